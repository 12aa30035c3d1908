"""Offline build of libb200phys.so for sm_100a (nvcc; no JIT, no torch extension).

The library is written in-tree to gpu-libero_b200/_lib/ so that it travels
with the repository snapshot.  Flags follow the reference FP32 build
(libero/libero/gpu/cmake/MjwarpBox.cmake:15): FMA contraction on, IEEE
division and square root, no flush-to-zero; never --use_fast_math.

Translation units: csrc/abi.cu (C ABI, launch shape) and six instances of
csrc/inst.cu (kernels for float / double in the three convex modes of
csrc/launch.h: no GJK / EPA, GJK / EPA for meshes, and with the zero-margin
box-box path), all compiled in parallel and linked into one shared library.
"""
import hashlib
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

ROOT = Path(__file__).resolve().parent
REPO = ROOT.parent
CSRC = ROOT / 'csrc'
OUT = Path(os.environ.get('B200PHYS_BUILD_OUT', ROOT / '_lib' / 'libb200phys.so'))
DEPENDS = sorted(CSRC.glob('*.cu')) + sorted(CSRC.glob('*.cuh')) + sorted(CSRC.glob('*.h')) + \
    sorted((REPO / 'include').glob('*.h'))
NVCC = os.environ.get('NVCC', '/usr/local/cuda/bin/nvcc')
FLAGS = ['-O3', '-std=c++17', '-gencode', 'arch=compute_100a,code=sm_100a', '-lineinfo',
         '--fmad=true', '--prec-div=true', '--prec-sqrt=true', '--ftz=false',
         '-Xcompiler', '-fPIC', '-I' + str(REPO / 'include'), '-I' + str(CSRC)]
INSTANCES = [(real, mode) for real in ('float', 'double') for mode in ('0', '1', '2')]


def stale():
    if not OUT.is_file():
        return True
    built = OUT.stat().st_mtime
    return any(p.stat().st_mtime > built for p in DEPENDS)


def build(force=False, verbose=False):
    if not force and not stale():
        return OUT
    OUT.parent.mkdir(parents=True, exist_ok=True)
    objdir = OUT.parent / ('obj_' + OUT.stem)
    objdir.mkdir(exist_ok=True)
    digest = hashlib.sha1(b''.join(p.read_bytes() for p in DEPENDS)).hexdigest()[:8]
    extra = os.environ.get('B200PHYS_NVCC_EXTRA', '').split()
    base = [NVCC] + FLAGS + extra + (['-Xptxas=-v'] if verbose else [])
    jobs = [base + ['-DB200PHYS_SOURCE_ID="b200phys-%s"' % digest, '-c', str(CSRC / 'abi.cu'),
                    '-o', str(objdir / 'abi.o')]]
    for real, convex in INSTANCES:
        jobs.append(base + ['-DB200_INST_REAL=%s' % real, '-DB200_INST_CONVEX=%s' % convex, '-c',
                            str(CSRC / 'inst.cu'), '-o', str(objdir / ('inst_%s_%s.o' % (real, convex)))])
    with ThreadPoolExecutor(len(jobs)) as pool:
        results = list(pool.map(lambda cmd: subprocess.run(cmd, capture_output=True, text=True), jobs))
    for r in results:
        if verbose or r.returncode:
            sys.stderr.write(r.stdout + r.stderr)
    if any(r.returncode for r in results):
        raise subprocess.CalledProcessError(1, 'nvcc')
    objs = [str(objdir / 'abi.o')] + [str(objdir / ('inst_%s_%s.o' % i)) for i in INSTANCES]
    subprocess.run([NVCC, '-shared', '-gencode', 'arch=compute_100a,code=sm_100a'] + objs + ['-o', str(OUT)],
                   check=True)
    return OUT


if __name__ == '__main__':
    build(force=True, verbose='-v' in sys.argv)
