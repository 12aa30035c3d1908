"""Offline build of libb200phys.so for sm_100a (nvcc; no JIT, no torch extension).

The library is written in-tree to gpu-libero_b200/_lib/ so that it travels
with the repository snapshot.  Flags follow the reference FP32 build
(libero/libero/gpu/cmake/MjwarpBox.cmake:15): FMA contraction on, IEEE
division and square root, no flush-to-zero; never --use_fast_math.
"""
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent
REPO = ROOT.parent
OUT = Path(os.environ.get('B200PHYS_BUILD_OUT', ROOT / '_lib' / 'libb200phys.so'))
SOURCES = [ROOT / 'csrc' / 'b200phys.cu']
DEPENDS = SOURCES + sorted((ROOT / 'csrc').glob('*.cuh')) + sorted((REPO / 'include').glob('*.h'))
NVCC = os.environ.get('NVCC', '/usr/local/cuda/bin/nvcc')
FLAGS = ['-O3', '-std=c++17', '-gencode', 'arch=compute_100a,code=sm_100a', '-lineinfo',
         '--fmad=true', '--prec-div=true', '--prec-sqrt=true', '--ftz=false',
         '-Xcompiler', '-fPIC', '-shared', '-I' + str(REPO / 'include')]


def stale():
    if not OUT.is_file():
        return True
    built = OUT.stat().st_mtime
    return any(p.stat().st_mtime > built for p in DEPENDS)


def build(force=False, verbose=False):
    if not force and not stale():
        return OUT
    OUT.parent.mkdir(parents=True, exist_ok=True)
    source_id = 'b200phys-' + str(abs(hash(tuple(p.read_bytes() for p in DEPENDS))) % (1 << 32))
    extra = os.environ.get('B200PHYS_NVCC_EXTRA', '').split()
    cmd = [NVCC] + FLAGS + extra + ['-DB200PHYS_SOURCE_ID="%s"' % source_id] + [str(s) for s in SOURCES] + ['-o', str(OUT)]
    if verbose:
        cmd.insert(1, '-Xptxas=-v')
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == '__main__':
    build(force=True, verbose='-v' in sys.argv)
