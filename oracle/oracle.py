"""ctypes loader of the CPU oracle (test infrastructure only).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module; the product path never does.  `make -C oracle` builds the two
libraries (float and double restatements of the reference substep).
"""
import ctypes as ct
import subprocess
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
BUILD = HERE / '_build'


def build():
    subprocess.run(['make', '-s', '-C', str(HERE)], check=True)


class Oracle:
    def __init__(self, precision='fp32'):
        name = 'liboracle_f32.so' if precision in ('fp32', 'float32') else 'liboracle_f64.so'
        path = BUILD / name
        if not path.is_file():
            build()
        self.lib = ct.CDLL(str(path))
        self.lib.oracle_step.restype = ct.c_int
        self.lib.oracle_step.argtypes = [ct.c_void_p, ct.c_void_p, ct.c_int, ct.c_int, ct.c_int, ct.c_int]
        self.lib.oracle_forward.restype = ct.c_int
        self.lib.oracle_forward.argtypes = [ct.c_void_p, ct.c_void_p, ct.c_int, ct.c_int, ct.c_int]

    def step(self, model, data, w0, w1, substeps, policy):
        rc = self.lib.oracle_step(ct.addressof(model), ct.addressof(data), w0, w1, substeps, policy)
        if rc:
            raise RuntimeError('oracle_step failed (%d)' % rc)

    def step_parallel(self, model, data, nworld, substeps, policy, threads):
        """Disjoint world ranges on `threads` host threads (ctypes drops the GIL)."""
        chunk = (nworld + threads - 1) // threads
        ranges = [(a, min(nworld, a + chunk)) for a in range(0, nworld, chunk)]
        with ThreadPoolExecutor(len(ranges)) as pool:
            list(pool.map(lambda r: self.step(model, data, r[0], r[1], substeps, policy), ranges))

    def forward(self, model, data, w0, w1, bootstrap):
        rc = self.lib.oracle_forward(ct.addressof(model), ct.addressof(data), w0, w1, bootstrap)
        if rc:
            raise RuntimeError('oracle_forward failed (%d)' % rc)
