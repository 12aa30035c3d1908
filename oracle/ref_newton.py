"""ctypes loader of the reference's own FP32 Newton leaves (test infrastructure only).

`make -C oracle ref REFERENCE=<reference checkout>` compiles the reference's
solver-state, constraint, Hessian and line-search leaves
(libero/libero/gpu/cuda/newton/mjwarp_{solver_state,constraint,hessian,linesearch}.cu)
unmodified, with the harness ref_newton.cu, into oracle/_ref/libref_newton.so.
The reference's direction leaf needs NVIDIA MathDx (absent); the harness
stands in for its Cholesky solve.  The library is built where the reference
checkout exists and travels prebuilt; where it is absent, `available()` is
False and the tests that use it skip.

`RefNewton.solve(batch)` runs the reference's Newton loop
(cuda_fp32/physics.py Newton.solve) on a batch of frozen problems in the
reference's row layout and returns its results and first-iteration values.
"""
import ctypes as ct
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / '_ref' / 'libref_newton.so'
P = ct.c_void_p

CASE_INTS = ('nworld', 'nv', 'rows', 'ncon', 'iterations', 'ls_iterations')
CASE_FLOATS = ('tolerance', 'ls_tolerance', 'meaninertia', 'impratio_invsqrt')
CASE_ARRAYS = (('nefc', np.int32), ('nf', np.int32), ('J', np.float32), ('D', np.float32), ('aref', np.float32),
               ('frictionloss', np.float32), ('row_type', np.int32), ('row_contact', np.int32),
               ('con_world', np.int32), ('con_dim', np.int32), ('con_address', np.int32),
               ('con_friction', np.float32), ('con_dist', np.float32), ('con_margin', np.float32),
               ('M', np.float32), ('qacc_smooth', np.float32), ('qacc_warmstart', np.float32),
               ('qfrc_smooth', np.float32))
OUT_ARRAYS = (('qacc', np.float32, 'nv'), ('qfrc_constraint', np.float32, 'nv'), ('force', np.float32, 'rows'),
              ('state', np.int32, 'rows'), ('niter', np.int32, 1), ('overflow', np.int32, 1),
              ('qacc0', np.float32, 'nv'), ('search0', np.float32, 'nv'), ('Ma0', np.float32, 'nv'),
              ('grad0', np.float32, 'nv'), ('jaref0', np.float32, 'rows'), ('state0', np.int32, 'rows'),
              ('H0', np.float32, 'nvnv'), ('alpha0', np.float32, 1), ('improvement0', np.float32, 1))


class RefNewtonCase(ct.Structure):
    _fields_ = [(k, ct.c_int) for k in CASE_INTS] + [(k, ct.c_float) for k in CASE_FLOATS] + \
        [(k, P) for k, _ in CASE_ARRAYS]


class RefNewtonOut(ct.Structure):
    _fields_ = [(k, P) for k, _, _ in OUT_ARRAYS]


def available():
    return LIB.is_file()


class RefNewton:
    def __init__(self):
        lib = self.lib = ct.CDLL(str(LIB))
        lib.refnt_solve.restype = ct.c_int
        lib.refnt_solve.argtypes = [ct.POINTER(RefNewtonCase), ct.POINTER(RefNewtonOut)]
        lib.refnt_case_bytes.restype = ct.c_size_t
        lib.refnt_out_bytes.restype = ct.c_size_t
        if lib.refnt_case_bytes() != ct.sizeof(RefNewtonCase) or lib.refnt_out_bytes() != ct.sizeof(RefNewtonOut):
            raise RuntimeError('libref_newton.so struct sizes differ from the loader')
        if not lib.refnt_abi_ok():
            raise RuntimeError('reference Newton leaf argument packs differ from the harness view')

    def solve(self, batch):
        """`batch`: the CASE_INTS / CASE_FLOATS scalars and CASE_ARRAYS arrays
        (world-major, rows padded to `rows`).  Returns the OUT_ARRAYS."""
        c = RefNewtonCase(**{k: int(batch[k]) for k in CASE_INTS}, **{k: float(batch[k]) for k in CASE_FLOATS})
        keep = []
        for k, dt in CASE_ARRAYS:
            a = np.ascontiguousarray(np.asarray(batch[k], dt).reshape(-1))
            if a.size == 0:
                a = np.zeros(1, dt)
            keep.append(a)
            setattr(c, k, a.ctypes.data)
        W, nv, rows = c.nworld, c.nv, c.rows
        size = dict(nv=nv, rows=rows, nvnv=nv * nv)
        out, o = {}, RefNewtonOut()
        for k, dt, n in OUT_ARRAYS:
            out[k] = np.zeros((W, size.get(n, n) if isinstance(n, str) else n), dt)
            setattr(o, k, out[k].ctypes.data)
        rc = self.lib.refnt_solve(ct.byref(c), ct.byref(o))
        if rc:
            raise RuntimeError('reference Newton leaves: CUDA error %d' % rc)
        out['H0'] = out['H0'].reshape(W, nv, nv)
        for k in ('niter', 'overflow', 'alpha0', 'improvement0'):
            out[k] = out[k][:, 0]
        return out
