"""ctypes loader of the CPU oracle (test infrastructure only).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module; the product path never does.  `make -C oracle` builds the two
libraries (float and double restatements of the reference substep).
"""
import ctypes as ct
import subprocess

import numpy as np
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
BUILD = HERE / '_build'


def build():
    subprocess.run(['make', '-s', '-C', str(HERE)], check=True)


class NewtonLeaf(ct.Structure):
    """One world's constraint rows for the Newton-piece leaves (oracle.c NewtonLeaf)."""
    _fields_ = ([(k, ct.c_int) for k in ('nv', 'nefc', 'ne', 'nf', 'ncon', 'ls_iterations')] +
                [(k, ct.c_double) for k in ('impratio_invsqrt', 'tolerance', 'ls_tolerance', 'meaninertia')] +
                [(k, ct.c_void_p) for k in ('M', 'J', 'D', 'frictionloss', 'qfrc_smooth', 'search', 'type', 'id',
                                            'state_in', 'con_dim', 'con_adr', 'con_friction', 'jaref', 'qacc', 'Ma',
                                            'force', 'H', 'alpha', 'improvement', 'state', 'ls_evals', 'overflow')])


class Oracle:
    def __init__(self, precision='fp32'):
        name = 'liboracle_f32.so' if precision in ('fp32', 'float32') else 'liboracle_f64.so'
        path = BUILD / name
        if not path.is_file():
            build()
        self.lib = ct.CDLL(str(path))
        self.dtype = np.float32 if name.endswith('f32.so') else np.float64
        self.real = ct.c_float if self.dtype == np.float32 else ct.c_double
        P = ct.c_void_p
        self.lib.oracle_leaf_positions.argtypes = [P] * 11
        self.lib.oracle_leaf_contacts.argtypes = [P] * 13
        self.lib.oracle_leaf_box.argtypes = [ct.c_int] + [P] * 6 + [self.real] + [P] * 3
        self.lib.oracle_leaf_integrate.argtypes = [P, P, P, ct.c_double]
        self.lib.oracle_leaf_convex.argtypes = ([ct.c_int] + [P] * 4 + [ct.c_int]) * 2 + [self.real] * 2 + \
            [ct.c_int] * 2 + [P] * 3
        self.lib.oracle_step.restype = ct.c_int
        self.lib.oracle_step.argtypes = [ct.c_void_p, ct.c_void_p, ct.c_int, ct.c_int, ct.c_int, ct.c_int]
        self.lib.oracle_forward.restype = ct.c_int
        self.lib.oracle_forward.argtypes = [ct.c_void_p, ct.c_void_p, ct.c_int, ct.c_int, ct.c_int]
        for leaf in ('rows', 'hessian', 'linesearch'):
            fn = getattr(self.lib, 'oracle_leaf_newton_' + leaf)
            fn.restype = ct.c_int
            fn.argtypes = [ct.POINTER(NewtonLeaf)]
        self.lib.oracle_newton_leaf_bytes.restype = ct.c_size_t
        if self.lib.oracle_newton_leaf_bytes() != ct.sizeof(NewtonLeaf):
            raise ValueError('NewtonLeaf layout differs between oracle.c and oracle.py')

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

    # ---- single-world leaves (golden-vector tests)
    def _ptr(self, a):
        return a.ctypes.data_as(ct.c_void_p)

    def positions(self, model, sizes, qpos):
        """Kinematics, CoM/CRB and the dense mass matrix of one world."""
        nb, ng, nv = sizes['nbody'], sizes['ngeom'], sizes['nv']
        out = dict(xpos=np.zeros((nb, 3)), xquat=np.zeros((nb, 4)), xipos=np.zeros((nb, 3)),
                   geom_xpos=np.zeros((ng, 3)), geom_xmat=np.zeros((ng, 9)), com=np.zeros((nb, 3)),
                   cinert=np.zeros((nb, 10)), cdof=np.zeros((nv, 6)), M=np.zeros((nv, nv)))
        out = {k: v.astype(self.dtype) for k, v in out.items()}
        q = np.ascontiguousarray(qpos, self.dtype)
        args = [ct.c_void_p(ct.addressof(model)), self._ptr(q)] + [self._ptr(out[k]) for k in
                ('xpos', 'xquat', 'xipos', 'geom_xpos', 'geom_xmat', 'com', 'cinert', 'cdof', 'M')]
        if self.lib.oracle_leaf_positions(*args):
            raise RuntimeError('oracle_leaf_positions failed')
        return out

    def contacts(self, model, sizes, qpos, qvel):
        """Contacts (geoms, dim, 28-real records) and constraint rows of one world."""
        nc, ne, nv = sizes['ncon_max'], sizes['nefc_max'], sizes['nv']
        ncon, nefc = ct.c_int(), ct.c_int()
        geoms, dims = np.zeros(2 * nc, np.int32), np.zeros(nc, np.int32)
        rec = np.zeros((nc, 28), self.dtype)
        J, D, aref = np.zeros((ne, nv), self.dtype), np.zeros(ne, self.dtype), np.zeros(ne, self.dtype)
        typ, ids = np.zeros(ne, np.int32), np.zeros(ne, np.int32)
        q, v = np.ascontiguousarray(qpos, self.dtype), np.ascontiguousarray(qvel, self.dtype)
        if self.lib.oracle_leaf_contacts(ct.addressof(model), self._ptr(q), self._ptr(v), ct.addressof(ncon),
                                         self._ptr(geoms), self._ptr(dims), self._ptr(rec), ct.addressof(nefc),
                                         self._ptr(J), self._ptr(D), self._ptr(aref), self._ptr(typ), self._ptr(ids)):
            raise RuntimeError('oracle_leaf_contacts failed')
        c, e = ncon.value, nefc.value
        return dict(ncon=c, geom=geoms[:2 * c].reshape(c, 2), dim=dims[:c], dist=rec[:c, 0], pos=rec[:c, 1:4],
                    frame=rec[:c, 4:13].reshape(c, 3, 3), margin=rec[:c, 13], friction=rec[:c, 14:19],
                    solref=rec[:c, 19:21], solimp=rec[:c, 21:26], solreffriction=rec[:c, 26:28], nefc=e,
                    J=J[:e], D=D[:e], aref=aref[:e], type=typ[:e], id=ids[:e])

    def box(self, type1, p1, R1, s1, p2, R2, s2, margin=0.0):
        """sphere/capsule/box (geom 1) against a box (geom 2) on raw poses."""
        arr = [np.ascontiguousarray(np.asarray(x, float).ravel(), self.dtype) for x in (p1, R1, s1, p2, R2, s2)]
        dist, pos, nrm = np.zeros(8, self.dtype), np.zeros(24, self.dtype), np.zeros(24, self.dtype)
        n = self.lib.oracle_leaf_box(type1, *[self._ptr(a) for a in arr], margin, self._ptr(dist), self._ptr(pos),
                                     self._ptr(nrm))
        return dist[:n].astype(float), pos[:3 * n].reshape(n, 3).astype(float), nrm[:3 * n].reshape(n, 3).astype(float)

    def integrate(self, model, qpos, qvel, dt):
        """qpos advanced by dt * qvel on the joint manifold (one world)."""
        q = np.ascontiguousarray(qpos, self.dtype).copy()
        v = np.ascontiguousarray(qvel, self.dtype)
        if self.lib.oracle_leaf_integrate(ct.addressof(model), self._ptr(q), self._ptr(v), dt):
            raise RuntimeError('oracle_leaf_integrate failed')
        return q

    def convex(self, kind1, p1, R1, s1, v1, kind2, p2, R2, s2, v2, margin=0.0, tol=1e-6, iterations=50,
               epa_iterations=32):
        """Convex narrowphase of two shapes on raw poses; v1 / v2 are local
        mesh vertices (None for primitives).  Returns (dist, pos, normal) or
        None; `self.epa_overflow` tells whether EPA's pools filled."""
        def arr(x, n):
            return np.ascontiguousarray(np.zeros(n) if x is None else np.asarray(x, float).ravel(), self.dtype)
        a = [arr(p1, 3), arr(R1, 9), arr(s1, 3), arr(v1, 3), arr(p2, 3), arr(R2, 9), arr(s2, 3), arr(v2, 3)]
        n1 = 0 if v1 is None else len(np.asarray(v1).reshape(-1, 3))
        n2 = 0 if v2 is None else len(np.asarray(v2).reshape(-1, 3))
        dist, pos, nrm = np.zeros(1, self.dtype), np.zeros(3, self.dtype), np.zeros(3, self.dtype)
        n = self.lib.oracle_leaf_convex(kind1, *[self._ptr(x) for x in a[:4]], n1, kind2,
                                        *[self._ptr(x) for x in a[4:]], n2, margin, tol, iterations,
                                        epa_iterations, self._ptr(dist), self._ptr(pos), self._ptr(nrm))
        self.epa_overflow = bool(n & 2)
        return (float(dist[0]), pos.astype(float), nrm.astype(float)) if n & 1 else None

    # ---- Newton pieces on one world's explicit rows (golden-vector tests)
    def newton(self, piece, case):
        """Run one Newton piece ('rows', 'hessian' or 'linesearch') on the rows
        of `case` (a dict of arrays in the reference's row layout); returns
        the piece's outputs."""
        r = self.dtype
        nv, n = int(case['nv']), len(case['type'])
        keep = []

        def arr(x, dtype):
            a = np.ascontiguousarray(np.asarray(x, dtype).reshape(-1))
            keep.append(a)
            return a.ctypes.data

        s = NewtonLeaf()
        s.nv, s.nefc, s.ne, s.nf = nv, n, int(case.get('ne', 0)), int(case.get('nf', 0))
        s.ncon, s.ls_iterations = len(case['con_dim']), int(case.get('ls_iterations', 0))
        s.impratio_invsqrt = float(case['impratio'])
        for k in ('tolerance', 'ls_tolerance', 'meaninertia'):
            setattr(s, k, float(case.get(k, 0.0)))
        s.M = arr(case.get('M', np.eye(nv)), r)
        s.J = arr(case['J'], r)
        s.D = arr(case['D'], r)
        s.frictionloss = arr(case.get('frictionloss', np.zeros(n)), r)
        s.type, s.id = arr(case['type'], np.int32), arr(case['id'], np.int32)
        s.state_in = arr(case.get('state', np.zeros(n)), np.int32)
        s.con_dim, s.con_adr = arr(case['con_dim'], np.int32), arr(case['con_adr'], np.int32)
        s.con_friction = arr(case['con_friction'], r)
        # in/out arrays: always copies, so the caller's inputs stay untouched
        jaref = np.array(case['jaref'], r, copy=True, order='C')
        qacc = np.array(case.get('qacc', np.zeros(nv)), r, copy=True, order='C')
        Ma = np.array(case.get('Ma', np.zeros(nv)), r, copy=True, order='C')
        s.jaref, s.qacc, s.Ma = jaref.ctypes.data, qacc.ctypes.data, Ma.ctypes.data
        s.qfrc_smooth = arr(case.get('qfrc_smooth', np.zeros(nv)), r)
        s.search = arr(case.get('search', np.zeros(nv)), r)
        force, H = np.zeros(n, r), np.zeros(nv * nv, r)
        state, alpha, improvement = np.zeros(n, np.int32), np.zeros(1, r), np.zeros(1, r)
        evals, overflow = np.zeros(1, np.int32), np.zeros(1, np.int32)
        s.force, s.H, s.state = force.ctypes.data, H.ctypes.data, state.ctypes.data
        s.alpha, s.improvement = alpha.ctypes.data, improvement.ctypes.data
        s.ls_evals, s.overflow = evals.ctypes.data, overflow.ctypes.data
        if getattr(self.lib, 'oracle_leaf_newton_' + piece)(ct.byref(s)):
            raise RuntimeError('oracle_leaf_newton_%s rejected the case' % piece)
        if piece == 'rows':
            return dict(force=force.astype(float), state=state)
        if piece == 'hessian':
            return dict(H=H.reshape(nv, nv).astype(float))
        return dict(alpha=float(alpha[0]), improvement=float(improvement[0]), ls_evals=int(evals[0]),
                    overflow=int(overflow[0]), qacc=qacc.astype(float), Ma=Ma.astype(float), jaref=jaref.astype(float))
