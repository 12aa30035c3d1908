"""ctypes loader of the reference's own FP32 collision leaves (test infrastructure only).

`make -C oracle ref REFERENCE=<reference checkout>` compiles the reference's
broadphase, plane, box and convex leaves unmodified, with the harness
ref_contacts.cu, into oracle/_ref/libref_contacts.so.  The library is built
where the reference checkout exists and travels prebuilt; where it is absent,
`available()` is False and the tests that use it skip.

`collide(scene, xpos, xmat)` runs the reference's collision sequence
(cuda_fp32/physics.py:95-100: broadphase, convex, planes, boxes) on given geom
poses and returns its pooled contact list.

The same target builds oracle/_ref/libref_native_{f64,f32}.so from
ref_native.cu: the reference's native MuJoCo 2.3.7 sphere-sphere,
sphere-capsule and capsule-capsule colliders (collision_detect_primitive.cuh)
with its real_t as double and as float, for the families its FP32 engine
lacks.  `RefNative.collide` runs them on given poses.
"""
import ctypes as ct
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / '_ref' / 'libref_contacts.so'
NATIVE_LIBS = {'fp64': HERE / '_ref' / 'libref_native_f64.so', 'fp32': HERE / '_ref' / 'libref_native_f32.so'}
P = ct.c_void_p


class RefGeomModel(ct.Structure):
    _fields_ = ([(k, ct.c_int) for k in ('ngeom', 'npairs', 'nmesh', 'nmeshvert', 'nmeshpoly', 'nmeshpolyvert',
                                          'nmeshpolymap', 'ccd_iterations', 'boxbox_primitive')] +
                [('ccd_tolerance', ct.c_float)] +
                [(k, P) for k in ('geom_type', 'geom_dataid', 'geom_condim', 'geom_priority', 'pairs', 'aabb',
                                  'rbound', 'margin', 'gap', 'size', 'solmix', 'solref', 'solimp', 'friction',
                                  'mesh_vertadr', 'mesh_vertnum', 'mesh_polyadr', 'mesh_polynum',
                                  'mesh_polyvertadr', 'mesh_polyvertnum', 'mesh_polyvert', 'mesh_polymapadr',
                                  'mesh_polymapnum', 'mesh_polymap', 'mesh_vert', 'mesh_polynormal')])


class RefContacts(ct.Structure):
    _fields_ = [('capacity', ct.c_int), ('count', ct.c_int), ('candidates', ct.c_int)] + \
        [(k, P) for k in ('geom', 'world', 'dim', 'dist', 'pos', 'frame', 'overflow')]


def build(reference=None):
    """Compile the leaves from the reference checkout given as `reference` or
    by the GPU_LIBERO_REFERENCE environment variable; False without one."""
    reference = reference or os.environ.get('GPU_LIBERO_REFERENCE')
    if not reference or not Path(reference, 'libero', 'libero', 'gpu', 'cuda', 'collision').is_dir():
        return False
    subprocess.run(['make', '-s', '-C', str(HERE), 'ref', 'REFERENCE=' + str(reference)], check=True)
    return LIB.is_file()


def available():
    return LIB.is_file()


class RefCollision:
    def __init__(self):
        self.lib = ct.CDLL(str(LIB))
        self.lib.refc_collide.restype = ct.c_int
        self.lib.refc_collide.argtypes = [ct.POINTER(RefGeomModel), ct.c_int, P, P, ct.POINTER(RefContacts)]
        self.lib.refc_model_bytes.restype = ct.c_size_t
        self.lib.refc_contacts_bytes.restype = ct.c_size_t
        if self.lib.refc_model_bytes() != ct.sizeof(RefGeomModel) or \
                self.lib.refc_contacts_bytes() != ct.sizeof(RefContacts):
            raise RuntimeError('libref_contacts.so struct sizes differ from the loader')
        if not self.lib.refc_abi_ok():
            raise RuntimeError('reference leaf argument packs differ from the harness view')

    def collide(self, scene, xpos, xmat, capacity=None):
        """Reference contacts for geom poses xpos [W, ngeom*3], xmat [W, ngeom*9] (float32)."""
        s, I, Rl = scene.sizes, scene.ints, scene.reals
        ng = s['ngeom']
        W = xpos.shape[0]
        keep = []

        def i32(a):
            a = np.ascontiguousarray(np.asarray(a, np.int32).reshape(-1))
            keep.append(a)
            return a.ctypes.data if a.size else None

        def f32(a):
            a = np.ascontiguousarray(np.asarray(a, np.float32).reshape(-1))
            keep.append(a)
            return a.ctypes.data if a.size else None

        pairs = np.sort(np.asarray(I['pair_geom'], np.int32).reshape(-1, 2), axis=1)
        types = np.asarray(I['geom_type'])
        boxes = np.flatnonzero(types == 6)
        margin = np.asarray(Rl['geom_margin'], float)
        boxbox_margin = any(margin[a] + margin[b] > 0 for a, b in pairs if types[a] == 6 and types[b] == 6)
        m = RefGeomModel(ngeom=ng, npairs=len(pairs), nmesh=s['nmesh'], nmeshvert=s['nmeshvert'],
                         nmeshpoly=s['nmeshpoly'], nmeshpolyvert=s['nmeshpolyvert'], nmeshpolymap=s['nmeshpolymap'],
                         ccd_iterations=s['ccd_iterations'], boxbox_primitive=int(boxbox_margin or boxes.size == 0),
                         ccd_tolerance=float(scene.scalars['ccd_tolerance']))
        for k in ('geom_type', 'geom_dataid', 'geom_condim', 'geom_priority', 'mesh_vertadr', 'mesh_vertnum',
                  'mesh_polyadr', 'mesh_polynum', 'mesh_polyvertadr', 'mesh_polyvertnum', 'mesh_polyvert',
                  'mesh_polymapadr', 'mesh_polymapnum', 'mesh_polymap'):
            setattr(m, k, i32(I[k]))
        m.pairs = i32(pairs)
        for k, name in (('aabb', 'geom_aabb'), ('rbound', 'geom_rbound'), ('margin', 'geom_margin'),
                        ('gap', 'geom_gap'), ('size', 'geom_size'), ('solmix', 'geom_solmix'),
                        ('solref', 'geom_solref'), ('solimp', 'geom_solimp'), ('friction', 'geom_friction'),
                        ('mesh_vert', 'mesh_vert'), ('mesh_polynormal', 'mesh_polynormal')):
            setattr(m, k, f32(Rl[name]))
        cap = int(capacity or W * len(pairs) * 8 + 64)
        out = RefContacts(capacity=cap)
        arrays = dict(geom=np.zeros((cap, 2), np.int32), world=np.zeros(cap, np.int32), dim=np.zeros(cap, np.int32),
                      dist=np.zeros(cap, np.float32), pos=np.zeros((cap, 3), np.float32),
                      frame=np.zeros((cap, 9), np.float32), overflow=np.zeros(W, np.int32))
        for k, a in arrays.items():
            setattr(out, k, a.ctypes.data)
        xp = np.ascontiguousarray(xpos, np.float32)
        xm = np.ascontiguousarray(xmat, np.float32)
        rc = self.lib.refc_collide(ct.byref(m), W, xp.ctypes.data, xm.ctypes.data, ct.byref(out))
        if rc:
            raise RuntimeError('reference collision leaves: CUDA error %d' % rc)
        n = min(out.count, cap)
        res = {k: (a[:n] if k != 'overflow' else a) for k, a in arrays.items()}
        res.update(count=out.count, candidates=out.candidates, capacity=cap)
        return res


def native_available():
    return all(p.is_file() for p in NATIVE_LIBS.values())


class RefNative:
    """The reference's native sphere / capsule colliders on given geom poses,
    with real_t of the given precision ('fp64' or 'fp32')."""

    def __init__(self, precision='fp64'):
        lib = self.lib = ct.CDLL(str(NATIVE_LIBS[precision]))
        lib.refn_real_bits.restype = ct.c_int
        lib.refn_max_hits.restype = ct.c_int
        lib.refn_collide.restype = ct.c_int
        lib.refn_collide.argtypes = [ct.c_int] * 3 + [P] * 8
        self.bits = 64 if precision == 'fp64' else 32
        if lib.refn_real_bits() != self.bits:
            raise RuntimeError('%s has real_t of %d bits' % (NATIVE_LIBS[precision].name, lib.refn_real_bits()))
        self.dtype = np.float64 if self.bits == 64 else np.float32
        self.max_hits = lib.refn_max_hits()

    def collide(self, scene, xpos, xmat, pairs, margin):
        """Contacts of `pairs` [P, 2] (each pair's margin in `margin` [P]) for geom
        poses xpos [W, ngeom*3], xmat [W, ngeom*9].  Returns count [W, P] (-1 for a
        family these colliders do not cover) and hits [W, P, max_hits, 7]: dist,
        pos[3], normal[3], in the library's precision."""
        ng = scene.sizes['ngeom']
        f = self.dtype
        xp = np.ascontiguousarray(xpos, f).reshape(-1, ng * 3)
        xm = np.ascontiguousarray(xmat, f).reshape(-1, ng * 9)
        W = xp.shape[0]
        types = np.ascontiguousarray(scene.ints['geom_type'], np.int32)
        size = np.ascontiguousarray(scene.reals['geom_size'], f)
        pr = np.ascontiguousarray(pairs, np.int32).reshape(-1, 2)
        mg = np.ascontiguousarray(margin, f).reshape(-1)
        count = np.zeros((W, len(pr)), np.int32)
        hits = np.zeros((W, len(pr), self.max_hits, 7), f)
        rc = self.lib.refn_collide(W, ng, len(pr), types.ctypes.data, size.ctypes.data, xp.ctypes.data,
                                   xm.ctypes.data, pr.ctypes.data, mg.ctypes.data, count.ctypes.data,
                                   hits.ctypes.data)
        if rc:
            raise RuntimeError('reference native colliders: CUDA error %d' % rc)
        return count, hits
