"""ctypes boundary of the B200 physics library (C ABI in include/b200phys.h).

The struct layouts are generated from include/b200phys_fields.h, the same
X-macro lists the C/CUDA side compiles, so the host and device agree on every
offset.  The reference binds its per-leaf libraries the same way: a ctypes
POD argument struct whose size is checked against the library's
``*_arguments_bytes()`` export before any launch
(libero/libero/gpu/host/backends/cuda_fp32/controller.py:92-96), and a
nonzero launch return raises ``RuntimeError('... CUDA error N')``
(cuda_fp32/bridges.py:57-60).
"""
import ctypes as ct
import os
import re
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
REPO = ROOT.parent
HEADER = REPO / 'include' / 'b200phys_fields.h'
LIBRARY = ROOT / '_lib' / 'libb200phys.so'


def _macro(text, name):
    """Body of the multi-line `#define name(X) ...` macro."""
    lines = text[text.index('#define ' + name + '(X)'):].splitlines()
    body = []
    for line in lines:
        body.append(line.rstrip().rstrip('\\'))
        if not line.rstrip().endswith('\\'):
            break
    return ' '.join(body)[len('#define ' + name + '(X)'):]


def _entries(text, name):
    body = _macro(text, name)
    out = []
    for m in re.finditer(r'X\(([^()]*(?:\([^()]*\)[^()]*)*)\)', body):
        parts = [p.strip() for p in m.group(1).split(',', 1)]
        out.append((parts[0], parts[1] if len(parts) > 1 else None))
    return out


class Layout:
    """Field lists parsed from include/b200phys_fields.h."""

    def __init__(self, path=HEADER):
        text = Path(path).read_text()
        self.int_scalars = [n for n, _ in _entries(text, 'B200_MODEL_INT_SCALARS')]
        self.real_scalars = [n for n, _ in _entries(text, 'B200_MODEL_REAL_SCALARS')]
        self.int_arrays = _entries(text, 'B200_MODEL_INT_ARRAYS')
        self.real_arrays = _entries(text, 'B200_MODEL_REAL_ARRAYS')
        self.data_real = _entries(text, 'B200_DATA_REAL')
        self.data_int = _entries(text, 'B200_DATA_INT')


LAYOUT = Layout()


class B200Model(ct.Structure):
    _fields_ = ([('real', ct.c_void_p), ('ints', ct.c_void_p)] +
                [(n, ct.c_int) for n in LAYOUT.int_scalars] +
                [(n, ct.c_double) for n in LAYOUT.real_scalars] +
                [('off_' + n, ct.c_int) for n, _ in LAYOUT.int_arrays] +
                [('off_' + n, ct.c_int) for n, _ in LAYOUT.real_arrays])


class B200Data(ct.Structure):
    _fields_ = ([('nworld', ct.c_int), ('world_offset', ct.c_int)] +
                [(n, ct.c_void_p) for n, _ in LAYOUT.data_real] +
                [(n, ct.c_void_p) for n, _ in LAYOUT.data_int])


def evaluate(expr, sizes):
    return int(eval(expr, {'__builtins__': {}}, dict(sizes)))


# packed parameter rows larger than this are refused (the copies live in HBM
# and are read through L2 by every world of their residue class)
MAX_ROW_BYTES = 1 << 32


class PackedModel:
    """A scene's arrays packed into one real buffer and one int32 buffer.

    rows: per-world parameter rows, {real array name: array of P rows}, each
    row the array's full length (a [P, ...] array is flattened per row).  World
    w (global index) reads row w % P of each such array, the reference's
    broadcast rule (cuda/dynamics/mjwarp_constraint_build.cu:18-20,
    ``p.data + (w % p.rows) * width``).  The real buffer then holds
    nvariant = lcm(P, ...) copies of every real array, variant_stride reals
    apart; copy v carries row v % P of each array given, and the scene's own
    values elsewhere.  Arrays derived from others (geom_aabb / geom_rbound from
    geom sizes, body_invweight0 / dof_invweight0 from masses) are not
    recomputed: give their rows too, or build the rows from compiled scenes
    with scene.parameter_rows.  Int arrays and scalars are one per model."""

    def __init__(self, scene, precision='fp32', rows=None):
        self.scene = scene
        self.dtype = np.float32 if precision in ('fp32', 'float32') else np.float64
        self.sizes = dict(scene.sizes)
        self.sizes['real_bytes'] = np.dtype(self.dtype).itemsize
        ints, reals, self.offsets, lengths = [], [], {}, {}
        at = 0
        for name, expr in LAYOUT.int_arrays:
            n = evaluate(expr, self.sizes)
            value = np.asarray(scene.ints[name], np.int32).reshape(-1)
            if value.size != n:
                raise ValueError('model int array %s has %d entries, expected %d' % (name, value.size, n))
            ints.append(value)
            self.offsets[name] = at
            at += n
        self.ints = np.ascontiguousarray(np.concatenate(ints + [np.zeros(1, np.int32)]))
        at = 0
        for name, expr in LAYOUT.real_arrays:
            n = evaluate(expr, self.sizes)
            value = np.asarray(scene.reals[name], np.float64).reshape(-1)
            if value.size != n:
                raise ValueError('model real array %s has %d entries, expected %d' % (name, value.size, n))
            reals.append(value)
            self.offsets[name] = at
            lengths[name] = n
            at += n
        base = np.concatenate(reals + [np.zeros(1)])
        # one copy per parameter row, each starting on a 128-byte boundary
        stride = -(-base.size // 32) * 32
        table = {}
        for name, value in (rows or {}).items():
            if name not in lengths:
                raise ValueError('parameter rows for %r: not a model real array' % (name,))
            value = np.asarray(value, np.float64)
            if value.ndim >= 1 and value.shape[0] >= 1:
                value = value.reshape(value.shape[0], -1)
            if value.ndim != 2 or value.shape[0] < 1 or value.shape[1] != lengths[name]:
                raise ValueError('parameter rows for %s: expected [P >= 1, %d] values, got shape %s'
                                 % (name, lengths[name], np.shape(value)))
            if not np.all(np.isfinite(value)):
                raise ValueError('parameter rows for %s hold non-finite values' % name)
            table[name] = value
        nvariant = 1
        for value in table.values():
            nvariant = int(np.lcm(nvariant, value.shape[0]))
            if nvariant * stride * self.sizes['real_bytes'] > MAX_ROW_BYTES:
                raise ValueError('parameter rows need %d model copies (the lcm of their row counts); '
                                 'more than %d bytes' % (nvariant, MAX_ROW_BYTES))
        packed = np.zeros((nvariant, stride))
        packed[:, :base.size] = base
        for name, value in table.items():
            o = self.offsets[name]
            packed[:, o:o + lengths[name]] = value[np.arange(nvariant) % value.shape[0]]
        self.nvariant, self.variant_stride = nvariant, stride
        self.sizes['nvariant'], self.sizes['variant_stride'] = nvariant, stride
        self.reals = np.ascontiguousarray(packed.reshape(-1).astype(self.dtype))

    def row_values(self, name, world):
        """The values of real array `name` that global world `world` reads."""
        o = self.offsets[name] + (world % self.nvariant) * self.variant_stride
        return self.reals[o:o + evaluate(dict(LAYOUT.real_arrays)[name], self.sizes)]

    def struct(self, real_ptr, int_ptr):
        m = B200Model()
        m.real, m.ints = real_ptr, int_ptr
        for n in LAYOUT.int_scalars:
            setattr(m, n, int(self.sizes[n]))
        for n in LAYOUT.real_scalars:
            setattr(m, n, float(self.scene.scalars[n]))
        # The FP32 engine floors the Newton tolerance at 1e-6
        # (cuda_fp32/model.py:71); the FP64 engine keeps the model's own.
        if self.dtype == np.float64:
            m.tolerance = float(self.scene.options.get('tolerance', m.tolerance))
        for n, _ in LAYOUT.int_arrays + LAYOUT.real_arrays:
            setattr(m, 'off_' + n, self.offsets[n])
        return m

    def host_struct(self):
        """B200Model over the host buffers; the struct keeps this owner alive."""
        st = self.struct(self.reals.ctypes.data, self.ints.ctypes.data)
        st._owner = self
        return st

    def data_widths(self):
        real = {n: evaluate(e, self.sizes) for n, e in LAYOUT.data_real}
        ints = {n: evaluate(e, self.sizes) for n, e in LAYOUT.data_int}
        return real, ints


def data_struct(arrays, nworld, world_offset=0, pointer=None):
    """B200Data from a dict name -> array; `pointer(array)` gives its address."""
    if pointer is None:
        pointer = lambda a: a.ctypes.data  # noqa: E731
    d = B200Data()
    d.nworld, d.world_offset = nworld, world_offset
    for n, _ in LAYOUT.data_real + LAYOUT.data_int:
        a = arrays.get(n)
        setattr(d, n, pointer(a) if a is not None else None)
    return d


class Library:
    """The product library (libb200phys.so); raises if it is missing."""

    def __init__(self, path=LIBRARY):
        path = Path(os.environ.get('B200PHYS_LIBRARY', path))
        if not path.is_file():
            raise FileNotFoundError('libb200phys.so is not built (%s); run __graft_entry__.build()' % path)
        self.path = path
        self.lib = ct.CDLL(str(path))
        lib = self.lib
        lib.b200phys_source_id.restype = ct.c_char_p
        for name in ('b200phys_model_bytes', 'b200phys_data_bytes'):
            getattr(lib, name).restype = ct.c_size_t
        lib.b200phys_arch.restype = ct.c_int
        lib.b200phys_world_smem_bytes.restype = ct.c_size_t
        lib.b200phys_world_smem_bytes.argtypes = [ct.POINTER(B200Model)]
        lib.b200phys_prepare.restype = ct.c_int
        lib.b200phys_prepare.argtypes = [ct.POINTER(B200Model)]
        lib.b200phys_step_launch.restype = ct.c_int
        lib.b200phys_step_launch.argtypes = [ct.POINTER(B200Model), ct.POINTER(B200Data), ct.c_int, ct.c_int,
                                             ct.c_void_p]
        lib.b200phys_order_launch.restype = ct.c_int
        lib.b200phys_order_launch.argtypes = [ct.POINTER(B200Model), ct.POINTER(B200Data), ct.c_void_p]
        lib.b200phys_forward_launch.restype = ct.c_int
        lib.b200phys_forward_launch.argtypes = [ct.POINTER(B200Model), ct.POINTER(B200Data), ct.c_int,
                                                ct.c_void_p, ct.c_void_p]
        for symbol, expected in (('b200phys_model_bytes', ct.sizeof(B200Model)),
                                 ('b200phys_data_bytes', ct.sizeof(B200Data))):
            got = getattr(lib, symbol)()
            if got != expected:
                raise ValueError('b200phys ABI differs: %s = %d, host expects %d' % (symbol, got, expected))

    @property
    def source_id(self):
        return self.lib.b200phys_source_id().decode()

    @property
    def arch(self):
        return int(self.lib.b200phys_arch())

    def smem_bytes(self, model):
        return int(self.lib.b200phys_world_smem_bytes(ct.byref(model)))

    def prepare(self, model):
        rc = self.lib.b200phys_prepare(ct.byref(model))
        if rc:
            raise RuntimeError('b200phys_prepare failed: CUDA error %d' % rc)

    def step(self, model, data, substeps, policy, stream):
        rc = self.lib.b200phys_step_launch(ct.byref(model), ct.byref(data), int(substeps), int(policy),
                                           ct.c_void_p(stream))
        if rc:
            raise RuntimeError('b200phys_step_launch failed: CUDA error %d' % rc)

    def order(self, model, data, stream):
        rc = self.lib.b200phys_order_launch(ct.byref(model), ct.byref(data), ct.c_void_p(stream))
        if rc:
            raise RuntimeError('b200phys_order_launch failed: CUDA error %d' % rc)

    def forward(self, model, data, bootstrap, mask_ptr, stream):
        rc = self.lib.b200phys_forward_launch(ct.byref(model), ct.byref(data), int(bootstrap),
                                              ct.c_void_p(mask_ptr or 0), ct.c_void_p(stream))
        if rc:
            raise RuntimeError('b200phys_forward_launch failed: CUDA error %d' % rc)


EXPORTS = ('b200phys_source_id', 'b200phys_arch', 'b200phys_model_bytes', 'b200phys_data_bytes',
           'b200phys_world_smem_bytes', 'b200phys_prepare', 'b200phys_step_launch', 'b200phys_forward_launch',
           'b200phys_order_launch')


def alloc_numpy(packed, nworld):
    """Zeroed world-major host buffers for every data field."""
    real, ints = packed.data_widths()
    arrays = {n: np.zeros((nworld, w), packed.dtype) for n, w in real.items()}
    arrays.update({n: np.zeros((nworld, w), np.int32) for n, w in ints.items()})
    return arrays
