"""Engine selection with the B200 engine added.

Mirrors libero/libero/gpu/host/backends/selection.py:5-17 (``resolve_engine``)
and its error behaviour, adding ``physics_engine="b200"`` (FP32 by default,
FP64 when ``precision`` asks for it).  ``auto`` keeps the reference's choices.
"""

PRECISIONS = ('fp32', 'float32', 'fp64', 'float64')


def resolve_engine(engine='auto', precision=None):
    if engine not in ('auto', 'native', 'mjwarp', 'cuda_fp32', 'b200'):
        raise ValueError('physics_engine must be auto, native, mjwarp, cuda_fp32 or b200')
    if precision is not None and precision not in PRECISIONS:
        raise ValueError('precision must be fp32 or fp64')
    bits = 32 if precision in (None, 'fp32', 'float32') else 64
    if engine == 'auto':
        return 'cuda_fp32' if bits == 32 else 'native'
    if engine == 'mjwarp' and bits == 64:
        raise ValueError('MJWarp requires FP32; use physics_engine="native" for FP64')
    if engine == 'cuda_fp32' and bits == 64:
        raise ValueError('Independent cuda_fp32 requires FP32')
    return engine


def make_env(*args, physics_engine='auto', precision=None, **kwargs):
    """Construct the engine a reference caller asked for, if it is this one."""
    engine = resolve_engine(physics_engine, precision)
    if engine != 'b200':
        raise NotImplementedError('engine %r is the reference\'s own; this package provides "b200"' % engine)
    from .runtime import B200BatchEnv
    return B200BatchEnv(*args, physics_engine='b200', precision=precision or 'fp32', **kwargs)
