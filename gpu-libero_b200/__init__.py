"""B200-native batched rigid-body physics step (GPU-LIBERO physics_engine="b200").

Importing this package never touches the GPU.  `runtime.B200BatchEnv` and
`runtime.Runtime` require a CUDA device and the built libb200phys.so.
"""
from . import native, scene, selection  # noqa: F401

__all__ = ['native', 'scene', 'selection']
