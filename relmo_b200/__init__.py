"""relmo_b200: B200-native (sm_100a) fan-out / fan-in message-passing ops.

A drop-in for relmo's ``relm_mp`` op library on CUDA: ``relmo_b200.ops.mp``
mirrors ``relmo.ops.mp`` (same functions, arguments, errors) and registers the
same ``torch.ops.relm_mp`` schemas, backed by hand-written CUDA kernels
(``librelm_mp_b200.so``, C ABI in ``include/relm_mp.h``).

Importing the package loads nothing; the native library is loaded on first
use by ``relmo_b200.ops.mp_runtime.ensure_loaded``.
"""

__all__ = ["ops"]
