"""B200-native (sm_100a) paged-KV-cache hot path for mini-engine.

Drop-in replacement for the paged-KV entry points of the reference engine's
``mini_engine/kernels`` package (decode attention, ragged paged prefill, KV
scatter/append, copy-on-write, device-side batch metadata), implemented as
hand-written CUDA kernels in ``libminikv.so`` behind a C ABI
(``include/minikv.h``) and called from Python through ctypes.
"""

from . import _lib

__all__ = ["_lib"]
