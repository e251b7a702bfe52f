"""ctypes binding of libminikv (the C ABI declared in include/minikv.h).

The shared library is built in-tree (``python -m myvllm_mini_engine_b200.build``
or ``__graft_entry__.build()``) and loaded from this package directory.  There
is no CPU fallback: if the library is missing or fails to load, every op
raises RuntimeError.  A library built from other sources than the ones next
to it (its compiled-in ``minikv_source_hash`` differs) is refused the same way.
"""

from __future__ import annotations

import contextlib
import ctypes
import os
from pathlib import Path

import torch

LIB_NAME = "libminikv.so"
LIB_PATH = Path(__file__).resolve().parent / LIB_NAME

F32, F16, BF16 = 0, 1, 2
OK, EINVAL, ECUDA, EUNSUPPORTED = 0, 1, 2, 3
DTYPE_CODES = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}

_p, _i64, _int, _f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float

# name -> (restype, argtypes); must match include/minikv.h
SIGNATURES = {
    "minikv_abi_version": (_int, []),
    "minikv_source_hash": (ctypes.c_char_p, []),
    "minikv_last_error": (ctypes.c_char_p, []),
    "minikv_device_status": (_int, [ctypes.POINTER(ctypes.c_uint), _int, _p]),
    "minikv_set_wait_limit": (_int, [ctypes.c_uint64, _p]),
    "minikv_paged_decode_workspace_bytes": (_i64, [_i64] * 7 + [_int]),
    "minikv_paged_decode": (_int, [_p] * 6 + [_p, _i64] + [_i64] * 7 + [_int, _p]),
    "minikv_paged_decode_chained": (_int, [_p] * 6 + [_p, _i64] + [_i64] * 7 + [_int, _p]),
    "minikv_paged_decode_append": (_int, [_p] * 8 + [_p, _i64] + [_i64] * 7 + [_int, _int, _p]),
    "minikv_paged_decode_noalloc": (_int, [_p] * 6 + [_i64] * 7 + [_int, _p]),
    "minikv_kv_scatter_slots": (_int, [_p] * 5 + [_i64] * 7 + [_int, _p]),
    "minikv_kv_scatter_slots_fp8": (_int, [_p] * 5 + [_i64] * 7 + [_f32, _f32, _int, _int, _p]),
    "minikv_paged_decode_fp8_workspace_bytes": (_i64, [_i64] * 7 + [_int]),
    "minikv_paged_decode_fp8": (_int, [_p] * 6 + [_p, _i64] + [_i64] * 7 + [_f32, _f32, _int, _int, _p]),
    "minikv_paged_decode_fp8_append": (_int, [_p] * 8 + [_p, _i64] + [_i64] * 7 + [_f32, _f32, _int, _int, _int, _p]),
    "minikv_paged_prefill_fp8_workspace_bytes": (_i64, [_i64] * 9 + [_int]),
    "minikv_paged_prefill_fp8": (_int, [_p] * 8 + [_p, _i64] + [_i64] * 9 + [_f32, _f32, _int, _int, _p]),
    "minikv_kv_append_batch": (_int, [_p] * 6 + [_i64] * 8 + [_int, _p]),
    "minikv_kv_write_range": (_int, [_p, _p, _p, _i64, _i64, _p, _p] + [_i64] * 7 + [_int, _p]),
    "minikv_copy_blocks": (_int, [_p, _p, _p] + [_i64] * 4 + [_int, _p]),
    "minikv_paged_prefill_workspace_bytes": (_i64, [_i64] * 9 + [_int]),
    "minikv_paged_prefill": (_int, [_p] * 8 + [_p, _i64] + [_i64] * 9 + [_int, _p]),
    "minikv_build_prefill_metadata": (_int, [_p] * 5 + [_i64] * 4 + [_p] * 7 + [_p]),
    "minikv_build_decode_tables": (_int, [_p] * 6 + [_i64, _i64] + [_p] * 3 + [_p]),
    "minikv_rms_norm": (_int, [_p] * 5 + [_i64, _i64, ctypes.c_double, _int, _p]),
    "minikv_silu_mul": (_int, [_p, _p, _i64, _i64, _int, _p]),
    "minikv_argmax_workspace_bytes": (_i64, [_i64, _i64]),
    "minikv_argmax_rows": (_int, [_p, _i64, _i64, _i64, _int, _p, _i64, _p, _p]),
    "minikv_qk_rope_append": (_int, [_p, _i64] + [_p] * 9 + [_i64] * 7 + [ctypes.c_double, _int, _p]),
    "minikv_pack_linear": (_int, [_p, _p, _i64, _i64, _i64, _int, _p]),
    "minikv_linear": (_int, [_p, _i64, _p, _p, ctypes.c_double, _p, _p, _i64, _i64, _i64, _int, _p]),
    "minikv_linear_residual": (_int, [_p, _i64, _p, _p, _p, _p, _i64, _i64, _i64, _int, _p]),
    "minikv_linear_silu_mul": (_int, [_p, _i64, _p, _p, ctypes.c_double, _p, _p, _i64, _i64, _i64, _int, _p]),
    "minikv_linear_qk_rope_append": (_int, [_p, _i64, _p, _p, ctypes.c_double] + [_p] * 10 + [_i64] * 8
                                     + [_int, _p]),
}

_LIB = None


def load():
    """Load libminikv once; raise RuntimeError (never fall back) on failure."""
    global _LIB
    if _LIB is not None:
        return _LIB
    path = Path(os.environ.get("MINIKV_LIBRARY", LIB_PATH))
    if not path.is_file():
        raise RuntimeError(f"{path} is missing: build it with `python -m myvllm_mini_engine_b200.build`; "
                           "this package has no CPU fallback")
    try:
        lib = ctypes.CDLL(str(path))
    except OSError as error:
        raise RuntimeError(f"cannot load {path}: {error}") from error
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    if lib.minikv_abi_version() != 1:
        raise RuntimeError("libminikv ABI version mismatch; rebuild the library")
    from . import build

    if build.CSRC.is_dir():  # an installed copy without its sources cannot be checked
        expected, found = build.source_hash(), lib.minikv_source_hash().decode()
        if found != expected:
            raise RuntimeError(f"{path} was built from other sources (hash {found[:12]}, sources "
                               f"{expected[:12]}): rebuild it with `python -m myvllm_mini_engine_b200.build`")
    _LIB = lib
    return lib


def dtype_code(dtype):
    try:
        return DTYPE_CODES[dtype]
    except KeyError:
        raise RuntimeError("FP32/FP16/BF16 required") from None


_NO_SWITCH = contextlib.nullcontext()


def on_device(device):
    """Context that makes ``device`` the current CUDA device; free when it already is."""
    if device.index is None or device.index == torch.cuda.current_device():
        return _NO_SWITCH
    return torch.cuda.device(device)


_RAW_STREAM = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_of(device) -> int:
    """Handle of ``device``'s current CUDA stream (``torch.cuda.current_stream(device).cuda_stream``).

    Read without building a Stream object, which costs microseconds of host
    time on every kernel call.
    """
    if _RAW_STREAM is not None:
        return _RAW_STREAM(device.index if device.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(device).cuda_stream


def check(status: int, what: str) -> None:
    if status != OK:
        message = load().minikv_last_error().decode(errors="replace")
        raise RuntimeError(f"{what}: {message}")


def ptr(tensor) -> int | None:
    return tensor.data_ptr() if tensor is not None and tensor.numel() else None


def device_status(device=None, *, clear=True) -> int:
    """Synchronise the current stream and return (and clear) the device status bits."""
    lib = load()
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    value = ctypes.c_uint(0)
    with torch.cuda.device(device):
        check(lib.minikv_device_status(ctypes.byref(value), int(clear), stream_of(device)), "device status")
    return value.value


DEFAULT_WAIT_LIMIT_NS = 2_000_000_000


def set_wait_limit(limit_ns: int, device=None) -> None:
    """Limit of the kernels' slot waits (see ``minikv_set_wait_limit``); tests shorten it to drive the timeout path."""
    lib = load()
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(device):
        check(lib.minikv_set_wait_limit(int(limit_ns), stream_of(device)), "set_wait_limit")
