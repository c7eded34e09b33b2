"""ctypes binding of ``libmetallora_b200.so`` (the C ABI in include/metallora_b200.h).

Loading is lazy; a missing library or an unsupported device raises
``DeviceError`` -- there is no CPU fallback anywhere in this package.
"""
from __future__ import annotations

import ctypes as C
import os
import threading
from pathlib import Path

from .exceptions import DeviceError, MetalLoRAError, ShapeError

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libmetallora_b200.so"

MLORA_OK = 0
MLORA_ERR_INVALID_ARG = -1
MLORA_ERR_UNSUPPORTED = -2
MLORA_ERR_CUDA = -3
MLORA_ERR_WORKSPACE = -4
MLORA_ERR_DEVICE = -5

BWD_ACCUMULATE = 1
BWD_DEFER_DX = 2
BWD_DX_ONLY = 4
BWD_GRADS_16BIT = 8

QUANT_NF4 = 1
QUANT_INT4 = 2
QUANT_INT8 = 3

DTYPE_BF16 = 0
DTYPE_F16 = 1
DTYPE_F32 = 2

_lib = None
_lock = threading.Lock()

vp = C.c_void_p
i64 = C.c_int64
f32 = C.c_float
i32 = C.c_int
sz = C.c_size_t

# name -> (restype, argtypes); kept in the order of include/metallora_b200.h
SIGNATURES: dict[str, tuple] = {
    "mlora_version": (i32, []),
    "mlora_status_string": (C.c_char_p, [i32]),
    "mlora_last_error_message": (C.c_char_p, []),
    "mlora_device_supported": (i32, [i32]),
    "mlora_device_status": (i32, [C.POINTER(C.c_uint32), i32]),
    "mlora_launch_count": (C.c_longlong, []),
    "mlora_profile_enable": (i32, [i32]),
    "mlora_profile_read": (i32, [C.POINTER(C.c_double), C.POINTER(C.c_longlong), i32, i32]),
    "mlora_lora_forward_workspace_bytes": (sz, [i64, i64, i64, i64, i32]),
    "mlora_lora_forward": (i32, [vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, f32, i32, vp, sz, vp]),
    "mlora_lora_backward_workspace_bytes": (sz, [i64, i64, i64, i64, i32]),
    "mlora_lora_backward": (i32, [vp, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, f32, f32,
                                  i32, vp, sz, vp]),
    "mlora_lora_backward_ex": (i32, [vp, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, f32,
                                     f32, i32, i32, vp, sz, vp]),
    "mlora_linear_workspace_bytes": (sz, [i64, i64, i64, i32]),
    "mlora_linear": (i32, [vp, vp, vp, i64, i64, i64, i32, vp, sz, vp]),
    "mlora_merge_workspace_bytes": (sz, [i64, i64, i64, i32]),
    "mlora_merge": (i32, [vp, vp, vp, vp, i64, i64, i64, f32, i32, vp, sz, vp]),
    "mlora_quantize": (i32, [vp, i32, i64, i64, i32, i64, vp, vp, vp, vp]),
    "mlora_dequantize": (i32, [i32, vp, vp, vp, i64, i64, i64, vp, i32, vp]),
    "mlora_qlora_forward_workspace_bytes": (sz, [i64, i64, i64, i64, i32, i64]),
    "mlora_qlora_backward_workspace_bytes": (sz, [i64, i64, i64, i64, i32, i64]),
    "mlora_qlora_lean_workspace_bytes": (sz, [i64, i64, i64, i64, i32, i64, i32]),
    "mlora_qlora_forward": (i32, [vp, i32, vp, vp, vp, i64, vp, vp, vp, vp, i64, i64, i64, i64,
                                  f32, i32, vp, sz, vp]),
    "mlora_qlora_backward": (i32, [vp, vp, i32, vp, vp, vp, i64, vp, vp, vp, vp, vp, vp, i64, i64,
                                   i64, i64, f32, f32, i32, i32, vp, sz, vp]),
    "mlora_qlora_prepared_scales_bytes": (sz, [i32, i64, i64, i64]),
    "mlora_multi_lora_forward_workspace_bytes": (sz, [i64, i64, i64, i64, i64, i32]),
    "mlora_lora_embedding_workspace_bytes": (sz, [i64, i64, i64, i32, i32]),
    "mlora_lora_kv_cache_workspace_bytes": (sz, [i64, i64, i64, i64, i32]),
    "mlora_peer_allreduce": (i32, [vp, vp, i32, i32, C.c_uint32, vp, i64, f32, vp, vp]),
    "mlora_lora_kv_cache_update": (i32, [vp] * 9 + [i64] * 6 + [f32, i32, vp, sz, vp]),
    "mlora_lora_embedding_forward": (i32, [vp, vp, vp, vp, vp, i64, i64, i64, i64, f32, i32, vp,
                                           sz, vp]),
    "mlora_lora_embedding_backward": (i32, [vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, i64,
                                            f32, i32, i32, vp, sz, vp]),
    "mlora_multi_lora_forward": (i32, [vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, f32, i32,
                                       vp, sz, vp]),
    "mlora_qlora_prepare_scales": (i32, [i32, vp, vp, i64, i64, i64, vp, vp]),
    "mlora_qlora_forward_ex": (i32, [vp, i32, vp, vp, vp, vp, i64, vp, vp, vp, vp, i64, i64, i64,
                                     i64, f32, i32, vp, sz, vp]),
    "mlora_qlora_backward_ex": (i32, [vp, vp, i32, vp, vp, vp, vp, i64, vp, vp, vp, vp, vp, vp,
                                      i64, i64, i64, i64, f32, f32, i32, i32, vp, sz, vp]),
    "mlora_adamw_step": (i32, [vp, vp, vp, vp, vp, i64, f32, f32, f32, f32, f32, i32, vp, vp]),
    "mlora_sgd_step": (i32, [vp, vp, i64, f32, i32, vp, vp]),
    "mlora_adam_state_step": (i32, [vp, f32, f32, vp]),
    "mlora_grad_norm_workspace_bytes": (sz, []),
    "mlora_grad_norm_clip": (i32, [vp, i64, f32, vp, vp, sz, vp]),
    "mlora_lora_grads_static_scratch_bytes": (sz, []),
    "mlora_lora_grads_static": (i32, [vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, f32, f32, i32,
                                      vp]),
}


def load(path: str | os.PathLike | None = None):
    """Loads (once) and returns the library handle with typed signatures."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = Path(path) if path else LIB_PATH
        if not p.is_file():
            raise DeviceError(
                f"{p} is missing: build it with `python -m metallora_b200.build` "
                "(the CUDA extension is required; there is no CPU fallback)")
        lib = C.CDLL(str(p))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def last_error() -> str:
    return load().mlora_last_error_message().decode(errors="replace")


def check(status: int, what: str) -> None:
    """Maps a C-ABI status to the reference's exception family."""
    if status == MLORA_OK:
        return
    msg = f"{what}: {last_error()}"
    if status in (MLORA_ERR_INVALID_ARG, MLORA_ERR_UNSUPPORTED, MLORA_ERR_WORKSPACE):
        raise ShapeError(msg)
    if status == MLORA_ERR_DEVICE:
        raise DeviceError(msg)
    raise MetalLoRAError(msg)


KERNEL_KINDS = ("gemm", "rank", "wgrad", "elementwise", "quant", "gemv", "optim")


def launch_count() -> int:
    return int(load().mlora_launch_count())


def profile_enable(on: bool) -> None:
    check(load().mlora_profile_enable(1 if on else 0), "mlora_profile_enable")


def profile_read(reset: bool = True) -> dict[str, tuple[float, int]]:
    """{kind: (total_ms, launches)} of the launches timed since the last reset."""
    n = len(KERNEL_KINDS)
    ms = (C.c_double * n)()
    cnt = (C.c_longlong * n)()
    check(load().mlora_profile_read(ms, cnt, n, 1 if reset else 0), "mlora_profile_read")
    return {k: (float(ms[i]), int(cnt[i])) for i, k in enumerate(KERNEL_KINDS)}


def device_status(reset: bool = False) -> int:
    out = C.c_uint32(0)
    check(load().mlora_device_status(C.byref(out), 1 if reset else 0), "mlora_device_status")
    return int(out.value)
