"""ctypes bindings to ``oracle/_ref/libmlref.so`` -- the reference's own Metal
compute shaders compiled for the CPU (see oracle/build_ref.py and
oracle/ref_driver.cpp).  TEST INFRASTRUCTURE ONLY: used by tests/ and by
tests/golden/make_golden.py to pin the numpy oracle.

Shapes follow the reference shaders: x is [batch, seq, K]; fp16 buffers are
passed as numpy float16 arrays.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

LIB_PATH = Path(__file__).resolve().parent / "_ref" / "libmlref.so"
_lib = None


def available() -> bool:
    return LIB_PATH.is_file()


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.is_file():
            raise FileNotFoundError(f"{LIB_PATH} not built (python oracle/build_ref.py)")
        _lib = C.CDLL(str(LIB_PATH))
        _lib.mlref_dequant_nf4.restype = C.c_float
        _lib.mlref_dequant_nf4.argtypes = [C.c_ubyte, C.c_int, C.c_float]
        _lib.mlref_dequant_int4.restype = C.c_float
        _lib.mlref_dequant_int4.argtypes = [C.c_ubyte, C.c_int, C.c_float, C.c_float]
        _lib.mlref_lora_maintenance.argtypes = [C.c_void_p, C.c_float, C.c_float]
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "reference kernels take row-contiguous buffers"
    return C.c_void_p(a.ctypes.data)


U = C.c_uint
F = C.c_float


def lora_forward_fused(x, W0, A, B, alpha):
    """kernels.py:41-144 (live Metal forward), fp32."""
    x = np.ascontiguousarray(x, np.float32)
    if x.ndim == 2:
        x = x[None]
    bsz, seq, K = x.shape
    D, R = W0.shape[0], A.shape[0]
    W0, A, B = (np.ascontiguousarray(t, np.float32) for t in (W0, A, B))
    out = np.zeros((bsz, seq, D), np.float32)
    lib().mlref_lora_forward_fused(_p(x), _p(W0), _p(A), _p(B), _p(out), U(bsz), U(seq), U(K),
                                   U(D), U(R), F(alpha))
    return out


def lora_backward_fused(grad_output, x, A, B, alpha, clip):
    """kernels.py:249-308: per-token clamped atomic dA/dB, fp32."""
    g = np.ascontiguousarray(grad_output, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    bsz, seq, K = x.shape
    R, D = A.shape[0], B.shape[0]
    A, B = np.ascontiguousarray(A, np.float32), np.ascontiguousarray(B, np.float32)
    gA = np.zeros((R, K), np.float32)
    gB = np.zeros((D, R), np.float32)
    lib().mlref_lora_backward_fused(_p(g), _p(x), _p(A), _p(B), _p(gA), _p(gB), U(bsz), U(seq),
                                    U(K), U(D), U(R), F(alpha), F(clip))
    return gA, gB


def lora_adamw_step(param, grad, m, v, gpu_state, lr, b1, b2, eps, wd):
    """kernels.py:314-344; returns updated (param, grad, m, v)."""
    p, g, m, v = (np.array(t, np.float32, copy=True) for t in (param, grad, m, v))
    st = np.ascontiguousarray(gpu_state, np.float32)
    lib().mlref_lora_adamw_step(_p(p), _p(g), _p(m), _p(v), _p(st), U(p.size), F(lr), F(b1),
                                F(b2), F(eps), F(wd))
    return p, g, m, v


def lora_maintenance(gpu_state, b1, b2):
    st = np.array(gpu_state, np.float32, copy=True)
    lib().mlref_lora_maintenance(_p(st), b1, b2)
    return st


def dequant_nf4_scalar(packed_byte, high, absmax):
    return lib().mlref_dequant_nf4(int(packed_byte), int(high), float(absmax))


def dequant_int4_scalar(packed_byte, high, scale, zero):
    return lib().mlref_dequant_int4(int(packed_byte), int(high), float(scale), float(zero))


def qlora_forward_nf4(W0_quant, absmax, x, A, B, alpha, block_size):
    """lora_quantized.metal:97-164; x/A/B/out fp16."""
    x = np.ascontiguousarray(x, np.float16)
    if x.ndim == 2:
        x = x[None]
    bsz, seq, K = x.shape
    D, R = W0_quant.shape[0], A.shape[0]
    Wq = np.ascontiguousarray(W0_quant, np.uint8)
    am = np.ascontiguousarray(absmax, np.float32)
    A, B = np.ascontiguousarray(A, np.float16), np.ascontiguousarray(B, np.float16)
    out = np.zeros((bsz, seq, D), np.float16)
    lib().mlref_qlora_forward_nf4(_p(Wq), _p(am), _p(x), _p(A), _p(B), _p(out), U(bsz), U(seq),
                                  U(K), U(D), U(R), F(alpha), U(block_size))
    return out


def qlora_forward_int4(W0_quant, scales, zeros, x, A, B, alpha):
    """lora_quantized.metal:29-93 (per-row fp32 scale/zero); x/A/B/out fp16."""
    x = np.ascontiguousarray(x, np.float16)
    if x.ndim == 2:
        x = x[None]
    bsz, seq, K = x.shape
    D, R = W0_quant.shape[0], A.shape[0]
    Wq = np.ascontiguousarray(W0_quant, np.uint8)
    s = np.ascontiguousarray(scales, np.float32)
    z = np.ascontiguousarray(zeros, np.float32)
    A, B = np.ascontiguousarray(A, np.float16), np.ascontiguousarray(B, np.float16)
    out = np.zeros((bsz, seq, D), np.float16)
    lib().mlref_qlora_forward_int4(_p(Wq), _p(s), _p(z), _p(x), _p(A), _p(B), _p(out), U(bsz),
                                   U(seq), U(K), U(D), U(R), F(alpha))
    return out


def train_forward(x, W0, A, B, alpha):
    """lora_train.metal:27-86 -> (out fp16, Ax_cache fp32)."""
    x = np.ascontiguousarray(x, np.float16)
    bsz, seq, K = x.shape
    D, R = W0.shape[0], A.shape[0]
    W0, A, B = (np.ascontiguousarray(t, np.float16) for t in (W0, A, B))
    out = np.zeros((bsz, seq, D), np.float16)
    ax = np.zeros((bsz, seq, R), np.float32)
    lib().mlref_train_forward(_p(x), _p(W0), _p(A), _p(B), _p(out), _p(ax), U(bsz), U(seq), U(K),
                              U(D), U(R), F(alpha))
    return out, ax


def train_backward(grad_output, x, ax_cache, A, B, alpha, clip):
    """lora_train.metal:90-154 -> (grad_A, grad_B) fp32."""
    g = np.ascontiguousarray(grad_output, np.float16)
    x = np.ascontiguousarray(x, np.float16)
    bsz, seq, K = x.shape
    R, D = A.shape[0], B.shape[0]
    axc = np.ascontiguousarray(ax_cache, np.float32)
    A, B = np.ascontiguousarray(A, np.float16), np.ascontiguousarray(B, np.float16)
    gA = np.zeros((R, K), np.float32)
    gB = np.zeros((D, R), np.float32)
    lib().mlref_train_backward(_p(g), _p(x), _p(axc), _p(A), _p(B), _p(gA), _p(gB), U(bsz),
                               U(seq), U(K), U(D), U(R), F(alpha), F(clip))
    return gA, gB


def optimizer_step(A, B, grad_A, grad_B, m_A, v_A, m_B, v_B, lr, b1, b2, eps, wd, step,
                   accum_steps=1):
    """lora_train.metal:158-210 -> updated (A, B, grad_A, grad_B, m_A, v_A, m_B, v_B)."""
    A = np.array(A, np.float16, copy=True)
    B = np.array(B, np.float16, copy=True)
    gA, gB, mA, vA, mB, vB = (np.array(t, np.float32, copy=True)
                              for t in (grad_A, grad_B, m_A, v_A, m_B, v_B))
    lib().mlref_optimizer_step(_p(A), _p(B), _p(gA), _p(gB), _p(mA), _p(vA), _p(mB), _p(vB),
                               F(lr), F(b1), F(b2), F(eps), F(wd), U(step), U(A.size),
                               U(B.size), U(accum_steps))
    return A, B, gA, gB, mA, vA, mB, vB


def multi_adapter(x, W0, adapters_A, adapters_B, adapter_ids, alpha):
    """kernels/lora_kernels.metal:440-508 (fp32): per-sample adapter over a
    shared base.  x [B, S, K] (K <= 4096, a multiple of 4), W0 [D, K],
    adapters_A [n, R, K] (R <= 128), adapters_B [n, D, R], adapter_ids [B]."""
    x = np.ascontiguousarray(x, np.float32)
    bsz, seq, K = x.shape
    n, R, _ = adapters_A.shape
    D = W0.shape[0]
    W0, Aa, Ba = (np.ascontiguousarray(t, np.float32) for t in (W0, adapters_A, adapters_B))
    ids = np.ascontiguousarray(adapter_ids, np.uint32)
    out = np.zeros((bsz, seq, D), np.float32)
    lib().mlref_multi_adapter(_p(x), _p(W0), _p(Aa), _p(Ba), _p(ids), _p(out), U(bsz), U(seq),
                              U(K), U(D), U(R), U(n), F(alpha))
    return out


KV_MAX_SEQ = 8192  # the shader's fixed cache length (lora_kernels.metal:584)


def kv_cache_update(x, W_K, W_V, A_K, B_K, A_V, B_V, k_cache, v_cache, cur_pos, alpha):
    """kernels/lora_kernels.metal:514-586 (fp16 storage): projects one new token
    per sequence x [B, D] and writes row ``cur_pos`` of the [B, 8192, D]
    caches; returns the updated copies of (k_cache, v_cache)."""
    x = np.ascontiguousarray(x, np.float16)
    bsz, D = x.shape
    R = A_K.shape[0]
    ws = [np.ascontiguousarray(t, np.float16) for t in (W_K, W_V, A_K, B_K, A_V, B_V)]
    kc = np.array(k_cache, np.float16, copy=True)
    vc = np.array(v_cache, np.float16, copy=True)
    assert kc.shape == (bsz, KV_MAX_SEQ, D) and vc.shape == kc.shape
    lib().mlref_kv_cache_update(_p(x), *[_p(w) for w in ws], _p(kc), _p(vc), U(bsz),
                                U(cur_pos), U(D), U(R), F(alpha))
    return kc, vc
