"""Kernel-level API over the C ABI, taking and returning ``torch.Tensor``.

Mirrors the reference's kernel module (python/metal_lora/kernels.py): the same
entry-point names (``is_metal_available``, ``lora_forward_metal``,
``lora_backward_metal``, ``lora_adamw_step_metal``,
``persistent_gpu_state_init/step``), backed by sm_100a CUDA kernels instead of
Metal shaders.  Every call enqueues on the current torch CUDA stream and never
synchronises; workspaces come from torch's caching allocator.

Activations and weights are bf16 or fp16 (fp32 accumulation), or fp32, which
runs as split-precision bf16 tensor-core GEMMs (three partial products per
product of two fp32 values, ~2^-16 relative error each).
"""
from __future__ import annotations

import torch

from . import _lib
from .exceptions import DeviceError, ShapeError

_DT = {torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_F16, torch.float32: _lib.DTYPE_F32}


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _need_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise DeviceError("metallora_b200 kernels take CUDA tensors (no CPU fallback)")


def _dtype_code(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise ShapeError(f"unsupported dtype {t.dtype}; use bfloat16, float16 or float32") from None


def _workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def is_metal_available() -> bool:
    """True when the CUDA extension loads and the current device is sm_100.

    Same name and meaning as the reference's ``kernels.is_metal_available()``
    (kernels.py:502): "can the custom kernels run here"."""
    try:
        lib = _lib.load()
    except DeviceError:
        return False
    if not torch.cuda.is_available():
        return False
    return bool(lib.mlora_device_supported(torch.cuda.current_device()))


def rank_tile(r: int) -> int:
    """Padded rank the tensor-core kernels use (power of two >= 16)."""
    R = 16
    while R < r:
        R *= 2
    return R


def _pad_rank(a: torch.Tensor, b: torch.Tensor, alpha: float):
    """Zero-pads A [r, K] / B [N, r] to a multiple-of-8 rank (16-byte rows) and
    rescales alpha so that alpha'/r' == alpha/r.  Zero rows/columns add nothing."""
    r = a.shape[0]
    r8 = (r + 7) // 8 * 8
    if r8 == r:
        return a, b, alpha, r
    a_p = torch.zeros((r8, a.shape[1]), dtype=a.dtype, device=a.device)
    a_p[:r] = a
    b_p = torch.zeros((b.shape[0], r8), dtype=b.dtype, device=b.device)
    b_p[:, :r] = b
    return a_p, b_p, alpha * r8 / r, r8


def _check_2d(name: str, t: torch.Tensor, shape: tuple, dtype: torch.dtype) -> None:
    if tuple(t.shape) != tuple(shape):
        raise ShapeError(f"{name} shape mismatch: expected {tuple(shape)}, got {tuple(t.shape)}")
    if t.dtype != dtype:
        raise ShapeError(f"{name} dtype mismatch: expected {dtype}, got {t.dtype}")


def lora_linear_fwd(x2d: torch.Tensor, w0: torch.Tensor, a: torch.Tensor, b: torch.Tensor,
                    alpha: float, save_xa: bool = False):
    """y = x.W0^T + (alpha/r).(x.A^T).B^T for 2-D x [M, K].

    Returns (y, saved_xa); saved_xa is the [R, ceil8(M)] rank intermediate the
    backward can reuse (bf16/fp16 only), else None."""
    _need_cuda(x2d, w0, a, b)
    dt = x2d.dtype
    code = _dtype_code(x2d)
    M, K = x2d.shape
    N = w0.shape[0]
    a, b, alpha, r = _pad_rank(a, b, alpha)
    _check_2d("W0", w0, (N, K), dt)
    _check_2d("A", a, (r, K), dt)
    _check_2d("B", b, (N, r), dt)
    x2d, w0, a, b = (t.contiguous() for t in (x2d, w0, a, b))
    y = torch.empty((M, N), dtype=dt, device=x2d.device)
    saved = None
    if save_xa and dt != torch.float32:
        saved = torch.empty((rank_tile(r), (M + 7) // 8 * 8), dtype=dt, device=x2d.device)
    if M == 0:  # no tokens: empty output, nothing to launch
        return y, saved
    lib = _lib.load()
    ws = _workspace(lib.mlora_lora_forward_workspace_bytes(M, K, N, r, code), x2d.device)
    st = lib.mlora_lora_forward(_ptr(x2d), _ptr(w0), _ptr(a), _ptr(b), _ptr(y), _ptr(saved), M, K,
                                N, r, float(alpha), code, _ptr(ws), ws.numel(), _stream())
    _lib.check(st, "mlora_lora_forward")
    return y, saved


def lora_linear_bwd(dy2d: torch.Tensor, x2d: torch.Tensor, w0: torch.Tensor | None,
                    a: torch.Tensor, b: torch.Tensor, alpha: float,
                    saved_xa: torch.Tensor | None = None, clip_value: float = 0.0,
                    need_dx: bool = True, da_out: torch.Tensor | None = None,
                    db_out: torch.Tensor | None = None, accumulate: bool = True,
                    grad_dtype: torch.dtype | None = None):
    """(dx, dA, dB) of the LoRA linear for 2-D dy [M, N], x [M, K].

    dA/dB are fp32 (master-gradient precision), or x's 16-bit dtype when
    ``grad_dtype`` names it (written by the kernel, no cast launch); clip_value
    > 0 clips them elementwise after the full reduction (ops.py:155).  With ``da_out`` and
    ``db_out`` (contiguous fp32 [r, K] / [N, r], rank a multiple of 8) the
    gradients are ADDED into those buffers (written over them when
    ``accumulate`` is False) and returned."""
    _need_cuda(dy2d, x2d, a, b)
    dt = x2d.dtype
    code = _dtype_code(x2d)
    M, K = x2d.shape
    N = dy2d.shape[1]
    r_orig = a.shape[0]
    a_p, b_p, alpha_p, r = _pad_rank(a, b, alpha)
    if dt == torch.float32:
        saved_xa = None
    _check_2d("grad_output", dy2d, (M, N), dt)
    _check_2d("A", a_p, (r, K), dt)
    _check_2d("B", b_p, (N, r), dt)
    if need_dx:
        if w0 is None:
            raise ShapeError("dx needs W0")
        _check_2d("W0", w0, (N, K), dt)
        w0 = w0.contiguous()
    dy2d, x2d, a_p, b_p = (t.contiguous() for t in (dy2d, x2d, a_p, b_p))
    lib = _lib.load()
    dx = torch.empty((M, K), dtype=dt, device=x2d.device) if need_dx else None
    flags = 0
    into = da_out is not None or db_out is not None
    if into:
        if r != r_orig:
            raise ShapeError("gradient accumulation buffers need a rank that is a multiple of 8")
        for name, t, shp in (("da_out", da_out, (r, K)), ("db_out", db_out, (N, r))):
            if t is None or t.dtype != torch.float32 or tuple(t.shape) != shp or \
                    not t.is_contiguous():
                raise ShapeError(f"{name} must be a contiguous fp32 tensor of shape {shp}")
        da, db = da_out, db_out
        flags = _lib.BWD_ACCUMULATE if accumulate else 0
    else:
        gdt = torch.float32
        if grad_dtype is not None and grad_dtype == dt and dt != torch.float32:
            gdt, flags = dt, _lib.BWD_GRADS_16BIT
        da = torch.empty((r, K), dtype=gdt, device=x2d.device)
        db = torch.empty((N, r), dtype=gdt, device=x2d.device)
    if M == 0:  # no tokens: the sums over tokens are zero; nothing to launch
        if not (into and accumulate):
            da.zero_()
            db.zero_()
        if into:
            return dx, da, db
        return dx, da[:r_orig].contiguous(), db[:, :r_orig].contiguous()
    ws = _workspace(lib.mlora_lora_backward_workspace_bytes(M, K, N, r, code), x2d.device)
    st = lib.mlora_lora_backward_ex(_ptr(dy2d), _ptr(x2d), _ptr(w0) if need_dx else None,
                                    _ptr(a_p), _ptr(b_p), _ptr(saved_xa), _ptr(dx), _ptr(da),
                                    _ptr(db), M, K, N, r, float(alpha_p), float(clip_value), code,
                                    flags, _ptr(ws), ws.numel(), _stream())
    _lib.check(st, "mlora_lora_backward")
    if into:
        return dx, da, db
    if r != r_orig:
        da, db = da[:r_orig].contiguous(), db[:, :r_orig].contiguous()
    return dx, da, db


def lora_linear_bwd_split(dy2d: torch.Tensor, x2d: torch.Tensor, w0: torch.Tensor,
                          a: torch.Tensor, b: torch.Tensor, alpha: float,
                          saved_xa: torch.Tensor | None, da_out: torch.Tensor,
                          db_out: torch.Tensor, accumulate: bool = True):
    """The 16-bit backward in two launches (MLORA_BWD_DEFER_DX, then
    MLORA_BWD_DX_ONLY): enqueues everything but the dx GEMM -- dA/dB land in
    ``da_out``/``db_out`` (fp32, added or written as ``accumulate`` says) --
    and returns ``finish``, which enqueues the dx GEMM and returns dx.  Work
    that needs only dA/dB (a gradient exchange on another stream) can be
    started between the two and overlaps the GEMM."""
    _need_cuda(dy2d, x2d, a, b)
    dt = x2d.dtype
    if dt == torch.float32:
        raise ShapeError("the split backward takes bf16/fp16 tensors")
    code = _dtype_code(x2d)
    M, K = x2d.shape
    N = dy2d.shape[1]
    r = a.shape[0]
    if r % 8:
        raise ShapeError("gradient buffers need a rank that is a multiple of 8")
    _check_2d("grad_output", dy2d, (M, N), dt)
    _check_2d("W0", w0, (N, K), dt)
    _check_2d("A", a, (r, K), dt)
    _check_2d("B", b, (N, r), dt)
    for name, t, shp in (("da_out", da_out, (r, K)), ("db_out", db_out, (N, r))):
        if t.dtype != torch.float32 or tuple(t.shape) != shp or not t.is_contiguous():
            raise ShapeError(f"{name} must be a contiguous fp32 tensor of shape {shp}")
    dy2d, x2d, w0, a, b = (t.contiguous() for t in (dy2d, x2d, w0, a, b))
    lib = _lib.load()
    dx = torch.empty((M, K), dtype=dt, device=x2d.device)
    ws = _workspace(lib.mlora_lora_backward_workspace_bytes(M, K, N, r, code), x2d.device)
    flags = _lib.BWD_ACCUMULATE if accumulate else 0
    if M == 0:  # no tokens: zero gradients (unless added to), empty dx
        if not accumulate:
            da_out.zero_()
            db_out.zero_()
        return lambda: dx

    def call(phase):
        st = lib.mlora_lora_backward_ex(_ptr(dy2d), _ptr(x2d), _ptr(w0), _ptr(a), _ptr(b),
                                        _ptr(saved_xa), _ptr(dx), _ptr(da_out), _ptr(db_out), M, K,
                                        N, r, float(alpha), 0.0, code, flags | phase, _ptr(ws),
                                        ws.numel(), _stream())
        _lib.check(st, "mlora_lora_backward_ex")

    call(_lib.BWD_DEFER_DX)

    def finish() -> torch.Tensor:
        call(_lib.BWD_DX_ONLY)
        return dx
    return finish


def linear(x2d: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """y = x.W^T (merged-weight forward, ops.py:106-114)."""
    _need_cuda(x2d, w)
    code = _dtype_code(x2d)
    M, K = x2d.shape
    N = w.shape[0]
    _check_2d("W", w, (N, K), x2d.dtype)
    x2d, w = x2d.contiguous(), w.contiguous()
    y = torch.empty((M, N), dtype=x2d.dtype, device=x2d.device)
    if M == 0:
        return y
    lib = _lib.load()
    ws = _workspace(lib.mlora_linear_workspace_bytes(M, K, N, code), x2d.device)
    st = lib.mlora_linear(_ptr(x2d), _ptr(w), _ptr(y), M, K, N, code, _ptr(ws), ws.numel(),
                          _stream())
    _lib.check(st, "mlora_linear")
    return y


def merge(w0: torch.Tensor, a: torch.Tensor, b: torch.Tensor, alpha: float,
          out: torch.Tensor | None = None) -> torch.Tensor:
    """W0 + (alpha/r).B.A (ops.py:162-172); ``out`` may be ``w0`` (in place)."""
    _need_cuda(w0, a, b)
    code = _dtype_code(w0)
    N, K = w0.shape
    a_p, b_p, alpha_p, r = _pad_rank(a, b, alpha)
    _check_2d("A", a_p, (r, K), w0.dtype)
    _check_2d("B", b_p, (N, r), w0.dtype)
    w0, a_p, b_p = w0.contiguous(), a_p.contiguous(), b_p.contiguous()
    lib = _lib.load()
    if out is None:
        out = torch.empty_like(w0)
    ws = _workspace(lib.mlora_merge_workspace_bytes(N, K, r, code), w0.device)
    st = lib.mlora_merge(_ptr(w0), _ptr(a_p), _ptr(b_p), _ptr(out), N, K, r, float(alpha_p), code,
                         _ptr(ws), ws.numel(), _stream())
    _lib.check(st, "mlora_merge")
    return out


def lora_forward_metal(x, w0, a, b, alpha: float = 16.0, batch_size=None, seq_len=None,
                       use_simd=None):
    """Fused LoRA forward (reference: kernels.py:507-566).  x is [B, S, K] or
    [S, K]; batch_size/seq_len/use_simd are accepted for signature parity."""
    shp = x.shape
    y, _ = lora_linear_fwd(x.reshape(-1, shp[-1]), w0, a, b, alpha)
    return y.reshape(*shp[:-1], w0.shape[0])


def lora_backward_metal(grad_output, x, a, b, alpha: float = 16.0, clip_value: float = 1.0):
    """(grad_A, grad_B) of the LoRA branch, clipped to +-clip_value (reference:
    kernels.py:569-612 / ops.py:143-155), returned in A's/B's dtype."""
    g = grad_output.reshape(-1, grad_output.shape[-1])
    xx = x.reshape(-1, x.shape[-1])
    _, da, db = lora_linear_bwd(g, xx, None, a, b, alpha, None, clip_value, need_dx=False)
    return da.to(a.dtype), db.to(b.dtype)


# ------------------------------------------------------------------ optimizer --

def persistent_gpu_state_init(beta1: float = 0.9, beta2: float = 0.999, device=None):
    """Device Adam state [step, beta1^step, beta2^step] (kernels.py:471-481).

    Starts at step 0 ([0, 1, 1]); ``persistent_gpu_state_step`` advances it
    before each update, so the first update uses step 1 and beta^1 -- the
    formula tests/test_parity.py:57-64 pins.  (The reference initialises to
    [1, b1, b2] and also steps before the first update, so its first update
    uses beta^2.)"""
    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    return torch.tensor([0.0, 1.0, 1.0], dtype=torch.float32, device=dev)


def persistent_gpu_state_step(gpu_state: torch.Tensor, beta1: float = 0.9, beta2: float = 0.999):
    """state := [t+1, b1^(t+1), b2^(t+1)] on the device (kernels.py:484-499)."""
    _need_cuda(gpu_state)
    _lib.check(_lib.load().mlora_adam_state_step(_ptr(gpu_state), beta1, beta2, _stream()),
               "mlora_adam_state_step")


def lora_adamw_step_metal(param, grad, m, v, gpu_state, lr: float, beta1: float, beta2: float,
                          eps: float, wd: float, grad_scale: torch.Tensor | None = None):
    """In-place AdamW step (kernels.py:615-643): updates param, m, v and zeroes
    grad.  param bf16/fp16/fp32; grad, m, v fp32 and contiguous."""
    _need_cuda(param, grad, m, v, gpu_state)
    for name, t in (("grad", grad), ("m", m), ("v", v)):
        if t.dtype != torch.float32 or t.numel() != param.numel() or not t.is_contiguous():
            raise ShapeError(f"{name} must be contiguous fp32 with param's size")
    if not param.is_contiguous():
        raise ShapeError("param must be contiguous")
    st = _lib.load().mlora_adamw_step(_ptr(param), _ptr(grad), _ptr(m), _ptr(v), _ptr(gpu_state),
                                      param.numel(), lr, beta1, beta2, eps, wd,
                                      _dtype_code(param), _ptr(grad_scale), _stream())
    _lib.check(st, "mlora_adamw_step")


def sgd_step(param, grad, lr: float, grad_scale: torch.Tensor | None = None):
    """In-place p -= lr * g (zeroes grad)."""
    _need_cuda(param, grad)
    st = _lib.load().mlora_sgd_step(_ptr(param), _ptr(grad), param.numel(), lr, _dtype_code(param),
                                    _ptr(grad_scale), _stream())
    _lib.check(st, "mlora_sgd_step")


def grad_norm_clip(grad: torch.Tensor, max_norm: float, out: torch.Tensor | None = None):
    """Device [clip scale, norm] of a flat fp32 gradient (trainer.py:237-240)."""
    _need_cuda(grad)
    if grad.dtype != torch.float32 or not grad.is_contiguous():
        raise ShapeError("grad must be contiguous fp32")
    lib = _lib.load()
    if out is None:
        out = torch.empty(2, dtype=torch.float32, device=grad.device)
    ws = _workspace(lib.mlora_grad_norm_workspace_bytes(), grad.device)
    st = lib.mlora_grad_norm_clip(_ptr(grad), grad.numel(), float(max_norm), _ptr(out), _ptr(ws),
                                  ws.numel(), _stream())
    _lib.check(st, "mlora_grad_norm_clip")
    return out


# --------------------------------------------------------- quantised bases --

def _qlora_ws_bytes(lib, qw, M, K, N, r, backward, need_w=True):
    """Staged workspace (a bf16 copy of deq(W), fastest) unless the weight asks
    for the lean fused-dequant kernel, or the call does not read the weight."""
    if getattr(qw, "lean", False) or not need_w:
        return lib.mlora_qlora_lean_workspace_bytes(M, K, N, r, qw.code, qw.group, int(backward))
    fn = (lib.mlora_qlora_backward_workspace_bytes if backward
          else lib.mlora_qlora_forward_workspace_bytes)
    return fn(M, K, N, r, qw.code, qw.group)


def qlora_linear_fwd(x2d: torch.Tensor, qw, a: torch.Tensor, b: torch.Tensor, alpha: float,
                     save_xa: bool = False):
    """y = x.deq(W)^T + (alpha/r).(x.A^T).B^T for a quantised base ``qw``
    (metallora_b200.quant.QuantizedWeight); x, A, B bf16.  ``qw.lean`` selects
    the fused kernel that dequantises in its main loop (no dense copy of W)."""
    _need_cuda(x2d, a, b)
    if x2d.dtype != torch.bfloat16:
        raise ShapeError("quantised-base LoRA takes bf16 activations")
    M, K = x2d.shape
    N = qw.shape[0]
    if qw.shape[1] != K:
        raise ShapeError(f"x has {K} features, the quantised weight {qw.shape[1]}")
    a, b, alpha, r = _pad_rank(a, b, alpha)
    _check_2d("A", a, (r, K), torch.bfloat16)
    _check_2d("B", b, (N, r), torch.bfloat16)
    x2d, a, b = x2d.contiguous(), a.contiguous(), b.contiguous()
    y = torch.empty((M, N), dtype=torch.bfloat16, device=x2d.device)
    saved = (torch.empty((rank_tile(r), (M + 7) // 8 * 8), dtype=torch.bfloat16,
                         device=x2d.device) if save_xa else None)
    if M == 0:  # no tokens: empty output, nothing to launch
        return y, saved
    lib = _lib.load()
    ws = _workspace(_qlora_ws_bytes(lib, qw, M, K, N, r, backward=False), x2d.device)
    st = lib.mlora_qlora_forward_ex(_ptr(x2d), qw.code, _ptr(qw.codes), _ptr(qw.scales),
                                    _ptr(qw.zeros), _ptr(qw.prepared_scales()), qw.group, _ptr(a),
                                    _ptr(b), _ptr(y), _ptr(saved), M, K, N, r, float(alpha),
                                    _lib.DTYPE_BF16, _ptr(ws), ws.numel(), _stream())
    _lib.check(st, "mlora_qlora_forward_ex")
    return y, saved


def qlora_linear_bwd(dy2d: torch.Tensor, x2d: torch.Tensor, qw, a: torch.Tensor, b: torch.Tensor,
                     alpha: float, saved_xa: torch.Tensor | None = None, clip_value: float = 0.0,
                     need_dx: bool = True, da_out: torch.Tensor | None = None,
                     db_out: torch.Tensor | None = None, accumulate: bool = True):
    """(dx, dA, dB) through a frozen quantised base (staged or lean as the forward);
    ``da_out``/``db_out``/``accumulate`` as in ``lora_linear_bwd``."""
    _need_cuda(dy2d, x2d, a, b)
    M, K = x2d.shape
    N = dy2d.shape[1]
    r_orig = a.shape[0]
    a_p, b_p, alpha_p, r = _pad_rank(a, b, alpha)
    _check_2d("grad_output", dy2d, (M, N), torch.bfloat16)
    _check_2d("A", a_p, (r, K), torch.bfloat16)
    _check_2d("B", b_p, (N, r), torch.bfloat16)
    dy2d, x2d, a_p, b_p = (t.contiguous() for t in (dy2d, x2d, a_p, b_p))
    lib = _lib.load()
    dx = torch.empty((M, K), dtype=torch.bfloat16, device=x2d.device) if need_dx else None
    flags = 0
    into = da_out is not None or db_out is not None
    if into:
        if r != r_orig:
            raise ShapeError("gradient accumulation buffers need a rank that is a multiple of 8")
        da, db = da_out, db_out
        flags = _lib.BWD_ACCUMULATE if accumulate else 0
    else:
        da = torch.empty((r, K), dtype=torch.float32, device=x2d.device)
        db = torch.empty((N, r), dtype=torch.float32, device=x2d.device)
    if M == 0:  # no tokens: the sums over tokens are zero; nothing to launch
        if not (into and accumulate):
            da.zero_()
            db.zero_()
        if into:
            return dx, da, db
        return dx, da[:r_orig].contiguous(), db[:, :r_orig].contiguous()
    ws = _workspace(_qlora_ws_bytes(lib, qw, M, K, N, r, backward=True, need_w=need_dx),
                    x2d.device)
    st = lib.mlora_qlora_backward_ex(_ptr(dy2d), _ptr(x2d), qw.code, _ptr(qw.codes),
                                     _ptr(qw.scales), _ptr(qw.zeros),
                                     _ptr(qw.prepared_scales()) if need_dx else None, qw.group,
                                     _ptr(a_p), _ptr(b_p), _ptr(saved_xa), _ptr(dx), _ptr(da),
                                     _ptr(db), M, K, N, r, float(alpha_p), float(clip_value),
                                     _lib.DTYPE_BF16, flags, _ptr(ws), ws.numel(), _stream())
    _lib.check(st, "mlora_qlora_backward_ex")
    if into:
        return dx, da, db
    if r != r_orig:
        da, db = da[:r_orig].contiguous(), db[:, :r_orig].contiguous()
    return dx, da, db


# ------------------------------------------------------ stacked adapters --

MAX_STACKED_RANK = 256  # n_adapters * rank per launch


def multi_lora_fwd(x2d: torch.Tensor, w0: torch.Tensor | None, a_stack: torch.Tensor,
                   b_stack: torch.Tensor, ids: torch.Tensor, r: int, alpha: float) -> torch.Tensor:
    """y = (x.w0^T if w0 is given) + (alpha/r) (x.A_g^T).B_g^T with g = ids[m] per
    token, over n adapters stacked as a_stack [n*r, K] and b_stack [N, n*r]
    (one launch of the rank kernel for all of them, then the tcgen05 GEMM);
    ids is an int32 CUDA tensor [M]; an id outside [0, n) adds no LoRA term."""
    _need_cuda(x2d, a_stack, b_stack, ids, w0)
    M, K = x2d.shape
    nr, K2 = a_stack.shape
    N = b_stack.shape[0]
    if K2 != K or b_stack.shape[1] != nr or nr % r:
        raise ShapeError("a_stack [n*r, K] and b_stack [N, n*r] do not match x / r")
    if w0 is not None:
        _check_2d("W0", w0, (N, K), x2d.dtype)
    if ids.dtype != torch.int32 or ids.numel() != M:
        raise ShapeError("ids must be an int32 tensor with one entry per token")
    n = nr // r
    x2d, a_stack, b_stack = x2d.contiguous(), a_stack.contiguous(), b_stack.contiguous()
    y = torch.empty((M, N), dtype=x2d.dtype, device=x2d.device)
    if M == 0:
        return y
    lib = _lib.load()
    code = _dtype_code(x2d)
    ws = _workspace(lib.mlora_multi_lora_forward_workspace_bytes(M, K, N, r, n, code), x2d.device)
    st = lib.mlora_multi_lora_forward(_ptr(x2d), _ptr(w0), _ptr(a_stack), _ptr(b_stack),
                                      _ptr(ids.contiguous()), _ptr(y), M, K, N, r, n, float(alpha),
                                      code, _ptr(ws), ws.numel(), _stream())
    _lib.check(st, "mlora_multi_lora_forward")
    return y


# ------------------------------------------------------------ embedding --

def _as_idx(indices: torch.Tensor) -> torch.Tensor:
    return indices.reshape(-1).to(torch.int32).contiguous()


def lora_embedding_fwd(indices: torch.Tensor, table: torch.Tensor, a: torch.Tensor,
                       b: torch.Tensor, alpha: float) -> torch.Tensor:
    """table[idx] + (alpha/r) b[idx].a for every index (LoRAEmbedding.__call__,
    layers.py:220-225); returns [*indices.shape, D]."""
    _need_cuda(indices, table, a, b)
    V, D = table.shape
    r = a.shape[0]
    _check_2d("A", a, (r, D), table.dtype)
    _check_2d("B", b, (V, r), table.dtype)
    idx = _as_idx(indices)
    T = idx.numel()
    code = _dtype_code(table)
    out = torch.empty((T, D), dtype=table.dtype, device=table.device)
    if T == 0:
        return out.reshape(*indices.shape, D)
    lib = _lib.load()
    ws = _workspace(lib.mlora_lora_embedding_workspace_bytes(T, D, r, code, 0), table.device)
    st = lib.mlora_lora_embedding_forward(_ptr(idx), _ptr(table.contiguous()), _ptr(a.contiguous()),
                                          _ptr(b.contiguous()), _ptr(out), T, V, D, r, float(alpha),
                                          code, _ptr(ws), ws.numel(), _stream())
    _lib.check(st, "mlora_lora_embedding_forward")
    return out.reshape(*indices.shape, D)


def lora_embedding_bwd(dy: torch.Tensor, indices: torch.Tensor, a: torch.Tensor, b: torch.Tensor,
                       alpha: float, da_out: torch.Tensor | None = None,
                       db_out: torch.Tensor | None = None):
    """fp32 (dA [r, D], dB [V, r]) of the LoRA embedding; dB rows are summed over
    each index's tokens in token order (deterministic).  With da_out/db_out the
    gradients are added into them."""
    _need_cuda(dy, indices, a, b)
    V, r = b.shape
    D = a.shape[1]
    idx = _as_idx(indices)
    T = idx.numel()
    dy2 = dy.reshape(T, D).contiguous()
    sorted_idx, order = torch.sort(idx, stable=True)
    order = order.to(torch.int32)
    lib = _lib.load()
    code = _dtype_code(dy2)
    flags = 0
    if da_out is not None and db_out is not None:
        da, db, flags = da_out, db_out, _lib.BWD_ACCUMULATE
    else:
        da = torch.empty((r, D), dtype=torch.float32, device=dy.device)
        db = torch.empty((V, r), dtype=torch.float32, device=dy.device)
    if T == 0:  # no tokens: zero gradients (or nothing added); nothing to launch
        if not flags:
            da.zero_()
            db.zero_()
        return da, db
    ws = _workspace(lib.mlora_lora_embedding_workspace_bytes(T, D, r, code, 1), dy.device)
    st = lib.mlora_lora_embedding_backward(_ptr(dy2), _ptr(idx), _ptr(sorted_idx), _ptr(order),
                                           _ptr(a.contiguous()), _ptr(b.contiguous()), _ptr(da),
                                           _ptr(db), T, V, D, r, float(alpha), code, flags,
                                           _ptr(ws), ws.numel(), _stream())
    _lib.check(st, "mlora_lora_embedding_backward")
    return da, db


# ------------------------------------------------------- KV-cache update --

def lora_kv_cache_update(x2d: torch.Tensor, wk: torch.Tensor, wv: torch.Tensor, ak: torch.Tensor,
                         bk: torch.Tensor, av: torch.Tensor, bv: torch.Tensor,
                         k_cache: torch.Tensor, v_cache: torch.Tensor, cur_pos: int,
                         alpha: float) -> None:
    """Projects one new token per sequence through the K and V LoRA linears and
    writes the rows straight into k_cache/v_cache [batch, max_seq, ...] at
    position cur_pos (lora_kv_cache_update, kernels/lora_kernels.metal:514-586)."""
    _need_cuda(x2d, wk, wv, ak, bk, av, bv, k_cache, v_cache)
    batch, D_in = x2d.shape
    D_kv = wk.shape[0]
    max_seq = k_cache.shape[1]
    if k_cache.shape[0] != batch or k_cache[0, 0].numel() != D_kv or v_cache.shape != k_cache.shape:
        raise ShapeError("caches must be [batch, max_seq, D_kv] (trailing dims may be heads, dim)")
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ShapeError("caches must be contiguous")
    r_orig = ak.shape[0]
    ak, bk, alpha_k, r = _pad_rank(ak, bk, alpha)
    av, bv, _, _ = _pad_rank(av, bv, alpha)
    for name, t, shape in (("W_K", wk, (D_kv, D_in)), ("W_V", wv, (D_kv, D_in)),
                           ("A_K", ak, (r, D_in)), ("A_V", av, (r, D_in)),
                           ("B_K", bk, (D_kv, r)), ("B_V", bv, (D_kv, r))):
        _check_2d(name, t, shape, x2d.dtype)
    del r_orig
    if batch == 0:  # no sequences: nothing to write
        return
    lib = _lib.load()
    code = _dtype_code(x2d)
    ws = _workspace(lib.mlora_lora_kv_cache_workspace_bytes(batch, D_in, D_kv, r, code), x2d.device)
    st = lib.mlora_lora_kv_cache_update(
        _ptr(x2d.contiguous()), _ptr(wk.contiguous()), _ptr(wv.contiguous()), _ptr(ak.contiguous()),
        _ptr(bk.contiguous()), _ptr(av.contiguous()), _ptr(bv.contiguous()), _ptr(k_cache),
        _ptr(v_cache), batch, int(cur_pos), max_seq, D_in, D_kv, r, float(alpha_k), code, _ptr(ws),
        ws.numel(), _stream())
    _lib.check(st, "mlora_lora_kv_cache_update")
