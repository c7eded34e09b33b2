"""The LoRA-linear C-ABI calls as PyTorch custom operators, ``torch.ops.metal_lora.*``.

The reference exposes its path as JIT-compiled Metal kernel objects called
from Python (python/metal_lora/kernels.py:370-464, used by
``lora_forward_metal`` :507-566 and ``lora_backward_metal`` :569-612).  Here
the same calls are registered with ``torch.library`` so that torch's tracers
(FX, ``torch.export``, ``torch.compile``) see one opaque operator per kernel
launch sequence instead of a Python function they cannot look into:

* ``metal_lora::lora_fwd(x, w0, a, b, alpha) -> (y, saved)`` -- the fused
  forward ``y = x.W0^T + (alpha/r).(x.A^T).B^T`` (ops.py:91-94) for x of any
  leading shape; ``saved`` is the rank intermediate ``(alpha/r).(x.A^T)`` the
  backward reuses (empty for fp32).  Autograd is registered: its backward is
  ``lora_bwd``, plus a plain GEMM for W0 when W0 requires a gradient.
* ``metal_lora::lora_bwd(dy, x, w0, a, b, saved, alpha, clip_value, need_dx)
  -> (dx, dA, dB)`` -- dx in x's dtype (empty when ``need_dx`` is False), dA
  [r, K] and dB [N, r] in fp32, clipped elementwise to +-clip_value after the
  full reduction when clip_value > 0 (ops.py:144-155).
* ``metal_lora::merge(w0, a, b, alpha) -> W'`` -- ``W0 + (alpha/r).B.A``
  (ops.py:162-172).
* ``metal_lora::linear(x, w) -> y`` -- the merged-weight forward ``x.W^T``
  (ops.py:106-114).
* ``metal_lora::qlora_fwd(x, codes, scales, zeros, prepared, scheme, group,
  lean, a, b, alpha) -> (y, saved)`` and ``qlora_bwd(...) -> (dx, dA, dB)`` --
  the same over a frozen NF4 / INT4 / INT8 base in the reference's packed
  layout (kernels/lora_quantized.metal:29-164); autograd registered on
  ``qlora_fwd``.  ``prepared`` is the weight's TMA-ready scale table
  (``QuantizedWeight.prepared_scales()``), or None to build it in the call.
* ``metal_lora::adamw_step(param, grad, m, v, gpu_state, lr, beta1, beta2,
  eps, wd, grad_scale)`` -- the in-place AdamW update of one LoRA tensor
  (kernels.py:615-643; operation order of kernels.py:333-343): param, m and v
  are updated and grad is zeroed (mutated arguments, no outputs);
  ``metal_lora::adam_state_step(gpu_state, beta1, beta2)`` advances the device
  step state [t, beta1^t, beta2^t] (kernels.py:484-499).

Each operator has a fake (shape) implementation, so it traces without a GPU.
The real implementations are the calls of :mod:`metallora_b200.kernels`; CPU
tensors raise :class:`DeviceError` there (no CPU fallback).  A and B may be of
a wider dtype than x: they are cast to x's dtype for the kernels and their
gradients are returned in their own dtype.

``LoRALinear`` and ``ops.lora_forward`` keep their own autograd function over
the same kernel calls, because it also carries the trainer's in-kernel
gradient buffers and cached casts, which an operator schema cannot express.
"""
from __future__ import annotations

import torch
from torch.library import custom_op

from . import kernels as _k
from .exceptions import ShapeError
from .quant import SCHEMES, QuantizedWeight

_NS = "metal_lora"


def _rows(x: torch.Tensor):
    m = 1
    for d in x.shape[:-1]:
        m = m * d
    return m


def _check(x: torch.Tensor, w0: torch.Tensor, a: torch.Tensor, b: torch.Tensor) -> None:
    K = x.shape[-1]
    N = w0.shape[0]
    r = a.shape[0]
    if w0.dim() != 2 or w0.shape[1] != K:
        raise ShapeError(f"W0 must be [out, {K}], got {tuple(w0.shape)}")
    if a.dim() != 2 or a.shape[1] != K:
        raise ShapeError(f"A must be [rank, {K}], got {tuple(a.shape)}")
    if b.dim() != 2 or tuple(b.shape) != (N, r):
        raise ShapeError(f"B must be [{N}, {r}], got {tuple(b.shape)}")


def _saved_shape(x: torch.Tensor, r: int):
    """Shape of the rank intermediate the forward saves: [padded rank, ceil8(M)]
    for 16-bit x (the rank kernel's transposed output), none for fp32."""
    if x.dtype == torch.float32:
        return (0,)
    return (_k.rank_tile((r + 7) // 8 * 8), (_rows(x) + 7) // 8 * 8)


# ---------------------------------------------------------------- lora_fwd --

@custom_op(f"{_NS}::lora_fwd", mutates_args=())
def lora_fwd(x: torch.Tensor, w0: torch.Tensor, a: torch.Tensor, b: torch.Tensor,
             alpha: float) -> tuple[torch.Tensor, torch.Tensor]:
    """Fused LoRA forward (ops.py:91-94); returns (y, saved intermediate)."""
    _check(x, w0, a, b)
    dt = x.dtype
    y, saved = _k.lora_linear_fwd(x.reshape(-1, x.shape[-1]), w0, a.to(dt), b.to(dt), alpha,
                                  save_xa=True)
    if saved is None:
        saved = x.new_empty((0,))
    return y.reshape(*x.shape[:-1], w0.shape[0]), saved


@lora_fwd.register_fake
def _lora_fwd_fake(x, w0, a, b, alpha):
    _check(x, w0, a, b)
    y = x.new_empty((*x.shape[:-1], w0.shape[0]))
    return y, x.new_empty(_saved_shape(x, a.shape[0]))


def _lora_fwd_setup(ctx, inputs, output):
    x, w0, a, b, alpha = inputs
    ctx.mark_non_differentiable(output[1])
    ctx.save_for_backward(x, w0, a, b, output[1])
    ctx.alpha = alpha


def _lora_fwd_backward(ctx, dy, _dsaved):
    x, w0, a, b, saved = ctx.saved_tensors
    need_dx = ctx.needs_input_grad[0]
    dx, da, db = torch.ops.metal_lora.lora_bwd(dy, x, w0, a, b, saved, ctx.alpha, 0.0, need_dx)
    dw0 = None
    if ctx.needs_input_grad[1]:
        # trainable base weight (freeze_base=False): plain library GEMM
        g2 = dy.reshape(-1, dy.shape[-1])
        dw0 = (g2.t().float() @ x.reshape(-1, x.shape[-1]).float()).to(w0.dtype)
    return (dx if need_dx else None, dw0,
            da.to(a.dtype) if ctx.needs_input_grad[2] else None,
            db.to(b.dtype) if ctx.needs_input_grad[3] else None, None)


lora_fwd.register_autograd(_lora_fwd_backward, setup_context=_lora_fwd_setup)


# ---------------------------------------------------------------- lora_bwd --

@custom_op(f"{_NS}::lora_bwd", mutates_args=())
def lora_bwd(dy: torch.Tensor, x: torch.Tensor, w0: torch.Tensor, a: torch.Tensor,
             b: torch.Tensor, saved: torch.Tensor, alpha: float, clip_value: float,
             need_dx: bool) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(dx, dA, dB) of the LoRA linear (autodiff of ops.py:91-94; dA/dB as
    ops.py:144-155); ``saved`` is lora_fwd's second output or an empty tensor."""
    _check(x, w0, a, b)
    dt = x.dtype
    K, N = x.shape[-1], w0.shape[0]
    sv = saved if saved.numel() > 0 else None
    dx, da, db = _k.lora_linear_bwd(dy.reshape(-1, N), x.reshape(-1, K), w0 if need_dx else None,
                                    a.to(dt), b.to(dt), alpha, sv, clip_value, need_dx=need_dx)
    dx = dx.reshape(x.shape) if need_dx else x.new_empty((0,))
    return dx, da, db


@lora_bwd.register_fake
def _lora_bwd_fake(dy, x, w0, a, b, saved, alpha, clip_value, need_dx):
    _check(x, w0, a, b)
    if tuple(dy.shape) != (*x.shape[:-1], w0.shape[0]):
        raise ShapeError(f"grad_output shape {tuple(dy.shape)} does not match the output")
    dx = x.new_empty(x.shape) if need_dx else x.new_empty((0,))
    da = a.new_empty(a.shape, dtype=torch.float32)
    db = b.new_empty(b.shape, dtype=torch.float32)
    return dx, da, db


# ------------------------------------------------------- merge and linear --

@custom_op(f"{_NS}::merge", mutates_args=())
def merge(w0: torch.Tensor, a: torch.Tensor, b: torch.Tensor, alpha: float) -> torch.Tensor:
    """``W0 + (alpha/A.shape[0]).B.A`` (ops.py:162-172) on the merge kernel."""
    dt = w0.dtype
    return _k.merge(w0, a.to(dt), b.to(dt), alpha)


@merge.register_fake
def _merge_fake(w0, a, b, alpha):
    if a.shape[1] != w0.shape[1] or tuple(b.shape) != (w0.shape[0], a.shape[0]):
        raise ShapeError("merge: A must be [r, in] and B [out, r]")
    return w0.new_empty(w0.shape)


@custom_op(f"{_NS}::linear", mutates_args=())
def linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """Merged-weight forward ``x.W^T`` (ops.py:106-114) for x of any leading shape."""
    y = _k.linear(x.reshape(-1, x.shape[-1]), w)
    return y.reshape(*x.shape[:-1], w.shape[0])


@linear.register_fake
def _linear_fake(x, w):
    if w.dim() != 2 or w.shape[1] != x.shape[-1]:
        raise ShapeError(f"W must be [out, {x.shape[-1]}], got {tuple(w.shape)}")
    return x.new_empty((*x.shape[:-1], w.shape[0]))


# ------------------------------------------------------ quantised bases --

def _qweight(x, codes, scales, zeros, prepared, scheme, group, lean) -> QuantizedWeight:
    if scheme not in SCHEMES:
        raise ShapeError(f"unknown scheme {scheme!r}; use one of {sorted(SCHEMES)}")
    qw = QuantizedWeight(scheme, codes, scales, zeros, int(group), (codes.shape[0], x.shape[-1]),
                         bool(lean))
    if prepared is not None:
        object.__setattr__(qw, "_prepared", prepared)
    return qw


def _check_q(x, codes, a, b, scheme):
    K, N, r = x.shape[-1], codes.shape[0], a.shape[0]
    per_byte = 1 if scheme == "int8" else 2
    if codes.dim() != 2 or codes.shape[1] * per_byte != K:
        raise ShapeError(f"codes must be [out, {K // per_byte}] for {scheme} with {K} inputs, "
                         f"got {tuple(codes.shape)}")
    if a.dim() != 2 or a.shape[1] != K:
        raise ShapeError(f"A must be [rank, {K}], got {tuple(a.shape)}")
    if b.dim() != 2 or tuple(b.shape) != (N, r):
        raise ShapeError(f"B must be [{N}, {r}], got {tuple(b.shape)}")


@custom_op(f"{_NS}::qlora_fwd", mutates_args=())
def qlora_fwd(x: torch.Tensor, codes: torch.Tensor, scales: torch.Tensor,
              zeros: torch.Tensor | None, prepared: torch.Tensor | None, scheme: str, group: int,
              lean: bool, a: torch.Tensor, b: torch.Tensor,
              alpha: float) -> tuple[torch.Tensor, torch.Tensor]:
    """LoRA forward over a quantised base: ``x.deq(W)^T + (alpha/r).(x.A^T).B^T``
    (lora_quantized.metal:29-164 with the adapter of ops.py:91-94); bf16 x."""
    _check_q(x, codes, a, b, scheme)
    qw = _qweight(x, codes, scales, zeros, prepared, scheme, group, lean)
    y, saved = _k.qlora_linear_fwd(x.reshape(-1, x.shape[-1]), qw, a.to(x.dtype), b.to(x.dtype),
                                   alpha, save_xa=True)
    return y.reshape(*x.shape[:-1], codes.shape[0]), saved


@qlora_fwd.register_fake
def _qlora_fwd_fake(x, codes, scales, zeros, prepared, scheme, group, lean, a, b, alpha):
    _check_q(x, codes, a, b, scheme)
    return (x.new_empty((*x.shape[:-1], codes.shape[0])),
            x.new_empty(_saved_shape(x, a.shape[0])))


def _qlora_fwd_setup(ctx, inputs, output):
    x, codes, scales, zeros, prepared, scheme, group, lean, a, b, alpha = inputs
    ctx.mark_non_differentiable(output[1])
    ctx.save_for_backward(x, codes, scales, zeros, prepared, a, b, output[1])
    ctx.meta = (scheme, group, lean, alpha)


def _qlora_fwd_backward(ctx, dy, _dsaved):
    x, codes, scales, zeros, prepared, a, b, saved = ctx.saved_tensors
    scheme, group, lean, alpha = ctx.meta
    need_dx = ctx.needs_input_grad[0]
    dx, da, db = torch.ops.metal_lora.qlora_bwd(dy, x, codes, scales, zeros, prepared, scheme,
                                                group, lean, a, b, saved, alpha, 0.0, need_dx)
    return (dx if need_dx else None, None, None, None, None, None, None, None,
            da.to(a.dtype) if ctx.needs_input_grad[8] else None,
            db.to(b.dtype) if ctx.needs_input_grad[9] else None, None)


qlora_fwd.register_autograd(_qlora_fwd_backward, setup_context=_qlora_fwd_setup)


@custom_op(f"{_NS}::qlora_bwd", mutates_args=())
def qlora_bwd(dy: torch.Tensor, x: torch.Tensor, codes: torch.Tensor, scales: torch.Tensor,
              zeros: torch.Tensor | None, prepared: torch.Tensor | None, scheme: str, group: int,
              lean: bool, a: torch.Tensor, b: torch.Tensor, saved: torch.Tensor, alpha: float,
              clip_value: float, need_dx: bool) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(dx, dA, dB) through a frozen quantised base; dA/dB fp32."""
    _check_q(x, codes, a, b, scheme)
    qw = _qweight(x, codes, scales, zeros, prepared, scheme, group, lean)
    K, N = x.shape[-1], codes.shape[0]
    sv = saved if saved.numel() > 0 else None
    dx, da, db = _k.qlora_linear_bwd(dy.reshape(-1, N), x.reshape(-1, K), qw, a.to(x.dtype),
                                     b.to(x.dtype), alpha, sv, clip_value, need_dx=need_dx)
    dx = dx.reshape(x.shape) if need_dx else x.new_empty((0,))
    return dx, da, db


@qlora_bwd.register_fake
def _qlora_bwd_fake(dy, x, codes, scales, zeros, prepared, scheme, group, lean, a, b, saved,
                    alpha, clip_value, need_dx):
    _check_q(x, codes, a, b, scheme)
    dx = x.new_empty(x.shape) if need_dx else x.new_empty((0,))
    return (dx, a.new_empty(a.shape, dtype=torch.float32),
            b.new_empty(b.shape, dtype=torch.float32))


def qlora_linear(x: torch.Tensor, qweight: QuantizedWeight, a: torch.Tensor, b: torch.Tensor,
                 alpha: float = 16.0) -> torch.Tensor:
    """``y`` of ``torch.ops.metal_lora.qlora_fwd`` for a ``QuantizedWeight``:
    the traceable form of ``ops.qlora_forward``."""
    qw = qweight
    prepared = getattr(qw, "_prepared", None)
    if prepared is None and qw.codes.is_cuda:
        prepared = qw.prepared_scales()
    return torch.ops.metal_lora.qlora_fwd(x, qw.codes, qw.scales, qw.zeros, prepared, qw.scheme,
                                          qw.group, qw.lean, a, b, float(alpha))[0]


# ---------------------------------------------------------------- optimizer --

@custom_op(f"{_NS}::adamw_step", mutates_args=("param", "grad", "m", "v"))
def adamw_step(param: torch.Tensor, grad: torch.Tensor, m: torch.Tensor, v: torch.Tensor,
               gpu_state: torch.Tensor, lr: float, beta1: float, beta2: float, eps: float,
               wd: float, grad_scale: torch.Tensor | None = None) -> None:
    """In-place AdamW step of one tensor (kernels.py:615-643): param, m, v
    updated, grad zeroed; ``grad_scale`` (device float[2], element 0) scales
    the gradient (the trainer's global-norm clip factor)."""
    _k.lora_adamw_step_metal(param, grad, m, v, gpu_state, lr, beta1, beta2, eps, wd,
                             grad_scale=grad_scale)


@adamw_step.register_fake
def _adamw_step_fake(param, grad, m, v, gpu_state, lr, beta1, beta2, eps, wd, grad_scale=None):
    for name, t in (("grad", grad), ("m", m), ("v", v)):
        if t.dtype != torch.float32 or t.numel() != param.numel():
            raise ShapeError(f"{name} must be fp32 with param's size")
    return None


@custom_op(f"{_NS}::adam_state_step", mutates_args=("gpu_state",))
def adam_state_step(gpu_state: torch.Tensor, beta1: float, beta2: float) -> None:
    """gpu_state := [t+1, beta1^(t+1), beta2^(t+1)] on the device (kernels.py:484-499)."""
    _k.persistent_gpu_state_step(gpu_state, beta1, beta2)


@adam_state_step.register_fake
def _adam_state_step_fake(gpu_state, beta1, beta2):
    return None


def lora_linear(x: torch.Tensor, w0: torch.Tensor, a: torch.Tensor, b: torch.Tensor,
                alpha: float = 16.0) -> torch.Tensor:
    """``y`` of ``torch.ops.metal_lora.lora_fwd``: the traceable form of
    ``ops.lora_forward`` without dropout."""
    return torch.ops.metal_lora.lora_fwd(x, w0, a, b, float(alpha))[0]
