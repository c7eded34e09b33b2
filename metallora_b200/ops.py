"""LoRA operations (reference: python/metal_lora/ops.py), on sm_100a kernels.

Same function names, arguments and defaults as the reference so callers can
switch imports.  ``use_metal``/``kernel_kwargs`` are accepted and ignored: there
is exactly one implementation, the CUDA one, and no fallback.  All tensors must
be CUDA tensors; bf16, fp16 or fp32 (fp32 runs as split-precision bf16
tensor-core GEMMs, see ``kernels``).
"""
from __future__ import annotations

import torch

from . import kernels as _k
from .exceptions import ShapeError


def _sink_accumulates(sink) -> bool:
    return sink is None or len(sink) < 3 or bool(sink[2])


class _LoRALinearFn(torch.autograd.Function):
    """y = x.W0^T + s.(x.A^T).B^T with the fused backward (dx, dA, dB in one
    launch sequence).  W0 gets a gradient only when it requires one (the
    reference freezes it by default, layers.py:77-78).

    A/B may be kept in a wider dtype than x (fp32 master factors with bf16
    compute): they are cast for the kernels and their gradients returned in
    their own dtype.  ``compute`` optionally supplies ready-made casts, and
    ``sink`` = (gA, gB) fp32 buffers receives the LoRA gradients by in-kernel
    accumulation instead of autograd (the trainer's flat gradient buffer);
    (gA, gB, False) writes them over the buffers' contents instead.  A fourth
    element ``on_grads`` (a callable) is called once dA/dB are enqueued and
    before the dx GEMM is: work it starts on another stream (a gradient
    exchange) overlaps that GEMM."""

    @staticmethod
    def forward(ctx, x2d, w0, a, b, alpha, compute, sink):
        a_c, b_c = compute if compute is not None else (a.to(x2d.dtype), b.to(x2d.dtype))
        y, saved = _k.lora_linear_fwd(x2d, w0, a_c, b_c, alpha, save_xa=True)
        ctx.save_for_backward(x2d, w0, a_c, b_c, saved)
        ctx.alpha = alpha
        ctx.sink = sink
        ctx.ab_dtypes = (a.dtype, b.dtype)
        return y

    @staticmethod
    def backward(ctx, dy):
        x2d, w0, a_c, b_c, saved = ctx.saved_tensors
        need_dx = ctx.needs_input_grad[0]
        sink = ctx.sink
        on_grads = sink[3] if sink is not None and len(sink) > 3 else None
        if on_grads is not None and need_dx and x2d.dtype != torch.float32:
            finish = _k.lora_linear_bwd_split(dy.contiguous(), x2d, w0, a_c, b_c, ctx.alpha,
                                              saved, sink[0], sink[1],
                                              accumulate=_sink_accumulates(sink))
            on_grads()
            dx, da, db = finish(), sink[0], sink[1]
        else:
            same = ctx.ab_dtypes[0] == ctx.ab_dtypes[1] == x2d.dtype  # 16-bit grads direct
            dx, da, db = _k.lora_linear_bwd(dy.contiguous(), x2d, w0 if need_dx else None, a_c,
                                            b_c, ctx.alpha, saved, 0.0, need_dx=need_dx,
                                            da_out=sink[0] if sink else None,
                                            db_out=sink[1] if sink else None,
                                            accumulate=_sink_accumulates(sink),
                                            grad_dtype=x2d.dtype if same else None)
            if on_grads is not None:
                on_grads()
        dw0 = None
        if ctx.needs_input_grad[1]:
            # trainable base weight (freeze_base=False): plain library GEMM
            dw0 = (dy.t().float() @ x2d.float()).to(w0.dtype)
        if dx is not None and not need_dx:
            dx = None
        if sink is not None:
            return dx, dw0, None, None, None, None, None
        da = da.to(ctx.ab_dtypes[0]) if ctx.needs_input_grad[2] else None
        db = db.to(ctx.ab_dtypes[1]) if ctx.needs_input_grad[3] else None
        return dx, dw0, da, db, None, None, None


class _QLoRALinearFn(torch.autograd.Function):
    """The LoRA linear over a frozen quantised base (QLoRA): no gradient for
    the base; A/B handled as in _LoRALinearFn."""

    @staticmethod
    def forward(ctx, x2d, a, b, qw, alpha, compute, sink):
        a_c, b_c = compute if compute is not None else (a.to(x2d.dtype), b.to(x2d.dtype))
        y, saved = _k.qlora_linear_fwd(x2d, qw, a_c, b_c, alpha, save_xa=True)
        ctx.save_for_backward(x2d, a_c, b_c, saved)
        ctx.qw, ctx.alpha, ctx.sink = qw, alpha, sink
        ctx.ab_dtypes = (a.dtype, b.dtype)
        return y

    @staticmethod
    def backward(ctx, dy):
        x2d, a_c, b_c, saved = ctx.saved_tensors
        sink = ctx.sink
        need_dx = ctx.needs_input_grad[0]
        dx, da, db = _k.qlora_linear_bwd(dy.contiguous(), x2d, ctx.qw, a_c, b_c, ctx.alpha, saved,
                                         0.0, need_dx=need_dx,
                                         da_out=sink[0] if sink else None,
                                         db_out=sink[1] if sink else None,
                                         accumulate=_sink_accumulates(sink))
        if sink is not None and len(sink) > 3 and sink[3] is not None:
            sink[3]()
        if sink is not None:
            return dx, None, None, None, None, None, None
        da = da.to(ctx.ab_dtypes[0]) if ctx.needs_input_grad[1] else None
        db = db.to(ctx.ab_dtypes[1]) if ctx.needs_input_grad[2] else None
        return dx, da, db, None, None, None, None


def qlora_forward(x, qweight, A, B, alpha: float = 16.0, _compute=None, _sink=None):  # noqa: N803
    """LoRA forward over a quantised base (``quant.QuantizedWeight``):
    ``x.deq(W)^T + (alpha/rank).(x.A^T).B^T`` with the dequantisation fused
    into the GEMM (replaces qlora_forward_nf4/int4, lora_quantized.metal:29-164)."""
    shp = x.shape
    out = _QLoRALinearFn.apply(x.reshape(-1, shp[-1]), A, B, qweight, float(alpha), _compute,
                               _sink)
    return out.reshape(*shp[:-1], qweight.shape[0])


def _apply(x2d, W0, A, B, alpha, compute=None, sink=None):
    return _LoRALinearFn.apply(x2d, W0, A, B, float(alpha), compute, sink)


def lora_forward(x, W0, A, B, alpha: float = 16.0, dropout: float = 0.0,  # noqa: N803
                 training: bool = False, use_metal: bool = True, kernel_kwargs: dict | None = None,
                 _compute=None, _sink=None):
    """LoRA forward ``h = x.W0^T + (alpha/rank).(x.A^T).B^T`` (ops.py:32-103).

    x is [batch, seq, in] or [seq, in] (any leading shape works); rank is read
    from ``B.shape[1]`` (ops.py:73).  With ``training`` and ``dropout > 0`` the
    dropout mask multiplies the LoRA term only, as at ops.py:96-98.
    """
    if x.shape[-1] != W0.shape[1]:
        raise ShapeError(f"x last dim {x.shape[-1]} != in_features {W0.shape[1]}")
    shp = x.shape
    x2d = x.reshape(-1, shp[-1])
    if training and dropout > 0:
        # ops.py:96-98: output = w0x + scale * bax * mask / (1 - dropout)
        zero_b = torch.zeros_like(B)
        w0x = _apply(x2d, W0, A, zero_b, alpha)
        scale = alpha / B.shape[1]
        bax = (x2d @ A.t()) @ B.t()
        mask = torch.bernoulli(torch.full_like(bax, 1.0 - dropout))
        out = w0x + scale * bax * mask / (1.0 - dropout)
    else:
        out = _apply(x2d, W0, A, B, alpha, _compute, _sink)
    return out.reshape(*shp[:-1], W0.shape[0])


def lora_forward_inference(x, w_merged):
    """Merged-weight forward (ops.py:106-114): ``x.W'^T`` with no adapter."""
    shp = x.shape
    y = _k.linear(x.reshape(-1, shp[-1]), w_merged)
    return y.reshape(*shp[:-1], w_merged.shape[0])


def lora_backward(grad_output, x, A, B, alpha: float = 16.0, clip_value: float = 1.0,  # noqa: N803
                  use_metal: bool = True):
    """Gradients of A and B (ops.py:117-155), clipped elementwise to
    +-clip_value after the full reduction, returned in A's/B's dtype."""
    g = grad_output.reshape(-1, grad_output.shape[-1])
    xx = x.reshape(-1, x.shape[-1])
    clip = float(clip_value) if clip_value is not None else 0.0
    _, da, db = _k.lora_linear_bwd(g, xx, None, A, B, alpha, None, clip, need_dx=False)
    return da.to(A.dtype), db.to(B.dtype)


# ops.py:158-159
lora_backward_efficient = lora_backward


def merge_lora_weights(W0, A, B, alpha: float = 16.0):  # noqa: N803
    """``W0 + (alpha/A.shape[0]) . B.A`` (ops.py:162-172) on the merge kernel."""
    return _k.merge(W0, A, B, alpha)


def unmerge_lora_weights(w_merged, W0, A, B, alpha: float = 16.0):  # noqa: N803
    """Recovers (A, B) from merged weights by truncated SVD (ops.py:175-193).
    Not on the hot path: uses torch.linalg.svd."""
    rank = A.shape[0]
    scale = alpha / rank
    delta = (w_merged.float() - W0.float()) / scale
    u, s, vt = torch.linalg.svd(delta, full_matrices=False)
    sqrt_s = torch.sqrt(s[:rank])
    a_rec = torch.diag(sqrt_s) @ vt[:rank, :]
    b_rec = u[:, :rank] @ torch.diag(sqrt_s)
    return a_rec.to(A.dtype), b_rec.to(B.dtype)


def multi_adapter_forward(x, W0, adapters_A, adapters_B, adapter_ids, alpha: float = 16.0):  # noqa: N803
    """Per-sample adapters over a shared base (the ``lora_multi_adapter`` kernel,
    kernels/lora_kernels.metal:440-508): ``y[b] = x[b].W0^T + (alpha/r)
    (x[b].A_id^T).B_id^T`` with ``id = adapter_ids[b]``.

    x [B, S, K]; W0 [N, K] or None (LoRA term only); adapters_A [n, r, K];
    adapters_B [n, N, r]; adapter_ids: ints, one per sample.  Only the
    adapters the batch uses are stacked; more than fit one launch
    (n * r <= 256) are applied in groups.
    """
    if x.dim() == 2:
        x = x.unsqueeze(0)
    Bsz, S, K = x.shape
    n_all, r, _ = adapters_A.shape
    N = adapters_B.shape[1]
    # ids are small host data: grouping and per-token ids are built on the host
    # (a CUDA tensor of ids is read back once)
    ids = [int(i) for i in (adapter_ids.tolist() if torch.is_tensor(adapter_ids) else adapter_ids)]
    if len(ids) != Bsz:
        raise ShapeError(f"{len(ids)} adapter ids for {Bsz} samples")
    if any(i < 0 or i >= n_all for i in ids):
        raise ShapeError(f"adapter ids must be in [0, {n_all})")
    x2d = x.reshape(-1, K)
    used = sorted(set(ids))
    r8 = (r + 7) // 8 * 8
    per = max(1, _k.MAX_STACKED_RANK // r8)
    y = None
    for g0 in range(0, len(used), per):
        group = used[g0:g0 + per]
        sel = torch.tensor(group, dtype=torch.int64).to(x.device, non_blocking=True)
        a, b = adapters_A.index_select(0, sel).to(x.dtype), adapters_B.index_select(0, sel).to(x.dtype)
        if r8 != r:  # zero-padded rank, alpha/r unchanged
            a = torch.nn.functional.pad(a, (0, 0, 0, r8 - r))
            b = torch.nn.functional.pad(b, (0, r8 - r))
        a_stack = a.reshape(len(group) * r8, K)
        b_stack = b.permute(1, 0, 2).reshape(N, len(group) * r8)
        slot = {g: j for j, g in enumerate(group)}
        tok_host = torch.tensor([slot.get(i, -1) for i in ids], dtype=torch.int32)
        tok = tok_host.repeat_interleave(S).to(x.device, non_blocking=True)
        base = W0.to(x.dtype) if (W0 is not None and y is None) else None
        part = _k.multi_lora_fwd(x2d, base, a_stack, b_stack, tok, r8, float(alpha) * r8 / r)
        y = part if y is None else y + part
    return y.reshape(Bsz, S, N)
