"""CPU oracle for the LoRA-linear path.  TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
may import this module, and only as the checker or the timed CPU stand-in:
the product (``metallora_b200``) never calls it.

It restates, in numpy, the reference's pure-MLX op path -- the numerically
authoritative path of Wilbatronic/MetalLora -- in the same op order:

* forward           ``python/metal_lora/ops.py:69-103``
* A/B gradients     ``python/metal_lora/ops.py:143-155`` (clip of the final grads)
* dx                chain rule of ``ops.py:91-94``: ``dy@W0 + s*(dy@B)@A``
* merge             ``python/metal_lora/ops.py:162-172``
* layer wrapper     ``python/metal_lora/layers.py:83-106`` (reshape, bias after)
* global-norm clip  ``python/metal_lora/trainer.py:237-240``
* AdamW step        ``kernels.py:333-343`` (pinned by tests/test_parity.py:57-64)

Parity status: pinned.  ``tests/test_oracle_pin.py`` checks every function here
against the reference's own kernels run on the CPU (``oracle/_ref``, built by
``oracle/build_ref.py`` from the reference's MSL sources) and against the
golden vectors in ``tests/golden/`` that were generated from it.  MLX itself
(the reference's CPU backend) is not installable here, so the pin goes through
the reference's Metal kernels, which compute the same math.

All functions take and return numpy arrays.  ``acc`` selects the arithmetic
type (float32 by default, float64 for "truth" used to size tolerances).
"""
from __future__ import annotations

import numpy as np


def _as(a, acc):
    return np.asarray(a, dtype=acc)


def lora_forward(x, W0, A, B, alpha=16.0, acc=np.float32):
    """``ops.lora_forward`` pure-MLX path (ops.py:69-103), dropout 0.

    x [..., K] (2-D or 3-D like the reference), W0 [N, K], A [r, K], B [N, r].
    rank is read from ``B.shape[1]`` as at ops.py:73.
    """
    x = _as(x, acc)
    W0, A, B = _as(W0, acc), _as(A, acc), _as(B, acc)
    rank = B.shape[1]
    scale = acc(alpha / rank)
    w0x = np.matmul(x, W0.T)
    ax = np.matmul(x, A.T)
    bax = np.matmul(ax, B.T)
    return w0x + scale * bax


def lora_forward_with_cache(x, W0, A, B, alpha=16.0, acc=np.float32):
    """Forward that also returns ``ax = x@A.T`` (what the fused kernels save
    for the backward; lora_train.metal:66 stores the same quantity)."""
    x = _as(x, acc)
    W0, A, B = _as(W0, acc), _as(A, acc), _as(B, acc)
    scale = acc(alpha / B.shape[1])
    ax = np.matmul(x, A.T)
    return np.matmul(x, W0.T) + scale * np.matmul(ax, B.T), ax


def lora_layer_forward(x, W0, A, B, alpha=16.0, bias=None, acc=np.float32):
    """``LoRALinear.__call__`` (layers.py:83-106): any leading shape, bias added
    after the op."""
    x = _as(x, acc)
    shp = x.shape
    out = lora_forward(x.reshape(-1, shp[-1]), W0, A, B, alpha, acc)
    if bias is not None:
        out = out + _as(bias, acc)
    return out.reshape(*shp[:-1], out.shape[-1])


def lora_backward(grad_output, x, A, B, alpha=16.0, clip_value=1.0, acc=np.float32):
    """``ops.lora_backward`` pure-MLX path (ops.py:143-155) -> (grad_a, grad_b).

    Inputs are 3-D [batch, seq, features] as the reference requires
    (transpose axes (0, 2, 1) at ops.py:149,153).  rank from ``A.shape[0]``
    (ops.py:144).  ``clip_value=None`` skips the final clip (the autodiff
    gradients the trainer sees).
    """
    g = _as(grad_output, acc)
    x = _as(x, acc)
    A, B = _as(A, acc), _as(B, acc)
    if g.ndim == 2:
        g, x = g[None], x[None]
    rank = A.shape[0]
    scale = acc(alpha / rank)
    ax = np.matmul(x, A.T)
    grad_b = scale * np.sum(np.matmul(np.transpose(g, (0, 2, 1)), ax), axis=0)
    bt_grad = np.matmul(g, B)
    grad_a = scale * np.sum(np.matmul(np.transpose(bt_grad, (0, 2, 1)), x), axis=0)
    if clip_value is None:
        return grad_a, grad_b
    return np.clip(grad_a, -clip_value, clip_value), np.clip(grad_b, -clip_value, clip_value)


def lora_grad_x(grad_output, W0, A, B, alpha=16.0, acc=np.float32):
    """dx of ``w0x + s*((x@A.T)@B.T)`` (ops.py:91-94): ``dy@W0 + s*(dy@B)@A``."""
    g = _as(grad_output, acc)
    W0, A, B = _as(W0, acc), _as(A, acc), _as(B, acc)
    scale = acc(alpha / B.shape[1])
    return np.matmul(g, W0) + scale * np.matmul(np.matmul(g, B), A)


def merge_lora_weights(W0, A, B, alpha=16.0, acc=np.float32):
    """ops.py:162-172: ``W0 + (alpha / A.shape[0]) * (B @ A)``."""
    W0, A, B = _as(W0, acc), _as(A, acc), _as(B, acc)
    scale = acc(alpha / A.shape[0])
    return W0 + scale * np.matmul(B, A)


def clip_grad_norm(grads, max_norm, acc=np.float32):
    """trainer.py:237-240: scale every grad by min(1, max_norm/(||g||+1e-6))."""
    gs = [_as(g, acc) for g in grads]
    norm = np.sqrt(sum(np.sum(g * g, dtype=acc) for g in gs)).astype(acc)
    scale = np.minimum(acc(1.0), acc(max_norm) / (norm + acc(1e-6))).astype(acc)
    return [g * scale for g in gs], float(norm)


def adamw_step(param, grad, m, v, lr, beta1, beta2, eps, wd, step, acc=np.float32, b1t=None,
               b2t=None):
    """AdamW with bias correction, as written in the live kernel
    kernels.py:333-343 (and, up to the order of the g*g product, in
    tests/test_parity.py:57-64):
    m = b1*m + (1-b1)*g; v = b2*v + ((1-b2)*g)*g;
    p -= lr*(m/(1-b1^t) / (sqrt(v/(1-b2^t)) + eps) + wd*p).
    The operation order is the kernel's, so fp32 results are bit-identical to it.
    ``b1t``/``b2t`` override beta^step (the kernel reads them from its device
    state, where they are running products).  Returns (param, m, v)."""
    p, g = _as(param, acc), _as(grad, acc)
    m, v = _as(m, acc), _as(v, acc)
    b1t = acc(beta1) ** acc(step) if b1t is None else acc(b1t)
    b2t = acc(beta2) ** acc(step) if b2t is None else acc(b2t)
    m = acc(beta1) * m + (acc(1) - acc(beta1)) * g
    v = acc(beta2) * v + ((acc(1) - acc(beta2)) * g) * g
    m_hat = m / (acc(1) - b1t)
    v_hat = v / (acc(1) - b2t)
    p = p - acc(lr) * (m_hat / (np.sqrt(v_hat) + acc(eps)) + acc(wd) * p)
    return p, m, v


def lora_flops(M, K, N, r, backward=False):
    """Algorithmic FLOPs of one call (no credit for recomputation):
    forward 2M(KN + Kr + rN); backward (dx, dA, dB) 2M(NK + 2Nr + 2rK)."""
    if backward:
        return 2.0 * M * (N * K + 2 * N * r + 2 * r * K)
    return 2.0 * M * (K * N + K * r + r * N)


def multi_adapter_forward(x, W0, A_all, B_all, ids, alpha, dtype=np.float64):  # noqa: N803
    """Per-sample adapters over a shared base, as the reference's
    ``lora_multi_adapter`` kernel computes it (kernels/lora_kernels.metal:
    440-508): for sample b, ``out = x[b].W0^T + (alpha/rank).(x[b].A_id^T).B_id^T``
    with ``id = ids[b]``; ``W0 = None`` gives the LoRA term alone and
    ``alpha = rank`` gives ``MultiAdapterManager.forward_batched``
    (python/metal_lora/optimizations.py:193-217, einsum bsk,brk->bsr then
    bsr,bdr->bsd).  x [B, S, K]; A_all [n, r, K]; B_all [n, N, r]."""
    x = np.asarray(x, dtype)
    out = []
    for b, g in enumerate(ids):
        A = np.asarray(A_all[g], dtype)
        B = np.asarray(B_all[g], dtype)
        ax = x[b] @ A.T
        y = (alpha / A.shape[0]) * (ax @ B.T)
        if W0 is not None:
            y = x[b] @ np.asarray(W0, dtype).T + y
        out.append(y)
    return np.stack(out)


def embedding_forward(idx, E, A, B, alpha, dtype=np.float64):  # noqa: N803
    """LoRAEmbedding.__call__ (python/metal_lora/layers.py:220-225):
    base_emb = E[idx]; lora_emb = B[idx] @ A; out = base_emb + (alpha/rank) lora_emb.
    E [V, D], A [rank, D], B [V, rank]."""
    E, A, B = (np.asarray(t, dtype) for t in (E, A, B))
    idx = np.asarray(idx)
    return E[idx] + (alpha / A.shape[0]) * (B[idx] @ A)


def embedding_backward(dy, idx, A, B, alpha, dtype=np.float64):  # noqa: N803
    """Gradients of embedding_forward with respect to A and B (the table is
    frozen, layers.py:217-218): dA = s B[idx]^T dy, dB[v] = s sum_{t: idx=v} dy[t] A^T."""
    A, B = np.asarray(A, dtype), np.asarray(B, dtype)
    idx = np.asarray(idx).reshape(-1)
    dy = np.asarray(dy, dtype).reshape(idx.size, -1)
    s = alpha / A.shape[0]
    dA = s * (B[idx].T @ dy)
    dB = np.zeros_like(B)
    np.add.at(dB, idx, s * (dy @ A.T))
    return dA, dB
