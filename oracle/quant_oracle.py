"""CPU oracle for the quantised-base LoRA path.  TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
may use this module; the product never imports it.

Restates in numpy:

* the NF4 codebook, ``kernels/lora_quantized.metal:10-15`` -- the reference's
  4-decimal literals, kept identical because dequantised values must be
  bit-exact with the reference;
* ``dequant_nf4`` (lora_quantized.metal:22-25): ``LEVELS[idx] * absmax`` in fp32,
  absmax index ``d*ceil(K/bs) + k//bs`` (:122,:135);
* ``dequant_int4`` (lora_quantized.metal:17-20): ``(q - zero) * scale`` in fp32;
* the nibble order of both shaders: byte ``W[d*K/2 + k/2]``, low nibble = even
  k, high nibble = odd k (:70-74, :140-144);
* the forward of ``qlora_forward_nf4`` / ``qlora_forward_int4`` as
  "dequantise, then the pure-MLX LoRA forward".

Group-wise int4/int8 (fp16 scale and zero per (row, group of ``group`` along K))
generalise the reference's per-row int4 (lora_quantized.metal:64-65); with
``group == K`` they reduce to it (with fp16 instead of fp32 scale/zero).

The reference ships no quantiser, so the quantisers below are this project's
definition (parity for them is unpinned; the GPU quantiser is checked
bit-exact against them):

* NF4: per (row, block of ``bs`` along K) ``absmax = max|w|``; code =
  argmin_i |w/absmax - LEVELS[i]|, ties to the lower index; an all-zero block
  gets absmax 0 and code 7 (level 0.0).
* int<b> asymmetric: per (row, group) ``scale = (max-min)/(2^b-1)`` computed in
  fp32 and rounded UP to fp16 (so the group's range always fits; 1.0 when it
  is 0), ``zero = clamp(rint(-min/scale), 0, 2^b-1)`` stored fp16,
  ``q = clamp(rint(w/scale) + zero, 0, 2^b-1)`` with round-half-even.

Dequantisation is pinned bit-exact against the reference's own
``dequant_nf4``/``dequant_int4`` (oracle/_ref) in tests/test_oracle_pin.py.
"""
from __future__ import annotations

import numpy as np

NF4_LEVELS = np.array(
    [-1.0, -0.6962, -0.5251, -0.3949, -0.2844, -0.1848, -0.0911, 0.0,
     0.0796, 0.1609, 0.2461, 0.3379, 0.4407, 0.5627, 0.7230, 1.0],
    dtype=np.float32,
)


# ---------------------------------------------------------------- packing ----

def pack_nibbles(q: np.ndarray) -> np.ndarray:
    """[N, K] uint8 codes (0..15), K even -> [N, K/2] bytes, low nibble = even k."""
    q = np.asarray(q, dtype=np.uint8)
    assert q.shape[1] % 2 == 0
    return (q[:, 0::2] & 0xF) | ((q[:, 1::2] & 0xF) << 4)


def unpack_nibbles(packed: np.ndarray, K: int) -> np.ndarray:
    """[N, K/2] bytes -> [N, K] codes (lora_quantized.metal:70-74)."""
    p = np.asarray(packed, dtype=np.uint8)
    out = np.empty((p.shape[0], K), dtype=np.uint8)
    out[:, 0::2] = p & 0xF
    out[:, 1::2] = (p >> 4) & 0xF
    return out


# -------------------------------------------------------------- dequantise ---

def dequant_nf4(packed, absmax, K, block_size=64) -> np.ndarray:
    """fp32 ``NF4_LEVELS[idx] * absmax[d*ceil(K/bs) + k//bs]`` (bit-exact)."""
    codes = unpack_nibbles(packed, K)
    N = codes.shape[0]
    nb = -(-K // block_size)
    am = np.asarray(absmax, dtype=np.float32).reshape(N, nb)
    am_full = np.repeat(am, block_size, axis=1)[:, :K]
    return NF4_LEVELS[codes] * am_full


def dequant_int_grouped(q, scales, zeros, K, group=128) -> np.ndarray:
    """fp32 ``(float(q) - float(zero)) * float(scale)`` per (row, group).

    ``q`` is [N, K] uint8 (unpacked: use ``unpack_nibbles`` for int4);
    ``scales``/``zeros`` are fp16 [N, ceil(K/group)]."""
    q = np.asarray(q, dtype=np.uint8)
    N = q.shape[0]
    ng = -(-K // group)
    s = np.asarray(scales, dtype=np.float16).astype(np.float32).reshape(N, ng)
    z = np.asarray(zeros, dtype=np.float16).astype(np.float32).reshape(N, ng)
    s_full = np.repeat(s, group, axis=1)[:, :K]
    z_full = np.repeat(z, group, axis=1)[:, :K]
    return (q.astype(np.float32) - z_full) * s_full


def dequant_int4_grouped(packed, scales, zeros, K, group=128) -> np.ndarray:
    return dequant_int_grouped(unpack_nibbles(packed, K), scales, zeros, K, group)


# --------------------------------------------------------------- quantise ---

def quantize_nf4(W, block_size=64):
    """fp32 [N, K] (K even) -> (packed [N, K/2] uint8, absmax [N, ceil(K/bs)] fp32)."""
    W = np.asarray(W, dtype=np.float32)
    N, K = W.shape
    nb = -(-K // block_size)
    pad = nb * block_size - K
    Wp = np.pad(W, ((0, 0), (0, pad))) if pad else W
    blocks = Wp.reshape(N, nb, block_size)
    absmax = np.max(np.abs(blocks), axis=2).astype(np.float32)
    safe = np.where(absmax == 0, np.float32(1), absmax)
    normed = (blocks / safe[:, :, None]).astype(np.float32)
    dist = np.abs(normed[..., None] - NF4_LEVELS)  # argmin takes the first (lowest) index on ties
    codes = np.argmin(dist, axis=-1).astype(np.uint8)
    codes = np.where((absmax == 0)[:, :, None], np.uint8(7), codes)
    codes = codes.reshape(N, nb * block_size)[:, :K]
    return pack_nibbles(codes), absmax


def quantize_int_grouped(W, bits, group=128):
    """fp32 [N, K] -> (q [N, K] uint8, scales fp16 [N, G], zeros fp16 [N, G])."""
    W = np.asarray(W, dtype=np.float32)
    N, K = W.shape
    ng = -(-K // group)
    qmax = np.float32(2 ** bits - 1)
    pad = ng * group - K
    if pad:
        # padded lanes repeat the row's last element so they do not move min/max
        Wp = np.concatenate([W, np.repeat(W[:, -1:], pad, axis=1)], axis=1)
    else:
        Wp = W
    g = Wp.reshape(N, ng, group)
    wmin = g.min(axis=2)
    wmax = g.max(axis=2)
    s32 = ((wmax - wmin) / qmax).astype(np.float32)
    scale = s32.astype(np.float16)
    low = scale.astype(np.float32) < s32
    scale[low] = np.nextafter(scale[low], np.float16(np.inf))  # round up
    scale = np.where(scale == 0, np.float16(1.0), scale)
    s32 = scale.astype(np.float32)
    zero = np.clip(np.rint((-wmin) / s32), 0, qmax).astype(np.float32)
    q = np.clip(np.rint(g / s32[:, :, None]) + zero[:, :, None], 0, qmax)
    q = q.astype(np.uint8).reshape(N, ng * group)[:, :K]
    return q, scale, zero.astype(np.float16)


def quantize_int4_grouped(W, group=128):
    q, s, z = quantize_int_grouped(W, 4, group)
    return pack_nibbles(q), s, z


def quantize_int8_grouped(W, group=128):
    return quantize_int_grouped(W, 8, group)


# ---------------------------------------------------------------- forward ---

def qlora_forward(x, W_deq, A, B, alpha, acc=np.float32):
    """``qlora_forward_*`` math: dequantised base + LoRA, restated as the
    pure-MLX forward on the dequantised weight (lora_quantized.metal:68-92)."""
    from .lora_oracle import lora_forward
    return lora_forward(x, W_deq, A, B, alpha, acc)
