"""Generates the golden vectors in tests/golden/*.npz.

The outputs come from the reference's own kernels run on the CPU
(``oracle/_ref/libmlref.so``, built from the reference's MSL sources by
``oracle/build_ref.py``); the inputs are seeded here (numpy PCG64, seed 0),
because the reference ships no fixtures and its MLX RNG cannot run here.

    python oracle/build_ref.py && python tests/golden/make_golden.py

Fixtures (all small):
  lora_fp32.npz   kernels.py:41-144 forward, kernels.py:249-308 dA/dB (clip
                  large so the per-token clamp is inactive, plus clip 0.05),
                  kernels.py:314-362 AdamW + maintenance step
  qlora_nf4.npz   lora_quantized.metal qlora_forward_nf4 + dequant_nf4 of every code
  qlora_int4.npz  lora_quantized.metal qlora_forward_int4 + dequant_int4
  train_fp16.npz  lora_train.metal forward (+Ax cache), backward, optimizer step
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import quant_oracle as qo  # noqa: E402
from oracle import ref  # noqa: E402

OUT = Path(__file__).resolve().parent


def lora_fp32(rng):
    bsz, seq, K, N, r, alpha = 2, 16, 128, 256, 16, 32.0
    x = rng.standard_normal((bsz, seq, K)).astype(np.float32)
    W0 = (rng.standard_normal((N, K)) / np.sqrt(K)).astype(np.float32)
    A = rng.uniform(-1 / np.sqrt(K), 1 / np.sqrt(K), (r, K)).astype(np.float32)
    B = (rng.standard_normal((N, r)) * np.sqrt(0.02)).astype(np.float32)
    dy = rng.standard_normal((bsz, seq, N)).astype(np.float32)
    y = ref.lora_forward_fused(x, W0, A, B, alpha)
    ga, gb = ref.lora_backward_fused(dy, x, A, B, alpha, 1e30)
    ga_c, gb_c = ref.lora_backward_fused(dy, x, A, B, alpha, 0.05)
    n = 1000
    p = rng.standard_normal(n).astype(np.float32)
    g = rng.standard_normal(n).astype(np.float32)
    m = (rng.standard_normal(n) * 0.1).astype(np.float32)
    v = np.abs(rng.standard_normal(n) * 0.01).astype(np.float32)
    state = np.array([1.0, 0.9, 0.999], np.float32)
    p1, g1, m1, v1 = ref.lora_adamw_step(p, g, m, v, state, 1e-3, 0.9, 0.999, 1e-8, 0.01)
    state2 = ref.lora_maintenance(state, 0.9, 0.999)
    np.savez_compressed(OUT / "lora_fp32.npz", x=x, W0=W0, A=A, B=B, dy=dy, alpha=alpha, y=y,
                        grad_A=ga, grad_B=gb, grad_A_clip005=ga_c, grad_B_clip005=gb_c,
                        adam_param=p, adam_grad=g, adam_m=m, adam_v=v, adam_state=state,
                        adam_param_out=p1, adam_grad_out=g1, adam_m_out=m1, adam_v_out=v1,
                        state_after_step=state2)


def qlora_nf4(rng):
    bsz, seq, K, N, r, alpha, bs = 1, 8, 256, 256, 16, 32.0, 64
    W = (rng.standard_normal((N, K)) / np.sqrt(K)).astype(np.float32)
    packed, absmax = qo.quantize_nf4(W, bs)
    x = rng.standard_normal((bsz, seq, K)).astype(np.float16)
    A = rng.uniform(-1 / 16, 1 / 16, (r, K)).astype(np.float16)
    B = (rng.standard_normal((N, r)) * 0.1).astype(np.float16)
    y = ref.qlora_forward_nf4(packed, absmax, x, A, B, alpha, bs)
    # every code in both nibbles, against a few absmax values
    codes = np.arange(256, dtype=np.uint8)
    am_vals = np.array([1.0, 0.03125, 0.0123, 3.7], np.float32)
    table = np.array([[[ref.dequant_nf4_scalar(c, h, a) for a in am_vals] for h in (0, 1)]
                      for c in codes], np.float32)
    np.savez_compressed(OUT / "qlora_nf4.npz", W=W, packed=packed, absmax=absmax, x=x, A=A, B=B,
                        alpha=alpha, block_size=bs, y=y, dequant_codes=codes,
                        dequant_absmax=am_vals, dequant_table=table)


def qlora_int4(rng):
    bsz, seq, K, N, r, alpha = 1, 8, 256, 256, 16, 32.0
    q = rng.integers(0, 16, (N, K), dtype=np.uint8)
    packed = qo.pack_nibbles(q)
    scales = (np.abs(rng.standard_normal(N)) * 0.01 + 1e-3).astype(np.float32)
    zeros = rng.integers(0, 16, N).astype(np.float32)
    x = rng.standard_normal((bsz, seq, K)).astype(np.float16)
    A = rng.uniform(-1 / 16, 1 / 16, (r, K)).astype(np.float16)
    B = (rng.standard_normal((N, r)) * 0.1).astype(np.float16)
    y = ref.qlora_forward_int4(packed, scales, zeros, x, A, B, alpha)
    sel = rng.integers(0, N * K, 512)
    d, k = sel // K, sel % K
    deq = np.array([ref.dequant_int4_scalar(packed[di, ki // 2], ki % 2, scales[di], zeros[di])
                    for di, ki in zip(d, k)], np.float32)
    np.savez_compressed(OUT / "qlora_int4.npz", packed=packed, scales=scales, zeros=zeros, x=x,
                        A=A, B=B, alpha=alpha, y=y, sel_row=d, sel_col=k, sel_dequant=deq)


def train_fp16(rng):
    bsz, seq, K, N, r, alpha = 1, 8, 128, 256, 8, 16.0
    x = rng.standard_normal((bsz, seq, K)).astype(np.float16)
    W0 = (rng.standard_normal((N, K)) / np.sqrt(K)).astype(np.float16)
    A = rng.uniform(-1 / np.sqrt(K), 1 / np.sqrt(K), (r, K)).astype(np.float16)
    B = (rng.standard_normal((N, r)) * 0.1).astype(np.float16)
    dy = rng.standard_normal((bsz, seq, N)).astype(np.float16)
    y, ax = ref.train_forward(x, W0, A, B, alpha)
    ga, gb = ref.train_backward(dy, x, ax, A, B, alpha, 1e30)
    mA = np.zeros(A.size, np.float32)
    vA = np.zeros(A.size, np.float32)
    mB = np.zeros(B.size, np.float32)
    vB = np.zeros(B.size, np.float32)
    outs = ref.optimizer_step(A, B, ga.ravel(), gb.ravel(), mA, vA, mB, vB, 1e-3, 0.9, 0.999,
                              1e-8, 0.0, 1)
    np.savez_compressed(OUT / "train_fp16.npz", x=x, W0=W0, A=A, B=B, dy=dy, alpha=alpha, y=y,
                        ax=ax, grad_A=ga, grad_B=gb, opt_A=outs[0], opt_B=outs[1],
                        opt_mA=outs[4], opt_vA=outs[5], opt_mB=outs[6], opt_vB=outs[7])


def main():
    if not ref.available():
        raise SystemExit("oracle/_ref/libmlref.so missing: run python oracle/build_ref.py first")
    rng = np.random.default_rng(0)
    lora_fp32(rng)
    qlora_nf4(rng)
    qlora_int4(rng)
    train_fp16(rng)
    for f in sorted(OUT.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
