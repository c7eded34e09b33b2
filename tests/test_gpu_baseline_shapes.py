"""GPU parity against the oracle at the full sizes of the benchmark
configurations (the other GPU test files cover ragged and small shapes):

* fp32 LoRALinear forward, x [4, 512, 4096], 4096 -> 4096, rank 16, alpha 32,
  and the merged (to_inference_mode) output: rel 1e-4 (reference path
  python/metal_lora/ops.py:91-94, merge :162-172, layers.py:108-117);
* NF4 base 11008 x 4096 (block 64, fp32 absmax), rank 64, alpha 128, at 512
  and 4096 tokens: forward and dx/dA/dB at the bf16 tolerance 2e-2
  (kernels/lora_quantized.metal:97-164 dequantisation, then ops.py:91-94 and
  its gradients :144-155);
* INT4/INT8 group-128 bases (fp16 scale and zero), 4096 -> 4096 and
  4096 -> 14336, rank 16, at 1 and 4096 tokens: forward unmerged and merged
  (dequantised base + (alpha/r) B.A in bf16), 2e-2.

Inputs follow the configurations' distributions: x ~ N(0,1), W ~ N(0,1/4096)
(variance), A ~ U(+-1/64), B ~ N(0, 0.02) (variance), seeded.  Tolerances are
normwise ||gpu - oracle|| / ||oracle|| per output plus the elementwise bound
|d| <= rtol |ref| + 3 rtol rms(ref).  The oracle runs the dequantised weight
in fp32 numpy (its own rounding, ~1e-6 relative, is far below the bf16
tolerance) and the fp32 config in fp64.
"""
import numpy as np
import pytest
import torch

from oracle import lora_oracle as lo
from oracle import quant_oracle as qo
from tests.test_gpu_lora import assert_close, status_ok

pytestmark = pytest.mark.gpu


def _draw(M, K, N, r, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g)
    W = torch.randn(N, K, generator=g) / 64
    A = (torch.rand(r, K, generator=g) * 2 - 1) / 64
    B = torch.randn(N, r, generator=g) * 0.02 ** 0.5
    dy = torch.randn(M, N, generator=g)
    return x, W, A, B, dy


def _np(t, dtype=np.float64):
    return t.detach().float().cpu().numpy().astype(dtype)


def test_fp32_forward_and_merged_full_size(cuda):
    """fp32, x [4, 512, 4096], 4096 -> 4096, rank 16, alpha 32, through
    LoRALinear; then to_inference_mode and the merged forward."""
    from metallora_b200.layers import LoRALinear
    x, W, A, B, _ = _draw(2048, 4096, 4096, 16, 0)
    layer = LoRALinear(4096, 4096, rank=16, alpha=32.0, device=cuda, dtype=torch.float32)
    with torch.no_grad():
        layer.W0.copy_(W)
        layer.A.copy_(A)
        layer.B.copy_(B)
    xd = x.reshape(4, 512, 4096).to(cuda)
    with torch.no_grad():
        y = layer(xd)
    torch.cuda.synchronize()
    xh, Wh, Ah, Bh = (t.numpy().astype(np.float64) for t in (x, W, A, B))
    ref = lo.lora_forward(xh, Wh, Ah, Bh, 32.0, np.float64)
    assert_close(y.reshape(2048, 4096), ref, 1e-4)
    layer.to_inference_mode()
    ref_w = lo.merge_lora_weights(Wh, Ah, Bh, 32.0, np.float64)
    assert_close(layer.W0, ref_w, 1e-4)
    assert int(torch.count_nonzero(layer.A)) == 0 and int(torch.count_nonzero(layer.B)) == 0
    with torch.no_grad():
        ym = layer(xd)
    torch.cuda.synchronize()
    assert_close(ym.reshape(2048, 4096), ref, 1e-4)
    assert status_ok()


@pytest.mark.parametrize("M", [512, 4096])
def test_nf4_full_shape_forward_backward(cuda, M):
    """NF4 11008 x 4096 (out x in), block 64, rank 64, alpha 128."""
    from metallora_b200 import kernels as K
    from metallora_b200 import quant
    Kd, N, r, alpha = 4096, 11008, 64, 128.0
    x, W, A, B, dy = _draw(M, Kd, N, r, 1)
    qw = quant.quantize(W.to(cuda), "nf4", 64)
    # the GPU quantiser against the oracle's on a band of rows (bit-exact)
    p_ref, am_ref = qo.quantize_nf4(W[:256].numpy(), 64)
    np.testing.assert_array_equal(qw.codes[:256].cpu().numpy(), p_ref)
    np.testing.assert_array_equal(qw.scales[:256].cpu().numpy(), am_ref)
    xb, Ab, Bb, dyb = (t.to(torch.bfloat16).to(cuda) for t in (x, A, B, dy))
    y, saved = K.qlora_linear_fwd(xb, qw, Ab, Bb, alpha, save_xa=True)
    dx, da, db = K.qlora_linear_bwd(dyb, xb, qw, Ab, Bb, alpha, saved, 0.0, True)
    torch.cuda.synchronize()
    Wf = qo.dequant_nf4(qw.codes.cpu().numpy(), qw.scales.cpu().numpy(), Kd, 64)
    xh, Ah, Bh, dyh = (_np(t, np.float32) for t in (xb, Ab, Bb, dyb))
    assert_close(y, lo.lora_forward(xh, Wf, Ah, Bh, alpha, np.float32), 2e-2)
    assert_close(dx, lo.lora_grad_x(dyh, Wf, Ah, Bh, alpha, np.float32), 2e-2)
    ga, gb = lo.lora_backward(dyh, xh, Ah, Bh, alpha, None, np.float64)
    assert_close(da, ga, 2e-2)
    assert_close(db, gb, 2e-2)
    assert status_ok()


@pytest.mark.parametrize("M", [1, 4096])
@pytest.mark.parametrize("N", [4096, 14336])
@pytest.mark.parametrize("scheme", ["int4", "int8"])
def test_int_grouped_full_shape_unmerged_and_merged(cuda, scheme, N, M):
    """INT4/INT8 group 128 (fp16 scale and zero), 4096 -> N, rank 16."""
    from metallora_b200 import kernels as K
    from metallora_b200 import quant
    Kd, r, alpha = 4096, 16, 32.0
    x, W, A, B, _ = _draw(M, Kd, N, r, 2)
    qw = quant.quantize(W.to(cuda), scheme, 128)
    bits = 4 if scheme == "int4" else 8
    q_ref, s_ref, z_ref = qo.quantize_int_grouped(W[:128].numpy(), bits, 128)
    np.testing.assert_array_equal(qw.scales[:128].cpu().numpy(), s_ref)
    np.testing.assert_array_equal(qw.zeros[:128].cpu().numpy(), z_ref)
    codes = qw.codes.cpu().numpy()
    q = qo.unpack_nibbles(codes, Kd) if bits == 4 else codes
    np.testing.assert_array_equal(q[:128], q_ref)
    Wf = qo.dequant_int_grouped(q, qw.scales.cpu().numpy(), qw.zeros.cpu().numpy(), Kd, 128)
    xb, Ab, Bb = (t.to(torch.bfloat16).to(cuda) for t in (x, A, B))
    y, _ = K.qlora_linear_fwd(xb, qw, Ab, Bb, alpha)
    Wm = K.merge(quant.dequantize(qw, torch.bfloat16), Ab, Bb, alpha)
    ym = K.linear(xb, Wm)
    torch.cuda.synchronize()
    xh, Ah, Bh = (_np(t, np.float32) for t in (xb, Ab, Bb))
    ref = lo.lora_forward(xh, Wf, Ah, Bh, alpha, np.float32)
    assert_close(y, ref, 2e-2)
    assert_close(ym, ref, 2e-2)
    # the merged weight itself against the oracle's merge of the dequantised base
    ref_w = lo.merge_lora_weights(Wf, Ah, Bh, alpha, np.float32)
    rows = slice(0, 512)
    assert_close(Wm[rows], ref_w[rows], 2e-2)
    assert status_ok()
