"""GPU tests of the quantised-base path (NF4, INT4, INT8).

* quantisers: bit-exact against oracle/quant_oracle.py;
* dequantisers: fp32 values bit-exact against the oracle and the reference's
  own dequant (golden table from kernels/lora_quantized.metal);
* fused QLoRA forward/backward: within the bf16 tolerance of the oracle, and
  bitwise equal to the dense kernels run on the dequantised bf16 weight (the
  dequantisation inside the main loop produces exactly those operands).
"""
import numpy as np
import pytest
import torch

from oracle import lora_oracle as lo
from oracle import quant_oracle as qo
from tests.conftest import rel_err

pytestmark = pytest.mark.gpu


def _w(N, K, seed, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(N, K, generator=g) / K ** 0.5).to(dtype)


@pytest.mark.parametrize("wdtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("scheme,group", [("nf4", 64), ("nf4", 128), ("int4", 128), ("int4", 64),
                                          ("int8", 128), ("int8", 256)])
def test_quantize_and_dequantize_bit_exact(cuda, scheme, group, wdtype):
    from metallora_b200 import quant
    W = _w(96, 640, 1, wdtype)
    Wh = W.float().numpy()
    qw = quant.quantize(W.to(cuda), scheme, group)
    torch.cuda.synchronize()
    if scheme == "nf4":
        p, am = qo.quantize_nf4(Wh, group)
        np.testing.assert_array_equal(qw.codes.cpu().numpy(), p)
        np.testing.assert_array_equal(qw.scales.cpu().numpy(), am)
        ref = qo.dequant_nf4(p, am, 640, group)
    else:
        bits = 4 if scheme == "int4" else 8
        q, s, z = qo.quantize_int_grouped(Wh, bits, group)
        codes = qo.pack_nibbles(q) if bits == 4 else q
        np.testing.assert_array_equal(qw.codes.cpu().numpy(), codes)
        np.testing.assert_array_equal(qw.scales.cpu().numpy(), s)
        np.testing.assert_array_equal(qw.zeros.cpu().numpy(), z)
        ref = qo.dequant_int_grouped(q, s, z, 640, group)
    np.testing.assert_array_equal(quant.dequantize(qw, torch.float32).cpu().numpy(), ref)
    bf = quant.dequantize(qw, torch.bfloat16)
    assert torch.equal(bf.cpu(), torch.from_numpy(ref).to(torch.bfloat16))


def test_dequantize_matches_reference_nf4_table(cuda, golden):
    """Every code byte, both nibbles, against the reference's dequant_nf4."""
    from metallora_b200 import quant
    g = golden("qlora_nf4.npz")
    codes = torch.from_numpy(np.tile(g["dequant_codes"][None, :], (4, 1))).to(cuda)  # [4, 256]
    am = torch.from_numpy(np.repeat(g["dequant_absmax"][:, None], 8, axis=1)).to(cuda)  # [4, 8]
    qw = quant.from_reference_layout("nf4", codes, am, None, (4, 512), 64)
    out = quant.dequantize(qw, torch.float32).cpu().numpy()  # [4, 512]
    table = g["dequant_table"]  # [byte, nibble, absmax]
    for i in range(4):
        np.testing.assert_array_equal(out[i, 0::2], table[:, 0, i])
        np.testing.assert_array_equal(out[i, 1::2], table[:, 1, i])


SHAPES = [(256, 512, 768, 16), (300, 1024, 520, 8), (1, 4096, 1024, 64), (513, 256, 256, 32),
          (130, 512, 264, 16)]


@pytest.mark.parametrize("lean", [False, True], ids=["staged", "lean"])
@pytest.mark.parametrize("scheme,group", [("nf4", 64), ("int4", 128), ("int8", 128),
                                          ("nf4", 256)])
@pytest.mark.parametrize("shape", SHAPES)
def test_qlora_forward_backward(cuda, scheme, group, shape, lean):
    """staged = dequantise into the workspace + dense kernels; lean = the fused
    kernel that dequantises in its main loop."""
    from metallora_b200 import kernels as K
    from metallora_b200 import quant
    M, Kd, N, r = shape
    g = torch.Generator().manual_seed(3)
    qw = quant.quantize(_w(N, Kd, 2).to(cuda), scheme, group, lean=lean)
    x = torch.randn(M, Kd, generator=g).to(torch.bfloat16).to(cuda)
    A = ((torch.rand(r, Kd, generator=g) * 2 - 1) / Kd ** 0.5).to(torch.bfloat16).to(cuda)
    B = (torch.randn(N, r, generator=g) * 0.1).to(torch.bfloat16).to(cuda)
    dy = torch.randn(M, N, generator=g).to(torch.bfloat16).to(cuda)
    Wb = quant.dequantize(qw, torch.bfloat16)
    h = lambda t: t.float().cpu().numpy().astype(np.float64)  # noqa: E731
    Wf = quant.dequantize(qw, torch.float32).cpu().numpy()
    ref = lo.lora_forward(h(x), Wf, h(A), h(B), 32.0, np.float64)
    # tensor-core paths (staged or fused dequant): the operand is exactly
    # bf16(deq(W)), so each equals the dense kernel on that weight; the decode
    # path (M <= 16, no saved intermediate) multiplies the integer codes and
    # scales each quad in fp32, so it agrees with the dense decode within bf16
    # rounding
    y_fast, _ = K.qlora_linear_fwd(x, qw, A, B, 32.0)
    y, saved = K.qlora_linear_fwd(x, qw, A, B, 32.0, save_xa=True)
    y_dense_fast, _ = K.lora_linear_fwd(x, Wb, A, B, 32.0)
    y_dense, _ = K.lora_linear_fwd(x, Wb, A, B, 32.0, save_xa=True)
    torch.cuda.synchronize()
    assert torch.equal(y, y_dense)
    assert rel_err(h(y_fast), h(y_dense_fast)) < 1e-2
    assert rel_err(h(y), ref) < 2e-2 and rel_err(h(y_fast), ref) < 2e-2
    dx, da, db = K.qlora_linear_bwd(dy, x, qw, A, B, 32.0, saved, 0.0, True)
    dxd, dad, dbd = K.lora_linear_bwd(dy, x, Wb, A, B, 32.0, saved, 0.0, True)
    torch.cuda.synchronize()
    assert torch.equal(dx, dxd) and torch.equal(da, dad) and torch.equal(db, dbd)
    assert rel_err(h(dx), lo.lora_grad_x(h(dy), Wf, h(A), h(B), 32.0, np.float64)) < 2e-2
    from metallora_b200 import _lib
    assert _lib.device_status(reset=True) == 0


@pytest.mark.parametrize("scheme,group", [("nf4", 64), ("int4", 128), ("int8", 128), ("nf4", 256),
                                          ("int4", 64), ("int8", 256)])
@pytest.mark.parametrize("M", [1, 5, 16])
@pytest.mark.parametrize("shape", [(4096, 11008, 64), (11008, 4096, 16), (512, 1000, 8)])
def test_qlora_decode(cuda, scheme, group, M, shape):
    """Decode kernel (M <= 16) against the oracle's dequantised weight in fp64,
    and bitwise repeatable."""
    from metallora_b200 import kernels as K
    from metallora_b200 import quant
    Kd, N, r = shape
    g = torch.Generator().manual_seed(21)
    qw = quant.quantize(_w(N, Kd, 8).to(cuda), scheme, group)
    x = torch.randn(M, Kd, generator=g).to(torch.bfloat16).to(cuda)
    A = ((torch.rand(r, Kd, generator=g) * 2 - 1) / Kd ** 0.5).to(torch.bfloat16).to(cuda)
    B = (torch.randn(N, r, generator=g) * 0.1).to(torch.bfloat16).to(cuda)
    y1, _ = K.qlora_linear_fwd(x, qw, A, B, 32.0)
    y2, _ = K.qlora_linear_fwd(x, qw, A, B, 32.0)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
    h = lambda t: t.float().cpu().numpy().astype(np.float64)  # noqa: E731
    Wf = quant.dequantize(qw, torch.float32).cpu().numpy()
    assert rel_err(h(y1), lo.lora_forward(h(x), Wf, h(A), h(B), 32.0, np.float64)) < 1e-2
    from metallora_b200 import _lib
    assert _lib.device_status(reset=True) == 0


def test_reference_qlora_nf4_golden_through_gpu(cuda, golden):
    """The reference's qlora_forward_nf4 output on its own inputs (fp16 there,
    bf16 here) within the bf16 tolerance."""
    from metallora_b200 import kernels as K
    from metallora_b200 import quant
    g = golden("qlora_nf4.npz")
    N, K2 = g["packed"].shape
    qw = quant.from_reference_layout("nf4", torch.from_numpy(g["packed"]).to(cuda),
                                     torch.from_numpy(g["absmax"]).to(cuda), None, (N, 2 * K2),
                                     int(g["block_size"]))
    bf = lambda a: torch.from_numpy(a.astype(np.float32)).to(torch.bfloat16).to(cuda)  # noqa: E731
    y, _ = K.qlora_linear_fwd(bf(g["x"].reshape(-1, 2 * K2)), qw, bf(g["A"]), bf(g["B"]),
                              float(g["alpha"]))
    assert rel_err(y.float().cpu().numpy(), g["y"].reshape(y.shape).astype(np.float64)) < 2e-2


def test_qlora_layer_and_trainer(cuda, tmp_path):
    from metallora_b200.layers import LoRALinear
    from metallora_b200.trainer import LoRATrainer, TrainingConfig
    layer = LoRALinear(512, 768, rank=16, alpha=32.0, device=cuda, dtype=torch.bfloat16)
    with torch.no_grad():
        layer.W0.copy_(_w(768, 512, 4).to(cuda))
        layer.B.normal_(0, 0.1)
    x = torch.randn(4, 64, 512, device=cuda, dtype=torch.bfloat16)
    y_dense = layer(x)
    layer.quantize_base("nf4", 64)
    assert layer.W0.numel() == 0 and layer.qweight.nbytes() < 768 * 512 // 2 + 768 * 8 * 4 + 1
    y_q = layer(x)
    assert float((y_q.float() - y_dense.float()).norm().detach() / y_dense.float().norm().detach()) < 0.15
    model = torch.nn.Sequential(layer)
    tr = LoRATrainer(model, TrainingConfig(rank=16, alpha=32.0, output_dir=str(tmp_path)))
    tgt = torch.randn_like(y_q)
    l0 = tr._training_step({"input_ids": x, "target_output": tgt})["loss"]
    for _ in range(20):
        l1 = tr._training_step({"input_ids": x, "target_output": tgt})["loss"]
    assert l1 < l0
