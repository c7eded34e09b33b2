"""Pack format of quantised bases (``quant.save_quantized`` / ``load_quantized``,
``utils.save_quantized_bases`` / ``load_quantized_bases``).

CPU: round trips of NF4 / INT4 / INT8 weights are exact, and malformed packs
(wrong format tag, wrong shape or dtype, missing zero-points) are rejected.
GPU: a model whose bases were quantised on the GPU, saved and loaded into a
fresh model gives the same forward bit for bit.
"""
import json

import pytest
import torch
from torch import nn

from metallora_b200 import quant, utils
from metallora_b200.exceptions import AdapterError, QuantizationError
from metallora_b200.layers import LoRALinear


def _cpu_qweight(scheme, N=24, K=256, seed=0):
    g = torch.Generator().manual_seed(seed)
    group = 64 if scheme == "nf4" else 128
    codes = torch.randint(0, 256, (N, K // (1 if scheme == "int8" else 2)), generator=g,
                          dtype=torch.int32).to(torch.uint8)
    if scheme == "nf4":
        scales, zeros = torch.rand(N, K // group, generator=g), None
    else:
        scales = torch.rand(N, K // group, generator=g).half()
        zeros = torch.randint(0, 16, (N, K // group), generator=g).half()
    return quant.from_reference_layout(scheme, codes, scales, zeros, (N, K), group)


def test_pack_round_trip(tmp_path):
    ws = {"l0.q": _cpu_qweight("nf4"), "l0.up": _cpu_qweight("int4", N=40, seed=1),
          "l1.down": _cpu_qweight("int8", K=384, seed=2)}
    quant.save_quantized(ws, tmp_path / "p.safetensors")
    back = quant.load_quantized(tmp_path / "p.safetensors")
    assert set(back) == set(ws)
    for name, qw in ws.items():
        got = back[name]
        assert (got.scheme, got.group, got.shape) == (qw.scheme, qw.group, qw.shape)
        assert torch.equal(got.codes, qw.codes) and torch.equal(got.scales, qw.scales)
        assert (got.zeros is None) == (qw.zeros is None)
        if qw.zeros is not None:
            assert torch.equal(got.zeros, qw.zeros)


def test_pack_rejects_malformed():
    tensors, meta = quant.pack_quantized({"w": _cpu_qweight("int4")})
    with pytest.raises(QuantizationError):
        quant.unpack_quantized(tensors, {"format": "other", "weights": meta["weights"]})
    bad = dict(tensors)
    bad["w.codes"] = bad["w.codes"][:, :-1]
    with pytest.raises(QuantizationError):
        quant.unpack_quantized(bad, meta)
    bad = dict(tensors)
    bad["w.scales"] = bad["w.scales"].float()
    with pytest.raises(QuantizationError):
        quant.unpack_quantized(bad, meta)
    bad = {k: v for k, v in tensors.items() if k != "w.zeros"}
    with pytest.raises(QuantizationError):
        quant.unpack_quantized(bad, meta)
    m = json.loads(meta["weights"])
    m["w"]["scheme"] = "int3"
    with pytest.raises(QuantizationError):
        quant.unpack_quantized(tensors, {"format": meta["format"], "weights": json.dumps(m)})


class _Two(nn.Module):
    def __init__(self):
        super().__init__()
        self.a = LoRALinear(256, 24, rank=8, alpha=16.0)
        self.b = LoRALinear(256, 40, rank=8, alpha=16.0)


def test_model_bases_round_trip_cpu(tmp_path):
    src = _Two()
    src.a.qweight = _cpu_qweight("nf4", N=24)
    src.b.qweight = _cpu_qweight("int8", N=40, seed=3)
    utils.save_quantized_bases(src, tmp_path)
    dst = _Two()
    utils.load_quantized_bases(dst, tmp_path)
    for m_src, m_dst in ((src.a, dst.a), (src.b, dst.b)):
        assert torch.equal(m_dst.qweight.codes, m_src.qweight.codes)
        assert m_dst.W0.numel() == 0
    with pytest.raises(AdapterError):
        utils.save_quantized_bases(_Two(), tmp_path / "none")
    wrong = nn.Module()
    wrong.a = LoRALinear(256, 32, rank=8)
    with pytest.raises(AdapterError):
        utils.load_quantized_bases(wrong, tmp_path)


@pytest.mark.gpu
def test_model_bases_round_trip_gpu(cuda, tmp_path):
    torch.manual_seed(0)
    src = _Two().to(cuda).to(torch.bfloat16)
    with torch.no_grad():
        for m in (src.a, src.b):
            m.W0.copy_(torch.randn_like(m.W0) / 16)
            m.B.copy_(torch.randn_like(m.B) * 0.1)
    src.a.quantize_base("nf4")
    src.b.quantize_base("int4")
    utils.save_quantized_bases(src, tmp_path)
    utils.save_adapter(src, tmp_path)
    dst = _Two().to(cuda).to(torch.bfloat16)
    utils.load_quantized_bases(dst, tmp_path)
    utils.load_adapter(dst, tmp_path)
    x = torch.randn(64, 256, device=cuda).to(torch.bfloat16)
    with torch.no_grad():
        for m_src, m_dst in ((src.a, dst.a), (src.b, dst.b)):
            assert m_dst.qweight.codes.is_cuda
            assert torch.equal(m_dst(x), m_src(x))
