"""Property tests (hypothesis) of the host-side logic the kernels rely on:
rank padding keeps alpha/r and the product, the padded rank tile, token
shards, and the quantised-base pack format."""
import pytest
import torch
from hypothesis import given, settings
from hypothesis import strategies as st

from metallora_b200 import kernels, quant
from metallora_b200.distributed import shard_bounds
from metallora_b200.exceptions import QuantizationError


@settings(max_examples=40, deadline=None)
@given(r=st.integers(1, 256), k=st.integers(1, 40), n=st.integers(1, 40),
       alpha=st.floats(0.5, 512.0))
def test_pad_rank_keeps_the_scaled_product(r, k, n, alpha):
    g = torch.Generator().manual_seed(r * 1000 + k)
    a = torch.randn(r, k, generator=g, dtype=torch.float64)
    b = torch.randn(n, r, generator=g, dtype=torch.float64)
    a_p, b_p, alpha_p, r_p = kernels._pad_rank(a, b, alpha)
    assert r_p % 8 == 0 and r <= r_p < r + 8
    assert a_p.shape == (r_p, k) and b_p.shape == (n, r_p)
    assert not a_p[r:].any() and not b_p[:, r:].any()
    assert abs(alpha_p / r_p - alpha / r) <= 1e-12 * alpha / r
    torch.testing.assert_close((alpha_p / r_p) * b_p @ a_p, (alpha / r) * b @ a)


@given(r=st.integers(1, 4096))
def test_rank_tile_is_the_smallest_power_of_two_at_least_16(r):
    t = kernels.rank_tile(r)
    assert t >= max(r, 16) and t & (t - 1) == 0
    assert t == 16 or t // 2 < r


@given(n=st.integers(1, 10 ** 7), world=st.integers(1, 64))
def test_shards_partition_the_tokens(n, world):
    spans = [shard_bounds(n, rank, world) for rank in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
    sizes = [e - b for b, e in spans]
    assert max(sizes) - min(sizes) <= 1


@settings(max_examples=30, deadline=None)
@given(scheme=st.sampled_from(["nf4", "int4", "int8"]), n=st.integers(1, 48),
       k_groups=st.integers(1, 4), seed=st.integers(0, 2 ** 16))
def test_pack_round_trip_and_truncation(scheme, n, k_groups, seed):
    g = torch.Generator().manual_seed(seed)
    group = 64 if scheme == "nf4" else 128
    k = group * k_groups
    per_byte = 1 if scheme == "int8" else 2
    codes = torch.randint(0, 256, (n, k // per_byte), generator=g, dtype=torch.int32)
    codes = codes.to(torch.uint8)
    if scheme == "nf4":
        scales, zeros = torch.rand(n, k_groups, generator=g), None
    else:
        scales = torch.rand(n, k_groups, generator=g).half()
        zeros = torch.randint(0, 16, (n, k_groups), generator=g).half()
    qw = quant.from_reference_layout(scheme, codes, scales, zeros, (n, k), group)
    tensors, meta = quant.pack_quantized({"w": qw})
    back = quant.unpack_quantized(tensors, meta)["w"]
    assert torch.equal(back.codes, codes) and torch.equal(back.scales, scales)
    assert back.shape == (n, k) and back.group == group and back.scheme == scheme
    cut = dict(tensors)
    cut["w.scales"] = cut["w.scales"][:, :-1] if k_groups > 1 else cut["w.scales"][:0]
    with pytest.raises(QuantizationError):
        quant.unpack_quantized(cut, meta)
