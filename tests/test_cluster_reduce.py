"""Rank-projection and weight-gradient kernels reduce their split partial sums
across a thread-block cluster through distributed shared memory.  These
shapes drive every cluster size (1, 2, 4, 8 splits on 148 SMs), padded ranks
and rank 256 (two 128-column passes); results are checked against an fp32
torch computation on the same bf16 inputs (normwise relative error, bf16
tolerance 2e-2) and for bitwise repeatability."""
import pytest
import torch

from metallora_b200 import _lib, kernels

SHAPES = [  # (M, K, N, r): fwd/bwd rank splits, weight-gradient splits
    (4096, 4096, 512, 16),   # 8, 8, 8
    (1024, 512, 768, 64),    # 2, 2, 4
    (256, 256, 384, 128),    # 1, 1, 1
    (16384, 1024, 256, 32),  # 2, 2, 8
    (2048, 4096, 512, 256),  # 8, 8, 8 (two column passes)
    (640, 1024, 256, 24),    # 4, 4, 2 (rank padded to 32)
]


def _rel(got, ref):
    return float((got.float() - ref).norm() / ref.norm().clamp_min(1e-30))


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,N,r", SHAPES)
def test_cluster_split_reduction(cuda, M, K, N, r):
    g = torch.Generator(device=cuda).manual_seed(11)
    bf = torch.bfloat16
    x = torch.randn(M, K, device=cuda, generator=g).to(bf)
    w = (torch.randn(N, K, device=cuda, generator=g) / K ** 0.5).to(bf)
    a = (torch.randn(r, K, device=cuda, generator=g) / K ** 0.5).to(bf)
    b = (torch.randn(N, r, device=cuda, generator=g) * 0.1).to(bf)
    dy = torch.randn(M, N, device=cuda, generator=g).to(bf)
    alpha = 2.0 * r
    s = alpha / r
    y, saved = kernels.lora_linear_fwd(x, w, a, b, alpha, save_xa=True)
    dx, da, db = kernels.lora_linear_bwd(dy, x, w, a, b, alpha, saved)
    dx2, da2, db2 = kernels.lora_linear_bwd(dy, x, w, a, b, alpha, saved)
    torch.cuda.synchronize()
    assert _lib.device_status(reset=True) == 0
    assert torch.equal(da, da2) and torch.equal(db, db2) and torch.equal(dx, dx2)

    xf, wf, af, bf32, dyf = (t.float() for t in (x, w, a, b, dy))
    xa = s * xf @ af.t()
    u = s * dyf @ bf32
    assert _rel(y, xf @ wf.t() + xa @ bf32.t()) < 2e-2
    assert _rel(dx, dyf @ wf + u @ af) < 2e-2
    assert _rel(da, u.t() @ xf) < 2e-2
    assert _rel(db, dyf.t() @ xa) < 2e-2
