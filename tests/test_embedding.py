"""LoRAEmbedding (layers.py:194-230): oracle on CPU; forward, gradients,
merge and bad indices on the GPU."""
import numpy as np
import pytest
import torch

from oracle import lora_oracle as lo
from tests.conftest import rel_err


def _case(V, D, r, T, seed):
    g = torch.Generator().manual_seed(seed)
    E = torch.randn(V, D, generator=g) * 0.02
    A = (torch.rand(r, D, generator=g) * 2 - 1) / D ** 0.5
    B = torch.randn(V, r, generator=g) * 0.1
    idx = torch.randint(0, V, (T,), generator=g)
    idx[: T // 4] = idx[0]  # repeated indices
    return E, A, B, idx


def test_oracle_embedding_matches_gather_plus_lora():
    E, A, B, idx = _case(50, 24, 8, 40, 0)
    out = lo.embedding_forward(idx.numpy(), E.numpy(), A.numpy(), B.numpy(), 16.0)
    for t, i in enumerate(idx.tolist()):
        ref = E[i].double().numpy() + 2.0 * (B[i].double().numpy() @ A.double().numpy())
        np.testing.assert_allclose(out[t], ref, rtol=1e-12, atol=1e-12)
    # gradient of <dy, out> by finite differences on one entry of A and of B
    dy = np.random.default_rng(1).standard_normal(out.shape)
    dA, dB = lo.embedding_backward(dy, idx.numpy(), A.numpy(), B.numpy(), 16.0)
    eps = 1e-6
    for mat, grad, (i, j) in ((A, dA, (3, 5)), (B, dB, (int(idx[0]), 2))):
        p = mat.double().numpy().copy()
        p[i, j] += eps
        args = (p, B.numpy()) if mat is A else (A.numpy(), p)
        f1 = (dy * lo.embedding_forward(idx.numpy(), E.numpy(), *args, 16.0)).sum()
        f0 = (dy * out).sum()
        assert abs((f1 - f0) / eps - grad[i, j]) < 1e-4 * max(1.0, abs(grad[i, j]))


TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2, torch.float16: 2e-2}


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("V,D,r,T", [(1000, 512, 8, 300), (32000, 4096, 16, 2048), (77, 264, 64, 5)])
def test_embedding_forward_backward_gpu(cuda, dtype, V, D, r, T):
    from metallora_b200 import _lib
    from metallora_b200 import kernels as K
    E, A, B, idx = _case(V, D, r, T, 3)
    h = lambda t: t.to(dtype).double().numpy()  # noqa: E731
    out = K.lora_embedding_fwd(idx.to(cuda), E.to(dtype).to(cuda), A.to(dtype).to(cuda),
                               B.to(dtype).to(cuda), 16.0)
    dy = torch.randn(T, D, generator=torch.Generator().manual_seed(4))
    da, db = K.lora_embedding_bwd(dy.to(dtype).to(cuda), idx.to(cuda), A.to(dtype).to(cuda),
                                  B.to(dtype).to(cuda), 16.0)
    da2, db2 = K.lora_embedding_bwd(dy.to(dtype).to(cuda), idx.to(cuda), A.to(dtype).to(cuda),
                                    B.to(dtype).to(cuda), 16.0)
    torch.cuda.synchronize()
    ref = lo.embedding_forward(idx.numpy(), h(E), h(A), h(B), 16.0)
    rda, rdb = lo.embedding_backward(h(dy), idx.numpy(), h(A), h(B), 16.0)
    assert rel_err(out.double().cpu().numpy(), ref) < TOL[dtype]
    assert rel_err(da.double().cpu().numpy(), rda) < TOL[dtype]
    assert rel_err(db.double().cpu().numpy(), rdb) < TOL[dtype]
    assert torch.equal(da, da2) and torch.equal(db, db2)  # deterministic
    untouched = torch.ones(V, dtype=torch.bool)
    untouched[idx] = False
    assert torch.count_nonzero(db.cpu()[untouched]) == 0
    assert _lib.device_status(reset=True) == 0


@pytest.mark.gpu
def test_embedding_bad_index_reports_and_zeroes(cuda):
    from metallora_b200 import _lib
    from metallora_b200 import kernels as K
    E, A, B, _ = _case(64, 128, 8, 4, 5)
    idx = torch.tensor([3, 64, -1, 7], device=cuda)
    _lib.device_status(reset=True)
    out = K.lora_embedding_fwd(idx, E.bfloat16().to(cuda), A.bfloat16().to(cuda),
                               B.bfloat16().to(cuda), 16.0)
    torch.cuda.synchronize()
    assert _lib.device_status(reset=True) == 0x107
    assert torch.count_nonzero(out[1:3]) == 0 and torch.count_nonzero(out[0]) > 0


@pytest.mark.gpu
def test_lora_embedding_module_trains_and_merges(cuda):
    from metallora_b200.layers import LoRAEmbedding
    emb = LoRAEmbedding(500, 256, rank=8, alpha=16.0, device=cuda, dtype=torch.bfloat16)
    with torch.no_grad():
        emb.B.normal_(0, 0.1)
    idx = torch.randint(0, 500, (4, 33), device=cuda)
    out = emb(idx)
    assert out.shape == (4, 33, 256)
    merged = emb.merge_weights()
    assert rel_err(merged[idx].float().cpu().numpy().astype(np.float64),
                   out.detach().float().cpu().numpy().astype(np.float64)) < 2e-2
    target = torch.randn_like(out)
    opt = torch.optim.SGD([emb.A, emb.B], lr=5.0)
    losses = []
    for _ in range(10):
        opt.zero_grad()
        loss = ((emb(idx).float() - target.float()) ** 2).mean()
        loss.backward()
        opt.step()
        losses.append(float(loss.detach()))
    assert emb.embeddings.grad is None and losses[-1] < losses[0]
