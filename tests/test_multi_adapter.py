"""Several adapters in one batch (MultiAdapterManager / lora_multi_adapter):
the oracle on CPU, the manager's bookkeeping, and the tcgen05 path on the GPU."""
import numpy as np
import pytest
import torch

from oracle import lora_oracle as lo
from tests.conftest import rel_err


def _adapters(n, r, K, N, seed):
    g = torch.Generator().manual_seed(seed)
    A = (torch.rand(n, r, K, generator=g) * 2 - 1) / K ** 0.5
    B = torch.randn(n, N, r, generator=g) * 0.1
    return A, B


def test_oracle_multi_matches_single_adapter_forward():
    A, B = _adapters(3, 8, 32, 24, 0)
    x = np.random.default_rng(1).standard_normal((4, 5, 32))
    W0 = np.random.default_rng(2).standard_normal((24, 32)) / 6
    ids = [2, 0, 2, 1]
    y = lo.multi_adapter_forward(x, W0, A.numpy(), B.numpy(), ids, 16.0)
    for b, g in enumerate(ids):
        ref = lo.lora_forward(x[b], W0, A[g].numpy(), B[g].numpy(), 16.0, np.float64)
        np.testing.assert_allclose(y[b], ref, rtol=1e-12, atol=1e-12)


def test_manager_bookkeeping():
    from metallora_b200.optimizations import MultiAdapterManager
    m = MultiAdapterManager(torch.nn.Identity(), max_adapters=2)
    A, B = _adapters(3, 8, 16, 16, 3)
    assert m.add_adapter("a", {"l.A": A[0], "l.B": B[0]}) == 0
    assert m.add_adapter("b", {"l.A": A[1], "l.B": B[1]}) == 1
    with pytest.raises(ValueError):
        m.add_adapter("c", {"l.A": A[2], "l.B": B[2]})
    m.remove_adapter("a")
    assert m.list_adapters() == ["b"]
    assert m.add_adapter("c", {"l.A": A[2], "l.B": B[2]}) == 2  # ids are not reused


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("n,r,with_base", [(4, 16, True), (4, 16, False), (16, 16, True),
                                            (3, 24, True), (20, 16, True), (5, 12, False)])
def test_multi_adapter_forward_gpu(cuda, dtype, n, r, with_base):
    """Ragged sequence length, repeated and unused adapters; 20 x 16 exceeds one
    launch (n * r <= 256) and runs in two groups; r = 12 is zero-padded."""
    from metallora_b200.ops import multi_adapter_forward
    K, N, S = 512, 776, 37
    A, B = _adapters(n, r, K, N, 5)
    g = torch.Generator().manual_seed(6)
    ids = [(7 * b) % n for b in range(max(6, n))]  # n = 20: all distinct, two groups
    x = torch.randn(len(ids), S, K, generator=g)
    W0 = torch.randn(N, K, generator=g) / K ** 0.5
    h = lambda t: t.to(dtype).float().numpy().astype(np.float64)  # noqa: E731
    y = multi_adapter_forward(x.to(dtype).to(cuda), W0.to(dtype).to(cuda) if with_base else None,
                              A.to(dtype).to(cuda), B.to(dtype).to(cuda), ids, alpha=32.0)
    torch.cuda.synchronize()
    ref = lo.multi_adapter_forward(h(x), h(W0) if with_base else None, h(A), h(B), ids, 32.0)
    assert y.shape == (len(ids), S, N)
    assert rel_err(y.float().cpu().numpy(), ref) < 2e-2
    from metallora_b200 import _lib
    assert _lib.device_status(reset=True) == 0


@pytest.mark.gpu
def test_manager_forward_batched_gpu(cuda):
    from metallora_b200.optimizations import MultiAdapterManager
    K, N, r = 256, 264, 8
    A, B = _adapters(3, r, K, N, 9)
    m = MultiAdapterManager(torch.nn.Identity(), device=cuda)
    ids = [m.add_adapter(f"a{i}", {"layer.A": A[i], "layer.B": B[i]}) for i in range(3)]
    x = torch.randn(4, 9, K).to(cuda)
    sel = [ids[2], ids[0], ids[2], ids[1]]
    y = m.forward_batched(x, sel)
    torch.cuda.synchronize()
    h = lambda t: t.to(torch.bfloat16).float().cpu().numpy().astype(np.float64)  # noqa: E731
    ref = lo.multi_adapter_forward(h(x), None, h(A), h(B), [2, 0, 2, 1], float(r))
    assert y.dtype == x.dtype and rel_err(y.float().cpu().numpy(), ref) < 2e-2
