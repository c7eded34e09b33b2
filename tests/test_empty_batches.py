"""Zero-token batches: every wrapper returns correctly shaped empty outputs and
zero LoRA gradients (the sum over no tokens), as torch.nn.Linear does, without
launching a kernel of the library."""
import pytest
import torch

from metallora_b200 import _lib, kernels, ops, quant
from metallora_b200.layers import LoRAEmbedding, LoRALinear


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_empty_token_batch(cuda, dtype):
    K, N, r = 256, 264, 12  # rank 12: padded to 16 inside, sliced back
    layer = LoRALinear(K, N, rank=r, alpha=32.0, device=cuda, dtype=dtype)
    with torch.no_grad():
        layer.B.copy_(torch.randn_like(layer.B))
    n0 = _lib.launch_count()
    x = torch.randn(2, 0, K, device=cuda, dtype=dtype, requires_grad=True)
    y = layer(x)
    assert y.shape == (2, 0, N) and y.dtype == dtype
    y.backward(torch.randn_like(y))
    assert x.grad.shape == x.shape
    assert layer.A.grad.shape == layer.A.shape and not layer.A.grad.any()
    assert layer.B.grad.shape == layer.B.shape and not layer.B.grad.any()
    da, db = ops.lora_backward(torch.empty(0, N, device=cuda, dtype=dtype),
                               torch.empty(0, K, device=cuda, dtype=dtype), layer.A.detach(),
                               layer.B.detach())
    assert da.shape == layer.A.shape and not da.any() and not db.any()
    assert kernels.linear(torch.empty(0, K, device=cuda, dtype=dtype),
                          layer.W0.detach()).shape == (0, N)
    # gradient sinks: written over -> zeros; added to -> unchanged
    if dtype == torch.bfloat16:
        a16 = torch.zeros(16, K, device=cuda, dtype=dtype)
        b16 = torch.zeros(N, 16, device=cuda, dtype=dtype)
        ga = torch.full((16, K), 3.0, device=cuda)
        gb = torch.full((N, 16), 3.0, device=cuda)
        e_dy, e_x = (torch.empty(0, n, device=cuda, dtype=dtype) for n in (N, K))
        kernels.lora_linear_bwd(e_dy, e_x, layer.W0.detach(), a16, b16, 32.0, da_out=ga,
                                db_out=gb, accumulate=True)
        assert bool((ga == 3.0).all()) and bool((gb == 3.0).all())
        kernels.lora_linear_bwd(e_dy, e_x, layer.W0.detach(), a16, b16, 32.0, da_out=ga,
                                db_out=gb, accumulate=False)
        assert not ga.any() and not gb.any()
    torch.cuda.synchronize()
    assert _lib.launch_count() == n0


@pytest.mark.gpu
def test_empty_batch_quantised_and_embedding(cuda):
    K, N, r = 256, 264, 16
    layer = LoRALinear(K, N, rank=r, alpha=32.0, device=cuda, dtype=torch.bfloat16)
    with torch.no_grad():
        layer.W0.copy_(torch.randn_like(layer.W0) / 16)
    layer.quantize_base("nf4")
    emb = LoRAEmbedding(100, K, rank=r, alpha=32.0).to(cuda)
    n0 = _lib.launch_count()
    x = torch.randn(0, K, device=cuda, dtype=torch.bfloat16, requires_grad=True)
    y = layer(x)
    y.backward(torch.randn_like(y))
    assert y.shape == (0, N) and x.grad.shape == (0, K) and not layer.A.grad.any()
    idx = torch.empty(3, 0, dtype=torch.int64, device=cuda)
    out = emb(idx)
    assert out.shape[:2] == (3, 0)
    ids = torch.empty(0, dtype=torch.int32, device=cuda)
    a_st = torch.zeros(2 * r, K, device=cuda, dtype=torch.bfloat16)
    b_st = torch.zeros(N, 2 * r, device=cuda, dtype=torch.bfloat16)
    assert kernels.multi_lora_fwd(torch.empty(0, K, device=cuda, dtype=torch.bfloat16), None,
                                  a_st, b_st, ids, r, 32.0).shape == (0, N)
    torch.cuda.synchronize()
    assert _lib.launch_count() == n0
