"""LoRA KV-cache update (lora_kv_cache_update / LoRAKVCache): bookkeeping on
CPU, fused projection into the cache slot on the GPU."""
import numpy as np
import pytest
import torch

from oracle import lora_oracle as lo
from tests.conftest import rel_err


def test_cache_update_bookkeeping():
    from metallora_b200.optimizations import LoRAKVCache
    c = LoRAKVCache(2, 8, 2, 4, dtype=torch.float32)
    k, v = c.update(torch.ones(2, 3, 2, 4), torch.full((2, 3, 2, 4), 2.0))
    assert k.shape == (2, 3, 2, 4) and float(v.sum()) == 2.0 * 48
    c.update(torch.ones(2, 5, 2, 4), torch.ones(2, 5, 2, 4))
    with pytest.raises(ValueError):
        c.update(torch.ones(2, 1, 2, 4), torch.ones(2, 1, 2, 4))
    c.reset()
    assert c.cur_pos == 0


@pytest.mark.gpu
@pytest.mark.parametrize("batch", [1, 4, 16, 40])
@pytest.mark.parametrize("r", [16, 12])
def test_kv_cache_update_gpu(cuda, batch, r):
    """Up to 16 sequences run the decode kernel, 40 the tcgen05 path; D_kv <
    D_in (grouped KV heads); r = 12 is zero-padded.  Only row cur_pos changes."""
    from metallora_b200 import kernels as K
    D_in, D_kv, max_seq, pos = 512, 256, 64, 37
    g = torch.Generator().manual_seed(batch + r)
    bf = torch.bfloat16
    x = torch.randn(batch, D_in, generator=g).to(bf)
    wk, wv = (torch.randn(D_kv, D_in, generator=g) / D_in ** 0.5 for _ in range(2))
    ak, av = ((torch.rand(r, D_in, generator=g) * 2 - 1) / D_in ** 0.5 for _ in range(2))
    bk, bv = (torch.randn(D_kv, r, generator=g) * 0.1 for _ in range(2))
    kc = torch.zeros(batch, max_seq, 4, D_kv // 4, dtype=bf, device=cuda)
    vc = torch.zeros_like(kc)
    dev = lambda t: t.to(bf).to(cuda)  # noqa: E731
    K.lora_kv_cache_update(dev(x), dev(wk), dev(wv), dev(ak), dev(bk), dev(av), dev(bv), kc, vc, pos,
                           32.0)
    torch.cuda.synchronize()
    h = lambda t: t.to(bf).double().numpy()  # noqa: E731
    for cache, w, a, b in ((kc, wk, ak, bk), (vc, wv, av, bv)):
        got = cache[:, pos].reshape(batch, D_kv).double().cpu().numpy()
        assert rel_err(got, lo.lora_forward(h(x), h(w), h(a), h(b), 32.0, np.float64)) < 2e-2
        others = torch.cat([cache[:, :pos], cache[:, pos + 1:]], dim=1)
        assert torch.count_nonzero(others) == 0


@pytest.mark.gpu
def test_cache_project_and_update_with_layers(cuda):
    from metallora_b200.layers import LoRALinear
    from metallora_b200.optimizations import LoRAKVCache
    kp = LoRALinear(256, 128, rank=8, alpha=16.0, device=cuda, dtype=torch.bfloat16)
    vp = LoRALinear(256, 128, rank=8, alpha=16.0, device=cuda, dtype=torch.bfloat16)
    with torch.no_grad():
        for layer in (kp, vp):
            layer.W0.normal_(0, 1 / 16)
            layer.B.normal_(0, 0.1)
    cache = LoRAKVCache(3, 16, 2, 64, dtype=torch.bfloat16, device=cuda)
    for step in range(3):
        x = torch.randn(3, 1, 256, device=cuda, dtype=torch.bfloat16)
        k, v = cache.project_and_update(x, kp, vp)
        assert k.shape == (3, step + 1, 2, 64)
        ref_k = kp(x).reshape(3, 2, 64)
        assert rel_err(k[:, step].float().cpu().numpy().astype(np.float64),
                       ref_k.detach().float().cpu().numpy().astype(np.float64)) < 2e-2
