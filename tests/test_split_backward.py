"""The backward split in two launches (MLORA_BWD_DEFER_DX, then
MLORA_BWD_DX_ONLY) gives the same dx, dA, dB as one call, and the on_grads
hook of a gradient sink runs between the two (before the dx GEMM)."""
import pytest
import torch

from metallora_b200 import _lib, kernels


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,N,r", [(512, 256, 384, 16), (300, 512, 256, 8)])
def test_split_backward_matches_single_call(cuda, M, K, N, r):
    g = torch.Generator(device=cuda).manual_seed(3)
    x = torch.randn(M, K, device=cuda, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device=cuda, generator=g) / K ** 0.5).to(torch.bfloat16)
    a = (torch.randn(r, K, device=cuda, generator=g) / K ** 0.5).to(torch.bfloat16)
    b = (torch.randn(N, r, device=cuda, generator=g) * 0.1).to(torch.bfloat16)
    dy = torch.randn(M, N, device=cuda, generator=g).to(torch.bfloat16)
    _, saved = kernels.lora_linear_fwd(x, w, a, b, 2.0 * r, save_xa=True)
    dx1, da1, db1 = kernels.lora_linear_bwd(dy, x, w, a, b, 2.0 * r, saved)
    da2 = torch.full((r, K), 7.0, device=cuda)
    db2 = torch.full((N, r), 7.0, device=cuda)
    finish = kernels.lora_linear_bwd_split(dy, x, w, a, b, 2.0 * r, saved, da2, db2,
                                           accumulate=False)
    dx2 = finish()
    torch.cuda.synchronize()
    assert torch.equal(dx1, dx2) and torch.equal(da1, da2) and torch.equal(db1, db2)
    assert _lib.device_status(reset=True) == 0


@pytest.mark.gpu
def test_sink_hook_runs_before_dx(cuda):
    from metallora_b200.layers import LoRALinear
    torch.manual_seed(0)
    layer = LoRALinear(256, 384, rank=16, alpha=32.0, device=cuda, dtype=torch.bfloat16)
    with torch.no_grad():
        layer.W0.copy_(torch.randn(384, 256, device=cuda) / 16)
        layer.B.copy_(torch.randn(384, 16, device=cuda) * 0.1)
    ga, gb = torch.zeros(16, 256, device=cuda), torch.zeros(384, 16, device=cuda)
    seen = []
    layer._grad_sink = (ga, gb, False, lambda: seen.append(ga.clone()))
    x = torch.randn(512, 256, device=cuda).to(torch.bfloat16).requires_grad_(True)
    dy = torch.randn(512, 384, device=cuda).to(torch.bfloat16)
    layer(x).backward(dy)
    torch.cuda.synchronize()
    assert len(seen) == 1 and torch.equal(seen[0], ga)  # dA complete when the hook ran
    layer._grad_sink = None
    x2 = x.detach().clone().requires_grad_(True)
    layer(x2).backward(dy)
    assert torch.equal(x.grad, x2.grad)
    assert torch.allclose(layer.A.grad.float(), ga, rtol=1e-2, atol=1e-3)


def test_split_flags_rejected_for_fp32_and_conflicts():
    lib = _lib.load()
    p = 1 << 20  # aligned stand-in pointers: validation fails before any launch
    head = [p, p, p, p, p, None, p, p, p, 128, 128, 128, 16, 32.0, 0.0]
    assert lib.mlora_lora_backward_ex(*head, _lib.DTYPE_F32, _lib.BWD_DEFER_DX, None, 0,
                                      None) == -1
    assert b"split backward" in lib.mlora_last_error_message()
    assert lib.mlora_lora_backward_ex(*head, _lib.DTYPE_BF16, _lib.BWD_DEFER_DX | _lib.BWD_DX_ONLY,
                                      None, 0, None) == -1
    assert b"exclude each other" in lib.mlora_last_error_message()


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_16bit_grads_equal_rounded_fp32(cuda, dtype):
    """MLORA_BWD_GRADS_16BIT writes dA/dB in the operands' dtype: the same
    values as the fp32 gradients rounded once (what a cast would give)."""
    M, K, N, r = 384, 256, 512, 16
    g = torch.Generator(device=cuda).manual_seed(5)
    x = torch.randn(M, K, device=cuda, generator=g).to(dtype)
    w = (torch.randn(N, K, device=cuda, generator=g) / K ** 0.5).to(dtype)
    a = (torch.randn(r, K, device=cuda, generator=g) / K ** 0.5).to(dtype)
    b = (torch.randn(N, r, device=cuda, generator=g) * 0.1).to(dtype)
    dy = torch.randn(M, N, device=cuda, generator=g).to(dtype)
    dx1, da1, db1 = kernels.lora_linear_bwd(dy, x, w, a, b, 32.0)
    dx2, da2, db2 = kernels.lora_linear_bwd(dy, x, w, a, b, 32.0, grad_dtype=dtype)
    assert da2.dtype == dtype and db2.dtype == dtype
    assert torch.equal(dx1, dx2)
    assert torch.equal(da1.to(dtype), da2) and torch.equal(db1.to(dtype), db2)
