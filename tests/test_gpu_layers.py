"""GPU tests of the reference-facing module API: LoRALinear (autograd),
to_inference_mode, ops, apply_lora_to_model and adapter round trips."""
import numpy as np
import pytest
import torch
from torch import nn

from oracle import lora_oracle as lo
from tests.conftest import rel_err

pytestmark = pytest.mark.gpu


def _init(layer, seed=0):
    g = torch.Generator(device=layer.W0.device).manual_seed(seed)
    with torch.no_grad():
        layer.W0.copy_(torch.randn(layer.W0.shape, device=layer.W0.device, generator=g)
                       / layer.in_features ** 0.5)
        layer.B.copy_(torch.randn(layer.B.shape, device=layer.B.device, generator=g) * 0.1)


@pytest.mark.parametrize("dtype,tol", [(torch.bfloat16, 2e-2), (torch.float32, 1e-4)])
@pytest.mark.parametrize("shape", [(4, 32), (64,), (2, 3, 5)])
def test_lora_linear_autograd_matches_oracle(cuda, dtype, tol, shape):
    from metallora_b200.layers import LoRALinear
    layer = LoRALinear(256, 384, rank=8, alpha=16.0, use_bias=True, device=cuda, dtype=dtype)
    _init(layer)
    with torch.no_grad():
        layer.bias.copy_(torch.linspace(-1, 1, 384, device=cuda))
    x = torch.randn(*shape, 256, device=cuda, dtype=dtype, requires_grad=True)
    y = layer(x)
    assert y.shape == (*shape, 384)
    dy = torch.randn_like(y)
    y.backward(dy)
    h = lambda t: t.detach().float().cpu().numpy().astype(np.float64)  # noqa: E731
    X, W, A, B, DY = h(x).reshape(-1, 256), h(layer.W0), h(layer.A), h(layer.B), h(dy).reshape(-1, 384)
    ref = lo.lora_layer_forward(X, W, A, B, 16.0, h(layer.bias), np.float64)
    assert rel_err(h(y).reshape(-1, 384), ref) < tol
    assert rel_err(h(x.grad).reshape(-1, 256), lo.lora_grad_x(DY, W, A, B, 16.0, np.float64)) < tol
    ga, gb = lo.lora_backward(DY, X, A, B, 16.0, None, np.float64)
    assert rel_err(h(layer.A.grad), ga) < tol and rel_err(h(layer.B.grad), gb) < tol
    assert layer.W0.grad is None  # frozen base (layers.py:77-78)


def test_fresh_layer_outputs_base_only(cuda):
    """B starts at zero (layers.py:73), so a fresh layer computes x.W0^T."""
    from metallora_b200.layers import LoRALinear
    layer = LoRALinear(128, 256, rank=4, device=cuda, dtype=torch.bfloat16)
    _init(layer)
    with torch.no_grad():
        layer.B.zero_()
    x = torch.randn(16, 128, device=cuda, dtype=torch.bfloat16)
    y = layer(x)
    ref = x.float() @ layer.W0.float().t()
    assert float((y.detach().float() - ref).norm() / ref.norm()) < 1e-2


@pytest.mark.parametrize("dtype,tol", [(torch.bfloat16, 2e-2), (torch.float32, 1e-4)])
def test_to_inference_mode_equals_unmerged(cuda, dtype, tol):
    from metallora_b200.layers import LoRALinear
    layer = LoRALinear(512, 512, rank=16, alpha=32.0, device=cuda, dtype=dtype).eval()
    _init(layer, 3)
    x = torch.randn(4, 64, 512, device=cuda, dtype=dtype)
    with torch.no_grad():
        y0 = layer(x)
        layer.to_inference_mode()
        y1 = layer(x)
    assert torch.count_nonzero(layer.A) == 0 and torch.count_nonzero(layer.B) == 0
    assert layer.A.shape == (16, 512) and layer.B.shape == (512, 16)
    assert float((y1.float() - y0.float()).norm() / y0.float().norm()) < tol


def test_ops_api_shapes_and_forward_2d_3d(cuda):
    from metallora_b200.ops import lora_forward, lora_forward_inference, merge_lora_weights
    x = torch.randn(4, 16, 64, device=cuda)
    w0 = torch.randn(128, 64, device=cuda)
    a = torch.randn(8, 64, device=cuda)
    b = torch.randn(128, 8, device=cuda)
    assert lora_forward(x, w0, a, b).shape == (4, 16, 128)
    assert lora_forward(x[0], w0, a, b).shape == (16, 128)
    m = merge_lora_weights(w0, a, b)
    assert m.shape == (128, 64)
    y_m = lora_forward_inference(x, m)
    y = lora_forward(x, w0, a, b)
    assert float((y_m - y).norm() / y.norm()) < 1e-4


def test_apply_lora_save_load_round_trip(cuda, tmp_path):
    from metallora_b200.layers import LoRALinear
    from metallora_b200.utils import (apply_lora_to_model, count_lora_parameters, load_adapter,
                                      save_adapter)

    class Block(nn.Module):
        def __init__(self):
            super().__init__()
            self.q_proj = nn.Linear(64, 64, bias=False)
            self.v_proj = nn.Linear(64, 64, bias=True)
            self.mlp = nn.Linear(64, 128)

    model = nn.Sequential(Block(), Block()).to(cuda)
    apply_lora_to_model(model, rank=8, alpha=16.0)
    assert isinstance(model[0].q_proj, LoRALinear) and isinstance(model[1].v_proj, LoRALinear)
    assert isinstance(model[0].mlp, nn.Linear)
    stats = count_lora_parameters(model)
    assert stats["lora_layers"] == 4 and stats["trainable"] == 4 * (8 * 64 + 64 * 8)
    with torch.no_grad():
        for mod in model.modules():
            if isinstance(mod, LoRALinear):
                mod.B.normal_()
    x = torch.randn(3, 64, device=cuda)
    y0 = model[0].q_proj(x)
    save_adapter(model, tmp_path, "adapt")
    with torch.no_grad():
        for mod in model.modules():
            if isinstance(mod, LoRALinear):
                mod.A.zero_()
                mod.B.zero_()
    load_adapter(model, tmp_path, "adapt")
    assert torch.equal(model[0].q_proj(x), y0)


def test_cpu_tensors_fail_loudly():
    from metallora_b200.exceptions import DeviceError
    from metallora_b200.ops import lora_forward
    with pytest.raises(DeviceError):
        lora_forward(torch.randn(2, 8), torch.randn(8, 8), torch.randn(8, 8), torch.randn(8, 8))
