"""Host-side API behaviour that needs no GPU: validation errors and parameter
bookkeeping (reference tests/test_kernels.py:20-119), adapter file format."""
import json

import pytest
import torch
from torch import nn

from metallora_b200 import ConfigurationError, validate_alpha, validate_rank
from metallora_b200.layers import LoRALinear
from metallora_b200.utils import (apply_lora_to_model, count_lora_parameters, get_lora_summary,
                                  load_adapter, save_adapter)


def test_init_valid():
    layer = LoRALinear(64, 128, rank=8, alpha=16.0)
    assert (layer.in_features, layer.out_features, layer.rank, layer.alpha) == (64, 128, 8, 16.0)
    assert layer.W0.shape == (128, 64) and layer.A.shape == (8, 64) and layer.B.shape == (128, 8)
    assert torch.count_nonzero(layer.W0) == 0 and torch.count_nonzero(layer.B) == 0
    assert float(layer.A.abs().max()) <= 1 / 8  # U(-1/sqrt(in), 1/sqrt(in))
    assert not layer.W0.requires_grad


@pytest.mark.parametrize("kw", [{"rank": 0}, {"rank": 300}, {"alpha": -1.0}, {"dropout": 1.5}])
def test_init_invalid(kw):
    with pytest.raises(ConfigurationError):
        LoRALinear(64, 128, **kw)


def test_trainable_params():
    layer = LoRALinear(64, 128, rank=8)
    params = layer.trainable_parameters()
    assert set(params) == {"A", "B"}
    assert layer.num_trainable_params() == 8 * 64 + 128 * 8


def test_validators():
    validate_rank(8)
    validate_rank(1)
    validate_rank(256)
    for bad in (0, 300, "8"):
        with pytest.raises(ConfigurationError):
            validate_rank(bad)
    validate_alpha(16.0)
    validate_alpha(1)
    for bad in (-1.0, 0):
        with pytest.raises(ConfigurationError):
            validate_alpha(bad)


def test_from_linear_and_surgery_on_cpu():
    model = nn.Sequential(nn.ModuleDict({"q_proj": nn.Linear(32, 16), "o_proj": nn.Linear(16, 32),
                                         "fc": nn.Linear(32, 32)}))
    apply_lora_to_model(model, rank=4, alpha=8.0, target_modules=["q_proj"])
    blk = model[0]
    assert isinstance(blk["q_proj"], LoRALinear) and isinstance(blk["o_proj"], nn.Linear)
    assert blk["q_proj"].bias is not None
    s = count_lora_parameters(model)
    assert s["lora_layers"] == 1 and s["trainable"] == 4 * 32 + 16 * 4
    assert "LoRA layers: 1" in get_lora_summary(model)


def test_adapter_file_format(tmp_path):
    from safetensors.torch import load_file
    model = nn.Sequential(nn.ModuleDict({"q_proj": nn.Linear(32, 16)}))
    apply_lora_to_model(model, rank=4, target_modules=["q_proj"])
    with torch.no_grad():
        model[0]["q_proj"].B.fill_(0.25)
    save_adapter(model, tmp_path, "mine")
    tensors = load_file(str(tmp_path / "mine.safetensors"))
    assert set(tensors) == {"0.q_proj.A", "0.q_proj.B"}
    cfg = json.loads((tmp_path / "mine_config.json").read_text())
    assert cfg["adapter_name"] == "mine" and cfg["num_params"] == 4 * 32 + 16 * 4
    other = nn.Sequential(nn.ModuleDict({"q_proj": nn.Linear(32, 16)}))
    apply_lora_to_model(other, rank=4, target_modules=["q_proj"])
    load_adapter(other, tmp_path, "mine")
    assert torch.equal(other[0]["q_proj"].B, model[0]["q_proj"].B)
    assert torch.equal(other[0]["q_proj"].A, model[0]["q_proj"].A)


def test_lora_trainable_module_on_cpu():
    """LoRATrainableModule (trainer.py:115-170): targets q/v/k/o_proj by
    default, freezes the base, A ~ N(0, 0.02^2) and B = 0, reference key names,
    set/get round trip and parameter counts."""
    import torch
    from torch import nn

    from metallora_b200.layers import LoRALinear
    from metallora_b200.trainer import LoRATrainableModule

    class Block(nn.Module):
        def __init__(self):
            super().__init__()
            self.q_proj = nn.Linear(64, 32, bias=False)
            self.v_proj = nn.Linear(64, 48, bias=False)
            self.mlp = nn.Linear(64, 64)

    torch.manual_seed(0)
    base = Block()
    n_base = sum(p.numel() for p in base.parameters())
    wrapped = LoRATrainableModule(base, rank=8, alpha=16.0)
    assert isinstance(base.q_proj, LoRALinear) and isinstance(base.v_proj, LoRALinear)
    assert isinstance(base.mlp, nn.Linear) and not base.mlp.weight.requires_grad
    params = wrapped.get_lora_params()
    assert set(params) == {"q_proj.lora_A", "q_proj.lora_B", "v_proj.lora_A", "v_proj.lora_B"}
    assert params["q_proj.lora_A"].shape == (8, 64) and params["v_proj.lora_B"].shape == (48, 8)
    assert not params["q_proj.lora_B"].any()
    assert 0.01 < float(params["q_proj.lora_A"].std()) < 0.03
    assert wrapped.num_trainable_params() == 8 * (64 + 32) + 8 * (64 + 48)
    assert wrapped.num_total_params() == n_base + wrapped.num_trainable_params()
    new = {k: torch.full_like(v, 0.5) for k, v in params.items()}
    wrapped.set_lora_params(new)
    assert all(torch.equal(v, new[k]) for k, v in wrapped.get_lora_params().items())
    trainable = {n for n, p in wrapped.named_parameters() if p.requires_grad}
    assert trainable == {"base_model.q_proj.A", "base_model.q_proj.B",
                         "base_model.v_proj.A", "base_model.v_proj.B"}
