"""Adapter I/O and model surgery (reference: python/metal_lora/utils.py).

The on-disk format follows the reference: ``{adapter_name}.safetensors`` holding
``{module}.A`` / ``{module}.B`` for every LoRA module, next to
``{adapter_name}_config.json`` = ``{"adapter_name", "num_params"}``
(utils.py:10-32).  This build also records ``rank`` and ``alpha`` per module in
the config so a load can be validated; readers of the reference format ignore
the extra keys.
"""
from __future__ import annotations

import json
from pathlib import Path

import torch
from torch import nn

from .exceptions import AdapterError


def _lora_modules(model: nn.Module):
    for name, module in model.named_modules():
        if hasattr(module, "A") and hasattr(module, "B") and isinstance(module.A, torch.Tensor):
            yield name, module


def save_adapter(model: nn.Module, path: str | Path, adapter_name: str = "default") -> None:
    """utils.py:10-32."""
    from safetensors.torch import save_file

    save_path = Path(path)
    save_path.mkdir(parents=True, exist_ok=True)
    params: dict[str, torch.Tensor] = {}
    modules = {}
    for name, module in _lora_modules(model):
        params[f"{name}.A"] = module.A.detach().contiguous().cpu()
        params[f"{name}.B"] = module.B.detach().contiguous().cpu()
        modules[name] = {"rank": int(module.A.shape[0]), "alpha": float(getattr(module, "alpha", 0))}
    save_file(params, str(save_path / f"{adapter_name}.safetensors"))
    config = {
        "adapter_name": adapter_name,
        "num_params": sum(p.numel() for p in params.values()),
        "modules": modules,
    }
    with open(save_path / f"{adapter_name}_config.json", "w") as f:
        json.dump(config, f, indent=2)


def load_adapter(model: nn.Module, path: str | Path, adapter_name: str = "default") -> nn.Module:
    """utils.py:35-51: assigns ``{name}.A`` / ``{name}.B`` to matching modules."""
    from safetensors.torch import load_file

    load_path = Path(path) / f"{adapter_name}.safetensors"
    if not load_path.is_file():
        raise AdapterError(f"adapter file not found: {load_path}")
    params = load_file(str(load_path))
    for name, module in _lora_modules(model):
        a_key, b_key = f"{name}.A", f"{name}.B"
        if a_key in params and b_key in params:
            a, b = params[a_key], params[b_key]
            if tuple(a.shape) != tuple(module.A.shape) or tuple(b.shape) != tuple(module.B.shape):
                raise AdapterError(f"{name}: adapter shapes {tuple(a.shape)}/{tuple(b.shape)} do "
                                   f"not match {tuple(module.A.shape)}/{tuple(module.B.shape)}")
            with torch.no_grad():
                module.A.copy_(a.to(module.A.device, module.A.dtype))
                module.B.copy_(b.to(module.B.device, module.B.dtype))
    return model


def save_quantized_bases(model: nn.Module, path: str | Path, name: str = "base") -> None:
    """Writes the quantised bases of every LoRA module of ``model`` (those made
    by ``LoRALinear.quantize_base``) to ``{path}/{name}.safetensors`` in the
    pack format of ``quant.save_quantized``, keyed by module name."""
    from .quant import save_quantized

    weights = {mname: m.qweight for mname, m in _lora_modules(model)
               if getattr(m, "qweight", None) is not None}
    if not weights:
        raise AdapterError("the model has no quantised base to save")
    save_path = Path(path)
    save_path.mkdir(parents=True, exist_ok=True)
    save_quantized(weights, save_path / f"{name}.safetensors")


def load_quantized_bases(model: nn.Module, path: str | Path, name: str = "base",
                         lean: bool = False) -> nn.Module:
    """Installs the quantised bases saved by ``save_quantized_bases`` into the
    matching LoRA modules (their dense W0 is released, as ``quantize_base``
    does); each weight must match the module's [out, in] shape."""
    from .quant import load_quantized

    load_path = Path(path) / f"{name}.safetensors"
    if not load_path.is_file():
        raise AdapterError(f"quantised base file not found: {load_path}")
    modules = dict(_lora_modules(model))
    for mname, qw in load_quantized(load_path, lean=lean).items():
        m = modules.get(mname)
        if m is None:
            raise AdapterError(f"no LoRA module named {mname!r} in the model")
        if tuple(qw.shape) != (m.out_features, m.in_features):
            raise AdapterError(f"{mname}: quantised base {tuple(qw.shape)} does not match "
                               f"({m.out_features}, {m.in_features})")
        dev = m.A.device
        m.qweight = type(qw)(qw.scheme, qw.codes.to(dev), qw.scales.to(dev),
                             None if qw.zeros is None else qw.zeros.to(dev), qw.group, qw.shape,
                             qw.lean)
        m.W0 = nn.Parameter(torch.empty(0, device=dev, dtype=m.W0.dtype), requires_grad=False)
    return model


def apply_lora_to_model(model: nn.Module, rank: int = 8, alpha: float = 16.0,
                        target_modules: list[str] | None = None, dropout: float = 0.0) -> nn.Module:
    """utils.py:54-80: replaces every ``nn.Linear`` whose dotted name contains a
    target substring (default q/v/k/o_proj) with ``LoRALinear.from_linear``."""
    from .layers import LoRALinear

    target_modules = target_modules or ["q_proj", "v_proj", "k_proj", "o_proj"]

    def should_apply(name: str) -> bool:
        return any(t in name for t in target_modules)

    def replace_linear(module: nn.Module, prefix: str = "") -> None:
        for child_name, child in list(module.named_children()):
            full_name = f"{prefix}.{child_name}" if prefix else child_name
            if isinstance(child, nn.Linear) and should_apply(full_name):
                setattr(module, child_name,
                        LoRALinear.from_linear(child, rank=rank, alpha=alpha, dropout=dropout))
            else:
                replace_linear(child, full_name)

    replace_linear(model)
    return model


def count_lora_parameters(model: nn.Module) -> dict[str, int | float]:
    """utils.py:83-100."""
    trainable = total = layers = 0
    for _, module in model.named_modules():
        if hasattr(module, "num_trainable_params"):
            trainable += module.num_trainable_params()
            total += module.num_total_params()
            layers += 1
    return {"trainable": trainable, "total": total, "lora_layers": layers,
            "ratio": trainable / total if total > 0 else 0.0}


def merge_all_lora(model: nn.Module) -> nn.Module:
    """utils.py:103-108."""
    for _, module in model.named_modules():
        if hasattr(module, "to_inference_mode"):
            module.to_inference_mode()
    return model


def get_lora_summary(model: nn.Module) -> str:
    """utils.py:111-120."""
    stats = count_lora_parameters(model)
    return "\n".join([
        f"LoRA layers: {stats['lora_layers']}",
        f"Trainable: {stats['trainable']:,}",
        f"Total: {stats['total']:,}",
        f"Ratio: {stats['ratio']:.2%}",
    ])
