"""Quantised base weights (NF4, group-wise INT4/INT8) for QLoRA.

Storage follows the reference shaders' layout (kernels/lora_quantized.metal):
packed codes ``[N, K/2]`` bytes with the low nibble holding the even k
(:70-74) -- ``[N, K]`` for INT8 -- and per-row, per-block scales:
fp32 absmax ``[N, ceil(K/group)]`` for NF4 (:122, :135), fp16 scale and zero
``[N, ceil(K/group)]`` for INT4/INT8 (the reference's per-row int4 is
``group = K``).  ``quantize`` runs on the GPU (the reference ships no
quantiser); ``dequantize`` returns fp32 values bit-identical to the
reference's ``dequant_nf4``/``dequant_int4``.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib
from .exceptions import QuantizationError, ShapeError
from .kernels import _dtype_code, _need_cuda, _ptr, _stream

SCHEMES = {"nf4": _lib.QUANT_NF4, "int4": _lib.QUANT_INT4, "int8": _lib.QUANT_INT8}
DEFAULT_GROUP = {"nf4": 64, "int4": 128, "int8": 128}


@dataclass
class QuantizedWeight:
    """A quantised [out_features, in_features] weight."""
    scheme: str
    codes: torch.Tensor
    scales: torch.Tensor
    zeros: torch.Tensor | None
    group: int
    shape: tuple[int, int]
    lean: bool = False  # fused in-loop dequant (no transient bf16 copy of W per call)

    @property
    def code(self) -> int:
        return SCHEMES[self.scheme]

    @property
    def device(self):
        return self.codes.device

    def nbytes(self) -> int:
        n = self.codes.numel() + self.scales.numel() * self.scales.element_size()
        if self.zeros is not None:
            n += self.zeros.numel() * self.zeros.element_size()
        return n

    def dequantize(self, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        return dequantize(self, dtype)

    def prepared_scales(self) -> torch.Tensor:
        """The TMA-ready scale table [groups, rows rounded to 4] the GPU kernels
        read (built once, on first use, and kept with the weight)."""
        t = getattr(self, "_prepared", None)
        if t is None or t.device != self.codes.device:
            lib = _lib.load()
            N, K = self.shape
            nbytes = lib.mlora_qlora_prepared_scales_bytes(self.code, N, K, self.group)
            t = torch.empty(nbytes, dtype=torch.uint8, device=self.codes.device)
            st = lib.mlora_qlora_prepare_scales(self.code, _ptr(self.scales), _ptr(self.zeros), N,
                                                K, self.group, _ptr(t), _stream())
            _lib.check(st, "mlora_qlora_prepare_scales")
            object.__setattr__(self, "_prepared", t)
        return t

    def state_dict(self) -> dict[str, torch.Tensor]:
        d = {"codes": self.codes, "scales": self.scales}
        if self.zeros is not None:
            d["zeros"] = self.zeros
        return d


def quantize(w: torch.Tensor, scheme: str = "nf4", group: int | None = None,
             lean: bool = False) -> QuantizedWeight:
    """Quantises a 2-D CUDA weight [N, K] (bf16/fp16/fp32).  ``lean`` makes the
    LoRA kernels dequantise inside the GEMM main loop instead of staging a
    bf16 copy of the weight in their workspace (less memory, slower)."""
    if scheme not in SCHEMES:
        raise QuantizationError(f"unknown scheme {scheme!r}; use one of {sorted(SCHEMES)}")
    _need_cuda(w)
    if w.dim() != 2:
        raise ShapeError("quantize takes a 2-D weight [out_features, in_features]")
    group = group or DEFAULT_GROUP[scheme]
    N, K = w.shape
    if scheme != "int8" and K % 2:
        raise QuantizationError("4-bit codes pack two per byte: in_features must be even")
    G = -(-K // group)
    w = w.contiguous()
    dev = w.device
    codes = torch.empty((N, K if scheme == "int8" else K // 2), dtype=torch.uint8, device=dev)
    if scheme == "nf4":
        scales = torch.empty((N, G), dtype=torch.float32, device=dev)
        zeros = None
    else:
        scales = torch.empty((N, G), dtype=torch.float16, device=dev)
        zeros = torch.empty((N, G), dtype=torch.float16, device=dev)
    st = _lib.load().mlora_quantize(_ptr(w), _dtype_code(w), N, K, SCHEMES[scheme], group,
                                    _ptr(codes), _ptr(scales), _ptr(zeros), _stream())
    _lib.check(st, "mlora_quantize")
    return QuantizedWeight(scheme, codes, scales, zeros, group, (N, K), lean)


def dequantize(qw: QuantizedWeight, dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Dense [N, K] weights: fp32 = the reference's dequantised values (bit
    exact); bf16/fp16 = those values rounded, the operand the GEMMs use."""
    N, K = qw.shape
    out = torch.empty((N, K), dtype=dtype, device=qw.device)
    st = _lib.load().mlora_dequantize(qw.code, _ptr(qw.codes), _ptr(qw.scales), _ptr(qw.zeros), N,
                                      K, qw.group, _ptr(out), _dtype_code(out), _stream())
    _lib.check(st, "mlora_dequantize")
    return out


def from_reference_layout(scheme: str, codes, scales, zeros, shape, group,
                          lean: bool = False) -> QuantizedWeight:
    """Wraps tensors already in the reference layout (e.g. loaded from disk)."""
    if scheme not in SCHEMES:
        raise QuantizationError(f"unknown scheme {scheme!r}")
    return QuantizedWeight(scheme, codes.contiguous(), scales.contiguous(),
                           None if zeros is None else zeros.contiguous(), int(group),
                           (int(shape[0]), int(shape[1])), lean)


# ------------------------------------------------------------ pack format --
# The reference has no on-disk form for a quantised base.  This one keeps the
# kernels' layout unchanged: one safetensors file holding, per weight,
# ``{name}.codes`` (uint8), ``{name}.scales`` (fp32 absmax for NF4, fp16 for
# INT4/INT8) and, for INT4/INT8, ``{name}.zeros`` (fp16); the safetensors
# header metadata carries ``format`` = PACK_FORMAT and ``weights`` = a JSON map
# name -> {scheme, group, out_features, in_features}.  Files written here load
# without any conversion and are validated shape by shape on load.

PACK_FORMAT = "metallora-qbase-1"


def _expected_shapes(scheme: str, N: int, K: int, group: int):
    per_byte = 1 if scheme == "int8" else 2
    groups = -(-K // group)
    codes = (N, -(-K // per_byte))
    scale_dt = torch.float32 if scheme == "nf4" else torch.float16
    return codes, (N, groups), scale_dt


def pack_quantized(weights: dict[str, QuantizedWeight]) -> tuple[dict, dict]:
    """(tensors, metadata) of the pack format for ``{name: QuantizedWeight}``;
    tensors are copied to host memory."""
    tensors: dict[str, torch.Tensor] = {}
    meta = {}
    for name, qw in weights.items():
        tensors[f"{name}.codes"] = qw.codes.detach().contiguous().cpu()
        tensors[f"{name}.scales"] = qw.scales.detach().contiguous().cpu()
        if qw.zeros is not None:
            tensors[f"{name}.zeros"] = qw.zeros.detach().contiguous().cpu()
        meta[name] = {"scheme": qw.scheme, "group": int(qw.group),
                      "out_features": int(qw.shape[0]), "in_features": int(qw.shape[1])}
    import json
    return tensors, {"format": PACK_FORMAT, "weights": json.dumps(meta, sort_keys=True)}


def unpack_quantized(tensors: dict, metadata: dict, device=None,
                     lean: bool = False) -> dict[str, QuantizedWeight]:
    """Inverse of ``pack_quantized``; every tensor is checked against the
    shape and dtype its scheme, group and weight shape imply."""
    import json
    if (metadata or {}).get("format") != PACK_FORMAT:
        raise QuantizationError(f"not a {PACK_FORMAT} pack (metadata {metadata!r})")
    out = {}
    for name, m in json.loads(metadata["weights"]).items():
        scheme, group = m["scheme"], int(m["group"])
        N, K = int(m["out_features"]), int(m["in_features"])
        if scheme not in SCHEMES:
            raise QuantizationError(f"{name}: unknown scheme {scheme!r}")
        codes_shape, scales_shape, scale_dt = _expected_shapes(scheme, N, K, group)
        want = {"codes": (codes_shape, torch.uint8), "scales": (scales_shape, scale_dt)}
        if scheme != "nf4":
            want["zeros"] = (scales_shape, torch.float16)
        got = {}
        for part, (shape, dt) in want.items():
            t = tensors.get(f"{name}.{part}")
            if t is None:
                raise QuantizationError(f"{name}: missing {part}")
            if tuple(t.shape) != shape or t.dtype != dt:
                raise QuantizationError(f"{name}.{part}: expected {shape} {dt}, got "
                                        f"{tuple(t.shape)} {t.dtype}")
            got[part] = t.to(device) if device is not None else t
        out[name] = from_reference_layout(scheme, got["codes"], got["scales"], got.get("zeros"),
                                          (N, K), group, lean=lean)
    return out


def save_quantized(weights: dict[str, QuantizedWeight], path) -> None:
    """Writes ``{name: QuantizedWeight}`` to one safetensors file in the pack format."""
    from safetensors.torch import save_file
    tensors, meta = pack_quantized(weights)
    save_file(tensors, str(path), metadata=meta)


def load_quantized(path, device=None, lean: bool = False) -> dict[str, QuantizedWeight]:
    """Reads a pack written by ``save_quantized`` (onto ``device`` if given)."""
    from safetensors import safe_open
    tensors = {}
    with safe_open(str(path), framework="pt") as f:
        meta = f.metadata()
        for k in f.keys():
            tensors[k] = f.get_tensor(k)
    return unpack_quantized(tensors, meta, device=device, lean=lean)
