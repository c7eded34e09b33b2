"""LoRA layers (reference: python/metal_lora/layers.py) as ``torch.nn.Module``s.

``LoRALinear`` keeps the reference's parameter names (``W0``, ``A``, ``B``,
``bias``), initialisation (layers.py:69-78), validation (:53-60), reshape and
bias handling (:83-106), merge / inference mode (:108-117), ``from_linear``
(:119-139) and trainable-parameter accounting (:141-158).  Its forward and
backward run on the sm_100a kernels in ``ops``/``kernels``.
"""
from __future__ import annotations

import math

import torch
from torch import nn

from . import kernels as _k
from .exceptions import ConfigurationError, validate_alpha, validate_probability, validate_rank
from .logging import logger
from .ops import lora_forward, merge_lora_weights, qlora_forward


class LoRALinear(nn.Module):
    """Linear layer with LoRA adaptation: ``h = x.W0^T + (alpha/rank).(x.A^T).B^T``.

    Parameters mirror the reference (layers.py:41-50); ``device``/``dtype``
    are the usual torch factory arguments.  ``W0`` is a frozen ``Parameter``
    when ``freeze_base`` (the reference stops its gradient, layers.py:77-78).
    """

    def __init__(self, in_features: int, out_features: int, rank: int = 8, alpha: float = 16.0,
                 dropout: float = 0.0, use_bias: bool = False, freeze_base: bool = True,
                 device=None, dtype=None):
        super().__init__()
        if in_features <= 0:
            raise ConfigurationError(f"in_features must be positive, got {in_features}")
        if out_features <= 0:
            raise ConfigurationError(f"out_features must be positive, got {out_features}")
        validate_rank(rank)
        validate_alpha(alpha)
        validate_probability(dropout, "dropout")

        self.in_features = in_features
        self.out_features = out_features
        self.rank = rank
        self.alpha = alpha
        self.dropout = dropout
        self.freeze_base = freeze_base
        self.merged = False

        fk = {"device": device, "dtype": dtype}
        self.W0 = nn.Parameter(torch.zeros((out_features, in_features), **fk),
                               requires_grad=not freeze_base)
        bound = 1.0 / math.sqrt(in_features)
        self.A = nn.Parameter(torch.empty((rank, in_features), **fk).uniform_(-bound, bound))
        self.B = nn.Parameter(torch.zeros((out_features, rank), **fk))
        if use_bias:
            self.bias = nn.Parameter(torch.zeros((out_features,), **fk),
                                     requires_grad=not freeze_base)
        else:
            self.register_parameter("bias", None)
        self._best_config = None
        # Set by a trainer that keeps fp32 master factors in flat buffers:
        # (A, B) in the compute dtype, and (gA, gB) fp32 gradient sinks.
        self._compute_ab = None
        self._grad_sink = None
        self.qweight = None  # quantised base (quantize_base); W0 is then dropped
        logger.debug(f"LoRALinear: {in_features}→{out_features}, rank={rank}")

    @property
    def scale(self) -> float:
        return self.alpha / self.rank

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """layers.py:83-106: any leading shape; the bias is added after the op."""
        if self.qweight is not None:
            out = qlora_forward(x, self.qweight, self.A, self.B, alpha=self.alpha,
                                _compute=self._compute_ab, _sink=self._grad_sink)
        elif self.merged:
            out = _k.linear(x.reshape(-1, x.shape[-1]), self.W0).reshape(*x.shape[:-1],
                                                                         self.out_features)
        else:
            out = lora_forward(x, self.W0, self.A, self.B, alpha=self.alpha, dropout=self.dropout,
                               training=self.training, _compute=self._compute_ab,
                               _sink=self._grad_sink)
        if self.bias is not None:
            out = out + self.bias
        return out

    @torch.no_grad()
    def merge_weights(self) -> torch.Tensor:
        """W0 + (alpha/rank).B.A (layers.py:108-110)."""
        return merge_lora_weights(self.W0, self.A, self.B, self.alpha)

    @torch.no_grad()
    def to_inference_mode(self) -> "LoRALinear":
        """layers.py:112-117: W0 := merged weight, A and B := zeros (shapes kept).

        The forward then skips the (all-zero) adapter and runs the plain GEMM,
        which gives the same result as running it."""
        self.W0.copy_(_k.merge(self.W0, self.A, self.B, self.alpha))
        self.A.zero_()
        self.B.zero_()
        self.merged = True
        return self

    @classmethod
    def from_linear(cls, linear: nn.Linear, rank: int = 8, alpha: float = 16.0,
                    dropout: float = 0.0) -> "LoRALinear":
        """layers.py:119-139: takes the weight (and bias) of an ``nn.Linear``."""
        w = linear.weight
        lora = cls(in_features=w.shape[1], out_features=w.shape[0], rank=rank, alpha=alpha,
                   dropout=dropout, use_bias=linear.bias is not None, freeze_base=True,
                   device=w.device, dtype=w.dtype)
        with torch.no_grad():
            lora.W0.copy_(w)
            if linear.bias is not None:
                lora.bias.copy_(linear.bias)
        return lora

    @torch.no_grad()
    def quantize_base(self, scheme: str = "nf4", group: int | None = None,
                      lean: bool = False) -> "LoRALinear":
        """Replaces the frozen base W0 by its quantised form (QLoRA): NF4 with
        per-block absmax, or group-wise INT4/INT8 (the formats of
        kernels/lora_quantized.metal).  The dense W0 is released.  ``lean``
        keeps the per-call workspace free of a dequantised copy (see
        metallora_b200.quant.quantize)."""
        from .quant import quantize
        if self.merged:
            raise ConfigurationError("quantize_base needs an unmerged layer")
        self.qweight = quantize(self.W0.detach(), scheme, group, lean=lean)
        self.W0 = nn.Parameter(torch.empty(0, device=self.W0.device, dtype=self.W0.dtype),
                               requires_grad=False)
        return self

    def trainable_parameters(self) -> dict:
        """layers.py:141-146: A and B (plus bias if the base is not frozen)."""
        params = {"A": self.A, "B": self.B}
        if self.bias is not None and not self.freeze_base:
            params["bias"] = self.bias
        return params

    def num_trainable_params(self) -> int:
        count = self.A.numel() + self.B.numel()
        if self.bias is not None and not self.freeze_base:
            count += self.bias.numel()
        return count

    def num_total_params(self) -> int:
        base = self.in_features * self.out_features if self.qweight is not None else self.W0.numel()
        count = base + self.A.numel() + self.B.numel()
        if self.bias is not None:
            count += self.bias.numel()
        return count

    def tune(self, warmup: int = 5, iters: int = 20):
        """layers.py:160-191 chose between Metal kernel variants; there is one
        kernel configuration here, so this only times it and records it."""
        if not _k.is_metal_available():
            return
        x = torch.randn((1, 128, self.in_features), device=self.W0.device, dtype=self.W0.dtype)
        for _ in range(warmup):
            self(x)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(iters):
            self(x)
        end.record()
        end.synchronize()
        self._best_config = {"ms": start.elapsed_time(end) / iters}
        logger.info(f"Tuned {self.in_features}x{self.out_features}: {self._best_config}")

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"rank={self.rank}, alpha={self.alpha}, merged={self.merged}")


class _LoRAEmbeddingFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, indices, table, a, b, alpha):
        ctx.save_for_backward(indices, a, b)
        ctx.alpha = alpha
        return _k.lora_embedding_fwd(indices, table, a, b, alpha)

    @staticmethod
    def backward(ctx, dy):
        indices, a, b = ctx.saved_tensors
        da, db = _k.lora_embedding_bwd(dy, indices, a, b, ctx.alpha)
        return None, None, da.to(a.dtype), db.to(b.dtype), None


class LoRAEmbedding(nn.Module):
    """Embedding with a LoRA delta (layers.py:194-230):
    ``out = E[idx] + (alpha/rank) * B[idx] . A`` with E [num_embeddings, dim]
    (frozen when ``freeze_base``), A [rank, dim] ~ U(+-1/sqrt(dim)), B
    [num_embeddings, rank] = 0, E ~ N(0, 0.02^2) -- the reference's
    initialisation (:207-213).  The forward gathers on the tensor cores
    (16-bit) or CUDA cores (fp32); gradients flow to A and B only."""

    def __init__(self, num_embeddings: int, embedding_dim: int, rank: int = 8,
                 alpha: float = 16.0, freeze_base: bool = True, device=None, dtype=None):
        super().__init__()
        if num_embeddings <= 0 or embedding_dim <= 0:
            raise ConfigurationError("num_embeddings and embedding_dim must be positive")
        validate_rank(rank)
        validate_alpha(alpha)
        self.num_embeddings = num_embeddings
        self.embedding_dim = embedding_dim
        self.rank = rank
        self.alpha = alpha
        fk = {"device": device, "dtype": dtype}
        self.embeddings = nn.Parameter(torch.randn((num_embeddings, embedding_dim), **fk) * 0.02,
                                       requires_grad=not freeze_base)
        bound = 1.0 / math.sqrt(embedding_dim)
        self.A = nn.Parameter(torch.empty((rank, embedding_dim), **fk).uniform_(-bound, bound))
        self.B = nn.Parameter(torch.zeros((num_embeddings, rank), **fk))

    @property
    def scale(self) -> float:
        return self.alpha / self.rank

    def forward(self, indices: torch.Tensor) -> torch.Tensor:
        if self.embeddings.requires_grad:
            raise ConfigurationError("LoRAEmbedding trains A and B only (freeze_base=True)")
        return _LoRAEmbeddingFn.apply(indices, self.embeddings, self.A, self.B, float(self.alpha))

    @torch.no_grad()
    def merge_weights(self) -> torch.Tensor:
        """layers.py:227-230: E + (alpha/rank) B.A."""
        return _k.merge(self.embeddings, self.A, self.B, float(self.alpha))
