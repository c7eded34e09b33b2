"""Batched inference with several LoRA adapters and a LoRA KV cache
(python/metal_lora/optimizations.py:129-220, :307-340).

``MultiAdapterManager`` and ``LoRAKVCache`` are on the LoRA-linear path; the
reference module's compression, memory pool, speculative decoding, lazy
loading and mixed-precision trainer are not part of this package.
"""
from __future__ import annotations

import torch
from torch import nn

from .ops import multi_adapter_forward


class MultiAdapterManager:
    """Holds adapters (one LoRA pair A [r, K], B [N, r] each) and runs a batch in
    which every sample uses its own adapter (optimizations.py:129-217).

    Ids are handed out in order and never reused (optimizations.py:144-155);
    storage is dense, so removing an adapter frees its slot.  The batched
    arrays are rebuilt lazily after a change (``_rebuild_batched``, :164-191),
    in ``dtype`` (the reference uses float16) on ``device``.
    """

    def __init__(self, base_model: nn.Module, max_adapters: int = 64, device=None,
                 dtype: torch.dtype = torch.bfloat16):
        self.base_model = base_model
        self.max_adapters = max_adapters
        self.adapters: dict[str, dict[str, torch.Tensor]] = {}
        self.adapter_ids: dict[str, int] = {}
        self.next_id = 0
        self.device = device
        self.dtype = dtype
        self.batched_a: torch.Tensor | None = None  # [n, r, K]
        self.batched_b: torch.Tensor | None = None  # [n, N, r]
        self._slot: dict[int, int] = {}  # adapter id -> row of the batched arrays
        self._needs_rebuild = True

    def add_adapter(self, name: str, weights: dict[str, torch.Tensor]) -> int:
        """Adds an adapter ({"<module>.A": [r, K], "<module>.B": [N, r]}); returns its id."""
        if len(self.adapters) >= self.max_adapters:
            raise ValueError(f"Max adapters ({self.max_adapters}) reached")
        adapter_id = self.next_id
        self.adapters[name] = weights
        self.adapter_ids[name] = adapter_id
        self.next_id += 1
        self._needs_rebuild = True
        return adapter_id

    def remove_adapter(self, name: str) -> None:
        if name in self.adapters:
            del self.adapters[name]
            del self.adapter_ids[name]
            self._needs_rebuild = True

    def list_adapters(self) -> list[str]:
        return list(self.adapters.keys())

    def _rebuild_batched(self) -> None:
        if not self.adapters or not self._needs_rebuild:
            return
        a_list, b_list, self._slot = [], [], {}
        for name, weights in self.adapters.items():
            a = next(v for k, v in weights.items() if k.endswith(".A"))
            b = next(v for k, v in weights.items() if k.endswith(".B"))
            self._slot[self.adapter_ids[name]] = len(a_list)
            dev = self.device if self.device is not None else a.device
            a_list.append(a.to(device=dev, dtype=self.dtype))
            b_list.append(b.to(device=dev, dtype=self.dtype))
        shapes = {(tuple(a.shape), tuple(b.shape)) for a, b in zip(a_list, b_list)}
        if len(shapes) != 1:
            raise ValueError("all adapters must share rank, in_features and out_features")
        self.batched_a = torch.stack(a_list)
        self.batched_b = torch.stack(b_list)
        self._needs_rebuild = False

    def forward_batched(self, x: torch.Tensor, adapter_ids: list[int]) -> torch.Tensor:
        """The LoRA term ``(x[b].A_id^T).B_id^T`` (unscaled, as at
        optimizations.py:193-217) for x [B, S, K], one adapter id per sample."""
        self._rebuild_batched()
        if self.batched_a is None:
            raise ValueError("no adapters loaded")
        slots = [self._slot[int(i)] for i in adapter_ids]
        r = self.batched_a.shape[1]
        y = multi_adapter_forward(x.to(self.dtype), None, self.batched_a, self.batched_b, slots,
                                  alpha=float(r))
        return y.to(x.dtype)


class LoRAKVCache:
    """KV cache for incremental LoRA decoding (optimizations.py:307-340): caches
    [batch, max_seq_len, num_heads, head_dim]; ``update`` appends K/V rows,
    ``project_and_update`` computes them from the new tokens with the K and V
    LoRALinear layers in one fused call that writes into the cache slot
    (kernels/lora_kernels.metal:514-586)."""

    def __init__(self, batch_size: int, max_seq_len: int, num_heads: int, head_dim: int,
                 dtype: torch.dtype = torch.float16, device=None):
        self.batch_size = batch_size
        self.max_seq_len = max_seq_len
        self.num_heads = num_heads
        self.head_dim = head_dim
        shape = (batch_size, max_seq_len, num_heads, head_dim)
        self.k_cache = torch.zeros(shape, dtype=dtype, device=device)
        self.v_cache = torch.zeros(shape, dtype=dtype, device=device)
        self.cur_pos = 0

    def update(self, k_new: torch.Tensor, v_new: torch.Tensor):
        """optimizations.py:327-336: write [batch, seq, heads, dim] at cur_pos."""
        seq_len = k_new.shape[1]
        end_pos = self.cur_pos + seq_len
        if end_pos > self.max_seq_len:
            raise ValueError(f"cache full: {end_pos} > {self.max_seq_len}")
        self.k_cache[:, self.cur_pos:end_pos] = k_new
        self.v_cache[:, self.cur_pos:end_pos] = v_new
        self.cur_pos = end_pos
        return self.k_cache[:, :end_pos], self.v_cache[:, :end_pos]

    def project_and_update(self, x: torch.Tensor, k_proj, v_proj):
        """x [batch, 1, D_in] (one new token per sequence); k_proj/v_proj are
        unmerged LoRALinear layers with dense bases and equal rank and alpha."""
        from .kernels import lora_kv_cache_update
        if self.cur_pos >= self.max_seq_len:
            raise ValueError("cache full")
        if k_proj.rank != v_proj.rank or k_proj.alpha != v_proj.alpha:
            raise ValueError("K and V projections must share rank and alpha")
        dt = self.k_cache.dtype
        x2d = x.reshape(self.batch_size, -1).to(dt)
        lora_kv_cache_update(x2d, k_proj.W0.to(dt), v_proj.W0.to(dt), k_proj.A.to(dt),
                             k_proj.B.to(dt), v_proj.A.to(dt), v_proj.B.to(dt), self.k_cache,
                             self.v_cache, self.cur_pos, k_proj.alpha)
        self.cur_pos += 1
        return self.k_cache[:, :self.cur_pos], self.v_cache[:, :self.cur_pos]

    def reset(self) -> None:
        self.cur_pos = 0
