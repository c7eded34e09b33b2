"""LoRA training (reference: python/metal_lora/trainer.py).

Keeps the reference's ``TrainingConfig`` (trainer.py:71-100), ``TrainingState``
(:103-112), ``LoRATrainableModule`` (:115-170), ``LoRATrainer`` (``_training_step`` :228-249, ``train`` :251-289,
``save``/``load`` :291-302), ``MetalAdamW`` (:21-68), ``train_lora`` (:305-318)
and ``quick_finetune`` (:321-331).  The reference's trainer wraps the model in a
module that never routes its LoRA tensors into the forward (trainer.py:133-170),
so its step does not train; this trainer implements the step the reference
intends and its examples run (examples/train_example.py:200-218): LoRALinear
modules are applied to the target projections, the loss is differentiated with
respect to the A/B factors only, the gradients are clipped by global norm
(trainer.py:237-240) and AdamW updates the factors.

Flat buffers: every A and B of the model is a view into one fp32 master array
(the factors the optimizer updates), with a compute-dtype copy (bf16 when the
base weights are bf16) refreshed by one copy per step, and one fp32 gradient
array that the backward kernels accumulate into.  The clip is then one
reduction kernel and AdamW one kernel launch for all adapters.  Under data
parallelism the gradient array is averaged over the ranks in per-layer buckets
(NCCL on a side stream), each started as soon as the backward has written it,
so the exchange overlaps the backward of the layers before it.  Data-parallel
replicas start from the first rank's factors (broadcast at construction), and
each step first checks on the host, through the process group's store, that
every peer reached it (``PeerLiveness``): a rank that leaves between steps
(``LoRATrainer.leave``) or stops turns the others' next step into a
DistributedError before any collective of that step is launched.
"""
from __future__ import annotations

import json
import time
from collections.abc import Iterator
from dataclasses import dataclass, field
from pathlib import Path

import torch
import torch.distributed as dist
from torch import nn

from . import kernels as _k
from .distributed import BucketedGradExchange, PeerLiveness, average_gradients
from .exceptions import ConfigurationError
from .layers import LoRALinear
from .logging import logger
from .utils import apply_lora_to_model


@dataclass
class TrainingConfig:
    """trainer.py:71-100 (same fields and defaults)."""
    rank: int = 16
    alpha: float = 32.0
    dropout: float = 0.0
    target_modules: list[str] = field(default_factory=lambda: ["q_proj", "v_proj"])

    learning_rate: float = 1e-4
    weight_decay: float = 0.01
    batch_size: int = 4
    gradient_accumulation_steps: int = 1
    max_grad_norm: float = 1.0

    optimizer: str = "adamw"
    beta1: float = 0.9
    beta2: float = 0.999
    eps: float = 1e-8

    warmup_steps: int = 100
    lr_scheduler: str = "cosine"

    use_fp16: bool = True
    gradient_checkpointing: bool = False

    log_interval: int = 10
    eval_interval: int = 100
    save_interval: int = 500

    output_dir: str = "./lora_output"


@dataclass
class TrainingState:
    """trainer.py:103-112."""
    global_step: int = 0
    epoch: int = 0
    best_loss: float = float("inf")
    train_loss: float = 0.0
    learning_rate: float = 0.0
    tokens_seen: int = 0
    start_time: float = 0.0


class LoRATrainableModule(nn.Module):
    """Makes a model LoRA-trainable (reference: trainer.py:115-170).

    Same constructor, default targets (q/v/k/o_proj), key names and counting
    methods as the reference wrapper.  The reference keeps A/B in side
    dictionaries that its forward never reads; here every targeted
    ``nn.Linear`` becomes a ``LoRALinear``, so the factors are used by the
    forward.  Like the reference (trainer.py:144-146), A starts as
    N(0, 0.02^2) and B as zeros; the base weights are frozen
    (trainer.py:147).  ``get_lora_params`` returns live references to the
    modules' A/B under the keys ``{module}.lora_A`` / ``{module}.lora_B``
    (trainer.py:149-154), which is also the key set of ``LoRATrainer.save``."""

    def __init__(self, base_model: nn.Module, rank: int = 16, alpha: float = 32.0,
                 target_modules: list[str] | None = None, dropout: float = 0.0):
        super().__init__()
        self.base_model = base_model
        self.rank = rank
        self.alpha = alpha
        self.dropout = dropout
        self.target_modules = target_modules or ["q_proj", "v_proj", "k_proj", "o_proj"]
        self._apply_lora()

    def _lora_layers(self) -> dict[str, LoRALinear]:
        return {n: m for n, m in self.base_model.named_modules() if isinstance(m, LoRALinear)}

    @torch.no_grad()
    def _apply_lora(self) -> None:
        before = set(self._lora_layers())
        apply_lora_to_model(self.base_model, rank=self.rank, alpha=self.alpha,
                            target_modules=self.target_modules, dropout=self.dropout)
        for name, m in self._lora_layers().items():
            if name not in before:
                m.A.copy_(torch.randn(m.A.shape, dtype=torch.float32).to(m.A) * 0.02)
                m.B.zero_()
        for p in self.base_model.parameters():
            p.requires_grad_(False)
        for m in self._lora_layers().values():
            m.A.requires_grad_(True)
            m.B.requires_grad_(True)

    def get_lora_params(self) -> dict[str, torch.Tensor]:
        params = {}
        for name, m in self._lora_layers().items():
            params[f"{name}.lora_A"] = m.A
            params[f"{name}.lora_B"] = m.B
        return params

    @torch.no_grad()
    def set_lora_params(self, params: dict[str, torch.Tensor]) -> None:
        """Copies ``{module}.lora_A`` / ``.lora_B`` values into the modules
        (trainer.py:156-161); keys of other modules are ignored."""
        layers = self._lora_layers()
        for key, value in params.items():
            for suffix, attr in ((".lora_A", "A"), (".lora_B", "B")):
                if key.endswith(suffix) and key[:-len(suffix)] in layers:
                    dst = getattr(layers[key[:-len(suffix)]], attr)
                    if tuple(value.shape) != tuple(dst.shape):
                        raise ConfigurationError(f"{key}: shape {tuple(value.shape)} does not "
                                                 f"match {tuple(dst.shape)}")
                    dst.copy_(value.to(dst.device, dst.dtype))

    def num_trainable_params(self) -> int:
        return sum(m.A.numel() + m.B.numel() for m in self._lora_layers().values())

    def num_total_params(self) -> int:
        """Base parameters plus the LoRA factors (trainer.py:166-167)."""
        lora = {id(m.A) for m in self._lora_layers().values()} | \
               {id(m.B) for m in self._lora_layers().values()}
        base = sum(p.numel() for p in self.base_model.parameters() if id(p) not in lora)
        return base + self.num_trainable_params()

    def forward(self, *args, **kwargs):
        return self.base_model(*args, **kwargs)


class FlatLoRAParams:
    """Rebinds the A/B factors of every LoRALinear in ``model`` as views of one
    fp32 master buffer, with a flat fp32 gradient buffer wired into the layers'
    backward and (if the layers compute in another dtype) a flat compute copy."""

    def __init__(self, model: nn.Module):
        self.layers: list[tuple[str, LoRALinear]] = [
            (n, m) for n, m in model.named_modules() if isinstance(m, LoRALinear)]
        if not self.layers:
            raise ConfigurationError("model has no LoRALinear modules")
        dev = self.layers[0][1].W0.device
        self.compute_dtype = self.layers[0][1].W0.dtype
        sizes = []
        for _, m in self.layers:
            if m.rank % 8:
                raise ConfigurationError("flat LoRA buffers need ranks that are multiples of 8")
            sizes += [m.A.numel(), m.B.numel()]
        self.numel = sum(sizes)
        self.master = torch.empty(self.numel, dtype=torch.float32, device=dev)
        self.grad = torch.zeros(self.numel, dtype=torch.float32, device=dev)
        self.compute = (None if self.compute_dtype == torch.float32 else
                        torch.empty(self.numel, dtype=self.compute_dtype, device=dev))
        self.slices: dict[str, tuple[int, int, tuple]] = {}
        off = 0
        with torch.no_grad():
            for name, m in self.layers:
                views = []
                for pname in ("A", "B"):
                    p = getattr(m, pname)
                    n = p.numel()
                    self.master[off:off + n].copy_(p.detach().reshape(-1).float())
                    self.slices[f"{name}.{pname}"] = (off, n, tuple(p.shape))
                    views.append((off, n, tuple(p.shape)))
                    off += n
                (oa, na, sa), (ob, nb, sb) = views
                m.A = nn.Parameter(self.master[oa:oa + na].view(sa))
                m.B = nn.Parameter(self.master[ob:ob + nb].view(sb))
                m._grad_sink = (self.grad[oa:oa + na].view(sa), self.grad[ob:ob + nb].view(sb))
                if self.compute is not None:
                    m._compute_ab = (self.compute[oa:oa + na].view(sa),
                                     self.compute[ob:ob + nb].view(sb))
        self.refresh_compute()

    def attach_exchange(self, group=None, bucket_bytes: int = 4 << 20):
        """A BucketedGradExchange over the flat gradient buffer, with each
        layer's gradient sink calling it once its dA/dB are written."""
        members = []
        for name, m in self.layers:
            oa = self.slices[f"{name}.A"][0]
            ob, nb, _ = self.slices[f"{name}.B"]
            members.append((oa, ob + nb))
        ex = BucketedGradExchange(self.grad, members, group, bucket_bytes)
        for i, (_, m) in enumerate(self.layers):
            ga, gb = m._grad_sink[:2]
            m._grad_sink = (ga, gb, True, lambda i=i: ex.ready(i))
        return ex

    def refresh_compute(self) -> None:
        """Copies the fp32 masters into the compute-dtype views (one kernel)."""
        if self.compute is not None:
            with torch.no_grad():
                self.compute.copy_(self.master)

    def named_tensors(self) -> dict[str, torch.Tensor]:
        return {k: self.master[o:o + n].view(s) for k, (o, n, s) in self.slices.items()}


class MetalAdamW:
    """AdamW on the flat buffers (reference: trainer.py:21-68 over the Metal
    kernels kernels.py:314-362).  One fused launch per step; weight_decay=0
    gives Adam; ``kind="sgd"`` plain SGD."""

    def __init__(self, params: FlatLoRAParams, learning_rate: float,
                 betas: tuple[float, float] = (0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.01, kind: str = "adamw"):
        self.params = params
        self.learning_rate = learning_rate
        self.beta1, self.beta2 = betas
        self.eps = eps
        self.weight_decay = weight_decay if kind == "adamw" else 0.0
        self.kind = kind
        dev = params.master.device
        self.gpu_state = _k.persistent_gpu_state_init(self.beta1, self.beta2, dev)
        self.m = torch.zeros_like(params.master)
        self.v = torch.zeros_like(params.master)

    def update(self, grad_scale: torch.Tensor | None = None) -> None:
        p = self.params
        if self.kind == "sgd":
            _k.sgd_step(p.master, p.grad, self.learning_rate, grad_scale)
        else:
            _k.persistent_gpu_state_step(self.gpu_state, self.beta1, self.beta2)
            _k.lora_adamw_step_metal(p.master, p.grad, self.m, self.v, self.gpu_state,
                                     self.learning_rate, self.beta1, self.beta2, self.eps,
                                     self.weight_decay, grad_scale)
        p.refresh_compute()

    def state_dict(self) -> dict:
        return {"m": self.m, "v": self.v, "gpu_state": self.gpu_state}

    def load_state_dict(self, sd: dict) -> None:
        self.m.copy_(sd["m"])
        self.v.copy_(sd["v"])
        self.gpu_state.copy_(sd["gpu_state"])


class LoRATrainer:
    """LoRA trainer (reference: trainer.py:173-302)."""

    def __init__(self, model: nn.Module, config: TrainingConfig | None = None,
                 process_group=None, overlap_grad_exchange: bool = True,
                 liveness_timeout: float | None = 30.0):
        self.config = config or TrainingConfig()
        c = self.config
        if not any(isinstance(m, LoRALinear) for m in model.modules()):
            apply_lora_to_model(model, rank=c.rank, alpha=c.alpha,
                                target_modules=c.target_modules, dropout=c.dropout)
        self.model = model
        for p in model.parameters():
            p.requires_grad_(False)
        self.params = FlatLoRAParams(model)
        self.optimizer = self._create_optimizer()
        self.state = TrainingState()
        self.group = process_group
        self._micro = 0
        # data parallel: per-layer gradient buckets averaged on a side stream
        # while the backward of earlier layers runs (None: one all-reduce of
        # the flat buffer after the backward)
        self.exchange = None
        data_parallel = dist.is_available() and dist.is_initialized() and \
            dist.get_world_size(process_group) > 1
        if data_parallel:
            # every replica starts from the first rank's LoRA factors (as
            # DistributedDataParallel does), so averaged gradients keep them equal
            src = dist.get_global_rank(process_group, 0) if process_group is not None else 0
            dist.broadcast(self.params.master, src=src, group=process_group)
            self.params.refresh_compute()
        if overlap_grad_exchange and data_parallel:
            self.exchange = self.params.attach_exchange(process_group)
        # data parallel: every training step first checks on the host that all
        # peers reached it (None: no check; a departed peer then surfaces as a
        # collective timeout)
        self.liveness = (PeerLiveness(process_group, liveness_timeout)
                         if data_parallel and liveness_timeout is not None else None)
        self._clip = torch.ones(2, dtype=torch.float32, device=self.params.master.device)
        Path(c.output_dir).mkdir(parents=True, exist_ok=True)

    def _create_optimizer(self) -> MetalAdamW:
        c = self.config
        kind = c.optimizer.lower()
        if kind not in ("adamw", "adam", "sgd"):
            raise ConfigurationError(f"unknown optimizer {c.optimizer}")
        return MetalAdamW(self.params, c.learning_rate, (c.beta1, c.beta2), c.eps,
                          c.weight_decay, kind)

    def _compute_loss(self, batch: dict[str, torch.Tensor]) -> torch.Tensor:
        """trainer.py:216-226: shifted cross-entropy on ``labels``, else MSE to
        ``target_output`` (or to the output itself)."""
        outputs = self.model(batch["input_ids"])
        if "labels" in batch:
            logits = outputs[:, :-1, :]
            labels = batch["labels"][:, 1:]
            return nn.functional.cross_entropy(logits.reshape(-1, logits.shape[-1]).float(),
                                               labels.reshape(-1))
        target = batch.get("target_output", outputs.detach())
        return torch.mean((outputs.float() - target.float()) ** 2)

    def backward(self, batch: dict[str, torch.Tensor]) -> torch.Tensor:
        """Forward + backward of one micro-batch; LoRA gradients accumulate in
        the flat fp32 buffer (under data parallelism, the last micro-batch
        before an optimizer step also starts each layer bucket's average as
        soon as its gradients are written)."""
        if self.exchange is not None:
            gas = max(1, self.config.gradient_accumulation_steps)
            self.exchange.armed = (self._micro + 1) % gas == 0
        loss = self._compute_loss(batch)
        scale = 1.0 / max(1, self.config.gradient_accumulation_steps)
        (loss * scale).backward()
        return loss.detach()

    def optimizer_step(self) -> None:
        """Data-parallel average (one all-reduce), global-norm clip
        (trainer.py:237-240), AdamW; all on the device, no host sync."""
        g = self.params.grad
        if self.exchange is not None:
            self.exchange.finish()
        else:
            average_gradients(g, self.group)
        if self.config.max_grad_norm > 0:
            _k.grad_norm_clip(g, self.config.max_grad_norm, out=self._clip)
            self.optimizer.update(self._clip[:1])
        else:
            self.optimizer.update(None)

    def leave(self) -> None:
        """Leaves data-parallel training between steps: the other ranks' next
        step raises DistributedError before it launches anything."""
        if self.liveness is not None:
            self.liveness.leave()

    def _training_step(self, batch: dict[str, torch.Tensor]) -> dict[str, float]:
        """trainer.py:228-249 (loss returned as a float, as the reference does)."""
        if self.liveness is not None:
            self.liveness.beat(self._micro)
            self.liveness.check(self._micro)
        loss = self.backward(batch)
        self._micro += 1
        if self._micro % max(1, self.config.gradient_accumulation_steps) == 0:
            self.optimizer_step()
            self.state.global_step += 1
        x = batch["input_ids"]
        self.state.tokens_seen += int(x.shape[0] * x.shape[1]) if x.dim() >= 2 else int(x.numel())
        return {"loss": float(loss)}

    def train(self, train_data: Iterator[dict[str, torch.Tensor]], num_epochs: int = 1,
              num_steps: int | None = None) -> dict[str, list[float]]:
        """trainer.py:251-289."""
        self.state.start_time = time.time()
        history: dict[str, list[float]] = {"loss": [], "step": []}
        from .utils import count_lora_parameters
        stats = count_lora_parameters(self.model)
        print(f"Trainable: {stats['trainable']:,} | Total: {stats['total']:,}")
        step = 0
        for epoch in range(num_epochs):
            self.state.epoch = epoch
            for batch in train_data:
                metrics = self._training_step(batch)
                step += 1
                if step % self.config.log_interval == 0:
                    print(f"Step {step} | Loss: {metrics['loss']:.4f}")
                    history["loss"].append(metrics["loss"])
                    history["step"].append(step)
                if step % self.config.save_interval == 0:
                    self.save(f"{self.config.output_dir}/checkpoint-{step}")
                if num_steps and step >= num_steps:
                    break
            if num_steps and step >= num_steps:
                break
        self.save(f"{self.config.output_dir}/final")
        return history

    def save(self, path: str | Path) -> None:
        """trainer.py:291-297: ``adapter.safetensors`` with ``{name}.lora_A`` /
        ``{name}.lora_B`` and ``config.json`` = {rank, alpha}; the optimizer
        state goes to ``optimizer.safetensors`` so training can resume."""
        from safetensors.torch import save_file
        p = Path(path)
        p.mkdir(parents=True, exist_ok=True)
        tensors = {}
        for name, t in self.params.named_tensors().items():
            mod, which = name.rsplit(".", 1)
            tensors[f"{mod}.lora_{which}"] = t.detach().contiguous().cpu()
        save_file(tensors, str(p / "adapter.safetensors"))
        opt = {k: v.detach().contiguous().cpu() for k, v in self.optimizer.state_dict().items()}
        save_file(opt, str(p / "optimizer.safetensors"))
        with open(p / "config.json", "w") as f:
            json.dump({"rank": self.config.rank, "alpha": self.config.alpha,
                       "global_step": self.state.global_step}, f)

    def load(self, path: str | Path) -> None:
        """trainer.py:299-302 (plus the optimizer state when present)."""
        from safetensors.torch import load_file
        p = Path(path)
        tensors = load_file(str(p / "adapter.safetensors"))
        views = self.params.named_tensors()
        with torch.no_grad():
            for key, t in tensors.items():
                mod, which = key.rsplit(".lora_", 1)
                views[f"{mod}.{which}"].copy_(t)
        if (p / "optimizer.safetensors").is_file():
            sd = load_file(str(p / "optimizer.safetensors"))
            self.optimizer.load_state_dict({k: v.to(self.params.master.device)
                                            for k, v in sd.items()})
        self.params.refresh_compute()
        logger.info(f"loaded adapter from {p}")


def train_lora(model: nn.Module, train_data, rank: int = 16, alpha: float = 32.0,
               learning_rate: float = 1e-4, num_epochs: int = 1,
               output_dir: str = "./lora_output") -> LoRATrainer:
    """trainer.py:305-318."""
    config = TrainingConfig(rank=rank, alpha=alpha, learning_rate=learning_rate,
                            output_dir=output_dir)
    trainer = LoRATrainer(model, config)
    trainer.train(train_data, num_epochs=num_epochs)
    return trainer


def quick_finetune(model: nn.Module, texts: list[str], tokenizer, rank: int = 8,
                   num_steps: int = 100) -> LoRATrainer:
    """trainer.py:321-331 (the tokenizer returns numpy ids; batches of 4)."""
    dev = next(model.parameters()).device

    def data_gen():
        for i in range(0, len(texts), 4):
            tokens = tokenizer(texts[i:i + 4], padding=True, return_tensors="np")
            ids = torch.as_tensor(tokens["input_ids"], device=dev)
            yield {"input_ids": ids, "labels": ids}

    trainer = LoRATrainer(model, TrainingConfig(rank=rank))
    trainer.train(data_gen(), num_steps=num_steps)
    return trainer
