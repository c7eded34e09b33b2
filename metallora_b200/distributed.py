"""Data parallelism for the LoRA-linear path: tokens shard across ranks (one
process per GPU); the forward needs no communication; training averages the
LoRA gradients (the only state that differs between ranks) with one
all-reduce over the flat gradient buffer.  The reference is single-device; this
is the multi-GPU layer of this implementation."""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from .exceptions import DistributedError

FAULT_ENV = "MLORA_FAULT_INJECT"


class InjectedFault(RuntimeError):
    """Raised by ``maybe_inject_fault`` on the rank and at the point that
    MLORA_FAULT_INJECT names."""


def maybe_inject_fault(point: str, rank: int | None = None) -> None:
    """Host-side fault injection for failure-detection tests.

    With MLORA_FAULT_INJECT = "<point>@<rank>" (several comma-separated), the
    rank ``rank`` (default: this process's rank in the default group) raises
    InjectedFault when it reaches ``point``.  Points: "before_allreduce" (the
    flat-gradient all-reduce) and "before_peer_allreduce" (the NVLink
    exchange).  The failure is made on the host, before anything is enqueued:
    no kernel or collective of the failing rank is in flight, and no GPU is
    faulted.  Unset, this is one environment lookup."""
    spec = os.environ.get(FAULT_ENV)
    if not spec:
        return
    if rank is None:
        rank = dist.get_rank() if dist.is_available() and dist.is_initialized() else 0
    for item in spec.split(","):
        name, _, who = item.strip().partition("@")
        if name == point and who.strip() != "" and int(who) == rank:
            raise InjectedFault(f"injected fault at {point} on rank {rank}")


def shard_bounds(n_tokens: int, rank: int, world: int) -> tuple[int, int]:
    """[begin, end) of this rank's contiguous token shard (sizes differ by at most 1)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world {world}")
    base, extra = divmod(n_tokens, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


def shard_tokens(x: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """This rank's slice of a [tokens, ...] (or [batch, seq, ...], flattened) tensor."""
    flat = x.reshape(-1, *x.shape[2:]) if x.dim() > 2 else x
    b, e = shard_bounds(flat.shape[0], rank, world)
    return flat[b:e]


def device_cpus(device) -> list[int] | None:
    """The host cores NVML reports as closest to a CUDA device (its NUMA
    node), or None when NVML or the device is unavailable.  Read-only: no
    setting of the device changes."""
    try:
        import pynvml
        pynvml.nvmlInit()
        try:
            props = torch.cuda.get_device_properties(device)
            bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
            handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            n = os.cpu_count() or 1
            words = pynvml.nvmlDeviceGetCpuAffinity(handle, (n + 63) // 64)
        finally:
            pynvml.nvmlShutdown()
    except Exception:  # no NVML, no GPU, or a device NVML does not list
        return None
    cpus = [w * 64 + b for w, m in enumerate(words) for b in range(64)
            if (int(m) >> b) & 1 and w * 64 + b < n]
    return cpus or None


def bind_to_device(device) -> list[int] | None:
    """Restricts this process to the host cores of ``device``'s NUMA node, so
    pinned host buffers it allocates afterwards sit next to the GPU's PCIe root
    (one process per GPU: each rank's host<->device copies then use its own
    socket's memory).  Returns the previous affinity (to restore), or None if
    the cores are unknown."""
    cpus = device_cpus(device)
    if not cpus or not hasattr(os, "sched_setaffinity"):
        return None
    before = sorted(os.sched_getaffinity(0))
    os.sched_setaffinity(0, cpus)
    return before


def average_gradients(flat_grad: torch.Tensor, group=None) -> None:
    """In-place mean of a flat gradient buffer over the process group (AVG on
    NCCL; SUM then scale elsewhere).

    A peer that raised, left or did not arrive ends the collective with the
    process group's timeout; the error surfaces here as DistributedError
    (gloo, and NCCL errors reported at the call).  On NCCL a timeout found
    later by torch's watchdog aborts the communicator instead."""
    if not (dist.is_available() and dist.is_initialized()):
        return
    world = dist.get_world_size(group)
    if world == 1:
        return
    rank = dist.get_rank(group)
    maybe_inject_fault("before_allreduce", rank)
    try:
        if dist.get_backend(group) == "nccl":
            dist.all_reduce(flat_grad, op=dist.ReduceOp.AVG, group=group)
        else:
            dist.all_reduce(flat_grad, group=group)
            flat_grad.mul_(1.0 / world)
    except RuntimeError as e:
        raise DistributedError(f"gradient all-reduce failed on rank {rank} of {world}: "
                               f"{str(e).splitlines()[0] if str(e) else type(e).__name__}") from e


class PeerLiveness:
    """Step-by-step membership check through the process group's key-value
    store, on the host.

    Before a rank launches a step's collectives it counts itself in for the
    step (``beat``) and waits, bounded by ``timeout_s``, until every rank of the
    group has been counted (``check``).  A peer that leaves between steps says
    so first (``leave``).  The survivors then raise DistributedError at their
    next check, before they enqueue anything, so no GPU kernel or NCCL
    collective is ever left waiting for a rank that is gone.  A peer that stops
    without saying so (a crash, a stall) surfaces as the same error once
    ``timeout_s`` has passed.  A step costs one atomic add and a few
    polls of the store, whatever the group size.

    Each instance uses its own key prefix.  Instances must be created in the
    same order on every rank, as collectives are."""

    _count = 0

    def __init__(self, group=None, timeout_s: float = 30.0, store=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.global_rank = (dist.get_global_rank(group, self.rank) if group is not None
                            else self.rank)
        self.store = store if store is not None else dist.distributed_c10d._get_default_store()
        self.timeout_s = float(timeout_s)
        PeerLiveness._count += 1
        self.prefix = f"mlora/live/{PeerLiveness._count}"

    def beat(self, step: int) -> None:
        """This rank has reached ``step`` (about to launch its collectives)."""
        self.store.add(f"{self.prefix}/arrived/{int(step)}", 1)

    def leave(self) -> None:
        """This rank leaves the group between steps; its peers' next check
        raises instead of waiting for it."""
        self.store.set(f"{self.prefix}/left_rank", str(self.global_rank))
        self.store.add(f"{self.prefix}/left", 1)

    def check(self, step: int) -> None:
        """Returns once every rank has reached ``step``; raises
        DistributedError if one has left, or has not arrived within
        ``timeout_s``."""
        import time
        key = f"{self.prefix}/arrived/{int(step)}"
        deadline = time.monotonic() + self.timeout_s
        pause = 1e-4
        while True:
            if self.store.add(f"{self.prefix}/left", 0) > 0:
                who = self.store.get(f"{self.prefix}/left_rank").decode()
                raise DistributedError(
                    f"rank {who} left the process group before step {step} "
                    f"(seen by rank {self.global_rank})")
            n = self.store.add(key, 0)
            if n >= self.world:
                if self.rank == 0 and step > 0:
                    # every rank has finished polling the previous step's count
                    self.store.delete_key(f"{self.prefix}/arrived/{int(step) - 1}")
                return
            if time.monotonic() > deadline:
                raise DistributedError(
                    f"only {n} of {self.world} ranks reached step {step} within "
                    f"{self.timeout_s:.1f} s (a rank left or stalled; seen by rank "
                    f"{self.global_rank})")
            time.sleep(pause)
            pause = min(pause * 2, 0.01)


def replicas_in_sync(t: torch.Tensor, group=None) -> bool:
    """True when every rank holds a bitwise-identical copy of ``t`` (checked
    through an all-gathered checksum)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size(group) == 1:
        return True
    v = t.detach().reshape(-1).view(torch.int32) if t.element_size() == 4 else \
        t.detach().reshape(-1).to(torch.float32).view(torch.int32)
    chk = torch.stack([v.sum(dtype=torch.int64), (v.to(torch.int64) * 31).sum()]).to(t.device)
    out = [torch.zeros_like(chk) for _ in range(dist.get_world_size(group))]
    dist.all_gather(out, chk, group=group)
    return all(torch.equal(o, out[0]) for o in out)


class PeerAllReduce:
    """Averages one small fp32 buffer over the ranks with a single kernel that
    reads the peers' copies over NVLink (``mlora_peer_allreduce``): a flag
    barrier, an in-rank-order sum (bitwise identical on every rank) and a
    closing barrier, so ``buffer`` may be overwritten once the call's kernel has
    run.  ``buffer`` (and the flags) live in symmetric memory; gradients are
    accumulated straight into it.  One-shot reads (world - 1) x the buffer per
    rank, so it is used for buffers up to ``MAX_BYTES``; larger ones, and
    process groups without symmetric memory, keep NCCL (``create`` returns None).
    """

    MAX_BYTES = 8 << 20

    def __init__(self, numel: int, group=None, device=None):
        import torch.distributed._symmetric_memory as symm_mem

        from . import _lib
        self._lib = _lib
        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self.numel = int(numel)
        dev = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        self.buffer = symm_mem.empty(self.numel, dtype=torch.float32, device=dev)
        self.flags = symm_mem.empty(max(self.world, 4), dtype=torch.int32, device=dev)
        self.buffer.zero_()
        self.flags.zero_()
        # every rank's flags are zero before any rank can raise one
        torch.cuda.synchronize(dev)
        name = self.group.group_name
        self._hb = symm_mem.rendezvous(self.buffer, name)
        self._hf = symm_mem.rendezvous(self.flags, name)
        dist.barrier(self.group)
        # arrival count, verdict seq and verdict (this GPU's memory)
        self.counter = torch.zeros(4, dtype=torch.int32, device=dev)
        self.seq = 0

    @classmethod
    def create(cls, numel: int, group=None, device=None) -> "PeerAllReduce | None":
        """A peer all-reduce for this group, or None where it does not apply."""
        if not (dist.is_available() and dist.is_initialized()) or not torch.cuda.is_available():
            return None
        g = group if group is not None else dist.group.WORLD
        if dist.get_world_size(g) < 2 or dist.get_backend(g) != "nccl":
            return None
        if numel * 4 > cls.MAX_BYTES:
            return None
        try:
            return cls(numel, g, device)
        except Exception:  # no peer access / symmetric memory on this system
            return None

    def allreduce(self, out: torch.Tensor, average: bool = True) -> torch.Tensor:
        """out = mean (or sum) over ranks of ``buffer``; out is a separate
        contiguous fp32 tensor of ``numel`` elements on this GPU."""
        if out.dtype != torch.float32 or out.numel() != self.numel or not out.is_contiguous():
            raise ValueError("out must be a contiguous fp32 tensor of the buffer's size")
        maybe_inject_fault("before_peer_allreduce", self.rank)
        self.seq += 1
        st = self._lib.load().mlora_peer_allreduce(
            self._hb.buffer_ptrs_dev, self._hf.buffer_ptrs_dev, self.rank, self.world, self.seq,
            out.data_ptr(), self.numel, (1.0 / self.world) if average else 1.0,
            self.counter.data_ptr(), torch.cuda.current_stream().cuda_stream)
        self._lib.check(st, "mlora_peer_allreduce")
        return out


class BucketedGradExchange:
    """Averages a flat gradient buffer over the ranks in buckets, each started
    as soon as the backward has written its part, so the exchange of later
    layers' gradients runs while earlier layers' backward still computes.

    ``members`` lists, in the flat buffer's order, the (begin, end) element
    range each gradient producer (one LoRALinear) writes.  Consecutive members
    are grouped into buckets of at least ``bucket_bytes``.  ``ready(i)`` is
    called once producer i's gradients are enqueued on the current stream;
    when every member of a bucket is ready, the bucket's slice is all-reduced
    (mean) -- on CUDA on a side stream after an event on the producing stream,
    elsewhere (gloo on CPU) at once.  ``finish()`` starts any bucket that did
    not fire (producers that took no part in this backward), in bucket order,
    and makes the current stream wait for the exchange.

    Every rank must run the same backward (the same producers in the same
    order), so that all ranks issue the same collectives in the same order.  A
    producer that reports twice in one step (a layer applied twice in one
    forward) raises DistributedError: its bucket would be averaged before all
    of its gradient had arrived."""

    def __init__(self, flat: torch.Tensor, members: list[tuple[int, int]], group=None,
                 bucket_bytes: int = 4 << 20):
        self.flat = flat
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.nccl = dist.get_backend(group) == "nccl"
        self.buckets: list[tuple[int, int, list[int]]] = []
        self.bucket_of: list[int] = []
        cur: list[int] = []
        start = None
        elt = flat.element_size()
        for i, (b, e) in enumerate(members):
            if cur and b != members[cur[-1]][1]:
                raise ValueError("members must tile the flat buffer contiguously")
            if not cur:
                start = b
            cur.append(i)
            self.bucket_of.append(len(self.buckets))
            if (e - start) * elt >= bucket_bytes or i == len(members) - 1:
                self.buckets.append((start, e, cur))
                cur = []
        self.cuda = flat.is_cuda
        self.stream = torch.cuda.Stream(device=flat.device) if self.cuda else None
        self.armed = True
        self.fired_order: list[int] = []
        self._reset()

    def _reset(self) -> None:
        self.seen = [False] * len(self.bucket_of)
        self.pending = [len(m) for _, _, m in self.buckets]
        self.fired = [False] * len(self.buckets)
        self.fired_order = []

    def _fire(self, k: int) -> None:
        b, e, _ = self.buckets[k]
        if not self.fired_order:
            maybe_inject_fault("before_allreduce", self.rank)
        self.fired[k] = True
        self.fired_order.append(k)
        part = self.flat[b:e]
        try:
            if self.cuda:
                ev = torch.cuda.Event()
                ev.record(torch.cuda.current_stream(self.flat.device))
                self.stream.wait_event(ev)
                with torch.cuda.stream(self.stream):
                    if self.nccl:
                        dist.all_reduce(part, op=dist.ReduceOp.AVG, group=self.group)
                    else:
                        dist.all_reduce(part, group=self.group)
                        part.mul_(1.0 / self.world)
            else:
                dist.all_reduce(part, group=self.group)
                part.mul_(1.0 / self.world)
        except RuntimeError as err:
            raise DistributedError(
                f"gradient bucket all-reduce failed on rank {self.rank} of {self.world}: "
                f"{str(err).splitlines()[0] if str(err) else type(err).__name__}") from err

    def ready(self, i: int) -> None:
        """Producer i's gradients are enqueued on the current stream."""
        if not self.armed:
            return
        if self.seen[i]:
            raise DistributedError(
                f"gradient producer {i} reported twice in one step (a layer used twice in one "
                "forward); construct the trainer with overlap_grad_exchange=False")
        self.seen[i] = True
        k = self.bucket_of[i]
        self.pending[k] -= 1
        if self.pending[k] == 0:
            self._fire(k)

    def finish(self) -> None:
        """Fires what is left and joins the exchange into the current stream."""
        for k in range(len(self.buckets)):
            if not self.fired[k]:
                self._fire(k)
        if self.cuda:
            torch.cuda.current_stream(self.flat.device).wait_stream(self.stream)
        self._reset()
