"""Benchmark of the LoRA-linear hot path (one JSON line on rank 0).

Workload (default): the bf16 fused LoRA forward+backward at 4096 -> 4096,
rank 16, alpha 32, 8192 tokens (batch 4 x seq 2048) per GPU -- one "step" is
forward (y) plus backward (dx, dA, dB) of that batch through ``LoRALinear``,
and for N > 1 GPUs the all-reduce of the LoRA gradients (weak scaling: every
rank processes its own 8192 tokens).  Inputs are synthetic (seeded normal /
uniform draws with the reference configuration's distributions); they total
~290 MB per GPU, larger than the 126 MB L2, so no flush is needed.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

``--impl reference`` times the reference's CPU path instead: the numpy
restatement of its pure-MLX op sequence (oracle/lora_oracle.py) on the host
cores, on bounded token samples of the same workload.

Other configurations of the same path (one JSON line per case):

    --workload stack   32 Llama-7B-shaped layers of projections (q,k,v,o 4096->4096,
                       gate,up 4096->11008, down 11008->4096), NF4 bases, rank 16,
                       one training step (fwd + bwd + clip + AdamW on A/B) over
                       8 x 4096 tokens, MSE to an N(0,1) target; tokens shard
                       across GPUs (strong scaling), LoRA grads all-reduced.
                       Per layer (n = per-token RMS norm, no weight):
                       a = (q(n(h))+k(n(h))+v(n(h)))/sqrt3; h = h + o(a);
                       h = h + down(gate(n(h))*up(n(h))).
    --workload nf4     NF4 11008x4096 base (block 64), rank 64, alpha 128:
                       forward and backward at 1, 16, 512, 4096 tokens.
    --workload int     INT4/INT8 group-128 bases, 4096->4096 and 4096->14336,
                       rank 16: forward unmerged and merged, 1..4096 tokens.
    --workload fp32    fp32 forward 4096->4096, rank 16, 2048 tokens, and merged.
    --workload multi   per-sample adapters: 16 samples x 512 tokens, 4096->4096,
                       r 16, 1/4/16/64 adapters (one rank pass over the stacked
                       adapters + the tcgen05 GEMM), against one adapter.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

WORKLOAD = {
    "workload": "lora_linear_fwd_bwd_bf16",
    "in_features": 4096,
    "out_features": 4096,
    "rank": 16,
    "alpha": 32.0,
    "tokens_per_gpu": 8192,
    "batch": 4,
    "seq_len": 2048,
}
METRIC = "LoRA-linear fwd+bwd tokens/s (bf16, 4096->4096, r16)"


def flops_per_token(K, N, r):
    fwd = 2.0 * (K * N + K * r + r * N)
    bwd = 2.0 * (N * K + 2 * N * r + 2 * r * K)
    return fwd + bwd


# The ncu capture of one lora_gemm_pair_kernel launch of this workload
# (forward y); its dram__bytes_read.sum / dram__bytes_write.sum rows give the
# roofline line's measured traffic.  Algorithmic bytes of that launch: x
# 64 MiB + W0 32 MiB + rank block (s.x.A^T 1 MiB, B 128 KiB) read, y 64 MiB
# written.
GEMM_PROFILE = Path("profiles") / "lora_gemm_pair_kernel_fwd_bf16_m8192_k4096_n4096_r16.md"
GEMM_ALGORITHMIC_BYTES = (64 + 32 + 1.125 + 64) * 2 ** 20


def profile_traffic(rel_path: Path):
    """(bytes per launch, source) from the dram__bytes_read.sum and
    dram__bytes_write.sum rows ("| metric | 111.2 MB |") of a committed ncu
    summary, or (None, reason)."""
    f = ROOT / rel_path
    if not f.is_file():
        return None, f"{rel_path} missing"
    vals = {}
    for ln in f.read_text().splitlines():
        cells = [c.strip() for c in ln.strip().strip("|").split("|")]
        if len(cells) >= 2 and cells[0] in ("dram__bytes_read.sum", "dram__bytes_write.sum"):
            num, _, unit = cells[1].partition(" ")
            scale = {"B": 1.0, "KB": 1e3, "MB": 1e6, "GB": 1e9}.get(unit.strip(), None)
            try:
                vals[cells[0]] = float(num) * scale
            except (TypeError, ValueError):
                pass
    if len(vals) != 2:
        return None, f"{rel_path} has no dram__bytes_read/write rows"
    return sum(vals.values()), (f"{rel_path}: ncu dram__bytes_read.sum + dram__bytes_write.sum "
                                "of one forward launch of this workload")


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.is_file():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def pick_peak(peaks, clocks, kind="bf16"):
    """The roofline denominator for a kernel timed under ``clocks`` (the
    sampler's summary of the timed region): the burst figure when no sample
    saw the power cap (a short region at full clock), the power-capped
    sustained figure otherwise.  Returns (peak, name, why)."""
    if kind == "hbm":
        return peaks["hbm_gbs"], f"{peaks['source']} hbm_gbs", "HBM copy bandwidth"
    capped = "sw_power_cap" in (clocks.get("reasons") or [])
    if capped:
        return (peaks["bf16_tflops_sustained"], f"{peaks['source']} bf16_tflops_sustained",
                "sw_power_cap active during the timed region")
    return (peaks["bf16_tflops"], f"{peaks['source']} bf16_tflops (burst)",
            f"no power-cap sample in the timed region (SM {clocks.get('sm_mhz')} MHz)")


# --------------------------------------------------------------- clocks ----

class ClockSampler:
    """Samples nvidia-smi clocks/throttle reasons in the background."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.samples: list[tuple[float, list[str]]] = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.gpu), "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append((time.time(), [f.strip() for f in line.split(",")]))

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self, t0: float, t1: float):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        inside = [s for t, s in self.samples if t0 - 0.15 <= t <= t1 + 0.15]
        if not inside:  # timed region shorter than the sampling period: nearest samples
            near = sorted(self.samples, key=lambda ts: min(abs(ts[0] - t0), abs(ts[0] - t1)))
            inside = [s for _, s in near[:3]]
        sm = [float(s[1]) for s in inside if s[1].replace(".", "").isdigit()]
        smax = [float(s[2]) for s in inside if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in inside for i in range(4)
                          if len(s) > 5 + i and s[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": reasons,
                "samples": len(inside)}


# --------------------------------------------------------- CPU baseline ----

def _bf16(a):
    """Round-to-nearest-even to bf16, kept in fp32."""
    a = np.asarray(a, np.float32)
    b = a.view(np.uint32)
    b = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16
    return b.astype(np.uint32).view(np.float32)


def _cpu_inputs(tokens: int, seed: int = 0):
    """The headline workload's inputs for `tokens` tokens (same distributions
    as our arm), bf16-rounded, in fp32 host arrays."""
    K, N, r = (WORKLOAD[k] for k in ("in_features", "out_features", "rank"))
    rng = np.random.default_rng(seed)
    return {"x": _bf16(rng.standard_normal((tokens, K))),
            "W": _bf16(rng.standard_normal((N, K)) / 64),
            "A": _bf16(rng.uniform(-1 / 64, 1 / 64, (r, K))),
            "B": _bf16(rng.standard_normal((N, r)) * np.sqrt(0.02)),
            "dy": _bf16(rng.standard_normal((tokens, N)))}


def _cpu_step(inp):
    """One step of the reference's CPU op path (forward, dx, dA, dB) in numpy."""
    from oracle import lora_oracle as lo
    alpha = WORKLOAD["alpha"]
    lo.lora_forward(inp["x"], inp["W"], inp["A"], inp["B"], alpha)
    lo.lora_grad_x(inp["dy"], inp["W"], inp["A"], inp["B"], alpha)
    lo.lora_backward(inp["dy"], inp["x"], inp["A"], inp["B"], alpha, None)


def _cpu_model() -> str:
    try:
        return next((ln.split(":", 1)[1].strip() for ln in open("/proc/cpuinfo")
                     if ln.startswith("model name")), "unknown")
    except OSError:
        return "unknown"


def _blas_threads() -> int:
    from threadpoolctl import threadpool_info
    return max([i.get("num_threads", 1) for i in threadpool_info()
                if i.get("user_api") == "blas"] or [1])


def cpu_baseline(tokens: int, reps: int, seed: int = 0):
    """Times the numpy restatement of the reference's CPU op path (forward,
    dx, dA, dB in fp32 on bf16-rounded inputs) on `tokens` tokens; inputs are
    built before the timed region."""
    from threadpoolctl import threadpool_limits
    inp = _cpu_inputs(tokens, seed)
    cores = len(os.sched_getaffinity(0))
    times = []
    # every host core (torchrun caps OpenBLAS at OMP_NUM_THREADS=1 otherwise)
    with threadpool_limits(limits=cores, user_api="blas"):
        for _ in range(reps + 1):
            t = time.perf_counter()
            _cpu_step(inp)
            times.append(time.perf_counter() - t)
        cores = _blas_threads()
    med = statistics.median(times[1:])  # first run warms caches/threads
    return {"value": tokens / med, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"{tokens} tokens x {reps} reps of fwd+dx+dA+dB (numpy fp32 on bf16-rounded "
                      f"inputs, OpenBLAS, {_cpu_model()})",
            "seconds_per_rep": med}


def nf4_cpu_baseline(qw, x, A, B, alpha, group, reps: int = 3):
    """Times the oracle's numpy restatement of the reference's NF4 forward
    (kernels/lora_quantized.metal:97-164: dequantise the NF4 weight in fp32,
    then y = x.W^T + s.(x.A^T).B^T) on the host cores, on the same weight and
    tokens: the CPU beside the decode kernel.  Median of ``reps`` calls after
    one warm-up; inputs are on the host before the timed region."""
    from threadpoolctl import threadpool_limits

    from oracle import lora_oracle as lo
    from oracle import quant_oracle as qo
    N, K = qw.shape
    codes = qw.codes.cpu().numpy()
    absmax = qw.scales.float().cpu().numpy()
    xf, Af, Bf = (t.float().cpu().numpy() for t in (x, A, B))
    cores = len(os.sched_getaffinity(0))
    times = []
    with threadpool_limits(limits=cores, user_api="blas"):
        for _ in range(reps + 1):
            t = time.perf_counter()
            W = qo.dequant_nf4(codes, absmax, K, group)
            lo.lora_forward(xf, W, Af, Bf, alpha, np.float32)
            times.append(time.perf_counter() - t)
        cores = _blas_threads()
    med = statistics.median(times[1:])
    return {"value": round(med * 1e3, 2), "unit": "ms per call", "cores": cores, "kind": "port",
            "sample": (f"one full call ({x.shape[0]} token(s), NF4 {N}x{K}, r {A.shape[0]}): "
                       f"numpy fp32 dequantisation + forward, median of {reps}, {_cpu_model()}")}


# ------------------------------------------------------------- our arm -----

def headline_config(world):
    """The `config` dict of the headline workload (both arms print it)."""
    return {**WORKLOAD, "parallelism": f"dp{world} (token shards, LoRA-grad all-reduce)",
            "l2": "inputs > L2 (~290 MB resident per GPU), no flush"}


def exchange_check(peer, layer, flat_grads, dev, world):
    """Outside the timed region: the peer kernel's average of the LoRA
    gradients against an NCCL all-reduce of the same buffer, whether every
    rank holds the same averaged gradient bits, and whether one AdamW step
    from them leaves A and B bitwise identical on every rank."""
    import torch
    import torch.distributed as dist

    from metallora_b200 import kernels as K
    from metallora_b200.distributed import replicas_in_sync
    torch.cuda.synchronize()
    if peer is not None:
        src = peer.buffer.clone()   # this step's dA/dB as written by the backward
        got = flat_grads.clone()    # the peer kernel's average of them
    else:
        src = flat_grads.clone()
        got = None
    ref = src.clone()
    dist.all_reduce(ref, op=dist.ReduceOp.SUM)
    ref.mul_(1.0 / world)
    out = {"exchange": "peer" if peer is not None else "nccl",
           "numel": int(src.numel())}
    if got is not None:
        diff = (got - ref).abs()
        scale = ref.abs().max().clamp_min(1e-30)
        out["bitwise_equal_nccl"] = bool(torch.equal(got, ref))
        out["max_rel_vs_nccl"] = float(diff.max() / scale)
        # fp32 sums of `world` terms in another order: a few ulps of the largest
        bound = 4 * world * 2.0 ** -24
        out["rel_bound"] = bound
        ok = out["max_rel_vs_nccl"] <= bound
    else:
        got = ref
        ok = True
    out["grads_in_sync"] = replicas_in_sync(got)
    # one AdamW step of A and B from the averaged gradient, then the replicas
    n_a = layer.A.numel()
    ab = torch.cat([layer.A.detach().reshape(-1).float(), layer.B.detach().reshape(-1).float()])
    g = got.clone()
    m, v = torch.zeros_like(ab), torch.zeros_like(ab)
    st = K.persistent_gpu_state_init(device=dev)
    K.persistent_gpu_state_step(st)
    K.lora_adamw_step_metal(ab, g, m, v, st, 1e-3, 0.9, 0.999, 1e-8, 0.01)
    out["params_in_sync_after_adamw"] = (replicas_in_sync(ab[:n_a]) and
                                         replicas_in_sync(ab[n_a:]))
    out["ok"] = bool(ok and out["grads_in_sync"] and out["params_in_sync_after_adamw"])
    return out


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from metallora_b200 import _lib, kernels
    from metallora_b200.distributed import bind_to_device
    from metallora_b200.layers import LoRALinear

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if not kernels.is_metal_available():
        raise SystemExit("metallora_b200 CUDA extension unavailable on this device")
    # this rank's host cores (and so its pinned buffers) on the GPU's NUMA node
    affinity_before = bind_to_device(dev)
    host_cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else None
    M = WORKLOAD["tokens_per_gpu"]
    K, N, r, alpha = (WORKLOAD[k] for k in ("in_features", "out_features", "rank", "alpha"))
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    layer = LoRALinear(K, N, rank=r, alpha=alpha, device=dev, dtype=torch.bfloat16)
    with torch.no_grad():
        layer.W0.copy_(torch.randn(N, K, device=dev, generator=g) / 64)
        # A and B are replicated parameters: the same on every rank
        ga = torch.Generator(device=dev).manual_seed(4321)
        layer.A.copy_((torch.rand(r, K, device=dev, generator=ga) * 2 - 1) / 64)
        layer.B.copy_(torch.randn(N, r, device=dev, generator=ga) * 0.02 ** 0.5)
    x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16).requires_grad_(True)
    dy = torch.randn(M, N, device=dev, generator=g).to(torch.bfloat16)
    flat_grads = None
    # N > 1: the LoRA gradients go straight into a symmetric buffer and are
    # averaged by one kernel over NVLink peer memory (NCCL where that is
    # unavailable)
    from metallora_b200.distributed import PeerAllReduce
    n_a, n_b = layer.A.numel(), layer.B.numel()
    peer = PeerAllReduce.create(n_a + n_b, device=dev) if world > 1 else None
    side = torch.cuda.Stream(device=dev) if peer is not None else None
    grads_ready = torch.cuda.Event() if peer is not None else None
    exchanged = torch.cuda.Event() if peer is not None else None

    def start_exchange():
        # dA/dB are enqueued and the dx GEMM is not yet: the exchange kernel
        # runs on a side stream beside that GEMM (its CTAs hold no shared
        # memory; block 0 alone polls the peers' flags, the rest back off)
        grads_ready.record(torch.cuda.current_stream())
        side.wait_event(grads_ready)
        with torch.cuda.stream(side):
            peer.allreduce(flat_grads)
        exchanged.record(side)

    if peer is not None:
        flat_grads = torch.empty(n_a + n_b, dtype=torch.float32, device=dev)
        # written over (not added to) every step: no zeroing between steps
        sink = (peer.buffer[:n_a].view(layer.A.shape), peer.buffer[n_a:].view(layer.B.shape),
                False)
        layer._grad_sink = sink + ((start_exchange,) if args.exchange_overlap else ())
    exchange_kind = "peer" if peer is not None else ("nccl" if world > 1 else "none")

    def step(xin, dyin):
        nonlocal flat_grads
        layer.A.grad = None
        layer.B.grad = None
        xin.grad = None
        y = layer(xin)
        y.backward(dyin)
        if peer is not None and args.exchange_overlap:
            # the next step's weight gradients overwrite the exchanged buffer
            torch.cuda.current_stream().wait_event(exchanged)
        elif peer is not None:
            peer.allreduce(flat_grads)
        elif world > 1:
            flat = torch.cat([layer.A.grad.reshape(-1), layer.B.grad.reshape(-1)]).float()
            dist.all_reduce(flat)
            flat_grads = flat
        return y

    # one clock sampler for the whole run; each measurement reads its window
    sampler = ClockSampler(local_rank if "CUDA_VISIBLE_DEVICES" not in os.environ else
                           int(os.environ["CUDA_VISIBLE_DEVICES"].split(",")[local_rank]))
    sampler.start()
    time.sleep(0.3)
    for _ in range(args.warmup):
        step(x, dy)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()

    def timed(profiled):
        """K steps between two events on the launching stream (barrier and
        synchronize on both sides), max over ranks.  ``profiled`` brackets
        every launch of the library with its own pair of events as well."""
        _lib.profile_read(reset=True)
        _lib.profile_enable(profiled)
        n0 = _lib.launch_count()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        w0 = time.time()
        ev0.record(stream)
        for _ in range(args.steps):
            step(x, dy)
        ev1.record(stream)
        torch.cuda.synchronize()
        w1 = time.time()
        if world > 1:
            dist.barrier()
        n = _lib.launch_count() - n0
        _lib.profile_enable(False)
        prof = _lib.profile_read(reset=True)
        ms = ev0.elapsed_time(ev1)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms, n, prof, w0, w1

    # the headline loop runs without per-launch events (they add ~20 us per
    # step); the same K steps then run again with them for the kernel breakdown
    ms, launches, _, t_wall0, t_wall1 = timed(False)
    ms_prof, _, prof, _, t_wall2 = timed(True)
    ms_per_step = ms / args.steps
    value = world * M * args.steps / (ms / 1e3)
    clocks = sampler.summary(t_wall0, t_wall2)

    # roofline: the dominant kernel is the tcgen05 GEMM (forward y and backward dx)
    peaks = load_peaks()
    gemm_ms, gemm_n = prof["gemm"]
    gemm_flops = 2.0 * M * N * (K + r)  # per launch: X.W^T (+ rank block); fwd and dx alike
    achieved = gemm_flops / (gemm_ms / gemm_n / 1e3) / 1e12 if gemm_n else None
    peak, peak_name, peak_why = pick_peak(peaks, clocks)
    traffic, traffic_src = profile_traffic(GEMM_PROFILE)
    breakdown = {k: {"ms_per_launch": round(v[0] / v[1], 4), "launches": v[1]}
                 for k, v in prof.items() if v[1]}
    nongemm = ms_prof / args.steps - gemm_ms / args.steps

    grad_check = exchange_check(peer, layer, flat_grads, dev, world) if world > 1 else None

    # end-to-end through the public API with host buffers (pinned), overlapped.
    # run_e2e averages the gradients itself, once per step on the compute
    # stream: the side-stream exchange hook comes off first, so that only one
    # exchange kernel (they wait on one another's flags) is ever in flight
    if peer is not None:
        layer._grad_sink = sink
    e2e = run_e2e(args, layer, M, K, N, dev, world, peer)
    e2e_all = run_e2e(args, layer, M, K, N, dev, world, peer, outputs="all")

    total_tflops = world * flops_per_token(K, N, r) * M * args.steps / (ms / 1e3) / 1e12
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) activations/grads, N(0,1/4096) base, U(+-1/64) A, "
                "N(0,0.02) B)",
        "config": headline_config(world),
        "grad_exchange": exchange_kind + (" (beside the dx GEMM, side stream)"
                                          if peer is not None and args.exchange_overlap else ""),
        "host_cores_per_rank": host_cores,
        "tflops": round(total_tflops, 1),
        "step_frac_of_peak": round(total_tflops / world / peak, 4),
        "roofline": {"bound": "tensor", "kernel": "lora_gemm_pair_kernel (tcgen05 cta_group::2)",
                     "achieved": round(achieved, 1) if achieved else None,
                     "peak": peak, "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 4) if achieved else None,
                     "peak_source": peak_name, "peak_why": peak_why,
                     "frac_of_burst": round(achieved / peaks["bf16_tflops"], 4) if achieved else None,
                     "frac_of_sustained": (round(achieved / peaks["bf16_tflops_sustained"], 4)
                                           if achieved else None),
                     "traffic": traffic, "traffic_unit": "bytes per launch",
                     "traffic_source": traffic_src,
                     "algorithmic_bytes": GEMM_ALGORITHMIC_BYTES,
                     "per_launch_gflop": round(gemm_flops / 1e9, 2),
                     "kernel_timing": f"per-launch events over a second pass of the {args.steps} "
                                      f"steps ({ms_prof / args.steps:.4f} ms/step with events)"},
        "kernels": breakdown,
        "non_gemm_ms_per_step": round(nongemm, 4),
        "gpu_launches": launches,
        "clocks": clocks,
        "e2e": e2e,
        "e2e_all_outputs": {k: e2e_all[k] for k in ("value", "unit", "h2d_bytes_per_step",
                                                    "d2h_bytes_per_step", "ms_per_step",
                                                    "returned")},
    }
    if grad_check is not None:
        line["grad_exchange_check"] = grad_check
    # free the headline tensors before the other configurations
    del x, dy, layer, flat_grads
    torch.cuda.empty_cache()
    if args.workloads == "all":
        line["workloads"] = run_workloads(args, rank, world, local_rank, sampler)
    sampler.stop()
    if rank == 0:
        if world == 1:  # the host baseline is taken at N=1 only, on every host core
            if affinity_before:
                os.sched_setaffinity(0, affinity_before)
            line["cpu_baseline"] = cpu_baseline(args.cpu_tokens, args.cpu_reps)
        print(json.dumps(line), flush=True)


def run_e2e(args, layer, M, K, N, dev, world, peer=None, outputs="api"):
    """Same step through the public API with host-resident inputs and results:
    per step, H2D of x and dy from pinned memory and D2H of the results.
    ``outputs="api"`` returns what the reference's public calls return: y
    (``lora_forward``, ops.py:32-103) and the LoRA gradients dA, dB
    (``lora_backward``, ops.py:117-155; at N > 1 their average over the ranks,
    by the same peer exchange as the device-resident leg).  dx is computed in
    every step and stays on the device, where a preceding layer's backward
    reads it.  ``outputs="all"`` also returns dx.  The two directions run on
    their own streams (PCIe is full duplex), the next step's inputs load while
    this step computes."""
    import torch
    import torch.distributed as dist

    steps = max(3, min(args.steps, 50))
    g = torch.Generator().manual_seed(99)
    xh = [torch.randn(M, K, generator=g).to(torch.bfloat16).pin_memory() for _ in range(2)]
    dyh = [torch.randn(M, N, generator=g).to(torch.bfloat16).pin_memory() for _ in range(2)]
    n_a, n_b = layer.A.numel(), layer.B.numel()
    if world > 1:
        grad_shapes = (("grads", (n_a + n_b,), torch.float32),)
    else:
        grad_shapes = (("dA", tuple(layer.A.shape), layer.A.dtype),
                       ("dB", tuple(layer.B.shape), layer.B.dtype))
    want_dx = outputs == "all"
    outs = {k: [torch.empty(s, dtype=dt).pin_memory() for _ in range(2)]
            for k, s, dt in (("y", (M, N), torch.bfloat16),
                             *((("dx", (M, K), torch.bfloat16),) if want_dx else ()),
                             *grad_shapes)}
    xd = [torch.empty(M, K, device=dev, dtype=torch.bfloat16) for _ in range(2)]
    dyd = [torch.empty(M, N, device=dev, dtype=torch.bfloat16) for _ in range(2)]
    avg = [torch.empty(n_a + n_b, dtype=torch.float32, device=dev) for _ in range(2)]
    comp = torch.cuda.current_stream()
    copy = torch.cuda.Stream(device=dev)   # host -> device
    drain = torch.cuda.Stream(device=dev)  # device -> host
    h2d = 2 * M * K + 2 * M * N
    d2h = 2 * M * N + (2 * M * K if want_dx else 0) + sum(
        int(np.prod(s)) * torch.empty(0, dtype=dt).element_size() for _, s, dt in grad_shapes)
    loaded = [torch.cuda.Event() for _ in range(2)]
    done = [torch.cuda.Event() for _ in range(2)]
    drained = [torch.cuda.Event() for _ in range(2)]
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    chunks = max(1, args.e2e_chunks)
    rows = [(M * c // chunks, M * (c + 1) // chunks) for c in range(chunks)]

    def load(i):
        b = i % 2
        with torch.cuda.stream(copy):
            if i >= 2:  # buffer b was the input of step i - 2
                copy.wait_event(done[b])
            for r0, r1 in rows:  # in row chunks, interleaved with the other direction
                xd[b][r0:r1].copy_(xh[b][r0:r1], non_blocking=True)
                dyd[b][r0:r1].copy_(dyh[b][r0:r1], non_blocking=True)
            loaded[b].record(copy)

    def run(n):
        """n pipelined steps between two events on the compute stream."""
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ev0.record(comp)
        load(0)
        for i in range(n):
            b = i % 2
            if i + 1 < n:
                load(i + 1)
            comp.wait_event(loaded[b])
            xin = xd[b].requires_grad_(True)
            layer.A.grad = None
            layer.B.grad = None
            y = layer(xin)
            y.backward(dyd[b])
            if world > 1:
                if i >= 2:  # avg[b] was drained to the host by step i - 2's copy
                    comp.wait_event(drained[b])
                if peer is not None:
                    peer.allreduce(avg[b])
                else:
                    flat = torch.cat([layer.A.grad.reshape(-1), layer.B.grad.reshape(-1)]).float()
                    dist.all_reduce(flat)
                    avg[b].copy_(flat.mul_(1.0 / world))
                grads = ((outs["grads"][b], avg[b]),)
            else:
                grads = ((outs["dA"][b], layer.A.grad), (outs["dB"][b], layer.B.grad))
            done[b].record(comp)
            dx = xin.grad
            with torch.cuda.stream(drain):
                drain.wait_event(done[b])
                for t in (y, dx, *(src for _, src in grads)):
                    t.record_stream(drain)
                for r0, r1 in rows:
                    outs["y"][b][r0:r1].copy_(y.detach()[r0:r1], non_blocking=True)
                    if want_dx:
                        outs["dx"][b][r0:r1].copy_(dx[r0:r1], non_blocking=True)
                for dst, src in grads:
                    dst.copy_(src, non_blocking=True)
                drained[b].record(drain)
            xin.grad = None
            xd[b].requires_grad_(False)
        comp.wait_stream(copy)
        comp.wait_stream(drain)
        ev1.record(comp)
        torch.cuda.synchronize()
        return ev0.elapsed_time(ev1)

    # untimed warm-up steps through the same buffers (first transfers from
    # freshly pinned pages and the first autograd passes), then the timed ones
    run(max(3, args.warmup))
    ms = run(steps)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return {"value": round(world * M * steps / (ms / 1e3), 1), "unit": "tokens/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": steps,
            "ms_per_step": round(ms / steps, 4),
            "copy_chunks": chunks,
            "returned": ("y, dA, dB (what lora_forward and lora_backward return); dx computed "
                         "on the device and left there" if not want_dx else "y, dx, dA, dB"),
            "path": "LoRALinear forward+backward, pinned host buffers, H2D and D2H on their "
                    "own streams overlapped with compute" +
                    (("; LoRA gradients averaged by the " +
                      ("NVLink peer exchange" if peer is not None else "NCCL all-reduce"))
                     if world > 1 else "")}


# ------------------------------------------------------------ stack (cfg4) --

STACK = {"workload": "llama7b_proj_stack_nf4_train_step", "layers": 32, "hidden": 4096,
         "intermediate": 11008, "rank": 16, "alpha": 32.0, "tokens": 32768, "quant": "nf4",
         "group": 64}


def stack_flops_per_token():
    h, i, r, L = STACK["hidden"], STACK["intermediate"], STACK["rank"], STACK["layers"]

    def lin(K, N):
        return flops_per_token(K, N, r)
    return L * (4 * lin(h, h) + 2 * lin(h, i) + lin(i, h))


def build_stack(dev, seed=0):
    import torch
    from torch import nn

    from metallora_b200.layers import LoRALinear
    h, i, r, a = STACK["hidden"], STACK["intermediate"], STACK["rank"], STACK["alpha"]
    g = torch.Generator(device=dev).manual_seed(seed)

    def proj(K, N):
        lin = LoRALinear(K, N, rank=r, alpha=a, device=dev, dtype=torch.bfloat16)
        with torch.no_grad():
            lin.W0.copy_(torch.randn(N, K, device=dev, generator=g) / K ** 0.5)
            lin.B.copy_(torch.randn(N, r, device=dev, generator=g) * 0.02 ** 0.5)
        return lin.quantize_base(STACK["quant"], STACK["group"])

    class Layer(nn.Module):
        def __init__(self):
            super().__init__()
            self.q_proj, self.k_proj, self.v_proj, self.o_proj = (proj(h, h) for _ in range(4))
            self.gate_proj, self.up_proj = proj(h, i), proj(h, i)
            self.down_proj = proj(i, h)

        def forward(self, x):
            # Llama-style pre-norm (per-token RMS, no weight): gate*up is quadratic
            # in its input, so without it the residual stream overflows bf16
            # within a few layers
            n = nn.functional.rms_norm(x, (h,), eps=1e-6)
            a_ = (self.q_proj(n) + self.k_proj(n) + self.v_proj(n)) * (1.0 / 3 ** 0.5)
            x = x + self.o_proj(a_)
            n = nn.functional.rms_norm(x, (h,), eps=1e-6)
            return x + self.down_proj(self.gate_proj(n) * self.up_proj(n))

    class Stack(nn.Module):
        def __init__(self):
            super().__init__()
            self.layers = nn.ModuleList(Layer() for _ in range(STACK["layers"]))

        def forward(self, x):
            for layer in self.layers:
                x = layer(x)
            return x

    return Stack()


def stack_measure(args, rank, world, local_rank, steps, warmup, sampler=None, overlap=True):
    """One configuration of the 32-layer NF4 stack: ``warmup`` untimed and
    ``steps`` timed LoRATrainer steps (forward, backward, gradient average
    over the ranks, global-norm clip, AdamW) on this rank's token shard; time
    is the max over ranks.  ``overlap``: per-layer gradient buckets averaged on
    a side stream while the backward of earlier layers runs; otherwise one
    all-reduce of the flat buffer after the backward."""
    import torch
    import torch.distributed as dist

    from metallora_b200 import _lib
    from metallora_b200.distributed import shard_bounds
    from metallora_b200.trainer import LoRATrainer, TrainingConfig

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    model = build_stack(dev)
    cfg = TrainingConfig(rank=STACK["rank"], alpha=STACK["alpha"], learning_rate=1e-4,
                         output_dir="/tmp/mlora_bench_out", log_interval=10 ** 9,
                         save_interval=10 ** 9)
    tr = LoRATrainer(model, cfg, overlap_grad_exchange=overlap)
    b, e = shard_bounds(STACK["tokens"], rank, world)
    g = torch.Generator(device=dev).manual_seed(7 + rank)
    x = torch.randn(1, e - b, STACK["hidden"], device=dev, generator=g).to(torch.bfloat16)
    tgt = torch.randn(1, e - b, STACK["hidden"], device=dev, generator=g).to(torch.bfloat16)
    batch = {"input_ids": x, "target_output": tgt}
    for _ in range(warmup):
        tr._training_step(batch)
    torch.cuda.synchronize()
    own_sampler = sampler is None
    if own_sampler:
        sampler = ClockSampler(local_rank)
        sampler.start()
        time.sleep(0.3)
    _lib.profile_read(reset=True)
    _lib.profile_enable(True)
    launches0 = _lib.launch_count()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.time()
    ev0.record()
    losses = []
    for _ in range(steps):
        losses.append(tr._training_step(batch)["loss"])
    ev1.record()
    torch.cuda.synchronize()
    t1 = time.time()
    if world > 1:
        dist.barrier()
    launches = _lib.launch_count() - launches0
    _lib.profile_enable(False)
    prof = _lib.profile_read(reset=True)
    if own_sampler:
        sampler.stop()
    clocks = sampler.summary(t0, t1)
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    in_sync = None
    if world > 1:
        from metallora_b200.distributed import replicas_in_sync
        in_sync = replicas_in_sync(tr.params.master)
    tokens = STACK["tokens"] * steps
    value = tokens / (ms / 1e3)
    tflops = stack_flops_per_token() * value / 1e12
    peaks = load_peaks()
    peak, peak_name, peak_why = pick_peak(peaks, clocks)
    g_ms = prof["gemm"][0]
    kern_total = sum(v[0] for v in prof.values())
    out = {
        "metric": "LoRA projection-stack training step tokens/s (NF4 bases, bf16)",
        "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": steps,
        "warmup": warmup, "ms_per_step": round(ms / steps, 3), "higher_is_better": True,
        "scaling": "strong", "dtype": "bf16", "data": "synthetic",
        "config": {**STACK, "parallelism": f"dp{world} (token shards, LoRA-grad all-reduce)",
                   "grad_exchange": ("per-layer buckets on a side stream, overlapped with the "
                                     "backward" if overlap else "one flat all-reduce after the "
                                     "backward") if world > 1 else "none"},
        "tflops": round(tflops, 1),
        "roofline": {"bound": "tensor", "achieved": round(tflops / world, 1), "peak": peak,
                     "unit": "TFLOP/s", "frac": round(tflops / world / peak, 4),
                     "per": "GPU, whole step", "peak_source": peak_name, "peak_why": peak_why},
        "kernels_ms_per_step": {k: round(v[0] / steps, 2) for k, v in prof.items() if v[1]},
        "kernel_launches_per_step": {k: v[1] // steps for k, v in prof.items() if v[1]},
        "gemm_share_of_kernel_time": round(g_ms / max(1e-9, kern_total), 3),
        "kernel_ms_per_step": round(kern_total / steps, 2),
        "gpu_launches": launches, "loss_first_last": [losses[0], losses[-1]],
        "clocks": clocks,
        "mem_gb": round(torch.cuda.max_memory_allocated(dev) / 1e9, 1),
    }
    if in_sync is not None:
        out["replicas_in_sync"] = in_sync
    del tr, model, x, tgt, batch
    torch.cuda.empty_cache()
    return out


def run_stack(args, rank, world, local_rank):
    line = stack_measure(args, rank, world, local_rank, args.steps, args.warmup,
                         overlap=not args.no_overlap)
    line["vs_baseline"] = None
    if rank == 0:
        print(json.dumps(line), flush=True)


# ------------------------------------------------------ config sweeps ----

def graph_ms(fn, reps=20, inner=5):
    """Mean device time of one call replayed from a CUDA graph (launch overhead
    hidden).  ``fn`` is a callable, or a list of callables captured in turn
    (e.g. the same op on distinct weight copies, so that weights stream from
    HBM rather than L2)."""
    import torch
    fns = fn if isinstance(fn, (list, tuple)) else [fn]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            for f in fns:
                f()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(inner):
            for f in fns:
                f()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps / inner / len(fns)


L2_BYTES = 126 * 2 ** 20


def events_ms(fn, reps=20, warm=3):
    """Mean time of fn() between CUDA events (launch overhead included)."""
    import torch
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def sweep(kind, sampler=None, quick=False, tokens=None):
    """Measurements of one of the other configurations on cuda:0, one dict per
    case.  kind: "fp32" (fp32 forward 4096->4096 r16, 2048 tokens, and the
    merged weight), "nf4" (NF4 11008x4096 block 64, r64, forward and backward
    at 1/16/512/4096 tokens), "int" (INT4/INT8 group 128, 4096->4096 and
    4096->14336, r16, forward unmerged and merged), "multi" (per-sample
    adapters).  ``quick`` keeps the cases the default bench line reports
    (tokens 1 and 4096 for INT, no lean-path comparison)."""
    import torch

    from metallora_b200 import _lib
    from metallora_b200 import kernels as K
    from metallora_b200 import quant
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peaks = load_peaks()
    gen = torch.Generator(device=dev).manual_seed(0)
    out = []

    def window(t0):
        return sampler.summary(t0, time.time()) if sampler is not None else {}

    def tensor_roofline(flops, ms, clocks):
        peak, name, _ = pick_peak(peaks, clocks)
        ach = flops / ms / 1e9
        return {"bound": "tensor", "achieved": round(ach, 1), "peak": peak, "unit": "TFLOP/s",
                "frac": round(ach / peak, 4), "peak_source": name}

    def hbm_roofline(nbytes, ms):
        ach = nbytes / ms / 1e6
        return {"bound": "hbm", "achieved": round(ach, 1), "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": round(ach / peaks["hbm_gbs"], 4),
                "peak_source": f"{peaks['source']} hbm_gbs", "weights": "HBM-cold (rotated copies)"}

    def lora_bytes(qw, W, A, B, M, Kd, N):
        wb = qw.nbytes() if qw is not None else W.numel() * 2
        return wb + (A.numel() + B.numel()) * 2 + 2 * M * (Kd + N)

    if kind == "fp32":
        t0 = time.time()
        M, Kd, N, r = 2048, 4096, 4096, 16
        x = torch.randn(M, Kd, device=dev, generator=gen)
        W = torch.randn(N, Kd, device=dev, generator=gen) / 64
        A = (torch.rand(r, Kd, device=dev, generator=gen) * 2 - 1) / 64
        B = torch.randn(N, r, device=dev, generator=gen) * 0.02 ** 0.5
        t = graph_ms(lambda: K.lora_linear_fwd(x, W, A, B, 32.0))
        Wm = K.merge(W, A, B, 32.0)
        tm = graph_ms(lambda: K.linear(x, Wm))
        y, _ = K.lora_linear_fwd(x, W, A, B, 32.0)
        ym = K.linear(x, Wm)
        ref = x.double() @ W.double().t() + 2.0 * (x.double() @ A.double().t()) @ B.double().t()
        rel = float((y.double() - ref).norm() / ref.norm())
        relm = float((ym.double() - ref).norm() / ref.norm())
        fl = 2.0 * M * (Kd * N + Kd * r + r * N)
        clocks = window(t0)
        out.append({"workload": "fp32_fwd_4096x4096_r16_2048tok", "tokens": M, "ms": round(t, 4),
                    "tflops": round(fl / t / 1e9, 1), "merged_ms": round(tm, 4),
                    "rel_err_vs_fp64": rel, "merged_rel_err_vs_fp64": relm, "tolerance": 1e-4,
                    "tokens_per_s": round(M / t * 1e3, 1),
                    "roofline": {**tensor_roofline(fl, t, clocks),
                                 "note": "fp32 as 3 bf16 products (hi.hi, hi.lo, lo.hi): "
                                         "algorithmic fp32 FLOPs over the bf16 peak",
                                 "executed_bf16_frac": round(
                                     3 * fl / t / 1e9 / pick_peak(peaks, clocks)[0], 4),
                                 "executed_note": "the 3 bf16 products the tensor cores run "
                                                  "(3x the algorithmic FLOPs) over the same "
                                                  "peak; the hi/lo split passes of x and W0 "
                                                  "are inside the timed call"},
                    "clocks": clocks})
        return out
    if kind == "multi":
        # per-sample adapters (16 samples x 512 tokens, 4096 -> 4096, r 16)
        from metallora_b200.ops import multi_adapter_forward
        Kd, N, r, S, Bsz = 4096, 4096, 16, 512, 16
        x = torch.randn(Bsz, S, Kd, device=dev, generator=gen).to(torch.bfloat16)
        W = (torch.randn(N, Kd, device=dev, generator=gen) / 64).to(torch.bfloat16)
        for n in (1, 4, 16, 64):
            A = ((torch.rand(n, r, Kd, device=dev, generator=gen) * 2 - 1) / 64).to(torch.bfloat16)
            Bm = (torch.randn(n, N, r, device=dev, generator=gen) * 0.1).to(torch.bfloat16)
            ids = [b % n for b in range(Bsz)]
            # host-side grouping of the ids: timed with events, not a graph
            t = events_ms(lambda: multi_adapter_forward(x, W, A, Bm, ids, 32.0))
            fl = 2.0 * Bsz * S * (Kd * N + Kd * r + r * N)
            out.append({"workload": "multi_adapter_fwd_4096x4096_r16", "tokens": Bsz * S,
                        "adapters": n, "distinct_in_batch": min(n, Bsz), "ms": round(t, 4),
                        "tflops": round(fl / t / 1e9, 1)})
        t1 = events_ms(lambda: K.lora_linear_fwd(x.reshape(-1, Kd), W, A[0], Bm[0], 32.0))
        out.append({"workload": "single_adapter_fwd_4096x4096_r16", "tokens": Bsz * S,
                    "ms": round(t1, 4)})
        return out
    if kind == "nf4":
        cases = [("nf4", 64, 4096, 11008, 64, 128.0, M) for M in (1, 16, 512, 4096)
                 if tokens is None or M in tokens]
    else:
        toks = (1, 4096) if quick else (1, 16, 128, 512, 4096)
        cases = [(s, 128, 4096, N, 16, 32.0, M) for s in ("int4", "int8") for N in (4096, 14336)
                 for M in toks if tokens is None or M in tokens]
    for scheme, group, Kd, N, r, alpha, M in cases:
        t0 = time.time()
        W = (torch.randn(N, Kd, device=dev, generator=gen) / Kd ** 0.5).to(torch.bfloat16)
        qw = quant.quantize(W, scheme, group)
        A = ((torch.rand(r, Kd, device=dev, generator=gen) * 2 - 1) / Kd ** 0.5).to(torch.bfloat16)
        B = (torch.randn(N, r, device=dev, generator=gen) * 0.1).to(torch.bfloat16)
        x = torch.randn(M, Kd, device=dev, generator=gen).to(torch.bfloat16)
        dy = torch.randn(M, N, device=dev, generator=gen).to(torch.bfloat16)
        fl = 2.0 * M * (Kd * N + Kd * r + r * N)
        d = {"workload": f"{scheme}_g{group}_{Kd}x{N}_r{r}", "tokens": M}
        byts = lora_bytes(qw, W, A, B, M, Kd, N)
        if M <= 16:
            # decode: rotate over weight copies totalling > 1.5x L2 so every
            # call streams its weight from HBM
            copies = [qw] + [quant.quantize(W, scheme, group)
                             for _ in range(int(1.5 * L2_BYTES // byts))]
            tf = graph_ms([lambda c=c: K.qlora_linear_fwd(x, c, A, B, alpha) for c in copies],
                          reps=10, inner=2)
            d["weight_copies"] = len(copies)
            del copies
            if kind == "nf4" and M == 1:
                d["cpu_baseline"] = nf4_cpu_baseline(qw, x, A, B, alpha, group)
        else:
            tf = graph_ms(lambda: K.qlora_linear_fwd(x, qw, A, B, alpha))
        d.update({"fwd_ms": round(tf, 4), "fwd_tflops": round(fl / tf / 1e9, 1),
                  "fwd_gbs": round(byts / tf / 1e6, 1), "algorithmic_bytes": byts})
        if M > 16 and not quick:  # the fused in-loop-dequant kernel (lean workspace)
            import dataclasses
            ql = dataclasses.replace(qw, lean=True)
            d["lean_fwd_ms"] = round(graph_ms(lambda: K.qlora_linear_fwd(x, ql, A, B, alpha)), 4)
        if kind == "nf4":
            _, saved = K.qlora_linear_fwd(x, qw, A, B, alpha, save_xa=True)
            tb = graph_ms(lambda: K.qlora_linear_bwd(dy, x, qw, A, B, alpha, saved))
            flb = 2.0 * M * (N * Kd + 2 * N * r + 2 * r * Kd)
            d.update({"bwd_ms": round(tb, 4), "bwd_tflops": round(flb / tb / 1e9, 1),
                      "fwd_bwd_tflops": round((fl + flb) / (tf + tb) / 1e9, 1)})
            if M > 16:
                # where the call's time goes: the library's per-launch events by
                # kernel kind (eager calls, after the graph timings above)
                for tag, fn in (("fwd", lambda: K.qlora_linear_fwd(x, qw, A, B, alpha)),
                                ("bwd", lambda: K.qlora_linear_bwd(dy, x, qw, A, B, alpha,
                                                                   saved))):
                    reps = 5
                    fn()
                    torch.cuda.synchronize()
                    _lib.profile_read(reset=True)
                    _lib.profile_enable(True)
                    for _ in range(reps):
                        fn()
                    torch.cuda.synchronize()
                    _lib.profile_enable(False)
                    prof = _lib.profile_read(reset=True)
                    d[f"{tag}_kernels_ms"] = {k: round(v[0] / reps, 4) for k, v in prof.items()
                                              if v[1]}
                    d[f"{tag}_kernel_launches"] = {k: v[1] // reps for k, v in prof.items()
                                                   if v[1]}
        else:
            Wm = K.merge(quant.dequantize(qw, torch.bfloat16), A, B, alpha)
            if M <= 16:
                wms = [Wm] + [Wm.clone() for _ in range(int(1.5 * L2_BYTES // (Wm.numel() * 2)))]
                tm = graph_ms([lambda w=w: K.linear(x, w) for w in wms], reps=10, inner=2)
                del wms
            else:
                tm = graph_ms(lambda: K.linear(x, Wm))
            d.update({"merged_fwd_ms": round(tm, 4),
                      "merged_gbs": round((Wm.numel() * 2 + 2 * M * (Kd + N)) / tm / 1e6, 1)})
        clocks = window(t0)
        if M <= 16:
            d["fwd_roofline"] = hbm_roofline(byts, tf)
        else:
            d["fwd_roofline"] = tensor_roofline(fl, tf, clocks)
        if "bwd_ms" in d and M > 16:
            d["fwd_bwd_roofline"] = tensor_roofline(fl + flb, tf + tb, clocks)
        d["clocks"] = clocks
        out.append(d)
        del W, qw, A, B, x, dy
    torch.cuda.empty_cache()
    return out


def run_workloads(args, rank, world, local_rank, sampler):
    """The other configurations, measured after the headline: at N = 1 the
    fp32 forward (cfg0), NF4 (cfg2) and INT4/INT8 (cfg3) cases on cuda:0; at
    every N the 32-layer NF4 stack training step (cfg4, all ranks)."""
    out = {}

    def guarded(name, fn):
        try:
            out[name] = fn()
        except Exception as e:  # recorded in the line, not hidden
            out[name] = {"error": f"{type(e).__name__}: {e}"[:400]}

    if world == 1:
        guarded("cfg0_fp32", lambda: sweep("fp32", sampler)[0])
        guarded("cfg2_nf4", lambda: sweep("nf4", sampler, quick=True))
        guarded("cfg3_int", lambda: sweep("int", sampler, quick=True))
    guarded("cfg4_stack", lambda: stack_measure(args, rank, world, local_rank, steps=3, warmup=2,
                                                sampler=sampler))
    return out


def run_sweep(args):
    for d in sweep(args.workload, tokens=args.tokens):
        print(json.dumps(d), flush=True)


# -------------------------------------------------------- reference arm ----

def run_reference(args, rank):
    """The reference's CPU path on the host cores, on the headline workload
    itself (8192 tokens per step unless --ref-tokens says otherwise): inputs
    built once, then W untimed and K timed steps of the numpy restatement
    (forward, dx, dA, dB), every step on the same resident inputs (as our
    arm's `value` leg keeps its inputs in HBM).  Each step is timed on its
    own; `value` uses the median step."""
    if rank != 0:
        return
    from threadpoolctl import threadpool_limits
    tokens = args.ref_tokens
    world = int(os.environ.get("WORLD_SIZE", "1"))
    inp = _cpu_inputs(tokens)
    times = []
    with threadpool_limits(limits=len(os.sched_getaffinity(0)), user_api="blas"):
        for _ in range(args.warmup):
            _cpu_step(inp)
        for _ in range(args.steps):
            t = time.perf_counter()
            _cpu_step(inp)
            times.append(time.perf_counter() - t)
        cores = _blas_threads()
    med = statistics.median(times)
    value = tokens / med
    sample = (f"{tokens} tokens per step (the full per-GPU batch), median of {args.steps} timed "
              f"steps after {args.warmup} warm-up, fwd+dx+dA+dB (numpy fp32 on bf16-rounded "
              f"inputs built once, OpenBLAS, {_cpu_model()}, {cores} threads)")
    K, N, r = WORKLOAD["in_features"], WORKLOAD["out_features"], WORKLOAD["rank"]
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * med, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (same distributions as our arm)",
        "config": headline_config(world),
        "impl": "reference",
        "runs_on": "host CPU, rank 0 only",
        "step_seconds": {"median": round(med, 4), "min": round(min(times), 4),
                         "max": round(max(times), 4)},
        "tflops": round(flops_per_token(K, N, r) * value / 1e12, 4),
        "cpu_baseline": {"value": round(value, 1), "unit": "tokens/s", "cores": cores,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 1), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "MLX (the reference's CPU backend) cannot be installed here; its pure-MLX op "
                "sequence (ops.py:91-94,144-155) is timed as the numpy restatement",
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["lora", "stack", "nf4", "int", "fp32", "multi"],
                    default="lora")
    ap.add_argument("--tokens", type=int, nargs="+", default=None,
                    help="--workload nf4 / int: only these token counts")
    ap.add_argument("--cpu-tokens", type=int, default=2048)
    ap.add_argument("--cpu-reps", type=int, default=3)
    ap.add_argument("--ref-tokens", type=int, default=WORKLOAD["tokens_per_gpu"])
    ap.add_argument("--workloads", choices=["all", "none"], default="all",
                    help="after the headline, also measure the other configurations "
                         "(fp32, NF4, INT4/INT8 at N=1; the NF4 stack at every N)")
    ap.add_argument("--no-overlap", action="store_true",
                    help="--workload stack: one flat all-reduce after the backward")
    ap.add_argument("--e2e-chunks", type=int, default=1,
                    help="e2e leg: host<->device copies in this many row chunks per tensor")
    ap.add_argument("--exchange-after", dest="exchange_overlap", action="store_false",
                    help="headline at N > 1: run the peer gradient exchange after the "
                         "backward instead of beside the dx GEMM")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.workload == "stack":
            run_stack(args, rank, world, local_rank)
        elif args.workload in ("nf4", "int", "fp32", "multi"):
            if rank == 0:
                run_sweep(args)
        else:
            run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
