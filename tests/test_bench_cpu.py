"""bench.py's contract on the CPU: the reference arm prints one JSON line with
the keys the driver reads, its value counts only the timed steps (inputs are
built before), and our arm and smoke() fail loudly without a GPU instead of
falling back to the CPU."""
import json
import subprocess
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]


def _run(*args, timeout=300):
    return subprocess.run([sys.executable, "bench.py", *args], cwd=ROOT, capture_output=True,
                          text=True, timeout=timeout)


def test_reference_arm_json_line():
    p = _run("--impl", "reference", "--steps", "2", "--warmup", "3", "--ref-tokens", "64")
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "tokens/s" and d["higher_is_better"]
    assert d["steps"] == 2 and d["warmup"] == 3 and d["n_gpus"] == 1
    assert d["value"] > 0
    # value counts the timed steps only: tokens * steps / (steps * ms_per_step)
    assert abs(d["value"] - 64 * 1e3 / d["ms_per_step"]) / d["value"] < 0.01
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert "64 tokens per step" in cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    assert d["config"]["workload"] == "lora_linear_fwd_bwd_bf16"


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the behaviour without a GPU")
def test_our_arm_and_smoke_fail_without_gpu():
    p = _run("--steps", "1", "--warmup", "3", timeout=300)
    assert p.returncode != 0
    assert not any(ln.startswith("{") for ln in p.stdout.splitlines())
    sys.path.insert(0, str(ROOT))
    import __graft_entry__
    with pytest.raises(Exception):
        __graft_entry__.smoke()


def test_nf4_cpu_baseline_shape():
    """The NF4 decode row's CPU baseline times the oracle's restatement of the
    reference's NF4 forward on the given weight and reports the fields the
    bench line carries."""
    import types

    import numpy as np
    sys.path.insert(0, str(ROOT))
    import bench
    from oracle import quant_oracle as qo
    rng = np.random.default_rng(0)
    N, K, r = 96, 256, 8
    codes, absmax = qo.quantize_nf4((rng.standard_normal((N, K)) / 16).astype(np.float32), 64)[:2]
    qw = types.SimpleNamespace(codes=torch.from_numpy(codes), scales=torch.from_numpy(absmax),
                               shape=(N, K))
    x = torch.randn(1, K).to(torch.bfloat16)
    A = (torch.rand(r, K) / 16).to(torch.bfloat16)
    B = (torch.randn(N, r) * 0.1).to(torch.bfloat16)
    cb = bench.nf4_cpu_baseline(qw, x, A, B, 16.0, 64, reps=2)
    assert cb["kind"] == "port" and cb["unit"] == "ms per call"
    assert cb["value"] > 0 and cb["cores"] >= 1
    assert f"NF4 {N}x{K}" in cb["sample"] and f"r {r}" in cb["sample"]
