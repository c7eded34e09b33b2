"""GPU tests of the optimizer kernels and the LoRA trainer step against the
oracle (AdamW: kernels.py:314-344 operation order, bit-exact in fp32; clip:
trainer.py:237-240)."""
import numpy as np
import pytest
import torch
from torch import nn

from oracle import lora_oracle as lo
from tests.conftest import rel_err

pytestmark = pytest.mark.gpu


def test_adamw_kernel_bit_exact(cuda):
    from metallora_b200 import kernels as K
    rng = np.random.default_rng(0)
    n = 100_003
    p, g = rng.standard_normal(n).astype(np.float32), rng.standard_normal(n).astype(np.float32)
    m = (rng.standard_normal(n) * 0.1).astype(np.float32)
    v = np.abs(rng.standard_normal(n) * 0.01).astype(np.float32)
    state = K.persistent_gpu_state_init(0.9, 0.999, cuda)
    tp, tg, tm, tv = (torch.from_numpy(a.copy()).to(cuda) for a in (p, g, m, v))
    for step in (1, 2, 3):
        K.persistent_gpu_state_step(state, 0.9, 0.999)
        K.lora_adamw_step_metal(tp, tg, tm, tv, state, 1e-3, 0.9, 0.999, 1e-8, 0.01)
        # oracle uses the device's beta powers (successive fp32 products)
        st = state.cpu().numpy()
        assert st[0] == step
        p, m, v = lo.adamw_step(p, g, m, v, 1e-3, 0.9, 0.999, 1e-8, 0.01, step, b1t=st[1],
                                b2t=st[2])
        np.testing.assert_array_equal(tm.cpu().numpy(), m)
        np.testing.assert_array_equal(tv.cpu().numpy(), v)
        np.testing.assert_array_equal(tp.cpu().numpy(), p)
        assert torch.count_nonzero(tg) == 0  # the kernel consumes and zeroes the gradient
        tg.copy_(torch.from_numpy(g))


def test_adamw_step1_matches_reference_golden(cuda, golden):
    """Against the reference kernel's own output at step 1 (tests/golden)."""
    from metallora_b200 import kernels as K
    gd = golden("lora_fp32.npz")
    t = {k: torch.from_numpy(gd[k].copy()).to(cuda)
         for k in ("adam_param", "adam_grad", "adam_m", "adam_v", "adam_state")}
    K.lora_adamw_step_metal(t["adam_param"], t["adam_grad"], t["adam_m"], t["adam_v"],
                            t["adam_state"], 1e-3, 0.9, 0.999, 1e-8, 0.01)
    np.testing.assert_array_equal(t["adam_param"].cpu().numpy(), gd["adam_param_out"])
    np.testing.assert_array_equal(t["adam_m"].cpu().numpy(), gd["adam_m_out"])
    np.testing.assert_array_equal(t["adam_v"].cpu().numpy(), gd["adam_v_out"])


def test_grad_norm_clip(cuda):
    from metallora_b200 import kernels as K
    g = torch.randn(1_000_001, device=cuda) * 0.01
    out = K.grad_norm_clip(g, 1.0)
    norm = float(g.double().norm())
    assert abs(float(out[1]) - norm) / norm < 1e-5
    assert abs(float(out[0]) - min(1.0, 1.0 / (norm + 1e-6))) < 1e-6
    out2 = K.grad_norm_clip(g, 0.5)
    assert abs(float(out2[0]) - 0.5 / (norm + 1e-6)) < 1e-6
    assert torch.equal(K.grad_norm_clip(g, 0.5), out2)  # deterministic


class TwoProj(nn.Module):
    def __init__(self, dev, dtype):
        super().__init__()
        self.q_proj = nn.Linear(256, 512, bias=False, device=dev, dtype=dtype)
        self.v_proj = nn.Linear(512, 256, bias=False, device=dev, dtype=dtype)

    def forward(self, x):
        return self.v_proj(self.q_proj(x))


def _model(dev, dtype=torch.bfloat16, seed=0):
    torch.manual_seed(seed)
    m = TwoProj(dev, dtype)
    with torch.no_grad():
        for lin in (m.q_proj, m.v_proj):
            lin.weight.normal_(0, lin.weight.shape[1] ** -0.5)
    return m


def _bf16(a):
    """fp64 -> bf16 (round to nearest even) -> fp64, as torch rounds."""
    t = torch.from_numpy(np.asarray(a, np.float64).astype(np.float32)).to(torch.bfloat16)
    return t.float().numpy().astype(np.float64)


def test_trainer_gradients_and_step_match_oracle(cuda):
    from metallora_b200.layers import LoRALinear
    from metallora_b200.trainer import LoRATrainer, TrainingConfig
    model = _model(cuda)
    cfg = TrainingConfig(rank=16, alpha=32.0, learning_rate=1e-3, max_grad_norm=0.05,
                         output_dir="/tmp/mlora_test_out")
    tr = LoRATrainer(model, cfg)
    with torch.no_grad():
        for mod in model.modules():
            if isinstance(mod, LoRALinear):
                mod.B.normal_(0, 0.1)  # the fp32 master views
    tr.params.refresh_compute()
    x = torch.randn(4, 64, 256, device=cuda, dtype=torch.bfloat16)
    tgt = torch.randn(4, 64, 256, device=cuda, dtype=torch.bfloat16)
    loss = tr.backward({"input_ids": x, "target_output": tgt})
    torch.cuda.synchronize()
    # oracle gradients through the two-layer chain, on the bf16 values the GPU used
    f = lambda t: t.detach().float().cpu().numpy().astype(np.float64)  # noqa: E731
    q, v = model.q_proj, model.v_proj
    Aq, Bq, Av, Bv = (f(t) for t in (q._compute_ab[0], q._compute_ab[1], v._compute_ab[0],
                                     v._compute_ab[1]))
    X = f(x).reshape(-1, 256)
    # every tensor the GPU path stores in bf16 between the two layers is
    # rounded to bf16 here too: the hidden state, the output, its gradient
    # (autograd hands the bf16 output a bf16 gradient) and the hidden state's
    # gradient
    H = _bf16(lo.lora_forward(X, f(q.W0), Aq, Bq, 32.0, np.float64))
    Y = _bf16(lo.lora_forward(H, f(v.W0), Av, Bv, 32.0, np.float64))
    T = f(tgt).reshape(-1, 256)
    assert abs(float(loss) - np.mean((Y - T) ** 2)) / np.mean((Y - T) ** 2) < 2e-2
    dY = _bf16(2 * (Y - T) / Y.size)
    gAv, gBv = lo.lora_backward(dY, H, Av, Bv, 32.0, None, np.float64)
    dH = _bf16(lo.lora_grad_x(dY, f(v.W0), Av, Bv, 32.0, np.float64))
    gAq, gBq = lo.lora_backward(dH, X, Aq, Bq, 32.0, None, np.float64)
    got = {k: t.cpu().numpy() for k, t in tr.params.named_tensors().items()}  # masters (before)
    grads = {n: tr.params.grad[o:o + c].view(s).cpu().numpy()
             for n, (o, c, s) in tr.params.slices.items()}
    for name, ref in (("q_proj.A", gAq), ("q_proj.B", gBq), ("v_proj.A", gAv),
                      ("v_proj.B", gBv)):
        assert rel_err(grads[name], ref) < 2e-2, name  # the bf16 tolerance
    # optimizer step = clip + AdamW on the device gradient, vs the oracle
    flat_g = tr.params.grad.cpu().numpy().copy()
    flat_p = tr.params.master.cpu().numpy().copy()
    tr.optimizer_step()
    torch.cuda.synchronize()
    (scaled,), norm = lo.clip_grad_norm([flat_g], 0.05)
    p_ref, _, _ = lo.adamw_step(flat_p, scaled, np.zeros_like(flat_p), np.zeros_like(flat_p),
                                1e-3, 0.9, 0.999, 1e-8, 0.01, 1)
    np.testing.assert_allclose(tr.params.master.cpu().numpy(), p_ref, rtol=1e-5, atol=1e-6)
    assert torch.count_nonzero(tr.params.grad) == 0
    assert got  # masters were readable


def test_trainer_fits_and_resumes(cuda, tmp_path):
    from metallora_b200.layers import LoRALinear
    from metallora_b200.trainer import LoRATrainer, TrainingConfig
    teacher = _model(cuda, seed=1)
    student = _model(cuda, seed=1)
    torch.manual_seed(5)
    with torch.no_grad():  # a rank-8 change the rank-16 adapter can represent exactly
        u = torch.randn(512, 8, device=cuda) * 0.1
        w = torch.randn(8, 256, device=cuda) * 0.1
        teacher.q_proj.weight.add_((u @ w).to(teacher.q_proj.weight.dtype))
    data = [torch.randn(8, 32, 256, device=cuda, dtype=torch.bfloat16) for _ in range(4)]
    cfg = TrainingConfig(rank=16, alpha=32.0, learning_rate=3e-3, log_interval=1000,
                         save_interval=1000, output_dir=str(tmp_path))
    tr = LoRATrainer(student, cfg)
    with torch.no_grad():
        targets = [teacher(x) for x in data]
    losses = []
    for epoch in range(30):
        for x, t in zip(data, targets):
            losses.append(tr._training_step({"input_ids": x, "target_output": t})["loss"])
    assert np.mean(losses[-4:]) < 0.3 * np.mean(losses[:4])
    tr.save(tmp_path / "ck")
    before = tr.params.master.clone()
    other = LoRATrainer(_model(cuda, seed=1), cfg)
    other.load(tmp_path / "ck")
    assert torch.equal(other.params.master, before)
    assert torch.equal(other.optimizer.m, tr.optimizer.m)
    assert sum(isinstance(m, LoRALinear) for m in other.model.modules()) == 2
