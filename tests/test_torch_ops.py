"""The custom operators ``torch.ops.metal_lora.*`` (``metallora_b200.torch_ops``).

CPU: registration, shape inference through the fake implementations (an FX
trace of a forward + backward needs no GPU), shape errors, and that real
calls on CPU tensors raise DeviceError (no CPU fallback).
GPU: the operators give bitwise the results of the module path
(``ops.lora_forward`` with autograd, ``kernels.merge``/``linear``) and agree
with a torch fp32 reference; ``torch.library.opcheck`` checks schema,
autograd registration and fake-tensor metadata against the real kernels.
"""
import pytest
import torch

from metallora_b200 import kernels, ops, torch_ops
from metallora_b200.exceptions import DeviceError, ShapeError

OPS = ("lora_fwd", "lora_bwd", "merge", "linear")


def _inputs(device, dtype, lead=(2, 3), K=64, N=40, r=12, ab_dtype=None, grad=False, seed=0):
    g = torch.Generator(device=device).manual_seed(seed)
    abt = ab_dtype or dtype
    x = torch.randn(*lead, K, device=device, generator=g).to(dtype)
    w0 = (torch.randn(N, K, device=device, generator=g) / K ** 0.5).to(dtype)
    a = ((torch.rand(r, K, device=device, generator=g) * 2 - 1) / K ** 0.5).to(abt)
    b = (torch.randn(N, r, device=device, generator=g) * 0.1).to(abt)
    dy = torch.randn(*lead, N, device=device, generator=g).to(dtype)
    if grad:
        for t in (x, a, b):
            t.requires_grad_(True)
    return x, w0, a, b, dy


def test_ops_registered():
    for name in OPS:
        assert hasattr(torch.ops.metal_lora, name), name
    schema = str(torch.ops.metal_lora.lora_fwd.default._schema)
    assert "float alpha" in schema and "-> (Tensor, Tensor)" in schema


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_fake_trace_forward_backward(dtype):
    """make_fx over forward + autograd.grad: the graph holds lora_fwd and
    lora_bwd, and the traced outputs carry the right shapes and dtypes
    (A/B gradients in A/B's own dtype)."""
    from torch.fx.experimental.proxy_tensor import make_fx

    def step(x, w0, a, b):
        y = torch_ops.lora_linear(x, w0, a, b, 32.0)
        loss = y.float().square().mean()
        gx, ga, gb = torch.autograd.grad(loss, (x, a, b))
        return y, gx, ga, gb

    x, w0, a, b, _ = _inputs("cpu", dtype, ab_dtype=torch.float32, grad=True)
    gm = make_fx(step, tracing_mode="fake")(x, w0, a, b)
    targets = [str(n.target) for n in gm.graph.nodes if n.op == "call_function"]
    assert "metal_lora.lora_fwd.default" in targets
    assert "metal_lora.lora_bwd.default" in targets
    outs = [n for n in gm.graph.nodes if n.op == "output"][0].args[0]
    metas = [o.meta["val"] for o in outs]
    assert tuple(metas[0].shape) == (2, 3, 40) and metas[0].dtype == dtype
    assert tuple(metas[1].shape) == (2, 3, 64) and metas[1].dtype == dtype
    assert tuple(metas[2].shape) == (12, 64) and metas[2].dtype == torch.float32
    assert tuple(metas[3].shape) == (40, 12) and metas[3].dtype == torch.float32


def test_fake_saved_intermediate_shape():
    """The forward's second output is the [padded rank, ceil8(M)] rank
    intermediate for 16-bit x and empty for fp32."""
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        for dtype, want in ((torch.bfloat16, (16, 8)), (torch.float32, (0,))):
            x, w0, a, b, _ = _inputs("cpu", dtype, lead=(5,), r=12)
            y, saved = torch.ops.metal_lora.lora_fwd(x, w0, a, b, 2.0)
            assert tuple(y.shape) == (5, 40) and tuple(saved.shape) == want
        x, w0, a, b, _ = _inputs("cpu", torch.bfloat16, lead=(300,), r=40)
        assert tuple(torch.ops.metal_lora.lora_fwd(x, w0, a, b, 2.0)[1].shape) == (64, 304)


def test_shape_errors_and_no_cpu_fallback():
    x, w0, a, b, dy = _inputs("cpu", torch.bfloat16)
    with pytest.raises(ShapeError):
        torch.ops.metal_lora.lora_fwd(x, w0, a[:, :32], b, 2.0)
    with pytest.raises(ShapeError):
        torch.ops.metal_lora.lora_fwd(x, w0, a, b[:, :4], 2.0)
    with pytest.raises(DeviceError):
        torch_ops.lora_linear(x, w0, a, b)
    with pytest.raises(DeviceError):
        torch.ops.metal_lora.merge(w0, a, b, 2.0)
    with pytest.raises(DeviceError):
        torch.ops.metal_lora.linear(x, w0)


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-30))


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("r", [16, 12])
def test_custom_op_matches_module_path(cuda, dtype, r):
    """Forward and all gradients through the operators equal, bit for bit, the
    autograd path LoRALinear uses (same kernels), at a ragged 3-D shape."""
    lead, K, N, alpha = (3, 100), 256, 264, 32.0
    x, w0, a, b, dy = _inputs(cuda, dtype, lead=lead, K=K, N=N, r=r, seed=11)
    res = []
    for fn in (lambda *t: ops.lora_forward(*t, alpha=alpha),
               lambda *t: torch_ops.lora_linear(*t, alpha)):
        xs, as_, bs = (t.detach().clone().requires_grad_(True) for t in (x, a, b))
        y = fn(xs, w0, as_, bs)
        y.backward(dy)
        res.append((y.detach(), xs.grad, as_.grad, bs.grad))
    for t1, t2 in zip(*res):
        assert t1.dtype == t2.dtype and t1.shape == t2.shape
        assert torch.equal(t1, t2)
    # and against a torch fp32 reference of the same op
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    xf, wf, af, bf = (t.detach().float() for t in (x, w0, a, b))
    s = alpha / r
    y_ref = xf @ wf.t() + s * (xf @ af.t()) @ bf.t()
    assert _rel(res[1][0], y_ref) < tol
    dyf = dy.float().reshape(-1, N)
    x2 = xf.reshape(-1, K)
    assert _rel(res[1][2], s * (dyf @ bf).t() @ x2) < tol
    assert _rel(res[1][3], s * dyf.t() @ (x2 @ af.t())) < tol


@pytest.mark.gpu
def test_custom_op_wide_ab_and_trainable_base(cuda):
    """fp32 A/B with bf16 activations (cast inside the operator, gradients in
    fp32) and a base weight that requires a gradient."""
    x, w0, a, b, dy = _inputs(cuda, torch.bfloat16, lead=(256,), K=128, N=136, r=16,
                              ab_dtype=torch.float32, grad=True, seed=3)
    w0.requires_grad_(True)
    y = torch_ops.lora_linear(x, w0, a, b, 16.0)
    y.backward(dy)
    assert a.grad.dtype == torch.float32 and b.grad.dtype == torch.float32
    assert w0.grad is not None and w0.grad.dtype == torch.bfloat16
    ref = dy.float().t() @ x.detach().float()
    assert _rel(w0.grad, ref) < 2e-2
    ab = (a.detach().bfloat16(), b.detach().bfloat16())
    _, saved = kernels.lora_linear_fwd(x.detach(), w0.detach(), *ab, 16.0, save_xa=True)
    _, da, db = kernels.lora_linear_bwd(dy, x.detach(), w0.detach(), *ab, 16.0, saved)
    assert torch.equal(a.grad, da) and torch.equal(b.grad, db)


@pytest.mark.gpu
def test_opcheck(cuda):
    from torch.library import opcheck

    x, w0, a, b, dy = _inputs(cuda, torch.bfloat16, lead=(2, 64), K=128, N=136, r=16, seed=5)
    fwd_args = (x, w0, a, b, 32.0)
    opcheck(torch.ops.metal_lora.lora_fwd.default, fwd_args,
            test_utils=("test_schema", "test_autograd_registration", "test_faketensor"))
    _, saved = torch.ops.metal_lora.lora_fwd(*fwd_args)
    plain = ("test_schema", "test_faketensor")
    opcheck(torch.ops.metal_lora.lora_bwd.default, (dy, x, w0, a, b, saved, 32.0, 0.0, True),
            test_utils=plain)
    opcheck(torch.ops.metal_lora.lora_bwd.default, (dy, x, w0, a, b, saved, 32.0, 0.5, False),
            test_utils=plain)
    opcheck(torch.ops.metal_lora.merge.default, (w0, a, b, 32.0), test_utils=plain)
    opcheck(torch.ops.metal_lora.linear.default, (x, w0), test_utils=plain)


@pytest.mark.gpu
def test_merge_and_linear_ops_match_kernels(cuda):
    x, w0, a, b, _ = _inputs(cuda, torch.bfloat16, lead=(300,), K=256, N=264, r=16, seed=9)
    wm = torch.ops.metal_lora.merge(w0, a, b, 32.0)
    assert torch.equal(wm, kernels.merge(w0, a, b, 32.0))
    y = torch.ops.metal_lora.linear(x, wm)
    assert torch.equal(y, kernels.linear(x, wm))
    # merged forward == unmerged forward (examples/basic_usage.py:114-140)
    assert _rel(y, torch_ops.lora_linear(x, w0, a, b, 32.0)) < 2e-2


def _q_inputs(device, scheme, M=64, K=128, N=136, r=16):
    g = torch.Generator(device=device).manual_seed(21)
    per_byte = 1 if scheme == "int8" else 2
    group = 64 if scheme == "nf4" else 128
    x = torch.randn(M, K, device=device, generator=g).to(torch.bfloat16)
    codes = torch.randint(0, 256, (N, K // per_byte), device=device, generator=g,
                          dtype=torch.int32).to(torch.uint8)
    if scheme == "nf4":
        scales = torch.rand(N, K // group, device=device, generator=g)
        zeros = None
    else:
        scales = (torch.rand(N, K // group, device=device, generator=g) * 0.01).half()
        zeros = torch.full((N, K // group), 8.0, device=device).half()
    a = (torch.randn(r, K, device=device, generator=g) / K ** 0.5).to(torch.bfloat16)
    b = (torch.randn(N, r, device=device, generator=g) * 0.1).to(torch.bfloat16)
    return x, codes, scales, zeros, group, a, b


@pytest.mark.parametrize("scheme", ["nf4", "int4", "int8"])
def test_qlora_fake_trace(scheme):
    from torch.fx.experimental.proxy_tensor import make_fx

    x, codes, scales, zeros, group, a, b = _q_inputs("cpu", scheme)
    a = a.float().requires_grad_(True)
    b = b.float().requires_grad_(True)
    x.requires_grad_(True)

    def step(x, codes, scales, zeros, a, b):
        y = torch.ops.metal_lora.qlora_fwd(x, codes, scales, zeros, None, scheme, group, False,
                                           a, b, 32.0)[0]
        return (y,) + torch.autograd.grad(y.float().sum(), (x, a, b))

    gm = make_fx(step, tracing_mode="fake")(x, codes, scales, zeros, a, b)
    targets = [str(n.target) for n in gm.graph.nodes if n.op == "call_function"]
    assert "metal_lora.qlora_fwd.default" in targets
    assert "metal_lora.qlora_bwd.default" in targets
    outs = [o.meta["val"] for o in [n for n in gm.graph.nodes if n.op == "output"][0].args[0]]
    assert [tuple(t.shape) for t in outs] == [(64, 136), (64, 128), (16, 128), (136, 16)]
    with pytest.raises(ShapeError):
        torch.ops.metal_lora.qlora_fwd(x.detach()[:, :64], codes, scales, zeros, None, scheme,
                                       group, False, a.detach(), b.detach(), 32.0)


@pytest.mark.gpu
@pytest.mark.parametrize("scheme,lean", [("nf4", False), ("nf4", True), ("int4", False),
                                         ("int8", False)])
def test_qlora_custom_op_matches_module_path(cuda, scheme, lean):
    """Quantised base: the operators equal the ops.qlora_forward autograd path
    bit for bit (forward, dx, dA, dB)."""
    from metallora_b200 import quant

    g = torch.Generator(device=cuda).manual_seed(13)
    M, K, N, r = 300, 256, 264, 16
    w = torch.randn(N, K, device=cuda, generator=g) / K ** 0.5
    qw = quant.quantize(w, scheme, lean=lean)
    x = torch.randn(3, M // 3, K, device=cuda, generator=g).to(torch.bfloat16)
    a = (torch.randn(r, K, device=cuda, generator=g) / K ** 0.5).to(torch.bfloat16)
    b = (torch.randn(N, r, device=cuda, generator=g) * 0.1).to(torch.bfloat16)
    dy = torch.randn(3, M // 3, N, device=cuda, generator=g).to(torch.bfloat16)
    res = []
    for fn in (lambda *t: ops.qlora_forward(t[0], qw, t[1], t[2], 32.0),
               lambda *t: torch_ops.qlora_linear(t[0], qw, t[1], t[2], 32.0)):
        xs, as_, bs = (t.detach().clone().requires_grad_(True) for t in (x, a, b))
        y = fn(xs, as_, bs)
        y.backward(dy)
        res.append((y.detach(), xs.grad, as_.grad, bs.grad))
    for t1, t2 in zip(*res):
        assert t1.dtype == t2.dtype and t1.shape == t2.shape
        assert torch.equal(t1, t2)
    # against torch fp32 on the dequantised weight
    wd = qw.dequantize(torch.float32)
    xf = x.float().reshape(-1, K)
    y_ref = xf @ wd.t() + (32.0 / r) * (xf @ a.float().t()) @ b.float().t()
    assert _rel(res[1][0].reshape(-1, N), y_ref) < 2e-2
    # the prepared scale table passed in or built in the call: same result
    y2 = torch.ops.metal_lora.qlora_fwd(x, qw.codes, qw.scales, qw.zeros, None, scheme, qw.group,
                                        lean, a, b, 32.0)[0]
    assert torch.equal(y2, res[1][0])


def test_adamw_ops_trace_and_errors():
    """The optimizer operators trace (mutating, no outputs) and keep the
    kernels' argument rules; CPU tensors raise DeviceError."""
    from torch.fx.experimental.proxy_tensor import make_fx

    def step(p, g, m, v, st):
        torch.ops.metal_lora.adam_state_step(st, 0.9, 0.999)
        torch.ops.metal_lora.adamw_step(p, g, m, v, st, 1e-3, 0.9, 0.999, 1e-8, 0.01)
        return p, g, m, v, st

    p = torch.randn(16, 8)
    g, m, v = torch.randn(16, 8), torch.zeros(16, 8), torch.zeros(16, 8)
    st = torch.tensor([0.0, 1.0, 1.0])
    gm = make_fx(step, tracing_mode="fake")(p, g, m, v, st)
    targets = [str(n.target) for n in gm.graph.nodes if n.op == "call_function"]
    assert "metal_lora.adamw_step.default" in targets
    assert "metal_lora.adam_state_step.default" in targets
    with pytest.raises(DeviceError):
        torch.ops.metal_lora.adamw_step(p, g, m, v, st, 1e-3, 0.9, 0.999, 1e-8, 0.01)
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        fp, fg = torch.empty(16, 8), torch.empty(16, 8, dtype=torch.float16)
        with pytest.raises(ShapeError):
            torch.ops.metal_lora.adamw_step(fp, fg, fp.clone(), fp.clone(), torch.empty(3),
                                            1e-3, 0.9, 0.999, 1e-8, 0.01)


@pytest.mark.gpu
def test_adamw_ops_match_kernel_calls(cuda):
    """Two AdamW steps through the operators equal, bit for bit, the same
    steps through kernels.lora_adamw_step_metal (bf16 and fp32 params)."""
    from torch.library import opcheck

    for dtype in (torch.bfloat16, torch.float32):
        g0 = torch.Generator(device=cuda).manual_seed(17)
        p0 = torch.randn(4096 + 5, device=cuda, generator=g0).to(dtype)
        grads = [torch.randn(p0.numel(), device=cuda, generator=g0) for _ in range(2)]
        out = []
        for use_ops in (False, True):
            p, m, v = p0.clone(), torch.zeros_like(p0, dtype=torch.float32), \
                torch.zeros_like(p0, dtype=torch.float32)
            st = kernels.persistent_gpu_state_init(device=cuda)
            for gr in grads:
                g = gr.clone()
                if use_ops:
                    torch.ops.metal_lora.adam_state_step(st, 0.9, 0.999)
                    torch.ops.metal_lora.adamw_step(p, g, m, v, st, 1e-3, 0.9, 0.999, 1e-8, 0.01)
                else:
                    kernels.persistent_gpu_state_step(st, 0.9, 0.999)
                    kernels.lora_adamw_step_metal(p, g, m, v, st, 1e-3, 0.9, 0.999, 1e-8, 0.01)
                assert not g.any()  # the step zeroes the gradient
            out.append((p, m, v, st))
        for t1, t2 in zip(*out):
            assert torch.equal(t1, t2)
    p = torch.randn(256, device=cuda)
    args = (p, torch.randn(256, device=cuda), torch.zeros(256, device=cuda),
            torch.zeros(256, device=cuda), torch.tensor([1.0, 0.9, 0.999], device=cuda),
            1e-3, 0.9, 0.999, 1e-8, 0.0)
    opcheck(torch.ops.metal_lora.adamw_step.default, args,
            test_utils=("test_schema", "test_faketensor"))
