"""The allocation-free weight-gradient entry point (mlora_lora_grads_static).

It exists for callers that cannot allocate device memory when the backward
runs, so it must produce the same dA/dB as the workspace-taking
mlora_lora_backward.  Both run the same kernels on the same inputs and the
backward is bitwise deterministic, so the results must be bit-identical.

This file is named to be collected last, and it works both alone in a fresh
process and after the other tests.  The built-in scratch keeps whatever the
previous call left, which no call may depend on: before the checked calls, a
larger call fills more of the array than they use, and the workspace path runs
on a workspace filled with NaN bytes.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

DTYPES = {torch.bfloat16: 0, torch.float16: 1}


def _inputs(M, K, N, r, seed, dev, dtype):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).to(dtype).to(dev)
    dy = torch.randn(M, N, generator=g).to(dtype).to(dev)
    a = ((torch.rand(r, K, generator=g) * 2 - 1) / K ** 0.5).to(dtype).to(dev)
    b = (torch.randn(N, r, generator=g) * 0.1).to(dtype).to(dev)
    return x, dy, a, b


def _with_workspace(lib, x, dy, a, b, alpha, clip):
    M, K = x.shape
    N, r = b.shape
    code = DTYPES[x.dtype]
    da = torch.full((r, K), float("nan"), dtype=torch.float32, device=x.device)
    db = torch.full((N, r), float("nan"), dtype=torch.float32, device=x.device)
    nbytes = lib.mlora_lora_backward_workspace_bytes(M, K, N, r, code)
    ws = torch.full((nbytes,), 0xFF, dtype=torch.uint8, device=x.device)  # NaN bytes
    st = lib.mlora_lora_backward(dy.data_ptr(), x.data_ptr(), None, a.data_ptr(), b.data_ptr(),
                                 None, None, da.data_ptr(), db.data_ptr(), M, K, N, r, alpha,
                                 clip, code, ws.data_ptr(), ws.numel(),
                                 torch.cuda.current_stream().cuda_stream)
    assert st == 0, lib.mlora_last_error_message()
    return da, db


def _static(lib, x, dy, a, b, alpha, clip):
    M, K = x.shape
    N, r = b.shape
    da = torch.full((r, K), float("nan"), dtype=torch.float32, device=x.device)
    db = torch.full((N, r), float("nan"), dtype=torch.float32, device=x.device)
    st = lib.mlora_lora_grads_static(dy.data_ptr(), x.data_ptr(), a.data_ptr(), b.data_ptr(),
                                     da.data_ptr(), db.data_ptr(), M, K, N, r, alpha, clip,
                                     DTYPES[x.dtype], torch.cuda.current_stream().cuda_stream)
    assert st == 0, lib.mlora_last_error_message()
    return da, db


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_static_scratch_matches_workspace_entry_point(cuda, dtype):
    from metallora_b200 import _lib
    lib = _lib.load()
    assert lib.mlora_lora_grads_static_scratch_bytes() == 32 << 20
    # a larger call first leaves its values in more of the shared array than
    # the checked calls below use
    big = _inputs(8192, 2048, 2048, 128, 7, cuda, dtype)
    assert lib.mlora_lora_backward_workspace_bytes(8192, 2048, 2048, 128, DTYPES[dtype]) <= 32 << 20
    _static(lib, *big, 16.0, 0.0)
    # two calls in a row, different shapes and data, each against the workspace path
    for (M, K, N, r, seed, clip) in [(1024, 512, 768, 16, 1, 0.0), (4096, 1024, 1024, 64, 2, 0.5)]:
        x, dy, a, b = _inputs(M, K, N, r, seed, cuda, dtype)
        ref_a, ref_b = _with_workspace(lib, x, dy, a, b, 32.0, clip)
        got_a, got_b = _static(lib, x, dy, a, b, 32.0, clip)
        torch.cuda.synchronize()
        assert torch.isfinite(got_a).all() and torch.isfinite(got_b).all()
        assert torch.equal(got_a, ref_a) and torch.equal(got_b, ref_b)
        if clip > 0:
            assert float(got_a.abs().max()) <= clip and float(got_b.abs().max()) <= clip
    assert _lib.device_status(reset=True) == 0


def test_static_scratch_rejects_oversized_shapes(cuda):
    from metallora_b200 import _lib
    lib = _lib.load()
    x = torch.empty(16, dtype=torch.bfloat16, device=cuda)
    f = torch.empty(16, dtype=torch.float32, device=cuda)
    M, K, N, r = 1 << 20, 4096, 4096, 64  # needs far more than the built-in array
    st = lib.mlora_lora_grads_static(x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(),
                                     f.data_ptr(), f.data_ptr(), M, K, N, r, 32.0, 0.0, 0,
                                     torch.cuda.current_stream().cuda_stream)
    assert st == _lib.MLORA_ERR_WORKSPACE
    assert b"built-in array" in lib.mlora_last_error_message()
