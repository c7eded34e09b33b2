"""The CTA-pair GEMM (cta_group::2, 256 x 256 tiles; used from 256 tokens) and
the single-CTA GEMM (128 x 256 tiles; MLORA_GEMM_PAIR=0) must agree: the same
LoRA forward and backward run in a child process with the single-CTA kernel
and here with the pair kernel, on the same seeded inputs.  Shapes cover ragged
M and N (a pair tile half outside the matrix) and the MN-major dx GEMM."""
import os
import subprocess
import sys

import pytest
import torch

CHILD = r"""
import sys, torch
from metallora_b200 import kernels
M, K, N, r = (int(v) for v in sys.argv[1:5])
g = torch.Generator(device="cuda").manual_seed(7)
x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
w = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5).to(torch.bfloat16)
a = (torch.randn(r, K, device="cuda", generator=g) / K ** 0.5).to(torch.bfloat16)
b = (torch.randn(N, r, device="cuda", generator=g) * 0.1).to(torch.bfloat16)
dy = torch.randn(M, N, device="cuda", generator=g).to(torch.bfloat16)
y, saved = kernels.lora_linear_fwd(x, w, a, b, 2.0 * r, save_xa=True)
dx, da, db = kernels.lora_linear_bwd(dy, x, w, a, b, 2.0 * r, saved)
torch.cuda.synchronize()
torch.save({"y": y.cpu(), "dx": dx.cpu(), "da": da.cpu(), "db": db.cpu()}, sys.argv[5])
"""


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,N,r", [(1024, 512, 768, 16), (300, 256, 200, 8), (512, 1024, 4096, 64)])
def test_pair_gemm_matches_single_cta(tmp_path, M, K, N, r):
    outs = {}
    for mode in ("0", "1"):
        path = tmp_path / f"out{mode}.pt"
        env = dict(os.environ, MLORA_GEMM_PAIR=mode)
        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        subprocess.run([sys.executable, "-c", CHILD, str(M), str(K), str(N), str(r), str(path)],
                       check=True, env=env, cwd=root, timeout=300)
        outs[mode] = torch.load(path)
    for k in ("y", "dx", "da", "db"):
        assert torch.equal(outs["0"][k], outs["1"][k]), k
