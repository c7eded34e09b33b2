"""Peer all-reduce (mlora_peer_allreduce).  On one GPU the kernel runs its full
protocol against itself (world 1: flags, counter reset, sequence numbers);
the multi-rank protocol runs in bench.py under torchrun on several GPUs."""
import pytest
import torch


@pytest.mark.gpu
def test_peer_allreduce_world_one(cuda):
    from metallora_b200 import _lib
    n = 4099  # a tail past the float4 body
    buf = torch.randn(n, device=cuda)
    flags = torch.zeros(4, dtype=torch.int32, device=cuda)
    counter = torch.zeros(1, dtype=torch.int32, device=cuda)
    bufs = torch.tensor([buf.data_ptr()], dtype=torch.int64, device=cuda)
    fl = torch.tensor([flags.data_ptr()], dtype=torch.int64, device=cuda)
    lib = _lib.load()
    for seq in range(1, 4):
        out = torch.empty_like(buf)
        st = lib.mlora_peer_allreduce(bufs.data_ptr(), fl.data_ptr(), 0, 1, seq, out.data_ptr(), n,
                                      0.5, counter.data_ptr(), torch.cuda.current_stream().cuda_stream)
        _lib.check(st, "mlora_peer_allreduce")
        torch.cuda.synchronize()
        assert torch.equal(out, buf * 0.5)
        assert int(flags[0]) == 2 * seq and int(counter[0]) == 0
    assert _lib.device_status(reset=True) == 0


def test_peer_allreduce_rejects_bad_arguments():
    from metallora_b200 import _lib
    lib = _lib.load()
    assert lib.mlora_peer_allreduce(None, None, 0, 1, 1, None, 4, 1.0, None, None) == -1
    assert lib.mlora_peer_allreduce(8, 8, 2, 2, 1, 16, 4, 1.0, 8, None) == -1  # rank >= world
    assert lib.mlora_peer_allreduce(8, 8, 0, 1, 0, 16, 4, 1.0, 8, None) == -1  # seq 0


@pytest.mark.gpu
def test_device_cpus_reports_numa_cores(cuda):
    """NVML names the host cores of the GPU's NUMA node (read-only query)."""
    import os

    from metallora_b200.distributed import device_cpus
    cpus = device_cpus(cuda)
    assert cpus and all(0 <= c < (os.cpu_count() or 1) for c in cpus)
