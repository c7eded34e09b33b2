"""Peer all-reduce (mlora_peer_allreduce).  On one GPU the kernel runs its full
protocol against itself (world 1: flags, counter reset, sequence numbers);
the multi-rank protocol runs in bench.py under torchrun on several GPUs, where
every N > 1 line compares it with an NCCL all-reduce of the same buffer."""
import pytest
import torch


def _ptrs(ts, dev):
    return torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64, device=dev)


@pytest.mark.gpu
@pytest.mark.parametrize("n", [4099, 148 * 256 * 4 * 3 + 5])  # one CTA / a full grid
def test_peer_allreduce_world_one(cuda, n):
    from metallora_b200 import _lib
    buf = torch.randn(n, device=cuda)
    flags = torch.zeros(4, dtype=torch.int32, device=cuda)
    counter = torch.zeros(4, dtype=torch.int32, device=cuda)
    bufs, fl = _ptrs([buf], cuda), _ptrs([flags], cuda)
    lib = _lib.load()
    for seq in range(1, 4):
        out = torch.empty_like(buf)
        st = lib.mlora_peer_allreduce(bufs.data_ptr(), fl.data_ptr(), 0, 1, seq, out.data_ptr(), n,
                                      0.5, counter.data_ptr(), torch.cuda.current_stream().cuda_stream)
        _lib.check(st, "mlora_peer_allreduce")
        torch.cuda.synchronize()
        assert torch.equal(out, buf * 0.5)
        assert int(flags[0]) == 2 * seq and int(counter[0]) == 0
        assert int(counter[1]) == seq and int(counter[2]) == 1  # the grid's verdict: go
    assert _lib.device_status(reset=True) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("n", [1024, 148 * 256 * 4 * 2])  # one CTA / every SM
def test_peer_allreduce_wait_runs_out(cuda, n):
    """Failure detection on the GPU without a fault: rank 0 of a two-rank
    exchange whose peer never raises its flags (a flag that nothing sets)
    gives up after the 2 s wait budget at the arrival barrier and again at the
    exit barrier, records status 0x108 (peer timeout), skips the reduction in
    every CTA (one verdict for the whole grid) and returns; the context stays
    usable for the next call."""
    import time

    from metallora_b200 import _lib
    buf0, buf1 = torch.randn(n, device=cuda), torch.randn(n, device=cuda)
    flags0 = torch.zeros(4, dtype=torch.int32, device=cuda)
    flags1 = torch.zeros(4, dtype=torch.int32, device=cuda)
    counter = torch.zeros(4, dtype=torch.int32, device=cuda)
    bufs, fl = _ptrs([buf0, buf1], cuda), _ptrs([flags0, flags1], cuda)
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    torch.cuda.synchronize()
    _lib.device_status(reset=True)
    out = torch.full_like(buf0, 7.0)
    t0 = time.monotonic()
    st = lib.mlora_peer_allreduce(bufs.data_ptr(), fl.data_ptr(), 0, 2, 1, out.data_ptr(), n,
                                  0.5, counter.data_ptr(), stream)
    _lib.check(st, "mlora_peer_allreduce")
    torch.cuda.synchronize()
    elapsed = time.monotonic() - t0
    assert _lib.device_status(reset=True) == 0x108
    assert 3.0 < elapsed < 20.0            # two bounded waits of 2 s
    assert bool((out == 7.0).all())        # no CTA wrote a partial reduction
    assert int(flags1[0]) == 2 and int(counter[0]) == 0  # exit flag raised, counter reset
    assert int(counter[1]) == 1 and int(counter[2]) == 0  # the grid's verdict: abort
    # the context still works: a world-1 exchange right after
    buf = torch.randn(n, device=cuda)
    f_solo = torch.zeros(4, dtype=torch.int32, device=cuda)
    solo, fl_solo = _ptrs([buf], cuda), _ptrs([f_solo], cuda)
    out2 = torch.empty_like(buf)
    counter.zero_()
    st = lib.mlora_peer_allreduce(solo.data_ptr(), fl_solo.data_ptr(), 0, 1, 1, out2.data_ptr(),
                                  n, 1.0, counter.data_ptr(), stream)
    _lib.check(st, "mlora_peer_allreduce")
    torch.cuda.synchronize()
    assert torch.equal(out2, buf) and _lib.device_status(reset=True) == 0


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
