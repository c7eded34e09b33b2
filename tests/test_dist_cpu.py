"""Multi-rank logic of the data-parallel layer on CPU ranks (gloo, world 2):
token sharding, gradient averaging and replica-sync checks."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from metallora_b200.distributed import (average_gradients, replicas_in_sync, shard_bounds,
                                        shard_tokens)


def test_shard_bounds_cover_all_tokens():
    for n in (1, 7, 8192, 8193):
        for world in (1, 2, 3, 8):
            spans = [shard_bounds(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [e - b for b, e in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_bounds(10, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=30))
    try:
        x = torch.arange(4 * 6 * 3, dtype=torch.float32).reshape(4, 6, 3)
        mine = shard_tokens(x, rank, world)
        g = torch.full((10,), float(rank + 1))
        average_gradients(g)
        same = replicas_in_sync(g)
        p = torch.full((5,), 1.0 + rank)  # deliberately different
        diff = replicas_in_sync(p)
        q.put((rank, mine.shape[0], g.tolist(), same, diff))
    finally:
        dist.destroy_process_group()


def test_gloo_average_and_sync():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [r[1] for r in res] == [12, 12]           # 24 tokens over 2 ranks
    for r in res:
        assert r[2] == [1.5] * 10                    # mean of 1 and 2
        assert r[3] is True and r[4] is False


def test_device_cpus_without_gpu_is_none():
    """NUMA binding degrades to a no-op where NVML or the device is missing."""
    import torch

    from metallora_b200.distributed import bind_to_device, device_cpus
    if torch.cuda.is_available():
        import pytest
        pytest.skip("CPU-only check")
    assert device_cpus(0) is None
    assert bind_to_device(0) is None


def test_fault_injection_spec(monkeypatch):
    from metallora_b200.distributed import FAULT_ENV, InjectedFault, maybe_inject_fault
    monkeypatch.delenv(FAULT_ENV, raising=False)
    maybe_inject_fault("before_allreduce", 1)
    monkeypatch.setenv(FAULT_ENV, "before_peer_allreduce@0, before_allreduce@1")
    maybe_inject_fault("before_allreduce", 0)
    maybe_inject_fault("before_peer_allreduce", 1)
    with pytest.raises(InjectedFault):
        maybe_inject_fault("before_allreduce", 1)
    with pytest.raises(InjectedFault):
        maybe_inject_fault("before_peer_allreduce", 0)


def _fault_worker(rank, world, port, q, mode):
    import datetime
    import time

    from metallora_b200.distributed import FAULT_ENV, InjectedFault
    from metallora_b200.exceptions import DistributedError
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    os.environ[FAULT_ENV] = "before_allreduce@1"
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=3))
    t0 = time.monotonic()
    try:
        g = torch.ones(8)
        average_gradients(g)
        q.put((rank, "ok", time.monotonic() - t0))
    except InjectedFault:
        q.put((rank, "injected", time.monotonic() - t0))
        if mode == "linger":
            time.sleep(8)  # alive, but never joins the collective
    except DistributedError:
        q.put((rank, "distributed_error", time.monotonic() - t0))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


@pytest.mark.parametrize("mode", ["exit", "linger"])
def test_peer_failure_surfaces_as_error(mode):
    """A rank that fails on the host before the gradient all-reduce (injected
    through MLORA_FAULT_INJECT) -- and then exits, or stays alive without
    joining -- makes its peer's all-reduce end with DistributedError within
    the process group's timeout instead of hanging."""
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_fault_worker, args=(r, world, port, q, mode))
             for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = dict((r, (kind, dt)) for r, kind, dt in (q.get(timeout=90) for _ in range(world)))
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
                p.join()
    assert res[1][0] == "injected"
    assert res[0][0] == "distributed_error"
    assert res[0][1] < 30.0


def _bucket_worker(rank, world, port, q):
    from metallora_b200.distributed import BucketedGradExchange
    from metallora_b200.exceptions import DistributedError
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=30))
    try:
        # seven producers of 3..9 floats; buckets of >= 32 bytes (8 floats)
        sizes = [3, 4, 5, 6, 7, 8, 9]
        members, off = [], 0
        for n in sizes:
            members.append((off, off + n))
            off += n
        flat = torch.zeros(off)
        ex = BucketedGradExchange(flat, members, bucket_bytes=32)
        buckets = [m for _, _, m in ex.buckets]
        res = {"buckets": buckets}
        for step in range(2):
            # the backward writes producers last-to-first; producer 1 takes no
            # part in this step (finish() must still average its bucket)
            for i in reversed(range(len(sizes))):
                if i == 1:
                    continue
                b, e = members[i]
                flat[b:e] = float((rank + 1) * (i + 1) + step)
                ex.ready(i)
            b, e = members[1]
            flat[b:e] = float((rank + 1) * 2 + step)
            fired_before_finish = list(ex.fired_order)
            ex.finish()
            res[f"fired{step}"] = fired_before_finish
            res[f"flat{step}"] = flat.tolist()
        # disarmed (a micro-batch before the last): nothing fires
        ex.armed = False
        ex.ready(6)
        res["disarmed_fired"] = list(ex.fired_order)
        ex.armed = True
        ex.ready(6)
        try:
            ex.ready(6)
            res["double"] = "no error"
        except DistributedError:
            res["double"] = "error"
        ex.finish()
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


def test_gloo_bucketed_exchange():
    """Per-layer gradient buckets: grouping, firing as soon as all members
    reported (in backward order), averaging, finish() for silent producers,
    disarming between micro-batches and the double-report error."""
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_bucket_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    r0 = res[0]
    assert r0["buckets"] == [[0, 1, 2], [3, 4], [5], [6]]
    # backward order 6,5,4,3,2,0: buckets 3, 2 and 1 fire as they complete;
    # bucket 0 waits for producer 1 until finish()
    assert r0["fired0"] == [3, 2, 1] and r0["fired1"] == [3, 2, 1]
    sizes = [3, 4, 5, 6, 7, 8, 9]
    for step in range(2):
        want = []
        for i, n in enumerate(sizes):
            want += [1.5 * (i + 1) + step] * n  # mean over ranks of (rank+1)(i+1)+step
        assert r0[f"flat{step}"] == want and res[1][f"flat{step}"] == want
    assert r0["disarmed_fired"] == [] and r0["double"] == "error"


def _live_worker(rank, world, port, q, mode):
    from metallora_b200.distributed import PeerLiveness
    from metallora_b200.exceptions import DistributedError
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=30))
    live = PeerLiveness(timeout_s=3.0)
    for step in range(3):  # all present: every check returns
        live.beat(step)
        live.check(step)
    if rank == 1:
        if mode == "leave":
            live.leave()
        q.put((rank, "gone", 0.0))
        q.close()
        q.join_thread()  # the message is written before the process goes
        if mode == "stall":
            __import__("time").sleep(8.0)  # alive, but never reaches step 3
        os._exit(0)
    t0 = __import__("time").monotonic()
    try:
        live.beat(3)
        live.check(3)
        out = "no error"
    except DistributedError as e:
        out = "left" if "left the process group" in str(e) else ("timeout" if "reached step" in str(e) else str(e))
    q.put((rank, out, __import__("time").monotonic() - t0))
    q.close()
    q.join_thread()
    os._exit(0)


@pytest.mark.parametrize("mode", ["leave", "stall"])
def test_peer_liveness(mode):
    """Host-side membership check: a peer that leaves between steps is seen
    at once by the survivor's next check; one that stops without a word is
    reported after the check's timeout.  Nothing waits on a collective."""
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_live_worker, args=(r, world, port, q, mode))
             for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = {r: (s, t) for r, s, t in (q.get(timeout=120) for _ in range(world))}
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
                p.join()
    assert res[1][0] == "gone"
    if mode == "leave":
        assert res[0][0] == "left" and res[0][1] < 2.0
    else:
        assert res[0][0] == "timeout" and 2.5 < res[0][1] < 10.0
