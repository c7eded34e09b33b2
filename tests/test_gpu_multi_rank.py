"""Data-parallel training on two GPUs (one process per GPU, NCCL), needing at
least two GPUs (skipped otherwise):

* two LoRATrainer steps whose per-layer gradient buckets are averaged on a
  side stream while the backward runs leave the replicas bitwise identical,
  and the averaged gradient equals the mean of both ranks' own gradients;
* failure detection without a GPU fault: rank 1 leaves between steps (after a
  synchronize, with nothing of its own in flight) and says so through the
  process group's store; rank 0's next step raises DistributedError from its
  host-side liveness check, before it launches any kernel or collective of
  that step, and its process exits.

NVLS is off (NCCL_NVLS_ENABLE=0) and no symmetric memory is used, so no
NVLink multicast object is bound when a rank leaves."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _model(dev, seed=0):
    from metallora_b200.layers import LoRALinear
    g = torch.Generator(device=dev).manual_seed(seed)
    m = torch.nn.Sequential(LoRALinear(256, 512, rank=16, alpha=32.0, device=dev,
                                       dtype=torch.bfloat16),
                            LoRALinear(512, 256, rank=16, alpha=32.0, device=dev,
                                       dtype=torch.bfloat16))
    with torch.no_grad():
        for lin in m:
            lin.W0.copy_(torch.randn(lin.W0.shape, device=dev, generator=g) / 16)
            lin.B.copy_(torch.randn(lin.B.shape, device=dev, generator=g) * 0.1)
    return m


def _worker(rank, world, port, q, mode):
    import datetime
    import time

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0",
                      TORCH_NCCL_BLOCKING_WAIT="1")
    from metallora_b200.distributed import replicas_in_sync
    from metallora_b200.exceptions import DistributedError
    from metallora_b200.trainer import LoRATrainer, TrainingConfig
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=8), device_id=dev)
    res = {"rank": rank}
    try:
        model = _model(dev)
        cfg = TrainingConfig(rank=16, alpha=32.0, learning_rate=1e-3, max_grad_norm=0.0,
                             output_dir=f"/tmp/mlora_mr_{rank}")
        tr = LoRATrainer(model, cfg, liveness_timeout=20.0)
        assert tr.exchange is not None
        res["init_in_sync"] = replicas_in_sync(tr.params.master)
        g = torch.Generator(device=dev).manual_seed(100 + rank)  # each rank its own shard
        batch = {"input_ids": torch.randn(2, 64, 256, device=dev, generator=g).to(torch.bfloat16),
                 "target_output": torch.randn(2, 64, 256, device=dev, generator=g).to(torch.bfloat16)}
        # the averaged gradient of one step against the mean of the ranks' own
        tr.backward(batch)
        tr.exchange.finish()
        avg = tr.params.grad.clone()
        res["avg_in_sync"] = replicas_in_sync(avg)
        tr.params.grad.zero_()
        tr.exchange.armed = False  # this rank's own gradient, not exchanged
        tr._compute_loss(batch).backward()
        own = tr.params.grad.clone()
        tr.params.grad.zero_()
        both = [torch.empty_like(own) for _ in range(world)]
        dist.all_gather(both, own)
        mean = sum(both) / world
        res["avg_rel_err"] = float((avg - mean).norm() / mean.norm())
        res["step_in_sync"] = []
        for _ in range(2):
            tr._training_step(batch)
            res["step_in_sync"].append(replicas_in_sync(tr.params.master))
        res["in_sync"] = replicas_in_sync(tr.params.master)
        torch.cuda.synchronize()
        if mode == "leave":
            if rank == 1:
                tr.leave()  # tells the peers through the store, then goes
                res["status"] = "left"
                q.put(res)
                q.close()
                q.join_thread()  # the report is written before the process goes
                os._exit(0)  # between steps: nothing of this rank is in flight
            t0 = time.monotonic()
            try:
                tr._training_step(batch)
                res["status"] = "no error"
            except DistributedError:
                res["status"] = "distributed_error"
            except Exception as e:  # noqa: BLE001 -- reported, then the test fails
                res["status"] = f"other: {type(e).__name__}: {str(e)[:200]}"
            res["seconds"] = time.monotonic() - t0
        q.put(res)
    except Exception as e:  # noqa: BLE001
        res["status"] = f"setup: {type(e).__name__}: {str(e)[:300]}"
        q.put(res)
    finally:
        if mode == "leave":
            q.close()
            q.join_thread()  # the report is written before the process goes
            os._exit(0)  # the survivor's communicator is gone with its process
        dist.destroy_process_group()


def _run(mode, timeout):
    import torch.multiprocessing as mp
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, mode)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = {}
        for _ in range(world):
            d = q.get(timeout=timeout)
            res[d["rank"]] = d
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
                p.join()
    hung = [p.pid for p in procs if p.exitcode is None]
    return res, hung


def _need_two():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")


def test_two_rank_bucketed_exchange_keeps_replicas_in_sync(cuda):
    _need_two()
    res, hung = _run("steps", 240)
    assert not hung
    for r in (0, 1):
        assert "status" not in res[r], res[r]
        assert res[r]["init_in_sync"] and res[r]["avg_in_sync"], res[r]
        assert res[r]["avg_rel_err"] < 1e-6, res[r]
        assert res[r]["in_sync"] is True, res[r]


def test_rank_leaving_between_steps_raises_on_survivor(cuda):
    _need_two()
    res, hung = _run("leave", 240)
    assert not hung
    assert res[1]["status"] == "left"
    assert res[0]["in_sync"] is True
    assert res[0]["status"] == "distributed_error", res[0]
    assert res[0]["seconds"] < 60.0
