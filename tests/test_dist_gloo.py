"""Host logic of the multi-process harness, with world-size-2 gloo ranks on
the CPU: row sharding, max-over-ranks timing, and failure detection (a rank
that dies surfaces as an error on its peer within the process-group timeout
instead of a hang). No GPU is used; failures are made on the host."""
import datetime
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _worker_shards(rank, world, port, q):
    _init(rank, world, port)
    try:
        import oracle
        B, S, H, D = 4, 16, 2, 64
        b = bench.local_batch(B, world, "strong")
        g = torch.Generator().manual_seed(0)
        q_all = torch.randn(B, S, H, D, generator=g)
        w = 1 + 0.1 * torch.randn(D, generator=g)
        gq = torch.randn(B, S, H, D, generator=g)
        inv = oracle.inv_freq(D, 1e4)
        # this rank's contiguous row shard; no collective on the data path
        shard = slice(rank * b, (rank + 1) * b)
        r = oracle.qk_norm_rope_fwd_bwd(q_all[shard], None, w, None, gq[shard], None, None, inv,
                                        1e-6)
        # the weight gradients of the shards add up to the unsharded one
        # (combined here only to check; training uses the DDP all-reduce)
        dw = r["dwq"].clone()
        dist.all_reduce(dw)
        full = oracle.qk_norm_rope_fwd_bwd(q_all, None, w, None, gq, None, None, inv, 1e-6)
        ok_dw = torch.allclose(dw, full["dwq"], atol=1e-10)
        ok_out = torch.equal(r["q_out"], full["q_out"][shard])
        slowest = bench.max_over_ranks(1.0 + rank, dist, torch.device("cpu"))
        q.put((rank, ok_dw, ok_out, slowest))
    finally:
        dist.destroy_process_group()


def test_row_shards_and_max_over_ranks():
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker_shards, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs)
    for rank, ok_dw, ok_out, slowest in res:
        assert ok_dw and ok_out, rank
        assert slowest == 2.0


def _worker_failure(rank, world, port, q):
    _init(rank, world, port, timeout_s=5)
    if rank == 1:
        raise SystemExit(3)  # a rank dies before the step's barrier
    t0 = time.time()
    try:
        dist.barrier()
        q.put(("no error", time.time() - t0))
    except Exception as e:  # noqa: BLE001 - any error is the expected outcome
        q.put((type(e).__name__, time.time() - t0))


def test_dead_rank_is_an_error_not_a_hang():
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker_failure, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    kind, waited = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert kind != "no error"
    assert waited < 60


def test_local_batch():
    assert bench.local_batch(8, 4, "weak") == 8
    assert bench.local_batch(8, 4, "strong") == 2
    with pytest.raises(ValueError):
        bench.local_batch(8, 3, "strong")
