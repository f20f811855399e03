"""CPU: the multi-GPU host logic with world_size-2 gloo ranks (no GPU).

* Every rank derives its shard from mcb_shard_plan_v1; gathered over ranks the
  shards tile the work exactly once (rows, (b,h) units, tokens with the K/V
  range of their batch element).
* The optional output reassembly (an all-gather of row shards) rebuilds the
  full output.
* Failure detection: a rank that leaves early makes the surviving rank's next
  collective fail within the process group's short timeout instead of hanging.
"""
import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def _plan_worker(rank, world, port, q):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch
    import matcoredsl_b200 as mcb
    dist = _init(rank, world, port)
    plans = {
        "rows": mcb.shard_plan("rows", 8192 * world, world, rank, align=128),
        "rows_strong": mcb.shard_plan("rows", 8192, world, rank, align=128),
        "units": mcb.shard_plan("units", 8 * 32, world, rank),
        "tokens": mcb.shard_plan("tokens", 4 * 2048, world, rank, group=2048, align=128),
    }
    gathered = [None] * world
    dist.all_gather_object(gathered, plans)
    # optional output reassembly: each rank holds its row shard of Y
    b, c, _, _ = plans["rows_strong"]
    local = torch.arange(b, b + c, dtype=torch.float32).unsqueeze(1).repeat(1, 4)
    full = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(full, local)
    y = torch.cat(full)
    if rank == 0:
        q.put((gathered, bool(torch.equal(y[:, 0], torch.arange(8192, dtype=torch.float32)))))
    dist.barrier()
    dist.destroy_process_group()


def _get(q, procs, timeout=120):
    """Queue result, failing fast if a worker died before producing one."""
    import queue
    import time
    t0 = time.time()
    while time.time() - t0 < timeout:
        try:
            return q.get(timeout=1)
        except queue.Empty:
            if all(p.exitcode not in (None, 0) for p in procs if p.exitcode is not None) and \
                    any(p.exitcode not in (None, 0) for p in procs):
                raise AssertionError(f"worker failed: {[p.exitcode for p in procs]}")
    raise AssertionError("timed out waiting for workers")


def _covers(shards, total):
    seen = 0
    for b, c, *_ in sorted(shards):
        if b != seen:
            return False
        seen = b + c
    return seen == total


def test_shard_plans_tile_the_work_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_plan_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    gathered, reassembled = _get(q, procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert reassembled
    assert _covers([g["rows"] for g in gathered], 16384)
    assert all(g["rows"][1] == 8192 for g in gathered)  # weak scaling: fixed per rank
    assert _covers([g["rows_strong"] for g in gathered], 8192)
    assert _covers([g["units"] for g in gathered], 256)
    assert _covers([g["tokens"] for g in gathered], 8192)
    for g in gathered:  # two whole batch elements each: K/V range == token range
        b, c, kb, kc = g["tokens"]
        assert (kb, kc) == (b, c) and c == 4096


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_token_plan_kv_ranges(mcb, world):
    shards = [mcb.shard_plan("tokens", 4 * 2048, world, r, group=2048, align=128)
              for r in range(world)]
    assert _covers(shards, 8192)
    for b, c, kb, kc in shards:
        assert kb <= b and b + c <= kb + kc  # owns tokens inside the K/V range it computes
        assert kb % 2048 == 0 and kc % 2048 == 0
        if world == 8:
            assert c == 1024 and kc == 2048  # 2 GPUs per batch element, redundant K/V


@pytest.mark.parametrize("world", [1, 3, 8, 148])
def test_row_plan_balanced(mcb, world):
    shards = [mcb.shard_plan("rows", 8192, world, r, align=128) for r in range(world)]
    assert _covers(shards, 8192)
    counts = [c for _, c, _, _ in shards]
    assert max(counts) - min(counts) <= 128
    assert all(b % 128 == 0 for b, _, _, _ in shards)


def test_invalid_plans_rejected(mcb):
    with pytest.raises(mcb.McbError):
        mcb.shard_plan("tokens", 4 * 2048, 3, 0, group=2048)  # 3 ranks cannot split 4 batches
    with pytest.raises(mcb.McbError):
        mcb.shard_plan("rows", 100, 2, 2)


def _dropout_worker(rank, world, port, q):
    import time
    dist = _init(rank, world, port, timeout_s=5)
    dist.barrier()
    if rank == 1:
        dist.destroy_process_group()  # leaves between steps, nothing in flight
        return
    t0 = time.time()
    try:
        dist.barrier()  # rank 1 never joins this one
        q.put(("no-error", time.time() - t0))
    except Exception as e:  # the short process-group timeout ends the wait
        q.put((type(e).__name__, time.time() - t0))


def test_rank_dropout_detected_by_timeout():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dropout_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    kind, waited = _get(q, procs)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert kind != "no-error"
    assert waited < 60
