"""GPU (two or more devices): the head-sharded attention block.

Two ranks, one process and one GPU each, hold one head group each of the
attention-residual block (BASELINE config 5's batch x heads sharding, for a
batch that does not split over the GPUs): mcb_attn_block_heads_v1 computes
each rank's partial output projection, mcb_reduce_scatter_v1 sums the two
partials and leaves each rank half of the rows, and mcb_residual_rmsnorm_v1
finishes those rows. The result must match the one-GPU region within the
bf16 bar (1e-2 relative Frobenius error); the reduce-scatter alone must sum
f32 exactly. The same block then runs three times with the exchange fused
into the output projection (mcb_attn_block_heads_pair_v1: each GPU's GEMM
stores the other GPU's rows into that GPU's receive buffer and raises a
counter there) and must match as well. Child processes with bounded waits; skipped on a box with fewer
than two GPUs."""
import os
import subprocess
import sys
import textwrap

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = textwrap.dedent(r'''
    import os, sys, time, torch
    sys.path.insert(0, sys.argv[1])
    import matcoredsl_b200 as mcb
    rank, world, id_file = int(sys.argv[2]), int(sys.argv[3]), sys.argv[4]
    torch.cuda.set_device(rank)
    if rank == 0:
        uid = mcb.Comm.unique_id()
        with open(id_file + ".tmp", "wb") as f:
            f.write(uid)
        os.replace(id_file + ".tmp", id_file)
    else:
        t0 = time.time()
        while not os.path.exists(id_file):
            assert time.time() - t0 < 60, "no communicator id from rank 0"
            time.sleep(0.05)
        uid = open(id_file, "rb").read()
    comm = mcb.Comm(uid, world, rank, rank)
    # reduce-scatter alone: integer-valued f32, so the sum is exact
    send = torch.arange(world * 1024, device="cuda", dtype=torch.float32) * (rank + 1)
    recv = torch.empty(1024, device="cuda", dtype=torch.float32)
    comm.reduce_scatter(send, recv)
    base = torch.arange(rank * 1024, (rank + 1) * 1024, device="cuda", dtype=torch.float32)
    assert torch.equal(recv, base * sum(r + 1 for r in range(world))), "reduce-scatter sum"
    # the head-sharded block: batch 1, seq 512, d_model 1024, 8 heads of 128
    g = torch.Generator(device="cuda"); g.manual_seed(41)
    S, D, H = 512, 1024, 8
    x = torch.randn(1, S, D, device="cuda", generator=g).to(torch.bfloat16)
    ws = [(torch.randn(D, D, device="cuda", generator=g) / D ** 0.5).to(torch.bfloat16)
          for _ in range(4)]
    dh = D // world
    cols = slice(rank * dh, (rank + 1) * dh)
    p = mcb.attn_block_heads(x, *[w[:, cols].contiguous() for w in ws[:3]],
                             ws[3][cols, :].contiguous(), H // world)
    rows = S // world
    mine = torch.empty(1, rows, D, device="cuda", dtype=torch.bfloat16)
    comm.reduce_scatter(p, mine)
    y = mcb.residual_rmsnorm(x[:, rank * rows:(rank + 1) * rows], mine, 1e-6)
    ref = mcb.attn_block(x, *ws, H, 1e-6)[:, rank * rows:(rank + 1) * rows]
    torch.cuda.synchronize()
    comm.close()
    err = ((y.float() - ref.float()).norm() / ref.float().norm()).item()
    assert err < 1e-2, err

    # the same block with the exchange fused into the output projection:
    # this GPU's GEMM stores the other GPU's rows into its receive buffer
    def swap(tag, data):
        mine_f = f"{id_file}.{tag}{rank}"
        with open(mine_f + ".tmp", "wb") as f:
            f.write(data)
        os.replace(mine_f + ".tmp", mine_f)
        other = f"{id_file}.{tag}{1 - rank}"
        t0 = time.time()
        while not os.path.exists(other):
            assert time.time() - t0 < 60, "no " + tag + " from the other rank"
            time.sleep(0.02)
        return open(other, "rb").read()
    xch = mcb.PeerExchange(rank, rows * D * 2)
    xch.connect(swap("h", xch.handle))
    for it in range(3):  # three steps: the counters and the buffer are reused
        y2 = mcb.attn_block_heads_pair(x, *[w[:, cols].contiguous() for w in ws[:3]],
                                       ws[3][cols, :].contiguous(), H // world, 1e-6, rank, xch)
        assert mcb.api.last_result.route == "attn_block_heads_pair_p2p"
        torch.cuda.synchronize()
        err2 = ((y2.float() - ref.reshape(rows, D).float()).norm() / ref.float().norm()).item()
        assert err2 < 1e-2, (it, err2)
        diff = ((y2.float() - y.reshape(rows, D).float()).norm() / ref.float().norm()).item()
        assert diff < 1e-2, (it, diff)
    assert mcb.device_status(rank) == 0
    swap("done", b"1")  # neither side frees its buffer while the other may still write it
    xch.close()
    print("rank", rank, "ok", err, err2)
''')


def test_two_rank_head_sharded_block(mcb, tmp_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    id_file = str(tmp_path / "comm_id")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", NCCL_DEBUG="WARN")
    procs = [subprocess.Popen([sys.executable, "-c", CHILD, ROOT, str(r), "2", id_file], env=env,
                              stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
             for r in range(2)]
    outs = []
    try:
        for p in procs:
            outs.append(p.communicate(timeout=240)[0])
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
    for r, (p, out) in enumerate(zip(procs, outs)):
        assert p.returncode == 0, f"rank {r} failed:\n{out[-3000:]}"
        assert f"rank {r} ok" in out
