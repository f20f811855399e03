"""GPU (two or more devices): the optional all-gather of output shards.

Two ranks, one process and one GPU each, run the config-2 operator on their
own rows (mcb_shard_plan_v1 "rows") and gather Y with mcb_allgather_v1; every
rank must then hold the bytes the whole GEMM gives on one GPU. Runs as child
processes with a bounded wait; skipped on a box with fewer than two GPUs."""
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
    # Rank 0 makes the id (its process hosts NCCL's bootstrap root) and hands
    # it to the other rank through a file; the wait for it is bounded.
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
    g = torch.Generator(device="cuda"); g.manual_seed(7)
    M, K, N = 1024, 512, 768
    x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(K, N, device="cuda", generator=g) / 32).to(torch.bfloat16)
    b = (torch.randn(N, device="cuda", generator=g) * 0.1).to(torch.bfloat16)
    begin, count, _, _ = mcb.shard_plan("rows", M, world, rank, align=128)
    assert count == M // world
    comm = mcb.Comm(uid, world, rank, rank)
    full = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    mine = full[begin:begin + count]
    mcb.gemm_epilogue(x[begin:begin + count], w, b, act="gelu_tanh", out=mine)
    comm.allgather(mine, full)          # in place: this rank's slot of full
    ref = mcb.gemm_epilogue(x, w, b, act="gelu_tanh")
    torch.cuda.synchronize()
    comm.close()
    assert torch.equal(full, ref), "gathered Y differs from the one-GPU result"
    print("rank", rank, "ok")
''')


def test_two_rank_row_shards_allgather(mcb, tmp_path):
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
