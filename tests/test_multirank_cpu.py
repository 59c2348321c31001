"""The multi-GPU host path of bench.py on CPU: two gloo ranks (world size 2,
127.0.0.1 rendezvous) exercise the max-over-ranks timing reduction, the
per-rank batch seeding of the batch-sharded replicas, and the reference arm's
rank-0-only output.  No GPU is involved."""
import json
import os
import socket
import subprocess
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    import bench
    ms = bench.max_over_ranks(10.0 + 5.0 * rank, dist, torch.device("cpu"))
    ids = bench.token_ids(2, 8, seed=bench.rank_token_seed(1, rank))
    gathered = [torch.zeros_like(ids) for _ in range(world)]
    dist.all_gather(gathered, ids)
    out.put((rank, ms, [g.tolist() for g in gathered]))
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_reduce_max_and_draw_distinct_batches():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ms, gathered in res:
        assert ms == 15.0                     # the slowest rank's time, on every rank
        assert gathered[0] != gathered[1]     # each replica processes its own batch


def test_single_process_needs_no_collective():
    sys.path.insert(0, ROOT)
    import bench
    assert bench.max_over_ranks(3.5, None, torch.device("cpu")) == 3.5


def test_reference_arm_prints_on_rank_zero_only(tmp_path):
    """Under torchrun only rank 0 runs the CPU reference arm; other ranks exit 0."""
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "0"], env=env, capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert r.returncode == 0
    assert r.stdout.strip() == ""
