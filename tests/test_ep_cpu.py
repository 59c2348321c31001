"""Expert parallelism on the CPU: the ownership and the exchange layout of
walsh_research_b200.ep with gloo ranks (world 2 and 4, 127.0.0.1), through
the all-to-all transport and a numpy evaluation of the experts, against the
single-process MoE of the oracle; and a rank that never joins the exchange,
which must end the others' exchange with an error instead of a hang."""
import datetime
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_ownership_covers_every_expert_once():
    from walsh_research_b200.ep import owned_experts
    for world in (1, 2, 4, 8, 16):
        seen = []
        for r in range(world):
            first, n = owned_experts(r, world, 16)
            seen += list(range(first, first + n))
        assert seen == list(range(16))
    with pytest.raises(ValueError):
        owned_experts(0, 3, 16)


def _case(T, C=512, seed=0):
    from oracle import walsh_oracle as O
    rng = np.random.default_rng(seed)
    E = C // 32
    p = {"router.gate.0.weight": rng.normal(0, 0.05, (C // 4, C)),
         "router.gate.2.weight": rng.normal(0, 0.5, (E, C // 4)),
         "experts.gate_weights": rng.integers(-1, 2, (E, 128, 32)).astype(np.float64),
         "experts.up_weights": rng.integers(-1, 2, (E, 128, 32)).astype(np.float64),
         "experts.down_weights": rng.integers(-1, 2, (E, 32, 128)).astype(np.float64)}
    return O, p


def _worker(rank, world, port, T, out, stall_rank):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=8))
    try:
        from walsh_research_b200.ep import ExpertParallel
        O, p = _case(T)
        rng = np.random.default_rng(100 + rank)
        u = rng.normal(size=(T, 512))
        w, mask, _ = O.router(u, p["router.gate.0.weight"], p["router.gate.2.weight"], 6)
        ep = ExpertParallel(max_tokens=T, C=512, dtype=torch.float64, transport="nccl", device="cpu")

        def experts_fn(rows, wrows, first, count, outb):
            r = rows.numpy().reshape(-1, 16, 32)
            wr = wrows.numpy()
            keep = np.zeros(16)
            keep[first:first + count] = 1.0
            y = O.experts(r, wr * keep, p["experts.gate_weights"], p["experts.up_weights"],
                          p["experts.down_weights"])
            outb.copy_(torch.from_numpy(y.reshape(outb.shape)))

        if rank == stall_rank:
            out.put((rank, "stalled", None))
            dist.barrier()  # never matched: the others are in the exchange
            return
        try:
            y = ep.moe(torch.from_numpy(u), torch.from_numpy(w), experts_fn).numpy().copy()
        except RuntimeError as e:
            out.put((rank, "error", str(e)[:200]))
            return
        want = O.experts(u.reshape(T, 16, 32), w, p["experts.gate_weights"], p["experts.up_weights"],
                         p["experts.down_weights"]).reshape(T, 512)
        out.put((rank, "ok", float(np.abs(y - want).max() / np.abs(want).max())))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, T, stall_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, T, q, stall_rank)) for r in range(world)]
    for pr in procs:
        pr.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for pr in procs:
        pr.join(timeout=60)
        if pr.is_alive():
            pr.kill()
    return sorted(res)


@pytest.mark.parametrize("world", [2, 4])
def test_exchange_equals_single_process_moe(world):
    res = _run(world, T=7)
    for rank, status, err in res:
        assert status == "ok", (rank, err)
        assert err < 1e-6  # the exchange carries routing weights as float32


def test_a_rank_that_never_joins_ends_the_exchange_with_an_error():
    res = _run(2, T=5, stall_rank=1)
    assert res[1][1] == "stalled"
    assert res[0][1] == "error"
