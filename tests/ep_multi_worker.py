"""One rank of the multi-GPU expert-parallel check, launched by
tests/test_gpu_ep_multi.py through torch.distributed.run (one process per
GPU, 127.0.0.1).  Each rank builds the same config-3 MoE layer, its own
tokens, and compares the ffn site evaluated expert-parallel (NVLink exchange
and the NCCL fallback) with the replicated evaluation of the same tokens;
then times both.  Prints one JSON line per rank."""
import datetime
import json
import os
import sys
import time

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def replicated(u, x, hmix, ff):
    from walsh_research_b200 import _lib, ops
    T = u.numel() // 512
    tc = ff.kernel_args(torch.float16)[7]
    gam = ff.experts.packed()[3]
    mask = torch.empty((T, 16), dtype=torch.uint8, device=u.device)
    probs = torch.empty((T, 16), dtype=torch.float32, device=u.device)
    w = torch.empty((T, 16), dtype=torch.float32, device=u.device)
    _lib.call("walsh_moe_router_tc_fwd", u.data_ptr(), _lib.dcode(u.dtype), T, tc[0].data_ptr(), tc[1].data_ptr(),
              ff.router.top_k, mask.data_ptr(), probs.data_ptr(), w.data_ptr(), None, _lib.stream())
    y = torch.empty_like(u)
    _lib.call("walsh_moe_experts_tc_fwd", u.data_ptr(), _lib.dcode(u.dtype), T, w.data_ptr(), tc[5].data_ptr(),
              tc[4].data_ptr(), gam.data_ptr(), y.data_ptr(), 0, None, _lib.dcode(u.dtype), None, None, _lib.stream())
    ops.mhc_post(x, y, hmix, out=x)
    return mask


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    import bench
    from walsh_research_b200.ep import ExpertParallel, moe_site
    ff = bench.build_model_cpu().layers[0].feed_forward.to(dev).eval()
    T = int(os.environ.get("EP_TOKENS", "10000"))
    g = torch.Generator(device="cpu").manual_seed(1000 + rank)
    u = torch.randn((1, T, 512), generator=g).to(dev, torch.float16)
    x0 = torch.randn((1, T, 4, 512), generator=g).to(dev, torch.float16)
    hmix = torch.rand((1, T, 24), generator=g).to(dev)
    out = {"rank": rank, "world": world, "tokens": T}
    with torch.no_grad():
        x_rep = x0.clone()
        m_rep = replicated(u, x_rep, hmix, ff)
        for transport in ("nvlink", "nccl"):
            ep = ExpertParallel(max_tokens=T, C=512, dtype=torch.float16, transport=transport)
            x_ep = x0.clone()
            m_ep, _ = moe_site(u, x_ep, hmix, ff, ep)
            torch.cuda.synchronize()
            ep.check()
            out[f"{transport}_equal"] = bool(torch.equal(x_ep, x_rep) and torch.equal(m_ep, m_rep))
            out[f"{transport}_maxdiff"] = float((x_ep.float() - x_rep.float()).abs().max())
            # timing: 20 sites back to back, CUDA events, max over ranks
            for _ in range(3):
                moe_site(u, x_ep, hmix, ff, ep)
            torch.cuda.synchronize()
            dist.barrier()
            s, e = torch.cuda.Event(True), torch.cuda.Event(True)
            s.record()
            for _ in range(20):
                moe_site(u, x_ep, hmix, ff, ep)
            e.record()
            torch.cuda.synchronize()
            ep.check()
            t = torch.tensor([s.elapsed_time(e) / 20], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            out[f"{transport}_us"] = float(t.item()) * 1e3
            ep.close()
        for _ in range(3):
            replicated(u, x_rep, hmix, ff)
        torch.cuda.synchronize()
        dist.barrier()
        s, e = torch.cuda.Event(True), torch.cuda.Event(True)
        s.record()
        for _ in range(20):
            replicated(u, x_rep, hmix, ff)
        e.record()
        torch.cuda.synchronize()
        t = torch.tensor([s.elapsed_time(e) / 20], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        out["replicated_us"] = float(t.item()) * 1e3
    out_dir = os.environ.get("EP_OUT_DIR")
    if out_dir:
        with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
            json.dump(out, f)
    print(json.dumps(out), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
