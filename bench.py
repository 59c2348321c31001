"""Benchmark: Walsh-512 prefill tokens/s on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl walsh|reference]

Workload (per rank, weak scaling): mHCWalsh Walsh-512 (L16, H32, C512, 16
experts top-6, channel modulation, 4 mHC streams, vocab 50257), bf16
activations, batch 64 x seq 1024 random token ids, seeded random weights with
ternary latents and router logits scaled to ~N(0, 1).  One step = one full
prefill forward (last-position logits).  The per-layer stream state
(64*1024*4*512 bf16 = 268 MB) exceeds the 126 MB L2, so no flush is needed
between steps.

Prints one JSON line (rank 0).  `value` times graph replays of the forward
with inputs resident in HBM; `e2e` times the public ``mHCWalsh.forward`` call
with the token ids copied from pinned host memory and the logits copied back
every step.  `--impl reference` times the reference's own PyTorch forward
(its src/model package, installed unmodified under baseline/_ref) on the host
cores, one B1xT1024 slice of the same workload per step in bf16 autocast; when
that install is absent it times the numpy oracle port instead and says so.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import select
import statistics
import subprocess
import sys
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIG = dict(block_size=1024, vocab_size=50257, n_layer=16, n_head=32, n_embd=512, dropout=0.0, bias=False,
              head_mixing=True, algebra="hadamard", hash_embeddings=False, use_moe=True, moe_threshold=0.1,
              moe_min_experts=1, moe_max_experts=6, use_channel_mod=True)
N_STREAMS = 4
BATCH, SEQ = 64, 1024
ROUTER_SCALE = 18.3
METRIC = "Walsh-512 prefill tokens/s"
UNIT = "tokens/s"
CPU_SAMPLE = (1, 1024)  # oracle sample per step: B1 x T1024
DECODE_BATCH, DECODE_CTX = 256, 1024
ATTN_TRAFFIC_B64 = 246.10e6  # ncu DRAM bytes of one prefill attention launch at B64 x T1024


def max_over_ranks(value: float, dist, device) -> float:
    """The largest per-rank value (step times are reported as the slowest
    rank's); `dist` is torch.distributed or None for a single process."""
    if not dist:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def rank_token_seed(base: int, rank: int) -> int:
    """Each rank draws its own batch (weak scaling: batch-sharded replicas)."""
    return base + rank


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


def build_model_cpu(seed=0):
    """The seeded recipe: package init, ternary latents i.i.d. uniform {-1,0,1},
    router output layer scaled so router logits are ~N(0,1)."""
    from walsh_research_b200.model import WalshConfig, mHCWalsh
    torch.manual_seed(seed)
    model = mHCWalsh(WalshConfig(**CONFIG), n_streams=N_STREAMS).eval()
    g = torch.Generator().manual_seed(seed)
    pat = re.compile(r"\.inner\.weight$|experts\.(gate|up|down)_weights$|channel_mod\.context_mlp\.\d\.weight$")
    with torch.no_grad():
        for name, p in sorted(model.named_parameters()):
            if pat.search(name):
                p.copy_(torch.randint(-1, 2, p.shape, generator=g).float())
        for layer in model.layers:
            layer.feed_forward.router.gate[2].weight.mul_(ROUTER_SCALE)
    return model


OCTO_CONFIG = dict(CONFIG, algebra="octonion", use_moe=False)
OCTO_BATCH = 32


def build_octonion_cpu(seed=0):
    """Config 2: the same recipe on the octonion variant (SwiGLU FFN, no MoE)."""
    from walsh_research_b200.model import WalshConfig, mHCWalsh
    torch.manual_seed(seed)
    model = mHCWalsh(WalshConfig(**OCTO_CONFIG), n_streams=N_STREAMS).eval()
    g = torch.Generator().manual_seed(seed)
    pat = re.compile(r"attention\.w[qkvo]\.weight$|feed_forward\.(gate|up|down)_proj\.weight$|"
                     r"channel_mod\.context_mlp\.\d\.weight$")
    with torch.no_grad():
        for name, p in sorted(model.named_parameters()):
            if pat.search(name):
                p.copy_(torch.randint(-1, 2, p.shape, generator=g).float())
    return model


def token_ids(B, T, seed=1):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, CONFIG["vocab_size"], (B, T), generator=g)


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------

CLOCK_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


class ClockSampler:
    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        # a sample every 20 ms; the timed region starts once the first sample
        # has arrived (at most 5 s of waiting).  That first sample only signals
        # that the sampler runs: it was taken before the timed region and is
        # dropped, so the kept samples fall inside it
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={CLOCK_FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "20"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        if self.proc is not None:
            try:
                ready, _, _ = select.select([self.proc.stdout], [], [], 5.0)
                if ready:
                    self.proc.stdout.readline()
            except (OSError, ValueError):
                pass
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in self.lines:
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# reference arm / CPU baseline: the reference's own PyTorch forward on the host
# cores (its src/model package, installed unmodified under baseline/_ref);
# the numpy oracle port stands in only when that install is absent
# ---------------------------------------------------------------------------

REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def reference_model_cpu():
    """The reference's mHCWalsh (src/model/mhc.py:538-681) built from its own
    package with this bench's seeded weights loaded through its
    ``load_state_dict`` (the state-dict layouts are identical).  Returns
    (model, None), or (None, reason) when the reference cannot be imported."""
    if not os.path.isdir(os.path.join(REF_DIR, "src", "model")):
        return None, "reference package not installed under baseline/_ref"
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    try:
        from src.model import WalshConfig as RefConfig, mHCWalsh as RefWalsh
    except Exception as e:  # noqa: BLE001 - any import failure means: use the port
        return None, f"reference import failed: {type(e).__name__}: {e}"
    ours = build_model_cpu()
    torch.manual_seed(0)
    ref = RefWalsh(RefConfig(**CONFIG), n_streams=N_STREAMS).eval()
    ref.load_state_dict(ours.state_dict(), strict=True)
    return ref, None


def cpu_model_name():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def time_reference_torch(ref, steps, warmup):
    """Mean seconds of one B1xT1024 forward of the reference on the host cores
    (bf16 autocast, the config's dtype; every host thread)."""
    torch.set_num_threads(os.cpu_count() or 1)
    B, T = CPU_SAMPLE
    idx = token_ids(B, T, seed=2)
    times = []
    with torch.no_grad(), torch.autocast("cpu", dtype=torch.bfloat16):
        for _ in range(warmup):
            ref(idx)
        for _ in range(steps):
            t0 = time.perf_counter()
            ref(idx)
            times.append(time.perf_counter() - t0)
    sec = sum(times) / len(times)
    return B * T / sec, sec


def oracle_inputs():
    model = build_model_cpu()
    sd = {k: v.detach().float().numpy() for k, v in model.state_dict().items()
          if k != "freqs_cis" and not k.endswith(".H")}
    return sd


def time_oracle(sd, steps, warmup):
    from oracle import walsh_oracle as O
    B, T = CPU_SAMPLE
    idx = token_ids(B, T, seed=2).numpy()
    for _ in range(warmup):
        O.mhc_walsh_forward(CONFIG, sd, idx, N_STREAMS, dtype=np.float32)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        O.mhc_walsh_forward(CONFIG, sd, idx, N_STREAMS, dtype=np.float32)
        times.append(time.perf_counter() - t0)
    sec = sum(times) / len(times)
    return B * T / sec, sec


def cpu_threads():
    try:
        import threadpoolctl
        info = threadpoolctl.threadpool_info()
        return max([i.get("num_threads", 1) for i in info] or [os.cpu_count()])
    except Exception:
        return os.cpu_count()


def cpu_baseline(steps, warmup):
    """The CPU leg: the reference's PyTorch forward when installed (kind
    "reference"), else the numpy oracle port (kind "port").  Returns the
    cpu_baseline object, the seconds per step and the dtype label."""
    B, T = CPU_SAMPLE
    ref, why = reference_model_cpu()
    if ref is not None:
        value, sec = time_reference_torch(ref, steps, warmup)
        return ({"value": value, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "reference",
                 "sample": f"one B{B}xT{T} forward per step of the reference's own mHCWalsh (src/model, "
                           f"PyTorch on the host CPU, bf16 autocast) with the same architecture and weights",
                 "cpu": cpu_model_name()}, sec, "bf16 (CPU autocast)")
    value, sec = time_oracle(oracle_inputs(), steps, warmup)
    return ({"value": value, "unit": UNIT, "cores": cpu_threads(), "kind": "port",
             "sample": f"numpy oracle float32, one B{B}xT{T} forward per step (same architecture and weights)",
             "cpu": cpu_model_name(), "why_port": why}, sec, "f32")


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cpu, sec, dtype = cpu_baseline(args.steps, args.warmup)
    value = cpu["value"]
    B, T = CPU_SAMPLE
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": dtype, "data": "synthetic",
            "config": {"workload": f"Walsh-512 mHC+MoE+chmod prefill (config 3 architecture), sample B{B}xT{T}",
                       "global_batch": B, "seq_len": T},
            "cpu_baseline": cpu,
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# the B200 arm
# ---------------------------------------------------------------------------

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="walsh", choices=["walsh", "reference"])
    ap.add_argument("--batch", type=int, default=BATCH)
    ap.add_argument("--ctx", type=int, default=DECODE_CTX,
                    help="KV-cache length of --profile decode (a short cache keeps ncu captures small)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decode", action="store_true", help="skip the decode measurement")
    ap.add_argument("--no-octonion", action="store_true", help="skip the config-2 octonion measurement")
    ap.add_argument("--no-micro", action="store_true", help="skip the config-1 HadamardLinear microbenchmark")
    ap.add_argument("--no-2048", action="store_true", help="skip the config-4 Walsh-2048 decode measurement")
    ap.add_argument("--ep", action="store_true",
                    help="with N > 1: also time the prefill with expert-parallel MoE layers (NVLink exchange)")
    ap.add_argument("--profile", nargs="?", const="prefill", choices=["prefill", "decode", "octonion", "decode2048", "hlin"],
                    help="run one warm-up and one eager forward only (for ncu launch lists)")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.profile:
        return run_profile(args)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    from walsh_research_b200 import ops
    from walsh_research_b200.model.mhc import MAP_EPS, site_params

    B, T = args.batch, SEQ
    model = build_model_cpu().to(dev).eval()
    model.compute_dtype = torch.bfloat16
    idx_host = token_ids(B, T, seed=rank_token_seed(1, rank)).pin_memory()
    idx = idx_host.to(dev)

    # graph-captured forward: inputs resident in HBM
    with torch.no_grad():
        for _ in range(2):
            model(idx)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        from walsh_research_b200 import _lib
        n0 = _lib.launch_count
        with torch.cuda.graph(graph):
            logits_g, _ = model(idx)
        launches_per_forward = _lib.launch_count - n0
        for _ in range(args.warmup):
            graph.replay()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clk:
            torch.cuda.synchronize()
            start.record()
            for _ in range(args.steps):
                graph.replay()
            end.record()
            torch.cuda.synchronize()
        ms = start.elapsed_time(end) / args.steps
        ms = max_over_ranks(ms, dist, dev)
        value = world * B * T / (ms / 1e3)

        # end to end through the public API: H2D ids, forward, D2H logits; once
        # with the model's own CUDA-graph replay (mHCWalsh.enable_cuda_graphs:
        # the serving mode, one host launch per forward) and once eagerly (one
        # host call per kernel, bound by the host when its cores are busy)
        logits_host = torch.empty((B, 1, CONFIG["vocab_size"]), dtype=torch.float32).pin_memory()
        e_steps = max(3, args.steps)

        def time_e2e():
            for _ in range(3):
                idx_w = idx_host.to(dev, non_blocking=True)
                lg, _ = model(idx_w)
                logits_host.copy_(lg, non_blocking=True)
            torch.cuda.synchronize()
            if dist:
                dist.barrier()
            start.record()
            for _ in range(e_steps):
                idx_dev = idx_host.to(dev, non_blocking=True)
                lg, _ = model(idx_dev)
                logits_host.copy_(lg, non_blocking=True)
            end.record()
            torch.cuda.synchronize()
            return max_over_ranks(start.elapsed_time(end) / e_steps, dist, dev)
        e_ms_eager = time_e2e()
        model.enable_cuda_graphs()
        e_ms = time_e2e()
        model.enable_cuda_graphs(False)
        e2e = {"value": world * B * T / (e_ms / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": idx_host.numel() * idx_host.element_size(),
               "d2h_bytes_per_step": logits_host.numel() * logits_host.element_size(),
               "mode": "mHCWalsh.forward with enable_cuda_graphs()",
               "eager_value": world * B * T / (e_ms_eager / 1e3)}

        # dominant kernel timed alone with CUDA events on the launching stream:
        # prefill attention of one layer (q/k/v of layer 0 recomputed in place)
        roof = dominant_kernel_roofline(model, idx, B, T, dev)
    del graph, logits_g
    torch.cuda.empty_cache()
    ep_line = measure_prefill_ep(model, idx, B, T, dev, args.steps, max(3, args.warmup), world, dist) \
        if (args.ep and world > 1) else None
    decode = None if args.no_decode else measure_decode(model, dev, args.steps, max(3, args.warmup), rank, world, dist)
    octo = None if args.no_octonion else measure_octonion(dev, args.steps, max(3, args.warmup), rank, world, dist)
    micro = None if args.no_micro else measure_hlin_microbench(dev)
    d2048 = None if args.no_2048 else measure_decode_2048(dev, args.steps, max(3, args.warmup), rank, world, dist)

    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu, _, _ = cpu_baseline(steps=3, warmup=1)
    hbm, tflops, src = peaks()
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16 operands, f32 accumulate (16-bit mode)", "data": "synthetic",
            "config": {"workload": "config 3: Walsh-512 mHC+MoE(16e top-6)+chmod prefill", "global_batch": world * B,
                       "batch_per_gpu": B, "seq_len": T, "parallelism": f"replicas x{world} (batch-sharded)",
                       "l2": "working set > L2 (stream state 268 MB per layer), no flush"},
            "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "clocks": clk.summary(), "decode": decode,
            "octonion": octo, "hlin_microbench": micro, "decode_2048": d2048, "prefill_ep": ep_line,
            "gpu_launches": launches_per_forward * args.steps,
            "peaks": src}
    print(json.dumps(line), flush=True)


def measure_prefill_ep(model, idx, B, T, dev, steps, warmup, world, dist):
    """Config-3 prefill with every MoE layer expert-parallel (each rank owns
    16 / N experts and evaluates them for every rank's tokens, through the
    NVLink exchange kernels), against the same eager forward with replicated
    experts; CUDA events, max over ranks.  Eager (no graph): the exchange
    epochs are host arguments."""
    from walsh_research_b200.ep import ExpertParallel
    ep = ExpertParallel(max_tokens=B * T, C=CONFIG["n_embd"], dtype=torch.float16, transport="nvlink")
    out = {}
    with torch.no_grad():
        for mode in ("replicated", "expert_parallel"):
            model.enable_expert_parallel(ep if mode == "expert_parallel" else None)
            for _ in range(warmup):
                model(idx)
            torch.cuda.synchronize()
            dist.barrier()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(steps):
                model(idx)
            e.record()
            torch.cuda.synchronize()
            ms = max_over_ranks(s.elapsed_time(e) / steps, dist, dev)
            out[mode] = {"value": world * B * T / (ms / 1e3), "unit": UNIT, "ms_per_step": ms}
        ep.check()
        model.enable_expert_parallel(None)
    ep.close()
    out["config"] = {"experts_per_rank": 16 // world, "transport": "NVLink exchange kernels", "mode": "eager"}
    return out


def run_profile(args):
    """One warm-up forward then one profiled forward, eager (no graph)."""
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    if args.profile == "hlin":
        # config 1: HadamardLinear(n, n), n = 512 then 2048, over 65536 bf16
        # tokens (16384 for n = 2048 with --batch below 64), three calls each
        from walsh_research_b200.model.fht_cuda import HadamardLinear
        g = torch.Generator().manual_seed(0)
        for n in (512, 2048):
            lin = HadamardLinear(n, n)
            with torch.no_grad():
                lin.weight.copy_(torch.randint(-1, 2, lin.weight.shape, generator=g).float())
                lin.alpha.copy_(torch.rand(lin.alpha.shape, generator=g) + 0.5)
            lin = lin.to(dev)
            ntok = 65536 if (n == 512 or args.batch >= BATCH) else 16384
            x = torch.randn((ntok, n), generator=g).to(dev, torch.bfloat16)
            with torch.no_grad():
                for _ in range(3):
                    y = lin(x)
            torch.cuda.synchronize()
            print(f"profile hlin {n} x {ntok} done", float(y.float().abs().mean()), flush=True)
            del x, y
        return
    model = build_model_cpu().to(dev).eval()
    model.compute_dtype = torch.bfloat16
    if args.profile == "decode2048":
        from walsh_research_b200.model import KVCache
        model = build_walsh2048_cpu().to(dev).eval()
        model.compute_dtype = torch.bfloat16
        B, ctx = W2048_BATCH, W2048_CTX
        H, C, L = W2048_CONFIG["n_head"], W2048_CONFIG["n_embd"], W2048_CONFIG["n_layer"]
        kv = KVCache(L, ctx, H, C // H, dev, dtype=torch.float16, batch_size=B)
        for t in kv.k_cache + kv.v_cache:
            t.normal_()
        ids = token_ids(B, 2, seed=13).to(dev)
        with torch.no_grad():
            kv.cached_len = ctx - 2
            model(ids[:, :1], kv_cache=kv, start_pos=ctx - 2)
            kv.cached_len = ctx - 1
            torch.cuda.synchronize()
            torch.cuda.nvtx.range_push("walsh_forward")
            model(ids[:, 1:], kv_cache=kv, start_pos=ctx - 1)
            torch.cuda.nvtx.range_pop()
            torch.cuda.synchronize()
        print("profile decode2048 step done", flush=True)
        return
    if args.profile == "decode":
        from walsh_research_b200.model import KVCache
        B, ctx = DECODE_BATCH, args.ctx
        H, C = CONFIG["n_head"], CONFIG["n_embd"]
        kv = KVCache(CONFIG["n_layer"], ctx, H, C // H, dev, dtype=torch.float16, batch_size=B)
        P = ctx - 2
        with torch.no_grad():
            model(token_ids(B, P, seed=3).to(dev), kv_cache=kv, start_pos=0)
            kv.increment(P)
            ids = token_ids(B, 2, seed=5).to(dev)
            model(ids[:, :1], kv_cache=kv, start_pos=P)
            kv.increment(1)
            torch.cuda.synchronize()
            torch.cuda.nvtx.range_push("walsh_forward")
            model(ids[:, 1:], kv_cache=kv, start_pos=P + 1)
            torch.cuda.nvtx.range_pop()
            torch.cuda.synchronize()
        print("profile decode step done", flush=True)
        return
    B = args.batch
    if args.profile == "octonion":
        model = build_octonion_cpu().to(dev).eval()
        model.compute_dtype = torch.bfloat16
        B = OCTO_BATCH
    idx = token_ids(B, SEQ).to(dev)
    with torch.no_grad():
        model(idx)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("walsh_forward")
        model(idx)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
    print("profile forward done", flush=True)


def measure_decode(model, dev, steps, warmup, rank=0, world=1, dist=None, B=None, ctx=None):
    """Steady-state batched decode (Walsh-512, B sequences, KV cache of ctx
    positions): the cache is prefilled to ctx - (warmup + steps) tokens, then
    each step appends one token per sequence.  Every position gets its own
    captured CUDA graph (the cache row and RoPE row are launch arguments), so
    the timed region replays the graphs of the last `steps` positions back to
    back.  The KV cache (16 layers x 2 x B x 32 x ctx x 16 fp16 = 8.6 GB at
    B256 x ctx1024) is far larger than L2.  `e2e` runs the same steps eagerly
    through the public forward with the token ids copied from pinned host
    memory and the logits copied back every step."""
    from walsh_research_b200 import _lib
    from walsh_research_b200.model import KVCache
    B = B or DECODE_BATCH
    ctx = ctx or DECODE_CTX
    H, C, L = CONFIG["n_head"], CONFIG["n_embd"], CONFIG["n_layer"]
    n = warmup + steps
    P = ctx - n
    kv = KVCache(L, ctx, H, C // H, dev, dtype=torch.float16, batch_size=B)
    prompt = token_ids(B, P, seed=rank_token_seed(3, rank)).to(dev)
    ids_host = token_ids(B, n, seed=rank_token_seed(5, rank)).pin_memory()
    ids = ids_host.to(dev)
    with torch.no_grad():
        model(prompt, kv_cache=kv, start_pos=0)
        kv.increment(P)
        model(ids[:, :1], kv_cache=kv, start_pos=P)      # eager warm-up of the decode path
        torch.cuda.synchronize()
        graphs, outs = [], []
        pool = None
        n0 = _lib.launch_count
        for i in range(n):
            kv.cached_len = P + i
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=pool):
                lg, _ = model(ids[:, i:i + 1], kv_cache=kv, start_pos=P + i)
            pool = g.pool()
            graphs.append(g)
            outs.append(lg)
        launches_per_step = (_lib.launch_count - n0) // n
        kv.cached_len = P
        for i in range(warmup):
            graphs[i].replay()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        start.record()
        for i in range(warmup, n):
            graphs[i].replay()
        end.record()
        torch.cuda.synchronize()
        ms = start.elapsed_time(end) / steps
        ms = max_over_ranks(ms, dist, dev)
        del graphs, outs

        # eager end to end through the public API
        logits_host = torch.empty((B, 1, CONFIG["vocab_size"]), dtype=torch.float32).pin_memory()
        kv.cached_len = P
        for i in range(warmup):
            lg, _ = model(ids_host[:, i:i + 1].to(dev, non_blocking=True), kv_cache=kv, start_pos=P + i)
            logits_host.copy_(lg, non_blocking=True)
            kv.increment(1)
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        start.record()
        for i in range(warmup, n):
            lg, _ = model(ids_host[:, i:i + 1].to(dev, non_blocking=True), kv_cache=kv, start_pos=P + i)
            logits_host.copy_(lg, non_blocking=True)
            kv.increment(1)
        end.record()
        torch.cuda.synchronize()
        e_ms = start.elapsed_time(end) / steps
        e_ms = max_over_ranks(e_ms, dist, dev)
    del kv
    torch.cuda.empty_cache()
    kv_bytes = L * 2 * B * H * ctx * (C // H) * 2
    return {"metric": "Walsh-512 decode tokens/s", "value": world * B / (ms / 1e3), "unit": UNIT,
            "ms_per_step": ms, "steps": steps, "warmup": warmup,
            "config": {"workload": f"Walsh-512 batched decode, B{B} per GPU, KV cache ctx {ctx} (positions "
                                   f"{P + warmup}..{ctx - 1} timed), fp16 KV cache, bf16 stream",
                       "batch_per_gpu": B, "ctx": ctx, "kv_cache_bytes": kv_bytes,
                       "l2": "KV cache 8.6 GB > L2, no flush"},
            "e2e": {"value": world * B / (e_ms / 1e3), "unit": UNIT,
                    "h2d_bytes_per_step": B * 8, "d2h_bytes_per_step": B * CONFIG["vocab_size"] * 4},
            "gpu_launches": launches_per_step * steps}


W2048_CONFIG = dict(CONFIG, block_size=2048, n_layer=24, n_head=64, n_embd=2048)
W2048_BATCH, W2048_CTX = 256, 2048


def build_walsh2048_cpu(seed=0):
    """Config 4: Walsh-2048 (L24, H64, C2048, 64 experts top-6) with the seeded
    recipe (ternary latents i.i.d. uniform {-1, 0, 1})."""
    from walsh_research_b200.model import WalshConfig, mHCWalsh
    torch.manual_seed(seed)
    model = mHCWalsh(WalshConfig(**W2048_CONFIG), n_streams=N_STREAMS).eval()
    g = torch.Generator().manual_seed(seed)
    pat = re.compile(r"\.inner\.weight$|experts\.(gate|up|down)_weights$|channel_mod\.context_mlp\.\d\.weight$")
    with torch.no_grad():
        for name, p in sorted(model.named_parameters()):
            if pat.search(name):
                p.copy_(torch.randint(-1, 2, p.shape, generator=g).float())
    return model


def measure_decode_2048(dev, steps, warmup, rank=0, world=1, dist=None):
    """Config 4: Walsh-2048 batched decode, B256 sequences at KV-cache positions
    2048 - (warmup + steps) .. 2047.  The KV cache (24 layers x 2 x 256 x 64 x
    2048 x 32 fp16 = 103 GB) is filled with seeded N(0, 1) values rather than
    by a prefill: a decode step does the same work whatever the cached values.
    One captured graph per position, as for the Walsh-512 decode line."""
    from walsh_research_b200 import _lib
    from walsh_research_b200.model import KVCache
    B, ctx = W2048_BATCH, W2048_CTX
    H, C, L = W2048_CONFIG["n_head"], W2048_CONFIG["n_embd"], W2048_CONFIG["n_layer"]
    model = build_walsh2048_cpu().to(dev).eval()
    model.compute_dtype = torch.bfloat16
    n = warmup + steps
    P = ctx - n
    kv = KVCache(L, ctx, H, C // H, dev, dtype=torch.float16, batch_size=B)
    gen = torch.Generator(device=dev).manual_seed(11 + rank)
    for t in kv.k_cache + kv.v_cache:
        t.normal_(generator=gen)
    ids = token_ids(B, n, seed=rank_token_seed(13, rank)).to(dev)
    kv.cached_len = P
    with torch.no_grad():
        model(ids[:, :1], kv_cache=kv, start_pos=P)   # eager warm-up (weight preparation)
        torch.cuda.synchronize()
        graphs, pool = [], None
        n0 = _lib.launch_count
        for i in range(n):
            kv.cached_len = P + i
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=pool):
                model(ids[:, i:i + 1], kv_cache=kv, start_pos=P + i)
            pool = g.pool()
            graphs.append(g)
        launches = (_lib.launch_count - n0) // n
        for i in range(warmup):
            graphs[i].replay()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for i in range(warmup, n):
            graphs[i].replay()
        end.record()
        torch.cuda.synchronize()
        ms = start.elapsed_time(end) / steps
        ms = max_over_ranks(ms, dist, dev)
    del graphs, kv, model
    torch.cuda.empty_cache()
    hbm, _, _ = peaks()
    kv_read = L * 2 * B * H * ctx * (C // H) * 2
    return {"metric": "Walsh-2048 decode tokens/s (config 4)", "value": world * B / (ms / 1e3), "unit": UNIT,
            "ms_per_step": ms, "steps": steps, "warmup": warmup,
            "config": {"workload": f"Walsh-2048 (L24 H64 C2048, 64 experts top-6) batched decode, B{B} per GPU, "
                                   f"KV cache ctx {ctx} filled with seeded values", "batch_per_gpu": B,
                       "ctx": ctx, "kv_cache_bytes": kv_read, "l2": "KV cache 103 GB > L2, no flush"},
            "kv_read_floor_ms": kv_read / (hbm * 1e9) * 1e3,
            "gpu_launches": launches * steps}


def measure_octonion(dev, steps, warmup, rank=0, world=1, dist=None):
    """Config 2 prefill (octonion Walsh-512, B32 x T1024 per GPU): graph
    replays of the forward with the ids resident in HBM, as for config 3."""
    from walsh_research_b200 import _lib
    model = build_octonion_cpu().to(dev).eval()
    model.compute_dtype = torch.bfloat16
    B, T = OCTO_BATCH, SEQ
    idx = token_ids(B, T, seed=rank_token_seed(7, rank)).to(dev)
    with torch.no_grad():
        for _ in range(2):
            model(idx)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        n0 = _lib.launch_count
        with torch.cuda.graph(g):
            model(idx)
        launches = _lib.launch_count - n0
        for _ in range(warmup):
            g.replay()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(steps):
            g.replay()
        end.record()
        torch.cuda.synchronize()
        ms = start.elapsed_time(end) / steps
        ms = max_over_ranks(ms, dist, dev)
    del g, model
    torch.cuda.empty_cache()
    return {"metric": "Walsh-512 octonion prefill tokens/s", "value": world * B * T / (ms / 1e3), "unit": UNIT,
            "ms_per_step": ms, "steps": steps, "warmup": warmup,
            "config": {"workload": "config 2: octonion Walsh-512 (SwiGLU 1368, head mixing, chmod) prefill",
                       "batch_per_gpu": B, "seq_len": T, "l2": "stream state 134 MB per layer > L2, no flush"},
            "gpu_launches": launches * steps}


def measure_hlin_microbench(dev, iters=20):
    """Config 1: HadamardLinear(n, n) on bf16 activations [T, n] (N(0, 1)), ternary
    weights i.i.d. uniform {-1, 0, 1}, alpha ~ U(0.5, 1.5), beta at the reference
    init.  Each entry times `iters` calls through the module's forward with CUDA
    events, cycling over enough input/output buffers that one pass over them
    exceeds L2 (no flush needed): `us` called from Python one by one,
    `us_graph` the same calls replayed from a CUDA graph (device time).  n =
    512 from HLIN_DENSE_FROM tokens on runs the dense tcgen05 GEMM form, below
    it and for n = 2048 the packed kernel.  Algorithmic bytes per call:
    T (32 in_o + 32 out_o) 2 + 32 out_o ceil(in_o / 4) + 4 * 32 (in_o + out_o)."""
    from walsh_research_b200.model.fht_cuda import HadamardLinear
    hbm, _, _ = peaks()
    g = torch.Generator().manual_seed(0)
    out = []
    for n in (512, 2048):
        lin = HadamardLinear(n, n)
        with torch.no_grad():
            lin.weight.copy_(torch.randint(-1, 2, lin.weight.shape, generator=g).float())
            lin.alpha.copy_(torch.rand(lin.alpha.shape, generator=g) + 0.5)
        lin = lin.to(dev)
        in_o = out_o = n // 32
        for T in (1, 64, 4096, 65536):
            nbuf = max(1, min(8, int(256e6 // (T * n * 2 * 2)) + 1))
            xs = [torch.randn((T, n), generator=g).to(dev, torch.bfloat16) for _ in range(nbuf)]
            with torch.no_grad():
                for i in range(3):
                    lin(xs[i % nbuf])
                torch.cuda.synchronize()
                s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s0.record()
                for i in range(iters):
                    lin(xs[i % nbuf])
                s1.record()
                torch.cuda.synchronize()
            sec = s0.elapsed_time(s1) / iters / 1e3
            # the same calls replayed from a CUDA graph: device time without
            # the Python and launch overhead of each call
            with torch.no_grad():
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr):
                    for i in range(iters):
                        lin(xs[i % nbuf])
                gr.replay()
                torch.cuda.synchronize()
                s0.record()
                gr.replay()
                s1.record()
                torch.cuda.synchronize()
            gsec = s0.elapsed_time(s1) / iters / 1e3
            del gr
            nbytes = T * (32 * in_o + 32 * out_o) * 2 + 32 * out_o * ((in_o + 3) // 4) + 4 * 32 * (in_o + out_o)
            e = {"n": n, "T": T, "us": sec * 1e6, "GB/s": nbytes / sec / 1e9, "us_graph": gsec * 1e6}
            if T >= 4096:
                e["roofline_frac"] = nbytes / sec / 1e9 / hbm
                e["roofline_frac_graph"] = nbytes / gsec / 1e9 / hbm
            out.append(e)
            del xs
    torch.cuda.empty_cache()
    return {"metric": "HadamardLinear latency / HBM roofline (config 1)", "dtype": "bf16 in/out, fp32 accumulate",
            "peak_GBs": hbm, "entries": out}


def dominant_kernel_roofline(model, idx, B, T, dev):
    """Time the prefill attention kernel alone (CUDA events, current stream)."""
    from walsh_research_b200 import ops
    H, C = CONFIG["n_head"], CONFIG["n_embd"]
    hd = C // H
    # the model's attention operands in 16-bit mode are fp16
    q = torch.randn((B, H, T, hd), device=dev).to(torch.float16)
    k = torch.randn((B, H, T, hd), device=dev).to(torch.float16)
    v = torch.randn((B, H, T, hd), device=dev).to(torch.float16)
    o = torch.empty((B, T, H, hd), device=dev, dtype=torch.float16)
    for _ in range(3):
        ops.attention(q, k, v, 0, out=o)
    n = 10
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    s.record()
    for _ in range(n):
        ops.attention(q, k, v, 0, out=o)
    e.record()
    torch.cuda.synchronize()
    sec = s.elapsed_time(e) / n / 1e3
    flops = 4.0 * B * H * hd * (T * (T + 1) / 2)
    hbm, tflops, src = peaks()
    achieved = flops / sec / 1e12
    # DRAM bytes read + written by one launch of this kernel at B64 x T1024, from one ncu
    # capture (dram__bytes_read.sum 201.34 MB + dram__bytes_write.sum 44.76 MB)
    traffic = ATTN_TRAFFIC_B64 * B / 64 if T == SEQ else None
    return {"kernel": "walsh_attn_fwd (prefill, causal, hd16, fp16)", "bound": "tensor", "achieved": achieved,
            "peak": tflops, "unit": "TFLOP/s", "frac": achieved / tflops, "traffic": traffic,
            "traffic_unit": "bytes per launch", "algorithmic_bytes": 4 * B * H * T * hd * 2,
            "flops_per_launch": flops, "launch_ms": sec * 1e3, "peak_source": src}


if __name__ == "__main__":
    main()
