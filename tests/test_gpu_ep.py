"""Expert parallelism on one GPU: the exchange kernels (walsh_ep_dispatch /
_combine / _wait) and the owned-expert tensor-core kernel with a world of
one, against the replicated MoE; the bounded device wait on a flag that no
peer sets; and the whole model with its MoE layers expert-parallel.  Runs
of two or more GPUs are in tests/test_gpu_ep_multi.py."""
import ctypes
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


@pytest.fixture(scope="module")
def group():
    import torch.distributed as dist
    if not dist.is_initialized():
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(_free_port()))
        dist.init_process_group("gloo", rank=0, world_size=1)
        yield None
        dist.destroy_process_group()
    else:
        yield None


def _moe_layer(seed=0):
    import bench
    torch.manual_seed(seed)
    model = bench.build_model_cpu()
    return model.layers[0].feed_forward.cuda().eval()


@pytest.mark.parametrize("T", [300, 10000])
def test_single_rank_exchange_equals_replicated(group, T):
    from walsh_research_b200 import ops
    from walsh_research_b200.ep import ExpertParallel, moe_site
    ff = _moe_layer()
    rng = np.random.default_rng(T)
    u = torch.from_numpy(rng.normal(size=(1, T, 512)).astype(np.float32)).to(DEV, torch.float16)
    x = torch.from_numpy(rng.normal(size=(1, T, 4, 512)).astype(np.float32)).to(DEV, torch.float16)
    hmix = torch.from_numpy(rng.uniform(0.1, 0.5, size=(1, T, 24)).astype(np.float32)).to(DEV)
    ep = ExpertParallel(max_tokens=T, C=512, dtype=torch.float16, transport="nvlink")
    x_ep = x.clone()
    mask, probs = moe_site(u, x_ep, hmix, ff, ep)
    ep.check()
    # replicated: the same router GEMM, all experts (unfused), then the same epilogue kernel
    from walsh_research_b200 import _lib
    tc = ff.kernel_args(torch.float16)[7]
    gam = ff.experts.packed()[3]
    E = 16
    m2 = torch.empty((T, E), dtype=torch.uint8, device=DEV)
    p2 = torch.empty((T, E), dtype=torch.float32, device=DEV)
    wts = torch.empty((T, E), dtype=torch.float32, device=DEV)
    _lib.call("walsh_moe_router_tc_fwd", u.data_ptr(), _lib.dcode(u.dtype), T, tc[0].data_ptr(), tc[1].data_ptr(),
              ff.router.top_k, m2.data_ptr(), p2.data_ptr(), wts.data_ptr(), None, _lib.stream())
    y = torch.empty_like(u)
    _lib.call("walsh_moe_experts_tc_fwd", u.data_ptr(), _lib.dcode(u.dtype), T, wts.data_ptr(), tc[5].data_ptr(),
              tc[4].data_ptr(), gam.data_ptr(), y.data_ptr(), 0, None, _lib.dcode(u.dtype), None, None, _lib.stream())
    x_rep = x.clone()
    ops.mhc_post(x_rep, y, hmix, out=x_rep)
    torch.cuda.synchronize()
    assert torch.equal(mask, m2)
    assert torch.equal(ep.y_full[:T].view(1, T, 512), y)      # same kernel, same rows
    assert torch.equal(x_ep, x_rep)
    assert _lib.call("walsh_tc05_error", 1) == 0


def test_wait_on_a_flag_nobody_sets_times_out_and_the_next_exchange_runs(group):
    """The wait kernel gives up after its clock budget (about 1 ms here) and
    reports WALSH_ERR_TIMEOUT through the status word; the context stays
    usable."""
    from walsh_research_b200 import _lib
    from walsh_research_b200.ep import ExpertParallel, ExpertParallelError, moe_site
    ep = ExpertParallel(max_tokens=64, C=512, dtype=torch.float16, transport="nvlink")
    _lib.call("walsh_ep_wait", ep.flags.data_ptr(), 0, 1, ctypes.c_uint32(0xABCDE), 2_000_000, ep.status.data_ptr(),
              _lib.stream())
    torch.cuda.synchronize()
    assert int(ep.status.item()) == -6
    with pytest.raises(ExpertParallelError):
        ep.check()
    ff = _moe_layer()
    u = torch.randn((1, 64, 512), device=DEV).to(torch.float16)
    x = torch.randn((1, 64, 4, 512), device=DEV).to(torch.float16)
    hmix = torch.rand((1, 64, 24), device=DEV)
    moe_site(u, x, hmix, ff, ep)
    ep.check()
    assert torch.isfinite(x.float()).all()


def test_model_expert_parallel_equals_replicated(group):
    """16-bit forward of the 2-layer fixture model at B10 x T1000 (the
    prefill-shaped MoE: the same router GEMM on both paths) with its MoE
    layers through the exchange (world of one): the first layer's
    selections are identical, and the logits equal the replicated forward's
    to the 16-bit rounding of the unfused site epilogue."""
    import cases
    from walsh_research_b200.ep import ExpertParallel
    from walsh_research_b200.model import WalshConfig, mHCWalsh
    cfg, n, idx, sd = cases.model_inputs("model_h512")
    cfg = dict(cfg, block_size=1024)
    m = mHCWalsh(WalshConfig(**cfg), n_streams=n)
    m.load_state_dict({k: torch.from_numpy(np.array(v)) for k, v in sd.items()}, strict=False)
    m = m.to(DEV).eval()
    m.compute_dtype = torch.bfloat16
    ids = torch.from_numpy(np.random.default_rng(3).integers(0, cfg["vocab_size"], (10, 1000))).to(DEV)
    with torch.no_grad():
        ref, _ = m(ids)
        mask_ref = m.layers[0].feed_forward._last_expert_mask.clone()
        ep = ExpertParallel(max_tokens=10 * 1000, C=512, dtype=torch.float16, transport="nvlink")
        m.enable_expert_parallel(ep)
        got, _ = m(ids)
        ep.check()
        m.enable_expert_parallel(None)
    assert torch.equal(mask_ref, m.layers[0].feed_forward._last_expert_mask)
    err = float((got - ref).abs().max())
    assert err < 5e-3, err
