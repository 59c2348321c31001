"""The router's threshold rule (opt-in; the reference's forward uses top-k,
src/model/moe.py:432-436, while its HadamardRouter docstring and arguments
describe the threshold rule, src/model/moe.py:383-403) on every kernel path
that routes: the float32 CUDA-core MoE kernel (C = 512 and 2048), the
decode-sized router (16-bit, C = 512 and 2048), the tcgen05 router-GEMM
epilogue (16-bit, prefill sizes) and the mma.sync MoE kernel.

Per path: (1) the selection equals the rule applied to the kernel's own
probabilities, bit for bit (the rule's logic, independent of rounding);
(2) the probabilities are within 1e-5 (float32), 2.5e-3 (fp16 inputs) or
1e-2 (bf16 inputs) of float64;
(3) wherever every decision margin of a token (each probability's distance to
the threshold, and the probability gap at the cut) exceeds twice that error,
the selection equals float64's; (4) the expert output with the GPU's
selections equals the oracle's (1e-5 relative float32, 2e-2 16-bit).
"""
import types

import numpy as np
import pytest
import torch

from oracle import walsh_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rule(probs, thr, kmin, kmax):
    order = np.argsort(-probs, axis=-1, kind="stable")[..., :kmax]
    kt = np.clip((probs > thr).sum(-1, keepdims=True), kmin, kmax)
    mask = np.zeros_like(probs)
    np.put_along_axis(mask, order, (np.arange(kmax) < kt).astype(probs.dtype), axis=-1)
    return mask


def _margin(probs, thr, kmin, kmax):
    """Smallest decision margin per token: distance of any probability to the
    threshold, and the gap between the last taken and first untaken."""
    srt = -np.sort(-probs, axis=-1)
    kt = np.clip((probs > thr).sum(-1), kmin, kmax)
    idx = np.arange(probs.shape[0])
    cut = srt[idx, kt - 1] - srt[idx, np.minimum(kt, probs.shape[-1] - 1)]
    return np.minimum(np.abs(probs - thr).min(-1), cut)


def _moe_module(C, seed, logit_scale):
    from walsh_research_b200.model.moe import HadamardMoE
    torch.manual_seed(seed)
    cfg = types.SimpleNamespace(n_embd=C)
    m = HadamardMoE(cfg, threshold=0.1, min_experts=2, max_experts=6)
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        m.router.gate[0].weight.copy_(torch.randn(m.router.gate[0].weight.shape, generator=g) / np.sqrt(C))
        h = m.router.gate[0].weight.shape[0]
        m.router.gate[2].weight.copy_(torch.randn(m.router.gate[2].weight.shape, generator=g) * logit_scale / np.sqrt(h))
        for w in (m.experts.gate_weights, m.experts.up_weights, m.experts.down_weights):
            w.copy_(torch.randint(-1, 2, w.shape, generator=g).float())
    m.router.routing_mode = "threshold"
    return m


PATHS = [
    # (C, ntok, dtype, MOE_TC05, router logit scale)
    (512, 1000, torch.float32, True, 2.0),     # CUDA-core moe_kernel
    (2048, 300, torch.float32, True, 3.0),
    (512, 300, torch.float16, True, 2.0),      # decode-sized router (walsh_moe_hidden_fwd)
    (2048, 300, torch.bfloat16, True, 3.0),
    (512, 20000, torch.float16, True, 2.0),    # tcgen05 router GEMM epilogue
    (512, 10000, torch.bfloat16, False, 2.0),  # mma.sync moe_mma512_kernel
]


@pytest.mark.parametrize("C,ntok,dtype,tc05,scale", PATHS)
def test_threshold_routing_paths(C, ntok, dtype, tc05, scale, parity_report):
    from walsh_research_b200 import ops
    m = _moe_module(C, C + ntok, scale)
    thr, kmin, kmax = 0.1, 2, 6
    rng = np.random.default_rng(ntok)
    u = torch.from_numpy(rng.normal(size=(1, ntok, C)).astype(np.float32)).to(dtype)
    un = u.double().numpy()[0]
    sd = {k: v.detach().double().numpy() for k, v in m.state_dict().items()}
    m = m.to(DEV).eval()
    old = ops.MOE_TC05
    ops.MOE_TC05 = tc05
    try:
        with torch.no_grad():
            y = m(u.to(DEV))
    finally:
        ops.MOE_TC05 = old
    mask = m._last_expert_mask.view(ntok, -1).cpu().numpy()
    probs = m._last_router_probs.view(ntok, -1).float().cpu().numpy().astype(np.float64)
    # (1) the rule on the kernel's own probabilities, exactly
    np.testing.assert_array_equal(mask, _rule(probs, thr, kmin, kmax))
    # (2) probabilities against float64
    _, want_mask, want_probs = O.router(un, sd["router.gate.0.weight"], sd["router.gate.2.weight"], kmax,
                                        threshold=thr, min_experts=kmin)
    perr = float(np.abs(probs - want_probs).max())
    # router inputs rounded to 16 bits: fp16 keeps 11 significant bits, bf16 8
    bound = {torch.float32: 1e-5, torch.float16: 2.5e-3, torch.bfloat16: 1e-2}[dtype]
    assert perr < bound
    # (3) away from every decision edge the selections equal float64's
    clear = _margin(want_probs, thr, kmin, kmax) > 2 * bound
    assert np.array_equal(mask[clear], want_mask[clear])
    # (4) the expert output with the GPU's selections
    ref, _, _ = O.moe(un[None], sd, "", kmax, forced_mask=mask[None])
    got = y.float().cpu().numpy()
    err = float(np.abs(got - ref).max() / np.abs(ref).max())
    assert err < (1e-5 if dtype == torch.float32 else 2e-2)
    n = mask.sum(-1)
    parity_report(f"{dtype} C{C} ntok {ntok}: experts per token {n.min():.0f}..{n.max():.0f} "
                  f"(mean {n.mean():.2f}); clear tokens {int(clear.sum())}/{ntok} identical; prob err {perr:.2e}; "
                  f"output rel err {err:.2e}")
    assert n.min() >= kmin and n.max() <= kmax and n.min() < n.max()


def test_threshold_routing_model_fp32_matches_oracle(parity_report):
    """Whole model (2-layer Walsh-512 fixture weights) in threshold mode:
    logits within 1e-4 of the float64 oracle run with the same rule."""
    import cases
    from walsh_research_b200.model import WalshConfig, mHCWalsh
    cfg, n, idx, sd = cases.model_inputs("model_h512")
    model = mHCWalsh(WalshConfig(**cfg), n_streams=n)
    model.load_state_dict({k: torch.from_numpy(np.array(v)) for k, v in sd.items()}, strict=False)
    model = model.to(DEV).eval()
    model.set_moe_routing("threshold")
    with torch.no_grad():
        logits, _ = model(torch.from_numpy(np.array(idx)).to(DEV))
    masks = [l.feed_forward._last_expert_mask.cpu().numpy() for l in model.layers]
    ocfg = dict(cfg, moe_routing="threshold")
    trace = {}
    ref, _ = O.mhc_walsh_forward(ocfg, sd, idx, n, trace=trace)
    for l, m in enumerate(masks):
        np.testing.assert_array_equal(m, trace["router_mask"][l])
    err = float(np.abs(logits.cpu().numpy() - ref).max() / np.abs(ref).max())
    ks = np.concatenate([m.sum(-1).ravel() for m in masks])
    parity_report(f"logits rel err {err:.2e}; experts per token {ks.min():.0f}..{ks.max():.0f}")
    assert err < 1e-4
