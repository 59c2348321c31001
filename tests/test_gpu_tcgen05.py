"""The tcgen05 GEMM mainloop (TMA + tensor memory) against the mma.sync
mainloop and the oracle, for every fused epilogue: ragged M/N/K tiles, both
16-bit operand types, and the device status word of the bounded waits."""
import numpy as np
import pytest
import torch

from oracle import walsh_oracle as O
from test_gpu_parity import DEV, T, rel

pytestmark = pytest.mark.gpu


@pytest.fixture
def mainloop():
    from walsh_research_b200 import _lib
    _lib.call("walsh_tc05_error", 1)
    prev = _lib.call("walsh_octo_set_mainloop", 1)

    def run(fn, tcgen05):
        _lib.call("walsh_octo_set_mainloop", 1 if tcgen05 else 0)
        out = fn()
        torch.cuda.synchronize()
        return out
    yield run
    _lib.call("walsh_octo_set_mainloop", prev)
    assert _lib.call("walsh_tc05_error", 1) == 0


def _layer(fin, fout, rng):
    from walsh_research_b200.model.cayley_dickson_cuda import OctonionFusedLinear
    m = OctonionFusedLinear(fin, fout)
    with torch.no_grad():
        m.weight.copy_(torch.from_numpy(rng.uniform(-1, 1, (8, fout // 8, fin // 8)).astype(np.float32)))
        m.beta.copy_(torch.from_numpy(rng.uniform(0.05, 0.2, (fout // 8,)).astype(np.float32)))
    return m.to(DEV)


@pytest.mark.parametrize("M,fin,fout", [(1, 512, 512), (128, 512, 512), (1000, 1368, 512), (333, 512, 1368),
                                        (4099, 512, 1536), (77, 64, 48)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_plain_gemm_matches_mma_sync_and_oracle(mainloop, M, fin, fout, dtype):
    rng = np.random.default_rng(M + 3 * fin + fout)
    m = _layer(fin, fout, rng)
    x = T(rng.normal(size=(M, fin)).astype(np.float32), dtype)
    a = mainloop(lambda: m.forward_flat(x), True)
    b = mainloop(lambda: m.forward_flat(x), False)
    w, be = m.weight.detach().cpu().numpy(), m.beta.detach().cpu().numpy()
    ref = O.octonion_linear(x.float().cpu().numpy(), w, be)
    tol = 3e-3 if dtype == torch.float16 else 1e-2
    assert rel(a, ref) < tol
    # same products, fp32 accumulation in a different order: outputs agree to the output rounding
    assert rel(a, b.float().cpu().numpy()) < (2e-3 if dtype == torch.float16 else 8e-3)


@pytest.mark.parametrize("tokens", [37, 5000])
def test_qkv_swiglu_post_epilogues_match_mma_sync(mainloop, tokens):
    from walsh_research_b200 import ops
    from walsh_research_b200.model import WalshConfig
    from walsh_research_b200.model.cayley_dickson_cuda import SwiGLUMLP, qkv_operands
    from walsh_research_b200.model.chassis import CausalSelfAttention, precompute_freqs_cis
    rng = np.random.default_rng(tokens)
    cfg = WalshConfig(n_embd=512, n_head=32, algebra="octonion", head_mixing=True)
    attn = CausalSelfAttention(cfg)
    mlp = SwiGLUMLP(cfg)
    with torch.no_grad():
        for lin in (attn.wq, attn.wk, attn.wv, attn.wo, mlp.gate_proj, mlp.up_proj, mlp.down_proj):
            lin.weight.copy_(torch.from_numpy(rng.uniform(-1, 1, tuple(lin.weight.shape)).astype(np.float32)))
    attn, mlp = attn.to(DEV), mlp.to(DEV)
    B = 1
    Tn, ctx, start = tokens, tokens + 9, 9
    u = T(rng.normal(size=(B, Tn, 512)).astype(np.float32), torch.float16)
    f = precompute_freqs_cis(16, ctx + 16)
    cos, sin = f.real[start:start + Tn].float().contiguous().to(DEV), f.imag[start:start + Tn].float().contiguous().to(DEV)

    def qkv():
        q = torch.zeros((B, 32, Tn, 16), dtype=torch.float16, device=DEV)
        kc = torch.zeros((B, 32, ctx, 16), dtype=torch.float16, device=DEV)
        vc = torch.zeros_like(kc)
        attn._octonion_qkv(u, cos, sin, start, q, kc, vc)
        return torch.cat([q.flatten(), kc.flatten(), vc.flatten()])
    assert rel(mainloop(qkv, True), mainloop(qkv, False).float().cpu().numpy()) < 2e-3

    h = mainloop(lambda: mlp.hidden_act(u), True)
    h2 = mainloop(lambda: mlp.hidden_act(u), False)
    assert rel(h, h2.float().cpu().numpy()) < 2e-3

    xs = T(rng.normal(size=(B * Tn, 4, 512)).astype(np.float32), torch.float16)
    hmix = torch.rand((B * Tn, 24), device=DEV)

    def post():
        w, s = mlp.down_operands(h.dtype)
        return ops.octo_post(h, w, s, xs, hmix)
    assert rel(mainloop(post, True), mainloop(post, False).float().cpu().numpy()) < 2e-3


def test_bounded_wait_times_out_and_context_survives():
    """A wait that can never complete gives up after its clock budget, the status
    word reports WALSH_ERR_TIMEOUT, and the next GEMM runs normally."""
    from walsh_research_b200 import _lib
    _lib.call("walsh_tc05_error", 1)
    _lib.call("walsh_tc05_wait_selftest", 2_000_000, _lib.stream())   # about 1 ms of SM clocks
    torch.cuda.synchronize()
    assert _lib.call("walsh_tc05_error", 1) == -6
    assert _lib.call("walsh_tc05_error", 0) == 0
    rng = np.random.default_rng(1)
    m = _layer(512, 512, rng)
    x = T(rng.normal(size=(300, 512)).astype(np.float32), torch.float16)
    y = m.forward_flat(x)
    torch.cuda.synchronize()
    w, be = m.weight.detach().cpu().numpy(), m.beta.detach().cpu().numpy()
    assert rel(y, O.octonion_linear(x.float().cpu().numpy(), w, be)) < 3e-3
    assert _lib.call("walsh_tc05_error", 1) == 0


@pytest.mark.parametrize("B,H,Tq,start", [(2, 3, 1024, 0), (1, 4, 300, 0), (2, 2, 77, 130), (1, 2, 129, 500),
                                          (3, 2, 6, 0), (1, 2, 1000, 24), (2, 1, 640, 0)])
@pytest.mark.parametrize("mode", [1, 2])
def test_attention_tcgen05_matches_mma_sync_and_oracle(B, H, Tq, start, mode):
    """fp16 prefill attention, head dim 16: the tcgen05 kernels (mode 1: S and
    P V in Tensor Memory; mode 2: S in Tensor Memory, softmax and P V on
    mma.sync) against the mma.sync whole-head kernel and float64 sdpa on the
    same fp16 inputs; full and partial 128-row query tiles, cached prefixes."""
    from walsh_research_b200 import _lib, ops
    from test_gpu_parity import _attn_ref
    rng = np.random.default_rng(B * 1000 + Tq + start)
    ctx = start + Tq + 3
    q = T((rng.normal(size=(B, H, Tq, 16)) * 2).astype(np.float32), torch.float16)
    k = T(rng.normal(size=(B, H, ctx, 16)).astype(np.float32), torch.float16)
    v = T(rng.normal(size=(B, H, ctx, 16)).astype(np.float32), torch.float16)
    _lib.call("walsh_tc05_error", 1)
    prev = _lib.call("walsh_attn_set_path", mode)
    try:
        a = ops.attention(q, k, v, start)
        torch.cuda.synchronize()
        _lib.call("walsh_attn_set_path", 0)
        b = ops.attention(q, k, v, start)
        torch.cuda.synchronize()
    finally:
        _lib.call("walsh_attn_set_path", prev)
    assert _lib.call("walsh_tc05_error", 1) == 0
    ref = _attn_ref(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(), start)
    assert rel(a, ref) < 3e-3
    assert rel(a, b.float().cpu().numpy()) < 3e-3


@pytest.mark.parametrize("n", [9472, 10000, 33000])
@pytest.mark.parametrize("udt,xdt", [(torch.float16, torch.float16), (torch.bfloat16, torch.bfloat16),
                                     (torch.float16, torch.bfloat16)])
def test_moe_tcgen05_matches_mma_sync_kernel(n, udt, xdt):
    """Prefill MoE on tcgen05 (router GEMM with the routing in its epilogue +
    expert-pair kernel with the site epilogue) against the single mma.sync
    kernel on the same inputs: equal selections except where the k-th and
    (k+1)-th probabilities are within the router's rounding; equal routing
    weights, expert outputs and fused site updates elsewhere; ragged last tile."""
    from walsh_research_b200 import _lib, ops
    from test_gpu_parity import _moe_module, cases
    d = cases.op_case("moe")
    rng = np.random.default_rng(n)
    m = _moe_module(d)
    args = m.kernel_args(udt)
    u = T(rng.normal(size=(n, 512)).astype(np.float32), udt)
    xs = T(rng.normal(size=(n, 4, 512)).astype(np.float32), xdt)
    hm = torch.rand((n, 24), device=DEV)

    def run(tc05):
        prev = ops.MOE_TC05
        ops.MOE_TC05 = tc05
        try:
            y, mask, probs, w = ops.moe(u, *args[:7], want_stats=True, tc=args[7])
            f = ops.moe(u, *args[:7], fuse=(xs, hm, torch.empty_like(xs)), tc=args[7])
            torch.cuda.synchronize()
            return y.float().cpu().numpy(), mask.cpu().numpy(), probs.cpu().numpy(), w.cpu().numpy(), \
                f.float().cpu().numpy()
        finally:
            ops.MOE_TC05 = prev
    _lib.call("walsh_tc05_error", 1)
    y1, m1, p1, w1, f1 = run(True)
    assert _lib.call("walsh_tc05_error", 1) == 0
    y0, m0, p0, w0, f0 = run(False)
    srt = -np.sort(-p0, axis=-1)
    near = (srt[:, 5] - srt[:, 6]) < 2e-3
    diff = (m1 != m0).any(-1)
    assert not (diff & ~near).any()
    ok = ~diff
    assert np.abs(p1 - p0).max() < 2e-3
    assert np.abs(w1 - w0)[ok].max() < 2e-3
    scale = np.abs(y0).max()
    assert np.abs(y1 - y0)[ok].max() / scale < 1e-2
    fs = np.abs(f0).max()
    assert np.abs(f1 - f0)[ok].max() / fs < 1e-2


@pytest.mark.parametrize("M,fin,fout", [(256, 512, 512), (256, 512, 1536), (37, 512, 1368), (129, 64, 200)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_narrow_tiles_equal_wide_tiles(mainloop, M, fin, fout, dtype):
    """Few-row GEMMs run with 64-wide CTA tiles (more CTAs on the same
    columns): the same K order per output, so the results equal the 256-wide
    tiling bit for bit (plain epilogue, ragged N; the q/k/v epilogue with RoPE
    and the KV-cache rows)."""
    from walsh_research_b200 import _lib
    rng = np.random.default_rng(M + fin + fout)
    m = _layer(fin, fout, rng)
    x = T(rng.normal(size=(M, fin)).astype(np.float32), dtype)
    prev = _lib.call("walsh_octo_set_narrow", -1)
    try:
        _lib.call("walsh_octo_set_narrow", 1)
        a = mainloop(lambda: m.forward_flat(x), True)
        _lib.call("walsh_octo_set_narrow", 0)
        b = mainloop(lambda: m.forward_flat(x), True)
    finally:
        _lib.call("walsh_octo_set_narrow", prev)
    assert torch.equal(a, b)


def test_narrow_tiles_qkv_epilogue_equal_wide(mainloop):
    from walsh_research_b200 import _lib
    from walsh_research_b200.model import WalshConfig
    from walsh_research_b200.model.chassis import CausalSelfAttention, precompute_freqs_cis
    rng = np.random.default_rng(99)
    cfg = WalshConfig(n_embd=512, n_head=32, algebra="octonion", head_mixing=True)
    attn = CausalSelfAttention(cfg)
    with torch.no_grad():
        for lin in (attn.wq, attn.wk, attn.wv):
            lin.weight.copy_(torch.from_numpy(rng.uniform(-1, 1, tuple(lin.weight.shape)).astype(np.float32)))
    attn = attn.to(DEV)
    B, Tn, ctx, start = 256, 1, 40, 33
    u = T(rng.normal(size=(B, Tn, 512)).astype(np.float32), torch.float16)
    f = precompute_freqs_cis(16, ctx + 16)
    cos, sin = f.real[start:start + Tn].float().contiguous().to(DEV), f.imag[start:start + Tn].float().contiguous().to(DEV)

    def qkv():
        q = torch.zeros((B, 32, Tn, 16), dtype=torch.float16, device=DEV)
        kc = torch.zeros((B, 32, ctx, 16), dtype=torch.float16, device=DEV)
        vc = torch.zeros_like(kc)
        attn._octonion_qkv(u, cos, sin, start, q, kc, vc)
        return torch.cat([q.flatten(), kc.flatten(), vc.flatten()])
    prev = _lib.call("walsh_octo_set_narrow", -1)
    try:
        _lib.call("walsh_octo_set_narrow", 1)
        a = mainloop(qkv, True)
        _lib.call("walsh_octo_set_narrow", 0)
        b = mainloop(qkv, True)
    finally:
        _lib.call("walsh_octo_set_narrow", prev)
    assert torch.equal(a, b)


@pytest.mark.parametrize("M,fin,fout", [(1, 512, 512), (100, 512, 256), (4099, 512, 1536), (20003, 512, 512),
                                        (777, 1368, 512), (333, 512, 1368)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_tma_store_epilogue_equals_row_stores(mainloop, M, fin, fout, dtype):
    """The plain epilogue's TMA-store form (each warp's scaled 32 x 32 block
    staged in shared memory with the 64-byte swizzle, clipped by the output
    map at ragged M; narrow tiles for few rows) against each lane storing its
    own row: the same rounding of the same sums, so equal bit for bit.  N not
    a multiple of 32 keeps the row stores."""
    from walsh_research_b200 import _lib
    rng = np.random.default_rng(M + 7 * fin + fout)
    m = _layer(fin, fout, rng)
    x = T(rng.normal(size=(M, fin)).astype(np.float32), dtype)
    prev = _lib.call("walsh_octo_set_tma_store", -1)
    try:
        _lib.call("walsh_octo_set_tma_store", 1)
        a = mainloop(lambda: m.forward_flat(x), True)
        _lib.call("walsh_octo_set_tma_store", 0)
        b = mainloop(lambda: m.forward_flat(x), True)
    finally:
        _lib.call("walsh_octo_set_tma_store", prev)
    assert torch.equal(a, b)
    w, be = m.weight.detach().cpu().numpy(), m.beta.detach().cpu().numpy()
    rows = np.r_[0:min(M, 200), max(0, M - 200):M]
    ref = O.octonion_linear(x[rows].float().cpu().numpy(), w, be)
    assert rel(a[rows], ref) < (3e-3 if dtype == torch.float16 else 1e-2)
