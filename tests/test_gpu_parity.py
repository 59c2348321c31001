"""GPU parity: the sm_100a kernels (through libwalsh's C ABI) against the
golden fixtures produced by the reference's own code and, at larger sizes,
against the numpy oracle.

Tolerances (max |ours - ref| / max |ref| unless stated):
  * ternary packing / unpacking / top-k selection: bit-exact
  * float32 activations: 1e-5 per op, 1e-4 for whole-model logits
  * bfloat16 activations: 2e-2 max-abs on logits (fp32 reference), with the
    routing sets matched; per-op 2e-2 relative.
"""
import os

import numpy as np
import pytest
import torch

import cases
from oracle import walsh_oracle as O

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
DEV = "cuda"


def golden(name):
    return np.load(os.path.join(GOLDEN, name + ".npz"))


def T(a, dtype=torch.float32):
    return torch.from_numpy(np.array(a)).to(DEV, dtype)


def rel(a, b):
    a = a.detach().float().cpu().numpy() if torch.is_tensor(a) else np.asarray(a)
    b = np.asarray(b, dtype=np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def build_model(name, dtype=torch.float32):
    from walsh_research_b200.model import WalshConfig, mHCWalsh
    cfg, n, idx, sd = cases.model_inputs(name)
    model = mHCWalsh(WalshConfig(**cfg), n_streams=n)
    model.load_state_dict({k: torch.from_numpy(np.array(v)) for k, v in sd.items()}, strict=False)
    model = model.to(DEV).eval()
    model.compute_dtype = dtype
    return cfg, n, idx, sd, model


# ---------------------------------------------------------------------------
# ternary weights
# ---------------------------------------------------------------------------

def test_pack_unpack_bit_exact():
    from walsh_research_b200 import ops
    d, g = cases.op_case("pack"), golden("pack")
    for k in ("w_a", "w_b", "w_c"):
        packed, _ = ops.quantize_pack(T(d[k]))
        assert np.array_equal(packed.cpu().numpy(), g[k + "_packed"]), k
        back = ops.unpack(T(g[k + "_packed"], torch.uint8), d[k].shape[-1])
        assert np.array_equal(back.cpu().numpy(), d[k]), k


def test_quantize_matches_reference():
    from walsh_research_b200.model.moe import quantize_ternary as qs
    from walsh_research_b200.model.physics import quantize_ternary as qu
    d, g = cases.op_case("quant"), golden("quant")
    np.testing.assert_allclose(qu(T(d["w_unscaled"])).cpu().numpy(), g["unscaled"], atol=2e-7, rtol=0)
    ours = qs(T(d["w_scaled"])).cpu().numpy()
    assert np.array_equal(np.sign(ours), np.sign(g["scaled"]))
    np.testing.assert_allclose(ours, g["scaled"], rtol=3e-7, atol=0)


def test_quantize_ragged_k_and_odd_rows():
    from walsh_research_b200 import ops
    rng = np.random.default_rng(5)
    w = rng.normal(size=(7, 13, 171)).astype(np.float32)
    packed, gamma = ops.quantize_pack(T(w))
    assert packed.shape == (7, 13, 43)
    np.testing.assert_array_equal(packed.cpu().numpy(), O.pack_ternary(O.quantize_ternary(w)))
    np.testing.assert_allclose(gamma.item(), O.absmean_gamma(w), rtol=2e-7)


# ---------------------------------------------------------------------------
# Hadamard algebra
# ---------------------------------------------------------------------------

def _hlin(d):
    from walsh_research_b200.model.fht_cuda import HadamardLinear
    fin, fout = d["x"].shape[-1], d["weight"].shape[1] * 32
    layer = HadamardLinear(fin, fout)
    with torch.no_grad():
        layer.weight.copy_(torch.from_numpy(d["weight"]))
        layer.alpha.copy_(torch.from_numpy(d["alpha"]))
        layer.beta.copy_(torch.from_numpy(d["beta"]))
    return layer.to(DEV)


@pytest.mark.parametrize("name", ["hlin_512", "hlin_512_latent", "hlin_2048", "hlin_512x2048", "hlin_2048x512"])
def test_hadamard_linear_fp32(name):
    d, g = cases.op_case(name), golden(name)
    y = _hlin(d)(T(d["x"]))
    assert y.dtype == torch.float32
    assert rel(y, g["y"]) < 1e-5


@pytest.mark.parametrize("name", ["hlin_512", "hlin_2048"])
def test_hadamard_linear_bf16(name):
    d, g = cases.op_case(name), golden(name)
    y = _hlin(d)(T(d["x"], torch.bfloat16))
    assert y.dtype == torch.bfloat16
    assert rel(y, g["y"]) < 2e-2


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("F,ntok", [(512, 1), (512, 31), (512, 32), (512, 33), (512, 4097), (512, 150 * 32 * 2 + 5),
                                    (2048, 1), (2048, 15), (2048, 17), (2048, 148 * 16 * 3 + 7)])
def test_hadamard_linear_packed_weights_vs_oracle(dt, F, ntok):
    """The 16-bit HadamardLinear(F, F) that reads the 2-bit packed weights
    (ragged last tile, several tiles per persistent CTA) against the float64
    oracle on the same rounded inputs, and against the kernel it replaces
    (512: the mma.sync kernel with fp16 weight copies; 2048: the general
    kernel).  16-bit intermediates: 1e-2 of the largest output."""
    from walsh_research_b200 import _lib, ops
    rng = np.random.default_rng(ntok + F)
    io = F // 32
    d = dict(x=rng.normal(size=(1, ntok, F)).astype(np.float32), weight=rng.normal(size=(32, io, io)).astype(np.float32),
             alpha=rng.uniform(0.5, 1.5, (32, io)).astype(np.float32),
             beta=rng.uniform(0.1, 0.4, (32, io)).astype(np.float32))
    layer = _hlin(d)
    x = T(d["x"], dt)
    _lib.call("walsh_hlin_pk_error", 1)
    ops.HLIN_DENSE = False
    try:
        y = layer(x)
    finally:
        ops.HLIN_DENSE = True
    assert y.dtype == dt
    ref = O.hadamard_linear(x.double().cpu().numpy(), d["weight"], d["alpha"], d["beta"])
    assert rel(y, ref) < 1e-2
    if dt == torch.bfloat16 or F == 2048:
        ops.HLIN_PACKED = False
        try:
            y_old = layer(x)
        finally:
            ops.HLIN_PACKED = True
        assert rel(y, y_old.float().cpu().numpy()) < 1e-2
    torch.cuda.synchronize()
    assert _lib.call("walsh_hlin_pk_error", 1) == 0


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("alpha_hi", [1.5, 300.0])
def test_hadamard_linear_dense_weights_match_float_matrix(dt, alpha_hi):
    """The dense matrix of the GEMM form (integer H W H sums times alpha and
    a power of two, rounded once to the 16-bit type) times its row scale
    against the layer's float64-built float32 matrix, entry by entry: within
    the 16-bit type's rounding.  alpha up to 300 exercises the power-of-two
    normalisation that keeps float16 entries in range."""
    from walsh_research_b200 import ops
    rng = np.random.default_rng(5)
    F, io = 512, 16
    d = dict(x=np.zeros((1, 1, F), np.float32), weight=rng.normal(size=(32, io, io)).astype(np.float32),
             alpha=rng.uniform(alpha_hi / 6, alpha_hi, (32, io)).astype(np.float32),
             beta=rng.uniform(0.1, 0.4, (32, io)).astype(np.float32))
    layer = _hlin(d)
    w, scale = layer.dense16(dt)
    assert w.dtype == dt and w.shape == (F, F) and w.abs().max().item() <= 1.0
    got = (w.float() * scale[:, None]).cpu().numpy()
    ref = layer.dense().cpu().numpy()
    ulp = 2.0 ** (-8 if dt == torch.bfloat16 else -11)
    err = np.abs(got - ref) / np.maximum(np.abs(ref), 1e-30)
    assert err[ref != 0].max() <= ulp * 1.01
    assert np.all(got[ref == 0] == 0)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("ntok", [1, 33, 4097, 150 * 128 + 77, 32768 + 5])
def test_hadamard_linear_dense_vs_oracle_and_packed(dt, ntok):
    """HadamardLinear(512, 512) as one tcgen05 GEMM over the dense matrix
    (the default from HLIN_DENSE_FROM tokens on; forced here for every size:
    narrow tiles for few tokens, ragged last row tile): against the float64
    oracle on the same rounded inputs and against the packed kernel, within
    1e-2 of the largest output (16-bit operands)."""
    from walsh_research_b200 import _lib, ops
    rng = np.random.default_rng(ntok)
    F, io = 512, 16
    d = dict(x=rng.normal(size=(1, ntok, F)).astype(np.float32), weight=rng.normal(size=(32, io, io)).astype(np.float32),
             alpha=rng.uniform(0.5, 1.5, (32, io)).astype(np.float32),
             beta=rng.uniform(0.1, 0.4, (32, io)).astype(np.float32))
    layer = _hlin(d)
    x = T(d["x"], dt)
    _lib.call("walsh_tc05_error", 1)
    prev, ops.HLIN_DENSE_FROM = ops.HLIN_DENSE_FROM, 1
    try:
        y = layer(x)
    finally:
        ops.HLIN_DENSE_FROM = prev
    torch.cuda.synchronize()
    assert _lib.call("walsh_tc05_error", 1) == 0
    assert y.dtype == dt
    ref = O.hadamard_linear(x.double().cpu().numpy(), d["weight"], d["alpha"], d["beta"])
    assert rel(y, ref) < 1e-2
    ops.HLIN_DENSE = False
    try:
        y_pk = layer(x)
    finally:
        ops.HLIN_DENSE = True
    assert rel(y, y_pk.float().cpu().numpy()) < 1e-2


@pytest.mark.parametrize("fin,fout,ntok", [(512, 512, 4096 + 3), (2048, 2048, 517), (512, 2048, 33),
                                            (2048, 512, 1), (512, 512, 1)])
def test_hadamard_linear_vs_oracle_sizes(fin, fout, ntok):
    """Ragged token counts (tails of the token tiles) against the oracle."""
    rng = np.random.default_rng(ntok)
    d = dict(x=rng.normal(size=(1, ntok, fin)).astype(np.float32),
             weight=rng.integers(-1, 2, size=(32, fout // 32, fin // 32)).astype(np.float32),
             alpha=rng.uniform(0.5, 1.5, (32, fin // 32)).astype(np.float32),
             beta=rng.uniform(0.1, 0.3, (32, fout // 32)).astype(np.float32))
    y = _hlin(d)(T(d["x"]))
    ref = O.hadamard_linear(d["x"], d["weight"], d["alpha"], d["beta"])
    assert rel(y, ref) < 1e-5


@pytest.mark.parametrize("name", ["headmix", "headmix32"])
def test_head_mixer(name):
    from walsh_research_b200.model.fht_cuda import HadamardHeadMixerFused
    d, g = cases.op_case(name), golden(name)
    m = HadamardHeadMixerFused(d["x"].shape[-1])
    with torch.no_grad():
        m.W.copy_(torch.from_numpy(d["W"]))
        m.beta.copy_(torch.from_numpy(d["beta"]))
    m = m.to(DEV)
    assert rel(m(T(d["x"])), g["y"]) < 1e-5
    assert rel(m(T(d["x"], torch.bfloat16)), g["y"]) < 2e-2


# ---------------------------------------------------------------------------
# mHC
# ---------------------------------------------------------------------------

def test_sinkhorn():
    from walsh_research_b200.model import SinkhornKnopp
    d, g = cases.op_case("sinkhorn"), golden("sinkhorn")
    assert rel(SinkhornKnopp()(T(d["H"])), g["y"]) < 1e-5


def test_stream_mapping():
    from walsh_research_b200.model.mhc import ResidualStreamMapping
    d, g = cases.op_case("mapping"), golden("mapping")
    for kind in ("pre", "post", "res"):
        m = ResidualStreamMapping(512, 4, kind)
        with torch.no_grad():
            m.phi.weight.copy_(torch.from_numpy(d[f"{kind}_phi"]))
            m.alpha.copy_(torch.from_numpy(np.array(d[f"{kind}_alpha"])))
            m.bias.copy_(torch.from_numpy(d[f"{kind}_bias"]))
        h = m.to(DEV)(T(d["x"]))
        assert h.shape == g[kind].shape
        assert rel(h, g[kind]) < 1e-5, kind


@pytest.mark.parametrize("xdt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("kernel,ntok,C", [("two_pass", 10000, 512), ("single_pass", 9000, 512),
                                           ("single_pass", 37, 512), ("single_pass", 37, 2048),
                                           ("pipelined", 10000, 512), ("pipelined", 150 * 16 * 5 + 7, 512)])
def test_tensor_core_mapping_vs_oracle(xdt, kernel, ntok, C):
    """The tensor-core site prologues for either 16-bit stream type: the
    two-pass kernel (from 9472 tokens without phi fragments, or with the
    pipelined kernel switched off), the single-pass TMA kernel (phi in
    fragment order; below 9472 tokens, ragged last tile) and the persistent
    pipelined single-pass kernel (from 9472 tokens; several tiles per CTA and
    passes round the buffer ring, ragged last tile): H_pre/H_post/H_res vs the
    oracle on the same rounded stream values, and the pre-mixed, normed u."""
    from walsh_research_b200 import _lib
    from walsh_research_b200 import ops
    assert _lib.call("walsh_map_set_pipe", -1) == 1
    from walsh_research_b200.model.mhc import MAP_EPS, ResidualStreamMapping, mHCResidualStream, site_params
    rng = np.random.default_rng(41)
    st = mHCResidualStream(C, 4)
    with torch.no_grad():
        for m in (st.H_pre, st.H_post, st.H_res):
            m.phi.weight.copy_(torch.from_numpy(rng.normal(0, 0.02, tuple(m.phi.weight.shape)).astype(np.float32)))
            m.alpha.fill_(0.7)
            m.bias.copy_(torch.from_numpy(rng.normal(0, 0.5, tuple(m.bias.shape)).astype(np.float32)))
    st = st.to(DEV)
    x = T(rng.normal(size=(ntok, 4, C)).astype(np.float32) * 3, xdt)
    nw = T((1 + 0.1 * rng.normal(size=C)).astype(np.float32))
    phi, mp, phil, phif = site_params(st, xdt)
    _lib.call("walsh_map_error", 1)
    u, hmix = ops.mhc_map(x, phi, mp, MAP_EPS, nw, 1e-6, phi_lp=phil, u_dtype=torch.float16,
                          phi_frag=None if kernel == "two_pass" else phif)
    torch.cuda.synchronize()
    if kernel == "pipelined":
        # against the two-pass kernel on the same input: both are within the
        # oracle tolerances below, and they agree to fp16 rounding of u
        _lib.call("walsh_map_set_pipe", 0)
        try:
            u2, hmix2 = ops.mhc_map(x, phi, mp, MAP_EPS, nw, 1e-6, phi_lp=phil, u_dtype=torch.float16, phi_frag=phif)
        finally:
            _lib.call("walsh_map_set_pipe", 1)
        assert float((hmix - hmix2).abs().max()) < 1e-4
        assert rel(u, u2.float().cpu().numpy()) < 2e-3
    assert _lib.call("walsh_map_error", 1) == 0
    xf = x.float().cpu().numpy().astype(np.float64).reshape(1, ntok, 4 * C)
    p = {k: v.detach().cpu().numpy() for k, v in st.state_dict().items()}
    hp = O.stream_mapping(xf, p["H_pre.phi.weight"], p["H_pre.alpha"], p["H_pre.bias"], "pre")
    ho = O.stream_mapping(xf, p["H_post.phi.weight"], p["H_post.alpha"], p["H_post.bias"], "post")
    hr = O.stream_mapping(xf, p["H_res.phi.weight"], p["H_res.alpha"], p["H_res.bias"], "res")
    h = hmix.cpu().numpy()
    assert np.abs(h[:, :4] - hp.reshape(ntok, 4)).max() < 5e-3
    assert np.abs(h[:, 4:8] - ho.reshape(ntok, 4)).max() < 1e-2
    assert np.abs(h[:, 8:] - hr.reshape(ntok, 16)).max() < 5e-3
    pre = (h[:, None, :4] @ x.float().cpu().numpy().astype(np.float64))[:, 0]
    ref_u = O.rmsnorm(pre, nw.cpu().numpy().astype(np.float64))
    assert rel(u, ref_u) < 5e-3


def test_residual_stream_site_matches_oracle():
    """map (with norm) + an identity layer + post against the oracle."""
    from walsh_research_b200 import ops
    from walsh_research_b200.model.mhc import MAP_EPS
    rng = np.random.default_rng(3)
    C, B, Tn = 512, 3, 37
    x = (rng.normal(size=(B, Tn, 4, C)) * 0.5).astype(np.float32)
    phi = rng.normal(0, 0.02, (24, 4 * C)).astype(np.float32)
    al = rng.uniform(0.1, 0.5, 3).astype(np.float32)
    bias = np.concatenate([rng.normal(0, .5, 8), (2 * np.eye(4) + rng.normal(0, .5, (4, 4))).ravel()]).astype(np.float32)
    nw = (1 + rng.normal(0, .1, C)).astype(np.float32)
    mp = np.concatenate([al, [0], bias]).astype(np.float32)
    u, hmix = ops.mhc_map(T(x), T(phi), T(mp), MAP_EPS, T(nw), 1e-6)
    xf = x.reshape(B, Tn, 4 * C).astype(np.float64)
    hp = O.stream_mapping(xf, phi[:4], al[0], bias[:4], "pre")
    ho = O.stream_mapping(xf, phi[4:8], al[1], bias[4:8], "post")
    hr = O.stream_mapping(xf, phi[8:], al[2], bias[8:].reshape(4, 4), "res")
    u_ref = O.rmsnorm((hp @ x.astype(np.float64))[:, :, 0], nw)
    assert rel(hmix[..., :4], hp[..., 0, :]) < 1e-5
    assert rel(hmix[..., 4:8], ho[..., 0, :]) < 1e-5
    assert rel(hmix[..., 8:].reshape(B, Tn, 4, 4), hr) < 1e-5
    assert rel(u, u_ref) < 1e-5
    f = rng.normal(size=(B, Tn, C)).astype(np.float32)
    xo = ops.mhc_post(T(x), T(f), hmix)
    ref = hr @ x.astype(np.float64) + np.swapaxes(ho, -1, -2) @ f[:, :, None, :].astype(np.float64)
    assert rel(xo, ref) < 1e-5


# ---------------------------------------------------------------------------
# MoE and channel modulation
# ---------------------------------------------------------------------------

def _moe_module(d):
    from walsh_research_b200.model import WalshConfig
    from walsh_research_b200.model.moe import HadamardMoE
    m = HadamardMoE(WalshConfig(n_embd=512), max_experts=int(d["top_k"]))
    with torch.no_grad():
        m.router.gate[0].weight.copy_(torch.from_numpy(d["gate0"]))
        m.router.gate[2].weight.copy_(torch.from_numpy(d["gate2"]))
        m.experts.gate_weights.copy_(torch.from_numpy(d["gate_w"]))
        m.experts.up_weights.copy_(torch.from_numpy(d["up_w"]))
        m.experts.down_weights.copy_(torch.from_numpy(d["down_w"]))
    return m.to(DEV).eval()


def test_moe_fp32():
    d, g = cases.op_case("moe"), golden("moe")
    m = _moe_module(d)
    w, mask, probs = m.router(T(d["x"]))
    assert np.array_equal(mask.cpu().numpy().astype(np.uint8), g["mask"])
    assert rel(probs, g["probs"]) < 1e-5
    assert rel(w, g["weights"]) < 1e-5
    y = m(T(d["x"]))
    assert rel(y, g["y"]) < 1e-5
    assert np.array_equal(m._last_expert_mask.cpu().numpy().astype(np.uint8), g["mask"])
    # experts with caller-given weights
    ye = m.experts(T(d["x"]).view(2, 8, 16, 32), T(g["weights"]))
    assert rel(ye.reshape(2, 8, 512), g["y"]) < 1e-5


def test_moe_bf16_with_matched_routing():
    d, g = cases.op_case("moe"), golden("moe")
    m = _moe_module(d)
    y = m(T(d["x"], torch.bfloat16))
    mask = m._last_expert_mask.cpu().numpy().astype(np.uint8)
    probs = g["probs"]
    # tie rule: a differing selection is excused only where the k-th/(k+1)-th gap is < 1e-2 (bf16 input)
    srt = -np.sort(-probs, axis=-1)
    gap = srt[..., 5] - srt[..., 6]
    bad = (mask != g["mask"]).any(-1) & (gap > 1e-2)
    assert not bad.any()
    same = (mask == g["mask"]).all(-1)
    diff = np.abs(y.float().cpu().numpy() - g["y"])[same]
    assert diff.max() / np.abs(g["y"]).max() < 2e-2


def test_moe_large_vs_oracle_topk_sets():
    """2000 tokens with router gaps from scaled logits: selection sets bit-exact."""
    from walsh_research_b200 import ops
    d = cases.op_case("moe")
    rng = np.random.default_rng(9)
    x = rng.normal(size=(1, 2000, 512)).astype(np.float32)
    m = _moe_module(d)
    w1t, w2, gp, up, dp, gam, k, tc = m.kernel_args(torch.float32)
    y, mask, probs, w = ops.moe(T(x), w1t, w2, gp, up, dp, gam, k, want_stats=True, tc=tc)
    p = {"r.router.gate.0.weight": d["gate0"], "r.router.gate.2.weight": d["gate2"],
         "r.experts.gate_weights": d["gate_w"], "r.experts.up_weights": d["up_w"], "r.experts.down_weights": d["down_w"]}
    y_ref, mask_ref, probs_ref = O.moe(x.astype(np.float64), p, "r.", 6)
    srt = -np.sort(-probs_ref, axis=-1)
    tie = (srt[..., 5] - srt[..., 6]) < 1e-6
    diff = (mask.cpu().numpy() != mask_ref).any(-1)
    assert not (diff & ~tie).any()
    ok = ~diff
    assert np.abs(y.cpu().numpy() - y_ref)[ok].max() / np.abs(y_ref).max() < 1e-5


def test_channel_modulation():
    from walsh_research_b200.model.moe import HadamardChannelModulation
    d, g = cases.op_case("chmod"), golden("chmod")
    m = HadamardChannelModulation(512, use_ternary=True, residual_scale=0.5)
    with torch.no_grad():
        m.context_mlp[0].weight.copy_(torch.from_numpy(d["w0"]))
        m.context_mlp[2].weight.copy_(torch.from_numpy(d["w2"]))
        m.scale_temp.copy_(torch.from_numpy(d["scale_temp"]))
    m = m.to(DEV)
    assert rel(m(T(d["x"])), g["y"]) < 1e-5
    assert rel(m(T(d["x"], torch.bfloat16)), g["y"]) < 2e-2


def test_channel_modulation_long_segments_vs_oracle():
    """Segments longer than one stats chunk (ragged last chunk)."""
    from walsh_research_b200.model.moe import HadamardChannelModulation
    rng = np.random.default_rng(4)
    x = rng.normal(size=(3, 150, 512)).astype(np.float32)
    w0 = rng.integers(-1, 2, (128, 512)).astype(np.float32)
    w2 = rng.normal(size=(32, 128)).astype(np.float32)
    m = HadamardChannelModulation(512)
    with torch.no_grad():
        m.context_mlp[0].weight.copy_(torch.from_numpy(w0))
        m.context_mlp[2].weight.copy_(torch.from_numpy(w2))
        m.scale_temp.fill_(0.25)
    y = m.to(DEV)(T(x))
    assert rel(y, O.channel_mod(x.astype(np.float64), w0, w2, np.array([0.25]))) < 1e-5


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
def test_chmod_16bit_rows_in_place_match_fp32(dt):
    """16-bit rows at C = 512 (the vectorised stats and apply kernels, several
    rows per warp) against the fp32 kernels on the same values, in place as the
    block runs it (out aliases x), with the norm weight and the input added."""
    from walsh_research_b200 import ops
    from walsh_research_b200.model.moe import HadamardChannelModulation
    rng = np.random.default_rng(12)
    m = HadamardChannelModulation(512).to(DEV)
    w1, w2c, gam, temp = m.kernel_args()
    nseg, seg = 64, 1024
    x = T(rng.normal(size=(nseg * seg, 512)).astype(np.float32), dt)
    nw = T(rng.uniform(0.5, 1.5, size=512).astype(np.float32))
    ref, s_ref, h_ref = ops.chmod(x.float(), seg, w1, w2c, gam, temp, norm_w=nw, norm_eps=1e-6, add_input=True)
    y = x.clone()
    _, sc, sh = ops.chmod(y, seg, w1, w2c, gam, temp, norm_w=nw, norm_eps=1e-6, add_input=True, out=y)
    assert rel(sc, s_ref.cpu().numpy()) < 1e-4
    assert rel(sh, h_ref.cpu().numpy()) < 1e-4
    assert rel(y, ref.cpu().numpy()) < (2e-3 if dt == torch.float16 else 1.6e-2)


@pytest.mark.parametrize("C,nseg,seg_len,dt", [(512, 1024, 1, torch.float16), (2048, 1024, 1, torch.float16),
                                              (512, 600, 70, torch.bfloat16), (2048, 512, 3, torch.float32)])
def test_chmod_tensor_core_mlp_matches_cuda_core_mlp(C, nseg, seg_len, dt):
    """Modulation MLP with its first layer as a tensor-core GEMM over the
    three-way bf16 split of the segment means (walsh_chmod_mlp_tc) against
    the CUDA-core kernel (walsh_chmod_mlp) on the same stats: scale and shift
    to fp32 rounding, and the applied rows; decode-shaped (one row per
    segment) and multi-row segments with a ragged last stats chunk."""
    from walsh_research_b200 import ops
    from walsh_research_b200.model.moe import HadamardChannelModulation
    rng = np.random.default_rng(C + nseg + seg_len)
    m = HadamardChannelModulation(C).to(DEV)
    with torch.no_grad():
        m.context_mlp[0].weight.copy_(torch.from_numpy(rng.normal(size=(C // 4, C)).astype(np.float32)))
        m.context_mlp[2].weight.copy_(torch.from_numpy(rng.normal(size=(C // 16, C // 4)).astype(np.float32)))
        m.scale_temp.fill_(0.3)
    w1, w2c, gam, temp = m.kernel_args()
    x = T((rng.normal(size=(nseg * seg_len, C)) * 3).astype(np.float32), dt)
    nw = T(rng.uniform(0.5, 1.5, size=C).astype(np.float32))
    ops.CHMOD_ROWS_FUSED = False  # the three-step form on both sides
    try:
        y0, s0, h0 = ops.chmod(x, seg_len, w1, w2c, gam, temp, norm_w=nw, norm_eps=1e-6, add_input=True)
        y1, s1, h1 = ops.chmod(x, seg_len, w1, w2c, gam, temp, norm_w=nw, norm_eps=1e-6, add_input=True,
                               w1_dense=m.w1_dense())
    finally:
        ops.CHMOD_ROWS_FUSED = True
    # float64 MLP on the same segment means (RMSNorm'd rows x norm weight, averaged)
    xf = x.double().cpu().numpy().reshape(nseg, seg_len, C)
    xn = xf / np.sqrt((xf * xf).mean(-1, keepdims=True) + 1e-6) * nw.double().cpu().numpy()
    bulk = xn.mean(1)
    t1 = ops.unpack(w1, C).double().cpu().numpy()
    t2 = ops.unpack(w2c, C // 4).double().cpu().numpy()
    g = gam.double().cpu().numpy()
    a1 = bulk @ t1.T * g[0]
    a2 = (a1 / (1 + np.exp(-a1))) @ t2.T * g[1]
    E = C // 32
    s_ref, h_ref = 1 + 0.3 * np.tanh(a2[:, :E]), a2[:, E:]
    for got, want, cuda_core in ((s1, s_ref, s0), (h1, h_ref, h0)):
        # fp32 rounding of the two K = C sums (unit-variance test weights): the
        # tensor-core path is as close to float64 as the CUDA-core path
        err_tc, err_cc = rel(got, want), rel(cuda_core, want)
        assert err_tc < max(2 * err_cc, 1e-5), (err_tc, err_cc)
    tol = {torch.float32: 1e-4, torch.float16: 2e-3, torch.bfloat16: 1.6e-2}[dt]  # a few output ulps
    assert rel(y1, y0.float().cpu().numpy()) < tol


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("nrows", [1, 3, 4, 1023, 1024])
def test_chmod_single_row_segments_fused(nrows, dt):
    """Single-row segments (batched decode) in one launch (walsh_chmod_rows_fwd,
    ragged last CTA of 4 rows, in place): scale and shift against a float64 MLP
    on the same rounded rows, and the applied rows against the three-step
    kernels (stats, tensor-core or CUDA-core MLP, apply) on the same inputs."""
    from walsh_research_b200 import ops
    from walsh_research_b200.model.moe import HadamardChannelModulation
    C = 512
    rng = np.random.default_rng(nrows + 7)
    m = HadamardChannelModulation(C).to(DEV)
    with torch.no_grad():
        m.context_mlp[0].weight.copy_(torch.from_numpy(rng.normal(size=(C // 4, C)).astype(np.float32)))
        m.context_mlp[2].weight.copy_(torch.from_numpy(rng.normal(size=(C // 16, C // 4)).astype(np.float32)))
        m.scale_temp.fill_(0.3)
    w1, w2c, gam, temp = m.kernel_args()
    x = T((rng.normal(size=(nrows, C)) * 3).astype(np.float32), dt)
    nw = T(rng.uniform(0.5, 1.5, size=C).astype(np.float32))
    y = x.clone()
    _, s1, h1 = ops.chmod(y, 1, w1, w2c, gam, temp, norm_w=nw, norm_eps=1e-6, add_input=True, out=y)
    ops.CHMOD_ROWS_FUSED = False
    try:
        y0, s0, h0 = ops.chmod(x, 1, w1, w2c, gam, temp, norm_w=nw, norm_eps=1e-6, add_input=True,
                               w1_dense=m.w1_dense())
    finally:
        ops.CHMOD_ROWS_FUSED = True
    xf = x.double().cpu().numpy()
    bulk = xf / np.sqrt((xf * xf).mean(-1, keepdims=True) + 1e-6) * nw.double().cpu().numpy()
    t1 = ops.unpack(w1, C).double().cpu().numpy()
    t2 = ops.unpack(w2c, C // 4).double().cpu().numpy()
    g = gam.double().cpu().numpy()
    a1 = bulk @ t1.T * g[0]
    a2 = (a1 / (1 + np.exp(-a1))) @ t2.T * g[1]
    E = C // 32
    s_ref, h_ref = 1 + 0.3 * np.tanh(a2[:, :E]), a2[:, E:]
    for got, want, three_step in ((s1, s_ref, s0), (h1, h_ref, h0)):
        # float32 sums in channel order (two halves of 256) against the split
        # bf16 tensor-core GEMM: both at float32 rounding of K = 512 sums
        err_f, err_3 = rel(got, want), rel(three_step, want)
        assert err_f < max(4 * err_3, 3e-5), (err_f, err_3)
    tol = {torch.float16: 2e-3, torch.bfloat16: 1.6e-2}[dt]  # a few output ulps
    assert rel(y, y0.float().cpu().numpy()) < tol


@pytest.mark.parametrize("M,K,N", [(256, 512, 50257), (5, 2048, 1000), (300, 64, 40)])
def test_linear_split_tc_matches_float64_like_linear_split(M, K, N):
    """The split-bf16 float32 GEMM on tcgen05 (one GEMM with K tripled; odd N,
    ragged tiles) against float64, as accurate as the mma.sync split kernel."""
    from walsh_research_b200 import ops
    rng = np.random.default_rng(M + K + N)
    x = rng.normal(size=(M, K)).astype(np.float32)
    w = (rng.normal(size=(N, K)) * 0.02).astype(np.float32)
    ref = x.astype(np.float64) @ w.astype(np.float64).T
    y_tc = ops.linear_split_tc(T(x), ops.split3_weights(T(w)))
    y_mma = ops.linear_split(T(x), *ops.split_bf16(T(w)))
    err_tc, err_mma = rel(y_tc, ref), rel(y_mma, ref)
    assert err_tc < max(2 * err_mma, 1e-5), (err_tc, err_mma)


# ---------------------------------------------------------------------------
# whole model
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("name", ["model_h512", "model_h512_noscale", "model_h2048"])
def test_model_fp32_matches_reference(name):
    cfg, n, idx, sd, model = build_model(name)
    g = golden(name)
    with torch.no_grad():
        logits, _, h = model(T(idx, torch.int64), return_hidden=True)
        logits_last, _ = model(T(idx, torch.int64))
    assert rel(h, g["hidden"]) < 1e-4
    assert rel(logits, g["logits"]) < 1e-4
    assert rel(logits_last, g["logits"]) < 1e-4
    if "router_mask" in g.files:
        for l, layer in enumerate(model.layers):
            mask = layer.feed_forward._last_expert_mask.cpu().numpy().astype(np.uint8)
            assert np.array_equal(mask, g["router_mask"][l]), l
    model.check_token_ids()


def _bf16_model_check(name, idx=None, cfg_override=None):
    """bf16 forward vs the oracle run with the GPU's own expert selections
    forced: selections may differ from the float32 reference only on near-ties
    (k-th/(k+1)-th probability gap < 5e-3), logits within 2e-2 max-abs."""
    from walsh_research_b200.model import WalshConfig, mHCWalsh
    cfg, n, idx0, sd = cases.model_inputs(name)
    idx = idx0 if idx is None else idx
    cfg = dict(cfg, **(cfg_override or {}))
    model = mHCWalsh(WalshConfig(**cfg), n_streams=n)
    model.load_state_dict({k: torch.from_numpy(np.array(v)) for k, v in sd.items()}, strict=False)
    model = model.to(DEV).eval()
    model.compute_dtype = torch.bfloat16
    with torch.no_grad():
        logits, _ = model(T(idx, torch.int64))
    masks = [layer.feed_forward._last_expert_mask.cpu().numpy() for layer in model.layers]
    trace = {}
    ref_logits, _ = O.mhc_walsh_forward(cfg, sd, idx, n, trace=trace, forced_masks=masks)
    k = cfg["moe_max_experts"]
    for l, m in enumerate(masks):
        probs = np.asarray(trace["router_probs"][l])
        srt = -np.sort(-probs, axis=-1)
        gap = srt[..., k - 1] - srt[..., k]
        order = np.argsort(-probs, axis=-1, kind="stable")[..., :k]
        own = np.zeros_like(probs)
        np.put_along_axis(own, order, 1.0, axis=-1)
        differs = (own != m).any(-1)
        assert not (differs & (gap > 5e-3)).any(), f"layer {l}: selection differs away from a near-tie"
        assert differs.mean() < 0.05
    err = float(np.abs(logits.cpu().numpy() - ref_logits).max())
    assert err < 2e-2, err


def test_model_bf16_matches_reference():
    _bf16_model_check("model_h512")


def test_model_bf16_walsh2048():
    """C = 2048 (64 heads of 32, 64 experts) in 16-bit mode: the tcgen05 q/k/v
    GEMM (hd-32 RoPE epilogue) and folded output GEMM with the site epilogue,
    the CUDA-core MoE and mapping kernels and the hd-32 attention."""
    _bf16_model_check("model_h2048")


def test_model_bf16_larger_batch():
    idx = np.random.default_rng(31).integers(0, 50257, (4, 200))
    _bf16_model_check("model_h512", idx=idx, cfg_override={"block_size": 256})


def test_model_bf16_prefill_sized_batch():
    """B10 x T1000: enough tokens for the prefill-shaped (tensor-core, 128
    tokens per CTA) map and MoE kernels and the four-warp q/k/v and output
    kernels, which smaller batches do not reach."""
    idx = np.random.default_rng(37).integers(0, 50257, (10, 1000))
    _bf16_model_check("model_h512", idx=idx, cfg_override={"block_size": 1024})


def test_model_cuda_graph_replay_equals_eager():
    """enable_cuda_graphs: first call eager, second captured, later calls
    replayed; every call's logits equal the eager forward on the same ids
    (same kernels), fresh ids reach the replayed graph, an in-place weight
    update forces a new capture, and disabling restores the eager path."""
    cfg, n, idx, sd, model = build_model("model_h512", torch.bfloat16)
    rng = np.random.default_rng(41)
    ids = [T(rng.integers(0, cfg["vocab_size"], idx.shape), torch.int64) for _ in range(4)]
    with torch.no_grad():
        eager = [model(i)[0].clone() for i in ids]
        model.enable_cuda_graphs()
        for rep in range(2):
            for i, e in zip(ids, eager):
                lg, loss = model(i)
                assert loss is None
                assert rel(lg, e.cpu().numpy()) < 1e-6
        model.output.weight.mul_(1.5)          # tied embedding: changes the table and the head
        after = [model(ids[0])[0] for _ in range(3)]   # eager, capture, replay
        model.enable_cuda_graphs(False)
        ref = model(ids[0])[0]
    for lg in after:
        assert rel(lg, ref.cpu().numpy()) < 1e-6
    assert rel(ref, eager[0].cpu().numpy()) > 1e-3


def test_model_autocast_selects_bf16():
    cfg, n, idx, sd, model = build_model("model_h512")
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        logits, _ = model(T(idx, torch.int64))
    g = golden("model_h512")
    assert float(np.abs(logits.cpu().numpy() - g["logits"]).max()) < 2e-2


def test_model_larger_batch_vs_oracle():
    """B4 x T96 (several attention tiles, chmod chunks) against the oracle."""
    cfg, n, _, sd, model = build_model("model_h512")
    cfg = dict(cfg, block_size=128)
    from walsh_research_b200.model import WalshConfig, mHCWalsh
    model = mHCWalsh(WalshConfig(**cfg), n_streams=n)
    model.load_state_dict({k: torch.from_numpy(np.array(v)) for k, v in sd.items()}, strict=False)
    model = model.to(DEV).eval()
    idx = np.random.default_rng(8).integers(0, cfg["vocab_size"], (4, 96))
    with torch.no_grad():
        logits, _, h = model(T(idx, torch.int64), return_hidden=True)
    ref_logits, ref_h = O.mhc_walsh_forward(cfg, sd, idx, n)
    assert rel(h, ref_h) < 1e-4
    assert rel(logits, ref_logits) < 1e-4


def test_cached_decode_matches_reference():
    from walsh_research_b200.model import KVCache, WalshConfig, mHCWalsh
    cfg, n, toks, T0, steps, sd = cases.decode_inputs("decode_h512")
    model = mHCWalsh(WalshConfig(**cfg), n_streams=n)
    model.load_state_dict({k: torch.from_numpy(np.array(v)) for k, v in sd.items()}, strict=False)
    model = model.to(DEV).eval()
    C, H = cfg["n_embd"], cfg["n_head"]
    cache = KVCache(cfg["n_layer"], cfg["block_size"], H, C // H, torch.device(DEV), torch.float32)
    outs = []
    with torch.no_grad():
        lg, _ = model(T(toks[:, :T0], torch.int64), kv_cache=cache, start_pos=0)
        cache.increment(T0)
        outs.append(lg.cpu().numpy())
        for s in range(steps):
            lg, _ = model(T(toks[:, T0 + s:T0 + s + 1], torch.int64), kv_cache=cache, start_pos=cache.cached_len)
            cache.increment(1)
            outs.append(lg.cpu().numpy())
    assert rel(np.concatenate(outs, axis=1), golden("decode_h512")["logits"]) < 1e-4


def test_batched_decode_equals_per_sequence():
    """B=3 sequences decoded together equal each sequence decoded alone (B=1)."""
    from walsh_research_b200.model import KVCache, WalshConfig, mHCWalsh
    cfg, n, _, T0, steps, sd = cases.decode_inputs("decode_h512")
    model = mHCWalsh(WalshConfig(**cfg), n_streams=n)
    model.load_state_dict({k: torch.from_numpy(np.array(v)) for k, v in sd.items()}, strict=False)
    model = model.to(DEV).eval()
    C, H = cfg["n_embd"], cfg["n_head"]
    toks = np.random.default_rng(2).integers(0, cfg["vocab_size"], (3, T0 + steps))

    def run(tk):
        cache = KVCache(cfg["n_layer"], cfg["block_size"], H, C // H, torch.device(DEV), torch.float32,
                        batch_size=tk.shape[0])
        outs = []
        with torch.no_grad():
            lg, _ = model(T(tk[:, :T0], torch.int64), kv_cache=cache, start_pos=0)
            cache.increment(T0)
            outs.append(lg)
            for s in range(steps):
                lg, _ = model(T(tk[:, T0 + s:T0 + s + 1], torch.int64), kv_cache=cache, start_pos=cache.cached_len)
                cache.increment(1)
                outs.append(lg)
        return torch.cat(outs, 1).cpu().numpy()

    together = run(toks)
    for b in range(3):
        alone = run(toks[b:b + 1])
        assert rel(together[b:b + 1], alone) < 1e-5


def test_out_of_range_token_id_is_reported():
    cfg, n, idx, sd, model = build_model("model_h512")
    bad = idx.copy()
    bad[0, 3] = cfg["vocab_size"] + 5
    with torch.no_grad():
        model(T(bad, torch.int64))
    with pytest.raises(IndexError):
        model.check_token_ids()


# ---------------------------------------------------------------------------
# attention kernels directly (tensor-core bf16 path and fp32 path)
# ---------------------------------------------------------------------------

def _attn_ref(q, k, v, start_pos):
    """numpy causal attention of queries at positions start_pos.. over keys 0..start_pos+T-1."""
    B, H, Tq, D = q.shape
    Tk = start_pos + Tq
    mask = np.tril(np.ones((Tq, Tk), dtype=bool), k=start_pos)
    out = O.sdpa(q.astype(np.float64), k[:, :, :Tk].astype(np.float64), v[:, :, :Tk].astype(np.float64), mask)
    return out.transpose(0, 2, 1, 3)  # token-major [B, T, H, D]


@pytest.mark.parametrize("hd,Tq,start,ctx", [(16, 1000, 0, 1000), (32, 300, 0, 300), (16, 77, 130, 256),
                                             (32, 5, 60, 70), (16, 2, 40, 48), (16, 129, 0, 129),
                                             (16, 1999, 49, 2048), (16, 6, 0, 6)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_attention_kernel_vs_oracle(hd, Tq, start, ctx, dtype):
    from walsh_research_b200 import ops
    rng = np.random.default_rng(hd * 1000 + Tq)
    B, H = 2, 3
    q = rng.normal(size=(B, H, Tq, hd)).astype(np.float32) * 2
    k = rng.normal(size=(B, H, ctx, hd)).astype(np.float32)
    v = rng.normal(size=(B, H, ctx, hd)).astype(np.float32)
    qt, kt, vt = T(q, dtype), T(k, dtype), T(v, dtype)
    o = ops.attention(qt, kt, vt, start)
    # reference on the same (rounded) inputs
    ref = _attn_ref(qt.float().cpu().numpy(), kt.float().cpu().numpy(), vt.float().cpu().numpy(), start)
    tol = {torch.bfloat16: 1e-2, torch.float16: 3e-3, torch.float32: 1e-5}[dtype]
    assert rel(o, ref) < tol


@pytest.mark.parametrize("hd,Tq,start,ctx", [(16, 1, 1023, 1024), (32, 1, 2047, 2048), (16, 4, 3, 8),
                                             (16, 3, 500, 600), (32, 1, 0, 1), (32, 2, 130, 200),
                                             (16, 1, 4000, 4001)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_decode_attention_vs_oracle(hd, Tq, start, ctx, dtype):
    """The bandwidth decode kernel (Tq <= 4, 16-bit caches): long and short
    caches, fewer visible keys than key slots, several queries per step."""
    from walsh_research_b200 import ops
    rng = np.random.default_rng(hd * 7 + Tq * 131 + start)
    B, H = 3, 5
    q = rng.normal(size=(B, H, Tq, hd)).astype(np.float32) * 2
    k = rng.normal(size=(B, H, ctx, hd)).astype(np.float32)
    v = rng.normal(size=(B, H, ctx, hd)).astype(np.float32)
    qt, kt, vt = T(q, dtype), T(k, dtype), T(v, dtype)
    o = ops.attention(qt, kt, vt, start)
    ref = _attn_ref(qt.float().cpu().numpy(), kt.float().cpu().numpy(), vt.float().cpu().numpy(), start)
    # fp32 arithmetic on the rounded inputs; only the output rounding differs
    tol = 2e-3 if dtype == torch.float16 else 1e-2
    assert rel(o, ref) < tol


@pytest.mark.parametrize("udt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("n", [3000, 10000])
def test_moe_tensor_core_vs_oracle(udt, n):
    """16-bit MoE with the fused mHC epilogue (bf16 stream) at a decode-sized
    token count (router GEMM + warp-per-token kernel) and a prefill-sized one
    (128-token tensor-core kernel): selection sets equal the oracle's wherever
    the k-th/(k+1)-th probability gap exceeds the router's rounding error;
    outputs within 2e-2."""
    from walsh_research_b200 import ops
    d = cases.op_case("moe")
    rng = np.random.default_rng(19)
    x = rng.normal(size=(n, 512)).astype(np.float32)
    m = _moe_module(d)
    w1t, w2, gp, up, dp, gam, k, tc = m.kernel_args(udt)
    xb = T(x, udt)
    y, mask, probs, w = ops.moe(xb, w1t, w2, gp, up, dp, gam, k, want_stats=True, tc=tc)
    p = {"r.router.gate.0.weight": d["gate0"], "r.router.gate.2.weight": d["gate2"],
         "r.experts.gate_weights": d["gate_w"], "r.experts.up_weights": d["up_w"], "r.experts.down_weights": d["down_w"]}
    xr = xb.float().cpu().numpy().astype(np.float64)
    y_ref, mask_ref, probs_ref = O.moe(xr, p, "r.", 6)
    srt = -np.sort(-probs_ref, axis=-1)
    near = (srt[..., 5] - srt[..., 6]) < 5e-3
    diff = (mask.cpu().numpy() != mask_ref).any(-1)
    assert not (diff & ~near).any()
    assert diff.mean() < 0.05
    ok = ~diff
    assert np.abs(y.float().cpu().numpy() - y_ref)[ok].max() / np.abs(y_ref).max() < 2e-2
    # fused site epilogue equals post(x, y, hmix) computed from the unfused output
    xs = T(rng.normal(size=(n, 4, 512)).astype(np.float32), torch.bfloat16)
    hm = torch.rand((n, 24), device=DEV)
    fused = ops.moe(xb, w1t, w2, gp, up, dp, gam, k, fuse=(xs, hm, torch.empty_like(xs)), tc=tc)
    ref = ops.mhc_post(xs, y.to(xs.dtype), hm)
    assert rel(fused, ref.float().cpu().numpy()) < 1e-2


@pytest.mark.parametrize("udt", [torch.bfloat16, torch.float16])
def test_moe_decode_path_c2048_vs_oracle(udt):
    """C = 2048 (64 experts, top 6) through the router GEMM + warp-per-token
    kernel: the oracle run with the GPU's own selections gives the same output;
    selections differ from the oracle's own only on near-ties."""
    from walsh_research_b200 import ops
    from walsh_research_b200.model import WalshConfig
    from walsh_research_b200.model.moe import HadamardMoE
    rng = np.random.default_rng(23)
    m = HadamardMoE(WalshConfig(n_embd=2048), max_experts=6)
    with torch.no_grad():
        m.router.gate[0].weight.copy_(torch.from_numpy(rng.normal(0, 0.03, (512, 2048)).astype(np.float32)))
        m.router.gate[2].weight.copy_(torch.from_numpy(rng.normal(0, 0.1, (64, 512)).astype(np.float32)))
        for w in (m.experts.gate_weights, m.experts.up_weights, m.experts.down_weights):
            w.copy_(torch.from_numpy(rng.integers(-1, 2, tuple(w.shape)).astype(np.float32)))
    m = m.to(DEV).eval()
    n = 77
    xb = T(rng.normal(size=(n, 2048)).astype(np.float32), udt)
    w1t, w2, gp, up, dp, gam, k, tc = m.kernel_args(udt)
    y, mask, probs, w = ops.moe(xb, w1t, w2, gp, up, dp, gam, k, want_stats=True, tc=tc)
    p = {"r.router.gate.0.weight": m.router.gate[0].weight.detach().cpu().numpy(),
         "r.router.gate.2.weight": m.router.gate[2].weight.detach().cpu().numpy(),
         "r.experts.gate_weights": m.experts.gate_weights.detach().cpu().numpy(),
         "r.experts.up_weights": m.experts.up_weights.detach().cpu().numpy(),
         "r.experts.down_weights": m.experts.down_weights.detach().cpu().numpy()}
    xr = xb.float().cpu().numpy().astype(np.float64)
    mk = mask.cpu().numpy().astype(np.float64)
    assert (mk.sum(-1) == 6).all()
    y_ref, _, probs_ref = O.moe(xr, p, "r.", 6, forced_mask=mk)
    # router hidden layer stored in the operand dtype: bf16 keeps 8 bits, fp16 11
    assert np.abs(probs.cpu().numpy() - probs_ref).max() < (5e-3 if udt == torch.float16 else 2e-2)
    assert rel(y, y_ref) < 2e-2
    _, own, _ = O.moe(xr, p, "r.", 6)
    srt = -np.sort(-probs_ref, axis=-1)
    near = (srt[..., 5] - srt[..., 6]) < (5e-3 if udt == torch.float16 else 2e-2)
    assert not ((own != mk).any(-1) & ~near).any()


# ---------------------------------------------------------------------------
# tensor-core Hadamard kernels (bf16, C = 512)
# ---------------------------------------------------------------------------

def _rand_hlin(rng, latent=False):
    from walsh_research_b200.model.fht_cuda import HadamardLinear
    layer = HadamardLinear(512, 512)
    with torch.no_grad():
        layer.weight.copy_(torch.from_numpy(rng.integers(-1, 2, (32, 16, 16)).astype(np.float32)))
        layer.alpha.copy_(torch.from_numpy(rng.uniform(0.5, 1.5, (32, 16)).astype(np.float32)))
        layer.beta.copy_(torch.from_numpy(rng.uniform(0.1, 0.4, (32, 16)).astype(np.float32)))
    return layer.to(DEV)


@pytest.mark.parametrize("ntok", [1, 15, 16, 64, 4096 + 3])
def test_hadamard_linear_tc_vs_oracle(ntok):
    rng = np.random.default_rng(100 + ntok)
    layer = _rand_hlin(rng)
    x = T(rng.normal(size=(1, ntok, 512)).astype(np.float32), torch.bfloat16)
    y = layer(x)
    ref = O.hadamard_linear(x.float().cpu().numpy(), layer.weight.detach().cpu().numpy(),
                            layer.alpha.detach().cpu().numpy(), layer.beta.detach().cpu().numpy())
    assert rel(y, ref) < 2e-2


@pytest.mark.parametrize("B,Tn,ctx,start", [(2, 45, 80, 20), (10, 1000, 1100, 20)])
def test_qkv_tc_matches_fp32_path(B, Tn, ctx, start):
    """Tensor-core q/k/v + RoPE + cache write vs the fp32 kernel on the same
    inputs, at a decode-sized token count (one warp and one projection per CTA)
    and a prefill-sized one (four warps, all projections per CTA)."""
    from walsh_research_b200 import ops
    from walsh_research_b200.model.chassis import precompute_freqs_cis
    rng = np.random.default_rng(7)
    layers = [_rand_hlin(rng) for _ in range(3)]
    H, hd = 32, 16
    u = rng.normal(size=(B, Tn, 512)).astype(np.float32)
    f = precompute_freqs_cis(hd, ctx + 80)
    cos = f.real[start:start + Tn].float().contiguous().to(DEV)
    sin = f.imag[start:start + Tn].float().contiguous().to(DEV)
    outs = {}
    for dt in (torch.float32, torch.float16):
        q = torch.zeros((B, H, Tn, hd), dtype=dt, device=DEV)
        kc = torch.zeros((B, H, ctx, hd), dtype=dt, device=DEV)
        vc = torch.zeros_like(kc)
        ub = T(u, torch.float16).to(dt)
        if dt == torch.float16:
            trip = [(l.ternary_f16(),) + l.scales() for l in layers]
            ops.attn_qkv_tc(ub, H, *trip, cos, sin, start, q, kc, vc)
        else:
            trip = [(l.packed(),) + l.scales() for l in layers]
            ops.attn_qkv(ub, H, *trip, cos, sin, start, q, kc, vc)
        outs[dt] = (q, kc, vc)
    for a, b in zip(outs[torch.float16], outs[torch.float32]):
        assert rel(a, b.cpu().numpy()) < 5e-3
    # rows outside [start, start + Tn) of the caches stay untouched
    assert float(outs[torch.float16][1][:, :, :start].abs().max()) == 0.0
    assert float(outs[torch.float16][1][:, :, start + Tn:].abs().max()) == 0.0


@pytest.mark.parametrize("mix", [True, False])
@pytest.mark.parametrize("ntok", [300, 10000])
def test_attn_out_tc_matches_composition(mix, ntok):
    """head mixer + wo + site epilogue (one kernel) vs the three fp32 ops."""
    from walsh_research_b200 import ops
    from walsh_research_b200.model.fht_cuda import HadamardHeadMixerFused
    rng = np.random.default_rng(11)
    wo = _rand_hlin(rng)
    hm = HadamardHeadMixerFused(16)
    with torch.no_grad():
        hm.W.copy_(torch.from_numpy(rng.normal(0, 0.25, (32, 16, 16)).astype(np.float32)))
        hm.beta.copy_(torch.from_numpy(rng.uniform(0.2, 0.4, 16).astype(np.float32)))
    hm = hm.to(DEV)
    o = T(rng.normal(size=(ntok, 512)).astype(np.float32), torch.float16)
    xs = T(rng.normal(size=(ntok, 4, 512)).astype(np.float32), torch.bfloat16)
    hmix = torch.rand((ntok, 24), device=DEV)
    wmix, bmix = hm.weights_tc() if mix else (None, None)
    out = ops.attn_out_tc(o, wmix, bmix, wo.ternary_f16(), *wo.scales(), xs, hmix)
    assert out.dtype == torch.bfloat16
    of = o.float()
    if mix:
        of = hm.forward_tokens(of.view(ntok, 32, 16)).view(ntok, 512)
    f = wo(of)
    ref = ops.mhc_post(xs.float(), f, hmix)
    assert rel(out, ref.cpu().numpy()) < 2e-2


@pytest.mark.parametrize("M,K,N,strided", [(1, 512, 1031, False), (70, 2048, 512, True), (256, 512, 4099, False),
                                           (129, 64, 200, True)])
@pytest.mark.parametrize("xdt", [torch.float32, torch.bfloat16])
def test_linear_split_vs_float64(M, K, N, strided, xdt):
    """Split-bf16 tensor-core linear (stream_merge / logits) at float32 accuracy."""
    from walsh_research_b200 import ops
    rng = np.random.default_rng(M * 7 + K + N)
    ld = K * 3 if strided else K
    xs = rng.normal(size=(M, ld)).astype(np.float32) * 3
    w = (rng.normal(size=(N, K)) * 0.02).astype(np.float32)
    b = rng.normal(size=(N,)).astype(np.float32)
    xt = T(xs, xdt)
    hi, lo = ops.split_bf16(T(w))
    if strided:
        y = ops.linear_split(xt, hi, lo, T(b), ldx=ld, M=M)
    else:
        y = ops.linear_split(xt, hi, lo, T(b))
    xr = xt.float().cpu().numpy().astype(np.float64)[:, :K]
    ref = xr @ w.astype(np.float64).T + b
    assert rel(y, ref) < 3e-5


@pytest.mark.parametrize("D", [2048, 512, 33])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_embed_gather_rows_and_bad_index(D, dtype):
    """Embedding gather (vector path for 16-byte rows, element path otherwise):
    rows equal table[idx]; an out-of-range id gives a zero row and
    WALSH_ERR_INDEX in the status word."""
    from walsh_research_b200 import ops
    rng = np.random.default_rng(D)
    V, n = 1000, 5003
    table = T(rng.normal(size=(V, D)).astype(np.float32), dtype)
    idx = torch.from_numpy(rng.integers(0, V, size=n)).to(DEV)
    idx[17] = V + 3
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = ops.embed_gather(idx, table, err=err)
    ref = table[idx.clamp(0, V - 1)].clone()
    ref[17] = 0
    assert torch.equal(out, ref)
    assert int(err.item()) == -9
