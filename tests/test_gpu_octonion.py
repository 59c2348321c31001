"""Octonion (Cayley-Dickson) path on the GPU against the reference-generated
fixtures (tests/golden) and the numpy oracle: the layer, the head mixer,
the fused GEMM epilogues (q/k/v + RoPE, SwiGLU, mHC site) and the whole
octonion Walsh-512 forward in float32 and bfloat16."""
import math

import numpy as np
import pytest
import torch

import cases
from oracle import walsh_oracle as O
from test_gpu_parity import DEV, T, golden, rel

pytestmark = pytest.mark.gpu


def _octo_layer(fin, fout, rng):
    from walsh_research_b200.model.cayley_dickson_cuda import OctonionFusedLinear
    m = OctonionFusedLinear(fin, fout)
    with torch.no_grad():
        m.weight.copy_(torch.from_numpy(rng.uniform(-1, 1, (8, fout // 8, fin // 8)).astype(np.float32)))
        m.beta.copy_(torch.from_numpy(rng.uniform(0.05, 0.2, (fout // 8,)).astype(np.float32)))
    return m.to(DEV)


def _np(m):
    return m.weight.detach().cpu().numpy(), m.beta.detach().cpu().numpy()


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 2e-5), (torch.float16, 3e-3), (torch.bfloat16, 1e-2)])
def test_octonion_linear_matches_reference(dtype, tol):
    from walsh_research_b200.model.cayley_dickson_cuda import OctonionFusedLinear
    d, g = cases.op_case("octo_lin"), golden("octo_lin")
    m = OctonionFusedLinear(512, 512)
    with torch.no_grad():
        m.weight.copy_(torch.from_numpy(d["weight"]))
        m.beta.copy_(torch.from_numpy(d["beta"]))
    m = m.to(DEV)
    x = T(d["x"], dtype)
    parts = m(tuple(x.split(64, dim=-1)))
    assert len(parts) == 8 and parts[0].shape == (2, 8, 64)
    y = torch.cat(parts, dim=-1)
    ref = g["y"] if dtype == torch.float32 else O.octonion_linear(x.float().cpu().numpy(), d["weight"], d["beta"])
    assert rel(y, ref) < tol


@pytest.mark.parametrize("M,fin,fout", [(1, 512, 512), (1000, 1368, 512), (333, 512, 1368), (130, 64, 16)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_octonion_linear_tiles_vs_oracle(M, fin, fout, dtype):
    """Ragged M/N/K tiles (K = 1368 is not a multiple of the 32-wide K stage)."""
    rng = np.random.default_rng(M + fin + fout)
    m = _octo_layer(fin, fout, rng)
    x = rng.normal(size=(M, fin)).astype(np.float32)
    xt = T(x, dtype)
    y = m.forward_flat(xt)
    w, b = _np(m)
    ref = O.octonion_linear(xt.float().cpu().numpy(), w, b)
    assert rel(y, ref) < (2e-5 if dtype == torch.float32 else 3e-3)


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 3e-5), (torch.float16, 3e-3)])
def test_octonion_head_mixer_matches_reference(dtype, tol):
    from walsh_research_b200.model.cayley_dickson_cuda import OctonionHeadMixer
    d, g = cases.op_case("octo_headmix"), golden("octo_headmix")
    m = OctonionHeadMixer(16)
    with torch.no_grad():
        m.W.copy_(torch.from_numpy(d["W"]))
        m.beta.copy_(torch.from_numpy(d["beta"]))
    m = m.to(DEV)
    x = T(d["x"], dtype)
    y = m(x)
    ref = g["y"] if dtype == torch.float32 else O.octonion_head_mixer(x.float().cpu().numpy(), d["W"], d["beta"])
    assert rel(y, ref) < tol


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_swiglu_matches_oracle(dtype):
    """SwiGLU (gate/up interleaved GEMM with the product in the epilogue, then down)."""
    from walsh_research_b200.model import WalshConfig
    from walsh_research_b200.model.cayley_dickson_cuda import SwiGLUMLP
    rng = np.random.default_rng(5)
    cfg = WalshConfig(n_embd=512, n_head=32, algebra="octonion")
    mlp = SwiGLUMLP(cfg)
    assert mlp.hidden == 1368
    with torch.no_grad():
        for lin in (mlp.gate_proj, mlp.up_proj, mlp.down_proj):
            lin.weight.copy_(torch.from_numpy(rng.uniform(-1, 1, tuple(lin.weight.shape)).astype(np.float32)))
    mlp = mlp.to(DEV)
    x = rng.normal(size=(3, 70, 512)).astype(np.float32)
    xt = T(x, dtype)
    y = mlp(xt)
    p = {f"f.{n}.{k}": getattr(getattr(mlp, n), k).detach().cpu().numpy()
         for n in ("gate_proj", "up_proj", "down_proj") for k in ("weight", "beta")}
    ref = O.swiglu({"algebra": "octonion"}, p, "f.", xt.float().cpu().numpy().astype(np.float64), np.float64)
    assert rel(y, ref) < (3e-5 if dtype == torch.float32 else 5e-3)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_octonion_qkv_matches_composition(dtype):
    """One GEMM for q/k/v with beta, RoPE and the cache write at start_pos."""
    from walsh_research_b200 import ops
    from walsh_research_b200.model import WalshConfig
    from walsh_research_b200.model.chassis import CausalSelfAttention, precompute_freqs_cis
    rng = np.random.default_rng(3)
    cfg = WalshConfig(n_embd=512, n_head=32, algebra="octonion", head_mixing=True)
    attn = CausalSelfAttention(cfg)
    with torch.no_grad():
        for lin in (attn.wq, attn.wk, attn.wv):
            lin.weight.copy_(torch.from_numpy(rng.uniform(-1, 1, (8, 64, 64)).astype(np.float32)))
    attn = attn.to(DEV)
    B, Tn, H, hd, ctx, start = 2, 37, 32, 16, 64, 11
    u = T(rng.normal(size=(B, Tn, 512)).astype(np.float32), dtype)
    f = precompute_freqs_cis(hd, 128)
    cos, sin = f.real[start:start + Tn].float().contiguous().to(DEV), f.imag[start:start + Tn].float().contiguous().to(DEV)
    q = torch.zeros((B, H, Tn, hd), dtype=dtype, device=DEV)
    kc = torch.zeros((B, H, ctx, hd), dtype=dtype, device=DEV)
    vc = torch.zeros_like(kc)
    attn._octonion_qkv(u, cos, sin, start, q, kc, vc)
    un = u.float().cpu().numpy().astype(np.float64)
    c, s = cos.cpu().numpy(), sin.cpu().numpy()
    for lin, out, rope, rows in ((attn.wq, q, True, slice(0, Tn)), (attn.wk, kc, True, slice(start, start + Tn)),
                                 (attn.wv, vc, False, slice(start, start + Tn))):
        w, b = _np(lin)
        r = O.octonion_linear(un, w, b).reshape(B, Tn, H, hd)
        if rope:
            r = O.apply_rope(r, c, s)
        got = out[:, :, rows].float().cpu().numpy().transpose(0, 2, 1, 3)
        assert rel(got, r) < (3e-5 if dtype == torch.float32 else 3e-3)
    assert float(kc[:, :, :start].abs().max()) == 0.0 and float(kc[:, :, start + Tn:].abs().max()) == 0.0


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_octonion_post_epilogue(dtype):
    """f = beta . (a W^T) then x' = H_res x + H_post f, in place on the stream state."""
    from walsh_research_b200 import ops
    rng = np.random.default_rng(13)
    m = _octo_layer(512, 512, rng)
    ntok = 300
    a = T(rng.normal(size=(ntok, 512)).astype(np.float32), dtype)
    xdt = torch.float32 if dtype == torch.float32 else torch.bfloat16
    xs = T(rng.normal(size=(ntok, 4, 512)).astype(np.float32), xdt)
    hmix = torch.rand((ntok, 24), device=DEV)
    xin = xs.clone()
    ops.octo_post(a, m.operands(a.dtype), m.scale(), xs, hmix, out=xs)
    f = m.forward_flat(a).float()
    ref = ops.mhc_post(xin.float(), f, hmix)
    assert rel(xs, ref.cpu().numpy()) < (1e-5 if dtype == torch.float32 else 1e-2)


def _octo_model(dtype=torch.float32, cfg_override=None):
    from walsh_research_b200.model import WalshConfig, mHCWalsh
    cfg, n, idx, sd = cases.model_inputs("model_o512")
    cfg = dict(cfg, **(cfg_override or {}))
    model = mHCWalsh(WalshConfig(**cfg), n_streams=n)
    missing, unexpected = model.load_state_dict({k: torch.from_numpy(np.array(v)) for k, v in sd.items()},
                                                strict=False)
    assert not unexpected
    # buffers and the output projection tied to tok_embeddings
    assert all(k in ("freqs_cis", "output.weight") or k.endswith((".H", ".signs", ".widx")) for k in missing), missing
    model = model.to(DEV).eval()
    model.compute_dtype = dtype
    return cfg, n, idx, sd, model


def test_octonion_model_fp32_matches_reference():
    cfg, n, idx, sd, model = _octo_model()
    g = golden("model_o512")
    with torch.no_grad():
        logits, _, h = model(T(idx, torch.int64), return_hidden=True)
    assert rel(h, g["hidden"]) < 1e-4
    assert rel(logits, g["logits"]) < 1e-4


def test_octonion_model_bf16_matches_reference():
    cfg, n, idx, sd, model = _octo_model(torch.bfloat16)
    g = golden("model_o512")
    with torch.no_grad():
        logits, _ = model(T(idx, torch.int64))
    assert float(np.abs(logits.cpu().numpy() - g["logits"]).max()) < 2e-2


def test_octonion_model_larger_batch_vs_oracle():
    """B3 x T64 in both precisions against the float64 oracle."""
    cfg, n, _, sd, model = _octo_model()
    idx = np.random.default_rng(17).integers(0, cfg["vocab_size"], (3, 64))
    ref_logits, ref_h = O.mhc_walsh_forward(cfg, sd, idx, n)
    with torch.no_grad():
        logits, _, h = model(T(idx, torch.int64), return_hidden=True)
        assert rel(h, ref_h) < 1e-4
        assert rel(logits, ref_logits) < 1e-4
        model.compute_dtype = torch.bfloat16
        lb, _ = model(T(idx, torch.int64))
    assert float(np.abs(lb.cpu().numpy() - ref_logits).max()) < 2e-2


def test_octonion_cached_decode_matches_oracle():
    """Prefill of 9 tokens then 3 single-token steps through the batched KV
    cache, against the oracle's batch-1 cached decode of each sequence (the
    reference's KVCache semantics: channel modulation pools over the tokens
    of each call, so a cached step differs from a full re-forward)."""
    from walsh_research_b200.model import KVCache
    cfg, n, _, sd, model = _octo_model()
    idx = np.random.default_rng(23).integers(0, cfg["vocab_size"], (2, 12))
    it = T(idx, torch.int64)
    H, C, L = cfg["n_head"], cfg["n_embd"], cfg["n_layer"]
    kv = KVCache(L, 32, H, C // H, DEV, dtype=torch.float32, batch_size=2)
    outs = []
    with torch.no_grad():
        lg, _ = model(it[:, :9], kv_cache=kv, start_pos=0)
        kv.increment(9)
        outs.append(lg.cpu().numpy())
        for t in range(9, 12):
            lg, _ = model(it[:, t:t + 1], kv_cache=kv, start_pos=t)
            kv.increment(1)
            outs.append(lg.cpu().numpy())
    got = np.concatenate(outs, axis=1)
    for b in range(2):
        cache = O.KVCache(L, 32, H, C // H)
        ref = [O.mhc_walsh_forward(cfg, sd, idx[b:b + 1, :9], n, cache=cache, start_pos=0)[0]]
        cache.increment(9)
        for t in range(9, 12):
            ref.append(O.mhc_walsh_forward(cfg, sd, idx[b:b + 1, t:t + 1], n, cache=cache, start_pos=t)[0])
            cache.increment(1)
        assert rel(got[b:b + 1], np.concatenate(ref, axis=1)) < 1e-4
