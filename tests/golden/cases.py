"""Deterministic weights and inputs for the parity cases.

This module is test infrastructure.  It builds, from a seed alone, the state
dict (parameter name -> float32 numpy array, using the reference's parameter
names and shapes) and the inputs of every parity case, so that the golden
fixtures only have to store the reference's *outputs*.  Three consumers use
it: ``make_golden.py`` (loads the arrays into the reference's own modules and
records their outputs), the numpy oracle tests, and the GPU parity tests.

Parameter names and shapes follow the reference:
  * ``mHCWalsh`` / ``mHCLlamaBlock``     src/model/mhc.py:451-615
  * ``HadamardLinear``                    src/model/fht_cuda.py:436-487
  * ``HadamardHeadMixerFused``            src/model/fht_cuda.py:627-650
  * ``HadamardMoE`` / router / experts    src/model/moe.py:306-510
  * ``HadamardChannelModulation``         src/model/moe.py:610-679
  * ``OctonionTernaryLinearRef``          src/model/physics.py:53-64
  * ``OctonionHeadMixer``                 src/model/chassis.py:347-372
  * ``SwiGLUMLP``                         src/model/chassis.py:485-495

Distributions mirror the reference's initialisers in kind (N(0, 0.02) for
dense linears, identity patterns for stream_proj/stream_merge, ternary
latents for the algebra weights) but are perturbed (non-unit norms, random
alpha/bias/beta) so that every term of the forward pass is exercised.
"""
from __future__ import annotations

import math
import zlib

import numpy as np

# ---------------------------------------------------------------------------
# configurations
# ---------------------------------------------------------------------------

WALSH512 = dict(block_size=64, vocab_size=50257, n_layer=2, n_head=32, n_embd=512,
                dropout=0.0, bias=False, head_mixing=True, algebra="hadamard",
                hash_embeddings=False, use_moe=True, moe_threshold=0.1,
                moe_min_experts=1, moe_max_experts=6, use_channel_mod=True)

OCTO512 = dict(WALSH512, algebra="octonion", use_moe=False)

WALSH2048 = dict(WALSH512, vocab_size=4096, n_layer=1, n_head=64, n_embd=2048)

MODEL_CASES = {
    # name: (config, n_streams, B, T, weight seed, router scale)
    "model_h512": (WALSH512, 4, 2, 16, 11, 18.3),
    "model_h512_noscale": (WALSH512, 4, 2, 16, 12, 1.0),
    "model_o512": (OCTO512, 4, 2, 16, 13, 1.0),
    "model_h2048": (WALSH2048, 4, 1, 8, 14, 18.3),
}

# cached decode: prefill of T0 tokens (B=1, the reference's KV cache holds one
# sequence) followed by `steps` single-token steps.
DECODE_CASES = {
    "decode_h512": (WALSH512, 4, 8, 3, 21, 18.3),
}


def _rng(seed: int, name: str) -> np.random.Generator:
    return np.random.default_rng([seed, zlib.crc32(name.encode())])


def _ternary(rng, shape):
    return rng.integers(-1, 2, size=shape).astype(np.float32)


# ---------------------------------------------------------------------------
# parameter inventory of mHCWalsh (names/shapes exactly as the reference)
# ---------------------------------------------------------------------------

def swiglu_hidden(n_embd: int, algebra_dim: int) -> int:
    """SwiGLUMLP hidden width (src/model/chassis.py:488-491)."""
    h = int(2 * (4 * n_embd) / 3)
    return math.ceil(h / algebra_dim) * algebra_dim


def param_shapes(cfg: dict, n_streams: int) -> dict:
    C, V, n = cfg["n_embd"], cfg["vocab_size"], n_streams
    hd = C // cfg["n_head"]
    shapes = {
        "tok_embeddings.weight": (V, C),
        "stream_proj.weight": (n * C, C), "stream_proj.bias": (n * C,),
        "stream_merge.weight": (C, n * C), "stream_merge.bias": (C,),
        "norm.weight": (C,),
    }
    hadamard = cfg["algebra"] == "hadamard"
    G = 32 if hadamard else 8
    for l in range(cfg["n_layer"]):
        p = f"layers.{l}."
        shapes[p + "attention_norm.weight"] = (C,)
        shapes[p + "ffn_norm.weight"] = (C,)
        for w in ("wq", "wk", "wv", "wo"):
            if hadamard:
                shapes[p + f"attention.{w}.inner.weight"] = (32, C // 32, C // 32)
                shapes[p + f"attention.{w}.inner.alpha"] = (32, C // 32)
                shapes[p + f"attention.{w}.inner.beta"] = (32, C // 32)
            else:
                shapes[p + f"attention.{w}.weight"] = (8, C // 8, C // 8)
                shapes[p + f"attention.{w}.beta"] = (C // 8,)
        if cfg["head_mixing"]:
            shapes[p + "attention.head_mixer.W"] = (G, hd, hd)
            shapes[p + "attention.head_mixer.beta"] = (hd,)
        if cfg["use_moe"]:
            E = C // 32
            shapes[p + "feed_forward.router.gate.0.weight"] = (C // 4, C)
            shapes[p + "feed_forward.router.gate.2.weight"] = (E, C // 4)
            shapes[p + "feed_forward.experts.gate_weights"] = (E, 128, 32)
            shapes[p + "feed_forward.experts.up_weights"] = (E, 128, 32)
            shapes[p + "feed_forward.experts.down_weights"] = (E, 32, 128)
        else:
            Hd = swiglu_hidden(C, G)
            for nm, (o, i) in (("gate_proj", (Hd, C)), ("up_proj", (Hd, C)), ("down_proj", (C, Hd))):
                if hadamard:
                    shapes[p + f"feed_forward.{nm}.inner.weight"] = (32, o // 32, i // 32)
                    shapes[p + f"feed_forward.{nm}.inner.alpha"] = (32, i // 32)
                    shapes[p + f"feed_forward.{nm}.inner.beta"] = (32, o // 32)
                else:
                    shapes[p + f"feed_forward.{nm}.weight"] = (8, o // 8, i // 8)
                    shapes[p + f"feed_forward.{nm}.beta"] = (o // 8,)
        if cfg["use_channel_mod"]:
            E = C // 32
            shapes[p + "channel_mod.context_mlp.0.weight"] = (C // 4, C)
            shapes[p + "channel_mod.context_mlp.2.weight"] = (2 * E, C // 4)
            shapes[p + "channel_mod.scale_temp"] = (1,)
            shapes[p + "channel_mod_norm.weight"] = (C,)
        for site in ("attn_stream", "ffn_stream"):
            for kind, rows in (("H_pre", n), ("H_post", n), ("H_res", n * n)):
                q = p + f"{site}.{kind}."
                shapes[q + "alpha"] = ()
                shapes[q + "bias"] = (n, n) if kind == "H_res" else (1, n)
                shapes[q + "phi.weight"] = (rows, n * C)
    return shapes


def make_param(name: str, shape: tuple, seed: int, cfg: dict, n_streams: int,
               router_scale: float = 1.0) -> np.ndarray:
    rng = _rng(seed, name)
    C = cfg["n_embd"]
    hd = C // cfg["n_head"]
    n = n_streams
    if name == "tok_embeddings.weight":
        return rng.normal(0, 0.02, shape).astype(np.float32)
    if name == "stream_proj.weight":
        return (np.tile(np.eye(C, dtype=np.float32), (n, 1)) / math.sqrt(n)
                + rng.normal(0, 0.01, shape)).astype(np.float32)
    if name == "stream_merge.weight":
        return (np.tile(np.eye(C, dtype=np.float32), (1, n)) / n
                + rng.normal(0, 0.01, shape)).astype(np.float32)
    if name.endswith(("stream_proj.bias", "stream_merge.bias")):
        return rng.normal(0, 0.01, shape).astype(np.float32)
    if name.endswith("norm.weight"):
        return (1.0 + rng.normal(0, 0.1, shape)).astype(np.float32)
    if name.endswith(".inner.weight") or name.endswith("_weights") \
            or "context_mlp" in name:
        return _ternary(rng, shape)
    if name.endswith(".inner.alpha"):
        return rng.uniform(0.5, 1.5, shape).astype(np.float32)
    if name.endswith(".inner.beta"):
        # beta_init = sqrt(3/(2*in_o)) (src/model/fht_cuda.py:474-477); in_o
        # is read from the sibling weight's shape.
        wshape = param_shapes(cfg, n_streams)[name[:-len("beta")] + "weight"]
        base = math.sqrt(3.0 / (2.0 * wshape[2]))
        return (base * rng.uniform(0.8, 1.2, shape)).astype(np.float32)
    if name.endswith("head_mixer.W"):
        return rng.normal(0, 1.0 / math.sqrt(hd), shape).astype(np.float32)
    if name.endswith("head_mixer.beta"):
        return (math.sqrt(3.0 / (2.0 * hd)) * rng.uniform(0.8, 1.2, shape)).astype(np.float32)
    if name.endswith((".alpha",)) and shape == ():
        return np.array(rng.uniform(0.1, 0.5), dtype=np.float32)
    if name.endswith("H_res.bias"):
        return (2.0 * np.eye(n, dtype=np.float32) + rng.normal(0, 0.5, shape)).astype(np.float32)
    if name.endswith(("H_pre.bias", "H_post.bias")):
        return rng.normal(0, 0.5, shape).astype(np.float32)
    if name.endswith("phi.weight"):
        return rng.normal(0, 0.02, shape).astype(np.float32)
    if name.endswith("router.gate.0.weight"):
        return rng.normal(0, 0.02, shape).astype(np.float32)
    if name.endswith("router.gate.2.weight"):
        return (rng.normal(0, 0.02, shape) * router_scale).astype(np.float32)
    if name.endswith("scale_temp"):
        return np.array([0.3], dtype=np.float32)
    if name.endswith(".weight") and len(shape) == 3:   # octonion latent
        return _ternary(rng, shape)
    if name.endswith(".beta") and len(shape) == 1:     # octonion beta
        wshape = param_shapes(cfg, n_streams)[name[:-len("beta")] + "weight"]
        base = math.sqrt(3.0 / (2.0 * wshape[2]))
        return (base * rng.uniform(0.8, 1.2, shape)).astype(np.float32)
    raise KeyError(f"no generator rule for parameter {name} {shape}")


def make_state_dict(cfg: dict, n_streams: int, seed: int, router_scale: float = 1.0) -> dict:
    return {k: make_param(k, s, seed, cfg, n_streams, router_scale)
            for k, s in sorted(param_shapes(cfg, n_streams).items())}


def model_inputs(name: str):
    cfg, n, B, T, seed, rs = MODEL_CASES[name]
    idx = _rng(seed, "idx").integers(0, cfg["vocab_size"], size=(B, T)).astype(np.int64)
    return cfg, n, idx, make_state_dict(cfg, n, seed, rs)


def decode_inputs(name: str):
    cfg, n, T0, steps, seed, rs = DECODE_CASES[name]
    toks = _rng(seed, "idx").integers(0, cfg["vocab_size"], size=(1, T0 + steps)).astype(np.int64)
    return cfg, n, toks, T0, steps, make_state_dict(cfg, n, seed, rs)


# ---------------------------------------------------------------------------
# op-level cases
# ---------------------------------------------------------------------------

def op_case(name: str) -> dict:
    """Inputs and parameters of one op-level case (all float32 / int arrays)."""
    r = lambda tag: _rng(1000, name + "/" + tag)
    if name == "pack":
        return dict(w_a=_ternary(r("a"), (32, 16, 16)), w_b=_ternary(r("b"), (8, 64, 64)),
                    w_c=_ternary(r("c"), (4, 7, 12)))
    if name == "quant":
        return dict(w_unscaled=r("u").normal(0, 1, (32, 16, 16)).astype(np.float32),
                    w_scaled=r("s").normal(0, 1, (16, 128, 32)).astype(np.float32))
    if name.startswith("hlin_"):
        spec = {"hlin_512": (512, 512, (2, 8), False), "hlin_512_latent": (512, 512, (2, 8), True),
                "hlin_2048": (2048, 2048, (1, 4), False), "hlin_512x2048": (512, 2048, (1, 4), False),
                "hlin_2048x512": (2048, 512, (1, 4), False)}[name]
        fin, fout, bt, latent = spec
        in_o, out_o = fin // 32, fout // 32
        w = (r("w").normal(0, 1, (32, out_o, in_o)).astype(np.float32) if latent
             else _ternary(r("w"), (32, out_o, in_o)))
        return dict(x=r("x").normal(0, 1, bt + (fin,)).astype(np.float32), weight=w,
                    alpha=r("a").uniform(0.5, 1.5, (32, in_o)).astype(np.float32),
                    beta=(math.sqrt(3 / (2 * in_o)) * r("b").uniform(0.8, 1.2, (32, out_o))).astype(np.float32))
    if name in ("headmix", "headmix32"):
        hd, B, T = (16, 2, 8) if name == "headmix" else (32, 1, 4)
        return dict(x=r("x").normal(0, 1, (B, 32, T, hd)).astype(np.float32),
                    W=r("W").normal(0, 1 / math.sqrt(hd), (32, hd, hd)).astype(np.float32),
                    beta=(math.sqrt(3 / (2 * hd)) * r("b").uniform(0.8, 1.2, (hd,))).astype(np.float32))
    if name == "sinkhorn":
        return dict(H=r("H").normal(0, 2, (64, 4, 4)).astype(np.float32))
    if name == "mapping":
        d = dict(x=(r("x").normal(0, 1, (2, 8, 2048)) * 0.3).astype(np.float32))
        for kind, rows in (("pre", 4), ("post", 4), ("res", 16)):
            d[f"{kind}_phi"] = r(kind + "phi").normal(0, 0.02, (rows, 2048)).astype(np.float32)
            d[f"{kind}_alpha"] = np.array(r(kind + "a").uniform(0.1, 0.5), dtype=np.float32)
            d[f"{kind}_bias"] = ((2 * np.eye(4) if kind == "res" else 0)
                                 + r(kind + "b").normal(0, 0.5, (4, 4) if kind == "res" else (1, 4))).astype(np.float32)
        return d
    if name == "moe":
        C, E = 512, 16
        return dict(x=r("x").normal(0, 1, (2, 8, C)).astype(np.float32),
                    gate0=r("g0").normal(0, 0.02, (C // 4, C)).astype(np.float32),
                    gate2=(r("g2").normal(0, 0.02, (E, C // 4)) * 18.3).astype(np.float32),
                    gate_w=r("gw").normal(0, 1, (E, 128, 32)).astype(np.float32),
                    up_w=_ternary(r("uw"), (E, 128, 32)),
                    down_w=_ternary(r("dw"), (E, 32, 128)),
                    top_k=np.array(6))
    if name == "chmod":
        C, E = 512, 16
        return dict(x=r("x").normal(0, 1, (8, 6, C)).astype(np.float32),
                    w0=_ternary(r("w0"), (C // 4, C)), w2=r("w2").normal(0, 1, (2 * E, C // 4)).astype(np.float32),
                    scale_temp=np.array([0.7], dtype=np.float32))
    if name == "octo_lin":
        return dict(x=r("x").normal(0, 1, (2, 8, 512)).astype(np.float32),
                    weight=_ternary(r("w"), (8, 64, 64)),
                    beta=(math.sqrt(3 / 128) * r("b").uniform(0.8, 1.2, (64,))).astype(np.float32))
    if name == "octo_headmix":
        return dict(x=r("x").normal(0, 1, (2, 8, 8, 16)).astype(np.float32),
                    W=r("W").normal(0, 0.25, (8, 16, 16)).astype(np.float32),
                    beta=(math.sqrt(3 / 32) * r("b").uniform(0.8, 1.2, (16,))).astype(np.float32))
    if name == "hash_emb":
        V, C, nb, nt = 1000, 64, 1021, 3
        return dict(tables=r("t").normal(0, 0.02, (nt, nb, C)).astype(np.float32),
                    importance=r("i").normal(1.0, 0.1, (V, nt)).astype(np.float32),
                    x=r("x").integers(0, V, (2, 7)).astype(np.int64),
                    h=r("h").normal(0, 1, (2, 5, C)).astype(np.float32),
                    targets=r("y").integers(0, V, (2, 5)).astype(np.int64))
    raise KeyError(name)


OP_CASES = ["pack", "quant", "hlin_512", "hlin_512_latent", "hlin_2048", "hlin_512x2048",
            "hlin_2048x512", "headmix", "headmix32", "sinkhorn", "mapping", "moe", "chmod",
            "octo_lin", "octo_headmix", "hash_emb"]
