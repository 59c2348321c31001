"""CPU oracle: a numpy restatement of Walsh's forward hot path.

TEST INFRASTRUCTURE ONLY.  This module is the checker the parity tests (and
the CPU-baseline leg of ``bench.py``) compare the CUDA path against.  The
product path (``walsh_research_b200``) never imports it.

Each function restates one piece of the reference (pulseofthemachine/
Walsh-Research, ``src/model/*.py``) and cites the lines it follows.  Arrays
are numpy; computation runs in ``float64`` by default (pass ``dtype=np.float32``
for the faster single-precision variant used as the CPU baseline).  The
oracle is pinned against golden fixtures produced by running the reference's
own PyTorch code (``tests/golden/make_golden.py``).

State dicts are ``{parameter name: ndarray}`` with the reference's names.
"""
from __future__ import annotations

import math

import numpy as np

F32_EPS = float(np.finfo(np.float32).eps)

# Cayley-Dickson tables (src/model/constants.py:15-52)
SIGN_TABLE = np.array([
    [+1, -1, -1, -1, -1, -1, -1, -1],
    [+1, +1, +1, -1, +1, -1, -1, +1],
    [+1, -1, +1, +1, +1, +1, -1, -1],
    [+1, +1, -1, +1, +1, -1, +1, -1],
    [+1, -1, -1, -1, +1, +1, +1, +1],
    [+1, +1, -1, +1, -1, +1, -1, +1],
    [+1, +1, +1, -1, -1, +1, +1, -1],
    [+1, -1, +1, +1, -1, -1, +1, +1]], dtype=np.int64)
WEIGHT_IDX = np.array([
    [0, 1, 2, 3, 4, 5, 6, 7],
    [1, 0, 3, 2, 5, 4, 7, 6],
    [2, 3, 0, 1, 6, 7, 4, 5],
    [3, 2, 1, 0, 7, 6, 5, 4],
    [4, 5, 6, 7, 0, 1, 2, 3],
    [5, 4, 7, 6, 1, 0, 3, 2],
    [6, 7, 4, 5, 2, 3, 0, 1],
    [7, 6, 5, 4, 3, 2, 1, 0]], dtype=np.int64)


# ---------------------------------------------------------------------------
# ternary weights
# ---------------------------------------------------------------------------

def hadamard_matrix(n: int = 32, normalize: bool = True, dtype=np.float64) -> np.ndarray:
    """Sylvester Hadamard matrix (src/model/fht_cuda.py:32-56)."""
    H = np.ones((1, 1), dtype=dtype)
    while H.shape[0] < n:
        H = np.block([[H, H], [H, -H]])
    return H / math.sqrt(n) if normalize else H


def pack_ternary(w: np.ndarray) -> np.ndarray:
    """2-bit packing, -1->00, 0->01, +1->10, MSB first (src/model/fht_cuda.py:65-93).

    When the last dimension is not a multiple of 4 it is padded with zeros
    (code 01) up to the next multiple; for multiples of 4 the output is the
    reference's byte layout exactly."""
    w = np.asarray(w)
    K = w.shape[-1]
    Kp = (K + 3) // 4 * 4
    code = np.ones(w.shape[:-1] + (Kp,), dtype=np.uint8)
    code[..., :K] = (w.astype(np.int64) + 1).astype(np.uint8)
    code = code.reshape(w.shape[:-1] + (Kp // 4, 4))
    return ((code[..., 0] << 6) | (code[..., 1] << 4) | (code[..., 2] << 2) | code[..., 3]).astype(np.uint8)


def unpack_ternary(packed: np.ndarray, k: int) -> np.ndarray:
    """Inverse of :func:`pack_ternary` (src/model/fht_cuda.py:96-117)."""
    p = np.asarray(packed).astype(np.int64)
    v = np.stack([((p >> s) & 3) - 1 for s in (6, 4, 2, 0)], axis=-1)
    return v.reshape(p.shape[:-1] + (p.shape[-1] * 4,))[..., :k].astype(np.float32)


def bitmask_ternary_decode(bitmask: bytes, sign_bits: bytes, shape, num_nonzero: int) -> np.ndarray:
    """Ternary weights from the .walsh v4 bitmask + sign form
    (generate_compressed.py:70-105; written by compress.py:36-93): bit b of
    bitmask byte i marks position 8 i + b non-zero; the j-th non-zero (in
    position order) is +1 when bit j % 8 of sign byte j // 8 is set, else -1."""
    total = int(np.prod(shape))
    nz = np.unpackbits(np.frombuffer(bitmask, dtype=np.uint8), bitorder="little")[:total].astype(bool)
    signs = np.unpackbits(np.frombuffer(sign_bits, dtype=np.uint8), bitorder="little")[:num_nonzero]
    out = np.zeros(total, dtype=np.float32)
    pos = np.flatnonzero(nz)[:num_nonzero]
    out[pos] = np.where(signs[: len(pos)] == 1, 1.0, -1.0)
    return out.reshape(shape)


def absmean_gamma(w: np.ndarray) -> np.float32:
    """gamma = mean(|W|) + 1e-8 in float32 (src/model/physics.py:23-25, src/model/moe.py:277-279)."""
    return np.float32(np.abs(np.asarray(w, dtype=np.float64)).mean()) + np.float32(1e-8)


def quantize_ternary(w: np.ndarray) -> np.ndarray:
    """Unscaled BitNet absmean ternary: clamp(round_half_even(W/gamma), -1, 1)
    (src/model/physics.py:13-51).  The reference's STE returns
    ``w_c + (w_q - w_c).detach()`` whose value is w_q up to one float32 ulp."""
    w32 = np.asarray(w, dtype=np.float32)
    return np.clip(np.round(w32 / absmean_gamma(w32)), -1, 1).astype(np.float32)


def quantize_ternary_scaled(w: np.ndarray) -> np.ndarray:
    """Scaled ternary ``q * gamma`` with one gamma per tensor (src/model/moe.py:268-303)."""
    w32 = np.asarray(w, dtype=np.float32)
    g = absmean_gamma(w32)
    return (np.clip(np.round(w32 / g), -1, 1) * g).astype(np.float32)


# ---------------------------------------------------------------------------
# elementary ops
# ---------------------------------------------------------------------------

def silu(x):
    return x / (1.0 + np.exp(-x))


def sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def softmax(x, axis=-1):
    m = x.max(axis=axis, keepdims=True)
    e = np.exp(x - m)
    return e / e.sum(axis=axis, keepdims=True)


def rmsnorm(x, weight, eps=1e-6):
    """Chassis RMSNorm with weight, eps 1e-6 (src/model/chassis.py:96-106)."""
    return x / np.sqrt((x * x).mean(-1, keepdims=True) + eps) * weight


def rms_norm_plain(x, eps=F32_EPS):
    """``F.rms_norm`` without weight, eps = finfo(float32).eps (src/model/mhc.py:291)."""
    return x / np.sqrt((x * x).mean(-1, keepdims=True) + eps)


def hadamard_linear(x, w_latent, alpha, beta, dtype=np.float64):
    """HadamardLinear.forward: y = beta * H . W_t . H . (alpha * x)
    (src/model/fht_cuda.py:489-519).  ``w_latent`` is quantised with the
    unscaled ternary quantiser (src/model/physics.py:42-51)."""
    G = 32
    x = np.asarray(x, dtype=dtype)
    lead = x.shape[:-1]
    in_o = x.shape[-1] // G
    wq = quantize_ternary(w_latent).astype(dtype)
    out_o = wq.shape[1]
    H = hadamard_matrix(G, dtype=dtype)
    xs = x.reshape(-1, G, in_o) * alpha.astype(dtype)
    xm = np.matmul(H.T, xs)                                   # sum_g H[g,h] xs[g,i]
    yp = np.matmul(xm.transpose(1, 0, 2), wq.transpose(0, 2, 1)).transpose(1, 0, 2)  # per-group W_g
    ym = np.matmul(H.T, yp)
    return (ym * beta.astype(dtype)).reshape(lead + (G * out_o,))


def hadamard_head_mixer(x, W, beta, dtype=np.float64):
    """HadamardHeadMixerFused.forward on [B, 32, T, hd]
    (src/model/fht_cuda.py:652-670)."""
    x = np.asarray(x, dtype=dtype)
    H = hadamard_matrix(32, dtype=dtype)
    B, _, Tn, D = x.shape
    xf = np.matmul(H.T, x.reshape(B, 32, Tn * D)).reshape(B, 32, Tn, D)
    y = np.matmul(xf, W.astype(dtype)[None])                  # per-head W_h
    yf = np.matmul(H.T, y.reshape(B, 32, Tn * D)).reshape(B, 32, Tn, D)
    return yf * beta.astype(dtype)


def octonion_linear(x, w_latent, beta, dtype=np.float64):
    """OctonionTernaryLinearRef.forward on the concatenation of the 8 parts:
    y_i = beta * sum_j SIGN[i,j] x_j @ Wq[WIDX[i,j]]^T (src/model/physics.py:66-82)."""
    x = np.asarray(x, dtype=dtype)
    in_o = x.shape[-1] // 8
    wq = quantize_ternary(w_latent).astype(dtype)
    parts = [x[..., j * in_o:(j + 1) * in_o] for j in range(8)]
    ys = []
    for i in range(8):
        acc = 0
        for j in range(8):
            acc = acc + SIGN_TABLE[i, j] * (parts[j] @ wq[WEIGHT_IDX[i, j]].T)
        ys.append(acc * beta.astype(dtype))
    return np.concatenate(ys, axis=-1)


def octonion_head_mixer(x, W, beta, dtype=np.float64):
    """OctonionHeadMixer.forward on [B, 8, T, hd]: y_i = beta * sum_j s_ij x_j @ W[widx_ij]
    (src/model/chassis.py:374-399; note x @ W, not W^T)."""
    x = np.asarray(x, dtype=dtype)
    W = W.astype(dtype)
    out = []
    for i in range(8):
        acc = 0
        for j in range(8):
            acc = acc + SIGN_TABLE[i, j] * (x[:, j] @ W[WEIGHT_IDX[i, j]])
        out.append(acc * beta.astype(dtype))
    return np.stack(out, axis=1)


def precompute_rope(hd: int, end: int):
    """cos/sin of the RoPE table, theta = 1e4, computed in float32 like
    ``precompute_freqs_cis`` (src/model/chassis.py:332-337)."""
    k = np.arange(0, hd, 2, dtype=np.float32)[: hd // 2] / np.float32(hd)
    freqs = (np.float32(1.0) / (np.float32(10000.0) ** k)).astype(np.float32)
    ang = np.outer(np.arange(end, dtype=np.float32), freqs).astype(np.float32)
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def apply_rope(x, cos, sin):
    """Interleaved complex-pair rotation of [B, T, H, hd] (src/model/chassis.py:339-345)."""
    xr, xi = x[..., 0::2], x[..., 1::2]
    c, s = cos[None, :, None, :], sin[None, :, None, :]
    out = np.empty_like(x)
    out[..., 0::2] = xr * c - xi * s
    out[..., 1::2] = xr * s + xi * c
    return out


_POOL = None


def _pool():
    global _POOL
    if _POOL is None:
        import concurrent.futures as cf
        import os
        _POOL = cf.ThreadPoolExecutor(max_workers=os.cpu_count() or 1)
    return _POOL


def sdpa(q, k, v, mask, block=256):
    """scaled_dot_product_attention with a boolean keep-mask [Tq, Tk]; q,k,v [B, H, T, hd].
    Evaluated per (batch, head) in query blocks over each block's visible key
    prefix (numpy releases the GIL, so heads run on all host threads)."""
    B, H, Tq, D = q.shape
    scale = 1.0 / math.sqrt(D)
    out = np.empty(q.shape[:-1] + (v.shape[-1],), dtype=np.result_type(q, v))
    last = np.where(mask.any(1), mask.shape[1] - 1 - np.argmax(mask[:, ::-1], axis=1), -1)

    def one(bh):
        b, h = divmod(bh, H)
        for q0 in range(0, Tq, block):
            q1 = min(Tq, q0 + block)
            kend = int(last[q0:q1].max()) + 1
            s = (q[b, h, q0:q1] @ k[b, h, :kend].T) * scale
            s = np.where(mask[q0:q1, :kend], s, -np.inf)
            out[b, h, q0:q1] = softmax(s, -1) @ v[b, h, :kend]

    list(_pool().map(one, range(B * H)))
    return out


def sinkhorn(Hm, n_iter=20, eps=1e-8):
    """SinkhornKnopp.forward: exp, then n_iter x (column, row) normalisation
    (src/model/mhc.py:214-229)."""
    M = np.exp(Hm)
    for _ in range(n_iter):
        M = M / (M.sum(-2, keepdims=True) + eps)
        M = M / (M.sum(-1, keepdims=True) + eps)
    return M


def stream_mapping(x_flat, phi, alpha, bias, kind, n=4):
    """ResidualStreamMapping.forward (src/model/mhc.py:283-318).
    Returns [.., 1, n] for 'pre'/'post' and [.., n, n] for 'res'."""
    d = rms_norm_plain(x_flat) @ phi.T
    if kind == "res":
        Ht = alpha * d.reshape(d.shape[:-1] + (n, n)) + bias
        return sinkhorn(Ht)
    Ht = alpha * d + bias.reshape(-1)
    s = sigmoid(Ht)[..., None, :]
    return s if kind == "pre" else 2.0 * s


def router(x, w0, w2, top_k, threshold=None, min_experts=1):
    """HadamardRouter.forward (src/model/moe.py:418-447): softmax(W2 SiLU(W1 x)),
    top-k mask (ties to the lower expert index), renormalised weights.

    With ``threshold`` set: the threshold rule that HadamardRouter's docstring
    and arguments describe (src/model/moe.py:383-403) but its forward does not
    run -- every expert with p > threshold, at least ``min_experts`` and at most
    top_k of them, taken in descending probability (ties to the lower index)."""
    probs = softmax(silu(x @ w0.T) @ w2.T, -1)
    E = probs.shape[-1]
    k = min(top_k, E)
    order = np.argsort(-probs, axis=-1, kind="stable")[..., :k]
    if threshold is None:
        take = np.ones(order.shape, dtype=bool)
    else:
        above = (probs > threshold).sum(-1, keepdims=True)
        kt = np.clip(above, min_experts, k)
        take = np.arange(k) < kt
    mask = np.zeros_like(probs)
    np.put_along_axis(mask, order, take.astype(probs.dtype), axis=-1)
    masked = probs * mask
    weights = masked / np.maximum(masked.sum(-1, keepdims=True), 1e-8)
    return weights, mask, probs


def experts(xb, weights, gate_w, up_w, down_w):
    """FastMoEExperts.forward (src/model/moe.py:337-380): scaled-ternary SwiGLU
    per 32-wide block over all experts, times the routing weight."""
    dt = xb.dtype
    g = quantize_ternary_scaled(gate_w).astype(dt)
    u = quantize_ternary_scaled(up_w).astype(dt)
    dw = quantize_ternary_scaled(down_w).astype(dt)
    lead, E = xb.shape[:-2], xb.shape[-2]
    xe = xb.reshape(-1, E, xb.shape[-1]).transpose(1, 0, 2)          # [E, N, 32]
    gate = np.matmul(xe, g.transpose(0, 2, 1))                        # [E, N, 128]
    up = np.matmul(xe, u.transpose(0, 2, 1))
    out = np.matmul(silu(gate) * up, dw.transpose(0, 2, 1))           # [E, N, 32]
    out = out.transpose(1, 0, 2).reshape(lead + (E, -1))
    return out * weights[..., None]


def moe(x, p, prefix, top_k, forced_mask=None, threshold=None, min_experts=1):
    """HadamardMoE.forward (src/model/moe.py:512-542).  ``forced_mask`` (test
    hook) replaces the top-k selection with a given 0/1 mask; ``threshold``
    selects the router's threshold rule (see ``router``)."""
    C = x.shape[-1]
    E = C // 32
    w, mask, probs = router(x, p[prefix + "router.gate.0.weight"], p[prefix + "router.gate.2.weight"], top_k,
                            threshold, min_experts)
    if forced_mask is not None:
        masked = probs * forced_mask
        w = masked / np.maximum(masked.sum(-1, keepdims=True), 1e-8)
        mask = forced_mask
    out = experts(x.reshape(x.shape[:-1] + (E, 32)), w, p[prefix + "experts.gate_weights"],
                  p[prefix + "experts.up_weights"], p[prefix + "experts.down_weights"])
    return out.reshape(x.shape), mask, probs


def channel_mod(x, w0, w2, scale_temp, residual_scale=0.5):
    """HadamardChannelModulation.forward on [B', T, C] (src/model/moe.py:681-762):
    bulk mean over T, scaled-ternary MLP, scale = 1 + clamp(temp, .1, .5) tanh,
    out = x + r (x*scale + 0.1*shift - x) per 32-wide block."""
    Bp, T, C = x.shape
    nb = C // 32
    dt = x.dtype
    bulk = x.mean(axis=1)
    h = silu(bulk @ quantize_ternary_scaled(w0).astype(dt).T)
    mods = h @ quantize_ternary_scaled(w2).astype(dt).T
    raw, shift = mods[:, :nb], mods[:, nb:]
    st = float(np.clip(np.asarray(scale_temp, dtype=np.float64).reshape(-1)[0], 0.1, 0.5))
    scale = 1.0 + st * np.tanh(raw)
    xb = x.reshape(Bp, T, nb, 32)
    xm = xb * scale[:, None, :, None] + shift[:, None, :, None] * 0.1
    return (xb + residual_scale * (xm - xb)).reshape(Bp, T, C)


# ---------------------------------------------------------------------------
# model
# ---------------------------------------------------------------------------

class KVCache:
    """Batch-1 KV cache (src/model/chassis.py:262-330): [max_len, H, hd] per layer."""

    def __init__(self, n_layers, max_len, n_head, hd, dtype=np.float64):
        self.k = [np.zeros((max_len, n_head, hd), dtype) for _ in range(n_layers)]
        self.v = [np.zeros((max_len, n_head, hd), dtype) for _ in range(n_layers)]
        self.cached_len = 0

    def update(self, l, k, v):
        s, e = self.cached_len, self.cached_len + k.shape[1]
        self.k[l][s:e] = k[0]
        self.v[l][s:e] = v[0]
        return self.k[l][:e][None], self.v[l][:e][None]

    def increment(self, n=1):
        self.cached_len += n


def hash_embedding_matrix(tables, importance, indices, n_embd):
    """HashEmbedding._get_chunk_embeddings over the whole vocabulary
    (src/model/chassis.py:175-191): row v = sqrt(n_embd) * sum_i
    importance[v, i] * tables[i][indices[v, i]], summed table by table."""
    out = np.zeros((importance.shape[0], n_embd), dtype=np.result_type(tables, importance))
    for i in range(tables.shape[0]):
        out = out + tables[i][indices[:, i]] * importance[:, i:i + 1]
    return out * out.dtype.type(math.sqrt(n_embd))


def hash_indices(hash_a, hash_b, prime, vocab_size, bucket_size):
    """((a v + b) mod p) mod buckets for every token v, [V, num_tables]
    (src/model/chassis.py:141-148)."""
    v = np.arange(vocab_size, dtype=np.int64)
    return (((v[None, :] * np.asarray(hash_a).reshape(-1, 1) + np.asarray(hash_b).reshape(-1, 1)) % int(prime))
            % bucket_size).T


def _embedding(cfg, p):
    if cfg.get("hash_embeddings"):
        nt = sum(1 for k in p if k.startswith("tok_embeddings.emb_tables."))
        tables = np.stack([p[f"tok_embeddings.emb_tables.{i}.weight"] for i in range(nt)])
        return hash_embedding_matrix(tables, p["tok_embeddings.importance.weight"],
                                     np.asarray(p["tok_embeddings.all_indices"]).astype(np.int64), cfg["n_embd"])
    return p["tok_embeddings.weight"]


def _algebra_linear(cfg, p, name, x, dtype):
    if cfg["algebra"] == "hadamard":
        return hadamard_linear(x, p[name + ".inner.weight"], p[name + ".inner.alpha"],
                               p[name + ".inner.beta"], dtype)
    return octonion_linear(x, p[name + ".weight"], p[name + ".beta"], dtype)


def attention(cfg, p, prefix, x, cos, sin, cache=None, layer=0, dtype=np.float64):
    """CausalSelfAttention.forward (src/model/chassis.py:424-483)."""
    B, T, C = x.shape
    H = cfg["n_head"]
    hd = C // H
    q = _algebra_linear(cfg, p, prefix + "wq", x, dtype).reshape(B, T, H, hd)
    k = _algebra_linear(cfg, p, prefix + "wk", x, dtype).reshape(B, T, H, hd)
    v = _algebra_linear(cfg, p, prefix + "wv", x, dtype).reshape(B, T, H, hd)
    q, k = apply_rope(q, cos, sin), apply_rope(k, cos, sin)
    cached = cache is not None and cache.cached_len > 0
    if cache is not None:
        k, v = cache.update(layer, k, v)
    Tk = k.shape[1]
    mask = np.tril(np.ones((T, Tk), dtype=bool), k=Tk - T) if cached else np.tril(np.ones((T, T), dtype=bool))
    y = sdpa(q.transpose(0, 2, 1, 3), k.transpose(0, 2, 1, 3), v.transpose(0, 2, 1, 3), mask)
    if cfg["head_mixing"]:
        G = 32 if cfg["algebra"] == "hadamard" else 8
        W, beta = p[prefix + "head_mixer.W"], p[prefix + "head_mixer.beta"]
        yg = y.reshape(B, H // G, G, T, hd)
        mix = hadamard_head_mixer if G == 32 else octonion_head_mixer
        y = np.concatenate([mix(yg[:, g], W, beta, dtype) for g in range(H // G)], axis=1)
    y = y.transpose(0, 2, 1, 3).reshape(B, T, C)
    return _algebra_linear(cfg, p, prefix + "wo", y, dtype)


def swiglu(cfg, p, prefix, x, dtype):
    """SwiGLUMLP.forward (src/model/chassis.py:497-507)."""
    g = _algebra_linear(cfg, p, prefix + "gate_proj", x, dtype)
    u = _algebra_linear(cfg, p, prefix + "up_proj", x, dtype)
    return _algebra_linear(cfg, p, prefix + "down_proj", silu(g) * u, dtype)


def mhc_stream(p, prefix, x, fn, n=4):
    """mHCResidualStream.forward (src/model/mhc.py:345-381)."""
    B, T, _, C = x.shape
    xf = x.reshape(B, T, n * C)
    hp = stream_mapping(xf, p[prefix + "H_pre.phi.weight"], p[prefix + "H_pre.alpha"], p[prefix + "H_pre.bias"], "pre", n)
    ho = stream_mapping(xf, p[prefix + "H_post.phi.weight"], p[prefix + "H_post.alpha"], p[prefix + "H_post.bias"], "post", n)
    hr = stream_mapping(xf, p[prefix + "H_res.phi.weight"], p[prefix + "H_res.alpha"], p[prefix + "H_res.bias"], "res", n)
    out = fn((hp @ x)[:, :, 0])
    return hr @ x + np.swapaxes(ho, -1, -2) @ out[:, :, None, :]


def block(cfg, p, l, x, cos, sin, n=4, cache=None, dtype=np.float64, trace=None, forced_masks=None):
    """mHCLlamaBlock.forward (src/model/mhc.py:507-534)."""
    B, T, _, C = x.shape
    pre = f"layers.{l}."
    x = mhc_stream(p, pre + "attn_stream.", x,
                   lambda u: attention(cfg, p, pre + "attention.", rmsnorm(u, p[pre + "attention_norm.weight"]),
                                       cos, sin, cache, l, dtype), n)

    def ffn(u):
        un = rmsnorm(u, p[pre + "ffn_norm.weight"])
        if cfg["use_moe"]:
            fm = None if forced_masks is None else forced_masks[l]
            thr = cfg["moe_threshold"] if cfg.get("moe_routing", "topk") == "threshold" else None
            y, mask, probs = moe(un, p, pre + "feed_forward.", cfg["moe_max_experts"], fm, thr,
                                 cfg.get("moe_min_experts", 1))
            if trace is not None:
                trace.setdefault("router_mask", []).append(mask)
                trace.setdefault("router_probs", []).append(probs)
            return y
        return swiglu(cfg, p, pre + "feed_forward.", un, dtype)

    x = mhc_stream(p, pre + "ffn_stream.", x, ffn, n)
    if cfg["use_channel_mod"]:
        xf = x.reshape(B * n, T, C)
        xf = xf + channel_mod(rmsnorm(xf, p[pre + "channel_mod_norm.weight"]),
                              p[pre + "channel_mod.context_mlp.0.weight"],
                              p[pre + "channel_mod.context_mlp.2.weight"],
                              p[pre + "channel_mod.scale_temp"])
        x = xf.reshape(B, T, n, C)
    if trace is not None:
        trace.setdefault("layers", []).append(x)
    return x


def mhc_walsh_forward(cfg, p, idx, n_streams=4, cache=None, start_pos=0, dtype=np.float64,
                      trace=None, forced_masks=None):
    """mHCWalsh.forward for inference (src/model/mhc.py:617-681).
    Returns (logits [B, 1, V] of the last position, h_out [B, T, C])."""
    p = {k: np.asarray(v, dtype=dtype) if np.asarray(v).dtype.kind == "f" else np.asarray(v)
         for k, v in p.items()}
    B, T = idx.shape
    C = cfg["n_embd"]
    emb = _embedding(cfg, p)
    h = emb[idx] @ p["stream_proj.weight"].T + p["stream_proj.bias"]
    x = h.reshape(B, T, n_streams, C)
    cos, sin = precompute_rope(C // cfg["n_head"], 2 * cfg["block_size"])
    cos = cos[start_pos:start_pos + T].astype(dtype)
    sin = sin[start_pos:start_pos + T].astype(dtype)
    for l in range(cfg["n_layer"]):
        x = block(cfg, p, l, x, cos, sin, n_streams, cache, dtype, trace, forced_masks)
    hm = x.reshape(B, T, n_streams * C) @ p["stream_merge.weight"].T + p["stream_merge.bias"]
    h_out = rmsnorm(hm, p["norm.weight"])
    logits = h_out[:, -1:, :] @ emb.T
    return logits, h_out
