"""Functional wrappers over the C ABI: tensors in, tensors out.

Each function validates devices, allocates outputs with torch (the caching
allocator is the only allocator on the forward path), and launches one
libwalsh entry point on the current stream.  No function here computes
anything on the host.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import call, dcode, ptr, require_cuda, stream


def _c(t):
    return t if t.is_contiguous() else t.contiguous()


# ---------------------------------------------------------------------------
# ternary weights
# ---------------------------------------------------------------------------

def quantize_pack(w: torch.Tensor):
    """Absmean ternary quantisation + 2-bit packing along the last dim.
    Returns (packed uint8 [..., ceil(k/4)], gamma float32 [1])."""
    require_cuda(w)
    w = _c(w.detach().float())
    k = w.shape[-1]
    rows = w.numel() // k
    packed = torch.empty(w.shape[:-1] + ((k + 3) // 4,), dtype=torch.uint8, device=w.device)
    gamma = torch.empty(1, dtype=torch.float32, device=w.device)
    call("walsh_ternary_quantize_pack", ptr(w), rows, k, ptr(packed), ptr(gamma), stream())
    return packed, gamma


def unpack(packed: torch.Tensor, k: int) -> torch.Tensor:
    require_cuda(packed)
    packed = _c(packed)
    rows = packed.numel() // packed.shape[-1]
    out = torch.empty(packed.shape[:-1] + (k,), dtype=torch.float32, device=packed.device)
    call("walsh_ternary_unpack", ptr(packed), rows, k, ptr(out), stream())
    return out


# ---------------------------------------------------------------------------
# Hadamard algebra
# ---------------------------------------------------------------------------

def hadamard_linear(x, packed, alpha, beta, w_scale: float = 1.0, out_dtype=None):
    require_cuda(x)
    x = _c(x)
    in_o = alpha.shape[1]
    out_o = beta.shape[1]
    if x.shape[-1] != 32 * in_o:
        raise ValueError(f"HadamardLinear expects last dim {32 * in_o}, got {x.shape[-1]}")
    out_dtype = out_dtype or x.dtype
    y = torch.empty(x.shape[:-1] + (32 * out_o,), dtype=out_dtype, device=x.device)
    ntok = x.numel() // x.shape[-1]
    call("walsh_hadamard_linear_fwd", ptr(x), dcode(x.dtype), ntok, in_o, out_o, ptr(packed), float(w_scale),
         ptr(alpha), ptr(beta), ptr(y), dcode(out_dtype), stream())
    return y


def tc_eligible(x, dtype=torch.bfloat16) -> bool:
    """True when the tensor-core Hadamard kernels apply: rows of 512 in ``dtype``."""
    return x.dtype == dtype and x.shape[-1] == 512


def hadamard_linear_tc(x, w_f16, alpha, beta, w_scale: float = 1.0):
    require_cuda(x)
    x = _c(x)
    y = torch.empty_like(x)
    call("walsh_hadamard_linear_tc_fwd", ptr(x), x.numel() // 512, ptr(w_f16), float(w_scale), ptr(alpha),
         ptr(beta), ptr(y), stream())
    return y


# HadamardLinear(512, 512) and (2048, 2048) on 16-bit activations: True reads
# the 2-bit packed weights (walsh_hadamard_linear_pk_fwd), False the fp16
# weight copies of the mma.sync chain (512) or the general kernel (2048);
# kept for comparisons
HLIN_PACKED = True
HLIN_PACKED_FEATURES = (512, 2048)
# 16-bit HadamardLinear(512, 512) from this many tokens on runs as one
# tcgen05 GEMM over the layer's dense matrix (hadamard_linear_dense; device
# time at 16384 / 65536 tokens: 13.9 / 37.1 us against the packed kernel's
# 16.2 / 54.6 us); below it (4096 - 8192 tokens: 9.0 - 9.3 against 8.4 -
# 8.5 us), and for 2048 (where the dense GEMM has 4 times the multiply-adds
# per token of 512 and measured 464 us against 207 us), the packed kernel
HLIN_DENSE = True
HLIN_DENSE_FEATURES = (512,)
HLIN_DENSE_FROM = 16384


def hadamard_linear_dense_weights(packed, alpha, beta, features, dtype):
    """(w_dense [F, F] in dtype, scale float [F]) of HadamardLinear(F, F):
    y = scale . (x w_dense^T)."""
    require_cuda(packed)
    w = torch.empty((features, features), dtype=dtype, device=packed.device)
    scale = torch.empty((features,), dtype=torch.float32, device=packed.device)
    call("walsh_hadamard_linear_dense_weights", ptr(_c(packed)), ptr(_c(alpha)), ptr(_c(beta)), features,
         dcode(dtype), ptr(w), ptr(scale), stream())
    return w, scale


def hadamard_linear_dense(x, w_dense, scale):
    """y = HadamardLinear(x) for 16-bit x [..., F] on the tcgen05 GEMM; y in x's dtype."""
    require_cuda(x)
    x = _c(x)
    F = x.shape[-1]
    if w_dense.dtype != x.dtype:
        raise ValueError(f"dense HadamardLinear weights are {w_dense.dtype}; activations are {x.dtype}")
    y = torch.empty_like(x)
    call("walsh_hadamard_linear_dense_fwd", ptr(x), dcode(x.dtype), x.numel() // F, F, ptr(w_dense), ptr(scale),
         ptr(y), stream())
    return y


def hadamard_linear_pk(x, packed, alpha, beta):
    """y = HadamardLinear(x) for x [..., F] (F = 512 or 2048) in bfloat16 or
    float16, weights 2-bit packed [32, F/32, F/128]; y in x's dtype."""
    require_cuda(x)
    x = _c(x)
    F = x.shape[-1]
    y = torch.empty_like(x)
    call("walsh_hadamard_linear_pk_fwd", ptr(x), dcode(x.dtype), x.numel() // F, F, ptr(packed), ptr(alpha),
         ptr(beta), ptr(y), stream())
    return y


def attn_out_tc(o, wmix, beta_mix, wo, alpha_o, beta_o, x, hmix, out=None):
    """Head mixer (wmix may be None) + wo + mHC site epilogue; returns x_out."""
    require_cuda(o, x)
    o = _c(o)
    out = out if out is not None else torch.empty_like(x)
    call("walsh_attn_out_tc_fwd", ptr(o), o.numel() // 512, ptr(wmix), ptr(beta_mix), ptr(wo), ptr(alpha_o),
         ptr(beta_o), ptr(x), dcode(x.dtype), ptr(hmix), ptr(out), stream())
    return out


def head_mixer_tokens(x, W, beta, out=None):
    """Hadamard head mixing on token-major [..., n_head, hd]."""
    require_cuda(x)
    x = _c(x)
    n_head, hd = x.shape[-2], x.shape[-1]
    y = out if out is not None else torch.empty_like(x)
    ntok = x.numel() // (n_head * hd)
    call("walsh_head_mixer_fwd", ptr(x), dcode(x.dtype), ntok, n_head, hd, ptr(W), ptr(beta), ptr(y), stream())
    return y


# ---------------------------------------------------------------------------
# mHC
# ---------------------------------------------------------------------------

def phi_fragments(phi_lp):
    """phi [24, D] (16-bit) in mma.sync B-fragment order: [D/16, 32 lanes, 6 regs, 2]."""
    D = phi_lp.shape[1]
    return (phi_lp.reshape(3, 8, D // 16, 2, 4, 2).permute(2, 1, 4, 0, 3, 5)
            .reshape(D // 16, 32, 6, 2).contiguous())


def mhc_map(x, phi, mparams, map_eps, norm_w=None, norm_eps=1e-6, phi_lp=None, u_dtype=None, phi_frag=None):
    """x [..., 4, C] -> (u [..., C] in u_dtype (default x's), hmix float [..., 24]).
    ``phi_lp`` (phi in x's 16-bit dtype) enables the tensor-core kernels for 16-bit
    x; ``phi_frag`` (``phi_fragments(phi_lp)``) the single-pass one for C = 512."""
    require_cuda(x)
    x = _c(x)
    C = x.shape[-1]
    lead = x.shape[:-2]
    ntok = x.numel() // (4 * C)
    u_dtype = u_dtype or x.dtype
    u = torch.empty(lead + (C,), dtype=u_dtype, device=x.device)
    hmix = torch.empty(lead + (24,), dtype=torch.float32, device=x.device)
    if phi_lp is not None and phi_lp.dtype != x.dtype:
        phi_lp = phi_frag = None
    call("walsh_mhc_map", ptr(x), dcode(x.dtype), ntok, C, ptr(phi), ptr(phi_lp), ptr(phi_frag), ptr(mparams),
         float(map_eps),
         ptr(norm_w), float(norm_eps), ptr(u), dcode(u_dtype), ptr(hmix), stream())
    return u, hmix


def mhc_post(x, f, hmix, out=None):
    require_cuda(x, f)
    x, f = _c(x), _c(f.to(x.dtype))
    C = x.shape[-1]
    ntok = x.numel() // (4 * C)
    out = out if out is not None else torch.empty_like(x)
    call("walsh_mhc_post", ptr(x), ptr(f), ptr(hmix), dcode(x.dtype), ntok, C, ptr(out), stream())
    return out


def sinkhorn(h, iters=20, eps=1e-8):
    require_cuda(h)
    if h.shape[-2:] != (4, 4):
        raise ValueError("walsh_sinkhorn supports 4x4 matrices (n_streams = 4)")
    hf = _c(h.float())
    out = torch.empty_like(hf)
    call("walsh_sinkhorn", ptr(hf), hf.numel() // 16, int(iters), float(eps), ptr(out), stream())
    return out.to(h.dtype)


# ---------------------------------------------------------------------------
# MoE and channel modulation
# ---------------------------------------------------------------------------

# below this many tokens (about a wave of 64-token tiles) the MoE runs as a
# router GEMM plus the warp-per-token kernel instead of the 128-token kernels
MOE_GEMM_ROUTER_BELOW = 148 * 64
# from this many tokens the attention output (head mixer and wo folded into
# one dense matrix) is a tcgen05 GEMM with the mHC site epilogue; below it
# the mma.sync attn_out_tc kernel.  Measured at B256 decode (Walsh-512): the
# GEMM form 3.57 ms per step against 3.74 ms, so it applies from one token
ATTN_OUT_DENSE_FROM = 1
# from this many tokens the site update runs in that GEMM's epilogue; below
# it the GEMM stores the attention output and mhc_post (spread over all SMs)
# applies the site update, since a few hundred tokens give the fused GEMM
# only M/128 x C/256 CTAs (B256 decode: 3.13 ms per step against 3.31 ms
# fused at Walsh-512, 21.19 against 21.48 ms at Walsh-2048)
ATTN_OUT_FUSED_FROM = 4096
# prefill-sized C = 512 MoE on the tcgen05 router GEMM + expert kernel (False:
# the single mma.sync kernel of walsh_moe_fwd; kept for comparisons)
MOE_TC05 = True
_ONES = {}


def _ones(n, device):
    key = (n, str(device))
    if key not in _ONES:
        _ONES[key] = torch.ones(n, dtype=torch.float32, device=device)
    return _ONES[key]


def routing_struct(routing):
    """ctypes pointer for an expert-selection rule: None (the reference's
    top-k) or (min_experts, threshold) for the threshold rule."""
    if routing is None:
        return None
    kmin, thr = routing
    return ctypes.byref(_lib.MoeRouting(_lib.ROUTE_THRESHOLD, int(kmin), float(thr)))


def moe(u, w1t, w2, gate_p, up_p, down_p, gammas, top_k, weights_in=None, fuse=None, want_stats=False, tc=None,
        routing=None, stats_out=None):
    """Router + experts.  With ``fuse=(x, hmix, x_out)`` the mHC epilogue is
    applied and ``x_out`` returned; otherwise the expert output y.
    With ``want_stats`` also returns (mask uint8, probs, weights).
    ``tc``: (w1, w2, gate, up, down) bfloat16 copies enabling the tensor-core kernel.
    ``routing``: None for the reference's top-k selection, or (min_experts,
    threshold) for the threshold rule (every expert with p > threshold, at
    least min_experts, at most top_k).  ``stats_out``: (mask, probs, weights)
    buffers to write the statistics into instead of new tensors."""
    require_cuda(u)
    rt = routing_struct(routing)
    tcs = None
    if tc is not None:
        tcs = _lib.MoeTcWeights(*[ptr(t) for t in tc[:5]])
    tcp = ctypes.byref(tcs) if tcs is not None else None
    u = _c(u)
    C = u.shape[-1]
    E = C // 32
    ntok = u.numel() // C
    lead = u.shape[:-1]
    mask = probs = weights = None
    if want_stats and stats_out is not None:
        mask, probs, weights = stats_out
    elif want_stats:
        mask = torch.empty(lead + (E,), dtype=torch.uint8, device=u.device)
        probs = torch.empty(lead + (E,), dtype=torch.float32, device=u.device)
        weights = torch.empty(lead + (E,), dtype=torch.float32, device=u.device)
    if weights_in is not None:
        weights_in = _c(weights_in.float())
    if (tc is not None and gate_p is not None and weights_in is None and u.dtype != torch.float32
            and C in (512, 2048) and ntok < MOE_GEMM_ROUTER_BELOW and tc[0].dtype == u.dtype):
        x, hmix, x_out = fuse if fuse is not None else (None, None, None)
        y = torch.empty_like(u) if fuse is None else None
        # decode-sized: router layer 1 as a tcgen05 GEMM, the rest one warp per token
        hid = C // 4
        hpre = octo_linear(u.view(ntok, C), (tc[0], None), _ones(hid, u.device))
        call("walsh_moe_hidden_fwd", ptr(u), ptr(hpre), dcode(u.dtype), ntok, C, int(top_k), ptr(w2), ptr(gate_p),
             ptr(up_p), ptr(down_p), ptr(gammas), ptr(y), 0 if fuse is None else 1, ptr(x),
             dcode(x.dtype) if x is not None else dcode(u.dtype), ptr(hmix), ptr(x_out), ptr(mask), ptr(probs),
             ptr(weights), rt, stream())
        out = y if fuse is None else x_out
        return (out, mask, probs, weights) if want_stats else out
    if (MOE_TC05 and tc is not None and len(tc) > 5 and gate_p is not None and weights_in is None
            and u.dtype != torch.float32 and C == 512 and ntok >= MOE_GEMM_ROUTER_BELOW and tc[0].dtype == u.dtype
            and (fuse is None or fuse[0].dtype != torch.float32)):
        # prefill-sized: router GEMM with the routing in its epilogue, then the
        # experts and the site epilogue, both on the tcgen05 tensor cores
        if not want_stats:
            mask = torch.empty(lead + (E,), dtype=torch.uint8, device=u.device)
            probs = torch.empty(lead + (E,), dtype=torch.float32, device=u.device)
            weights = torch.empty(lead + (E,), dtype=torch.float32, device=u.device)
        call("walsh_moe_router_tc_fwd", ptr(u), dcode(u.dtype), ntok, ptr(tc[0]), ptr(tc[1]), int(top_k), ptr(mask),
             ptr(probs), ptr(weights), rt, stream())
        x, hmix, x_out = fuse if fuse is not None else (None, None, None)
        y = torch.empty_like(u) if fuse is None else None
        call("walsh_moe_experts_tc_fwd", ptr(u), dcode(u.dtype), ntok, ptr(weights), ptr(tc[5]), ptr(tc[4]),
             ptr(gammas), ptr(y), 0 if fuse is None else 1, ptr(x),
             dcode(x.dtype) if x is not None else dcode(u.dtype), ptr(hmix), ptr(x_out), stream())
        out = y if fuse is None else x_out
        return (out, mask, probs, weights) if want_stats else out
    if fuse is None:
        y = torch.empty_like(u)
        call("walsh_moe_fwd", ptr(u), dcode(u.dtype), ntok, C, int(top_k), ptr(w1t), ptr(w2), ptr(gate_p),
             ptr(up_p), ptr(down_p), ptr(gammas), ptr(y), 0, None, dcode(u.dtype), None, None, ptr(weights_in),
             ptr(mask), ptr(probs), ptr(weights), tcp, rt, stream())
        out = y
    else:
        x, hmix, x_out = fuse
        call("walsh_moe_fwd", ptr(u), dcode(u.dtype), ntok, C, int(top_k), ptr(w1t), ptr(w2), ptr(gate_p),
             ptr(up_p), ptr(down_p), ptr(gammas), None, 1, ptr(x), dcode(x.dtype), ptr(hmix), ptr(x_out),
             ptr(weights_in), ptr(mask), ptr(probs), ptr(weights), tcp, rt, stream())
        out = x_out
    return (out, mask, probs, weights) if want_stats else out


# from this many segments (batched decode: one per stream row) the
# channel-modulation MLP's first layer runs as a tensor-core GEMM
CHMOD_MLP_TC_FROM = 512
# single-row segments (seg_len 1, C 512, 16-bit rows) in one launch
# (walsh_chmod_rows_fwd); False keeps the stats / mlp / apply steps
CHMOD_ROWS_FUSED = True


def chmod(x, seg_len, w1_p, w2_p, gammas, scale_temp, norm_w=None, norm_eps=1e-6, add_input=True, out=None,
          residual_scale=0.5, w1_dense=None, scale_out=None, shift_out=None):
    """Channel modulation over rows of x viewed as [nseg, seg_len, C].
    ``w1_dense``: W1 as dense bfloat16 [C/4, C] (the ternary values), enabling
    the tensor-core first layer from CHMOD_MLP_TC_FROM segments.
    ``scale_out``/``shift_out``: float32 [nseg, C/32] buffers for the
    per-segment scale and shift (new tensors when None)."""
    require_cuda(x)
    x = _c(x)
    C = x.shape[-1]
    nrows = x.numel() // C
    if nrows % seg_len:
        raise ValueError("rows must be a multiple of the segment length")
    nseg = nrows // seg_len
    E = C // 32
    if (seg_len == 1 and C == 512 and CHMOD_ROWS_FUSED and x.dtype in (torch.bfloat16, torch.float16)
            and (out is None or out.dtype == x.dtype)):
        # one launch for single-row segments (batched decode)
        scale = scale_out if scale_out is not None else torch.empty((nseg, E), dtype=torch.float32, device=x.device)
        shift = shift_out if shift_out is not None else torch.empty((nseg, E), dtype=torch.float32, device=x.device)
        out = out if out is not None else torch.empty_like(x)
        call("walsh_chmod_rows_fwd", ptr(x), dcode(x.dtype), nrows, C, ptr(norm_w), float(norm_eps), ptr(w1_p),
             ptr(w2_p), ptr(gammas), ptr(scale_temp), float(residual_scale), 1 if add_input else 0, ptr(scale),
             ptr(shift), ptr(out), stream())
        return out, scale, shift
    chunk = call("walsh_chmod_chunk_rows", int(seg_len))
    nch = (seg_len + chunk - 1) // chunk
    partial = torch.empty((nseg, nch, C), dtype=torch.float32, device=x.device)
    call("walsh_chmod_stats", ptr(x), dcode(x.dtype), nrows, C, int(seg_len), ptr(norm_w), float(norm_eps),
         ptr(partial), stream())
    scale = scale_out if scale_out is not None else torch.empty((nseg, E), dtype=torch.float32, device=x.device)
    shift = shift_out if shift_out is not None else torch.empty((nseg, E), dtype=torch.float32, device=x.device)
    if w1_dense is not None and nseg >= CHMOD_MLP_TC_FROM and C % 64 == 0:
        nbytes = call("walsh_chmod_mlp_tc_scratch_bytes", nseg, C)
        scratch = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
        call("walsh_chmod_mlp_tc", ptr(partial), nseg, int(seg_len), C, ptr(w1_dense), ptr(w2_p), ptr(gammas),
             ptr(scale_temp), ptr(scratch), ptr(scale), ptr(shift), stream())
    else:
        call("walsh_chmod_mlp", ptr(partial), nseg, int(seg_len), C, ptr(w1_p), ptr(w2_p), ptr(gammas),
             ptr(scale_temp), ptr(scale), ptr(shift), stream())
    out = out if out is not None else torch.empty_like(x)
    call("walsh_chmod_apply", ptr(x), dcode(x.dtype), nrows, C, int(seg_len), ptr(norm_w), float(norm_eps),
         ptr(scale), ptr(shift), float(residual_scale), 1 if add_input else 0, ptr(out), stream())
    return out, scale, shift


# ---------------------------------------------------------------------------
# attention
# ---------------------------------------------------------------------------

def attn_qkv(u, n_head, wq, wk, wv, rope_cos, rope_sin, start_pos, q, k_cache, v_cache):
    """wq/wk/wv: (packed, alpha, beta) triples; rope_cos/sin [>=T, hd/2] hold the
    rows of the tokens' own positions; k/v land at cache rows start_pos.."""
    require_cuda(u)
    u = _c(u)
    B, T, C = u.shape
    call("walsh_attn_qkv_fwd", ptr(u), dcode(u.dtype), B, T, C, n_head,
         ptr(wq[0]), ptr(wq[1]), ptr(wq[2]), ptr(wk[0]), ptr(wk[1]), ptr(wk[2]),
         ptr(wv[0]), ptr(wv[1]), ptr(wv[2]), ptr(rope_cos), ptr(rope_sin), rope_cos.shape[0], int(start_pos),
         ptr(q), ptr(k_cache), ptr(v_cache), k_cache.shape[-2], dcode(q.dtype), stream())


def attn_qkv_tc(u, n_head, wq, wk, wv, rope_cos, rope_sin, start_pos, q, k_cache, v_cache):
    """attn_qkv on the tensor cores (C = 512; u, q and caches float16); wq/wk/wv: (w_f16, alpha, beta)."""
    require_cuda(u)
    u = _c(u)
    B, T, C = u.shape
    call("walsh_attn_qkv_tc_fwd", ptr(u), B, T, n_head,
         ptr(wq[0]), ptr(wq[1]), ptr(wq[2]), ptr(wk[0]), ptr(wk[1]), ptr(wk[2]),
         ptr(wv[0]), ptr(wv[1]), ptr(wv[2]), ptr(rope_cos), ptr(rope_sin), rope_cos.shape[0], int(start_pos),
         ptr(q), ptr(k_cache), ptr(v_cache), k_cache.shape[-2], stream())


def attention(q, k_cache, v_cache, start_pos, out=None):
    """q [B, H, T, hd], caches [B, H, ctx, hd] -> o [B, T, H, hd]."""
    require_cuda(q)
    B, H, T, hd = q.shape
    ctx = k_cache.shape[-2]
    o = out if out is not None else torch.empty((B, T, H, hd), dtype=q.dtype, device=q.device)
    call("walsh_attn_fwd", ptr(q), ptr(k_cache), ptr(v_cache), dcode(q.dtype), B, H, T, hd, ctx, int(start_pos),
         ptr(o), stream())
    return o


# ---------------------------------------------------------------------------
# octonion (Cayley-Dickson) GEMMs; w = (w_hi, w_lo or None) in the operand
# dtype the x dtype selects (float16 for float16 x, bfloat16 otherwise)
# ---------------------------------------------------------------------------

def octo_operand_dtype(x_dtype):
    return torch.float16 if x_dtype == torch.float16 else torch.bfloat16


def _octo_w(x, w):
    hi, lo = w
    if hi.dtype != octo_operand_dtype(x.dtype):
        raise ValueError(f"octonion weights are {hi.dtype}; {x.dtype} activations need {octo_operand_dtype(x.dtype)}")
    if x.dtype != torch.float32:
        lo = None
    return hi, lo


def octo_linear(x, w, scale, out=None):
    """y = scale . (x w^T); x [..., K] -> y [..., N] in x's dtype."""
    require_cuda(x)
    x = _c(x)
    hi, lo = _octo_w(x, w)
    N, K = hi.shape
    M = x.numel() // K
    y = out if out is not None else torch.empty(x.shape[:-1] + (N,), dtype=x.dtype, device=x.device)
    call("walsh_octo_linear_fwd", ptr(x), dcode(x.dtype), M, K, ptr(hi), ptr(lo), dcode(hi.dtype), N, ptr(scale),
         ptr(y), stream())
    return y


def octo_qkv(u, n_head, w, scale, rope_cos, rope_sin, start_pos, q, k_cache, v_cache):
    require_cuda(u)
    u = _c(u)
    B, T, C = u.shape
    hi, lo = _octo_w(u, w)
    call("walsh_octo_qkv_fwd", ptr(u), dcode(u.dtype), B, T, C, n_head, ptr(hi), ptr(lo), dcode(hi.dtype),
         ptr(scale), ptr(rope_cos), ptr(rope_sin), rope_cos.shape[0], int(start_pos), ptr(q), ptr(k_cache),
         ptr(v_cache), k_cache.shape[-2], stream())


def octo_swiglu(u, w, scale, hidden, out=None):
    """h = silu(gate(u)) * up(u) with gate/up rows interleaved in w [2 hidden, K]."""
    require_cuda(u)
    u = _c(u)
    hi, lo = _octo_w(u, w)
    K = hi.shape[1]
    M = u.numel() // K
    h = out if out is not None else torch.empty(u.shape[:-1] + (hidden,), dtype=u.dtype, device=u.device)
    call("walsh_octo_swiglu_fwd", ptr(u), dcode(u.dtype), M, K, ptr(hi), ptr(lo), dcode(hi.dtype), ptr(scale),
         int(hidden), ptr(h), stream())
    return h


def octo_post(a, w, scale, x, hmix, out=None):
    """f = scale . (a w^T), then x_out = H_res x + H_post f (x [..., 4, C])."""
    require_cuda(a, x)
    a = _c(a)
    hi, lo = _octo_w(a, w)
    C, K = hi.shape
    M = a.numel() // K
    out = out if out is not None else torch.empty_like(x)
    call("walsh_octo_post_fwd", ptr(a), dcode(a.dtype), M, K, ptr(hi), ptr(lo), dcode(hi.dtype), ptr(scale), C,
         ptr(x), dcode(x.dtype), ptr(hmix), ptr(out), stream())
    return out


# ---------------------------------------------------------------------------
# dense helpers
# ---------------------------------------------------------------------------

def embed_gather(idx, table, err=None, out=None):
    require_cuda(idx, table)
    idx = _c(idx.to(torch.int64))
    V, D = table.shape
    out = out if out is not None else torch.empty(idx.shape + (D,), dtype=table.dtype, device=table.device)
    call("walsh_embed_gather", ptr(idx), idx.numel(), ptr(table), dcode(table.dtype), V, D, ptr(out), ptr(err),
         stream())
    return out


def linear(x, w, bias=None, out_dtype=torch.float32, ldx=None, M=None, out=None):
    """y = x W^T + b with x rows of stride ldx (defaults to contiguous rows)."""
    require_cuda(x, w)
    w = _c(w)
    N, K = w.shape
    if ldx is None:
        x = _c(x)
        ldx = K
        M = x.numel() // K
        lead = x.shape[:-1]
    else:
        lead = (M,)
    y = out if out is not None else torch.empty(lead + (N,), dtype=out_dtype, device=x.device)
    call("walsh_linear_fwd", ptr(x), dcode(x.dtype), M, K, ldx, ptr(w), dcode(w.dtype), N,
         ptr(None if bias is None else _c(bias.float())), ptr(y), dcode(y.dtype), stream())
    return y


def split_bf16(w):
    """(w_hi, w_lo) bfloat16 with w_hi + w_lo = w to about 2^-16 relative."""
    wf = w.detach().float()
    hi = wf.to(torch.bfloat16)
    lo = (wf - hi.float()).to(torch.bfloat16)
    return hi.contiguous(), lo.contiguous()


def split_eligible(x, K, ldx=None) -> bool:
    esz = x.element_size()
    ld = K if ldx is None else ldx
    return (x.dtype in (torch.float32, torch.bfloat16, torch.float16) and K % 32 == 0 and x.data_ptr() % 16 == 0
            and (ld * esz) % 16 == 0)


def split3_weights(w):
    """[w_hi | w_lo | w_hi] bfloat16 [N, 3K] for linear_split_tc."""
    hi, lo = split_bf16(w)
    return torch.cat([hi, lo, hi], dim=1).contiguous()


def linear_split_tc(x, w3):
    """y = x W^T (float32 x [..., K], float32 y) on the tcgen05 tensor cores,
    W given as split3_weights(W); the same three split products as
    linear_split in one GEMM with K tripled."""
    require_cuda(x, w3)
    x = _c(x.float())
    N, K3 = w3.shape
    K = K3 // 3
    M = x.numel() // K
    y = torch.empty(x.shape[:-1] + (N,), dtype=torch.float32, device=x.device)
    scratch = torch.empty(call("walsh_linear_split_tc_scratch_bytes", M, K), dtype=torch.uint8, device=x.device)
    call("walsh_linear_split_tc_fwd", ptr(x), M, K, ptr(w3), N, ptr(scratch), ptr(y), stream())
    return y


def linear_split(x, w_hi, w_lo, bias=None, ldx=None, M=None, out=None):
    """y = x W^T + b (float32) with W given as its bf16 split (see split_bf16)."""
    require_cuda(x, w_hi, w_lo)
    N, K = w_hi.shape
    if ldx is None:
        x = _c(x)
        ldx = K
        M = x.numel() // K
        lead = x.shape[:-1]
    else:
        lead = (M,)
    y = out if out is not None else torch.empty(lead + (N,), dtype=torch.float32, device=x.device)
    call("walsh_linear_split_fwd", ptr(x), dcode(x.dtype), M, K, ldx, ptr(w_hi), ptr(w_lo), N,
         ptr(None if bias is None else _c(bias.float())), ptr(y), stream())
    return y


def rmsnorm(x, w, eps=1e-6, out_dtype=None):
    require_cuda(x)
    x = _c(x)
    C = x.shape[-1]
    out_dtype = out_dtype or x.dtype
    y = torch.empty(x.shape, dtype=out_dtype, device=x.device)
    call("walsh_rmsnorm", ptr(x), dcode(x.dtype), x.numel() // C, C, ptr(w), float(eps), ptr(y), dcode(out_dtype),
         stream())
    return y
