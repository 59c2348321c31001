"""Base decoder pieces (reference: src/model/chassis.py): config, RMSNorm,
RoPE table, batched KV cache, attention and the layer factories."""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional, Tuple

import torch
import torch.nn as nn

from .. import ops
from . import _prep
from .fht_cuda import HadamardHeadMixerFused, HadamardTernaryLinearTuple


@dataclass
class WalshConfig:
    """Same fields and defaults as the reference (src/model/chassis.py:33-51)."""
    block_size: int = 256
    vocab_size: int = 65
    n_layer: int = 6
    n_head: int = 6
    n_embd: int = 768
    dropout: float = 0.0
    bias: bool = False
    head_mixing: bool = False
    algebra: str = "octonion"
    hash_embeddings: bool = False
    use_moe: bool = False
    moe_threshold: float = 0.1
    moe_min_experts: int = 1
    moe_max_experts: int = 4
    use_channel_mod: bool = False


def get_linear_layer(config: WalshConfig):
    """(LayerClass, algebra_dim) for the config's algebra (src/model/chassis.py:54-65)."""
    if config.algebra == "hadamard":
        return HadamardTernaryLinearTuple, 32
    from .physics import OctonionTernaryLinear
    return OctonionTernaryLinear, 8


def get_head_mixer(config: WalshConfig, head_dim: int):
    """Head mixer for the config's algebra or None (src/model/chassis.py:68-94)."""
    if not config.head_mixing:
        return None
    if config.algebra == "hadamard":
        if config.n_head % 32 != 0:
            raise ValueError(f"Hadamard head_mixing requires n_head % 32 == 0, got {config.n_head}")
        return HadamardHeadMixerFused(head_dim)
    if config.n_head % 8 != 0:
        raise ValueError(f"Octonion head_mixing requires n_head % 8 == 0, got {config.n_head}")
    from .cayley_dickson_cuda import OctonionHeadMixer
    return OctonionHeadMixer(head_dim)


class RMSNorm(nn.Module):
    """x / sqrt(mean(x^2) + eps) * weight (src/model/chassis.py:96-106)."""

    def __init__(self, dim, eps=1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        return ops.rmsnorm(x, self.weight.detach().float().contiguous(), self.eps)


def precompute_freqs_cis(dim: int, end: int, theta: float = 10000.0) -> torch.Tensor:
    """Complex RoPE table [end, dim/2], float32 angles (src/model/chassis.py:332-337)."""
    freqs = 1.0 / (theta ** (torch.arange(0, dim, 2)[: dim // 2].float() / dim))
    ang = torch.outer(torch.arange(end, dtype=torch.float32), freqs).float()
    return torch.polar(torch.ones_like(ang), ang)


def rope_tables(module, freqs_cis: torch.Tensor):
    """(cos, sin) float32 [n_pos, hd/2] device tables from a complex RoPE table."""
    return _prep.cached(module, "rope", [freqs_cis],
                        lambda: (freqs_cis.real.float().contiguous(), freqs_cis.imag.float().contiguous()),
                        extra=(freqs_cis.shape[0],))


class KVCache:
    """KV cache with the reference's interface (src/model/chassis.py:262-330),
    extended to a batch: per layer [batch, n_head, max_seq_len, head_dim]
    (the reference keeps one sequence, [max_seq_len, n_head, head_dim])."""

    def __init__(self, n_layers: int, max_seq_len: int, n_head: int, head_dim: int,
                 device: torch.device, dtype: torch.dtype = torch.bfloat16, batch_size: int = 1):
        self.n_layers = n_layers
        self.max_seq_len = max_seq_len
        self.n_head = n_head
        self.head_dim = head_dim
        self.batch_size = batch_size
        self.dtype = dtype
        shape = (batch_size, n_head, max_seq_len, head_dim)
        self.k_cache: List[torch.Tensor] = [torch.zeros(shape, device=device, dtype=dtype) for _ in range(n_layers)]
        self.v_cache: List[torch.Tensor] = [torch.zeros(shape, device=device, dtype=dtype) for _ in range(n_layers)]
        self.cached_len = 0

    def update(self, layer_idx: int, k: torch.Tensor, v: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """Store k, v [B, new_len, H, hd] at cached_len; return the full [B, len, H, hd] views."""
        s, e = self.cached_len, self.cached_len + k.shape[1]
        self.k_cache[layer_idx][:, :, s:e] = k.transpose(1, 2).to(self.dtype)
        self.v_cache[layer_idx][:, :, s:e] = v.transpose(1, 2).to(self.dtype)
        return (self.k_cache[layer_idx][:, :, :e].transpose(1, 2),
                self.v_cache[layer_idx][:, :, :e].transpose(1, 2))

    def increment(self, n: int = 1):
        self.cached_len += n

    def reset(self):
        self.cached_len = 0


class CausalSelfAttention(nn.Module):
    """Algebra q/k/v/o projections, RoPE, causal attention over an optional
    KV cache and algebra head mixing (src/model/chassis.py:401-483)."""

    def __init__(self, config: WalshConfig):
        super().__init__()
        self.n_head = config.n_head
        self.n_embd = config.n_embd
        self.head_dim = config.n_embd // config.n_head
        self.head_mixing = config.head_mixing
        self.algebra = config.algebra
        LinearLayer, self.algebra_dim = get_linear_layer(config)
        self.mixer_dim = 32 if config.algebra == "hadamard" else 8
        self.wq = LinearLayer(config.n_embd, config.n_embd)
        self.wk = LinearLayer(config.n_embd, config.n_embd)
        self.wv = LinearLayer(config.n_embd, config.n_embd)
        self.wo = LinearLayer(config.n_embd, config.n_embd)
        self.dropout = config.dropout
        self.head_mixer = get_head_mixer(config, self.head_dim)

    def _triple(self, lin):
        inner = lin.inner
        return (inner.packed(),) + inner.scales()

    def _triple_tc(self, lin):
        inner = lin.inner
        return (inner.ternary_f16(),) + inner.scales()

    def _qkv_dense(self, dtype):
        """q | k | v HadamardLinear layers as one dense [3C, C] matrix (alpha, beta,
        the two transforms and the ternary blocks folded together, float32 then
        rounded to the operand dtype) with unit column scales: the operands of the
        tcgen05 q/k/v GEMM."""
        def build():
            W = torch.cat([self.wq.inner.dense(), self.wk.inner.dense(), self.wv.inner.dense()], dim=0)
            return (W.to(ops.octo_operand_dtype(dtype)).contiguous(), None), torch.ones(
                W.shape[0], device=W.device, dtype=torch.float32)
        ws = [p for lin in (self.wq, self.wk, self.wv) for p in (lin.weight, lin.inner.alpha, lin.inner.beta)]
        return _prep.cached(self, f"qkv_dense_{dtype}", ws, build)

    def _out_dense(self, dtype):
        """Head mixer then wo as one dense [C, C] matrix (the mixer applied to the
        identity rows, composed with wo's full matrix in float64, rounded to the
        operand dtype) with unit column scales: the operands of the tcgen05 output
        GEMM with the mHC site epilogue."""
        def build():
            C = self.n_embd
            eye = torch.eye(C, device=self.wo.weight.device, dtype=torch.float32)
            mix = eye if self.head_mixer is None else self.head_mixer.forward_tokens(
                eye.view(C, self.n_head, self.head_dim)).reshape(C, C)
            W = (self.wo.inner.dense().double() @ mix.double().t()).float()
            return (W.to(ops.octo_operand_dtype(dtype)).contiguous(), None), torch.ones(
                C, device=W.device, dtype=torch.float32)
        ws = [self.wo.weight, self.wo.inner.alpha, self.wo.inner.beta]
        if self.head_mixer is not None:
            ws += list(self.head_mixer.parameters())
        return _prep.cached(self, f"out_dense_{dtype}", ws, build)

    def _tc(self, x) -> bool:
        """16-bit Hadamard attention site on the tcgen05 GEMMs (dense q | k | v with
        RoPE and the cache write, folded mixer + wo with the site epilogue)."""
        return (self.algebra == "hadamard" and x.dtype == torch.float16 and self.n_embd in (512, 2048)
                and self.head_dim % 16 == 0)

    def forward_site(self, x, rope_cos, rope_sin, k_cache, v_cache, start_pos: int, xs, hmix):
        """Attention plus the mHC site epilogue: xs [B, T, n, C] <- H_res xs + H_post attn(x)."""
        if self.algebra != "hadamard":
            return self._octonion_site(x, rope_cos, rope_sin, k_cache, v_cache, start_pos, xs, hmix)
        if not self._tc(x) or xs.dtype not in (torch.bfloat16, torch.float16):
            f = self.forward_cached(x, rope_cos, rope_sin, k_cache, v_cache, start_pos, out_dtype=xs.dtype)
            return ops.mhc_post(xs, f, hmix, out=xs)
        B, T, C = x.shape
        H, hd = self.n_head, self.head_dim
        q = torch.empty((B, H, T, hd), dtype=x.dtype, device=x.device)
        # one tcgen05 GEMM over the dense q | k | v matrix, RoPE and the cache write in its epilogue
        w, sc = self._qkv_dense(x.dtype)
        ops.octo_qkv(x, H, w, sc, rope_cos, rope_sin, start_pos, q, k_cache, v_cache)
        o = ops.attention(q, k_cache, v_cache, start_pos)
        if B * T >= ops.ATTN_OUT_DENSE_FROM:
            # mixer and wo folded into one tcgen05 GEMM, the site update in its
            # epilogue (or, for few tokens, mhc_post after it)
            w, sc = self._out_dense(o.dtype)
            if B * T >= ops.ATTN_OUT_FUSED_FROM:
                return ops.octo_post(o.view(B, T, C), w, sc, xs, hmix, out=xs)
            f = ops.octo_linear(o.view(B, T, C), w, sc)
            return ops.mhc_post(xs, f, hmix, out=xs)
        wmix = bmix = None
        if self.head_mixer is not None:
            if hd != 16:
                o = self.head_mixer.forward_tokens(o, out=o)
            else:
                wmix, bmix = self.head_mixer.weights_tc()
        wo = self.wo.inner
        return ops.attn_out_tc(o.view(B, T, C), wmix, bmix, wo.ternary_f16(), *wo.scales(), xs, hmix, out=xs)

    def forward_cached(self, x, rope_cos, rope_sin, k_cache, v_cache, start_pos: int, out_dtype=None):
        """x [B, T, C] (already normed); rope rows for the T tokens; k/v written
        at cache rows start_pos.. (q/k/v in the caches' dtype); returns the wo
        output [B, T, C] in out_dtype (default x's)."""
        B, T, C = x.shape
        H, hd = self.n_head, self.head_dim
        q = torch.empty((B, H, T, hd), dtype=k_cache.dtype, device=x.device)
        if self.algebra == "hadamard":
            ops.attn_qkv(x, H, self._triple(self.wq), self._triple(self.wk), self._triple(self.wv),
                         rope_cos, rope_sin, start_pos, q, k_cache, v_cache)
        else:
            self._octonion_qkv(x, rope_cos, rope_sin, start_pos, q, k_cache, v_cache)
        o = ops.attention(q, k_cache, v_cache, start_pos)           # [B, T, H, hd]
        y = o.view(B, T, C)
        if self.algebra == "hadamard":
            if self.head_mixer is not None:
                o = self.head_mixer.forward_tokens(o, out=o)
            inner = self.wo.inner
            alpha, beta = inner.scales()
            return ops.hadamard_linear(y, inner.packed(), alpha, beta, 1.0, out_dtype=out_dtype or x.dtype)
        from .cayley_dickson_cuda import folded_output
        w, s = folded_output(self, y.dtype)
        f = ops.octo_linear(y, w, s)
        return f if out_dtype in (None, f.dtype) else f.to(out_dtype)

    def _octonion_qkv(self, x, rope_cos, rope_sin, start_pos, q, k_cache, v_cache):
        from .cayley_dickson_cuda import octonion_qkv
        octonion_qkv(self, x, rope_cos, rope_sin, start_pos, q, k_cache, v_cache)

    def _octonion_site(self, x, rope_cos, rope_sin, k_cache, v_cache, start_pos, xs, hmix):
        """q/k/v GEMM (RoPE, cache write) -> attention -> one GEMM for the head
        mixer and wo with the mHC site epilogue."""
        from .cayley_dickson_cuda import folded_output
        B, T, C = x.shape
        q = torch.empty((B, self.n_head, T, self.head_dim), dtype=k_cache.dtype, device=x.device)
        self._octonion_qkv(x, rope_cos, rope_sin, start_pos, q, k_cache, v_cache)
        o = ops.attention(q, k_cache, v_cache, start_pos)
        w, s = folded_output(self, o.dtype)
        return ops.octo_post(o.view(B, T, C), w, s, xs, hmix, out=xs)

    def forward(self, x, freqs_cis, kv_cache: Optional[KVCache] = None, layer_idx: int = 0):
        B, T, C = x.shape
        cos = freqs_cis[:T].real.float().contiguous()
        sin = freqs_cis[:T].imag.float().contiguous()
        if kv_cache is None:
            kc = torch.empty((B, self.n_head, T, self.head_dim), dtype=x.dtype, device=x.device)
            vc = torch.empty_like(kc)
            start = 0
        else:
            kc, vc, start = kv_cache.k_cache[layer_idx], kv_cache.v_cache[layer_idx], kv_cache.cached_len
            if kc.dtype != x.dtype or kc.shape[0] != B:
                raise ValueError("KV cache dtype/batch must match the activations")
        return self.forward_cached(x, cos, sin, kc, vc, start)
