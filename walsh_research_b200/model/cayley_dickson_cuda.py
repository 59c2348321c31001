"""Octonion (Cayley-Dickson) layers (reference: src/model/cayley_dickson_cuda.py,
src/model/physics.py:53-82, src/model/chassis.py:347-399, 485-507).

Same class names, constructor signatures, parameters and buffers as the
reference.  Each layer's eight ternary blocks are expanded once per
parameter version into the dense signed matrix
``W[(i, o), (j, k)] = SIGN[i][j] * Wq[WIDX[i][j]][o][k]`` (exact in fp16 and
bf16), so every octonion product runs as one tensor-core GEMM of libwalsh
with beta and the following op fused into its epilogue.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn

from .. import ops
from . import _prep
from .constants import SIGN_TABLE, WEIGHT_IDX


def dense_signed(blocks: torch.Tensor) -> torch.Tensor:
    """[8, R, S] blocks -> [8 R, 8 S] with block (i, j) = SIGN[i][j] * blocks[WIDX[i][j]]."""
    _, R, S = blocks.shape
    sign = torch.tensor(SIGN_TABLE, dtype=blocks.dtype, device=blocks.device)
    widx = torch.tensor(WEIGHT_IDX, dtype=torch.long, device=blocks.device)
    full = blocks[widx] * sign[:, :, None, None]           # [8 (i), 8 (j), R, S]
    return full.permute(0, 2, 1, 3).reshape(8 * R, 8 * S).contiguous()


def gemm_operands(w: torch.Tensor, dtype: torch.dtype, exact: bool):
    """(w_hi, w_lo) for activations of `dtype`: float16 w for float16
    activations, bfloat16 otherwise; w_lo (float32 activations only, and only
    when w is not exactly representable) carries w - w_hi."""
    op = ops.octo_operand_dtype(dtype)
    if dtype == torch.float32 and not exact:
        return ops.split_bf16(w)
    return w.to(op).contiguous(), None


class OctonionFusedLinear(nn.Module):
    """y_i = beta * sum_j SIGN[i][j] x_j @ Wq[WIDX[i][j]]^T over 8 parts
    (src/model/physics.py:53-82; src/model/cayley_dickson_cuda.py:622-668)."""

    def __init__(self, in_features, out_features, bias=False):
        super().__init__()
        assert in_features % 8 == 0 and out_features % 8 == 0
        self.in_o = in_features // 8
        self.out_o = out_features // 8
        self.weight = nn.Parameter(torch.rand(8, self.out_o, self.in_o) * 2 - 1)
        self.beta = nn.Parameter(torch.ones(self.out_o) * math.sqrt(3.0 / (2.0 * self.in_o)))

    def dense(self) -> torch.Tensor:
        """The signed expansion of the ternary blocks, float32 [8 out_o, 8 in_o]."""
        def build():
            packed, _ = ops.quantize_pack(self.weight)
            return dense_signed(ops.unpack(packed, self.in_o).float())
        return _prep.cached(self, "dense", [self.weight], build)

    def operands(self, dtype):
        return _prep.cached(self, f"op_{dtype}", [self.weight], lambda: gemm_operands(self.dense(), dtype, True))

    def scale(self):
        """beta for every output column: column (i, o) -> beta[o]."""
        return _prep.cached(self, "scale", [self.beta], lambda: self.beta.detach().float().repeat(8).contiguous())

    def forward_flat(self, x: torch.Tensor) -> torch.Tensor:
        return ops.octo_linear(x, self.operands(x.dtype), self.scale())

    def forward(self, x_parts):
        y = self.forward_flat(torch.cat(x_parts, dim=-1))
        return tuple(y.split(self.out_o, dim=-1))


OctonionTernaryLinear = OctonionFusedLinear
OctonionTernaryLinearRef = OctonionFusedLinear


class OctonionHeadMixer(nn.Module):
    """Octonion mixing of 8 heads: y_i = beta * sum_j SIGN[i][j] x_j @ W[WIDX[i][j]]
    (src/model/chassis.py:347-399; OctonionHeadMixerFused,
    src/model/cayley_dickson_cuda.py:1011-1042).  Input/output [B, 8, T, hd]."""

    def __init__(self, head_dim):
        super().__init__()
        self.head_dim = head_dim
        self.W = nn.Parameter(torch.randn(8, head_dim, head_dim) * 0.02)
        self.beta = nn.Parameter(torch.ones(head_dim) * math.sqrt(3.0 / (2.0 * head_dim)))
        self.register_buffer("signs", torch.tensor(SIGN_TABLE, dtype=torch.float32))
        self.register_buffer("widx", torch.tensor(WEIGHT_IDX, dtype=torch.long))

    def dense(self) -> torch.Tensor:
        """Mixing over the 8 heads' concatenated features as y = x M^T:
        block (i, j) of M is SIGN[i][j] W[WIDX[i][j]]^T, float32 [8 hd, 8 hd]."""
        return _prep.cached(self, "dense", [self.W], lambda: dense_signed(self.W.detach().float().transpose(1, 2)))

    def scale(self):
        return _prep.cached(self, "scale", [self.beta], lambda: self.beta.detach().float().repeat(8).contiguous())

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, H, T, D = x.shape
        assert H == 8, f"OctonionHeadMixer requires exactly 8 heads, got {H}"
        xt = x.permute(0, 2, 1, 3).reshape(B, T, 8 * D)
        w = _prep.cached(self, f"op_{x.dtype}", [self.W], lambda: gemm_operands(self.dense(), x.dtype, False))
        y = ops.octo_linear(xt, w, self.scale())
        return y.view(B, T, 8, D).permute(0, 2, 1, 3)


OctonionHeadMixerFused = OctonionHeadMixer


def folded_output(attn, dtype):
    """wo with the octonion head mixer folded in: f = beta_o . (o (Wo diag(s) Mix)^T),
    Mix the block-diagonal mixer over groups of 8 heads and s its beta.
    Returns ((w_hi, w_lo), scale)."""
    wo = attn.wo
    mixer = attn.head_mixer
    if mixer is None:
        return wo.operands(dtype), wo.scale()

    def build():
        C = attn.n_embd
        g = 8 * attn.head_dim
        M = mixer.dense().double()
        s = mixer.scale().double()
        mix = torch.zeros((C, C), dtype=torch.float64, device=M.device)
        for k in range(C // g):
            mix[k * g:(k + 1) * g, k * g:(k + 1) * g] = s[:, None] * M
        W = (wo.dense().double() @ mix).float()
        return gemm_operands(W, dtype, False)

    w = _prep.cached(attn, f"wo_fold_{dtype}", [wo.weight, mixer.W, mixer.beta], build)
    return w, wo.scale()


def qkv_operands(attn, dtype):
    """q | k | v rows of the three octonion layers stacked: ((w_hi, w_lo), scale [3C])."""
    def build():
        W = torch.cat([attn.wq.dense(), attn.wk.dense(), attn.wv.dense()], dim=0)
        s = torch.cat([attn.wq.scale(), attn.wk.scale(), attn.wv.scale()]).contiguous()
        return gemm_operands(W, dtype, True), s
    return _prep.cached(attn, f"qkv_{dtype}", [attn.wq.weight, attn.wk.weight, attn.wv.weight,
                                              attn.wq.beta, attn.wk.beta, attn.wv.beta], build)


def octonion_qkv(attn, x, rope_cos, rope_sin, start_pos, q, k_cache, v_cache):
    """q/k/v + RoPE + cache write for the octonion algebra (one GEMM)."""
    w, s = qkv_operands(attn, x.dtype)
    ops.octo_qkv(x, attn.n_head, w, s, rope_cos, rope_sin, start_pos, q, k_cache, v_cache)


def layer_dense(lin):
    """(dense float32 [out, in], column scale [out], exactly representable) of
    an algebra linear layer: octonion layers give their signed ternary
    expansion and beta; Hadamard layers their full matrix with alpha and beta
    folded in."""
    if isinstance(lin, OctonionFusedLinear):
        return lin.dense(), lin.scale(), True
    inner = lin.inner
    return inner.dense(), torch.ones(inner.out_features, device=inner.weight.device), False


class SwiGLUMLP(nn.Module):
    """silu(gate(x)) * up(x) -> down (src/model/chassis.py:485-507), as two
    GEMMs: gate and up interleaved with the SwiGLU product in the epilogue,
    then down (with the mHC site epilogue inside a block)."""

    def __init__(self, config):
        super().__init__()
        from .chassis import get_linear_layer
        LinearLayer, self.algebra_dim = get_linear_layer(config)
        hidden = int(2 * (4 * config.n_embd) / 3)
        hidden = math.ceil(hidden / self.algebra_dim) * self.algebra_dim
        self.hidden = hidden
        self.gate_proj = LinearLayer(config.n_embd, hidden)
        self.up_proj = LinearLayer(config.n_embd, hidden)
        self.down_proj = LinearLayer(hidden, config.n_embd)

    def _watch(self):
        return [p for m in (self.gate_proj, self.up_proj, self.down_proj) for p in m.parameters()]

    def gate_up_operands(self, dtype):
        """gate and up rows interleaved (row 2j gate unit j, row 2j + 1 up unit j)."""
        def build():
            wg, sg, eg = layer_dense(self.gate_proj)
            wu, su, eu = layer_dense(self.up_proj)
            W = torch.stack([wg, wu], dim=1).reshape(2 * self.hidden, -1)
            s = torch.stack([sg, su], dim=1).reshape(-1).float().contiguous()
            return gemm_operands(W, dtype, eg and eu), s
        return _prep.cached(self, f"gu_{dtype}", self._watch(), build)

    def down_operands(self, dtype):
        def build():
            wd, sd, ed = layer_dense(self.down_proj)
            return gemm_operands(wd, dtype, ed), sd.float().contiguous()
        return _prep.cached(self, f"down_{dtype}", self._watch(), build)

    def hidden_act(self, x):
        w, s = self.gate_up_operands(x.dtype)
        return ops.octo_swiglu(x, w, s, self.hidden)

    def forward(self, x):
        w, s = self.down_operands(x.dtype)
        return ops.octo_linear(self.hidden_act(x), w, s)

    def forward_site(self, u, x, hmix):
        """FFN site of an mHC block: x <- H_res x + H_post down(silu(gate u) * up u)."""
        h = self.hidden_act(u)
        w, s = self.down_operands(h.dtype)
        return ops.octo_post(h, w, s, x, hmix, out=x)
