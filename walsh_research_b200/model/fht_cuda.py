"""Hadamard-32 algebra layers (reference: src/model/fht_cuda.py).

Same class names, constructor signatures, parameters and buffers as the
reference, so reference checkpoints load unchanged.  Forward passes run the
sm_100a kernels of libwalsh; the latent weights are quantised and packed to
2 bits on the device once per parameter version.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn

from .. import ops
from . import _prep

ALGEBRA_DIM = 32


def hadamard_matrix(n: int, normalize: bool = True) -> torch.Tensor:
    """Sylvester Hadamard matrix, float32 (src/model/fht_cuda.py:32-56)."""
    assert n > 0 and (n & (n - 1)) == 0, f"n must be power of 2, got {n}"
    idx = torch.arange(n)
    both = idx[:, None] & idx[None, :]
    parity = torch.zeros_like(both)
    for b in range(n.bit_length()):
        parity ^= (both >> b) & 1
    H = 1.0 - 2.0 * parity.float()          # H[i, j] = (-1)^popcount(i & j)
    return H / math.sqrt(n) if normalize else H


def pack_ternary_weights(w: torch.Tensor) -> torch.Tensor:
    """[.., K] ternary {-1,0,+1} -> [.., ceil(K/4)] uint8 in the reference's
    2-bit encoding (src/model/fht_cuda.py:65-93).  Runs on the device."""
    packed, _ = ops.quantize_pack(w)
    return packed


def unpack_ternary_weights(packed: torch.Tensor, original_k: int) -> torch.Tensor:
    """Inverse of pack_ternary_weights (src/model/fht_cuda.py:96-117)."""
    return ops.unpack(packed, original_k)


def _ternary_init(out_o: int, in_o: int) -> torch.Tensor:
    # equal Frobenius norm per group (src/model/fht_cuda.py:464-468)
    w = torch.randn(ALGEBRA_DIM, out_o, in_o) * 0.02
    norms = w.view(ALGEBRA_DIM, -1).norm(dim=1, keepdim=True).unsqueeze(-1)
    return w / (norms + 1e-8) * 0.02 * math.sqrt(out_o * in_o)


class HadamardLinear(nn.Module):
    """y = beta . H . W_ternary . H . (alpha . x) (src/model/fht_cuda.py:436-519)."""

    ALGEBRA_DIM = ALGEBRA_DIM

    def __init__(self, in_features: int, out_features: int, bias: bool = False):
        super().__init__()
        assert in_features % ALGEBRA_DIM == 0 and out_features % ALGEBRA_DIM == 0
        self.in_o = in_features // ALGEBRA_DIM
        self.out_o = out_features // ALGEBRA_DIM
        self.in_features = in_features
        self.out_features = out_features
        self.weight = nn.Parameter(_ternary_init(self.out_o, self.in_o))
        self.alpha = nn.Parameter(torch.ones(ALGEBRA_DIM, self.in_o))
        self.beta = nn.Parameter(torch.ones(ALGEBRA_DIM, self.out_o) * math.sqrt(3.0 / (2.0 * self.in_o)))
        self.register_buffer("H", hadamard_matrix(ALGEBRA_DIM, normalize=True))

    def packed(self):
        """(2-bit weights [32, out_o, ceil(in_o/4)], alpha, beta) on the device."""
        return _prep.cached(self, "packed", [self.weight],
                            lambda: ops.quantize_pack(self.weight)[0])

    def ternary_f16(self):
        """Ternary values as float16 [32, out_o, in_o] (operands of the tensor-core kernels)."""
        return _prep.cached(self, "tern_f16", [self.weight],
                            lambda: ops.unpack(self.packed(), self.in_o).to(torch.float16).contiguous())

    def scales(self):
        return _prep.cached(self, "scales", [self.alpha, self.beta],
                            lambda: (self.alpha.detach().float().contiguous(), self.beta.detach().float().contiguous()))

    def dense(self) -> torch.Tensor:
        """The layer as one matrix, float32 [out, in]:
        W[(h, o), (p, i)] = beta[h, o] sum_g H[g, h] w[g, o, i] H[p, g] alpha[p, i]."""
        def build():
            Hm = hadamard_matrix(ALGEBRA_DIM, normalize=True).double().to(self.weight.device)
            w = ops.unpack(self.packed(), self.in_o).double()
            W = torch.einsum("gh,goi,pg->hopi", Hm, w, Hm)
            W = W * self.beta.detach().double()[:, :, None, None] * self.alpha.detach().double()[None, None]
            return W.reshape(self.out_features, self.in_features).float().contiguous()
        return _prep.cached(self, "dense", [self.weight, self.alpha, self.beta], build)

    def dense16(self, dtype):
        """(w_dense [out, in] in dtype, scale float [out]) of the dense GEMM form."""
        alpha, beta = self.scales()
        return _prep.cached(self, f"dense16_{dtype}", [self.weight, self.alpha, self.beta],
                            lambda: ops.hadamard_linear_dense_weights(self.packed(), alpha, beta, self.in_features,
                                                                      dtype))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        alpha, beta = self.scales()
        sixteen = x.dtype in (torch.bfloat16, torch.float16) and self.in_features == self.out_features
        if (sixteen and ops.HLIN_DENSE and self.in_features in ops.HLIN_DENSE_FEATURES
                and x.numel() >= ops.HLIN_DENSE_FROM * self.in_features):
            return ops.hadamard_linear_dense(x, *self.dense16(x.dtype))
        if ops.HLIN_PACKED and sixteen and self.in_features in ops.HLIN_PACKED_FEATURES:
            return ops.hadamard_linear_pk(x, self.packed(), alpha, beta)
        if ops.tc_eligible(x) and self.in_features == 512 and self.out_features == 512:
            return ops.hadamard_linear_tc(x, self.ternary_f16(), alpha, beta)
        return ops.hadamard_linear(x, self.packed(), alpha, beta, 1.0, out_dtype=x.dtype)

    def extra_repr(self) -> str:
        return f"in={self.in_features}, out={self.out_features}, algebra=hadamard32"


class HadamardTernaryLinearTuple(nn.Module):
    """Tuple interface around HadamardLinear (src/model/fht_cuda.py:526-569)."""

    ALGEBRA_DIM = ALGEBRA_DIM

    def __init__(self, in_features: int, out_features: int, bias: bool = False):
        super().__init__()
        self.inner = HadamardLinear(in_features, out_features, bias)
        self.in_o = self.inner.in_o
        self.out_o = self.inner.out_o

    @property
    def weight(self):
        return self.inner.weight

    @property
    def beta(self):
        return self.inner.beta

    def forward(self, x_parts: tuple) -> tuple:
        assert len(x_parts) == ALGEBRA_DIM, f"Expected {ALGEBRA_DIM} parts, got {len(x_parts)}"
        y = self.inner(torch.cat(x_parts, dim=-1))
        return tuple(y.split(self.out_o, dim=-1))


class HadamardHeadMixerFused(nn.Module):
    """Hadamard head mixing of 32 heads: y = beta . H (W_h x_h) H
    (src/model/fht_cuda.py:627-670).  Input/output [B, 32, T, head_dim]."""

    ALGEBRA_DIM = ALGEBRA_DIM

    def __init__(self, head_dim: int):
        super().__init__()
        self.head_dim = head_dim
        self.W = nn.Parameter(torch.randn(ALGEBRA_DIM, head_dim, head_dim) * 0.02)
        self.beta = nn.Parameter(torch.ones(head_dim) * math.sqrt(3.0 / (2.0 * head_dim)))
        self.register_buffer("H", hadamard_matrix(ALGEBRA_DIM, normalize=True))

    def weights(self):
        return _prep.cached(self, "w", [self.W, self.beta],
                            lambda: (self.W.detach().float().contiguous(), self.beta.detach().float().contiguous()))

    def weights_tc(self):
        """(W^T per head as float16 [32, hd_out, hd_in], beta float32)."""
        return _prep.cached(self, "wtc", [self.W, self.beta],
                            lambda: (self.W.detach().transpose(1, 2).to(torch.float16).contiguous(),
                                     self.beta.detach().float().contiguous()))

    def forward_tokens(self, y: torch.Tensor, out=None) -> torch.Tensor:
        """Token-major entry: y [..., n_head, hd], groups of 32 heads share W."""
        W, beta = self.weights()
        return ops.head_mixer_tokens(y, W, beta, out=out)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, H, T, D = x.shape
        assert H == ALGEBRA_DIM
        y = self.forward_tokens(x.permute(0, 2, 1, 3).contiguous())
        return y.permute(0, 2, 1, 3)


class HadamardHeadMixer(HadamardHeadMixerFused):
    """Reference implementation class of the same mixing (src/model/fht_cuda.py:576-624)."""


HadamardTernaryLinear = HadamardLinear
