"""Octonion (Cayley-Dickson) layers (reference: src/model/cayley_dickson_cuda.py,
src/model/physics.py:53-82, src/model/chassis.py:347-399, 485-507)."""
from __future__ import annotations

import math

import torch
import torch.nn as nn

from .constants import SIGN_TABLE, WEIGHT_IDX


class OctonionFusedLinear(nn.Module):
    """y_i = beta * sum_j SIGN[i][j] x_j @ Wq[WIDX[i][j]]^T over 8 parts."""

    def __init__(self, in_features, out_features, bias=False):
        super().__init__()
        assert in_features % 8 == 0 and out_features % 8 == 0
        self.in_o = in_features // 8
        self.out_o = out_features // 8
        self.weight = nn.Parameter(torch.rand(8, self.out_o, self.in_o) * 2 - 1)
        self.beta = nn.Parameter(torch.ones(self.out_o) * math.sqrt(3.0 / (2.0 * self.in_o)))

    def forward(self, x_parts):
        raise NotImplementedError("octonion kernels are not built yet")


class OctonionHeadMixer(nn.Module):
    def __init__(self, head_dim):
        super().__init__()
        self.head_dim = head_dim
        self.W = nn.Parameter(torch.randn(8, head_dim, head_dim) * 0.02)
        self.beta = nn.Parameter(torch.ones(head_dim) * math.sqrt(3.0 / (2.0 * head_dim)))
        self.register_buffer("signs", torch.tensor(SIGN_TABLE, dtype=torch.float32))
        self.register_buffer("widx", torch.tensor(WEIGHT_IDX, dtype=torch.long))

    def forward(self, x):
        raise NotImplementedError("octonion kernels are not built yet")


class SwiGLUMLP(nn.Module):
    def __init__(self, config):
        super().__init__()
        from .chassis import get_linear_layer
        LinearLayer, self.algebra_dim = get_linear_layer(config)
        hidden = int(2 * (4 * config.n_embd) / 3)
        hidden = math.ceil(hidden / self.algebra_dim) * self.algebra_dim
        self.gate_proj = LinearLayer(config.n_embd, hidden)
        self.up_proj = LinearLayer(config.n_embd, hidden)
        self.down_proj = LinearLayer(hidden, config.n_embd)

    def forward(self, x):
        raise NotImplementedError("octonion kernels are not built yet")
