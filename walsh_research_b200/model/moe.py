"""Hadamard MoE and channel modulation (reference: src/model/moe.py).

Forward passes run libwalsh's fused router/expert and channel-modulation
kernels.  Statistics the reference records on every call (aux loss, expert
mask, modulation stats) are kept as device tensors and only reduced when
asked for, so the forward path has no host synchronisation.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import numpy as np
import torch
import torch.nn as nn

from .. import ops
from . import _prep


def quantize_ternary(w: torch.Tensor) -> torch.Tensor:
    """Scaled absmean ternary q * gamma (src/model/moe.py:268-303), on the device."""
    packed, gamma = ops.quantize_pack(w)
    return ops.unpack(packed, w.shape[-1]) * gamma


class FastMoEExperts(nn.Module):
    """Ternary SwiGLU experts on 32-wide blocks (src/model/moe.py:306-380)."""

    def __init__(self, n_experts: int = 8, dim: int = 32, expansion: int = 4, use_ternary: bool = True):
        super().__init__()
        self.n_experts = n_experts
        self.dim = dim
        self.hidden = dim * expansion
        self.use_ternary = use_ternary
        if dim != 32 or self.hidden != 128 or not use_ternary:
            raise NotImplementedError("the fused expert kernel implements 32-wide ternary experts with hidden 128")
        self.gate_weights = nn.Parameter(torch.empty(n_experts, self.hidden, dim).uniform_(-1, 1))
        self.up_weights = nn.Parameter(torch.empty(n_experts, self.hidden, dim).uniform_(-1, 1))
        self.down_weights = nn.Parameter(torch.empty(n_experts, dim, self.hidden).uniform_(-1, 1))

    def packed(self):
        """(gate, up, down) 2-bit tensors and gammas float[3] on the device."""
        def build():
            g, gg = ops.quantize_pack(self.gate_weights)
            u, gu = ops.quantize_pack(self.up_weights)
            d, gd = ops.quantize_pack(self.down_weights)
            return g, u, d, torch.cat([gg, gu, gd])
        return _prep.cached(self, "packed", [self.gate_weights, self.up_weights, self.down_weights], build)

    def ternary_tc(self, dtype):
        """(gate, up, down) ternary values {-1, 0, +1} in ``dtype`` (bf16 or fp16; gamma
        not applied), the operands of the tensor-core expert kernel."""
        def build():
            g, u, d, _ = self.packed()
            return (ops.unpack(g, self.dim).to(dtype).contiguous(),
                    ops.unpack(u, self.dim).to(dtype).contiguous(),
                    ops.unpack(d, self.hidden).to(dtype).contiguous())
        return _prep.cached(self, f"tern_{dtype}", [self.gate_weights, self.up_weights, self.down_weights], build)

    def pair_tc(self, dtype):
        """Gate/up ternary values of expert pairs side by side, ``dtype`` [E/2, 256, 64]:
        for pair p rows 0..127 gate, 128..255 up; columns 0..31 expert 2p, 32..63
        expert 2p + 1 (the operand layout of walsh_moe_experts_tc_fwd)."""
        def build():
            g, u, _ = self.ternary_tc(dtype)
            E, H, D = g.shape
            gp = g.view(E // 2, 2, H, D).permute(0, 2, 1, 3).reshape(E // 2, H, 2 * D)
            up = u.view(E // 2, 2, H, D).permute(0, 2, 1, 3).reshape(E // 2, H, 2 * D)
            return torch.cat([gp, up], dim=1).contiguous()
        return _prep.cached(self, f"pair_{dtype}", [self.gate_weights, self.up_weights], build)

    def forward(self, x: torch.Tensor, expert_weights: torch.Tensor) -> torch.Tensor:
        B, T, E, D = x.shape
        g, u, d, gam = self.packed()
        y = ops.moe(x.reshape(B, T, E * D), None, None, g, u, d, gam, top_k=1, weights_in=expert_weights)
        return y.view(B, T, E, D)


class HadamardRouter(nn.Module):
    """softmax(W2 SiLU(W1 x)) with top-k selection (src/model/moe.py:383-447).
    ``threshold`` and ``min_experts`` are stored and, by default, unused: as in
    the reference, the selection is top-k with k = min(max_experts,
    n_experts).  ``routing_mode = "threshold"`` switches to the rule the
    reference's docstring describes: every expert with p > threshold, at least
    min_experts and at most k of them (opt-in; not the reference's forward)."""

    def __init__(self, n_embd: int, n_experts: int = 8, threshold: float = 0.1, min_experts: int = 1,
                 max_experts: int = 4):
        super().__init__()
        self.n_experts = n_experts
        self.threshold = threshold
        self.min_experts = min_experts
        self.max_experts = max_experts
        hidden = n_embd // 4
        self.gate = nn.Sequential(nn.Linear(n_embd, hidden, bias=False), nn.SiLU(),
                                  nn.Linear(hidden, n_experts, bias=False))
        for m in self.gate:
            if isinstance(m, nn.Linear):
                nn.init.normal_(m.weight, std=0.01)
        self.routing_mode = "topk"

    @property
    def top_k(self) -> int:
        return min(self.max_experts, self.n_experts)

    def routing(self):
        """The kernels' selection rule: None for the reference's top-k, or
        (min_experts, threshold) in threshold mode."""
        if self.routing_mode == "topk":
            return None
        if self.routing_mode == "threshold":
            return (max(1, min(int(self.min_experts), self.top_k)), float(self.threshold))
        raise ValueError(f"routing_mode must be 'topk' or 'threshold', got {self.routing_mode!r}")

    def weights_dev(self):
        """(W1 transposed [C, C/4], W2 [E, C/4]) float32 on the device."""
        return _prep.cached(self, "w", [self.gate[0].weight, self.gate[2].weight],
                            lambda: (self.gate[0].weight.detach().float().t().contiguous(),
                                     self.gate[2].weight.detach().float().contiguous()))

    def weights_tc(self, dtype):
        """(W1 [C/4, C], W2 [E, C/4]) copies in ``dtype`` (bf16 or fp16) for the tensor-core kernel."""
        return _prep.cached(self, f"w_{dtype}", [self.gate[0].weight, self.gate[2].weight],
                            lambda: (self.gate[0].weight.detach().to(dtype).contiguous(),
                                     self.gate[2].weight.detach().to(dtype).contiguous()))

    def forward(self, x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        w1t, w2 = self.weights_dev()
        tc = self.weights_tc(x.dtype) + (None, None, None) if x.dtype != torch.float32 else None
        _, mask, probs, weights = ops.moe(x, w1t, w2, None, None, None, None, self.top_k, want_stats=True, tc=tc,
                                          routing=self.routing())
        return weights, mask.float(), probs


class HadamardMoE(nn.Module):
    """Router + experts over the n_embd/32 Hadamard blocks (src/model/moe.py:450-598)."""
    BLOCK_DIM = 32

    def __init__(self, config, n_experts: int = None, expansion: int = 4, threshold: float = 0.1,
                 min_experts: int = 1, max_experts: int = 4, aux_loss_weight: float = 0.01):
        super().__init__()
        self.n_embd = config.n_embd
        if n_experts is None:
            n_experts = config.n_embd // self.BLOCK_DIM
        self.n_experts = n_experts
        self.block_dim = config.n_embd // n_experts
        self.aux_loss_weight = aux_loss_weight
        assert self.block_dim == self.BLOCK_DIM
        self.router = HadamardRouter(config.n_embd, n_experts, threshold, min_experts, max_experts)
        self.experts = FastMoEExperts(n_experts=n_experts, dim=self.block_dim, expansion=expansion)
        self._aux_loss = None
        self._last_router_probs = None
        self.register_buffer("_expert_counts", torch.zeros(n_experts), persistent=False)
        self.register_buffer("_total_tokens", torch.zeros(1), persistent=False)
        self.__dict__["_last_mask_u8"] = None

    def kernel_args(self, dtype=torch.float16):
        """Arguments of ops.moe for activations u of ``dtype``:
        (w1t, w2, gate, up, down, gammas, top_k, tc)."""
        w1t, w2 = self.router.weights_dev()
        g, u, d, gam = self.experts.packed()
        tc = None
        if dtype != torch.float32:
            tc = self.router.weights_tc(dtype) + self.experts.ternary_tc(dtype) + (self.experts.pair_tc(dtype),)
        return w1t, w2, g, u, d, gam, self.router.top_k, tc

    @property
    def _last_expert_mask(self):
        """0/1 float mask [B, T, E] of the last forward's selections (src/model/moe.py:529)."""
        m = self.__dict__.get("_last_mask_u8")
        return None if m is None else m.float()

    @_last_expert_mask.setter
    def _last_expert_mask(self, value):
        self.__dict__["_last_mask_u8"] = value

    def _record(self, mask, probs, ntok):
        self.__dict__["_last_mask_u8"] = mask  # kept as the kernel's uint8; converted on access
        self._last_router_probs = probs
        self._aux_loss = None  # reduced lazily by get_aux_loss
        if self.training:
            with torch.no_grad():
                self._expert_counts += mask.view(-1, self.n_experts).float().sum(0)
                self._total_tokens += ntok

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, T, C = x.shape
        w1t, w2, g, u, d, gam, k, tc = self.kernel_args(x.dtype)
        y, mask, probs, _ = ops.moe(x, w1t, w2, g, u, d, gam, k, want_stats=True, tc=tc,
                                    routing=self.router.routing())
        self._record(mask, probs, B * T)
        return y

    def _compute_aux_loss(self, router_probs, expert_mask):
        """Switch-style load-balance loss (src/model/moe.py:544-560)."""
        probs = router_probs.reshape(-1, self.n_experts)
        mask = expert_mask.reshape(-1, self.n_experts)
        return (mask.mean(0) * probs.mean(0)).sum() * self.n_experts

    def get_aux_loss(self) -> Optional[torch.Tensor]:
        if self._aux_loss is None and self._last_router_probs is not None:
            self._aux_loss = self._compute_aux_loss(self._last_router_probs, self._last_expert_mask)
        return self._aux_loss if self._aux_loss is not None else torch.tensor(0.0)

    def get_expert_stats(self) -> dict:
        """Expert load and Gini-based balance (src/model/moe.py:566-589)."""
        total = float(self._total_tokens.item())
        if total == 0:
            return {"expert_load": [0.0] * self.n_experts, "avg_experts": 0.0, "load_balance": 0.0}
        counts = self._expert_counts.cpu().numpy()
        load = counts / total
        s = np.sort(load)
        n = len(s)
        cum = np.cumsum(s)
        gini = (2 * np.sum(np.arange(1, n + 1) * s) - (n + 1) * cum[-1]) / (n * cum[-1] + 1e-8)
        return {"expert_load": load.tolist(), "avg_experts": float(counts.sum() / total),
                "load_balance": float(1 - abs(gini))}

    def reset_stats(self):
        self._expert_counts.zero_()
        self._total_tokens.zero_()

    def get_expert_usage(self) -> dict:
        return self.get_expert_stats()


class HadamardChannelModulation(nn.Module):
    """Bulk-state channel modulation (src/model/moe.py:610-771)."""
    BLOCK_DIM = 32

    def __init__(self, n_embd: int = 256, n_blocks: int = None, use_ternary: bool = True,
                 residual_scale: float = 0.5):
        super().__init__()
        if n_blocks is None:
            n_blocks = n_embd // self.BLOCK_DIM
        self.n_blocks = n_blocks
        self.block_dim = n_embd // n_blocks
        self.residual_scale = residual_scale
        self.use_ternary = use_ternary
        if self.block_dim != 32 or not use_ternary:
            raise NotImplementedError("the channel-modulation kernels implement ternary modulation of 32-wide blocks")
        hidden = n_embd // 4
        self.context_mlp = nn.Sequential(nn.Linear(n_embd, hidden, bias=False), nn.SiLU(),
                                         nn.Linear(hidden, n_blocks * 2, bias=False))
        nn.init.normal_(self.context_mlp[0].weight, std=0.02)
        nn.init.normal_(self.context_mlp[-1].weight, std=0.01)
        self.scale_temp = nn.Parameter(torch.ones(1) * 1.0)
        self._last_scale = None
        self._last_shift = None

    def packed(self):
        def build():
            w1, g1 = ops.quantize_pack(self.context_mlp[0].weight)
            w2, g2 = ops.quantize_pack(self.context_mlp[2].weight)
            return w1, w2, torch.cat([g1, g2])
        return _prep.cached(self, "packed", [self.context_mlp[0].weight, self.context_mlp[2].weight], build)

    def kernel_args(self):
        w1, w2, gam = self.packed()
        return w1, w2, gam, self.scale_temp.detach().float().contiguous()

    def w1_dense(self):
        """W1's ternary values as dense bfloat16 [C/4, C] (exact), for the
        tensor-core first layer of the modulation MLP."""
        def build():
            w1, _, _ = self.packed()
            return ops.unpack(w1, self.context_mlp[0].weight.shape[1]).to(torch.bfloat16).contiguous()
        return _prep.cached(self, "w1_dense", [self.context_mlp[0].weight], build)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, T, C = x.shape
        w1, w2, gam, temp = self.kernel_args()
        out, scale, shift = ops.chmod(x, T, w1, w2, gam, temp, norm_w=None, add_input=False,
                                      residual_scale=self.residual_scale)
        self._last_scale, self._last_shift = scale, shift
        return out

    def get_modulation_stats(self) -> dict:
        if self._last_scale is None:
            return {"scale_mean": 0.0, "scale_std": 0.0, "shift_mean": 0.0, "scale_temp": self.scale_temp.item()}
        return {"scale_mean": self._last_scale.mean().item(), "scale_std": self._last_scale.std().item(),
                "shift_mean": self._last_shift.abs().mean().item(), "scale_temp": self.scale_temp.item()}
