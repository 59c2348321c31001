"""Ternary quantiser and the octonion linear layer (reference: src/model/physics.py)."""
from __future__ import annotations

import torch

from .. import ops


def quantize_ternary(w: torch.Tensor, training: bool = True) -> torch.Tensor:
    """Unscaled absmean ternary {-1, 0, +1} (src/model/physics.py:13-51), on the device."""
    packed, _ = ops.quantize_pack(w)
    return ops.unpack(packed, w.shape[-1])


def __getattr__(name):
    # the octonion layer lives with its kernels; the reference exports it from here
    if name in ("OctonionTernaryLinear", "OctonionTernaryLinearRef", "OctonionFusedLinear"):
        from . import cayley_dickson_cuda
        return getattr(cayley_dickson_cuda, "OctonionFusedLinear")
    raise AttributeError(name)
