"""Caching of load-time derived device tensors (packed ternary weights,
transposed router weights, concatenated mHC projections, RoPE tables).

A derived value is keyed on the (storage pointer, version counter, dtype) of
its source parameters, so it is rebuilt after ``load_state_dict``, an in-place
update or ``.to()`` and reused otherwise.
"""
from __future__ import annotations

import torch


def _key(sources, extra):
    return tuple((s.data_ptr(), s._version, s.dtype, s.device) for s in sources) + tuple(extra)


def cached(module, name: str, sources, builder, extra=()):
    store = module.__dict__.setdefault("_walsh_prep", {})
    key = _key(sources, extra)
    hit = store.get(name)
    if hit is None or hit[0] != key:
        with torch.no_grad():
            hit = (key, builder())
        store[name] = hit
    return hit[1]


def clear(module):
    for m in module.modules():
        m.__dict__.pop("_walsh_prep", None)
