"""Thin wrappers of library calls used by several model modules."""
from __future__ import annotations

import torch

from .._lib import call, ptr, stream


def call_hash_rows(tables, importance, indices, C, scale, start, end):
    """walsh_hash_embed_rows over rows start .. end - 1; raises on an index
    outside the tables."""
    out = torch.empty((end - start, C), dtype=torch.float32, device=tables.device)
    err = torch.zeros(1, dtype=torch.int32, device=tables.device)
    call("walsh_hash_embed_rows", ptr(tables), tables.shape[1], ptr(importance), ptr(indices), tables.shape[0], C,
         float(scale), start, end - start, ptr(out), ptr(err), stream())
    if int(err.item()) != 0:
        raise IndexError("hash embedding index outside the tables")
    return out
