""".walsh v4 model files (the compressed format of the reference's
inference canister) loaded onto the device.

Container (compress.py:121-358 writes it, generate_compressed.py:112-262
reads it): b"SPIN", u16 version, u32 length + JSON config, then chunks of
<marker u8><name: u16 length + UTF-8> followed by a marker-specific body,
ended by b"END!".  Bodies:

  E, A  f32 scale + int8 array          embedding / hash table, value = q * scale
  B     u8 ndim, u32 dims, u32 nnz,     ternary weight as bitmask + signs
        u32 + bitmask, u32 + signs
  S L N H h I   f16 array               beta, alpha, norm, head mixer W / beta, importance
  R     f32 array [.., 2]               RoPE table as (real, imag) pairs
  J     i32 array                       hash indices

where an array is u8 dtype code (0 i8, 1 i32, 2 f16, 3 f32), u8 ndim, u32
dims, raw little-endian data.  The file parsing is host work; the ternary
bitmask decode runs on the GPU (walsh_bitmask_ternary_unpack) and also
yields this library's 2-bit packed layout of each ternary weight.
"""
from __future__ import annotations

import json
import struct

import numpy as np
import torch

from . import _lib
from ._lib import call, ptr, stream

_DT = {0: np.int8, 1: np.int32, 2: np.float16, 3: np.float32}
_FLOAT_ARRAY = {b"S", b"L", b"N", b"H", b"h", b"I"}


class _Reader:
    def __init__(self, data: bytes):
        self.d, self.o = data, 0

    def take(self, n):
        if self.o + n > len(self.d):
            raise ValueError("truncated .walsh file")
        b = self.d[self.o:self.o + n]
        self.o += n
        return b

    def u8(self):
        return self.take(1)[0]

    def u16(self):
        return struct.unpack("<H", self.take(2))[0]

    def u32(self):
        return struct.unpack("<I", self.take(4))[0]

    def f32(self):
        return struct.unpack("<f", self.take(4))[0]

    def name(self):
        return self.take(self.u16()).decode("utf-8")

    def array(self):
        code, ndim = self.u8(), self.u8()
        if code not in _DT:
            raise ValueError(f"unknown array dtype code {code}")
        shape = tuple(self.u32() for _ in range(ndim))
        dt = np.dtype(_DT[code])
        n = int(np.prod(shape)) if shape else 1
        return np.frombuffer(self.take(n * dt.itemsize), dtype=dt).reshape(shape).copy()


def parse_walsh(path_or_bytes):
    """(config dict, version, list of (marker, name, body)) of a .walsh file;
    bodies are numpy arrays, (scale, int8 array) for E/A, or a dict for B."""
    data = path_or_bytes if isinstance(path_or_bytes, (bytes, bytearray)) else open(path_or_bytes, "rb").read()
    r = _Reader(bytes(data))
    if r.take(4) != b"SPIN":
        raise ValueError("not a .walsh file (magic)")
    version = r.u16()
    config = json.loads(r.take(r.u32()).decode("utf-8"))
    chunks = []
    while r.o < len(r.d):
        marker = r.take(1)
        if marker == b"\x00":
            break
        if marker == b"E" and r.d[r.o:r.o + 3] == b"ND!":
            break
        name = r.name()
        if marker in (b"E", b"A"):
            scale = r.f32()
            chunks.append((marker, name, (scale, r.array())))
        elif marker == b"B":
            ndim = r.u8()
            shape = tuple(r.u32() for _ in range(ndim))
            nnz = r.u32()
            mask = r.take(r.u32())
            signs = r.take(r.u32())
            chunks.append((marker, name, {"shape": shape, "nnz": nnz, "mask": mask, "signs": signs}))
        elif marker in _FLOAT_ARRAY or marker in (b"R", b"J"):
            chunks.append((marker, name, r.array()))
        else:
            raise ValueError(f"unknown .walsh chunk marker {marker!r} ({name})")
    return config, version, chunks


def decode_ternary(body, device):
    """(dense float32 tensor, 2-bit packed uint8 tensor [.., ceil(k/4)]) of a
    'B' chunk, decoded on the device."""
    shape, nnz = body["shape"], body["nnz"]
    total = int(np.prod(shape))
    k = shape[-1]
    mask = torch.frombuffer(bytearray(body["mask"]), dtype=torch.uint8).to(device)
    signs = torch.frombuffer(bytearray(body["signs"] or b"\0"), dtype=torch.uint8).to(device)
    dense = torch.empty(shape, dtype=torch.float32, device=device)
    packed = torch.empty(shape[:-1] + ((k + 3) // 4,), dtype=torch.uint8, device=device)
    err = torch.zeros(1, dtype=torch.int32, device=device)
    call("walsh_bitmask_ternary_unpack", ptr(mask), len(body["mask"]), ptr(signs), max(len(body["signs"]), 1),
         total, nnz, k, ptr(dense), ptr(packed), ptr(err), stream())
    return dense, packed, err


def load_walsh(path, device="cuda"):
    """(state_dict, config, packed) of a .walsh file with every tensor on the
    device: the same names and values the reference's load_walsh returns
    (generate_compressed.py:112-262), and ``packed``: name -> 2-bit packed
    ternary weight (this library's layout) for each bitmask chunk."""
    _lib.require_cuda(torch.empty(0, device=device))
    config, _, chunks = parse_walsh(path)
    sd, packed, errs = {}, {}, []
    for marker, name, body in chunks:
        if marker in (b"E", b"A"):
            scale, q = body
            sd[name] = torch.from_numpy(q).to(device).float() * np.float32(scale)
        elif marker == b"B":
            dense, pk, err = decode_ternary(body, device)
            sd[name], packed[name] = dense, pk
            errs.append((name, err))
        elif marker == b"R":
            sd[name] = torch.view_as_complex(torch.from_numpy(body.astype(np.float32)).contiguous()).to(device)
        elif marker == b"J":
            sd[name] = torch.from_numpy(body.astype(np.int32)).to(device)
        else:
            sd[name] = torch.from_numpy(body.astype(np.float32)).to(device)
    for name, err in errs:
        if int(err.item()) != 0:
            raise ValueError(f"{name}: bitmask population differs from its non-zero count")
    return sd, config, packed


def load_walsh_model(path, device="cuda", n_streams=4):
    """An mHCWalsh built from a .walsh file's config with the file's tensors
    loaded (strict=False, as the reference loads them: the format carries
    the attention projections, their scales, norms, head mixers and the
    embedding; other parameters keep their initialisation).  Returns
    (model, missing keys)."""
    from .model import WalshConfig, mHCWalsh
    sd, config, _ = load_walsh(path, device)
    fields = {k: v for k, v in config.items() if k in WalshConfig.__dataclass_fields__}
    model = mHCWalsh(WalshConfig(**fields), n_streams=n_streams).to(device)
    if "tok_embeddings.weight" in sd and "output.weight" not in sd:
        sd["output.weight"] = sd["tok_embeddings.weight"]
    missing, unexpected = model.load_state_dict(sd, strict=False)
    if unexpected:
        raise ValueError(f"tensors the model does not have: {unexpected[:5]}")
    return model.eval(), missing
