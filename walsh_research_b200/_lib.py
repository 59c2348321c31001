"""ctypes binding of libwalsh.so (the C ABI declared in include/walsh.h).

The library is loaded from the package directory (built in-tree by
``python -m walsh_research_b200.build``).  There is no fallback: if it is
missing, every op raises.  Every wrapper checks the returned walsh_status and
raises ``WalshError`` with the library's own message.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import c_float, c_int, c_int64, c_void_p

import torch

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libwalsh.so")

F32, BF16, F16 = 0, 1, 2
P = c_void_p

# name -> argument types (restype is int/walsh_status unless listed in _RESTYPE)
SIGNATURES = {
    "walsh_status_str": [c_int],
    "walsh_abi_version": [],
    "walsh_ternary_quantize_pack": [P, c_int64, c_int, P, P, P],
    "walsh_ternary_unpack": [P, c_int64, c_int, P, P],
    "walsh_hadamard_linear_fwd": [P, c_int, c_int64, c_int, c_int, P, c_float, P, P, P, c_int, P],
    "walsh_head_mixer_fwd": [P, c_int, c_int64, c_int, c_int, P, P, P, P],
    "walsh_attn_qkv_fwd": [P, c_int, c_int, c_int, c_int, c_int, P, P, P, P, P, P, P, P, P, P, P, c_int, c_int,
                           P, P, P, c_int, c_int, P],
    "walsh_attn_fwd": [P, P, P, c_int, c_int, c_int, c_int, c_int, c_int, c_int, P, P],
    "walsh_hadamard_linear_tc_fwd": [P, c_int64, P, c_float, P, P, P, P],
    "walsh_attn_qkv_tc_fwd": [P, c_int, c_int, c_int, P, P, P, P, P, P, P, P, P, P, P, c_int, c_int, P, P, P,
                              c_int, P],
    "walsh_attn_out_tc_fwd": [P, c_int64, P, P, P, P, P, P, c_int, P, P, P],
    "walsh_mhc_map": [P, c_int, c_int64, c_int, P, P, P, P, c_float, P, c_float, P, c_int, P, P],
    "walsh_map_error": [c_int],
    "walsh_map_set_pipe": [c_int],
    "walsh_mhc_post": [P, P, P, c_int, c_int64, c_int, P, P],
    "walsh_sinkhorn": [P, c_int64, c_int, c_float, P, P],
    "walsh_moe_fwd": [P, c_int, c_int64, c_int, c_int, P, P, P, P, P, P, P, c_int, P, c_int, P, P, P, P, P, P, P,
                      P, P],
    "walsh_octo_set_mainloop": [c_int],
    "walsh_octo_set_narrow": [c_int],
    "walsh_octo_set_tma_store": [c_int],
    "walsh_tc05_error": [c_int],
    "walsh_attn_set_path": [c_int],
    "walsh_moe_router_tc_fwd": [P, c_int, c_int64, P, P, c_int, P, P, P, P, P],
    "walsh_moe_experts_tc_fwd": [P, c_int, c_int64, P, P, P, P, P, c_int, P, c_int, P, P, P],
    "walsh_tc05_wait_selftest": [ctypes.c_longlong, P],
    "walsh_octo_linear_fwd": [P, c_int, c_int64, c_int, P, P, c_int, c_int64, P, P, P],
    "walsh_octo_qkv_fwd": [P, c_int, c_int, c_int, c_int, c_int, P, P, c_int, P, P, P, c_int, c_int, P, P, P, c_int,
                           P],
    "walsh_octo_swiglu_fwd": [P, c_int, c_int64, c_int, P, P, c_int, P, c_int64, P, P],
    "walsh_octo_post_fwd": [P, c_int, c_int64, c_int, P, P, c_int, P, c_int, P, c_int, P, P, P],
    "walsh_moe_hidden_fwd": [P, P, c_int, c_int64, c_int, c_int, P, P, P, P, P, P, c_int, P, c_int, P, P, P, P, P,
                             P, P],
    "walsh_chmod_chunk_rows": [c_int],
    "walsh_chmod_stats": [P, c_int, c_int64, c_int, c_int, P, c_float, P, P],
    "walsh_chmod_mlp": [P, c_int, c_int, c_int, P, P, P, P, P, P, P],
    "walsh_chmod_apply": [P, c_int, c_int64, c_int, c_int, P, c_float, P, P, c_float, c_int, P, P],
    "walsh_chmod_rows_fwd": [P, c_int, c_int64, c_int, P, c_float, P, P, P, P, c_float, c_int, P, P, P, P],
    "walsh_chmod_mlp_tc": [P, c_int, c_int, c_int, P, P, P, P, P, P, P, P],
    "walsh_linear_split_tc_fwd": [P, c_int64, c_int, P, c_int64, P, P, P],
    "walsh_linear_split_tc_scratch_bytes": [c_int64, c_int],
    "walsh_chmod_mlp_tc_scratch_bytes": [c_int, c_int],
    "walsh_chmod_fwd_noalloc": [P, c_int, c_int64, c_int, c_int, P, c_float, P, P, P, P, c_float, c_int, P, P],
    "walsh_embed_gather": [P, c_int64, P, c_int, c_int64, c_int, P, P, P],
    "walsh_linear_fwd": [P, c_int, c_int64, c_int, c_int64, P, c_int, c_int64, P, P, c_int, P],
    "walsh_linear_split_fwd": [P, c_int, c_int64, c_int, c_int64, P, P, c_int64, P, P, P],
    "walsh_rmsnorm": [P, c_int, c_int64, c_int, P, c_float, P, c_int, P],
    "walsh_moe_experts_tc_part_fwd": [P, c_int, c_int64, P, P, P, P, c_int, c_int, P, P],
    "walsh_ep_dispatch": [P, c_int, c_int64, c_int, P, c_int, c_int, P, P, P, P, ctypes.c_uint32, P],
    "walsh_ep_combine": [P, c_int, c_int64, c_int, c_int, c_int, P, P, P, ctypes.c_uint32, P],
    "walsh_ep_wait": [P, c_int, c_int, ctypes.c_uint32, ctypes.c_longlong, P, P],
    "walsh_ipc_handle": [P, P, P],
    "walsh_ipc_open": [P, c_int64, P, P],
    "walsh_ipc_close": [P],
    "walsh_ipc_handle_bytes": [],
    "walsh_bitmask_ternary_unpack": [P, c_int64, P, c_int64, c_int64, c_int64, c_int, P, P, P, P],
    "walsh_hash_embed_rows": [P, c_int64, P, P, c_int, c_int, c_float, c_int64, c_int64, P, P, P],
    "walsh_hadamard_linear_pk_fwd": [P, c_int, c_int64, c_int, P, P, P, P, P],
    "walsh_hadamard_linear_dense_weights": [P, P, P, c_int, c_int, P, P, P],
    "walsh_hadamard_linear_dense_fwd": [P, c_int, c_int64, c_int, P, P, P, P],
    "walsh_hlin_pk_error": [c_int],
}
_RESTYPE = {"walsh_status_str": ctypes.c_char_p, "walsh_ipc_handle_bytes": c_int, "walsh_chmod_mlp_tc_scratch_bytes": ctypes.c_int64,
            "walsh_linear_split_tc_scratch_bytes": ctypes.c_int64}
# kernels each entry point launches (for the launch accounting reported by bench.py)
KERNELS_PER_CALL = {"walsh_ternary_quantize_pack": 2, "walsh_chmod_fwd_noalloc": 3, "walsh_octo_set_mainloop": 0, "walsh_octo_set_narrow": 0, "walsh_octo_set_tma_store": 0,
                    "walsh_chmod_mlp_tc": 3, "walsh_chmod_mlp_tc_scratch_bytes": 0,
                    "walsh_linear_split_tc_fwd": 2, "walsh_linear_split_tc_scratch_bytes": 0,
                    "walsh_tc05_error": 0, "walsh_attn_set_path": 0, "walsh_map_error": 0, "walsh_map_set_pipe": 0, "walsh_hlin_pk_error": 0, "walsh_chmod_chunk_rows": 0, "walsh_status_str": 0,
                    "walsh_abi_version": 0, "walsh_ipc_handle": 0, "walsh_ipc_open": 0, "walsh_ipc_close": 0,
                    "walsh_ipc_handle_bytes": 0}
launch_count = 0
# entry points that return a plain int rather than a status
_PLAIN_INT = {"walsh_abi_version", "walsh_chmod_chunk_rows", "walsh_octo_set_mainloop", "walsh_octo_set_narrow", "walsh_octo_set_tma_store", "walsh_tc05_error",
              "walsh_map_error", "walsh_attn_set_path", "walsh_map_set_pipe", "walsh_hlin_pk_error"}


class MoeTcWeights(ctypes.Structure):
    """walsh_moe_tc_weights: bfloat16 copies of the router / expert weights."""
    _fields_ = [("w1", P), ("w2", P), ("gate", P), ("up", P), ("down", P)]


ROUTE_TOPK, ROUTE_THRESHOLD = 0, 1


class MoeRouting(ctypes.Structure):
    """walsh_moe_routing: the expert-selection rule (NULL = the reference's top-k)."""
    _fields_ = [("mode", c_int), ("min_experts", c_int), ("threshold", c_float)]


class WalshError(RuntimeError):
    def __init__(self, name: str, code: int, msg: str):
        super().__init__(f"{name} failed: {msg} (status {code})")
        self.code = code


_lib = None


def lib() -> ctypes.CDLL:
    """Load libwalsh.so once.  Raises if the library was not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"libwalsh.so not found at {LIB_PATH}; build it with "
                               f"`python -m walsh_research_b200.build` (no CPU fallback exists)")
        L = ctypes.CDLL(LIB_PATH)
        for name, args in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = _RESTYPE.get(name, c_int)
        _lib = L
    return _lib


def status_str(code: int) -> str:
    return lib().walsh_status_str(code).decode()


def call(name: str, *args) -> int:
    global launch_count
    rc = getattr(lib(), name)(*args)
    launch_count += KERNELS_PER_CALL.get(name, 1)
    if name in _PLAIN_INT or name in _RESTYPE:
        return rc
    if rc != 0:
        raise WalshError(name, rc, status_str(rc))
    return rc


# ---------------------------------------------------------------------------
# tensor helpers
# ---------------------------------------------------------------------------

def ptr(t):
    """Device pointer of a tensor (None -> NULL)."""
    if t is None:
        return None
    return t.data_ptr()


def dcode(dtype: torch.dtype) -> int:
    if dtype == torch.float32:
        return F32
    if dtype == torch.bfloat16:
        return BF16
    if dtype == torch.float16:
        return F16
    raise TypeError(f"walsh kernels take float32, bfloat16 or float16 activations, got {dtype}")


def inner_dtype(stream_dtype: torch.dtype) -> torch.dtype:
    """Storage type of the normalised activations (u, q/k/v, attention output)
    for a residual stream of ``stream_dtype``: float16 next to a 16-bit
    stream (values are bounded by the normalisations, fp16 keeps 3 more
    mantissa bits than bf16), float32 next to a float32 stream."""
    return torch.float16 if stream_dtype in (torch.bfloat16, torch.float16) else stream_dtype


_RAW_STREAM = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream() -> int:
    """Handle of the current CUDA stream of the current device (read without
    building a torch.cuda.Stream object: a few microseconds less per op)."""
    if _RAW_STREAM is not None:
        return _RAW_STREAM(torch._C._cuda_getDevice())
    return torch.cuda.current_stream().cuda_stream


def require_cuda(*tensors):
    """The hot path runs only on CUDA tensors; there is no CPU fallback."""
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("walsh_research_b200 runs on CUDA devices only (no CPU fallback); "
                               f"got a tensor on {t.device}")
