"""C-ABI checks that need no GPU: the library loads, exports every symbol
include/walsh.h declares, and rejects bad arguments / injected faults on the
host before any CUDA call."""
import ctypes
import os
import re

import pytest

from walsh_research_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "walsh.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(walsh_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    names = declared_symbols()
    assert len(names) >= 15
    for n in names:
        assert hasattr(L, n), f"{n} declared in walsh.h but not exported"
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"


def test_status_strings_and_version():
    assert _lib.call("walsh_abi_version") >= 2
    assert _lib.status_str(0) == "ok"
    for code in range(-9, 0):
        assert _lib.status_str(code) != "unknown walsh status"


def test_null_pointer_rejected_before_launch():
    L = _lib.lib()
    rc = L.walsh_hadamard_linear_fwd(None, 0, 4, 16, 16, None, 1.0, None, None, None, 0, None)
    assert rc == -1
    rc = L.walsh_attn_fwd(None, None, None, 0, 1, 1, 1, 16, 8, 0, None, None)
    assert rc == -1


def test_bad_dtype_and_shape_rejected():
    L = _lib.lib()
    p = ctypes.c_void_p(16)  # never dereferenced: the check fails first
    assert L.walsh_hadamard_linear_fwd(p, 7, 4, 16, 16, p, 1.0, p, p, p, 0, None) == -3
    assert L.walsh_hadamard_linear_fwd(p, 0, 4, 16, 32, p, 1.0, p, p, p, 0, None) == -2
    # start_pos + T beyond the cache
    assert L.walsh_attn_fwd(p, p, p, 0, 1, 1, 4, 16, 8, 6, p, None) == -2
    # unsupported head_dim
    assert L.walsh_attn_fwd(p, p, p, 0, 1, 1, 4, 24, 8, 0, p, None) == -2


def test_fault_injection(monkeypatch):
    L = _lib.lib()
    monkeypatch.setenv("WALSH_INJECT_FAULT", "moe_fwd")
    p = ctypes.c_void_p(16)
    rc = L.walsh_moe_fwd(p, 0, 4, 512, 6, p, p, p, p, p, p, p, 0, None, 0, None, None, None, None, None, None, None,
                         None, None)
    assert rc == -7
    monkeypatch.setenv("WALSH_INJECT_FAULT", "sinkhorn")
    with pytest.raises(_lib.WalshError, match="injected"):
        _lib.call("walsh_sinkhorn", p, 1, 20, 1e-8, p, None)
    monkeypatch.setenv("WALSH_INJECT_FAULT", "all")
    assert L.walsh_rmsnorm(p, 0, 1, 8, p, 1e-6, p, 0, None) == -7


def test_cpu_tensors_are_rejected():
    import torch
    from walsh_research_b200 import ops
    with pytest.raises(RuntimeError, match="CUDA devices only"):
        ops.rmsnorm(torch.ones(2, 8), torch.ones(8))


@pytest.mark.parametrize("mode,kmin,thr", [(7, 1, 0.1), (1, 0, 0.1), (1, 7, 0.1), (1, 1, 1.5), (1, 1, float("nan"))])
def test_bad_routing_rule_rejected_on_host(mode, kmin, thr):
    """An unknown selection mode, min_experts outside [1, top_k] or a
    threshold outside [0, 1] is an argument error before any launch (the
    device pointers below are never dereferenced)."""
    L = _lib.lib()
    p = ctypes.c_void_p(256)
    rt = ctypes.byref(_lib.MoeRouting(mode, kmin, thr))
    rc = L.walsh_moe_fwd(p, 0, 4, 512, 6, p, p, p, p, p, p, p, 0, None, 0, None, None, None, None, None, None, None,
                         rt, None)
    assert rc == -1
    rc = L.walsh_moe_hidden_fwd(p, p, 1, 4, 512, 6, p, p, p, p, p, p, 0, None, 1, None, None, None, None, None, rt,
                                None)
    assert rc == -1
    rc = L.walsh_moe_router_tc_fwd(p, 1, 4, p, p, 6, p, p, p, rt, None)
    assert rc == -1
