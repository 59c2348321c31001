"""CPU test of the context-keyed address cache behind the allocation-free
entry point (walsh_chmod_fwd_noalloc): a new CUDA context on the same device,
as after a device reset, must miss the cache instead of reusing the address
of the old context's scratch array."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_context_address_cache(tmp_path):
    exe = tmp_path / "ctx_cache_check"
    src = os.path.join(ROOT, "tests", "native", "ctx_cache_check.cpp")
    inc = os.path.join(ROOT, "walsh_research_b200", "csrc")
    subprocess.run(["g++", "-std=c++17", "-O1", "-I" + inc, src, "-o", str(exe), "-pthread"], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "ctx_cache ok" in r.stdout
