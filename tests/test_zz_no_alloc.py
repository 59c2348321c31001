"""walsh_chmod_fwd_noalloc: channel modulation with library-owned scratch.

Some hosts cannot allocate device memory when a layer runs: a runtime whose
device memory is planned once at start-up, or a memory-budgeted serving
process.  The allocation-free entry point serves them by keeping its scratch
in a fixed array inside the library.  It runs the same three kernels as the
caller-scratch path (walsh_chmod_stats / _mlp / _apply through ops.chmod), so
its output must equal that path's bit for bit, on consecutive calls that
reuse the shared array.  The file is named to be collected last.  The
per-context set-up is checked three ways: in this process after every other
test has used the device, in a fresh process (where the set-up runs on the
entry point's first call there), and on a second device when one is visible.
"""
import ctypes
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from walsh_research_b200 import _lib, ops

SCRATCH_FLOATS = 1 << 20
ERR_SCRATCH = -10


def _round64(n):
    return (n + 63) // 64 * 64


def _scratch_floats(nrows, C, seg_len):
    nseg = nrows // seg_len
    nch = -(-seg_len // _lib.call("walsh_chmod_chunk_rows", seg_len))
    return _round64(nseg * nch * C) + 2 * _round64(nseg * (C // 32))


def _module(C, seed):
    from walsh_research_b200.model.moe import HadamardChannelModulation
    torch.manual_seed(seed)
    m = HadamardChannelModulation(C, use_ternary=True, residual_scale=0.5)
    with torch.no_grad():
        m.scale_temp.fill_(0.3)
    return m.cuda()


def _noalloc(x, seg_len, args, norm_w, eps, add_input, out, rscale=0.5):
    w1, w2, gam, st = args
    C = x.shape[-1]
    _lib.call("walsh_chmod_fwd_noalloc", x.data_ptr(), _lib.dcode(x.dtype), x.numel() // C, C, seg_len,
              _lib.ptr(norm_w), eps, w1.data_ptr(), w2.data_ptr(), gam.data_ptr(), st.data_ptr(), rscale,
              1 if add_input else 0, out.data_ptr(), _lib.stream())
    return out


def test_scratch_limit_rejected_on_host():
    """A problem larger than the fixed scratch fails before any device work
    (the pointers are never dereferenced; the size check comes first)."""
    L = _lib.lib()
    p = ctypes.c_void_p(256)
    C, seg_len = 512, 64
    nseg = SCRATCH_FLOATS // (C + 2 * 16) + 64
    assert _scratch_floats(nseg * seg_len, C, seg_len) > SCRATCH_FLOATS
    rc = L.walsh_chmod_fwd_noalloc(p, 1, ctypes.c_int64(nseg * seg_len), C, seg_len, None, ctypes.c_float(1e-6),
                                   p, p, p, p, ctypes.c_float(0.5), 1, p, None)
    assert rc == ERR_SCRATCH
    assert "allocation-free" in _lib.status_str(rc)


def _check_two_calls_in_a_row(index):
    dev = torch.device("cuda", index)
    torch.cuda.set_device(dev)
    g = torch.Generator(device="cpu").manual_seed(11)

    # call 1: the block's layout (bf16 stream rows [B*T*n, C], segment = T rows,
    # chassis RMSNorm weight, x added back)
    C, seg1, nseg1 = 512, 256, 8
    m1 = _module(C, 1)
    a1 = m1.kernel_args()
    x1 = torch.randn((nseg1 * seg1, C), generator=g).to(dev, torch.bfloat16)
    nw = (1.0 + 0.1 * torch.randn(C, generator=g)).to(dev)
    assert _scratch_floats(x1.shape[0], C, seg1) <= SCRATCH_FLOATS

    # call 2: float32, no norm weight, ragged last chunk, no input residual
    seg2, nseg2 = 150, 3
    m2 = _module(C, 2)
    a2 = m2.kernel_args()
    x2 = torch.randn((nseg2 * seg2, C), generator=g).to(dev)

    want1, _, _ = ops.chmod(x1, seg1, *a1[:3], a1[3], norm_w=nw, norm_eps=1e-6, add_input=True)
    want2, _, _ = ops.chmod(x2, seg2, *a2[:3], a2[3], norm_w=None, add_input=False)

    got1 = _noalloc(x1, seg1, a1, nw, 1e-6, True, torch.empty_like(x1))
    got2 = _noalloc(x2, seg2, a2, None, 1e-6, False, torch.empty_like(x2))
    torch.cuda.synchronize()
    # identical kernels and reduction order: tolerance 0 (bit-exact)
    assert torch.equal(got1, want1)
    assert torch.equal(got2, want2)

    # the first problem again, in place (out aliases x), after the scratch
    # was reused by a differently shaped call
    x1c = x1.clone()
    _noalloc(x1c, seg1, a1, nw, 1e-6, True, x1c)
    torch.cuda.synchronize()
    assert torch.equal(x1c, want1)
    assert np.isfinite(got1.float().cpu().numpy()).all()


@pytest.mark.gpu
def test_noalloc_matches_caller_scratch_path_two_calls_in_a_row():
    _check_two_calls_in_a_row(0)


@pytest.mark.gpu
@pytest.mark.skipif(os.environ.get("WALSH_NOALLOC_CHILD") == "1", reason="already the fresh process")
def test_noalloc_in_a_fresh_process():
    """The same check as the first call of a new process on the device."""
    env = dict(os.environ, WALSH_NOALLOC_CHILD="1")
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider",
                        __file__ + "::test_noalloc_matches_caller_scratch_path_two_calls_in_a_row"],
                       capture_output=True, text=True, env=env, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "1 passed" in r.stdout


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_noalloc_on_a_second_device():
    """Each device's context has its own copy of the array: the set-up on
    device 1 must not reuse device 0's address."""
    _check_two_calls_in_a_row(1)
    _check_two_calls_in_a_row(0)
    torch.cuda.set_device(0)
