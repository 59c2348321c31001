"""Expert parallelism across GPUs: tests/ep_multi_worker.py on every visible
GPU (2 to 8), one process each.  The ffn site evaluated expert-parallel --
through the NVLink exchange kernels and through the NCCL fallback -- must
equal the replicated evaluation of the same tokens bit for bit (the same
router and expert kernels on the same rows; the exchange only moves bytes).
NVLS is kept off (NCCL_NVLS_ENABLE=0)."""
import json
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2+ GPUs")
def test_expert_parallel_across_gpus_equals_replicated(parity_report, tmp_path):
    n = min(torch.cuda.device_count(), 8)
    n = 8 if n >= 8 else (4 if n >= 4 else 2)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", EP_TOKENS="10000", EP_OUT_DIR=str(tmp_path))
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(ROOT, "tests", "ep_multi_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    lines = [json.load(open(tmp_path / f"rank{k}.json")) for k in range(n)]
    for d in lines:
        assert d["nvlink_equal"], d
        assert d["nccl_equal"], d
    d = lines[0]
    parity_report(f"{n} GPUs, {d['tokens']} tokens per rank: ffn site expert-parallel equal to replicated "
                  f"(NVLink and NCCL transports); max over ranks: NVLink {d['nvlink_us']:.1f} us, "
                  f"NCCL {d['nccl_us']:.1f} us, replicated {d['replicated_us']:.1f} us")
