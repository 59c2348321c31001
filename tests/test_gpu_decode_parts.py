"""Batched decode in parts on separate CUDA streams (mHCWalsh._layers_in_parts)
against the same step on the whole batch: every kernel sees the same rows,
so logits, KV-cache rows, router statistics and modulation scales agree to
the last bit, eagerly and replayed from a captured CUDA graph."""
import numpy as np
import pytest
import torch

import cases

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _model(dtype):
    from walsh_research_b200.model import WalshConfig, mHCWalsh
    cfg, n, _, sd = cases.model_inputs("model_h512")
    cfg = dict(cfg, block_size=64)
    m = mHCWalsh(WalshConfig(**cfg), n_streams=n)
    m.load_state_dict({k: torch.from_numpy(np.array(v)) for k, v in sd.items()}, strict=False)
    m = m.to(DEV).eval()
    m.compute_dtype = dtype
    return cfg, m


def _step(m, cfg, ids, prompt, parts, graph):
    from walsh_research_b200 import _lib
    from walsh_research_b200.model import KVCache
    B = ids.shape[0]
    C, H = cfg["n_embd"], cfg["n_head"]
    idt = _lib.inner_dtype(m._act_dtype())
    kv = KVCache(cfg["n_layer"], cfg["block_size"], H, C // H, DEV, dtype=idt, batch_size=B)
    prev, m.decode_streams = m.decode_streams, parts
    with torch.no_grad():
        m(prompt, kv_cache=kv, start_pos=0)
        kv.increment(prompt.shape[1])
        if graph:
            m(ids, kv_cache=kv, start_pos=kv.cached_len)  # warm-up (same cache rows rewritten)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                logits, _ = m(ids, kv_cache=kv, start_pos=kv.cached_len)
            g.replay()
        else:
            logits, _ = m(ids, kv_cache=kv, start_pos=kv.cached_len)
    torch.cuda.synchronize()
    ff = m.layers[0].feed_forward
    cm = m.layers[0].channel_mod if m.layers[0].use_channel_mod else None
    out = {"logits": logits.float().cpu(), "k": kv.k_cache[1].float().cpu(), "v": kv.v_cache[1].float().cpu(),
           "probs": ff._last_router_probs.float().cpu().reshape(B, -1)}
    if cm is not None:
        out["scale"] = cm._last_scale.cpu()
    m.decode_streams = prev
    return out


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("graph", [False, True])
def test_decode_in_parts_equals_whole_batch(dtype, graph):
    cfg, m = _model(dtype)
    B = 160  # above DECODE_PARTS_FROM, odd part sizes with three parts
    assert B >= m.DECODE_PARTS_FROM
    rng = np.random.default_rng(17)
    prompt = torch.from_numpy(rng.integers(0, cfg["vocab_size"], (B, 5))).to(DEV)
    ids = torch.from_numpy(rng.integers(0, cfg["vocab_size"], (B, 1))).to(DEV)
    whole = _step(m, cfg, ids, prompt, 1, graph)
    for parts in (2, 3):
        split = _step(m, cfg, ids, prompt, parts, graph)
        for key in whole:
            if dtype == torch.float32:
                # float32 modulation MLP: the tensor-core form (split bf16
                # GEMM) from CHMOD_MLP_TC_FROM segments, the CUDA-core form
                # below, so a part may take the other one: float32 rounding
                d = (whole[key] - split[key]).abs().max().item()
                assert d <= 1e-4 * max(whole[key].abs().max().item(), 1e-30), (parts, key, d)
            else:
                assert torch.equal(whole[key], split[key]), (parts, key)
