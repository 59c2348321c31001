"""Cached, batched mHCWalsh.generate against the float64 oracle (reference
semantics: src/model/mhc.py:753-789 for the sampling step,
src/model/chassis.py:600-655 for the cached loop).

The two loops are different models of the sequence, in the reference as
here: channel modulation averages over the tokens of the current call
(src/model/moe.py:681-722), so a cached step (one new token) sees a
different bulk state than a re-forward of the whole context.  Each loop is
therefore checked against the oracle run the same way: the cached loop
against the oracle's one-sequence KV cache, the uncached loop against full
re-forwards."""
import numpy as np
import pytest
import torch

import cases
from oracle import walsh_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _model(dtype=torch.float32, block_size=64):
    from walsh_research_b200.model import WalshConfig, mHCWalsh
    cfg, n, _, sd = cases.model_inputs("model_h512")
    cfg = dict(cfg, block_size=block_size)
    m = mHCWalsh(WalshConfig(**cfg), n_streams=n)
    m.load_state_dict({k: torch.from_numpy(np.array(v)) for k, v in sd.items()}, strict=False)
    m = m.to(DEV).eval()
    m.compute_dtype = dtype
    return cfg, n, sd, m


def _oracle_greedy(cfg, n, sd, prompt, steps, cached):
    """Arg-max continuation of one prompt [T] by the oracle."""
    if not cached:
        seq = prompt[None]
        for _ in range(steps):
            logits, _ = O.mhc_walsh_forward(cfg, sd, seq, n)
            seq = np.concatenate([seq, logits[:, -1].argmax(-1)[:, None]], axis=1)
        return seq[0]
    C, H = cfg["n_embd"], cfg["n_head"]
    cache = O.KVCache(cfg["n_layer"], cfg["block_size"], H, C // H)
    logits, _ = O.mhc_walsh_forward(cfg, sd, prompt[None], n, cache=cache, start_pos=0)
    cache.increment(len(prompt))
    out = list(prompt) + [int(logits[0, -1].argmax())]
    for _ in range(steps - 1):
        logits, _ = O.mhc_walsh_forward(cfg, sd, np.array([[out[-1]]]), n, cache=cache, start_pos=cache.cached_len)
        cache.increment(1)
        out.append(int(logits[0, -1].argmax()))
    return np.array(out)


def test_greedy_generation_matches_the_oracle():
    """top_k = 1 makes every draw the arg-max: three prompts decoded together
    through the batched KV cache give, per sequence, the oracle's cached
    arg-max continuation; the uncached loop gives the oracle's re-forward
    continuation."""
    cfg, n, sd, m = _model()
    rng = np.random.default_rng(5)
    idx = torch.from_numpy(rng.integers(0, cfg["vocab_size"], (3, 12))).to(DEV)
    a = m.generate(idx, 6, top_k=1, use_cache=True)
    b = m.generate(idx, 4, top_k=1, use_cache=False)
    assert a.shape == (3, 18) and b.shape == (3, 16)
    assert torch.equal(a[:, :12], idx) and torch.equal(b[:, :12], idx)
    for i in range(3):
        p = idx[i].cpu().numpy()
        assert np.array_equal(a[i].cpu().numpy(), _oracle_greedy(cfg, n, sd, p, 6, True)), i
        assert np.array_equal(b[i].cpu().numpy(), _oracle_greedy(cfg, n, sd, p, 4, False)), i


def test_sampled_generation_follows_the_reference_loop():
    """With temperature and top-k the cached loop draws exactly what the
    reference's loop draws from the same logits and generator: prefill into
    the cache, sample, then one forward per new token."""
    from walsh_research_b200.model import KVCache
    cfg, n, sd, m = _model()
    rng = np.random.default_rng(6)
    idx = torch.from_numpy(rng.integers(0, cfg["vocab_size"], (2, 9))).to(DEV)
    g = torch.Generator(device=DEV).manual_seed(1234)
    got = m.generate(idx, 10, temperature=0.8, top_k=50, generator=g)
    g = torch.Generator(device=DEV).manual_seed(1234)
    C, H = cfg["n_embd"], cfg["n_head"]
    cache = KVCache(cfg["n_layer"], cfg["block_size"], H, C // H, idx.device, dtype=torch.float32, batch_size=2)
    with torch.no_grad():
        logits, _ = m(idx, kv_cache=cache, start_pos=0)
        cache.increment(idx.shape[1])
        seq = idx
        for _ in range(10):
            nxt = m._sample(logits[:, -1, :], 0.8, 50, g)
            seq = torch.cat((seq, nxt), dim=1)
            logits, _ = m(nxt, kv_cache=cache, start_pos=cache.cached_len)
            cache.increment(1)
    assert torch.equal(got, seq)
    g = torch.Generator(device=DEV).manual_seed(99)
    assert not torch.equal(got, m.generate(idx, 10, temperature=0.8, top_k=50, generator=g))


def test_cached_generation_stops_when_the_cache_is_full():
    """block_size 16, prompt 12: one token from the prefill, then one per
    cached step until 16 positions are cached (reference behaviour)."""
    cfg, n, sd, m = _model(block_size=16)
    idx = torch.from_numpy(np.random.default_rng(7).integers(0, cfg["vocab_size"], (2, 12))).to(DEV)
    out = m.generate(idx, 10, top_k=1)
    assert out.shape == (2, 17)


def test_16bit_generate_runs_and_starts_like_the_uncached_loop():
    """16-bit mode: the first token comes from the prefill forward in both
    loops (same kernels with and without the cache)."""
    cfg, n, sd, m = _model(torch.bfloat16)
    idx = torch.from_numpy(np.random.default_rng(8).integers(0, cfg["vocab_size"], (4, 20))).to(DEV)
    a = m.generate(idx, 6, top_k=1)
    b = m.generate(idx, 1, top_k=1, use_cache=False)
    assert a.shape == (4, 26)
    assert torch.equal(a[:, :21], b)
