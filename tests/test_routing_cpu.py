"""The router's threshold rule on the CPU: the oracle's selection against the
rule as stated (every expert with p > threshold, at least min_experts, at most
max_experts, in descending probability with ties to the lower index), and the
model-side switch that selects it.  The reference's forward uses top-k
(src/model/moe.py:432-436); the threshold rule is the one its HadamardRouter
docstring and arguments describe (src/model/moe.py:383-403)."""
import numpy as np
import pytest

from oracle import walsh_oracle as O


def _rule(p, thr, kmin, kmax):
    """Reference statement of the rule, one token at a time."""
    order = sorted(range(len(p)), key=lambda e: (-p[e], e))
    take = [e for e in order if p[e] > thr][:kmax]
    for e in order:
        if len(take) >= kmin:
            break
        if e not in take:
            take.append(e)
    m = np.zeros(len(p))
    m[take] = 1.0
    return m


@pytest.mark.parametrize("thr,kmin,kmax", [(0.1, 1, 6), (0.05, 2, 6), (0.3, 1, 4), (0.0, 1, 6), (1.0, 3, 6)])
def test_threshold_rule_matches_statement(thr, kmin, kmax):
    rng = np.random.default_rng(int(thr * 100) + kmin + kmax)
    C, E, H = 64, 16, 16
    x = rng.normal(size=(500, C))
    w0 = rng.normal(size=(H, C)) * 0.3
    w2 = rng.normal(size=(E, H)) * rng.uniform(0.2, 3.0)
    w, mask, probs = O.router(x, w0, w2, kmax, threshold=thr, min_experts=kmin)
    for t in range(x.shape[0]):
        np.testing.assert_array_equal(mask[t], _rule(probs[t], thr, kmin, kmax))
    n = mask.sum(-1)
    assert (n >= kmin).all() and (n <= kmax).all()
    np.testing.assert_allclose(w.sum(-1), 1.0, rtol=1e-12)
    assert (w[mask == 0] == 0).all()


def test_topk_is_the_default_and_unchanged():
    rng = np.random.default_rng(3)
    x = rng.normal(size=(200, 64))
    w0, w2 = rng.normal(size=(16, 64)), rng.normal(size=(16, 16))
    _, m_default, _ = O.router(x, w0, w2, 6)
    _, m_thr0, _ = O.router(x, w0, w2, 6, threshold=-1.0, min_experts=6)
    assert (m_default.sum(-1) == 6).all()
    np.testing.assert_array_equal(m_default, m_thr0)


def test_model_switch_selects_the_rule():
    from walsh_research_b200.model import WalshConfig, mHCWalsh
    cfg = dict(block_size=32, vocab_size=64, n_layer=2, n_head=32, n_embd=512, dropout=0.0, bias=False,
               head_mixing=True, algebra="hadamard", hash_embeddings=False, use_moe=True, moe_threshold=0.15,
               moe_min_experts=2, moe_max_experts=6, use_channel_mod=True)
    m = mHCWalsh(WalshConfig(**cfg), n_streams=4)
    r = m.layers[0].feed_forward.router
    assert r.routing() is None
    m.set_moe_routing("threshold")
    assert all(l.feed_forward.router.routing() == (2, 0.15) for l in m.layers)
    m.set_moe_routing("topk")
    assert r.routing() is None
    with pytest.raises(ValueError):
        m.set_moe_routing("sometimes")
