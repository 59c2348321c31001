"""Pin the numpy oracle against fixtures produced by the reference's own code."""
import os

import numpy as np
import pytest

import cases
from oracle import walsh_oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def golden(name):
    return np.load(os.path.join(GOLDEN, name + ".npz"))


def rel(a, b):
    return float(np.abs(np.asarray(a, np.float64) - b).max() / max(np.abs(b).max(), 1e-30))


def test_pack_bit_exact():
    d, g = cases.op_case("pack"), golden("pack")
    for k in ("w_a", "w_b", "w_c"):
        assert np.array_equal(O.pack_ternary(d[k]), g[k + "_packed"])
        assert np.array_equal(O.unpack_ternary(g[k + "_packed"], d[k].shape[-1]), d[k])


def test_pack_ragged_k_pads_with_zero_code():
    w = np.array([[1, -1, 0, 1, -1]], dtype=np.float32)
    p = O.pack_ternary(w)
    assert p.shape == (1, 2)
    assert p[0, 1] == 0b00010101  # -1 then three zero codes
    assert np.array_equal(O.unpack_ternary(p, 5), w)


def test_quantize_matches_reference():
    d, g = cases.op_case("quant"), golden("quant")
    # the reference's STE returns w_c + (w_q - w_c): equal to w_q up to 1 ulp
    np.testing.assert_allclose(O.quantize_ternary(d["w_unscaled"]), g["unscaled"], atol=2e-7, rtol=0)
    # same ternary pattern; gamma (a float32 mean) may differ by one ulp of summation order
    ours = O.quantize_ternary_scaled(d["w_scaled"])
    gamma = np.abs(g["scaled"]).max()
    assert np.array_equal(np.sign(ours), np.sign(g["scaled"]))
    assert np.array_equal(np.round(g["scaled"] / gamma), np.sign(g["scaled"]))
    np.testing.assert_allclose(ours, g["scaled"], rtol=3e-7, atol=0)


@pytest.mark.parametrize("name", ["hlin_512", "hlin_512_latent", "hlin_2048", "hlin_512x2048", "hlin_2048x512"])
def test_hadamard_linear(name):
    d, g = cases.op_case(name), golden(name)
    y = O.hadamard_linear(d["x"], d["weight"], d["alpha"], d["beta"])
    assert rel(y, g["y"]) < 2e-6


@pytest.mark.parametrize("name", ["headmix", "headmix32"])
def test_head_mixer(name):
    d, g = cases.op_case(name), golden(name)
    assert rel(O.hadamard_head_mixer(d["x"], d["W"], d["beta"]), g["y"]) < 2e-6


def test_sinkhorn():
    d, g = cases.op_case("sinkhorn"), golden("sinkhorn")
    assert rel(O.sinkhorn(d["H"].astype(np.float64)), g["y"]) < 2e-6


def test_stream_mapping():
    d, g = cases.op_case("mapping"), golden("mapping")
    x = d["x"].astype(np.float64)
    for kind in ("pre", "post", "res"):
        h = O.stream_mapping(x, d[f"{kind}_phi"], d[f"{kind}_alpha"], d[f"{kind}_bias"], kind)
        assert h.shape == g[kind].shape
        assert rel(h, g[kind]) < 2e-6


def test_moe():
    d, g = cases.op_case("moe"), golden("moe")
    p = {"r.router.gate.0.weight": d["gate0"], "r.router.gate.2.weight": d["gate2"],
         "r.experts.gate_weights": d["gate_w"], "r.experts.up_weights": d["up_w"],
         "r.experts.down_weights": d["down_w"]}
    y, mask, probs = O.moe(d["x"].astype(np.float64), p, "r.", int(d["top_k"]))
    assert np.array_equal(mask.astype(np.uint8), g["mask"])
    assert rel(probs, g["probs"]) < 2e-6
    assert rel(y, g["y"]) < 2e-6


def test_channel_mod():
    d, g = cases.op_case("chmod"), golden("chmod")
    y = O.channel_mod(d["x"].astype(np.float64), d["w0"], d["w2"], d["scale_temp"])
    assert rel(y, g["y"]) < 2e-6


def test_octonion_linear():
    d, g = cases.op_case("octo_lin"), golden("octo_lin")
    assert rel(O.octonion_linear(d["x"], d["weight"], d["beta"]), g["y"]) < 2e-6


def test_octonion_head_mixer():
    d, g = cases.op_case("octo_headmix"), golden("octo_headmix")
    assert rel(O.octonion_head_mixer(d["x"], d["W"], d["beta"]), g["y"]) < 2e-6


@pytest.mark.parametrize("name", list(cases.MODEL_CASES))
def test_model_forward(name):
    cfg, n, idx, sd = cases.model_inputs(name)
    g = golden(name)
    trace = {}
    logits, h = O.mhc_walsh_forward(cfg, sd, idx, n, trace=trace)
    if "router_mask" in g.files:
        assert np.array_equal(np.stack(trace["router_mask"]).astype(np.uint8), g["router_mask"])
    assert rel(h, g["hidden"]) < 1e-5
    assert rel(logits, g["logits"]) < 1e-5
    if name == "model_h512":
        for i in range(cfg["n_layer"]):
            assert rel(trace["layers"][i], g[f"layer{i}"]) < 1e-5


def test_cached_decode():
    cfg, n, toks, T0, steps, sd = cases.decode_inputs("decode_h512")
    g = golden("decode_h512")["logits"]
    C, H = cfg["n_embd"], cfg["n_head"]
    cache = O.KVCache(cfg["n_layer"], cfg["block_size"], H, C // H)
    outs = []
    lg, _ = O.mhc_walsh_forward(cfg, sd, toks[:, :T0], n, cache=cache, start_pos=0)
    cache.increment(T0)
    outs.append(lg)
    for s in range(steps):
        lg, _ = O.mhc_walsh_forward(cfg, sd, toks[:, T0 + s:T0 + s + 1], n, cache=cache, start_pos=cache.cached_len)
        cache.increment(1)
        outs.append(lg)
    assert rel(np.concatenate(outs, axis=1), g) < 1e-5


def test_fht_properties():
    """Restates the reference's two FHT property tests
    (inference/src/hadamard.rs:228-266): self-inverse and norm-preserving, tol 1e-5."""
    H = O.hadamard_matrix(32)
    x = np.arange(32, dtype=np.float64)
    assert np.abs(H @ (H @ x) - x).max() < 1e-5
    y = (np.arange(32) + 1) / 32.0
    assert abs(np.linalg.norm(H @ y) - np.linalg.norm(y)) < 1e-5


def test_hash_embedding_oracle_and_buffers_match_reference():
    """Hash embeddings (src/model/chassis.py:109-260): the oracle's matrix,
    lookup, output projection and cross entropy, and this package's hashing
    buffers, against the reference's own module (tests/golden/hash_emb.npz)."""
    import torch
    from walsh_research_b200.model.hash_embeddings import HashEmbedding
    d, g = cases.op_case("hash_emb"), np.load(os.path.join(GOLDEN, "hash_emb.npz"))
    nt, nb, C = d["tables"].shape
    V = d["importance"].shape[0]
    m = HashEmbedding(V, C, bucket_size=nb, num_tables=nt)
    np.testing.assert_array_equal(m.hash_a.numpy(), g["hash_a"])
    np.testing.assert_array_equal(m.hash_b.numpy(), g["hash_b"])
    np.testing.assert_array_equal(m.all_indices.numpy(), g["all_indices"])
    np.testing.assert_array_equal(O.hash_indices(g["hash_a"], g["hash_b"], 1000000007, V, nb), g["all_indices"])
    E = O.hash_embedding_matrix(d["tables"], d["importance"], g["all_indices"], C)
    np.testing.assert_allclose(E, g["all_embeddings"], rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(E[d["x"]], g["y"], rtol=1e-6, atol=1e-7)
    logits = d["h"].astype(np.float64) @ E.astype(np.float64).T
    np.testing.assert_allclose(logits, g["logits"], rtol=1e-5, atol=1e-6)
    lse = np.log(np.exp(logits - logits.max(-1, keepdims=True)).sum(-1)) + logits.max(-1)
    loss = float(np.mean(lse - np.take_along_axis(logits, d["targets"][..., None], -1)[..., 0]))
    assert abs(loss - float(g["loss"])) < 1e-5
