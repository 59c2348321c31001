"""The model package mirrors the reference's src.model API and state-dict
layout (checked on CPU: construction and load_state_dict only)."""
import numpy as np
import pytest
import torch

import cases
import walsh_research_b200.model as wm
from walsh_research_b200.model.mhc import mHCWalsh


@pytest.mark.parametrize("name", ["model_h512", "model_h2048"])
def test_state_dict_keys_and_shapes_match_reference(name):
    cfg, n, _, _ = cases.MODEL_CASES[name][0], cases.MODEL_CASES[name][1], None, None
    model = mHCWalsh(wm.WalshConfig(**cfg), n_streams=n)
    sd = model.state_dict()
    expected = cases.param_shapes(cfg, n)
    params = dict(model.named_parameters())
    assert set(params) == set(expected)
    for k, shape in expected.items():
        assert tuple(params[k].shape) == tuple(shape), k
    # persistent buffers the reference also saves
    hd = cfg["n_embd"] // cfg["n_head"]
    assert sd["freqs_cis"].shape == (2 * cfg["block_size"], hd // 2)
    assert sd["layers.0.attention.wq.inner.H"].shape == (32, 32)
    assert sd["layers.0.attention.head_mixer.H"].shape == (32, 32)
    assert "output.weight" in sd


def test_golden_weights_load_strictly():
    cfg, n, idx, sd = cases.model_inputs("model_h512")
    model = mHCWalsh(wm.WalshConfig(**cfg), n_streams=n)
    missing, unexpected = model.load_state_dict({k: torch.from_numpy(np.array(v)) for k, v in sd.items()},
                                                strict=False)
    assert not unexpected
    assert all(("freqs_cis" in m or m.endswith(".H") or m == "output.weight") for m in missing), missing


def test_hadamard_matrix_and_rope_table_match_reference_construction():
    from walsh_research_b200.model.fht_cuda import hadamard_matrix
    from walsh_research_b200.model.chassis import precompute_freqs_cis
    from oracle import walsh_oracle as O
    assert np.array_equal(hadamard_matrix(32, False).numpy(), O.hadamard_matrix(32, False))
    f = precompute_freqs_cis(16, 128)
    cos, sin = O.precompute_rope(16, 128)
    assert np.abs(f.real.numpy() - cos).max() < 1e-6 and np.abs(f.imag.numpy() - sin).max() < 1e-6


def test_forward_refuses_cpu():
    cfg = dict(cases.WALSH512, vocab_size=128, n_layer=1)
    model = mHCWalsh(wm.WalshConfig(**cfg), n_streams=4)
    with pytest.raises(RuntimeError, match="CUDA"):
        model(torch.zeros(1, 4, dtype=torch.long))


def test_cuda_graph_cache_host_logic(monkeypatch):
    """mHCWalsh's graph cache (enable_cuda_graphs), host side, with fakes for the
    CUDA graph calls: first call of a shape runs eagerly, the second captures
    and replays, later calls copy the ids in and replay; another shape or
    start_pos gets its own entry; an in-place parameter update drops the graph
    (eager again, then a new capture); disabling releases the graphs."""
    cfg = dict(cases.MODEL_CASES["model_h512"][0], n_layer=1)
    model = mHCWalsh(wm.WalshConfig(**cfg), n_streams=4)
    log = []

    class FakeGraph:
        def __init__(self):
            self.id = len([e for e in log if e[0] == "capture"])

        def replay(self):
            log.append(("replay", self.id))

    class FakeCapture:
        def __init__(self, g):
            self.g = g

        def __enter__(self):
            log.append(("capture", self.g.id))

        def __exit__(self, *a):
            return False

    def fake_forward(idx, targets, kv_cache, start_pos, return_hidden):
        log.append(("forward", tuple(idx.shape), start_pos))
        model._last_index_error = None
        return torch.zeros(idx.shape[0], 1, 4) + idx.sum().float(), None

    monkeypatch.setattr(torch.cuda, "CUDAGraph", FakeGraph)
    monkeypatch.setattr(torch.cuda, "graph", FakeCapture)
    monkeypatch.setattr(torch.cuda, "synchronize", lambda *a, **k: None)
    monkeypatch.setattr(model, "_forward", fake_forward)

    model.enable_cuda_graphs()
    a, b = torch.ones(2, 3, dtype=torch.long), torch.full((2, 3), 2, dtype=torch.long)
    with torch.no_grad():
        model._graph_forward(a, 0)                     # eager
        assert log[-1][0] == "forward"
        model._graph_forward(a, 0)                     # capture (one traced forward) + replay
        assert [e[0] for e in log[-3:]] == ["capture", "forward", "replay"]
        n = len(log)
        out, _ = model._graph_forward(b, 0)            # replay with the new ids copied in
        assert [e[0] for e in log[n:]] == ["replay"]
        graphs = model.__dict__["_walsh_graphs"]
        key = model._graph_key(a, 0)
        assert key[:4] == ((2, 3), 0, model._act_dtype(), a.device)
        assert torch.equal(graphs[key]["idx"], b)
        # another expert-selection rule is another graph: eager first
        model.layers[0].feed_forward.router.routing_mode = "threshold"
        model._graph_forward(a, 0)
        assert log[-1] == ("forward", (2, 3), 0)
        assert model._graph_key(a, 0) != key and key in graphs
        model.layers[0].feed_forward.router.routing_mode = "topk"
        model._graph_forward(a, 5)                     # other start_pos: its own entry, eager first
        assert log[-1] == ("forward", (2, 3), 5)
        with torch.no_grad():
            model.output.weight.mul_(2.0)              # parameter change: graph dropped
        n = len(log)
        model._graph_forward(a, 0)
        assert [e[0] for e in log[n:]] == ["forward"]
        assert key not in graphs
        model._graph_forward(a, 0)                     # recaptured
        assert "capture" in [e[0] for e in log[n:]]
    model.enable_cuda_graphs(False)
    assert model.__dict__["_walsh_graphs"] == {}


def test_split3_weight_layout_cpu():
    """Operand B of the tensor-core logits GEMM: [W_hi | W_lo | W_hi] in bf16,
    hi + lo = W to about 2^-16 relative, so that [x_hi | x_hi | x_lo] against
    it gives x_hi W_hi + x_hi W_lo + x_lo W_hi."""
    from walsh_research_b200 import ops
    w = torch.from_numpy(np.random.default_rng(3).normal(size=(37, 64)).astype(np.float32))
    w3 = ops.split3_weights(w)
    assert w3.dtype == torch.bfloat16 and tuple(w3.shape) == (37, 192) and w3.is_contiguous()
    hi, lo, hi2 = w3[:, :64].float(), w3[:, 64:128].float(), w3[:, 128:].float()
    assert torch.equal(hi, hi2)
    assert float(((hi + lo) - w).abs().max() / w.abs().max()) < 2.0 ** -15
    x = torch.from_numpy(np.random.default_rng(4).normal(size=(5, 64)).astype(np.float32))
    x_hi = x.to(torch.bfloat16).float()
    x_lo = (x - x_hi).to(torch.bfloat16).float()
    y = torch.cat([x_hi, x_hi, x_lo], 1).double() @ w3.double().t()
    ref = x.double() @ w.double().t()
    assert float((y - ref).abs().max() / ref.abs().max()) < 1e-4


def test_sampling_step_matches_the_reference_rule():
    """mHCWalsh._sample on CPU logits against the reference's own steps
    (temperature, top-k mask, softmax, multinomial) with the same generator."""
    import torch.nn.functional as F
    from walsh_research_b200.model.mhc import mHCWalsh
    logits = torch.randn(5, 300, generator=torch.Generator().manual_seed(0)) * 3
    for temp, k in ((1.0, None), (0.7, 20), (1.3, 1), (0.5, 0)):
        got = mHCWalsh._sample(logits, temp, k, torch.Generator().manual_seed(7))
        z = logits / temp
        if k is not None and k > 0:
            v, _ = torch.topk(z, min(k, z.size(-1)))
            z = z.clone()
            z[z < v[:, [-1]]] = -float("Inf")
        want = torch.multinomial(F.softmax(z, dim=-1), num_samples=1, generator=torch.Generator().manual_seed(7))
        assert torch.equal(got, want)
        if k == 1:
            assert torch.equal(got[:, 0], logits.argmax(-1))


def test_decode_parts_rule():
    """Which steps run in parts on separate streams (host logic): only cached
    steps of at most 4 tokens from DECODE_PARTS_FROM sequences, without
    gradients or expert parallelism, and never more parts than sequences."""
    cfg = dict(cases.WALSH512, vocab_size=128, n_layer=1)
    model = mHCWalsh(wm.WalshConfig(**cfg), n_streams=4)
    kv = object()
    big = model.DECODE_PARTS_FROM
    assert model.decode_streams == 1 and model._decode_parts(big, 1, kv) == 1  # off by default
    model.decode_streams = 2
    with torch.no_grad():
        assert model._decode_parts(big, 1, kv) == 2
        assert model._decode_parts(big, 4, kv) == 2
        assert model._decode_parts(big, 5, kv) == 1          # prefill-sized
        assert model._decode_parts(big - 1, 1, kv) == 1      # small batch
        assert model._decode_parts(big, 1, None) == 1        # no KV cache
        model.decode_streams = 1
        assert model._decode_parts(big, 1, kv) == 1
        model.decode_streams = 3
        assert model._decode_parts(big, 1, kv) == 3
        model.layers[0].__dict__["_ep"] = object()
        assert model._decode_parts(big, 1, kv) == 1          # expert parallel
        del model.layers[0].__dict__["_ep"]
    assert model._decode_parts(big, 1, kv) == 1              # gradients on


def test_hadamard_linear_form_selection_host_logic(monkeypatch):
    """HadamardLinear.forward's choice of device form, with the device calls
    replaced by recorders: 16-bit HadamardLinear(512, 512) from
    HLIN_DENSE_FROM tokens on takes the dense tensor-core GEMM (its matrix
    built once and cached), below that and for 2048 the packed 2-bit kernel,
    float32 the general kernel; HLIN_DENSE = False keeps the packed kernel."""
    from walsh_research_b200 import ops
    from walsh_research_b200.model.fht_cuda import HadamardLinear
    calls, built = [], []
    monkeypatch.setattr(ops, "quantize_pack", lambda w: (torch.zeros(1, dtype=torch.uint8), None))
    monkeypatch.setattr(ops, "hadamard_linear_dense_weights",
                        lambda p, a, b, F, dt: built.append(dt) or (torch.zeros(F, F, dtype=dt), torch.ones(F)))
    monkeypatch.setattr(ops, "hadamard_linear_dense", lambda x, w, s: calls.append("dense") or x)
    monkeypatch.setattr(ops, "hadamard_linear_pk", lambda x, p, a, b: calls.append("packed") or x)
    monkeypatch.setattr(ops, "tc_eligible", lambda x: False)
    monkeypatch.setattr(ops, "hadamard_linear", lambda x, *a, **k: calls.append("general") or x)
    for F in (512, 2048):
        lin = HadamardLinear(F, F)
        for T in (1, ops.HLIN_DENSE_FROM - 1, ops.HLIN_DENSE_FROM):
            for dt in (torch.bfloat16, torch.float16, torch.float32):
                calls.clear()
                lin(torch.empty((T, F), dtype=dt))
                if dt == torch.float32:
                    want = "general"
                elif F == 512 and T >= ops.HLIN_DENSE_FROM:
                    want = "dense"
                else:
                    want = "packed"
                assert calls == [want], (F, T, dt, calls)
    assert built == [torch.bfloat16, torch.float16]  # one dense matrix per 16-bit type, cached
    monkeypatch.setattr(ops, "HLIN_DENSE", False)
    calls.clear()
    HadamardLinear(512, 512)(torch.empty((ops.HLIN_DENSE_FROM, 512), dtype=torch.bfloat16))
    assert calls == ["packed"]
