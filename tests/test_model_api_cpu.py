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
