"""The .walsh v4 loader on the GPU: every tensor of the fixture file equals
the reference reader's (tests/golden/h512_small_loaded.npz, written by the
reference's generate_compressed.load_walsh), the device bitmask decode is
bit-exact against the oracle on large random tensors (several 32K-word
rounds of its scan), its 2-bit output equals this library's packer, and a
model built from the file runs."""
import os

import numpy as np
import pytest
import torch

from oracle import walsh_oracle as O

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_load_walsh_equals_the_reference_reader():
    from walsh_research_b200 import ops
    from walsh_research_b200.walsh_file import load_walsh
    want = np.load(os.path.join(GOLDEN, "h512_small_loaded.npz"))
    sd, config, packed = load_walsh(os.path.join(GOLDEN, "h512_small.walsh"))
    assert set(sd) == set(want.files) - {"__config__"}
    for name, t in sd.items():
        assert t.is_cuda
        np.testing.assert_array_equal(t.cpu().numpy(), want[name], err_msg=name)
    assert packed
    for name, pk in packed.items():
        mine, _ = ops.quantize_pack(sd[name])
        assert torch.equal(pk, mine), name
        np.testing.assert_array_equal(pk.cpu().numpy(), O.pack_ternary(want[name]), err_msg=name)


@pytest.mark.parametrize("shape,density", [((3, 7, 13), 0.5), ((32, 64, 64), 0.66), ((1, 3_000_017), 0.1),
                                           ((2000, 511), 0.9)])
def test_device_bitmask_decode_bit_exact(shape, density):
    from walsh_research_b200.walsh_file import decode_ternary
    rng = np.random.default_rng(int(np.prod(shape)))
    w = rng.choice([-1.0, 0.0, 1.0], size=shape, p=[density / 2, 1 - density, density / 2]).astype(np.float32)
    flat = w.ravel()
    mask = np.packbits(flat != 0, bitorder="little").tobytes()
    signs = np.packbits(flat[flat != 0] > 0, bitorder="little").tobytes()
    body = {"shape": shape, "nnz": int((flat != 0).sum()), "mask": mask, "signs": signs}
    dense, packed, err = decode_ternary(body, "cuda")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    np.testing.assert_array_equal(dense.cpu().numpy(), w)
    np.testing.assert_array_equal(packed.cpu().numpy(), O.pack_ternary(w))


def test_population_mismatch_is_reported():
    from walsh_research_b200.walsh_file import decode_ternary
    mask = bytes([0xFF, 0x00])
    body = {"shape": (4, 4), "nnz": 5, "mask": mask, "signs": bytes([0x1F])}
    _, _, err = decode_ternary(body, "cuda")
    torch.cuda.synchronize()
    assert int(err.item()) == -1


def test_model_from_walsh_file_runs():
    from walsh_research_b200.walsh_file import load_walsh_model
    model, missing = load_walsh_model(os.path.join(GOLDEN, "h512_small.walsh"))
    assert "layers.0.attention.wq.inner.weight" not in missing
    ids = torch.randint(0, 512, (2, 16), device="cuda")
    with torch.no_grad():
        logits, _ = model(ids)
    assert logits.shape == (2, 1, 512) and torch.isfinite(logits).all()
