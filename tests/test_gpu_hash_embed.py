"""Hash embeddings on the GPU (walsh_hash_embed_rows): the represented
matrix, the lookup, the output projection and the cross entropy against the
reference's own HashEmbedding (tests/golden/hash_emb.npz), and a whole
mHCWalsh with hash_embeddings=True against the oracle.  (The reference's
mHCWalsh imports the class from a module its checkout does not contain,
src/model/mhc.py:559-561; its chassis.py holds the class, which is what the
golden file records.)"""
import os

import numpy as np
import pytest
import torch

import cases
from oracle import walsh_oracle as O

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _module():
    from walsh_research_b200.model.hash_embeddings import HashEmbedding
    d = cases.op_case("hash_emb")
    nt, nb, C = d["tables"].shape
    m = HashEmbedding(d["importance"].shape[0], C, bucket_size=nb, num_tables=nt)
    with torch.no_grad():
        for i in range(nt):
            m.emb_tables[i].weight.copy_(torch.from_numpy(d["tables"][i]))
        m.importance.weight.copy_(torch.from_numpy(d["importance"]))
    return d, m.cuda()


def test_hash_embedding_matches_reference():
    g = np.load(os.path.join(GOLDEN, "hash_emb.npz"))
    d, m = _module()
    with torch.no_grad():
        E = m._get_all_embeddings()
        # the same products and sums in the same order: bit-exact
        np.testing.assert_array_equal(E.cpu().numpy(), g["all_embeddings"])
        np.testing.assert_array_equal(m._get_chunk_embeddings(100, 357).cpu().numpy(), g["all_embeddings"][100:357])
        y = m(torch.from_numpy(d["x"]).cuda())
        np.testing.assert_allclose(y.cpu().numpy(), g["y"], rtol=1e-6, atol=1e-8)
        h = torch.from_numpy(d["h"]).cuda()
        logits = m.output_projection(h)
        # the split-bfloat16 float32 GEMM (about 2^-16 of the largest logit)
        got = logits.cpu().numpy()
        assert np.abs(got - g["logits"]).max() / np.abs(g["logits"]).max() < 1e-4
        loss = m.chunked_cross_entropy(h, torch.from_numpy(d["targets"]).cuda())
    assert abs(float(loss) - float(g["loss"])) < 1e-5


def test_hash_embedding_model_matches_oracle():
    from walsh_research_b200.model import WalshConfig, mHCWalsh
    cfg, n, idx, sd = cases.model_inputs("model_h512")
    cfg = dict(cfg, vocab_size=1000, hash_embeddings=True)
    torch.manual_seed(3)
    m = mHCWalsh(WalshConfig(**cfg), n_streams=n)
    sd = {k: v for k, v in sd.items() if not k.startswith(("tok_embeddings", "output"))}
    m.load_state_dict({k: torch.from_numpy(np.array(v)) for k, v in sd.items()}, strict=False)
    with torch.no_grad():
        for t in m.tok_embeddings.emb_tables:
            t.weight.normal_(0, 0.05)
        m.tok_embeddings.importance.weight.normal_(1.0, 0.2)
    full = {k: v.detach().numpy().astype(np.float64) if v.is_floating_point() else v.detach().numpy()
            for k, v in m.state_dict().items() if k != "freqs_cis" and not k.endswith(".H")}
    m = m.cuda().eval()
    ids = np.random.default_rng(4).integers(0, 1000, (2, 16))
    with torch.no_grad():
        logits, _ = m(torch.from_numpy(ids).cuda())
        _, loss = m(torch.from_numpy(ids).cuda(), targets=torch.from_numpy(ids).cuda())
    ref, _ = O.mhc_walsh_forward(cfg, full, ids, n)
    err = float(np.abs(logits.cpu().numpy() - ref).max() / np.abs(ref).max())
    assert err < 1e-4, err
    assert torch.isfinite(loss)
