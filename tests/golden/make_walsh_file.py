"""Generate the .walsh v4 fixtures by running the reference's own writer and
reader.

Usage (in a container where the reference checkout is readable):

    python tests/golden/make_walsh_file.py --ref /path/to/Walsh-Research

1. Builds the seeded 2-layer Walsh-512 state dict of ``cases.py`` (the
   "model_h512" case, vocabulary cut to 512 so the file stays small) with
   float latents (not already ternary), in the reference's parameter names.
2. Saves it as a checkpoint {"model_args": config, "model": state_dict} and
   converts it with the reference's ``compress.compress_model``
   (compress.py:121-358) into ``tests/golden/h512_small.walsh``.
3. Reads that file back with the reference's ``generate_compressed.load_walsh``
   (generate_compressed.py:112-262) and stores every tensor it returns in
   ``tests/golden/h512_small_loaded.npz`` (keys are the parameter names;
   ``__config__`` holds the JSON config).

The .walsh file and the npz are what the tests compare this repository's
loader against; neither the reference nor this script is needed at test time.
"""
from __future__ import annotations

import argparse
import contextlib
import io
import json
import os
import sys
import tempfile

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import cases  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True)
    a = ap.parse_args()
    sys.path.insert(0, a.ref)
    import compress  # noqa: E402  (the reference's writer)
    import generate_compressed  # noqa: E402  (the reference's reader)

    cfg = dict(cases.WALSH512, vocab_size=512)
    rng = np.random.default_rng(77)
    sd = cases.make_state_dict(cfg, 4, seed=31, router_scale=18.3)
    # float latents for the algebra weights (the writer quantises them itself)
    for k in list(sd):
        if k.endswith(".inner.weight"):
            sd[k] = rng.normal(0, 1, sd[k].shape).astype(np.float32)
    state = {k: torch.from_numpy(np.array(v)) for k, v in sd.items()}
    state["output.weight"] = state["tok_embeddings.weight"]          # tied, as the model saves it
    with tempfile.TemporaryDirectory() as d:
        ckpt = os.path.join(d, "ckpt.pt")
        torch.save({"model_args": cfg, "model": state}, ckpt)
        out = os.path.join(HERE, "h512_small.walsh")
        with contextlib.redirect_stdout(io.StringIO()):
            compress.compress_model(ckpt, out)
    with contextlib.redirect_stdout(io.StringIO()):
        loaded, config = generate_compressed.load_walsh(out, verbose=False)
    arrays = {k: v.numpy() for k, v in loaded.items() if not torch.is_complex(v)}
    arrays["__config__"] = np.frombuffer(json.dumps(config).encode(), dtype=np.uint8)
    np.savez_compressed(os.path.join(HERE, "h512_small_loaded.npz"), **arrays)
    print(f"wrote h512_small.walsh ({os.path.getsize(out)} bytes) and {len(arrays) - 1} reference-loaded tensors")


if __name__ == "__main__":
    main()
