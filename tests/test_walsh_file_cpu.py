"""The .walsh v4 container on the CPU: this repository's parser and the
oracle's bitmask decode against the reference's own reader
(generate_compressed.load_walsh), whose output on the fixture file is
stored in tests/golden/h512_small_loaded.npz (tests/golden/make_walsh_file.py
wrote both with the reference's compress.py and generate_compressed.py)."""
import json
import os

import numpy as np
import pytest

from oracle import walsh_oracle as O
from walsh_research_b200.walsh_file import parse_walsh

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _fixture():
    return os.path.join(GOLDEN, "h512_small.walsh"), np.load(os.path.join(GOLDEN, "h512_small_loaded.npz"))


def test_parse_matches_the_reference_reader():
    path, want = _fixture()
    config, version, chunks = parse_walsh(path)
    assert version == 4
    assert config == json.loads(bytes(want["__config__"]).decode())
    names = set()
    for marker, name, body in chunks:
        names.add(name)
        if marker == b"B":
            got = O.bitmask_ternary_decode(body["mask"], body["signs"], body["shape"], body["nnz"])
        elif marker in (b"E", b"A"):
            scale, q = body
            got = q.astype(np.float32) * np.float32(scale)
        else:
            got = body.astype(np.float32)
        np.testing.assert_array_equal(got, want[name], err_msg=name)
    assert names == set(want.files) - {"__config__"}


def test_bitmask_decode_known_answer():
    # positions 0, 3, 9 non-zero with signs +, -, +; 12 positions
    mask = bytes([0b00001001, 0b00000010])
    signs = bytes([0b00000101])
    got = O.bitmask_ternary_decode(mask, signs, (3, 4), 3)
    np.testing.assert_array_equal(got, np.array([[1, 0, 0, -1], [0, 0, 0, 0], [0, 1, 0, 0]], dtype=np.float32))


def test_bad_files_are_rejected():
    path, _ = _fixture()
    data = open(path, "rb").read()
    with pytest.raises(ValueError, match="magic"):
        parse_walsh(b"XXXX" + data[4:])
    with pytest.raises(ValueError, match="truncated"):
        parse_walsh(data[: len(data) // 2])
