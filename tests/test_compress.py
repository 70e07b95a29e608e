"""The NVFP4 -> 1.58-bit block-64 ternary + rank-16 Q8 core compressor
(flash1017.rs:10342-10645), CPU side: the oracle restatement, pinned by the
reference's own test of it (flash1017.rs:10972-11009: the same input, shapes
and the property that the rank-16 core strictly reduces the Frobenius error),
plus hand-checkable cases of the ternary step."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def reference_test_input():
    """The input of flash1017.rs:10975-10989."""
    rows, cols = 64, 128
    w = np.array([((i * 7 + 3) % 16) | (((i * 13 + 5) % 16) << 4) for i in range(rows * cols // 2)],
                 dtype=np.uint8)
    s = np.array([0x38 if i % 2 == 0 else 0x3C for i in range(rows * cols // 16)], dtype=np.uint8)
    return w, s, np.float32(0.02), rows, cols


def test_reference_accuracy_property(oracle):
    w, s, gs, rows, cols = reference_test_input()
    c = oracle.compress_ternary_b64(w, s, gs, rows, cols, 42)
    assert c["packed"].size == rows * (cols // 4)
    assert c["row_scales"].size == rows
    assert c["core_b"].size == rows * 16
    assert c["core_a"].size == 16 * cols
    assert c["jepa_err_sq"] < c["ternary_err_sq"]
    assert 0 < c["ternary_err_sq"] < c["orig_frob_sq"]


def test_ternary_step_by_hand(oracle):
    """One row of 64 columns.  E2M1 code 0x2 = 1.0, 0xA = -1.0, 0x0 = 0, scale
    0x38 = 1.0, gs 1: 32 columns at +1, 16 at -1, 16 at 0 -> rms = sqrt(48/64);
    every candidate threshold (0.42..0.78 x rms < 1) selects the 48 nonzeros, so
    gamma = 1, codes 2 / 0 / 1, row scale 1/255, block scale 255, residual 0."""
    vals = [1.0] * 32 + [-1.0] * 16 + [0.0] * 16
    code = {1.0: 0x2, -1.0: 0xA, 0.0: 0x0}
    w = np.array([code[vals[2 * i]] | (code[vals[2 * i + 1]] << 4) for i in range(32)], dtype=np.uint8)
    s = np.full(4, 0x38, dtype=np.uint8)
    c = oracle.compress_ternary_b64(w, s, 1.0, 1, 64, 7)
    tern = {1.0: 2, -1.0: 0, 0.0: 1}
    want = np.array([sum(tern[vals[4 * j + u]] << (2 * u) for u in range(4)) for j in range(16)], np.uint8)
    assert np.array_equal(c["packed"], want)
    assert c["block_scales"][0] == 255
    assert c["row_scales"][0] == np.float32(1.0) / np.float32(255.0)
    assert c["ternary_err_sq"] == 0.0


def test_zero_block_and_bad_shape(oracle):
    """An all-zero block gets code 1 everywhere (0x55) and scale 0; cols must be
    a multiple of 64."""
    w = np.zeros(64, dtype=np.uint8)  # 1 row x 128 columns, all E2M1 zero
    s = np.full(8, 0x38, dtype=np.uint8)
    c = oracle.compress_ternary_b64(w, s, 1.0, 1, 128, 1)
    assert np.all(c["packed"] == 0x55) and np.all(c["block_scales"] == 0) and c["row_scales"][0] == 0.0
    with pytest.raises(ValueError):
        oracle.compress_ternary_b64(np.zeros(48, np.uint8), np.zeros(6, np.uint8), 1.0, 1, 96, 1)


def test_oracle_matches_golden_restatement(oracle):
    """The C oracle against the independent float32 / f64 restatement of
    tests/golden/make_golden.py on the same input: every output byte (SHA-256)
    and the three f64 error sums."""
    import hashlib
    import json
    g = json.load(open(os.path.join(ROOT, "tests", "golden", "compress.json")))
    w, s, gs, rows, cols = reference_test_input()
    c = oracle.compress_ternary_b64(w, s, gs, rows, cols, g["seed"])
    for k, digest in g["sha256"].items():
        assert hashlib.sha256(np.ascontiguousarray(c[k]).tobytes()).hexdigest() == digest, k
    for k in ("orig_frob_sq", "ternary_err_sq", "jepa_err_sq"):
        assert c[k] == g[k], k
