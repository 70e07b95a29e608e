"""The 106 GB format's compressor on the GPU (ffn_b200_compress_ternary_b64:
compress_nvfp4_matrix_to_158_jepa_q8, flash1017.rs:10377-10645) against the
oracle restatement, which the reference's own test pins (tests/test_compress.py).

Ternary codes, row scales and U8 block scales: bit-exact.  The rank-16 core:
its products run in the reference's order, so it matches too; the only
reordered sums are the Gram-Schmidt f64 dots and norms, which are rounded to
f32 before use, so at most rare last-bit differences can reach the int8 core:
the test allows 0.5 % of the core entries to differ by one step, and the core
scales 1e-5 relative.  A compressed expert then runs through the ternary
kernels and matches the oracle's expert made from the oracle's tensors
(max|dy|/max|y| <= 1e-3, cosine >= 0.99999)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def host(t):
    return t.detach().cpu().numpy()


def dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def compress_both(oracle, ffn, w, s, gs, rows, cols, seed):
    ref = oracle.compress_ternary_b64(w, s, gs, rows, cols, seed)
    m = ffn.TernaryMatrix.compress(dev(w), dev(s), gs, rows, cols, seed)
    return ref, m


def check_against_oracle(ref, m, what):
    a, a_sc, b, b_sc = m.core
    assert np.array_equal(host(m.p), ref["packed"]), f"{what}: ternary codes"
    assert np.array_equal(host(m.bs), ref["block_scales"]), f"{what}: block scales"
    assert np.array_equal(host(m.rs), ref["row_scales"]), f"{what}: row scales"
    for got, want, sc_got, sc_want, name in ((host(b), ref["core_b"], host(b_sc), ref["core_b_sc"], "core_b"),
                                              (host(a), ref["core_a"], host(a_sc), ref["core_a_sc"], "core_a")):
        d = np.abs(got.astype(np.int32) - want.astype(np.int32))
        assert d.max() <= 1 and (d > 0).mean() <= 0.005, f"{what}: {name} ({(d > 0).sum()} entries differ)"
        np.testing.assert_allclose(sc_got, sc_want, rtol=1e-5, atol=0, err_msg=f"{what}: {name} scales")


def test_reference_test_input(oracle, ffn, cuda):
    """The input of the reference's compressor test (flash1017.rs:10975-10995)."""
    rows, cols = 64, 128
    w = np.array([((i * 7 + 3) % 16) | (((i * 13 + 5) % 16) << 4) for i in range(rows * cols // 2)],
                 dtype=np.uint8)
    s = np.array([0x38 if i % 2 == 0 else 0x3C for i in range(rows * cols // 16)], dtype=np.uint8)
    ref, m = compress_both(oracle, ffn, w, s, np.float32(0.02), rows, cols, 42)
    check_against_oracle(ref, m, "reference test input")


@pytest.mark.parametrize("rows,cols,seed", [(256, 512, 7), (2048, 4096, 11), (96, 320, 3)])
def test_random_nvfp4(oracle, ffn, cuda, rows, cols, seed):
    w, s = oracle.gen_nvfp4(oracle.key(seed, 9, rows, cols), rows, cols)
    ref, m = compress_both(oracle, ffn, w, s, np.float32(0.5), rows, cols, seed)
    check_against_oracle(ref, m, f"{rows}x{cols}")


def test_zero_rows(oracle, ffn, cuda):
    """All-zero blocks: codes 0x55, scales 0, core of a zero residual = 0."""
    rows, cols = 32, 128
    w = np.zeros(rows * cols // 2, np.uint8)
    s = np.full(rows * cols // 16, 0x38, np.uint8)
    ref, m = compress_both(oracle, ffn, w, s, np.float32(1.0), rows, cols, 5)
    check_against_oracle(ref, m, "zero matrix")
    assert np.all(host(m.p) == 0x55) and np.all(host(m.core[0]) == 0)


def test_bad_shape(ffn, cuda):
    import torch
    w = torch.zeros(16 * 48, dtype=torch.uint8, device="cuda")
    s = torch.zeros(16 * 6, dtype=torch.uint8, device="cuda")
    with pytest.raises(ffn.FfnError):
        ffn.TernaryMatrix.compress(w, s, 1.0, 16, 96, 1)  # cols % 64 != 0


def test_compressed_expert_forward(oracle, ffn, cuda):
    """An NVFP4 expert compressed on the GPU runs through the ternary kernels
    and matches the oracle's expert built from the oracle's compressed tensors."""
    H, I = 512, 256
    shapes = ((I, H), (I, H), (H, I))
    src = [oracle.gen_nvfp4(oracle.key(21, 0, k, oracle.TAG_W1), r, c) for k, (r, c) in enumerate(shapes)]
    mats, ps, rss, bss, cores = [], [], [], [], []
    for k, ((w, s), (r, c)) in enumerate(zip(src, shapes)):
        ref, m = compress_both(oracle, ffn, w, s, np.float32(0.75), r, c, 100 + k)
        mats.append(m)
        ps.append(ref["packed"])
        rss.append(ref["row_scales"])
        bss.append(ref["block_scales"])
        cores.append(oracle.Core(ref["core_a"], ref["core_a_sc"], ref["core_b"], ref["core_b_sc"]))
    e = ffn.SwigluExpert(ffn.FMT_TERNARY, mats, I, H)
    oe = oracle.TernaryExpert(I, H, tuple(ps), tuple(rss), tuple(cores), 1.0, tuple(bss))
    x = ffn.gen_normal(ffn.path_key(22, 0, 0, ffn.TAG_X), 3 * H).view(3, H)
    y = host(e.forward(x))
    xs = host(x)
    ref = np.stack([oe.forward(np.ascontiguousarray(xs[t])) for t in range(3)])
    oracle.assert_close(y, ref, what="compressed expert")
