"""CPU tests: the oracle pinned against the golden fixtures (no GPU)."""
import hashlib
import json
import math
import os

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(name):
    return json.load(open(os.path.join(GOLD, name)))


def bench_x(n):
    return np.array([np.float32(math.sin(i * 0.013) * 0.5) for i in range(n)], dtype=np.float32)


def test_e4m3_decode_matches_torch_all_codes(oracle):
    """flash1017.rs:1031-1045 vs an independent decoder (torch.float8_e4m3fn)."""
    ref = np.array(_load("e4m3_torch.json")["bits"], dtype=np.uint32).view(np.float32)
    got = oracle.e4m3_table()
    same = (got.view(np.uint32) == ref.view(np.uint32)) | (np.isnan(got) & np.isnan(ref))
    assert same.all(), np.where(~same)
    assert np.isnan(got[0x7F]) and np.isnan(got[0xFF])
    assert got[0x38] == 1.0 and got[0x3C] == 1.5 and got[0x7E] == 448.0 and got[0x01] == 2.0**-9


def test_e2m1_lut_known_values(oracle):
    """flash1017.rs:17-20."""
    want = [0, .5, 1, 1.5, 2, 3, 4, 6, -0.0, -.5, -1, -1.5, -2, -3, -4, -6]
    got = [oracle.e2m1_to_f32(n) for n in range(16)]
    assert got == want
    assert math.copysign(1, got[8]) == -1  # -0.0 keeps its sign


def test_e4m3_encoder_round_trip_and_rne(oracle):
    tab = oracle.e4m3_table()
    for b in range(256):
        if not np.isnan(tab[b]) and tab[b] != 0:
            assert oracle.f32_to_e4m3(float(tab[b])) == b
    # ties to even between 1.0 (0x38) and 1.125 (0x39): 1.0625 -> 0x38; 1.1875 -> 0x3A
    assert oracle.f32_to_e4m3(1.0625) == 0x38
    assert oracle.f32_to_e4m3(1.1875) == 0x3A
    assert oracle.f32_to_e4m3(1e6) == 0x7E                     # saturates to 448
    assert oracle.f32_to_e4m3(2.0**-10) == 0x00                # half the smallest subnormal -> even
    assert oracle.f32_to_e4m3(3 * 2.0**-10) == 0x02            # 1.5 ulp -> 2 (even)


def test_nvfp4_known_answer_single_group(oracle):
    """1x16 row, scale 0x38 (1.0): y = gs * sum(LUT[n_k] * x_k) by hand."""
    w = np.array([0x10 * ((2 * k + 1) % 16) + (2 * k % 16) for k in range(8)], dtype=np.uint8)
    s = np.array([0x38], dtype=np.uint8)
    x = np.arange(1, 17, dtype=np.float32)
    lut = [0, .5, 1, 1.5, 2, 3, 4, 6, 0, -.5, -1, -1.5, -2, -3, -4, -6]
    want = sum(lut[k] * (k + 1) for k in range(16)) * 0.5
    assert oracle.nvfp4_matvec(w, s, 0.5, x, 1, 16)[0] == np.float32(want)


def test_nvfp4_reference_fixture(oracle):
    """The reference's own NVFP4 test fixture (flash1017.rs:10974-10990) through
    the oracle equals the independent Python restatement bit for bit."""
    ka = _load("known_answers.json")["nvfp4_fixture"]
    rows, cols = ka["rows"], ka["cols"]
    w = np.array([((i * 7 + 3) % 16) | (((i * 13 + 5) % 16) << 4) for i in range(rows * cols // 2)],
                 dtype=np.uint8)
    s = np.array([0x38 if i % 2 == 0 else 0x3C for i in range(rows * cols // 16)], dtype=np.uint8)
    y = oracle.nvfp4_matvec(w, s, ka["gs"], bench_x(cols), rows, cols)
    assert np.array_equal(y, np.array(ka["y"], dtype=np.float32))


def test_nvfp4_all_codes_and_scales(oracle):
    ka = _load("known_answers.json")["nvfp4_scales"]
    w = np.array(ka["w"], dtype=np.uint8)
    s = np.array(ka["s"], dtype=np.uint8)
    y = oracle.nvfp4_matvec(w, s, ka["gs"], bench_x(ka["cols"]), ka["rows"], ka["cols"])
    assert np.array_equal(y, np.array(ka["y"], dtype=np.float32))


def test_nvfp4_threads_do_not_change_results(oracle):
    w, s = oracle.gen_nvfp4(oracle.key(0, 0, 0, 1), 256, 512)
    x = oracle.gen_normal(oracle.key(0, 0, 0, 11), 512)
    oracle.set_threads(1)
    a = oracle.nvfp4_matvec(w, s, 1.0, x, 256, 512)
    oracle.set_threads(7)
    b = oracle.nvfp4_matvec(w, s, 1.0, x, 256, 512)
    oracle.set_threads(1)
    assert np.array_equal(a, b)


def test_ternary_known_answers(oracle):
    """flash1017.rs:2602-2621 (0x55 skip) and :2567-2601 (U8 block scales)."""
    ka = _load("known_answers.json")["ternary"]
    p = np.array(ka["p"], dtype=np.uint8)
    rs = np.array(ka["rs"], dtype=np.float32)
    x = bench_x(ka["cols"])
    y = oracle.ternary_matvec(p, rs, x, ka["rows"], ka["cols"])
    assert np.array_equal(y, np.array(ka["y"], dtype=np.float32))
    bs = np.array(ka["bs"], dtype=np.uint8)
    y2 = oracle.ternary_matvec(p, rs, x, ka["rows"], ka["cols"], bs=bs)
    assert np.array_equal(y2, np.array(ka["y_bs"], dtype=np.float32))


def test_ternary_code3_and_0x55_decode_to_zero(oracle):
    p = np.array([0xFF, 0x55, 0x06, 0x59], dtype=np.uint8)
    d = oracle.dequant_ternary(p, 1, 16)
    assert (d[0, :8] == 0).all()                       # code 3 and code 1 are zero
    assert list(d[0, 8:12]) == [1.0, 0.0, -1.0, -1.0]  # 0x06: codes 2,1,0,0
    assert list(d[0, 12:16]) == [0.0, 1.0, 0.0, 0.0]   # 0x59: codes 1,2,1,1
    x = np.arange(1, 17, dtype=np.float32)
    y = oracle.ternary_matvec(p, np.ones(1, dtype=np.float32), x, 1, 16)
    assert y[0] == np.float32((d[0] * x).sum())


def test_rank16_known_answer(oracle):
    """flash1017.rs:2446-2472 against the Python restatement."""
    ka = _load("known_answers.json")
    t, r = ka["ternary"], ka["rank16"]
    core = oracle.Core(np.array(r["a"], dtype=np.int8), np.array(r["a_sc"], dtype=np.float32),
                       np.array(r["b"], dtype=np.int8), np.array(r["b_sc"], dtype=np.float32))
    y = np.zeros(t["rows"], dtype=np.float32)
    oracle.rank16_apply_add(core, bench_x(t["cols"]), y, t["rows"], t["cols"])
    assert np.array_equal(y, np.array(r["y"], dtype=np.float32))


def test_ternary_with_core_is_matvec_plus_core(oracle):
    rows, cols = 64, 256
    p, rs = oracle.gen_ternary(oracle.key(1, 0, 0, 1), rows, cols)
    core = oracle.gen_core(oracle.key(1, 0, 0, 1), rows, cols)
    x = oracle.gen_normal(oracle.key(1, 0, 0, 11), cols)
    base = oracle.ternary_matvec(p, rs, x, rows, cols)
    oracle.rank16_apply_add(core, x, base, rows, cols)
    assert np.array_equal(base, oracle.ternary_matvec(p, rs, x, rows, cols, core=core))


def test_router_known_answer(oracle):
    """Top-6 selection and weights (flash1017.rs:7280-7376) vs the restatement."""
    ka = _load("known_answers.json")["router"]
    logits = np.array(ka["logits"], dtype=np.float32)[None, :]
    for fn, kidx, kw, tot in ((0, "ref_idx", "ref_w", 1.5), (1, "sig_idx", "sig_w", 1.0)):
        idx, wt, sc, bi = oracle.route(logits, 6, None, fn)
        assert list(idx[0]) == ka[kidx]
        np.testing.assert_allclose(wt[0], ka[kw], rtol=1e-6)
        assert abs(float(wt[0].sum()) - tot) < 1e-5
        assert (np.diff(bi[0]) <= 0).all()


def test_router_bias_changes_selection_not_weights(oracle):
    logits = np.zeros((1, 16), dtype=np.float32)
    logits[0, :] = np.linspace(-1, 1, 16)
    bias = np.zeros(16, dtype=np.float32)
    bias[0] = 10.0  # lowest logit forced into the selection by the noaux bias
    idx, wt, sc, _ = oracle.route(logits, 6, bias, 0)
    assert idx[0, 0] == 0
    assert abs(float(wt[0].sum()) - 1.5) < 1e-6  # weights use unbiased scores
    np.testing.assert_allclose(wt[0], sc[0] * 1.5 / sc[0].sum(), rtol=1e-6)


def test_swiglu_clamps(oracle):
    g = np.array([-50, -1, 0, 1, 12, 50, np.nan], dtype=np.float32)
    u = np.array([-50, -1, 0, 1, 12, 50, 1.0], dtype=np.float32)
    h = oracle.swiglu(g, u)
    assert h[5] == np.float32(100.0)    # silu(50) capped at 10, u clamped to 10
    assert abs(h[0]) < 1e-18            # silu(-50) ~ -1e-20
    assert h[4] == np.float32(100.0)
    assert h[6] == np.float32(10.0)     # min(NaN, 10) = 10 (Rust f32::min)


def test_generator_golden_checksums(oracle):
    def h(a):
        return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()

    g = _load("generator.json")
    w, s = oracle.gen_nvfp4(oracle.key(0, 0, 0, oracle.TAG_W1), 64, 4096)
    assert [h(w), h(s)] == g["nvfp4_64x4096"]
    p, r = oracle.gen_ternary(oracle.key(1, 0, 0, oracle.TAG_W1), 64, 4096)
    assert [h(p), h(r)] == g["ternary_64x4096"]
    c = oracle.gen_core(oracle.key(1, 0, 0, oracle.TAG_W1), 64, 4096)
    assert [h(c.a), h(c.a_sc), h(c.b), h(c.b_sc)] == g["core_64x4096"]
    assert h(oracle.gen_normal(oracle.key(2, 0, 0, oracle.TAG_X), 100000)) == g["normal_100000"]


def test_generator_distributions(oracle):
    w, s = oracle.gen_nvfp4(oracle.key(0, 0, 0, 1), 256, 4096)
    counts = np.bincount(np.concatenate([w & 15, w >> 4]), minlength=16)
    assert counts.min() > 0.9 * counts.mean()
    sc = oracle.e4m3_table()[s]
    assert abs(sc.mean() - math.sqrt(2 / math.pi) / 6) < 0.01
    p, rs = oracle.gen_ternary(oracle.key(1, 0, 0, 1), 256, 4096)
    d = oracle.dequant_ternary(p, 256, 4096)
    for v, pr in ((-1, .3), (0, .4), (1, .3)):
        assert abs((d == v).mean() - pr) < 0.01
    assert rs.min() >= 0.01 and rs.max() < 0.05
    x = oracle.gen_normal(oracle.key(0, 0, 0, 11), 200000)
    assert abs(x.mean()) < 0.01 and abs(x.std() - 1) < 0.01


def test_moe_layer_oracle_small(oracle):
    """Reference-order decode MoE on a tiny layer: combine == sum_k w_k y_k."""
    H, I, E, T = 64, 32, 8, 3
    experts = [oracle.gen_nvfp4_expert(5, 0, e, I, H) for e in range(E)]
    wr = oracle.gen_router(5, 0, E, H)
    x = oracle.gen_hidden(5, T, H)
    out, idx, wt = oracle.moe_layer(experts, wr, x, top_k=2, score_fn=1)
    for t in range(T):
        ref = np.zeros(H, dtype=np.float64)
        for k in range(2):
            ref += float(wt[t, k]) * experts[idx[t, k]].forward(np.ascontiguousarray(x[t]))
        np.testing.assert_allclose(out[t], ref, rtol=1e-5, atol=1e-6)


def test_tolerance_metrics(oracle):
    a = np.array([1.0, -2.0, 4.0])
    assert oracle.max_rel_err(a, a) == 0 and oracle.cosine(a, a) == pytest.approx(1.0)
    b = a + np.array([0, 0, 0.004])
    assert oracle.max_rel_err(b, a) == pytest.approx(1e-3)
    with pytest.raises(AssertionError):
        oracle.assert_close(a + np.array([0, 0, 0.01]), a)


def test_rms_norm_matches_restatement(oracle):
    """flash1017.rs:4880-4891 restated: sequential f32 sum of squares."""
    x = oracle.gen_normal(oracle.key(9, 0, 0, 11), 256) * np.float32(3.0)
    w = np.linspace(0.5, 1.5, 256).astype(np.float32)
    ss = np.float32(0)
    for v in x:
        ss = np.float32(ss + np.float32(v * v))
    inv = np.float32(1.0) / np.float32(np.sqrt(np.float32(ss / np.float32(256) + np.float32(1e-20))))
    want = np.array([np.float32(np.float32(x[i] * inv) * w[i]) for i in range(256)], dtype=np.float32)
    assert np.array_equal(oracle.rms_norm(x[None, :], w)[0], want)


def test_e8m0_decode_pinned(oracle):
    """flash1017.rs:1049-1057 on all 256 codes against the independent restatement."""
    ka = json.load(open(os.path.join(GOLD, "known_answers.json")))["e8m0"]
    got = [int(np.float32(oracle.e8m0_to_f32(b)).view(np.uint32)) for b in range(256)]
    assert got == ka["bits"]


def test_mxfp4_known_answer(oracle):
    """F:2717-2744 restated term by term (tests/golden/make_golden.py)."""
    ka = json.load(open(os.path.join(GOLD, "known_answers.json")))["mxfp4"]
    y = oracle.mxfp4_matvec(np.array(ka["w"], dtype=np.uint8), np.array(ka["s"], dtype=np.uint8),
                            bench_x(ka["cols"]), ka["rows"], ka["cols"])
    assert np.array_equal(y, np.array(ka["y"], dtype=np.float32))


def test_mxfp8_known_answer(oracle):
    """F:1960-1982 (32 x 32 E8M0 blocks) restated term by term."""
    ka = json.load(open(os.path.join(GOLD, "known_answers.json")))["mxfp8"]
    y = oracle.mxfp8_matvec(np.array(ka["w"], dtype=np.uint8), np.array(ka["s"], dtype=np.uint8),
                            bench_x(ka["cols"]), ka["rows"], ka["cols"])
    assert np.array_equal(y, np.array(ka["y"], dtype=np.float32))
