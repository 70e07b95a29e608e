"""The reference's hardware add-on entry points with host pointers, as the Rust
host calls them (hardware_addon.rs:143-174 vtable, :323-373 fused experts).

The fused decode sequence of flash1017.rs:7401-7472: the shared
expert overwrites `out` (accumulate = false), then the routed experts add
weight * expert(x) (accumulate = true), and only the last call asks for the
result (sync_now = true).  The library queues the accumulating calls and runs
them together as one routed layer; the results must equal the one-by-one
arithmetic of the oracle (out += w * y in call order).  The batched layer
(flash1017.rs:8126-8262): the shared expert's gx10_rust_mxfp8_mlp_batch call
hands x_all over, then one *_mlp_batch call per hit expert; expected values
follow the host's CPU twin (flash1017.rs:8266-8324)."""
import ctypes as C
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def bench_x(n, phase=0.0):
    return np.array([np.float32(math.sin(i * 0.013 + phase) * 0.5) for i in range(n)], dtype=np.float32)


def p(a):
    return a.ctypes.data_as(C.c_void_p)


def nv_expert(oracle, seed, I, H, gs=(0.5, 1.0, 0.75)):
    ms = [oracle.gen_nvfp4(oracle.key(seed, 0, k, oracle.TAG_W1), r, c)
          for k, (r, c) in enumerate(((I, H), (I, H), (H, I)))]
    return oracle.Nvfp4Expert(I, H, tuple(w for w, _ in ms), tuple(s for _, s in ms), gs)


def tn_expert(oracle, seed, I, H, proj=1.25):
    ms = [oracle.gen_ternary(oracle.key(seed, 1, k, oracle.TAG_W1), r, c)
          for k, (r, c) in enumerate(((I, H), (I, H), (H, I)))]
    return oracle.TernaryExpert(I, H, tuple(a for a, _ in ms), tuple(b for _, b in ms), None, proj)


def f8_expert(oracle, seed, I, H):
    rng = np.random.default_rng(seed)
    ws, ss = [], []
    for r, c in ((I, H), (I, H), (H, I)):
        w = rng.integers(0, 256, size=r * c, dtype=np.uint8)
        w[(w & 0x7F) == 0x7F] = 0x38
        ws.append(w)
        ss.append(rng.integers(118, 131, size=((r + 31) // 32) * (c // 32), dtype=np.uint8))
    return oracle.MxExpert(4, I, H, tuple(ws), tuple(ss))


def call(L, e, I, H, x, out, w, acc, sync):
    if hasattr(e, "gs"):  # NVFP4
        return L.gx10_rust_nvfp4_mlp_accum(I, H, p(e.w[0]), p(e.s[0]), C.c_float(e.gs[0]), p(e.w[1]),
                                           p(e.s[1]), C.c_float(e.gs[1]), p(e.w[2]), p(e.s[2]),
                                           C.c_float(e.gs[2]), p(x), p(out), C.c_float(w), acc, sync)
    if hasattr(e, "rs"):  # ternary: proj_scale is part of the expert, as in the oracle
        return L.gx10_rust_ternary_158_mlp_accum(I, H, p(e.p[0]), p(e.rs[0]), p(e.p[1]), p(e.rs[1]),
                                                 p(e.p[2]), p(e.rs[2]), C.c_float(e.proj_scale), p(x),
                                                 p(out), C.c_float(w), acc, sync)
    return L.gx10_rust_mxfp8_mlp_accum(I, H, p(e.w[0]), p(e.s[0]), p(e.w[1]), p(e.s[1]), p(e.w[2]),
                                       p(e.s[2]), p(x), p(out), C.c_float(w), acc, sync)


@pytest.fixture(scope="module")
def L(ffn):
    return ffn.lib()


def reference(oracle, seq, x, out0=0.0):
    """(experts, weights, accumulate) in call order -> out, one by one, from `out0`."""
    out = np.full(len(x), out0, dtype=np.float32)
    for e, w, acc in seq:
        y = e.forward(x)
        out = (out + np.float32(w) * y).astype(np.float32) if acc else (np.float32(w) * y)
    return out


def test_fused_decode_sequence(oracle, ffn, cuda, L):
    """Shared MXFP8 expert, then six routed NVFP4 / ternary experts, sync on the last."""
    H, I = 1024, 512
    shared = f8_expert(oracle, 1, I, H)
    routed = [nv_expert(oracle, 10 + k, I, H) if k % 2 == 0 else tn_expert(oracle, 10 + k, I, H) for k in range(6)]
    wts = [0.31, 0.22, 0.17, 0.13, 0.1, 0.07]
    x = bench_x(H)
    out = np.zeros(H, dtype=np.float32)
    assert call(L, shared, I, H, x, out, 1.0, False, False)
    for k, (e, w) in enumerate(zip(routed, wts)):
        assert call(L, e, I, H, x, out, w, True, k == 5)
    ref = reference(oracle, [(shared, 1.0, False)] + [(e, w, True) for e, w in zip(routed, wts)], x)
    oracle.assert_close(out, ref, rel=1e-4, what="fused decode sequence")


def test_queue_longer_than_a_batch(oracle, ffn, cuda, L):
    """20 accumulating calls (more than one queued batch) onto one output, sync
    on the last; then a second output."""
    H, I = 512, 256
    es = [nv_expert(oracle, 40 + k, I, H) for k in range(5)]
    x1, x2 = bench_x(H), bench_x(H, 1.0)
    o1 = np.full(H, 0.5, dtype=np.float32)
    o2 = np.zeros(H, dtype=np.float32)
    seq = []
    for k in range(20):
        e, w = es[k % 5], 0.05 * (k + 1)
        assert call(L, e, I, H, x1, o1, w, True, k == 19)
        seq.append((e, w, True))
    assert call(L, es[0], I, H, x2, o2, 2.0, False, True)
    r1 = reference(oracle, seq, x1, 0.5)
    oracle.assert_close(o1, r1, rel=1e-4, what="20 queued calls")
    oracle.assert_close(o2, 2.0 * es[0].forward(x2), rel=1e-4, what="second target")


def test_abandoned_sequence_is_never_written_back(oracle, ffn, cuda, L):
    """The host breaks out of a fused sequence before its sync_now call and
    frees `out` (flash1017.rs:7483-7486): no later call may write to that
    buffer.  The abandoned buffer keeps a sentinel here, through a call to
    another target, a call of another entry point, and a new batched layer."""
    H, I = 512, 256
    es = [nv_expert(oracle, 70 + k, I, H) for k in range(3)]
    x = bench_x(H)
    sentinel = np.float32(-7.25)
    gone = np.full(H, sentinel, dtype=np.float32)  # stands for the freed buffer
    assert call(L, es[0], I, H, x, gone, 1.0, False, False)
    assert call(L, es[1], I, H, x, gone, 0.5, True, False)  # ... and the host breaks out here
    fresh = np.zeros(H, dtype=np.float32)
    assert call(L, es[2], I, H, x, fresh, 1.0, False, True)
    assert np.all(gone == sentinel), "an abandoned sequence was written to its old target"
    oracle.assert_close(fresh, es[2].forward(x), rel=1e-4, what="the next sequence")
    # an abandoned sequence followed by another entry point (V3 matvec slot)
    assert call(L, es[0], I, H, x, gone, 1.0, False, False)
    fn = C.CFUNCTYPE(None, C.c_size_t, C.c_size_t, C.c_void_p, C.c_void_p, C.c_float, C.c_void_p, C.c_void_p)
    slot = C.c_void_p.from_address(L.merkaba_hardware_addon_v1() + 120).value  # matvec_nvfp4 (HA:143-174)
    y = np.zeros(I, dtype=np.float32)
    m = es[0]
    fn(slot)(I, H, p(m.w[0]), p(m.s[0]), m.gs[0], p(x), p(y))
    oracle.assert_close(y, oracle.nvfp4_matvec(m.w[0], m.s[0], m.gs[0], x, I, H), what="vtable matvec_nvfp4")
    assert np.all(gone == sentinel), "an abandoned sequence was written back by another entry point"
    # an abandoned batched layer, then the next layer's shared-expert call
    shared = f8_expert(oracle, 5, I, H)
    x_all = np.ascontiguousarray(np.stack([bench_x(H, 0.1 * t) for t in range(2)]), dtype=np.float32)
    old = np.full((2, H), sentinel, dtype=np.float32)
    assert L.gx10_rust_mxfp8_mlp_batch(I, H, 2, p(shared.w[0]), p(shared.s[0]), p(shared.w[1]),
                                       p(shared.s[1]), p(shared.w[2]), p(shared.s[2]), p(x_all), 2,
                                       p(old), False)
    dst = np.array([0, 1], dtype=np.uint64)
    wts = np.array([0.3, 0.2], dtype=np.float32)
    e = es[1]
    assert L.gx10_rust_nvfp4_mlp_batch(I, H, 2, p(e.w[0]), p(e.s[0]), e.gs[0], p(e.w[1]), p(e.s[1]),
                                       e.gs[1], p(e.w[2]), p(e.s[2]), e.gs[2], 0, p(dst), p(wts), 2,
                                       p(old), False)
    new = np.zeros((2, H), dtype=np.float32)
    assert L.gx10_rust_mxfp8_mlp_batch(I, H, 2, p(shared.w[0]), p(shared.s[0]), p(shared.w[1]),
                                       p(shared.s[1]), p(shared.w[2]), p(shared.s[2]), p(x_all), 2,
                                       p(new), True)
    assert np.all(old == sentinel), "an abandoned batched layer was written back"
    ref = np.stack([shared.forward(x_all[t]) for t in range(2)])
    oracle.assert_close(new, ref, rel=1e-4, what="the next batched layer")


def test_hbm_budget_evicts_and_copies_again(oracle, ffn, cuda, L):
    """A model larger than the HBM the weight copies may use (the reference's
    404 GB checkpoint on a 180 GB GPU): with a budget of three experts'
    weights, calls cycling through eight experts evict the least recently used
    copies and copy them again.  Every call succeeds (a false return would send
    the host to its CPU path), results equal the oracle, the copies stay within
    the budget, and a queued sequence of five experts, whose first copies are
    evicted while they are still queued, is still right."""
    H, I = 512, 256
    es = [nv_expert(oracle, 200 + k, I, H) for k in range(8)]
    ebytes = 3 * (I * H // 2 + I * H // 16)
    L.ffn_b200_release_host_ranges()
    L.ffn_b200_set_host_cache_budget(3 * ebytes)
    try:
        x = bench_x(H)
        for _ in range(2):
            for k, e in enumerate(es):
                out = np.zeros(H, dtype=np.float32)
                assert call(L, e, I, H, x, out, 1.0, False, True)
                oracle.assert_close(out, e.forward(x), rel=1e-4, what=f"expert {k} under the budget")
                assert L.ffn_b200_host_cache_bytes() <= 3 * ebytes
        out = np.zeros(H, dtype=np.float32)
        seq = []
        for k, e in enumerate(es[3:8]):
            assert call(L, e, I, H, x, out, 0.2 + 0.1 * k, k > 0, k == 4)
            seq.append((e, 0.2 + 0.1 * k, k > 0))
        oracle.assert_close(out, reference(oracle, seq, x), rel=1e-4, what="queued sequence under the budget")
    finally:
        L.ffn_b200_set_host_cache_budget(0)
        L.ffn_b200_release_host_ranges()


def test_calls_with_different_inputs(oracle, ffn, cuda, L):
    """Each queued call keeps its own x (the host may reuse its buffer)."""
    H, I = 512, 256
    es = [tn_expert(oracle, 60 + k, I, H) for k in range(3)]
    xbuf = np.zeros(H, dtype=np.float32)
    out = np.zeros(H, dtype=np.float32)
    ref = np.zeros(H, dtype=np.float32)
    for k, e in enumerate(es):
        xbuf[:] = bench_x(H, 0.3 * k)
        assert call(L, e, I, H, xbuf, out, 0.5, True, k == 2)
        ref = (ref + np.float32(0.5) * e.forward(bench_x(H, 0.3 * k))).astype(np.float32)
    oracle.assert_close(out, ref, rel=1e-4, what="per-call inputs")


# --------------------------------------------- batched layer (*_mlp_batch)
def host_batched_layer(oracle, L, shared, experts, sel, x_tok, I, H):
    """The reference host's batched fused layer (flash1017.rs:8088-8099,
    8126-8262): expert_hits in order of first appearance, x_all = the b_len
    token rows + one extra row per hit of every multi-hit expert, the shared
    MXFP8 expert over x_all, then one *_mlp_batch call per hit expert, sync on
    the last.  Returns (GPU out_batch, expected out_batch by the CPU twin's
    arithmetic, flash1017.rs:8266-8324)."""
    b_len = x_tok.shape[0]
    hits = []  # (expert id, [(token, weight)])
    for t, picks in enumerate(sel):
        for e, w in picks:
            for h in hits:
                if h[0] == e:
                    h[1].append((t, w))
                    break
            else:
                hits.append((e, [(t, w)]))
    rows = [x_tok[t] for t in range(b_len)]
    offs = []
    for e, hs in hits:
        if len(hs) == 1:
            offs.append(hs[0][0])
        else:
            offs.append(len(rows))
            rows += [x_tok[t] for t, _ in hs]
    x_all = np.ascontiguousarray(np.stack(rows), dtype=np.float32)
    out = np.zeros((b_len, H), dtype=np.float32)
    keep = [x_all]
    ok = L.gx10_rust_mxfp8_mlp_batch(I, H, b_len, p(shared.w[0]), p(shared.s[0]), p(shared.w[1]),
                                     p(shared.s[1]), p(shared.w[2]), p(shared.s[2]), p(x_all),
                                     x_all.shape[0], p(out), len(hits) == 0)
    assert ok
    for i, (e, hs) in enumerate(hits):
        ex = experts[e]
        dst = np.array([t for t, _ in hs], dtype=np.uint64)
        wts = np.array([w for _, w in hs], dtype=np.float32)
        keep += [dst, wts]
        last = i + 1 == len(hits)
        if hasattr(ex, "gs"):
            ok = L.gx10_rust_nvfp4_mlp_batch(I, H, len(hs), p(ex.w[0]), p(ex.s[0]), ex.gs[0], p(ex.w[1]),
                                             p(ex.s[1]), ex.gs[1], p(ex.w[2]), p(ex.s[2]), ex.gs[2],
                                             offs[i], p(dst), p(wts), b_len, p(out), last)
        else:
            ok = L.gx10_rust_ternary_158_mlp_batch(I, H, len(hs), p(ex.p[0]), p(ex.rs[0]), p(ex.p[1]),
                                                   p(ex.rs[1]), p(ex.p[2]), p(ex.rs[2]), ex.proj_scale,
                                                   offs[i], p(dst), p(wts), b_len, p(out), last)
        assert ok
    # expected: the CPU twin (shared matbatch, then per hit expert, per hit, axpy)
    ref = np.stack([shared.forward(x_all[t]) for t in range(b_len)])
    for i, (e, hs) in enumerate(hits):
        ex = experts[e]
        sc = np.float32(getattr(ex, "proj_scale", 1.0)) if not hasattr(ex, "gs") else None
        for k, (t, w) in enumerate(hs):
            y = ex.forward(np.ascontiguousarray(x_all[offs[i] + k]))
            ww = np.float32(w) if sc is None else np.float32(w) * sc
            ref[t] = (ref[t] + ww * y).astype(np.float32)
    return out, ref


def routed_pool(oracle, I, H, n, seed):
    return [nv_expert(oracle, seed + k, I, H) if k % 3 else tn_expert(oracle, seed + k, I, H, 1.25)
            for k in range(n)]


def test_batched_layer_sequence(oracle, ffn, cuda, L):
    """Four tokens, top-6 over 12 experts (NVFP4 and ternary with proj_scale
    1.25): the shared expert, then the hit experts with 1..4 tokens each."""
    H, I = 1024, 512
    shared = f8_expert(oracle, 2, I, H)
    experts = routed_pool(oracle, I, H, 12, 100)
    rng = np.random.default_rng(5)
    sel = [[(int(e), float(w)) for e, w in zip(rng.choice(12, 6, replace=False), rng.uniform(0.05, 0.4, 6))]
           for _ in range(4)]
    x_tok = np.stack([bench_x(H, 0.7 * t) for t in range(4)])
    out, ref = host_batched_layer(oracle, L, shared, experts, sel, x_tok, I, H)
    oracle.assert_close(out, ref, rel=1e-4, what="batched layer")


def test_batched_layer_more_calls_than_a_queue(oracle, ffn, cuda, L):
    """Sixteen tokens, top-6 over 192 experts: about 75 hit experts, more than
    one queue (64 calls) holds, and a second layer right after."""
    H, I = 512, 256
    shared = f8_expert(oracle, 3, I, H)
    experts = routed_pool(oracle, I, H, 192, 300)
    rng = np.random.default_rng(6)
    for layer in range(2):
        sel = [[(int(e), float(w)) for e, w in zip(rng.choice(192, 6, replace=False), rng.uniform(0.05, 0.4, 6))]
               for _ in range(16)]
        x_tok = np.stack([bench_x(H, 0.3 * t + layer) for t in range(16)])
        out, ref = host_batched_layer(oracle, L, shared, experts, sel, x_tok, I, H)
        oracle.assert_close(out, ref, rel=1e-4, what=f"batched layer {layer}")


def test_batched_layer_without_routed_experts(oracle, ffn, cuda, L):
    H, I = 512, 256
    shared = f8_expert(oracle, 4, I, H)
    x_tok = np.stack([bench_x(H, 0.5 * t) for t in range(3)])
    out, ref = host_batched_layer(oracle, L, shared, [], [[], [], []], x_tok, I, H)
    oracle.assert_close(out, ref, rel=1e-4, what="shared expert only")


def test_q4_backbone_flag_is_refused(oracle, ffn, cuda, L):
    """seq_len with bit 31 (the NVFP4 q4-backbone shared expert) returns false,
    so the host takes its CPU twin."""
    H, I = 512, 256
    shared = f8_expert(oracle, 5, I, H)
    x = np.stack([bench_x(H)] * 2)
    out = np.zeros((2, H), dtype=np.float32)
    assert not L.gx10_rust_mxfp8_mlp_batch(I, H, 2 | (1 << 31), p(shared.w[0]), p(shared.s[0]),
                                           p(shared.w[1]), p(shared.s[1]), p(shared.w[2]),
                                           p(shared.s[2]), p(x), 2, p(out), True)


def test_mxfp4_wide_scale_range_through_the_abi(oracle, ffn, cuda, L):
    """MXFP4 block scales over 2^-37 .. 2^13 through gx10_rust_mxfp4_matvec and
    gx10_rust_mxfp4_mlp_accum: the library derives the f16 decode's power-of-two
    bias from the largest scale, as the device-resident Mxfp4Matrix does."""
    H, I = 1024, 512
    rng = np.random.default_rng(9)
    ws = []
    for r, c in ((I, H), (I, H), (H, I)):
        ws.append((rng.integers(0, 256, size=r * c // 2, dtype=np.uint8),
                   rng.integers(90, 141, size=r * c // 32, dtype=np.uint8)))
    x = bench_x(H)
    y = np.zeros(I, dtype=np.float32)
    assert L.gx10_rust_mxfp4_matvec(I, H, p(ws[0][0]), p(ws[0][1]), p(x), p(y))
    oracle.assert_close(y, oracle.mxfp4_matvec(ws[0][0], ws[0][1], x, I, H), what="mxfp4 matvec, wide scales")
    oe = oracle.MxExpert(3, I, H, tuple(a for a, _ in ws), tuple(b for _, b in ws))
    out = np.zeros(H, dtype=np.float32)
    assert L.gx10_rust_mxfp4_mlp_accum(I, H, p(ws[0][0]), p(ws[0][1]), p(ws[1][0]), p(ws[1][1]),
                                       p(ws[2][0]), p(ws[2][1]), p(x), p(out), 0.5, False, True)
    oracle.assert_close(out, 0.5 * oe.forward(x), what="mxfp4 expert, wide scales")


def test_bad_shape_fails_at_the_call_and_leaves_a_clean_state(oracle, ffn, cuda, L):
    """Shapes the kernels cannot run (NVFP4 hidden % 64, MXFP4 hidden % 128) make
    that call return false (the host then runs its CPU twin), with the weight
    arrays sized for the claimed dims.  A pending sequence to another target is
    abandoned (never written back: the host recomputes it on its CPU path),
    and the next sequence is unaffected."""
    H, I = 512, 256
    es = [nv_expert(oracle, 70 + k, I, H) for k in range(2)]
    x = bench_x(H)
    out = np.zeros(H, dtype=np.float32)
    assert call(L, es[0], I, H, x, out, 0.5, True, False)  # queued
    bH = 96
    w = np.zeros(I * bH // 2, dtype=np.uint8)
    s = np.full(I * bH // 16, 0x38, dtype=np.uint8)
    bad = oracle.Nvfp4Expert(I, bH, (w, w, w), (s, s, s), (1.0, 1.0, 1.0))
    xb, ob = bench_x(bH), np.zeros(bH, dtype=np.float32)
    assert not call(L, bad, I, bH, xb, ob, 0.5, True, True)
    assert np.all(out == 0), "the abandoned sequence was written back"
    mH = 320
    mw = np.zeros(I * mH // 2, dtype=np.uint8)
    ms = np.full(I * mH // 32, 127, dtype=np.uint8)
    mo = np.zeros(mH, dtype=np.float32)
    xm = bench_x(mH)
    assert not L.gx10_rust_mxfp4_mlp_accum(I, mH, p(mw), p(ms), p(mw), p(ms), p(mw), p(ms), p(xm), p(mo),
                                           1.0, False, True)
    out2 = np.zeros(H, dtype=np.float32)
    assert call(L, es[0], I, H, x, out2, 1.0, False, False)
    assert call(L, es[1], I, H, x, out2, 0.25, True, True)
    ref = reference(oracle, [(es[0], 1.0, False), (es[1], 0.25, True)], x)
    oracle.assert_close(out2, ref, rel=1e-4, what="sequence after the failures")
