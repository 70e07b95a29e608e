"""MXFP4 experts on the GPU (FFN_B200_FMT_MXFP4: the reference's MTP routed
experts, CachedMxfp4Mat, flash1017.rs:2674-2747, E8M0 decode :1049-1057)
against the oracle: matvecs, the term-by-term golden fixture, experts, a MoE
layer, the reference-ABI entry points (gx10_rust_mxfp4_*) and the shard
loader.  Tolerance: max|y - ref| / max|ref| <= 1e-3 and cosine >= 0.99999."""
import ctypes as C
import json
import math
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def host(t):
    return t.detach().cpu().numpy()


def dev(a, cuda):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def bench_x(n):
    return np.array([np.float32(math.sin(i * 0.013) * 0.5) for i in range(n)], dtype=np.float32)


def mx_weights(rows, cols, seed, lo=110, hi=131):
    """E2M1 pairs (every code) and E8M0 scales uniform in [lo, hi)."""
    rng = np.random.default_rng(seed)
    w = rng.integers(0, 256, size=rows * cols // 2, dtype=np.uint8)
    s = rng.integers(lo, hi, size=rows * cols // 32, dtype=np.uint8)
    return w, s


def mx_matrix(ffn, w, s, rows, cols, cuda):
    dw, ds = dev(w, cuda), dev(s, cuda)
    return ffn.Mxfp4Matrix(dw, ds, ffn.Mxfp4Matrix.bias_for(ds), rows, cols)


def mx_expert(ffn, oracle, seed, inter, hidden, cuda, lo=110, hi=131):
    shapes = ((inter, hidden), (inter, hidden), (hidden, inter))
    ws = [mx_weights(r, c, seed + k, lo, hi) for k, (r, c) in enumerate(shapes)]
    mats = [mx_matrix(ffn, w, s, r, c, cuda) for (w, s), (r, c) in zip(ws, shapes)]
    e = ffn.SwigluExpert(ffn.FMT_MXFP4, mats, inter, hidden)
    oe = oracle.MxExpert(3, inter, hidden, tuple(w for w, _ in ws), tuple(s for _, s in ws))
    return e, oe


@pytest.mark.parametrize("rows,cols", [(32, 256), (2048, 4096), (4096, 2048), (96, 384)])
@pytest.mark.parametrize("seq", [1, 4, 8, 13])
def test_mxfp4_matvec(oracle, ffn, cuda, rows, cols, seq):
    w, s = mx_weights(rows, cols, rows * 7 + cols)
    m = mx_matrix(ffn, w, s, rows, cols, cuda)
    x = ffn.gen_normal(ffn.path_key(70, seq, cols, ffn.TAG_X), seq * cols).view(seq, cols)
    y = host(m.matvec(x))
    xs = host(x)
    ref = np.stack([oracle.mxfp4_matvec(w, s, xs[t], rows, cols) for t in range(seq)])
    oracle.assert_close(y, ref, what=f"mxfp4 {rows}x{cols} seq {seq}")


def test_mxfp4_needs_whole_scale_rows(ffn, cuda):
    """cols % 128: rows of E8M0 scales copy in whole 4-byte pieces; checked on
    the host before any launch."""
    w, s = mx_weights(96, 320, 3)
    m = mx_matrix(ffn, w, s, 96, 320, cuda)
    x = ffn.gen_normal(ffn.path_key(70, 1, 320, ffn.TAG_X), 320).view(1, 320)
    with pytest.raises(ffn.FfnError):
        m.matvec(x)


def test_mxfp4_wide_scale_range(oracle, ffn, cuda):
    """Block scales over 2^-37 .. 2^13: the blocks within 36 octaves of the
    largest decode exactly; the rest sit far below the tolerance."""
    rows, cols = 256, 2048
    w, s = mx_weights(rows, cols, 5, lo=90, hi=141)
    m = mx_matrix(ffn, w, s, rows, cols, cuda)
    assert m.gs == 2.0 ** (int(s.max()) - 140)
    x = ffn.gen_normal(ffn.path_key(71, 1, cols, ffn.TAG_X), 2 * cols).view(2, cols)
    y = host(m.matvec(x))
    xs = host(x)
    ref = np.stack([oracle.mxfp4_matvec(w, s, xs[t], rows, cols) for t in range(2)])
    oracle.assert_close(y, ref, what="mxfp4 wide scale range")


def test_mxfp4_known_answer_fixture(oracle, ffn, cuda):
    f = json.load(open(os.path.join(GOLD, "known_answers.json")))["mxfp4"]
    w, s = np.array(f["w"], dtype=np.uint8), np.array(f["s"], dtype=np.uint8)
    m = mx_matrix(ffn, w, s, f["rows"], f["cols"], cuda)
    y = host(m.matvec(dev(bench_x(f["cols"]), cuda)))[0]
    oracle.assert_close(y, np.array(f["y"], dtype=np.float32), what="mxfp4 fixture")


@pytest.mark.parametrize("seq", [1, 3, 8])
def test_mxfp4_expert(oracle, ffn, cuda, seq):
    H, I = 4096, 2048
    e, oe = mx_expert(ffn, oracle, 80, I, H, cuda)
    x = ffn.gen_normal(ffn.path_key(72, 0, 0, ffn.TAG_X), seq * H).view(seq, H)
    y = host(e.forward(x))
    xs = host(x)
    ref = np.stack([oe.forward(np.ascontiguousarray(xs[t])) for t in range(seq)])
    oracle.assert_close(y, ref, what=f"mxfp4 expert seq {seq}")


def test_mxfp4_moe_layer(oracle, ffn, cuda):
    """An MTP-like layer: MXFP4 experts, top-3 (flash1017.rs:9015-9110 routes
    3 of 128), plus NVFP4 experts in the same layer."""
    import torch
    E, H, I, T, K = 12, 512, 256, 19, 3
    experts, oes = [], []
    for e in range(E):
        if e % 4 == 3:
            ex = ffn.SwigluExpert.generate(ffn.FMT_NVFP4, 81, 0, e, I, H)
            experts.append(ex)
            oes.append(oracle.Nvfp4Expert(I, H, tuple(host(m.w) for m in ex.mats),
                                          tuple(host(m.s) for m in ex.mats),
                                          tuple(m.gs for m in ex.mats)))
        else:
            ex, oe = mx_expert(ffn, oracle, 900 + 3 * e, I, H, cuda)
            experts.append(ex)
            oes.append(oe)
    wr = ffn.gen_normal(ffn.path_key(82, 0, 0, ffn.TAG_ROUTER), E * H, 0.02).view(E, H)
    x = ffn.gen_normal(ffn.path_key(82, 0, 0, ffn.TAG_X), T * H).view(T, H)
    layer = ffn.MoeLayer(experts, wr, H, I, top_k=K, score_fn=0)
    assert layer.desc.has_mxfp4 == 1 and layer.desc.has_nvfp4 == 1
    out = host(layer.forward(x))
    ref, _, _ = oracle.moe_layer(oes, host(wr), host(x), top_k=K, score_fn=0)
    oracle.assert_close(out, ref, what="MoE layer with MXFP4 experts")
    # the grouped (NVFP4-only) path refuses MXFP4 experts
    g = ffn.MoeLayer(experts, wr, H, I, top_k=K, score_fn=0, path=ffn.PATH_GROUPED)
    with pytest.raises(ffn.FfnError):
        g.forward(x)
    torch.cuda.synchronize()


def test_mxfp4_reference_abi(oracle, ffn, cuda):
    """gx10_rust_mxfp4_matvec / gx10_rust_mxfp4_mlp_accum with host pointers."""
    L = ffn.lib()
    H, I = 1024, 512
    rows, cols = I, H
    w, s = mx_weights(rows, cols, 11)
    x = bench_x(cols)
    out = np.zeros(rows, dtype=np.float32)
    p = lambda a: a.ctypes.data_as(C.c_void_p)  # noqa: E731
    assert L.gx10_rust_mxfp4_matvec(rows, cols, p(w), p(s), p(x), p(out))
    oracle.assert_close(out, oracle.mxfp4_matvec(w, s, x, rows, cols), what="gx10_rust_mxfp4_matvec")
    shapes = ((I, H), (I, H), (H, I))
    ws = [mx_weights(r, c, 20 + k) for k, (r, c) in enumerate(shapes)]
    oe = oracle.MxExpert(3, I, H, tuple(a for a, _ in ws), tuple(b for _, b in ws))
    y = np.full(H, 0.25, dtype=np.float32)
    ok = L.gx10_rust_mxfp4_mlp_accum(I, H, p(ws[0][0]), p(ws[0][1]), p(ws[1][0]), p(ws[1][1]),
                                     p(ws[2][0]), p(ws[2][1]), p(x), p(y), 0.5, True, True)
    assert ok
    oracle.assert_close(y, 0.25 + 0.5 * oe.forward(x), what="gx10_rust_mxfp4_mlp_accum")


def test_mxfp4_shard_loader(oracle, ffn, cuda, tmp_path):
    """MTP experts as CachedMxfp4Mat::from_shard reads them: <p>.weight + <p>.scale."""
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from test_safetensors import write_shard
    H, I = 1024, 512
    tensors, ws = [], []
    for k, (m, r, c) in enumerate((("w1", I, H), ("w3", I, H), ("w2", H, I))):
        w, s = mx_weights(r, c, 40 + k)
        tensors += [(f"mtp.0.ffn.experts.7.{m}.weight", "U8", (r, c // 2), w.tobytes()),
                    (f"mtp.0.ffn.experts.7.{m}.scale", "F8_E8M0", (r, c // 32), s.tobytes())]
        ws.append((w, s))
    path = tmp_path / "mtp.safetensors"
    write_shard(path, tensors)
    st = ffn.SafetensorsShard(path)
    assert st.expert_bytes("mtp.0.ffn.experts.7", H, I)[0] == ffn.FMT_MXFP4
    ex = st.load_expert("mtp.0.ffn.experts.7", H, I)
    x = ffn.gen_normal(ffn.path_key(73, 0, 0, ffn.TAG_X), 2 * H).view(2, H)
    y = host(ex.forward(x))
    oe = oracle.MxExpert(3, I, H, tuple(a for a, _ in ws), tuple(b for _, b in ws))
    xs = host(x)
    ref = np.stack([oe.forward(np.ascontiguousarray(xs[t])) for t in range(2)])
    oracle.assert_close(y, ref, what="loaded MXFP4 expert")


# ------------------------------------------------------------------ MXFP8
def f8_weights(rows, cols, seed, lo=118, hi=131):
    """E4M3 codes (NaN codes 0x7F / 0xFF replaced) and E8M0 32 x 32 block scales."""
    rng = np.random.default_rng(seed)
    w = rng.integers(0, 256, size=rows * cols, dtype=np.uint8)
    w[(w & 0x7F) == 0x7F] = 0x38
    s = rng.integers(lo, hi, size=((rows + 31) // 32) * ((cols + 31) // 32), dtype=np.uint8)
    return w, s


def f8_matrix(ffn, w, s, rows, cols, cuda):
    dw, ds = dev(w, cuda), dev(s, cuda)
    return ffn.Mxfp8Matrix(dw, ds, ffn.Mxfp8Matrix.bias_for(ds), rows, cols)


@pytest.mark.parametrize("rows,cols", [(32, 128), (2048, 4096), (4096, 2048), (100, 384)])
@pytest.mark.parametrize("seq", [1, 4, 8, 11])
def test_mxfp8_matvec(oracle, ffn, cuda, rows, cols, seq):
    w, s = f8_weights(rows, cols, rows * 3 + cols)
    m = f8_matrix(ffn, w, s, rows, cols, cuda)
    x = ffn.gen_normal(ffn.path_key(74, seq, cols, ffn.TAG_X), seq * cols).view(seq, cols)
    y = host(m.matvec(x))
    xs = host(x)
    ref = np.stack([oracle.mxfp8_matvec(w, s, xs[t], rows, cols) for t in range(seq)])
    oracle.assert_close(y, ref, what=f"mxfp8 {rows}x{cols} seq {seq}")


def test_mxfp8_needs_whole_scale_rows(ffn, cuda):
    w, s = f8_weights(64, 320, 2)
    m = f8_matrix(ffn, w, s, 64, 320, cuda)
    x = ffn.gen_normal(ffn.path_key(74, 1, 320, ffn.TAG_X), 320).view(1, 320)
    with pytest.raises(ffn.FfnError):
        m.matvec(x)


def test_mxfp8_known_answer_fixture(oracle, ffn, cuda):
    """The term-by-term golden vector has cols 96: run it zero-padded to 128
    columns (zero weights, one more scale column) -- the same sums."""
    f = json.load(open(os.path.join(GOLD, "known_answers.json")))["mxfp8"]
    rows, cols = f["rows"], f["cols"]
    w = np.array(f["w"], dtype=np.uint8).reshape(rows, cols)
    s = np.array(f["s"], dtype=np.uint8).reshape((rows + 31) // 32, (cols + 31) // 32)
    wp = np.zeros((rows, 128), dtype=np.uint8)
    wp[:, :cols] = w
    sp = np.full((s.shape[0], 4), 127, dtype=np.uint8)
    sp[:, :s.shape[1]] = s
    m = f8_matrix(ffn, wp.ravel(), sp.ravel(), rows, 128, cuda)
    x = np.zeros(128, dtype=np.float32)
    x[:cols] = bench_x(cols)
    y = host(m.matvec(dev(x, cuda)))[0]
    oracle.assert_close(y, np.array(f["y"], dtype=np.float32), what="mxfp8 fixture")


@pytest.mark.parametrize("seq", [1, 5])
def test_mxfp8_shared_expert(oracle, ffn, cuda, seq):
    """The shared expert at the reference checkpoint's dims (H 5120, I 2304)."""
    H, I = 5120, 2304
    shapes = ((I, H), (I, H), (H, I))
    ws = [f8_weights(r, c, 50 + k) for k, (r, c) in enumerate(shapes)]
    mats = [f8_matrix(ffn, w, s, r, c, cuda) for (w, s), (r, c) in zip(ws, shapes)]
    e = ffn.SwigluExpert(ffn.FMT_MXFP8, mats, I, H)
    oe = oracle.MxExpert(4, I, H, tuple(a for a, _ in ws), tuple(b for _, b in ws))
    x = ffn.gen_normal(ffn.path_key(75, 0, 0, ffn.TAG_X), seq * H).view(seq, H)
    y = host(e.forward(x))
    xs = host(x)
    ref = np.stack([oe.forward(np.ascontiguousarray(xs[t])) for t in range(seq)])
    oracle.assert_close(y, ref, what=f"mxfp8 shared expert seq {seq}")
    with pytest.raises(ffn.FfnError):  # not a routed-expert format
        ffn.MoeLayer([e], ffn.gen_normal(1, H, 0.02).view(1, H), H, I, top_k=1)


def test_mxfp8_reference_abi(oracle, ffn, cuda):
    """gx10_rust_mxfp8_mlp_accum and the V3 vtable's matvec_mxfp8 slot."""
    L = ffn.lib()
    H, I = 1024, 512
    p = lambda a: a.ctypes.data_as(C.c_void_p)  # noqa: E731
    shapes = ((I, H), (I, H), (H, I))
    ws = [f8_weights(r, c, 60 + k) for k, (r, c) in enumerate(shapes)]
    oe = oracle.MxExpert(4, I, H, tuple(a for a, _ in ws), tuple(b for _, b in ws))
    x = bench_x(H)
    y = np.zeros(H, dtype=np.float32)
    assert L.gx10_rust_mxfp8_mlp_accum(I, H, p(ws[0][0]), p(ws[0][1]), p(ws[1][0]), p(ws[1][1]),
                                       p(ws[2][0]), p(ws[2][1]), p(x), p(y), 1.0, False, True)
    oracle.assert_close(y, oe.forward(x), what="gx10_rust_mxfp8_mlp_accum")
    fn = C.CFUNCTYPE(None, C.c_size_t, C.c_size_t, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p)
    vt = L.merkaba_hardware_addon_v1()
    slot = C.c_void_p.from_address(vt + 152).value  # matvec_mxfp8 (HA:143-174 layout)
    out = np.zeros(I, dtype=np.float32)
    fn(slot)(I, H, p(ws[0][0]), p(ws[0][1]), p(x), p(out))
    oracle.assert_close(out, oracle.mxfp8_matvec(ws[0][0], ws[0][1], x, I, H), what="vtable matvec_mxfp8")


def test_mxfp8_shard_loader(oracle, ffn, cuda, tmp_path):
    """Shared experts as CachedMxfp8Mat::from_shard reads them (.weight E4M3 + .scale)."""
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from test_safetensors import write_shard
    H, I = 1024, 512
    tensors, ws = [], []
    for k, (m, r, c) in enumerate((("w1", I, H), ("w3", I, H), ("w2", H, I))):
        w, s = f8_weights(r, c, 70 + k)
        tensors += [(f"layers.2.ffn.shared_experts.{m}.weight", "F8_E4M3", (r, c), w.tobytes()),
                    (f"layers.2.ffn.shared_experts.{m}.scale", "F8_E8M0",
                     ((r + 31) // 32, (c + 31) // 32), s.tobytes())]
        ws.append((w, s))
    path = tmp_path / "shared.safetensors"
    write_shard(path, tensors)
    st = ffn.SafetensorsShard(path)
    assert st.expert_bytes("layers.2.ffn.shared_experts", H, I)[0] == ffn.FMT_MXFP8
    ex = st.load_expert("layers.2.ffn.shared_experts", H, I)
    x = ffn.gen_normal(ffn.path_key(76, 0, 0, ffn.TAG_X), 2 * H).view(2, H)
    y = host(ex.forward(x))
    oe = oracle.MxExpert(4, I, H, tuple(a for a, _ in ws), tuple(b for _, b in ws))
    xs = host(x)
    ref = np.stack([oe.forward(np.ascontiguousarray(xs[t])) for t in range(2)])
    oracle.assert_close(y, ref, what="loaded MXFP8 shared expert")
