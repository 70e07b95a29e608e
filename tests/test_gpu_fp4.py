"""The MoE layer's block-scaled FP4 tensor-core path (FFN_B200_PATH_FP4,
tcgen05 kind::mxf4nvf4) against the CPU oracle, through the C-ABI.

The weights enter the tensor core unchanged, from the stage images
ffn_b200_pack_nvfp4_expert writes (E2M1 codes, E4M3 block scales; checked
byte for byte against a numpy restatement of the layout); the activations
enter as six NVFP4 residual terms (ffn_b200_quantize_nvfp4_terms).  The
quantiser is checked bit for bit against a numpy restatement of its rule, the
layer against the oracle at the path's tolerance (max|y-ref|/max|ref| <= 1e-3,
cosine >= 0.99999)."""
import ctypes as C

import numpy as np
import pytest

from test_gpu_parity import host, oracle_nvfp4_expert

pytestmark = pytest.mark.gpu


# ------------------------------------------------- quantiser restatement
def _ue4m3_ceil(s):
    """Smallest UE4M3 code with value >= s (s >= 0 float32), at most 0x7E."""
    s = s.astype(np.float32)
    bits = s.view(np.uint32).astype(np.int64)
    e = (bits >> 23) - 127
    mq = ((bits & 0x7FFFFF) + 0xFFFFF) >> 20
    carry = mq == 8
    mq = np.where(carry, 0, mq)
    e2 = e + carry
    normal = np.minimum(((e2 + 7) << 3) | mq, 0x7E)
    normal = np.where(e2 > 8, 0x7E, normal)
    sub = np.ceil(s.astype(np.float64) * 512.0).astype(np.int64)
    code = np.where(e >= -6, normal, sub)
    return np.where(s > 0, code, 0).astype(np.uint8)


def _ue4m3_value(c):
    c = c.astype(np.int64)
    e, m = c >> 3, c & 7
    return np.where(e == 0, m / 512.0, (8 + m) * np.exp2(e - 10.0)).astype(np.float32)


_E2M1 = np.array([0, .5, 1, 1.5, 2, 3, 4, 6], dtype=np.float32)


def _e2m1_rne(v):
    """E2M1 code of v (round to nearest, ties to even, saturated at +-6)."""
    a = np.abs(v)
    c = ((a > 0.25).astype(np.int64) + (a >= 0.75) + (a > 1.25) + (a >= 1.75) + (a > 2.5) +
         (a >= 3.5) + (a > 5.0))
    return np.where(np.signbit(v), c | 8, c).astype(np.uint8)  # a negative value keeps its sign at 0


def quantize_ref(x, terms=4):
    rows, K = x.shape
    codes = np.zeros((rows, terms, K // 2), np.uint8)
    scales = np.zeros((rows, terms, K // 16), np.uint8)
    exps = np.zeros((rows, terms), np.int32)
    r = x.astype(np.float32).copy()
    for t in range(terms):
        am = np.abs(r).max(1)
        for i in range(rows):
            e = 0
            if am[i] > 0:
                _, ex = np.frexp(am[i])
                e = int(max(-110, min(110, ex - 1 - 8)))
            exps[i, t] = e
        inv = np.exp2(-exps[:, t].astype(np.float64)).astype(np.float32)[:, None, None]
        sc = np.exp2(exps[:, t].astype(np.float64)).astype(np.float32)[:, None, None]
        b = r.reshape(rows, K // 16, 16)
        bm = (np.abs(b).max(2, keepdims=True) * inv).astype(np.float32)
        code = _ue4m3_ceil((bm / np.float32(6)).astype(np.float32)[..., 0])
        sv = _ue4m3_value(code)[..., None]
        with np.errstate(divide="ignore", invalid="ignore"):
            rcp = (np.float32(1) / sv).astype(np.float32)  # correctly rounded reciprocal
            q = np.where(sv > 0, ((b * inv).astype(np.float32) * rcp).astype(np.float32), 0).astype(np.float32)
        c = np.where(sv > 0, _e2m1_rne(q), 0).astype(np.uint8)
        val = np.where(c & 8, -_E2M1[c & 7], _E2M1[c & 7]).astype(np.float32)
        r = (b - val * (sv * sc)).astype(np.float32).reshape(rows, K)
        codes[:, t] = (c[..., 0::2] | (c[..., 1::2] << 4)).reshape(rows, K // 2)
        scales[:, t] = code
    return codes, scales, exps


def dequant_terms(codes, scales, exps):
    rows, terms, half = codes.shape
    K = 2 * half
    lo, hi = codes & 15, codes >> 4
    c = np.stack([lo, hi], -1).reshape(rows, terms, K)
    val = np.where(c & 8, -_E2M1[c & 7], _E2M1[c & 7]).astype(np.float64)
    s = _ue4m3_value(scales).astype(np.float64).repeat(16, axis=2)
    return (val * s * np.exp2(exps[..., None].astype(np.float64))).sum(1)


def gpu_quantize(ffn, cuda, x, terms=4):
    import torch
    rows, K = x.shape
    xd = torch.from_numpy(x).to(cuda)
    codes = torch.empty(rows, terms, K // 2, dtype=torch.uint8, device=cuda)
    scales = torch.empty(rows, terms, K // 16, dtype=torch.uint8, device=cuda)
    exps = torch.empty(rows, terms, dtype=torch.int32, device=cuda)
    p = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    if terms == 4:
        rc = ffn.lib().ffn_b200_quantize_nvfp4x4(rows, K, p(xd), K, p(codes), p(scales), p(exps), None)
    else:
        rc = ffn.lib().ffn_b200_quantize_nvfp4_terms(rows, K, terms, p(xd), K, p(codes), p(scales), p(exps),
                                                     None)
    ffn.check(rc, "quantize_nvfp4")
    torch.cuda.synchronize()
    return host(codes), host(scales), host(exps)


@pytest.mark.parametrize("K,terms", [(256, 4), (2048, 4), (4096, 4), (7168, 4), (2048, 6), (4096, 6)])
def test_quantizer_bit_exact_and_accurate(ffn, cuda, K, terms):
    rng = np.random.default_rng(K)
    rows = [rng.standard_normal(K), rng.standard_normal(K) * 1e-6, np.zeros(K),
            rng.standard_normal(K) * np.exp(rng.uniform(-12, 12, K)),  # wide dynamic range
            np.where(rng.random(K) < 0.9, 0.0, rng.standard_normal(K) * 50),  # mostly zero
            np.full(K, 3.0), rng.uniform(-100, 100, K)]
    x = np.stack(rows).astype(np.float32)
    got = gpu_quantize(ffn, cuda, x, terms)
    want = quantize_ref(x, terms)
    for g, w, name in zip(got, want, ("codes", "scales", "exponents")):
        assert np.array_equal(g, w), f"{name} differ at {np.argwhere(g != w)[:5]}"
    back = dequant_terms(*got)
    for i in range(len(rows)):
        den = np.abs(x[i]).max()
        if den == 0:
            assert np.all(back[i] == 0)
            continue
        # element-wise: a single value can keep up to ~max/6^terms; dot products average it out
        assert np.abs(back[i] - x[i]).max() / den < (1e-3 if terms == 4 else 1e-4), f"row {i}"


# ------------------------------------------------------------- the layer
def _layer(ffn, E, H, I, seed, path, score_fn=None):
    experts = [ffn.SwigluExpert.generate(ffn.FMT_NVFP4, seed, 0, e, I, H).pack_fp4() for e in range(E)]
    wr = ffn.gen_normal(ffn.path_key(seed, 0, 0, ffn.TAG_ROUTER), E * H, 0.02).view(E, H)
    kw = {} if score_fn is None else {"score_fn": score_fn}
    return experts, wr, lambda top_k, p=path: ffn.MoeLayer(experts, wr, H, I, top_k=top_k, path=p, **kw)


@pytest.mark.parametrize("E,H,I,T,K", [(16, 512, 256, 5, 6),     # one token per expert mostly
                                       (8, 512, 256, 40, 6),     # ~30 tokens per expert: 4 chunks each
                                       (16, 5120, 2304, 24, 6),  # the reference checkpoint's dims
                                       (32, 1024, 768, 1, 6)])   # a single token
def test_fp4_layer_vs_oracle(oracle, ffn, cuda, E, H, I, T, K):
    import torch
    experts, wr, make = _layer(ffn, E, H, I, 80 + T, ffn.PATH_FP4)
    x = ffn.gen_normal(ffn.path_key(80 + T, 0, 0, ffn.TAG_X), T * H).view(T, H)
    idx = torch.empty(T, K, dtype=torch.int32, device=cuda)
    out = host(make(K).forward(x, topk_idx=idx, residual=x))
    oe = [oracle_nvfp4_expert(oracle, e) for e in experts]
    xs = host(x)
    ref, ridx, _ = oracle.moe_layer(oe, host(wr), xs, top_k=K)
    assert np.array_equal(host(idx), ridx)
    oracle.assert_close(out - xs, ref, what=f"fp4 layer E{E} H{H} I{I} T{T}")


@pytest.mark.parametrize("mode", ["exact", "tensor"])
def test_fp4_layer_with_ffn_norm(oracle, ffn, cuda, mode):
    """The reference's ffn_norm before routing (RMSNorm, flash1017.rs:7637): on
    the FP4 path the norm, the router's f16 split and the experts' NVFP4 terms
    come from one kernel (xq_kernel).  With the exact router the norm's
    sum runs in the reference's order, so the top-6 sets match the oracle's
    exactly; the tensor router may differ only at near-ties."""
    import torch
    E, H, I, T, K = 32, 1024, 512, 16, 6
    experts, wr, _ = _layer(ffn, E, H, I, 95, ffn.PATH_FP4)
    nw = (1.0 + 0.1 * ffn.gen_normal(ffn.path_key(95, 0, 1, ffn.TAG_X), H)).contiguous()
    x = (3.0 * ffn.gen_normal(ffn.path_key(95, 0, 0, ffn.TAG_X), T * H)).view(T, H)
    rm = ffn.ROUTER_EXACT if mode == "exact" else ffn.ROUTER_TENSOR
    layer = ffn.MoeLayer(experts, wr, H, I, top_k=K, path=ffn.PATH_FP4, router_mode=rm, norm_w=nw,
                         norm_eps=1e-20)
    idx = torch.empty(T, K, dtype=torch.int32, device=cuda)
    out = host(layer.forward(x, topk_idx=idx, residual=x))
    oe = [oracle_nvfp4_expert(oracle, e) for e in experts]
    xs = host(x)
    ref, ridx, _ = oracle.moe_layer(oe, host(wr), xs, top_k=K, norm_w=host(nw), norm_eps=1e-20)
    if mode == "exact":
        assert np.array_equal(host(idx), ridx)
    else:
        xn = xs / np.sqrt((xs.astype(np.float64) ** 2).mean(axis=1, keepdims=True)) * host(nw)
        bs = oracle.biased_sorted(oracle.router_logits(host(wr), xn.astype(np.float32)), K)
        assert oracle.topk_agrees(host(idx), ridx, bs).all()
    same = (host(idx) == ridx).all(axis=1)
    oracle.assert_close((out - xs)[same], ref[same], what=f"fp4 layer with ffn_norm ({mode} router)")


def test_fp4_matches_gemv_path_and_is_deterministic(oracle, ffn, cuda):
    E, H, I, T, K = 24, 1024, 512, 48, 6
    experts, wr, make = _layer(ffn, E, H, I, 91, ffn.PATH_FP4)
    x = ffn.gen_normal(ffn.path_key(91, 0, 0, ffn.TAG_X), T * H).view(T, H)
    a = host(make(K).forward(x))
    b = host(make(K).forward(x))
    g = host(make(K, ffn.PATH_GEMV).forward(x))
    assert np.array_equal(a, b), "FP4 path not deterministic"
    oracle.assert_close(a, g, what="fp4 vs gemv path")


def test_fp4_rejects_scales_outside_ue4m3(oracle, ffn, cuda):
    """A scale byte with the sign bit set (or the E4M3 NaN 0x7F) is not a UE4M3
    value: packing refuses the expert, so the FP4 path never sees it, and the
    layer of unpacked experts runs on the GEMV slices (which decode E4M3)."""
    import torch
    E, H, I, T, K = 8, 512, 256, 6, 6
    experts = [ffn.SwigluExpert.generate(ffn.FMT_NVFP4, 93, 0, e, I, H) for e in range(E)]
    for bad in (0xB8, 0x7F):  # -1.0 in E4M3, NaN
        s = experts[3].mats[0].s
        keep = s[5].clone()
        s[5] = bad
        with pytest.raises(ffn.FfnError, match="UE4M3"):
            experts[3].pack_fp4()
        s[5] = keep
    assert experts[3].fp4 is None
    wr = ffn.gen_normal(ffn.path_key(93, 0, 0, ffn.TAG_ROUTER), E * H, 0.02).view(E, H)
    x = ffn.gen_normal(ffn.path_key(93, 0, 0, ffn.TAG_X), T * H).view(T, H)
    with pytest.raises(ffn.FfnError, match="packed"):
        ffn.MoeLayer(experts, wr, H, I, top_k=K, path=ffn.PATH_FP4).forward(x)
    ffn.profile_enable(True)
    out = host(ffn.MoeLayer(experts, wr, H, I, top_k=K).forward(x))
    torch.cuda.synchronize()
    prof = ffn.profile_read()
    ffn.profile_enable(False)
    assert "gateup_nvfp4" in prof and "fp4_gateup" not in prof and np.isfinite(out).all()


def test_fp4_stage_images(oracle, ffn, cuda):
    """ffn_b200_pack_nvfp4_expert against a numpy restatement of the layout:
    stage (row block, K step) = both blocks' 128-byte-swizzled code tiles, then
    their scale atoms (line l = rows l, l+32, l+64, l+96)."""
    H, I = 512, 768
    ex = ffn.SwigluExpert.generate(ffn.FMT_NVFP4, 97, 0, 0, I, H).pack_fp4()
    gu, dn = host(ex.fp4[0]), host(ex.fp4[1])
    assert gu.size == ffn.lib().ffn_b200_fp4_pack_bytes(I, H, 0) == 2 * I * (H // 2 + H // 16)
    assert dn.size == ffn.lib().ffn_b200_fp4_pack_bytes(I, H, 1) == H * (I // 2 + I // 16)
    w = [host(m.w).reshape(m.rows, m.cols // 2) for m in ex.mats]
    s = [host(m.s).reshape(m.rows, m.cols // 16) for m in ex.mats]

    def image(wa, sa, ra, wb, sb, rb_, kt):
        img = np.zeros(36864, dtype=np.uint8)
        for blk, (ww, ss, r0) in enumerate(((wa, sa, ra), (wb, sb, rb_))):
            for r in range(128):
                for c in range(8):
                    off = blk * 16384 + (r // 8) * 1024 + (r % 8) * 128 + ((c ^ (r % 8)) * 16)
                    img[off:off + 16] = ww[r0 + r, kt * 128 + c * 16: kt * 128 + c * 16 + 16]
            for k in range(4):
                for l in range(32):
                    off = 32768 + blk * 2048 + k * 512 + l * 16
                    for q in range(4):
                        img[off + 4 * q: off + 4 * q + 4] = ss[r0 + l + 32 * q, kt * 16 + 4 * k: kt * 16 + 4 * k + 4]
        return img

    kt_h, kt_i = H // 256, I // 256
    for rb in (0, I // 128 - 1):
        for kt in (0, kt_h - 1):
            want = image(w[0], s[0], rb * 128, w[1], s[1], rb * 128, kt)
            got = gu[(rb * kt_h + kt) * 36864:(rb * kt_h + kt + 1) * 36864]
            np.testing.assert_array_equal(got, want)
    for rb in (0, H // 256 - 1):
        for kt in (0, kt_i - 1):
            want = image(w[2], s[2], rb * 256, w[2], s[2], rb * 256 + 128, kt)
            got = dn[(rb * kt_i + kt) * 36864:(rb * kt_i + kt + 1) * 36864]
            np.testing.assert_array_equal(got, want)


def test_fp4_config2_all_tokens(oracle, ffn, cuda):
    """Benchmark config 2 (384 NVFP4 experts, H 4096, I 2048, 64 tokens, sigmoid
    top-6, seed 2) on the FP4 path: every token's top-6 and output against the
    oracle."""
    import torch
    E, H, I, T, K, seed = 384, 4096, 2048, 64, 6, 2
    experts, wr, make = _layer(ffn, E, H, I, seed, ffn.PATH_FP4, ffn.SCORE_SIGMOID)
    x = ffn.gen_normal(ffn.path_key(seed, 0, 0, ffn.TAG_X), T * H).view(T, H)
    idx = torch.empty(T, K, dtype=torch.int32, device=cuda)
    out = host(make(K).forward(x, topk_idx=idx))
    oracle.set_threads(16)
    xs = host(x)
    ridx, rwt, _, _ = oracle.route(oracle.router_logits(host(wr), xs), K, None, 1)
    assert np.array_equal(host(idx), ridx)
    used = sorted(set(ridx.ravel().tolist()))
    oe = {e: oracle_nvfp4_expert(oracle, experts[e]) for e in used}
    ref = np.zeros((T, H), dtype=np.float32)
    for t in range(T):
        xt = np.ascontiguousarray(xs[t])
        for k in range(K):
            oracle.axpy(ref[t], rwt[t, k], oe[ridx[t, k]].forward(xt))
    oracle.assert_close(out, ref, what="config 2, all 64 tokens, FP4 path")
    for t in range(T):
        oracle.assert_close(out[t], ref[t], what=f"config 2 token {t}")
