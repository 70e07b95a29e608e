"""Generates the committed golden fixtures in this folder.

Run from the repository root:  python tests/golden/make_golden.py

The fixtures pin the C oracle (oracle/ffn_oracle.c) to sources independent of
it, since the Rust reference itself cannot be executed here:
  * e4m3_torch.json   -- all 256 E4M3 codes decoded by torch.float8_e4m3fn.
  * known_answers.json -- outputs of pure-Python float32 restatements of the
    reference loops (terox27/Flash1017-Engine, crates/flash-core/src/
    flash1017.rs: NVFP4 :2331-2357, ternary :2602-2621 and :2567-2601, rank-16
    :2446-2472, router :7280-7376, MXFP4 :2717-2744, MXFP8 :1960-1982 with the
    E8M0 decode :1049-1057), evaluated term by term with numpy float32
    scalars in the reference's order, on deterministic inputs.  The NVFP4 input
    is the reference's own test fixture (flash1017.rs:10974-10990: nibbles
    (i*7+3)%16 / (i*13+5)%16, scales alternating 0x38/0x3C, global scale 0.02);
    x follows the reference's addon micro-benchmark pattern
    (hardware_addon.rs:1074: sin(0.013 i) * 0.5).
  * generator.json -- SHA-256 of seeded generator outputs (pins the generator
    that the CUDA library's device generator must reproduce byte for byte).
  * compress.json -- the 106 GB format's compressor (flash1017.rs:10342-10645:
    block-64 ternary quantisation, rank-16 subspace iteration with f64
    Gram-Schmidt, int8 core) restated term by term in numpy float32 scalars and
    Python f64 floats, on the reference's own compressor-test input: SHA-256 of
    every output array and the three f64 error sums.
"""
import hashlib
import json
import math
import os
import struct
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

F = np.float32
LUT4 = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0]
TLUT = [-1.0, 0.0, 1.0, 0.0]


def e4m3(b: int) -> F:
    """flash1017.rs:1031-1045 restated independently (struct bit casts)."""
    sign = (b & 0x80) << 24
    em = b & 0x7F
    if em == 0x7F:
        return F("nan")
    if em < 8:
        sub = F(em) * F(1.0 / 512.0)
        bits = struct.unpack("<I", struct.pack("<f", sub))[0]
        return F(struct.unpack("<f", struct.pack("<I", sign | bits))[0])
    return F(struct.unpack("<f", struct.pack("<I", sign | ((em + 960) << 20)))[0])


def e8m0(b: int) -> F:
    """flash1017.rs:1049-1057 restated: 0xFF NaN, 0 -> bits 0x00400000, else b << 23."""
    if b == 0xFF:
        return F("nan")
    bits = 0x00400000 if b == 0 else (b << 23)
    return F(struct.unpack("<f", struct.pack("<I", bits))[0])


def mxfp4_matvec_py(w, s, x, rows, cols):
    out = []
    spr = cols // 32
    for r in range(rows):
        wr = w[r * cols // 2:(r + 1) * cols // 2]
        acc = F(0)
        for g in range(spr):
            sc = e8m0(int(s[r * spr + g]))
            bsum = F(0)
            for k in range(16):
                b = int(wr[g * 16 + k])
                w0, w1 = F(LUT4[b & 15]), F(LUT4[b >> 4])
                bsum = F(bsum + F(F(w0 * x[g * 32 + 2 * k]) + F(w1 * x[g * 32 + 2 * k + 1])))
            acc = F(acc + F(bsum * sc))
        out.append(acc)
    return np.array(out, dtype=np.float32)


def mxfp8_matvec_py(w, s, x, rows, cols):
    out = []
    scols = (cols + 31) // 32
    for r in range(rows):
        acc = F(0)
        for bc in range(scols):
            sc = e8m0(int(s[(r // 32) * scols + bc]))
            bsum = F(0)
            for c in range(bc * 32, min(bc * 32 + 32, cols)):
                bsum = F(bsum + F(e4m3(int(w[r * cols + c])) * x[c]))
            acc = F(acc + F(bsum * sc))
        out.append(acc)
    return np.array(out, dtype=np.float32)


def nvfp4_matvec_py(w, s, gs, x, rows, cols):
    out = []
    gpr = cols // 16
    for r in range(rows):
        wr = w[r * cols // 2:(r + 1) * cols // 2]
        sr = s[r * gpr:(r + 1) * gpr]
        row_acc = F(0)
        for g in range(gpr):
            gsc = e4m3(int(sr[g]))
            gsum = F(0)
            for k in range(8):
                b = int(wr[g * 8 + k])
                v0, v1 = F(LUT4[b & 15]), F(LUT4[b >> 4])
                gsum = F(gsum + F(F(v0 * x[g * 16 + 2 * k]) + F(v1 * x[g * 16 + 2 * k + 1])))
            row_acc = F(row_acc + F(gsum * gsc))
        out.append(F(row_acc * F(gs)))
    return np.array(out, dtype=np.float32)


def _tern4(b, x, base):
    t = F(F(F(F(TLUT[b & 3]) * x[base]) + F(F(TLUT[(b >> 2) & 3]) * x[base + 1]))
          + F(F(TLUT[(b >> 4) & 3]) * x[base + 2]))
    return F(t + F(F(TLUT[(b >> 6) & 3]) * x[base + 3]))


def ternary_matvec_py(p, rs, x, rows, cols, bs=None):
    out = []
    pc = cols // 4
    for r in range(rows):
        row = p[r * pc:(r + 1) * pc]
        if bs is None:
            acc = F(0)
            for i, b in enumerate(row):
                b = int(b)
                if b == 0x55:
                    continue
                acc = F(acc + _tern4(b, x, 4 * i))
            out.append(F(acc * F(rs[r])))
        else:
            bpr = cols // 64
            row_acc = F(0)
            for blk in range(bpr):
                u8 = int(bs[r * bpr + blk])
                if u8 == 0:
                    continue
                bacc = F(0)
                for k in range(16):
                    b = int(row[blk * 16 + k])
                    if b == 0x55:
                        continue
                    bacc = F(bacc + _tern4(b, x, (blk * 16 + k) * 4))
                row_acc = F(row_acc + F(bacc * F(u8)))
            out.append(F(row_acc * F(rs[r])))
    return np.array(out, dtype=np.float32)


def rank16_py(a, a_sc, b, b_sc, x, y, rows, cols, rank=16):
    z = []
    for r in range(rank):
        dot = F(0)
        for c in range(cols):
            dot = F(dot + F(F(int(a[r * cols + c])) * x[c]))
        z.append(F(F(F(dot * F(a_sc[r])) * F(b_sc[r])) * F(1.0)))
    y = y.copy()
    for row in range(rows):
        acc = F(0)
        for r in range(rank):
            acc = F(acc + F(F(int(b[row * rank + r])) * z[r]))
        y[row] = F(y[row] + acc)
    return y


def route_py(logits, top_k, score_fn):
    """Selections by (biased desc, index asc); weights as the reference forms them."""
    cands = []
    for e in range(len(logits)):
        l = float(logits[e])
        if score_fn == 0:
            sp = l if l > 20 else (math.exp(l) if l < -20 else math.log(1 + math.exp(l)))
            sc = math.sqrt(max(sp, 0.0))
        else:
            sc = 1.0 / (1.0 + math.exp(-l))
        cands.append((e, sc))
    cands.sort(key=lambda c: (-c[1], c[0]))
    sel = cands[:top_k]
    tot = sum(c[1] for c in sel)
    num = 1.5 if score_fn == 0 else 1.0
    return [c[0] for c in sel], [c[1] * num / tot for c in sel]


def round_away(v) -> F:
    """Rust f32::round: halves away from zero."""
    return F(math.copysign(math.floor(abs(float(v)) + 0.5), float(v)))


def ortho16_py(m):
    """flash1017.rs:10342-10372 on a list of 16-float rows (in place)."""
    n = len(m)
    for k in range(16):
        for j in range(k):
            dot = 0.0
            for r in range(n):
                dot += float(m[r][k]) * float(m[r][j])
            d = F(dot)
            for r in range(n):
                m[r][k] = F(m[r][k] - F(d * m[r][j]))
        norm_sq = 0.0
        for r in range(n):
            v = float(m[r][k])
            norm_sq += v * v
        inv = F(1.0 / math.sqrt(norm_sq)) if norm_sq > 1e-24 else F(0.0)
        for r in range(n):
            m[r][k] = F(m[r][k] * inv)


def compress_py(w, s, gs, rows, cols, seed):
    """flash1017.rs:10377-10645 restated loop for loop."""
    gs = F(gs)
    pcols, groups, nblk, tcols = cols // 2, cols // 16, cols // 64, cols // 4
    e4 = [e4m3(b) for b in range(256)]
    packed = np.zeros(rows * tcols, np.uint8)
    row_scales = np.zeros(rows, np.float32)
    block_scales = np.zeros(rows * nblk, np.uint8)
    res = [[F(0.0)] * cols for _ in range(rows)]
    orig = terr = 0.0
    for r in range(rows):
        rr = res[r]
        for g in range(groups):
            g_sc = F(e4[int(s[r * groups + g])] * gs)
            for k in range(8):
                b = int(w[r * pcols + g * 8 + k])
                w0, w1 = F(F(LUT4[b & 15]) * g_sc), F(F(LUT4[b >> 4]) * g_sc)
                rr[g * 16 + 2 * k], rr[g * 16 + 2 * k + 1] = w0, w1
                orig += float(w0) * float(w0) + float(w1) * float(w1)
        gam = [F(0.0)] * nblk
        max_gamma = F(0.0)
        for blk in range(nblk):
            wb = rr[blk * 64:(blk + 1) * 64]
            sq = F(0.0)
            for v in wb:
                sq = F(sq + F(v * v))
            rms = F(np.sqrt(F(sq * F(1.0 / 64.0))))
            base = r * tcols + blk * 16
            if rms <= F(1e-12):
                packed[base:base + 16] = 0x55
                continue
            best_score, best_gamma, best_th = F(-1.0), F(0.0), F(F(0.58) * rms)
            for fac in (0.42, 0.54, 0.66, 0.78):
                th = F(F(fac) * rms)
                dot, cnt = F(0.0), 0
                for v in wb:
                    if v > th:
                        dot, cnt = F(dot + v), cnt + 1
                    elif v < -th:
                        dot, cnt = F(dot - v), cnt + 1
                if cnt > 0:
                    score = F(F(dot * dot) / F(cnt))
                    if score > best_score:
                        best_score, best_gamma, best_th = score, F(dot / F(cnt)), th
            gam[blk] = best_gamma
            if best_gamma > max_gamma:
                max_gamma = best_gamma
            for i, v in enumerate(wb):
                code = 2 if v > best_th else (0 if v < -best_th else 1)
                packed[base + (i >> 2)] |= code << ((i & 3) * 2)
        row_sc = F(max_gamma / F(255.0)) if max_gamma > F(1e-12) else F(0.0)
        row_scales[r] = row_sc
        for blk in range(nblk):
            u8 = int(min(max(round_away(F(gam[blk] / row_sc)), 0.0), 255.0)) if row_sc > F(0.0) else 0
            block_scales[r * nblk + blk] = u8
            qg = F(F(u8) * row_sc)
            for i in range(16):
                pb = int(packed[r * tcols + blk * 16 + i])
                v = []
                for u in range(4):
                    c = blk * 64 + 4 * i + u
                    rr[c] = F(rr[c] - F(F(TLUT[(pb >> (2 * u)) & 3]) * qg))
                    v.append(float(rr[c]))
                terr += v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3]
    M, G = (1 << 64) - 1, 0x9E3779B97F4A7C15
    rng = (seed ^ G) & M
    p = []
    for c in range(cols):
        row = []
        for k in range(16):
            rng = (rng + G) & M
            x = rng
            x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & M
            x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & M
            x ^= x >> 31
            row.append(F(F((x >> 40) - (1 << 23)) * F(1.0 / (1 << 23))))
        p.append(row)
    ortho16_py(p)
    for sweep in range(2):
        q = []
        for r in range(rows):
            acc = [F(0.0)] * 16
            for c in range(cols):
                v = res[r][c]
                for k in range(16):
                    acc[k] = F(acc[k] + F(v * p[c][k]))
            q.append(acc)
        ortho16_py(q)
        z = [[F(0.0)] * 16 for _ in range(cols)]
        for r in range(rows):
            for c in range(cols):
                v = res[r][c]
                for k in range(16):
                    z[c][k] = F(z[c][k] + F(v * q[r][k]))
        if sweep == 0:
            p = [list(row) for row in z]
            ortho16_py(p)
    core_b, core_a = np.zeros(rows * 16, np.int8), np.zeros(16 * cols, np.int8)
    b_sc, a_sc = np.zeros(16, np.float32), np.zeros(16, np.float32)
    captured = 0.0
    for k in range(16):
        mx = F(0.0)
        for r in range(rows):
            if abs(q[r][k]) > mx:
                mx = abs(q[r][k])
        b_sc[k] = F(mx / F(127.0)) if mx > F(1e-12) else F(0.0)
        if b_sc[k] > 0:
            inv = F(F(1.0) / b_sc[k])
            for r in range(rows):
                core_b[r * 16 + k] = int(min(max(round_away(F(q[r][k] * inv)), -127.0), 127.0))
        mz, cn = F(0.0), 0.0
        for c in range(cols):
            if abs(z[c][k]) > mz:
                mz = abs(z[c][k])
            cn += float(z[c][k]) * float(z[c][k])
        captured += cn
        a_sc[k] = F(mz / F(127.0)) if mz > F(1e-12) else F(0.0)
        if a_sc[k] > 0:
            inv = F(F(1.0) / a_sc[k])
            for c in range(cols):
                core_a[k * cols + c] = int(min(max(round_away(F(z[c][k] * inv)), -127.0), 127.0))
    return dict(packed=packed, row_scales=row_scales, block_scales=block_scales, core_b=core_b,
                core_b_sc=b_sc, core_a=core_a, core_a_sc=a_sc, orig_frob_sq=orig, ternary_err_sq=terr,
                jepa_err_sq=max(terr - captured, 0.0))


COMPRESS_ARRAYS = ("packed", "row_scales", "block_scales", "core_b", "core_b_sc", "core_a", "core_a_sc")


def bench_x(n):
    return np.array([F(math.sin(i * 0.013) * 0.5) for i in range(n)], dtype=np.float32)


def main():
    import torch
    import oracle as O

    codes = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    json.dump({"bits": [int(v) for v in codes.view(np.uint32)]},
              open(os.path.join(HERE, "e4m3_torch.json"), "w"))

    ka = {}
    # NVFP4 on the reference's compressor-test fixture (flash1017.rs:10974-10990)
    rows, cols = 64, 128
    w = np.array([((i * 7 + 3) % 16) | (((i * 13 + 5) % 16) << 4) for i in range(rows * cols // 2)],
                 dtype=np.uint8)
    s = np.array([0x38 if i % 2 == 0 else 0x3C for i in range(rows * cols // 16)], dtype=np.uint8)
    ka["nvfp4_fixture"] = {"rows": rows, "cols": cols, "gs": 0.02,
                           "y": nvfp4_matvec_py(w, s, 0.02, bench_x(cols), rows, cols).tolist()}
    # NVFP4 with all 16 codes and normal / subnormal scales
    rows2, cols2 = 16, 256
    w2 = np.array([(i * 37 + 11) & 0xFF for i in range(rows2 * cols2 // 2)], dtype=np.uint8)
    s2 = np.array([(i * 29 + 1) % 0x7F for i in range(rows2 * cols2 // 16)], dtype=np.uint8)
    ka["nvfp4_scales"] = {"rows": rows2, "cols": cols2, "gs": 0.75, "w": w2.tolist(),
                          "s": s2.tolist(),
                          "y": nvfp4_matvec_py(w2, s2, 0.75, bench_x(cols2), rows2, cols2).tolist()}
    # ternary: all codes (including 3) with 0x55 bytes mixed in
    rows3, cols3 = 32, 256
    p = np.array([(0x55 if (i % 7 == 0) else ((i * 73 + 5) & 0xFF)) for i in range(rows3 * cols3 // 4)],
                 dtype=np.uint8)
    rs = np.array([0.01 + 0.001 * r for r in range(rows3)], dtype=np.float32)
    bs = np.array([(i * 11) % 256 for i in range(rows3 * cols3 // 64)], dtype=np.uint8)
    xt = bench_x(cols3)
    ka["ternary"] = {"rows": rows3, "cols": cols3, "p": p.tolist(), "rs": rs.tolist(),
                     "y": ternary_matvec_py(p, rs, xt, rows3, cols3).tolist(),
                     "bs": bs.tolist(),
                     "y_bs": ternary_matvec_py(p, rs, xt, rows3, cols3, bs).tolist()}
    # MXFP4: all 16 E2M1 codes, E8M0 scales around 2^0 (120..134)
    rows4, cols4 = 16, 256
    w4 = np.array([(i * 53 + 7) & 0xFF for i in range(rows4 * cols4 // 2)], dtype=np.uint8)
    s4 = np.array([120 + (i * 5) % 15 for i in range(rows4 * cols4 // 32)], dtype=np.uint8)
    ka["mxfp4"] = {"rows": rows4, "cols": cols4, "w": w4.tolist(), "s": s4.tolist(),
                   "y": mxfp4_matvec_py(w4, s4, bench_x(cols4), rows4, cols4).tolist()}
    # MXFP8: E4M3 codes (NaN codes 0x7F / 0xFF avoided), 32 x 32 block scales
    rows5, cols5 = 64, 96
    w5 = np.array([(i * 29 + 3) & 0xFF for i in range(rows5 * cols5)], dtype=np.uint8)
    w5[(w5 & 0x7F) == 0x7F] = 0x3C
    s5 = np.array([118 + (i * 7) % 13 for i in range(((rows5 + 31) // 32) * ((cols5 + 31) // 32))],
                  dtype=np.uint8)
    ka["mxfp8"] = {"rows": rows5, "cols": cols5, "w": w5.tolist(), "s": s5.tolist(),
                   "y": mxfp8_matvec_py(w5, s5, bench_x(cols5), rows5, cols5).tolist()}
    ka["e8m0"] = {"bits": [int(np.float32(e8m0(b)).view(np.uint32)) for b in range(256)]}
    # rank-16 core added onto a zero output
    a = np.array([((i * 31 + 7) % 255) - 127 for i in range(16 * cols3)], dtype=np.int8)
    b = np.array([((i * 17 + 3) % 255) - 127 for i in range(rows3 * 16)], dtype=np.int8)
    a_sc = np.array([1e-4 * (1 + r) for r in range(16)], dtype=np.float32)
    b_sc = np.array([2e-4 * (16 - r) for r in range(16)], dtype=np.float32)
    y0 = np.zeros(rows3, dtype=np.float32)
    ka["rank16"] = {"a": a.tolist(), "b": b.tolist(), "a_sc": a_sc.tolist(), "b_sc": b_sc.tolist(),
                    "y": rank16_py(a, a_sc, b, b_sc, xt, y0, rows3, cols3).tolist()}
    # router: logits pattern over 384 experts, both score functions
    logits = np.array([F(math.sin(e * 0.37) * 3.0 + math.cos(e * 1.3)) for e in range(384)],
                      dtype=np.float32)
    r0, r1 = route_py(logits, 6, 0), route_py(logits, 6, 1)
    ka["router"] = {"logits": logits.tolist(), "ref_idx": r0[0], "ref_w": r0[1],
                    "sig_idx": r1[0], "sig_w": r1[1]}
    json.dump(ka, open(os.path.join(HERE, "known_answers.json"), "w"))

    def h(arr):
        return hashlib.sha256(np.ascontiguousarray(arr).tobytes()).hexdigest()

    gen = {}
    w_, s_ = O.gen_nvfp4(O.key(0, 0, 0, O.TAG_W1), 64, 4096)
    gen["nvfp4_64x4096"] = [h(w_), h(s_)]
    p_, r_ = O.gen_ternary(O.key(1, 0, 0, O.TAG_W1), 64, 4096)
    gen["ternary_64x4096"] = [h(p_), h(r_)]
    c_ = O.gen_core(O.key(1, 0, 0, O.TAG_W1), 64, 4096)
    gen["core_64x4096"] = [h(c_.a), h(c_.a_sc), h(c_.b), h(c_.b_sc)]
    gen["normal_100000"] = h(O.gen_normal(O.key(2, 0, 0, O.TAG_X), 100000))
    json.dump(gen, open(os.path.join(HERE, "generator.json"), "w"), indent=1)
    # compressor on the reference's compressor-test input (flash1017.rs:10975-10995)
    cp = compress_py(w, s, 0.02, rows, cols, 42)
    json.dump({"rows": rows, "cols": cols, "gs": 0.02, "seed": 42,
               "sha256": {k: h(cp[k]) for k in COMPRESS_ARRAYS},
               "orig_frob_sq": cp["orig_frob_sq"], "ternary_err_sq": cp["ternary_err_sq"],
               "jepa_err_sq": cp["jepa_err_sq"]},
              open(os.path.join(HERE, "compress.json"), "w"), indent=1)
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main()
