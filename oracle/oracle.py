"""TEST INFRASTRUCTURE ONLY -- numpy front end of the CPU oracle (ffn_oracle.c).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline legs may
import this module.  It restates the reference's CPU dot path
(terox27/Flash1017-Engine, ``crates/flash-core/src/flash1017.rs``) and supplies
the seeded synthetic generators whose bytes the CUDA library's device
generator reproduces exactly.

Parity pinning: see the header of ffn_oracle.c.  Known-answer vectors pin the
decoders; the summation-order restatement of the matvec loops is "parity
unpinned" against executed reference output (no Rust toolchain here).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle_ffn.so")

_lib = None


def build() -> str:
    """Compile ffn_oracle.c (make -C oracle)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(
            os.path.join(HERE, "ffn_oracle.c")
        ):
            build()
        L = C.CDLL(LIB_PATH)
        sz, f32, u64, i32 = C.c_size_t, C.c_float, C.c_uint64, C.c_int
        vp = C.c_void_p
        L.orc_e4m3_to_f32.restype = f32
        L.orc_e4m3_to_f32.argtypes = [C.c_uint8]
        L.orc_e2m1_to_f32.restype = f32
        L.orc_e2m1_to_f32.argtypes = [C.c_uint8]
        L.orc_f32_to_e4m3.restype = C.c_uint8
        L.orc_f32_to_e4m3.argtypes = [f32]
        L.orc_set_threads.argtypes = [i32]
        L.orc_get_threads.restype = i32
        L.orc_nvfp4_matvec.argtypes = [sz, sz, vp, vp, f32, vp, vp]
        L.orc_nvfp4_matbatch.argtypes = [sz, sz, sz, vp, vp, f32, vp, vp]
        L.orc_rank16_apply_add.argtypes = [sz, sz, sz, vp, vp, vp, vp, vp, vp, f32]
        L.orc_ternary_matvec.argtypes = [sz, sz, vp, vp, vp, vp, vp, vp]
        L.orc_ternary_matbatch.argtypes = [sz, sz, sz, vp, vp, vp, vp, vp, vp]
        L.orc_bf16_matvec.argtypes = [sz, sz, vp, vp, vp]
        L.orc_f32_matvec.argtypes = [sz, sz, vp, vp, vp]
        L.orc_swiglu.argtypes = [sz, vp, vp, f32, i32, vp]
        L.orc_axpy.argtypes = [sz, f32, vp, vp]
        L.orc_rms_norm.argtypes = [sz, vp, vp, f32, vp]
        L.orc_nvfp4_expert.argtypes = [sz, sz, vp, vp, vp, vp, vp, vp]
        L.orc_ternary_expert.argtypes = [sz, sz, vp, vp, vp, vp, f32, vp, vp, vp]
        L.orc_route.argtypes = [sz, sz, sz, vp, vp, i32, vp, vp, vp, vp]
        L.orc_e8m0_to_f32.restype = f32
        L.orc_e8m0_to_f32.argtypes = [C.c_uint8]
        L.orc_mxfp4_matvec.argtypes = [sz, sz, vp, vp, vp, vp]
        L.orc_mxfp8_matvec.argtypes = [sz, sz, vp, vp, vp, vp]
        L.orc_compress_ternary_b64.argtypes = [sz, sz, vp, vp, f32, C.c_uint64, vp, vp, vp, vp, vp, vp,
                                               vp, vp]
        L.orc_compress_ternary_b64.restype = C.c_int
        L.orc_mx_expert.argtypes = [i32, sz, sz, vp, vp, vp, vp, vp]
        L.orc_combine.argtypes = [sz, sz, sz, vp, vp, vp]
        L.orc_derive.restype = u64
        L.orc_derive.argtypes = [u64, u64]
        L.orc_gen_nvfp4.argtypes = [u64, sz, sz, vp, vp]
        L.orc_gen_ternary.argtypes = [u64, sz, sz, vp, vp]
        L.orc_gen_core.argtypes = [u64, sz, sz, sz, vp, vp, vp, vp]
        L.orc_gen_normal.argtypes = [u64, sz, f32, vp]
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


# ----------------------------------------------------------------- decoders
def e4m3_to_f32(b: int) -> float:
    return lib().orc_e4m3_to_f32(b)


def e2m1_to_f32(n: int) -> float:
    return lib().orc_e2m1_to_f32(n)


def f32_to_e4m3(v: float) -> int:
    return lib().orc_f32_to_e4m3(v)


def e4m3_table() -> np.ndarray:
    return np.array([e4m3_to_f32(b) for b in range(256)], dtype=np.float32)


def e8m0_to_f32(b: int) -> float:
    return float(lib().orc_e8m0_to_f32(b))


def mxfp4_matvec(w, s, x, rows, cols) -> np.ndarray:
    """F:2700-2746: E2M1 [rows, cols/2] with E8M0 scales per 32 columns."""
    out = np.empty(rows, dtype=np.float32)
    lib().orc_mxfp4_matvec(rows, cols, _p(w), _p(s), _p(np.ascontiguousarray(x, np.float32)), _p(out))
    return out


def mxfp8_matvec(w, s, x, rows, cols) -> np.ndarray:
    """F:1940-1984: E4M3 [rows, cols] with E8M0 scales per 32 x 32 block."""
    out = np.empty(rows, dtype=np.float32)
    lib().orc_mxfp8_matvec(rows, cols, _p(w), _p(s), _p(np.ascontiguousarray(x, np.float32)), _p(out))
    return out


def compress_ternary_b64(w: np.ndarray, s: np.ndarray, gs: float, rows: int, cols: int,
                         seed: int) -> dict:
    """The reference's NVFP4 -> 1.58-bit block-64 ternary + rank-16 Q8 core
    compressor (F:10377-10645): packed [rows, cols/4], row_scales [rows],
    block_scales [rows, cols/64], core_b [rows, 16] int8, core_b_sc [16],
    core_a [16, cols] int8, core_a_sc [16], and the f64 error sums
    orig_frob_sq, ternary_err_sq, jepa_err_sq."""
    out = dict(packed=np.empty(rows * cols // 4, np.uint8), row_scales=np.empty(rows, np.float32),
               block_scales=np.empty(rows * cols // 64, np.uint8), core_b=np.empty(rows * 16, np.int8),
               core_b_sc=np.empty(16, np.float32), core_a=np.empty(16 * cols, np.int8),
               core_a_sc=np.empty(16, np.float32))
    st = np.empty(3, np.float64)
    rc = lib().orc_compress_ternary_b64(rows, cols, _p(np.ascontiguousarray(w)), _p(np.ascontiguousarray(s)),
                                        float(gs), int(seed) & (2**64 - 1), _p(out["packed"]),
                                        _p(out["row_scales"]), _p(out["block_scales"]), _p(out["core_b"]),
                                        _p(out["core_b_sc"]), _p(out["core_a"]), _p(out["core_a_sc"]), _p(st))
    if rc:
        raise ValueError("compress_ternary_b64: cols must be a positive multiple of 64")
    out.update(orig_frob_sq=float(st[0]), ternary_err_sq=float(st[1]), jepa_err_sq=float(st[2]))
    return out


def dequant_nvfp4(w: np.ndarray, s: np.ndarray, gs: float, rows: int, cols: int) -> np.ndarray:
    """Decoded weight values e2m1 * e4m3 (F:2341-2351), as f32 [rows, cols]
    (the per-tensor scale is applied separately by the reference, F:2356)."""
    lut = np.array([e2m1_to_f32(i) for i in range(16)], dtype=np.float32)
    tab = e4m3_table()
    w = w.reshape(rows, cols // 2)
    vals = np.empty((rows, cols), dtype=np.float32)
    vals[:, 0::2] = lut[w & 0x0F]
    vals[:, 1::2] = lut[w >> 4]
    sc = np.repeat(tab[s.reshape(rows, cols // 16)], 16, axis=1)
    return (vals * sc).astype(np.float32)


def dequant_ternary(p: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """Decoded ternary codes {-1,0,+1} as f32 [rows, cols] (F:2566, F:2609-2618)."""
    lut = np.array([-1.0, 0.0, 1.0, 0.0], dtype=np.float32)
    p = p.reshape(rows, cols // 4)
    out = np.empty((rows, cols), dtype=np.float32)
    for i in range(4):
        out[:, i::4] = lut[(p >> (2 * i)) & 3]
    return out


# ------------------------------------------------------------------ matvecs
def nvfp4_matvec(w, s, gs, x, rows, cols) -> np.ndarray:
    out = np.zeros(rows, dtype=np.float32)
    lib().orc_nvfp4_matvec(rows, cols, _p(w), _p(s), float(gs), _p(x), _p(out))
    return out


def nvfp4_matbatch(w, s, gs, xb, rows, cols, seq) -> np.ndarray:
    out = np.zeros((seq, rows), dtype=np.float32)
    lib().orc_nvfp4_matbatch(rows, cols, seq, _p(w), _p(s), float(gs), _p(xb), _p(out))
    return out


class _Core(C.Structure):
    _fields_ = [("a", C.c_void_p), ("a_sc", C.c_void_p), ("b", C.c_void_p),
                ("b_sc", C.c_void_p), ("rank", C.c_size_t)]


@dataclass
class Core:
    """Rank-16 Q8 core: a = V^T [rank, cols] i8, b = U [rows, rank] i8 (F:2417-2420)."""
    a: np.ndarray
    a_sc: np.ndarray
    b: np.ndarray
    b_sc: np.ndarray

    @property
    def rank(self) -> int:
        return int(self.a_sc.shape[0])

    def cstruct(self) -> _Core:
        return _Core(_p(self.a), _p(self.a_sc), _p(self.b), _p(self.b_sc), self.rank)


def rank16_apply_add(core: Core, x, y, rows, cols, scale=1.0) -> None:
    lib().orc_rank16_apply_add(rows, cols, core.rank, _p(core.a), _p(core.a_sc), _p(core.b),
                               _p(core.b_sc), _p(x), _p(y), float(scale))


def ternary_matvec(p, rs, x, rows, cols, core: Core | None = None, bs=None) -> np.ndarray:
    out = np.zeros(rows, dtype=np.float32)
    cs = core.cstruct() if core is not None else None
    lib().orc_ternary_matvec(rows, cols, _p(p), _p(rs), _p(bs),
                             C.addressof(cs) if cs is not None else None, _p(x), _p(out))
    return out


def ternary_matbatch(p, rs, xb, rows, cols, seq, core: Core | None = None, bs=None):
    out = np.zeros((seq, rows), dtype=np.float32)
    cs = core.cstruct() if core is not None else None
    lib().orc_ternary_matbatch(rows, cols, seq, _p(p), _p(rs), _p(bs),
                               C.addressof(cs) if cs is not None else None, _p(xb), _p(out))
    return out


def f32_matvec(w, x, rows, cols) -> np.ndarray:
    out = np.zeros(rows, dtype=np.float32)
    lib().orc_f32_matvec(rows, cols, _p(w), _p(x), _p(out))
    return out


def bf16_matvec(w_u16, x, rows, cols) -> np.ndarray:
    out = np.zeros(rows, dtype=np.float32)
    lib().orc_bf16_matvec(rows, cols, _p(w_u16), _p(x), _p(out))
    return out


def swiglu(g, u, proj_scale=1.0, scaled=False) -> np.ndarray:
    h = np.zeros_like(g, dtype=np.float32)
    lib().orc_swiglu(g.size, _p(g), _p(u), float(proj_scale), int(scaled), _p(h))
    return h


def rms_norm(x, w, eps=1e-20) -> np.ndarray:
    """flash1017.rs:4880-4891, row by row for 2-D x."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    out = np.empty_like(x)
    for r in range(x.shape[0] if x.ndim == 2 else 1):
        xr = x[r] if x.ndim == 2 else x
        orow = out[r] if x.ndim == 2 else out
        lib().orc_rms_norm(xr.size, _p(np.ascontiguousarray(xr)), _p(w), float(eps),
                           orow.ctypes.data)
    return out


def axpy(dst, scale, src) -> None:
    lib().orc_axpy(dst.size, float(scale), _p(src), _p(dst))


# ------------------------------------------------------------ generators
def derive(parent: int, v: int) -> int:
    return int(lib().orc_derive(C.c_uint64(parent & (2**64 - 1)), C.c_uint64(v)))


def key(*path: int) -> int:
    """Stream key for a tensor: derive(derive(derive(ROOT, a), b), ...)."""
    k = 0x464C415348313031  # "FLASH101"
    for v in path:
        k = derive(k, int(v))
    return k


def gen_nvfp4(k: int, rows: int, cols: int):
    w = np.empty(rows * cols // 2, dtype=np.uint8)
    s = np.empty(rows * cols // 16, dtype=np.uint8)
    lib().orc_gen_nvfp4(C.c_uint64(k), rows, cols, _p(w), _p(s))
    return w, s


def gen_ternary(k: int, rows: int, cols: int):
    p = np.empty(rows * cols // 4, dtype=np.uint8)
    rs = np.empty(rows, dtype=np.float32)
    lib().orc_gen_ternary(C.c_uint64(k), rows, cols, _p(p), _p(rs))
    return p, rs


def gen_core(k: int, rows: int, cols: int, rank: int = 16) -> Core:
    a = np.empty(rank * cols, dtype=np.int8)
    b = np.empty(rows * rank, dtype=np.int8)
    a_sc = np.empty(rank, dtype=np.float32)
    b_sc = np.empty(rank, dtype=np.float32)
    lib().orc_gen_core(C.c_uint64(k), rows, cols, rank, _p(a), _p(a_sc), _p(b), _p(b_sc))
    return Core(a, a_sc, b, b_sc)


def gen_normal(k: int, n: int, stdev: float = 1.0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().orc_gen_normal(C.c_uint64(k), n, float(stdev), _p(out))
    return out


# ------------------------------------------------------------- experts / MoE
@dataclass
class Nvfp4Expert:
    """gate (w1), up (w3), down (w2) NVFP4 matrices of one SwiGLU expert."""
    inter: int
    hidden: int
    w: tuple  # (w1, w3, w2) packed
    s: tuple  # scales
    gs: tuple  # per-tensor scales

    def forward(self, x: np.ndarray) -> np.ndarray:
        y = np.zeros(self.hidden, dtype=np.float32)
        scratch = np.zeros(3 * self.inter, dtype=np.float32)
        wp = (C.c_void_p * 3)(*[_p(a) for a in self.w])
        sp = (C.c_void_p * 3)(*[_p(a) for a in self.s])
        gs = np.array(self.gs, dtype=np.float32)
        lib().orc_nvfp4_expert(self.inter, self.hidden, wp, sp, _p(gs), _p(x), _p(y),
                               _p(scratch))
        return y

    def nbytes(self) -> int:
        return sum(a.nbytes for a in self.w) + sum(a.nbytes for a in self.s) + 12


@dataclass
class MxExpert:
    """gate (w1), up (w3), down (w2) of an MXFP4 (fmt 3: the MTP routed
    experts, F:9103-9158) or MXFP8 (fmt 4: the shared expert, F:9132-9142)
    SwiGLU expert."""
    fmt: int
    inter: int
    hidden: int
    w: tuple
    s: tuple

    def forward(self, x: np.ndarray) -> np.ndarray:
        y = np.zeros(self.hidden, dtype=np.float32)
        scratch = np.zeros(3 * self.inter, dtype=np.float32)
        wp = (C.c_void_p * 3)(*[_p(a) for a in self.w])
        sp = (C.c_void_p * 3)(*[_p(a) for a in self.s])
        lib().orc_mx_expert(self.fmt, self.inter, self.hidden, wp, sp,
                            _p(np.ascontiguousarray(x, np.float32)), _p(y), _p(scratch))
        return y


@dataclass
class TernaryExpert:
    inter: int
    hidden: int
    p: tuple  # (w1, w3, w2) packed codes
    rs: tuple  # row scales
    cores: tuple | None  # (Core, Core, Core) or None
    proj_scale: float = 1.0
    bs: tuple | None = None  # (w1, w3, w2) U8 block scales [rows, cols/64], or None

    def forward(self, x: np.ndarray) -> np.ndarray:
        y = np.zeros(self.hidden, dtype=np.float32)
        scratch = np.zeros(3 * self.inter, dtype=np.float32)
        pp = (C.c_void_p * 3)(*[_p(a) for a in self.p])
        rp = (C.c_void_p * 3)(*[_p(a) for a in self.rs])
        cores = None
        if self.cores is not None:
            cores = (_Core * 3)(*[c.cstruct() for c in self.cores])
        bp = None
        if self.bs is not None:
            bp = (C.c_void_p * 3)(*[_p(a) for a in self.bs])
        lib().orc_ternary_expert(self.inter, self.hidden, pp, rp,
                                 C.addressof(cores) if cores is not None else None,
                                 bp, float(self.proj_scale), _p(x), _p(y), _p(scratch))
        return y

    def nbytes(self) -> int:
        n = sum(a.nbytes for a in self.p) + sum(a.nbytes for a in self.rs)
        if self.bs is not None:
            n += sum(a.nbytes for a in self.bs)
        if self.cores is not None:
            for c in self.cores:
                n += c.a.nbytes + c.b.nbytes + c.a_sc.nbytes + c.b_sc.nbytes
        return n


# Tensor tags used in generator key paths (shared with the device generator).
TAG_W1, TAG_W3, TAG_W2, TAG_ROUTER, TAG_X, TAG_BIAS = 1, 3, 2, 10, 11, 12


def gen_nvfp4_expert(seed: int, layer: int, expert: int, inter: int, hidden: int,
                     gs: float = 1.0) -> Nvfp4Expert:
    w1, s1 = gen_nvfp4(key(seed, layer, expert, TAG_W1), inter, hidden)
    w3, s3 = gen_nvfp4(key(seed, layer, expert, TAG_W3), inter, hidden)
    w2, s2 = gen_nvfp4(key(seed, layer, expert, TAG_W2), hidden, inter)
    return Nvfp4Expert(inter, hidden, (w1, w3, w2), (s1, s3, s2), (gs, gs, gs))


def gen_ternary_expert(seed: int, layer: int, expert: int, inter: int, hidden: int,
                       with_core: bool = True, proj_scale: float = 1.0) -> TernaryExpert:
    p1, r1 = gen_ternary(key(seed, layer, expert, TAG_W1), inter, hidden)
    p3, r3 = gen_ternary(key(seed, layer, expert, TAG_W3), inter, hidden)
    p2, r2 = gen_ternary(key(seed, layer, expert, TAG_W2), hidden, inter)
    cores = None
    if with_core:
        cores = (gen_core(key(seed, layer, expert, TAG_W1), inter, hidden),
                 gen_core(key(seed, layer, expert, TAG_W3), inter, hidden),
                 gen_core(key(seed, layer, expert, TAG_W2), hidden, inter))
    return TernaryExpert(inter, hidden, (p1, p3, p2), (r1, r3, r2), cores, proj_scale)


def gen_router(seed: int, layer: int, n_exp: int, hidden: int, stdev: float = 0.02):
    return gen_normal(key(seed, layer, 0, TAG_ROUTER), n_exp * hidden, stdev).reshape(
        n_exp, hidden)


def gen_hidden(seed: int, n_tok: int, hidden: int) -> np.ndarray:
    return gen_normal(key(seed, 0, 0, TAG_X), n_tok * hidden, 1.0).reshape(n_tok, hidden)


def route(logits: np.ndarray, top_k: int = 6, bias=None, score_fn: int = 1):
    """Router + top-k (F:7277-7376).  score_fn 0 = reference sqrt(softplus)+bias,
    weights score*1.5/sum; 1 = sigmoid, weights score/sum.  Returns
    (idx, weight, score, biased) each [n_tok, top_k]."""
    n_tok, n_exp = logits.shape
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    idx = np.zeros((n_tok, top_k), dtype=np.int32)
    wt = np.zeros((n_tok, top_k), dtype=np.float32)
    sc = np.zeros((n_tok, top_k), dtype=np.float32)
    bi = np.zeros((n_tok, top_k), dtype=np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    lib().orc_route(n_tok, n_exp, top_k, _p(logits), _p(b), int(score_fn), _p(idx), _p(wt),
                    _p(sc), _p(bi))
    return idx, wt, sc, bi


def topk_agrees(idx, ref_idx, ref_biased_sorted, tol=1e-5):
    """True per token when the selected set equals the reference's, or the
    reference's k-th and (k+1)-th biased scores are within `tol` (a near-tie,
    where a different summation order may legitimately pick either)."""
    ok = []
    for t in range(idx.shape[0]):
        same = set(idx[t].tolist()) == set(ref_idx[t].tolist())
        k = idx.shape[1]
        tie = abs(ref_biased_sorted[t, k - 1] - ref_biased_sorted[t, k]) <= tol
        ok.append(same or tie)
    return np.array(ok)


def biased_sorted(logits, k, bias=None, score_fn=1):
    """The k+1 largest biased scores per token (for topk_agrees)."""
    _, _, _, bi = route(logits, k + 1, bias, score_fn)
    return bi


def router_logits(wr: np.ndarray, x: np.ndarray) -> np.ndarray:
    n_exp, hidden = wr.shape
    xs = np.atleast_2d(x)
    out = np.zeros((xs.shape[0], n_exp), dtype=np.float32)
    for t in range(xs.shape[0]):
        out[t] = f32_matvec(wr, np.ascontiguousarray(xs[t]), n_exp, hidden)
    return out


def moe_layer(experts, wr, x, top_k=6, bias=None, score_fn=1, norm_w=None, norm_eps=1e-20):
    """Decode MoE layer, reference order (F:7637 ffn_norm when norm_w is given,
    F:7277-7376 routing, F:7521-7566 combine, no shared expert).  experts: list
    of expert objects with .forward(x).  Returns (out [n_tok, hidden], idx, wt)."""
    if norm_w is not None:
        x = rms_norm(x, norm_w, norm_eps)
    logits = router_logits(wr, x)
    idx, wt, _, _ = route(logits, top_k, bias, score_fn)
    n_tok, hidden = x.shape
    out = np.zeros((n_tok, hidden), dtype=np.float32)
    for t in range(n_tok):
        xt = np.ascontiguousarray(x[t])
        for k in range(top_k):
            y = experts[idx[t, k]].forward(xt)
            axpy(out[t], wt[t, k], y)
    return out, idx, wt


# ----------------------------------------------------------- comparisons
def max_rel_err(y: np.ndarray, ref: np.ndarray) -> float:
    """max|y - ref| / max|ref| (the tolerance metric of the configs)."""
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    den = np.max(np.abs(ref))
    return float(np.max(np.abs(y - ref)) / den) if den > 0 else float(np.max(np.abs(y)))


def cosine(y: np.ndarray, ref: np.ndarray) -> float:
    y = np.asarray(y, dtype=np.float64).ravel()
    ref = np.asarray(ref, dtype=np.float64).ravel()
    ny, nr = np.linalg.norm(y), np.linalg.norm(ref)
    if ny == 0 and nr == 0:
        return 1.0
    return float(np.dot(y, ref) / (ny * nr))


REL_TOL = 1e-3
COS_TOL = 0.99999


def assert_close(y, ref, rel=REL_TOL, cos=COS_TOL, what=""):
    e, c = max_rel_err(y, ref), cosine(y, ref)
    assert e <= rel and c >= cos, f"{what}: max_rel_err={e:.3e} (tol {rel}) cosine={c:.8f} (tol {cos})"
    return e, c
