"""ctypes binding of libffn_b200.so for Python callers (tests, bench, smoke).

The library's C-ABI (include/ffn_b200.h, include/merkaba_hw_addon.h) is the
product; this module only marshals torch CUDA tensors into it.  PyTorch here
is plumbing: device memory, streams and torch.distributed.  There is no Python
or CPU compute path: every function below runs a CUDA kernel of the library,
and using it without the built library raises.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libffn_b200.so")

FMT_NVFP4, FMT_TERNARY, FMT_MXFP4, FMT_MXFP8 = 0, 1, 2, 3
SCORE_REF, SCORE_SIGMOID = 0, 1
ROUTER_EXACT, ROUTER_TENSOR = 0, 1
PATH_AUTO, PATH_GEMV, PATH_GROUPED, PATH_FP4 = 0, 1, 2, 3
GROUPED_MIN_PAIRS = 48
ERRORS = {0: "OK", -1: "EINVAL", -2: "ECUDA", -3: "ENOSPC", -4: "ENCCL", -5: "EUNSUP"}

# Symbols the public headers declare (checked by the CPU test suite).
EXPORTS = [
    "merkaba_hardware_addon_v1",
    "gx10_rust_nvfp4_mlp_accum", "gx10_rust_ternary_158_mlp_accum",
    "gx10_rust_nvfp4_mlp_batch", "gx10_rust_ternary_158_mlp_batch",
    "gx10_rust_register_shard_bounds", "gx10_rust_register_host_range",
    "ffn_b200_version", "ffn_b200_last_error", "ffn_b200_launch_count", "ffn_b200_set_device",
    "ffn_b200_matvec_ws_bytes", "ffn_b200_nvfp4_matvec", "ffn_b200_ternary_matvec",
    "ffn_b200_expert_ws_bytes", "ffn_b200_expert_forward", "ffn_b200_expert_forward_noalloc",
    "ffn_b200_moe_ws_bytes", "ffn_b200_moe_layer",
    "ffn_b200_key", "ffn_b200_gen_nvfp4", "ffn_b200_gen_ternary", "ffn_b200_gen_core",
    "ffn_b200_gen_normal", "ffn_b200_dequant_nvfp4", "ffn_b200_dequant_ternary",
    "ffn_b200_set_batch_input", "ffn_b200_release_host_ranges", "ffn_b200_host_cache_bytes",
    "ffn_b200_profile_enable", "ffn_b200_profile_kinds", "ffn_b200_profile_read",
    "ffn_b200_ep_handle_bytes", "ffn_b200_ep_create", "ffn_b200_ep_connect", "ffn_b200_ep_part",
    "ffn_b200_ep_allreduce", "ffn_b200_ep_error", "ffn_b200_ep_destroy",
    "ffn_b200_mxfp4_matvec", "gx10_rust_mxfp4_matvec", "gx10_rust_mxfp4_mlp_accum",
    "ffn_b200_mxfp8_matvec", "gx10_rust_mxfp8_mlp_accum", "gx10_rust_mxfp8_mlp_batch",
    "ffn_b200_st_open", "ffn_b200_st_close", "ffn_b200_st_count", "ffn_b200_st_name",
    "ffn_b200_st_find", "ffn_b200_st_expert_bytes", "ffn_b200_st_load_expert",
    "ffn_b200_compress_ws_bytes", "ffn_b200_compress_ternary_b64",
    "ffn_b200_quantize_nvfp4x4", "ffn_b200_ep_moe_layer", "ffn_b200_set_host_cache_budget",
    "ffn_b200_topk", "ffn_b200_quantize_nvfp4_terms", "ffn_b200_fp4_pack_bytes",
    "ffn_b200_pack_nvfp4_expert",
]

# Kernel kinds of ffn_b200_profile_read (FFN_B200_K_*).
K_XPREP, K_ROUTER, K_TOPK, K_GROUP, K_GATEUP_NVFP4, K_DOWN_NVFP4 = 0, 1, 2, 3, 4, 5
K_GATEUP_TERNARY, K_DOWN_TERNARY, K_COREZ, K_COMBINE, K_MATVEC, K_OTHER = 6, 7, 8, 9, 10, 11
K_GEMM_GATEUP, K_GEMM_DOWN, K_QUANT, K_FP4_GATEUP, K_FP4_DOWN = 12, 13, 14, 15, 16
K_NAMES = ["xprep", "router", "topk", "group", "gateup_nvfp4", "down_nvfp4", "gateup_ternary",
           "down_ternary", "corez", "combine", "matvec", "other", "gemm_gateup", "gemm_down",
           "quant", "fp4_gateup", "fp4_down"]


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE, "-j8"], check=True)
    return LIB_PATH


class FfnError(RuntimeError):
    pass


# ------------------------------------------------------------ C structs
class NvMat(C.Structure):
    _fields_ = [("w", C.c_void_p), ("s", C.c_void_p), ("gs", C.c_float),
                ("reserved", C.c_uint32)]


class TnMat(C.Structure):
    _fields_ = [("p", C.c_void_p), ("rs", C.c_void_p), ("core_a", C.c_void_p),
                ("core_a_sc", C.c_void_p), ("core_b", C.c_void_p), ("core_b_sc", C.c_void_p),
                ("bs", C.c_void_p)]


class Expert(C.Structure):
    _fields_ = [("format", C.c_int32), ("proj_scale", C.c_float), ("nv", NvMat * 3),
                ("tn", TnMat * 3), ("fp4_gu", C.c_void_p), ("fp4_dn", C.c_void_p)]


class MoeDesc(C.Structure):
    _fields_ = [("hidden", C.c_size_t), ("inter", C.c_size_t), ("n_experts", C.c_size_t),
                ("top_k", C.c_size_t), ("experts", C.c_void_p), ("router_w", C.c_void_p),
                ("router_bias", C.c_void_p), ("score_fn", C.c_int32),
                ("router_mode", C.c_int32), ("expert_begin", C.c_int32),
                ("expert_end", C.c_int32), ("has_nvfp4", C.c_int32),
                ("has_ternary", C.c_int32), ("norm_w", C.c_void_p), ("norm_eps", C.c_float),
                ("path", C.c_int32), ("has_mxfp4", C.c_int32), ("fp4_packed", C.c_int32)]


assert C.sizeof(Expert) == 264, C.sizeof(Expert)

_lib = None


def lib() -> C.CDLL:
    """The loaded library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FfnError(f"{LIB_PATH} is missing: build it with `make -C {HERE}` "
                           "(or __graft_entry__.build())")
        L = C.CDLL(LIB_PATH)
        sz, vp, f32, i32, u64 = C.c_size_t, C.c_void_p, C.c_float, C.c_int, C.c_uint64
        L.ffn_b200_version.restype = C.c_char_p
        L.ffn_b200_last_error.restype = C.c_char_p
        L.ffn_b200_launch_count.restype = u64
        L.ffn_b200_set_device.argtypes = [i32]
        L.ffn_b200_matvec_ws_bytes.restype = sz
        L.ffn_b200_matvec_ws_bytes.argtypes = [sz, sz]
        L.ffn_b200_nvfp4_matvec.argtypes = [sz, sz, sz, C.POINTER(NvMat), vp, vp, vp, sz, vp]
        L.ffn_b200_ternary_matvec.argtypes = [sz, sz, sz, C.POINTER(TnMat), vp, vp, vp, sz, vp]
        L.ffn_b200_mxfp4_matvec.argtypes = [sz, sz, sz, C.POINTER(NvMat), vp, vp, vp, sz, vp]
        L.ffn_b200_quantize_nvfp4x4.argtypes = [sz, sz, vp, sz, vp, vp, vp, vp]
        L.ffn_b200_topk.argtypes = [sz, sz, sz, C.c_int32, vp, sz, vp, vp, vp, vp]
        L.ffn_b200_quantize_nvfp4_terms.argtypes = [sz, sz, sz, vp, sz, vp, vp, vp, vp]
        L.ffn_b200_fp4_pack_bytes.restype = sz
        L.ffn_b200_fp4_pack_bytes.argtypes = [sz, sz, C.c_int]
        L.ffn_b200_pack_nvfp4_expert.argtypes = [sz, sz, C.POINTER(Expert), vp, vp, vp]
        L.gx10_rust_mxfp4_matvec.argtypes = [sz, sz, vp, vp, vp, vp]
        L.gx10_rust_mxfp4_matvec.restype = C.c_bool
        L.gx10_rust_mxfp4_mlp_accum.argtypes = [sz, sz, vp, vp, vp, vp, vp, vp, vp, vp, f32,
                                                C.c_bool, C.c_bool]
        L.gx10_rust_mxfp4_mlp_accum.restype = C.c_bool
        L.ffn_b200_mxfp8_matvec.argtypes = [sz, sz, sz, C.POINTER(NvMat), vp, vp, vp, sz, vp]
        L.gx10_rust_mxfp8_mlp_accum.argtypes = [sz, sz, vp, vp, vp, vp, vp, vp, vp, vp, f32,
                                                C.c_bool, C.c_bool]
        L.gx10_rust_mxfp8_mlp_accum.restype = C.c_bool
        L.gx10_rust_mxfp8_mlp_batch.argtypes = [sz, sz, sz, vp, vp, vp, vp, vp, vp, vp, sz, vp,
                                                C.c_bool]
        L.gx10_rust_mxfp8_mlp_batch.restype = C.c_bool
        L.gx10_rust_nvfp4_mlp_accum.argtypes = [sz, sz, vp, vp, f32, vp, vp, f32, vp, vp, f32, vp,
                                                vp, f32, C.c_bool, C.c_bool]
        L.gx10_rust_nvfp4_mlp_accum.restype = C.c_bool
        L.gx10_rust_ternary_158_mlp_accum.argtypes = [sz, sz, vp, vp, vp, vp, vp, vp, f32, vp, vp,
                                                      f32, C.c_bool, C.c_bool]
        L.gx10_rust_ternary_158_mlp_accum.restype = C.c_bool
        L.gx10_rust_nvfp4_mlp_batch.argtypes = [sz, sz, sz, vp, vp, f32, vp, vp, f32, vp, vp, f32,
                                                sz, vp, vp, sz, vp, C.c_bool]
        L.gx10_rust_nvfp4_mlp_batch.restype = C.c_bool
        L.gx10_rust_ternary_158_mlp_batch.argtypes = [sz, sz, sz, vp, vp, vp, vp, vp, vp, f32, sz,
                                                      vp, vp, sz, vp, C.c_bool]
        L.gx10_rust_ternary_158_mlp_batch.restype = C.c_bool
        L.ffn_b200_compress_ws_bytes.restype = sz
        L.ffn_b200_compress_ws_bytes.argtypes = [sz, sz]
        L.ffn_b200_compress_ternary_b64.argtypes = [sz, sz, vp, vp, f32, u64, vp, vp, vp, vp, vp, vp,
                                                    vp, vp, sz, vp]
        L.ffn_b200_expert_ws_bytes.restype = sz
        L.ffn_b200_expert_ws_bytes.argtypes = [sz, sz, sz]
        L.ffn_b200_expert_forward.argtypes = [sz, sz, sz, C.POINTER(Expert), vp, vp, f32, i32,
                                              vp, sz, vp]
        L.ffn_b200_expert_forward_noalloc.argtypes = [sz, sz, sz, C.POINTER(Expert), vp, vp, f32,
                                                      i32, vp]
        L.ffn_b200_moe_ws_bytes.restype = sz
        L.ffn_b200_moe_ws_bytes.argtypes = [C.POINTER(MoeDesc), sz]
        L.ffn_b200_moe_layer.argtypes = [C.POINTER(MoeDesc), sz, vp, vp, vp, vp, vp, vp, sz, vp]
        L.ffn_b200_key.restype = u64
        L.ffn_b200_key.argtypes = [u64, u64]
        L.ffn_b200_gen_nvfp4.argtypes = [u64, sz, sz, vp, vp, vp]
        L.ffn_b200_gen_ternary.argtypes = [u64, sz, sz, vp, vp, vp]
        L.ffn_b200_gen_core.argtypes = [u64, sz, sz, vp, vp, vp, vp, vp]
        L.ffn_b200_gen_normal.argtypes = [u64, sz, f32, vp, vp]
        L.ffn_b200_dequant_nvfp4.argtypes = [sz, sz, vp, vp, vp, vp]
        L.ffn_b200_dequant_ternary.argtypes = [sz, sz, vp, vp, vp]
        L.ffn_b200_set_batch_input.argtypes = [vp, sz, sz]
        L.ffn_b200_host_cache_bytes.restype = sz
        L.ffn_b200_set_host_cache_budget.argtypes = [sz]
        L.merkaba_hardware_addon_v1.restype = vp
        L.ffn_b200_profile_enable.argtypes = [i32]
        L.ffn_b200_profile_kinds.argtypes = [C.c_uint32]
        L.ffn_b200_ep_handle_bytes.restype = sz
        L.ffn_b200_ep_create.argtypes = [i32, i32, sz, sz, vp, C.POINTER(vp)]
        L.ffn_b200_ep_connect.argtypes = [vp, vp]
        L.ffn_b200_ep_part.argtypes = [vp]
        L.ffn_b200_ep_part.restype = vp
        L.ffn_b200_ep_allreduce.argtypes = [vp, sz, vp, vp, vp]
        L.ffn_b200_ep_moe_layer.argtypes = [vp, C.POINTER(MoeDesc), sz, vp, vp, vp, vp, vp, vp, sz, vp]
        L.ffn_b200_ep_error.argtypes = [vp, C.POINTER(C.c_int)]
        L.ffn_b200_ep_destroy.argtypes = [vp]
        L.ffn_b200_profile_read.argtypes = [i32, C.POINTER(C.c_double), C.POINTER(C.c_uint64)]
        L.ffn_b200_st_open.argtypes = [C.c_char_p, C.POINTER(vp)]
        L.ffn_b200_st_close.argtypes = [vp]
        L.ffn_b200_st_count.argtypes = [vp]
        L.ffn_b200_st_count.restype = sz
        L.ffn_b200_st_name.argtypes = [vp, sz]
        L.ffn_b200_st_name.restype = C.c_char_p
        L.ffn_b200_st_find.argtypes = [vp, C.c_char_p, C.POINTER(C.c_char_p), C.POINTER(C.c_int64),
                                       C.POINTER(C.c_int), C.POINTER(vp), C.POINTER(sz)]
        L.ffn_b200_st_expert_bytes.argtypes = [vp, C.c_char_p, sz, sz, C.POINTER(C.c_int), C.POINTER(sz)]
        L.ffn_b200_st_load_expert.argtypes = [vp, C.c_char_p, sz, sz, vp, sz, vp, C.POINTER(Expert)]
        _lib = L
    return _lib


def check(rc: int, what: str = "") -> None:
    if rc != 0:
        msg = lib().ffn_b200_last_error().decode(errors="replace")
        raise FfnError(f"{what}: {ERRORS.get(rc, rc)}: {msg}")


def launch_count() -> int:
    return int(lib().ffn_b200_launch_count())


def profile_enable(on: bool) -> None:
    """Start (True: clears the totals) or stop per-kernel event timing."""
    check(lib().ffn_b200_profile_enable(int(on)), "profile_enable")


def profile_kinds(names=None) -> None:
    """Time only these kernel kinds (names from K_NAMES; None: all)."""
    mask = 0xFFFFFFFF if names is None else sum(1 << K_NAMES.index(n) for n in names)
    check(lib().ffn_b200_profile_kinds(C.c_uint32(mask)), "profile_kinds")


def profile_read() -> dict:
    """{kernel kind name: (total device ms, launches)} since profile_enable(True)."""
    out = {}
    for k, name in enumerate(K_NAMES):
        ms, n = C.c_double(), C.c_uint64()
        check(lib().ffn_b200_profile_read(k, C.byref(ms), C.byref(n)), "profile_read")
        if n.value:
            out[name] = (ms.value, int(n.value))
    return out


def key(parent: int, v: int) -> int:
    return int(lib().ffn_b200_key(parent & (2**64 - 1), v))


def path_key(*path: int) -> int:
    """Same key path as the oracle's generator: derive(derive(ROOT, a), b)..."""
    k = 0x464C415348313031
    for v in path:
        k = key(k, int(v))
    return k


# ----------------------------------------------------------- torch glue
def _torch():
    import torch
    return torch


def _ptr(t):
    return None if t is None else t.data_ptr()


def _stream(stream=None):
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


class EpExchange:
    """NVLink peer exchange of the expert-parallel partial outputs (one
    process per GPU, torch.distributed initialised).  Every rank's MoE layer
    writes its partial into `part` (residual None); allreduce() then forms
    residual + sum of the parts on every rank."""

    def __init__(self, rank: int, world: int, max_tokens: int, hidden: int, group=None):
        import torch.distributed as dist
        torch = _torch()
        n = int(lib().ffn_b200_ep_handle_bytes())
        h = (C.c_uint8 * n)()
        ep = C.c_void_p()
        check(lib().ffn_b200_ep_create(rank, world, max_tokens, hidden, C.cast(h, C.c_void_p),
                                       C.byref(ep)), "ep_create")
        self.ep = ep
        mine = torch.tensor(list(bytes(h)), dtype=torch.uint8, device="cuda")
        allh = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(allh, mine, group=group)
        blob = b"".join(bytes(t.cpu().tolist()) for t in allh)
        buf = (C.c_uint8 * len(blob)).from_buffer_copy(blob)
        check(lib().ffn_b200_ep_connect(ep, C.cast(buf, C.c_void_p)), "ep_connect")
        ptr = int(lib().ffn_b200_ep_part(ep))

        class _View:  # zero-copy torch view of the shared part buffer
            __cuda_array_interface__ = {"shape": (max_tokens, hidden), "typestr": "<f4",
                                        "data": (ptr, False), "version": 2}

        self.part = torch.as_tensor(_View(), device=torch.device("cuda", torch.cuda.current_device()))
        self.hidden = hidden

    def allreduce(self, n_tok: int, residual, out, stream=None):
        check(lib().ffn_b200_ep_allreduce(self.ep, n_tok, _ptr(residual), _ptr(out),
                                          _stream(stream)), "ep_allreduce")
        return out

    def error(self) -> int:
        flag = C.c_int(0)
        check(lib().ffn_b200_ep_error(self.ep, C.byref(flag)), "ep_error")
        return int(flag.value)

    def close(self):
        if self.ep:
            lib().ffn_b200_ep_destroy(self.ep)
            self.ep = None


class Workspace:
    """Grow-only device scratch buffer handed to the library's ws arguments."""

    def __init__(self, device=None):
        self.buf = None
        self.device = device

    def get(self, nbytes: int):
        torch = _torch()
        if self.buf is None or self.buf.numel() < nbytes:
            self.buf = None
            self.buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8,
                                   device=self.device or "cuda")
        return self.buf


_ws = {}


def _default_ws(device) -> Workspace:
    d = str(device)
    if d not in _ws:
        _ws[d] = Workspace(device)
    return _ws[d]


# ----------------------------------------------------------- matrices
class Nvfp4Matrix:
    """NVFP4 matrix on the device: w [rows, cols/2] u8, s [rows, cols/16] u8, gs."""

    def __init__(self, w, s, gs: float, rows: int, cols: int):
        self.w, self.s, self.gs, self.rows, self.cols = w, s, float(gs), rows, cols

    def cstruct(self) -> NvMat:
        return NvMat(_ptr(self.w), _ptr(self.s), self.gs, 0)

    @classmethod
    def generate(cls, k: int, rows: int, cols: int, gs: float = 1.0, device="cuda", stream=None):
        torch = _torch()
        w = torch.empty(rows * cols // 2, dtype=torch.uint8, device=device)
        s = torch.empty(rows * cols // 16, dtype=torch.uint8, device=device)
        check(lib().ffn_b200_gen_nvfp4(k, rows, cols, _ptr(w), _ptr(s), _stream(stream)),
              "gen_nvfp4")
        return cls(w, s, gs, rows, cols)

    def matvec(self, x, out=None, stream=None):
        """out [seq, rows] = x [seq, cols] W^T (x float32 CUDA)."""
        torch = _torch()
        x = x.contiguous()
        seq = x.numel() // self.cols
        if out is None:
            out = torch.empty(seq, self.rows, dtype=torch.float32, device=x.device)
        ws = _default_ws(x.device).get(lib().ffn_b200_matvec_ws_bytes(seq, self.cols))
        m = self.cstruct()
        check(lib().ffn_b200_nvfp4_matvec(self.rows, self.cols, seq, C.byref(m), _ptr(x),
                                          _ptr(out), _ptr(ws), ws.numel(), _stream(stream)),
              "nvfp4_matvec")
        return out

    def dequant(self, stream=None):
        torch = _torch()
        out = torch.empty(self.rows, self.cols, dtype=torch.float32, device=self.w.device)
        check(lib().ffn_b200_dequant_nvfp4(self.rows, self.cols, _ptr(self.w), _ptr(self.s),
                                           _ptr(out), _stream(stream)), "dequant_nvfp4")
        return out

    def nbytes(self) -> int:
        return self.w.numel() + self.s.numel()


class Mxfp4Matrix(Nvfp4Matrix):
    """MXFP4 matrix on the device (FMT_MXFP4, flash1017.rs:2674-2747): w
    [rows, cols/2] E2M1 pairs, s [rows, cols/32] E8M0 block scales, gs a power
    of two 2^B taken out of the block scales (1 for the reference's tensors)."""

    @staticmethod
    def bias_for(s_bytes) -> float:
        """gs = 2^B with B = (largest finite block scale byte) - 140: the
        largest block decodes to 2^13 in f16 (E2M1 6 x 2^13 < 65504)."""
        torch = _torch()
        t = s_bytes if torch.is_tensor(s_bytes) else torch.as_tensor(s_bytes)
        t = t[t != 0xFF]
        return 2.0 ** (int(t.max().item()) - 140) if t.numel() else 1.0

    def matvec(self, x, out=None, stream=None):
        torch = _torch()
        x = x.contiguous()
        seq = x.numel() // self.cols
        if out is None:
            out = torch.empty(seq, self.rows, dtype=torch.float32, device=x.device)
        ws = _default_ws(x.device).get(lib().ffn_b200_matvec_ws_bytes(seq, self.cols))
        m = self.cstruct()
        check(lib().ffn_b200_mxfp4_matvec(self.rows, self.cols, seq, C.byref(m), _ptr(x),
                                          _ptr(out), _ptr(ws), ws.numel(), _stream(stream)),
              "mxfp4_matvec")
        return out

    def nbytes(self) -> int:
        return self.w.numel() + self.s.numel()


class Mxfp8Matrix(Nvfp4Matrix):
    """MXFP8 matrix on the device (FMT_MXFP8, the shared expert's format,
    flash1017.rs:1920-1984): w [rows, cols] E4M3, s [ceil(rows/32), cols/32]
    E8M0 scales of 32 x 32 blocks, gs a power of two 2^B taken out of them."""

    @staticmethod
    def bias_for(s_bytes) -> float:
        """gs = 2^B, B = (largest finite scale byte) - 134: the largest block
        decodes to 2^7 in f16 (E4M3 448 x 2^7 < 65504)."""
        torch = _torch()
        t = s_bytes if torch.is_tensor(s_bytes) else torch.as_tensor(s_bytes)
        t = t[t != 0xFF]
        return 2.0 ** (int(t.max().item()) - 134) if t.numel() else 1.0

    def matvec(self, x, out=None, stream=None):
        torch = _torch()
        x = x.contiguous()
        seq = x.numel() // self.cols
        if out is None:
            out = torch.empty(seq, self.rows, dtype=torch.float32, device=x.device)
        ws = _default_ws(x.device).get(lib().ffn_b200_matvec_ws_bytes(seq, self.cols))
        m = self.cstruct()
        check(lib().ffn_b200_mxfp8_matvec(self.rows, self.cols, seq, C.byref(m), _ptr(x),
                                          _ptr(out), _ptr(ws), ws.numel(), _stream(stream)),
              "mxfp8_matvec")
        return out

    def nbytes(self) -> int:
        return self.w.numel() + self.s.numel()


class TernaryMatrix:
    """Packed ternary matrix p [rows, cols/4] u8 + rs [rows] f32 (+ optional
    rank-16 core a [16, cols] i8, a_sc [16], b [rows, 16] i8, b_sc [16]; +
    optional U8 block scales bs [rows, cols/64])."""

    def __init__(self, p, rs, rows, cols, core=None, bs=None):
        self.p, self.rs, self.rows, self.cols, self.core = p, rs, rows, cols, core
        self.bs = bs

    def cstruct(self) -> TnMat:
        c = self.core
        return TnMat(_ptr(self.p), _ptr(self.rs), _ptr(c[0]) if c else None,
                     _ptr(c[1]) if c else None, _ptr(c[2]) if c else None,
                     _ptr(c[3]) if c else None, _ptr(self.bs) if self.bs is not None else None)

    @classmethod
    def generate(cls, k: int, rows: int, cols: int, with_core: bool = True, device="cuda",
                 stream=None):
        torch = _torch()
        p = torch.empty(rows * cols // 4, dtype=torch.uint8, device=device)
        rs = torch.empty(rows, dtype=torch.float32, device=device)
        check(lib().ffn_b200_gen_ternary(k, rows, cols, _ptr(p), _ptr(rs), _stream(stream)),
              "gen_ternary")
        core = None
        if with_core:
            a = torch.empty(16 * cols, dtype=torch.int8, device=device)
            a_sc = torch.empty(16, dtype=torch.float32, device=device)
            b = torch.empty(rows * 16, dtype=torch.int8, device=device)
            b_sc = torch.empty(16, dtype=torch.float32, device=device)
            check(lib().ffn_b200_gen_core(k, rows, cols, _ptr(a), _ptr(a_sc), _ptr(b), _ptr(b_sc),
                                          _stream(stream)), "gen_core")
            core = (a, a_sc, b, b_sc)
        return cls(p, rs, rows, cols, core)

    @classmethod
    def compress(cls, w, s, gs: float, rows: int, cols: int, seed: int, stream=None):
        """The 106 GB format's compressor (ffn_b200_compress_ternary_b64): an
        NVFP4 matrix (device w [rows, cols/2], s [rows, cols/16], per-tensor
        scale gs) -> ternary codes, row scales, U8 block-64 scales and the
        rank-16 Q8 core of the residual."""
        torch = _torch()
        dev = w.device
        p = torch.empty(rows * cols // 4, dtype=torch.uint8, device=dev)
        rs = torch.empty(rows, dtype=torch.float32, device=dev)
        bs = torch.empty(rows * cols // 64, dtype=torch.uint8, device=dev)
        a = torch.empty(16 * cols, dtype=torch.int8, device=dev)
        a_sc = torch.empty(16, dtype=torch.float32, device=dev)
        b = torch.empty(rows * 16, dtype=torch.int8, device=dev)
        b_sc = torch.empty(16, dtype=torch.float32, device=dev)
        ws = _default_ws(dev).get(lib().ffn_b200_compress_ws_bytes(rows, cols))
        check(lib().ffn_b200_compress_ternary_b64(rows, cols, _ptr(w), _ptr(s), float(gs),
                                                  int(seed) & (2**64 - 1), _ptr(p), _ptr(rs),
                                                  _ptr(bs), _ptr(b), _ptr(b_sc), _ptr(a), _ptr(a_sc),
                                                  _ptr(ws), ws.numel(), _stream(stream)),
              "compress_ternary_b64")
        return cls(p, rs, rows, cols, (a, a_sc, b, b_sc), bs)

    def matvec(self, x, out=None, stream=None):
        torch = _torch()
        x = x.contiguous()
        seq = x.numel() // self.cols
        if out is None:
            out = torch.empty(seq, self.rows, dtype=torch.float32, device=x.device)
        ws = _default_ws(x.device).get(lib().ffn_b200_matvec_ws_bytes(seq, self.cols))
        m = self.cstruct()
        check(lib().ffn_b200_ternary_matvec(self.rows, self.cols, seq, C.byref(m), _ptr(x),
                                            _ptr(out), _ptr(ws), ws.numel(), _stream(stream)),
              "ternary_matvec")
        return out

    def dequant(self, stream=None):
        torch = _torch()
        out = torch.empty(self.rows, self.cols, dtype=torch.float32, device=self.p.device)
        check(lib().ffn_b200_dequant_ternary(self.rows, self.cols, _ptr(self.p), _ptr(out),
                                             _stream(stream)), "dequant_ternary")
        return out

    def nbytes(self) -> int:
        n = self.p.numel() + 4 * self.rs.numel()
        if self.bs is not None:
            n += self.bs.numel()
        if self.core:
            n += self.core[0].numel() + self.core[2].numel() + 128
        return n


# Tensor tags of the generator key paths (same values as the oracle's).
TAG_W1, TAG_W3, TAG_W2, TAG_ROUTER, TAG_X, TAG_BIAS = 1, 3, 2, 10, 11, 12


class SwigluExpert:
    """gate (w1), up (w3), down (w2) of one SwiGLU expert on the device."""

    def __init__(self, fmt, mats, inter, hidden, proj_scale=1.0):
        self.fmt, self.mats, self.inter, self.hidden = fmt, mats, inter, hidden
        self.proj_scale = float(proj_scale)
        self.fp4 = None  # (gate/up, down) stage images of the FP4 path

    def cstruct(self) -> Expert:
        e = Expert()
        e.format = self.fmt
        e.proj_scale = self.proj_scale
        for i, m in enumerate(self.mats):
            if self.fmt == FMT_TERNARY:
                e.tn[i] = m.cstruct()
            else:  # NVFP4 and MXFP4 use nv[]
                e.nv[i] = m.cstruct()
        if self.fp4 is not None:
            e.fp4_gu, e.fp4_dn = _ptr(self.fp4[0]), _ptr(self.fp4[1])
        return e

    def pack_fp4(self, gu=None, dn=None, stream=None):
        """The FP4 path's stage images of this NVFP4 expert
        (ffn_b200_pack_nvfp4_expert), into gu / dn (uint8 device tensors of
        ffn_b200_fp4_pack_bytes, e.g. views of one larger buffer) or new
        tensors; raises FfnError when a scale byte is not UE4M3.  Returns self."""
        torch = _torch()
        dev = self.mats[0].w.device
        nb = [lib().ffn_b200_fp4_pack_bytes(self.inter, self.hidden, w) for w in (0, 1)]
        if gu is None:
            gu = torch.empty(nb[0], dtype=torch.uint8, device=dev)
        if dn is None:
            dn = torch.empty(nb[1], dtype=torch.uint8, device=dev)
        if gu.numel() < nb[0] or dn.numel() < nb[1]:
            raise FfnError("pack_fp4: image buffers too small")
        e = self.cstruct()
        check(lib().ffn_b200_pack_nvfp4_expert(self.inter, self.hidden, C.byref(e), _ptr(gu), _ptr(dn),
                                               _stream(stream)), "pack_nvfp4_expert")
        self.fp4 = (gu, dn)
        return self

    @classmethod
    def generate(cls, fmt, seed, layer, expert, inter, hidden, gs=1.0, with_core=True,
                 proj_scale=1.0, device="cuda", stream=None):
        tags = (TAG_W1, TAG_W3, TAG_W2)
        shapes = ((inter, hidden), (inter, hidden), (hidden, inter))
        mats = []
        for tag, (r, c) in zip(tags, shapes):
            k = path_key(seed, layer, expert, tag)
            if fmt == FMT_NVFP4:
                mats.append(Nvfp4Matrix.generate(k, r, c, gs, device, stream))
            else:
                mats.append(TernaryMatrix.generate(k, r, c, with_core, device, stream))
        return cls(fmt, mats, inter, hidden, proj_scale)

    def forward(self, x, out=None, weight=1.0, accumulate=False, stream=None):
        torch = _torch()
        x = x.contiguous()
        seq = x.numel() // self.hidden
        if out is None:
            out = torch.zeros(seq, self.hidden, dtype=torch.float32, device=x.device)
        ws = _default_ws(x.device).get(lib().ffn_b200_expert_ws_bytes(self.inter, self.hidden, seq))
        e = self.cstruct()
        check(lib().ffn_b200_expert_forward(self.inter, self.hidden, seq, C.byref(e), _ptr(x),
                                            _ptr(out), float(weight), int(accumulate), _ptr(ws),
                                            ws.numel(), _stream(stream)), "expert_forward")
        return out

    def nbytes(self) -> int:
        return sum(m.nbytes() for m in self.mats)


class LoadedExpert(SwigluExpert):
    """An expert whose tensors were copied from a shard into one device buffer."""

    def __init__(self, desc: "Expert", buf, inter, hidden):
        super().__init__(desc.format, None, inter, hidden, desc.proj_scale)
        self.desc, self.buf = desc, buf

    def cstruct(self) -> "Expert":
        e = Expert.from_buffer_copy(self.desc)
        e.proj_scale = self.proj_scale
        return e

    def nbytes(self) -> int:
        return int(self.buf.numel())


class SafetensorsShard:
    """A .safetensors shard mapped read-only by the library (ffn_b200_st_*,
    the reference's Flash1017ShardInspector, flash1017.rs:108-235): tensor
    lookup and routed experts copied straight into HBM."""

    def __init__(self, path):
        h = C.c_void_p()
        check(lib().ffn_b200_st_open(os.fsencode(str(path)), C.byref(h)), "st_open")
        self._h = h

    def close(self):
        if self._h:
            lib().ffn_b200_st_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def names(self):
        L = lib()
        return [L.ffn_b200_st_name(self._h, i).decode() for i in range(L.ffn_b200_st_count(self._h))]

    def __contains__(self, name) -> bool:
        return name in set(self.names())

    def tensor(self, name):
        """(dtype, shape, bytes): a copy of the tensor's bytes from the mapping."""
        dt, nd, data, nb = C.c_char_p(), C.c_int(), C.c_void_p(), C.c_size_t()
        shape = (C.c_int64 * 8)()
        check(lib().ffn_b200_st_find(self._h, name.encode(), C.byref(dt), shape, C.byref(nd),
                                     C.byref(data), C.byref(nb)), "st_find")
        return dt.value.decode(), tuple(shape[i] for i in range(nd.value)), C.string_at(data, nb.value)

    def expert_bytes(self, prefix, hidden, inter):
        fmt, nb = C.c_int(), C.c_size_t()
        check(lib().ffn_b200_st_expert_bytes(self._h, prefix.encode(), hidden, inter, C.byref(fmt),
                                             C.byref(nb)), "st_expert_bytes")
        return fmt.value, nb.value

    def load_expert(self, prefix, hidden, inter, device="cuda", stream=None) -> LoadedExpert:
        torch = _torch()
        _, nb = self.expert_bytes(prefix, hidden, inter)
        buf = torch.empty(nb + 256, dtype=torch.uint8, device=device)
        off = (-buf.data_ptr()) % 256
        view = buf[off:off + nb]
        e = Expert()
        check(lib().ffn_b200_st_load_expert(self._h, prefix.encode(), hidden, inter, _ptr(view), nb,
                                            _stream(stream), C.byref(e)), "st_load_expert")
        ex = LoadedExpert(e, buf, inter, hidden)
        return ex

    def load_layer(self, layer, n_experts, hidden, inter, device="cuda", stream=None):
        """The routed experts layers.<layer>.ffn.experts.<e> (flash1017.rs:5219-5262)."""
        return [self.load_expert(f"layers.{layer}.ffn.experts.{e}", hidden, inter, device, stream)
                for e in range(n_experts)]


def gen_normal(k: int, n: int, stdev: float = 1.0, device="cuda", stream=None):
    torch = _torch()
    out = torch.empty(n, dtype=torch.float32, device=device)
    check(lib().ffn_b200_gen_normal(k, n, float(stdev), _ptr(out), _stream(stream)),
          "gen_normal")
    return out


def topk(logits, top_k, score_fn=SCORE_SIGMOID, bias=None, stream=None):
    """The MoE layer's top-k step on device logits, [n_tok, n_exp] or partial
    planes [n_part, n_tok, n_exp] (added in plane order): (idx int32, wt f32),
    each [n_tok, top_k] (ffn_b200_topk)."""
    torch = _torch()
    lg = logits if logits.dim() == 3 else logits.unsqueeze(0)
    lg = lg.contiguous()
    n_part, n_tok, n_exp = lg.shape
    idx = torch.empty(n_tok, top_k, dtype=torch.int32, device=lg.device)
    wt = torch.empty(n_tok, top_k, dtype=torch.float32, device=lg.device)
    b = None if bias is None else bias.contiguous()
    check(lib().ffn_b200_topk(n_tok, n_exp, top_k, int(score_fn), _ptr(lg), n_part,
                              None if b is None else _ptr(b), _ptr(idx), _ptr(wt), _stream(stream)),
          "topk")
    return idx, wt


def expert_table(experts, device="cuda"):
    """Device array of ffn_b200_expert structs (None entries: placeholders)."""
    torch = _torch()
    table = (Expert * len(experts))()
    fmts = set()
    for i, e in enumerate(experts):
        if e is not None:
            table[i] = e.cstruct()
            fmts.add(e.fmt)
    return torch.frombuffer(bytearray(bytes(table)), dtype=torch.uint8).to(device), fmts


class MoeLayer:
    """Routed SwiGLU MoE layer over device-resident experts."""

    def __init__(self, experts, router_w, hidden, inter, top_k=6, score_fn=SCORE_SIGMOID,
                 router_bias=None, router_mode=ROUTER_EXACT, expert_range=None, device="cuda",
                 table=None, ws=None, norm_w=None, norm_eps=1e-20, path=PATH_AUTO):
        self.experts = experts  # SwigluExpert list (None allowed outside expert_range)
        self.router_w = router_w
        self.router_bias = router_bias
        self.norm_w = norm_w
        self.hidden, self.inter, self.top_k = hidden, inter, top_k
        n = len(experts)
        if any(e is not None and e.fmt == FMT_MXFP8 for e in experts):
            raise FfnError("MoE tables hold NVFP4, MXFP4 and ternary experts; MXFP8 is for "
                           "dense (shared) experts")
        if table is None:
            self.table, fmts = expert_table(experts, device)
        else:  # a shared (table, formats) pair
            self.table, fmts = table
        # experts kept only as stage images (reference-layout pointers NULL) can
        # run nowhere but the FP4 path
        if any(e is not None and e.mats is not None and any(getattr(m, "w", 0) is None for m in e.mats)
               for e in experts):
            if path not in (PATH_AUTO, PATH_FP4):
                raise FfnError("experts held only as FP4 stage images run only on PATH_FP4")
            path = PATH_FP4
        lo, hi = expert_range if expert_range else (0, n)
        # the FP4 path reads stage images: every local expert must carry them
        # (the table must have been built after pack_fp4)
        packed = all(experts[e] is not None and getattr(experts[e], "fp4", None) is not None
                     for e in range(lo, hi))
        self.desc = MoeDesc(hidden, inter, n, top_k, _ptr(self.table), _ptr(router_w),
                            _ptr(router_bias), score_fn, router_mode, lo, hi,
                            int(FMT_NVFP4 in fmts or FMT_MXFP4 in fmts or not fmts),
                            int(FMT_TERNARY in fmts), _ptr(norm_w), float(norm_eps), int(path),
                            int(FMT_MXFP4 in fmts), int(packed))
        self.ws = ws if ws is not None else Workspace(device)

    def ws_bytes(self, n_tok: int) -> int:
        return int(lib().ffn_b200_moe_ws_bytes(C.byref(self.desc), n_tok))

    def forward_ep(self, exchange, x, out, residual=None, topk_idx=None, topk_w=None, stream=None):
        """This rank's experts (expert_range) with the expert-parallel exchange
        fused in: out = residual + the layer over every rank's experts."""
        x = x.contiguous()
        n_tok = x.numel() // self.hidden
        ws = self.ws.get(self.ws_bytes(n_tok))
        check(lib().ffn_b200_ep_moe_layer(exchange.ep, C.byref(self.desc), n_tok, _ptr(x), _ptr(residual),
                                          _ptr(out), _ptr(topk_idx), _ptr(topk_w), _ptr(ws), ws.numel(),
                                          _stream(stream)), "ep_moe_layer")
        return out

    def forward(self, x, out=None, residual=None, topk_idx=None, topk_w=None, stream=None):
        torch = _torch()
        x = x.contiguous()
        n_tok = x.numel() // self.hidden
        if out is None:
            out = torch.empty(n_tok, self.hidden, dtype=torch.float32, device=x.device)
        ws = self.ws.get(self.ws_bytes(n_tok))
        check(lib().ffn_b200_moe_layer(C.byref(self.desc), n_tok, _ptr(x), _ptr(residual),
                                       _ptr(out), _ptr(topk_idx), _ptr(topk_w), _ptr(ws),
                                       ws.numel(), _stream(stream)), "moe_layer")
        return out
