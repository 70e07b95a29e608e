"""CPU tests of the C-ABI boundary: the library loads, exports what the
headers declare, presents the reference's vtable layout, and validates
arguments before touching a GPU."""
import ctypes as C
import os
import re
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INC = os.path.join(ROOT, "include")


def header_functions():
    names = set()
    for h in ("ffn_b200.h", "merkaba_hw_addon.h"):
        text = open(os.path.join(INC, h)).read()
        for m in re.finditer(r"^FFN_B200_EXPORT [^;(]*?\b([a-z_0-9]+)\(", text, re.M):
            names.add(m.group(1))
    return names


def test_exports_cover_headers(ffn):
    declared = header_functions()
    assert declared == set(ffn.EXPORTS), declared ^ set(ffn.EXPORTS)
    L = ffn.lib()
    for name in declared:
        assert getattr(L, name) is not None


def test_only_declared_symbols_exported(ffn):
    out = subprocess.run(["nm", "-D", "--defined-only", ffn.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    syms = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    ours = {s for s in syms if s.startswith(("ffn_b200_", "gx10_rust_", "merkaba_"))}
    assert ours == set(ffn.EXPORTS)


def test_headers_compile_as_c_and_cpp(tmp_path):
    src = tmp_path / "t.c"
    src.write_text('#include "merkaba_hw_addon.h"\n#include "ffn_b200.h"\nint main(void){return 0;}\n')
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-I", INC, "-c", str(src), "-o",
                    str(tmp_path / "t.o")], check=True)
    cpp = tmp_path / "t.cpp"  # the C++ build runs the static_asserts on the vtable layout
    cpp.write_text(src.read_text())
    subprocess.run(["g++", "-std=c++17", "-Wall", "-Werror", "-I", INC, "-c", str(cpp), "-o",
                    str(tmp_path / "t2.o")], check=True)


class VTable(C.Structure):
    """hardware_addon.rs:143-174, read through ctypes."""
    _fields_ = [("abi_version", C.c_uint32), ("addon_id_ptr", C.c_void_p),
                ("addon_id_len", C.c_size_t), ("addon_desc_ptr", C.c_void_p),
                ("addon_desc_len", C.c_size_t)] + [
        (n, C.c_void_p) for n in (
            "dot_f32", "dot_i8_f32", "dot_q4_g32_f32", "dot_ternary_2bit_f32",
            "matvec_q4_g32", "matvec_q8", "matvec_bf16", "matbatch_q4_g32", "matbatch_q8",
            "matbatch_bf16", "matvec_nvfp4", "matbatch_nvfp4", "matvec_ternary_158",
            "matbatch_ternary_158", "matvec_mxfp8", "matbatch_mxfp8")]


def test_vtable_layout_and_slots(ffn):
    assert C.sizeof(VTable) == 168
    p = ffn.lib().merkaba_hardware_addon_v1()
    assert p
    vt = VTable.from_address(p)
    assert vt.abi_version == 0x4D485703
    assert C.string_at(vt.addon_id_ptr, vt.addon_id_len).decode() == "addon_b200_ffn"
    assert C.string_at(vt.addon_desc_ptr, vt.addon_desc_len).decode().startswith("B200")
    for name in ("dot_f32", "dot_i8_f32", "dot_q4_g32_f32", "dot_ternary_2bit_f32",
                 "matvec_bf16", "matbatch_bf16", "matvec_nvfp4", "matbatch_nvfp4",
                 "matvec_ternary_158", "matbatch_ternary_158", "matvec_mxfp8", "matbatch_mxfp8"):
        assert getattr(vt, name), name
    for name in ("matvec_q4_g32", "matvec_q8", "matbatch_q4_g32", "matbatch_q8"):
        assert not getattr(vt, name), name  # out of scope: None for the Rust host
    assert ffn.lib().merkaba_hardware_addon_v1() == p  # stable for the process lifetime


def test_argument_validation_without_gpu(ffn):
    """Bad shapes and pointers are rejected before any CUDA call."""
    L = ffn.lib()
    m = ffn.NvMat(None, None, 1.0, 0)
    rc = L.ffn_b200_nvfp4_matvec(16, 64, 1, C.byref(m), None, None, None, 0, None)
    assert rc == -1 and b"null" in L.ffn_b200_last_error()
    m = ffn.NvMat(16, 16, 1.0, 0)
    rc = L.ffn_b200_nvfp4_matvec(16, 48, 1, C.byref(m), None, None, None, 0, None)
    assert rc == -5 and b"multiple of 64" in L.ffn_b200_last_error()
    m = ffn.NvMat(24, 16, 1.0, 0)  # misaligned weights
    assert L.ffn_b200_nvfp4_matvec(16, 64, 1, C.byref(m), None, None, None, 0, None) == -1
    t = ffn.TnMat(16, 4, None, None, None, None)
    assert L.ffn_b200_ternary_matvec(16, 96, 1, C.byref(t), None, None, None, 0, None) == -5
    d = ffn.MoeDesc(4096, 2048, 384, 7, None, None, None, 1, 0, 0, 384, 1, 0, None, 0.0, 0)
    assert L.ffn_b200_moe_layer(C.byref(d), 4, None, None, None, None, None, None, 0, None) == -1
    d = ffn.MoeDesc(4096, 2048, 384, 6, 64, 64, None, 1, 0, 0, 385, 1, 0, None, 0.0, 0)
    assert L.ffn_b200_moe_layer(C.byref(d), 4, None, None, None, None, None, None, 0, None) == -1
    d = ffn.MoeDesc(4096, 2048, 384, 6, 64, 64, None, 7, 0, 0, 384, 1, 0, None, 0.0, 0)
    assert L.ffn_b200_moe_layer(C.byref(d), 4, None, None, None, None, None, None, 0, None) == -1
    d = ffn.MoeDesc(4096, 2048, 384, 6, 64, 64, None, 1, 9, 0, 384, 1, 0, None, 0.0, 0)
    assert L.ffn_b200_moe_layer(C.byref(d), 4, None, None, None, None, None, None, 0, None) == -1
    d = ffn.MoeDesc(4096, 2048, 384, 6, 64, 64, None, 1, 0, 0, 384, 1, 0, None, 0.0, 0)
    rc = L.ffn_b200_moe_layer(C.byref(d), 4, 64, None, 64, None, None, 64, 16, None)
    assert rc == -3  # workspace too small


def test_workspace_sizes_scale(ffn):
    L = ffn.lib()
    d = ffn.MoeDesc(4096, 2048, 384, 6, None, None, None, 1, 0, 0, 384, 1, 0, None, 0.0, 0)
    a, b = L.ffn_b200_moe_ws_bytes(C.byref(d), 64), L.ffn_b200_moe_ws_bytes(C.byref(d), 256)
    assert 0 < a < b
    assert b >= 256 * 6 * 4096 * 4  # y [P, H] f32 dominates
    assert L.ffn_b200_expert_ws_bytes(2048, 4096, 1) < L.ffn_b200_expert_ws_bytes(2048, 4096, 8)


def test_generator_key_matches_oracle(ffn, oracle):
    for path in ((0, 0, 0, 1), (4, 39, 383, 2), (2, 0, 0, 11)):
        assert ffn.path_key(*path) == oracle.key(*path)
