"""Safetensors expert loader (ffn_b200_st_*): the reference's shard mapping and
tensor lookup (Flash1017ShardInspector, flash1017.rs:108-235) and the expert
matrix constructors (:2295-2309, :2495-2525, :2415-2440).

Shards are written here the way the reference's 106 GB writer lays them out
(flash1017.rs:10836-10880: JSON header padded to 8 bytes, tensors 8-byte
aligned), with weights from the oracle's generators.  CPU tests: header
parsing, lookup, expert planning and malformed files.  GPU tests: experts
loaded into HBM run through the kernels and match the oracle on the same
bytes, at the benchmark configs' dims and at the reference checkpoint's own dims
(H 5120, I 2304, flash1017.rs:7268-7269)."""
import json
import os
import struct
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(ROOT, "flash1017-engine_b200"), os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def write_shard(path, tensors, metadata=None):
    """tensors: [(name, dtype, shape, bytes)]."""
    header, blobs, off = {}, [], 0
    if metadata is not None:
        header["__metadata__"] = metadata
    for name, dt, shape, data in tensors:
        header[name] = {"dtype": dt, "shape": list(shape), "data_offsets": [off, off + len(data)]}
        pad = (-(off + len(data))) % 8
        blobs.append(bytes(data) + b"\0" * pad)
        off += len(data) + pad
    h = json.dumps(header).encode()
    h += b" " * ((-len(h)) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def nvfp4_tensors(O, prefix, seed, inter, hidden, gs=(0.5, 0.75, 1.25)):
    """(tensor list, oracle expert) of one NVFP4 expert."""
    out, ws, ss = [], [], []
    for k, (m, rows, cols) in enumerate((("w1", inter, hidden), ("w3", inter, hidden), ("w2", hidden, inter))):
        w, s = O.gen_nvfp4(O.key(seed, 0, k, O.TAG_W1), rows, cols)
        out += [(f"{prefix}.{m}.weight", "U8", (rows, cols // 2), w.tobytes()),
                (f"{prefix}.{m}.weight_scale", "F8_E4M3", (rows, cols // 16), s.tobytes()),
                (f"{prefix}.{m}.weight_scale_2", "F32", (1,), np.float32(gs[k]).tobytes())]
        ws.append(w)
        ss.append(s)
    return out, O.Nvfp4Expert(inter, hidden, tuple(ws), tuple(ss), gs)


def ternary_tensors(O, prefix, seed, inter, hidden, block_scales=True, core=True):
    out, ps, rss, bss, cores = [], [], [], [], []
    rng = np.random.default_rng(seed)
    for k, (m, rows, cols) in enumerate((("w1", inter, hidden), ("w3", inter, hidden), ("w2", hidden, inter))):
        p, rs = O.gen_ternary(O.key(seed, 1, k, O.TAG_W1), rows, cols)
        out += [(f"{prefix}.{m}.packed_ternary", "U8", (rows, cols // 4), p.tobytes()),
                (f"{prefix}.{m}.row_scales", "F32", (rows,), rs.tobytes())]
        ps.append(p)
        rss.append(rs)
        if block_scales:
            bs = rng.integers(0, 256, size=rows * cols // 64, dtype=np.uint8)
            out.append((f"{prefix}.{m}.block_scales", "U8", (rows, cols // 64), bs.tobytes()))
            bss.append(bs)
        if core:
            c = O.gen_core(O.key(seed, 2, k, O.TAG_W1), rows, cols)
            out += [(f"{prefix}.{m}.core_b_q8", "I8", (rows, 16), c.b.tobytes()),
                    (f"{prefix}.{m}.core_b_scale", "F32", (16,), c.b_sc.tobytes()),
                    (f"{prefix}.{m}.core_a_q8", "I8", (16, cols), c.a.tobytes()),
                    (f"{prefix}.{m}.core_a_scale", "F32", (16,), c.a_sc.tobytes())]
            cores.append(c)
    oe = O.TernaryExpert(inter, hidden, tuple(ps), tuple(rss), tuple(cores) if core else None, 1.0,
                         tuple(bss) if block_scales else None)
    return out, oe


@pytest.fixture(scope="module")
def O():
    import oracle
    return oracle


@pytest.fixture(scope="module")
def F():
    import ffn_b200
    return ffn_b200


@pytest.fixture
def shard(tmp_path, O):
    H, I = 512, 256
    t1, o1 = nvfp4_tensors(O, "layers.3.ffn.experts.0", 1, I, H)
    t2, o2 = ternary_tensors(O, "layers.3.ffn.experts.1", 2, I, H)
    t3, o3 = ternary_tensors(O, "layers.3.ffn.experts.2", 3, I, H, block_scales=False, core=False)
    router = np.arange(3 * H, dtype=np.uint16)
    extra = [("layers.3.ffn.gate.weight", "BF16", (3, H), router.tobytes())]
    path = tmp_path / "model-00004-of-00048.safetensors"
    write_shard(path, t1 + extra + t2 + t3, metadata={"format": "pt", "note": "a \"quoted\" \u00e9 value"})
    return path, (H, I), (o1, o2, o3), t1 + extra + t2 + t3


# ------------------------------------------------------------------ CPU
def test_header_and_lookup(F, shard):
    path, (H, I), _, tensors = shard
    st = F.SafetensorsShard(path)
    assert st.names() == [t[0] for t in tensors]
    for name, dt, shape, data in tensors:
        d, s, b = st.tensor(name)
        assert (d, s, b) == (dt, tuple(shape), data), name
    with pytest.raises(F.FfnError):
        st.tensor("layers.3.ffn.experts.9.w1.weight")
    st.close()


def test_expert_planning(F, shard):
    path, (H, I), _, _ = shard
    st = F.SafetensorsShard(path)
    fmt, nb = st.expert_bytes("layers.3.ffn.experts.0", H, I)
    assert fmt == F.FMT_NVFP4
    # 3 x (weights + scales), each piece 256-byte aligned
    assert nb >= 3 * (I * H // 2 + I * H // 16)
    fmt, nb1 = st.expert_bytes("layers.3.ffn.experts.1", H, I)
    fmt2, nb2 = st.expert_bytes("layers.3.ffn.experts.2", H, I)
    assert fmt == fmt2 == F.FMT_TERNARY and nb1 > nb2  # block scales + cores
    with pytest.raises(F.FfnError):  # wrong dims
        st.expert_bytes("layers.3.ffn.experts.0", 2 * H, I)
    with pytest.raises(F.FfnError):  # absent expert
        st.expert_bytes("layers.3.ffn.experts.7", H, I)


@pytest.mark.parametrize("case", ["short", "header_len", "json", "offsets", "not_object", "dup_field"])
def test_malformed_shards(F, tmp_path, case):
    path = tmp_path / f"{case}.safetensors"
    good = json.dumps({"a": {"dtype": "U8", "shape": [4], "data_offsets": [0, 4]}}).encode()
    if case == "short":
        blob = b"\x01\x02"
    elif case == "header_len":
        blob = struct.pack("<Q", 10 ** 6) + good
    elif case == "json":
        h = good[:-3]
        blob = struct.pack("<Q", len(h)) + h + b"\0" * 4
    elif case == "offsets":
        h = json.dumps({"a": {"dtype": "U8", "shape": [64], "data_offsets": [0, 64]}}).encode()
        blob = struct.pack("<Q", len(h)) + h + b"\0" * 8
    elif case == "not_object":
        h = b"[1, 2, 3]"
        blob = struct.pack("<Q", len(h)) + h
    else:  # a tensor listed twice
        h = b'{"a": {"dtype": "U8", "shape": [4], "data_offsets": [0, 4]}, ' \
            b'"a": {"dtype": "U8", "shape": [4], "data_offsets": [0, 4]}}'
        blob = struct.pack("<Q", len(h)) + h + b"\0" * 4
    path.write_bytes(blob)
    with pytest.raises(F.FfnError):
        F.SafetensorsShard(path)


def test_missing_file(F, tmp_path):
    with pytest.raises(F.FfnError):
        F.SafetensorsShard(tmp_path / "absent.safetensors")


# ------------------------------------------------------------------ GPU
@pytest.mark.gpu
def test_loaded_experts_match_oracle(F, O, shard):
    import torch
    path, (H, I), oes, _ = shard
    st = F.SafetensorsShard(path)
    x = F.gen_normal(F.path_key(60, 0, 0, F.TAG_X), 3 * H).view(3, H)
    xs = x.cpu().numpy()
    for e, oe in enumerate(oes):
        ex = st.load_expert(f"layers.3.ffn.experts.{e}", H, I)
        y = ex.forward(x).cpu().numpy()
        ref = np.stack([oe.forward(np.ascontiguousarray(xs[t])) for t in range(3)])
        O.assert_close(y, ref, what=f"loaded expert {e}")
    torch.cuda.synchronize()


@pytest.mark.gpu
def test_loaded_layer_moe_matches_oracle(F, O, shard):
    path, (H, I), oes, _ = shard
    st = F.SafetensorsShard(path)
    experts = st.load_layer(3, 3, H, I)
    wr = F.gen_normal(F.path_key(61, 0, 0, F.TAG_ROUTER), 3 * H, 0.02).view(3, H)
    x = F.gen_normal(F.path_key(61, 0, 0, F.TAG_X), 9 * H).view(9, H)
    out = F.MoeLayer(experts, wr, H, I, top_k=2, score_fn=0).forward(x).cpu().numpy()
    ref, _, _ = O.moe_layer(list(oes), wr.cpu().numpy(), x.cpu().numpy(), top_k=2, score_fn=0)
    O.assert_close(out, ref, what="MoE layer of loaded experts")


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["nvfp4", "ternary"])
def test_reference_checkpoint_dims(F, O, tmp_path, fmt):
    """The reference checkpoint's expert dims, H 5120 and I 2304 (flash1017.rs:
    7268-7269), through the same kernels."""
    H, I = 5120, 2304
    pre = "layers.0.ffn.experts.5"
    if fmt == "nvfp4":
        t, oe = nvfp4_tensors(O, pre, 7, I, H)
    else:
        t, oe = ternary_tensors(O, pre, 8, I, H)
    path = tmp_path / "dims.safetensors"
    write_shard(path, t)
    ex = F.SafetensorsShard(path).load_expert(pre, H, I)
    x = F.gen_normal(F.path_key(62, 0, 0, F.TAG_X), 2 * H).view(2, H)
    y = ex.forward(x).cpu().numpy()
    xs = x.cpu().numpy()
    ref = np.stack([oe.forward(np.ascontiguousarray(xs[k])) for k in range(2)])
    O.assert_close(y, ref, what=f"{fmt} expert at H 5120, I 2304")
