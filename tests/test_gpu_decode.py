"""The expert decode kernels (csrc/expert_decode.cu): one NVFP4, MXFP4 or
ternary SwiGLU expert over 1..8 tokens (NVFP4 from 3 tokens on the tensor
cores), as ffn_b200_expert_forward runs it
for those formats and batch sizes, against the oracle's expert
(flash1017.rs:7537-7561 over CachedNvfp4Mat / CachedMxfp4Mat /
CachedTernary158Mat rows with their rank-16 cores, flash1017.rs:2331-2357,
2717-2744, 2538-2627, 2396-2473) and the output update out (+)= w * y
(flash1017.rs:4900-4905).  Tolerance:
max|y - ref| / max|ref| <= 1e-3 and cosine >= 0.99999.  Each case also checks
that the call issued exactly the two decode launches (ternary experts with
gate/up cores: three, the cores' z kernel first; the GEMV chain issues at
least three, four with cores)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def host(t):
    return np.ascontiguousarray(t.detach().cpu().numpy())


def _nvfp4(ffn, oracle, seed, inter, hidden):
    e = ffn.SwigluExpert.generate(ffn.FMT_NVFP4, seed, 0, 0, inter, hidden)
    oe = oracle.Nvfp4Expert(inter, hidden, tuple(host(m.w) for m in e.mats),
                            tuple(host(m.s) for m in e.mats), tuple(m.gs for m in e.mats))
    return e, oe


LAUNCHES = 2


def _run(ffn, e, x, out=None, weight=1.0, accumulate=False):
    n0 = ffn.launch_count()
    y = e.forward(x, out=out, weight=weight, accumulate=accumulate)
    return host(y), ffn.launch_count() - n0


@pytest.mark.parametrize("seq", [1, 2, 3, 8])
def test_decode_nvfp4_config0(oracle, ffn, cuda, seq):
    H, I = 4096, 2048
    e, oe = _nvfp4(ffn, oracle, 0, I, H)
    x = ffn.gen_normal(ffn.path_key(0, 0, seq, ffn.TAG_X), seq * H).view(seq, H)
    y, launches = _run(ffn, e, x)
    assert launches == LAUNCHES
    xs = host(x)
    ref = np.stack([oe.forward(np.ascontiguousarray(xs[t])) for t in range(seq)])
    oracle.assert_close(y, ref, what=f"decode nvfp4 seq {seq}")


@pytest.mark.parametrize("seq", [1, 5])
def test_decode_accumulate(oracle, ffn, cuda, seq):
    """out += w * y on top of existing contents, twice, deterministic."""
    import torch
    H, I = 4096, 2048
    e, oe = _nvfp4(ffn, oracle, 3, I, H)
    x = ffn.gen_normal(ffn.path_key(3, 1, seq, ffn.TAG_X), seq * H).view(seq, H)
    base = ffn.gen_normal(ffn.path_key(3, 2, seq, ffn.TAG_X), seq * H).view(seq, H)
    w = 0.37
    out = base.clone()
    _, launches = _run(ffn, e, x, out=out, weight=w, accumulate=True)
    assert launches == LAUNCHES
    y2 = host(e.forward(x, out=out, weight=w, accumulate=True))
    xs, b = host(x), host(base)
    ref = np.stack([oe.forward(np.ascontiguousarray(xs[t])) for t in range(seq)])
    expect = (b + np.float32(w) * ref) + np.float32(w) * ref
    oracle.assert_close(y2 - b, expect - b, what=f"decode accumulate seq {seq}")
    again = base.clone()
    e.forward(x, out=again, weight=w, accumulate=True)
    e.forward(x, out=again, weight=w, accumulate=True)
    assert torch.equal(again, out)


@pytest.mark.parametrize("seq", [2, 4])
@pytest.mark.parametrize("inter,hidden", [(512, 1024), (1024, 512), (1024, 8192), (4096, 2048)])
def test_decode_shapes(oracle, ffn, cuda, inter, hidden, seq):
    """Rows per CTA from 3 up to 56, one to sixteen column chunks; 2 tokens on
    the CUDA cores, 4 on the tensor cores (4 to 64 column blocks over 16
    warps)."""
    e, oe = _nvfp4(ffn, oracle, 11, inter, hidden)
    x = ffn.gen_normal(ffn.path_key(11, inter, hidden, ffn.TAG_X), seq * hidden).view(seq, hidden)
    y, launches = _run(ffn, e, x)
    assert launches == LAUNCHES
    xs = host(x)
    ref = np.stack([oe.forward(np.ascontiguousarray(xs[t])) for t in range(seq)])
    oracle.assert_close(y, ref, what=f"decode nvfp4 {inter}x{hidden}")


def test_decode_fallback_shapes(oracle, ffn, cuda):
    """Shapes the decode kernels do not take (inter 2304: not a multiple of 512;
    9 tokens) run on the GEMV chain with the same results."""
    for inter, hidden, seq in ((2304, 5120, 1), (2048, 4096, 9)):
        e, oe = _nvfp4(ffn, oracle, 12, inter, hidden)
        x = ffn.gen_normal(ffn.path_key(12, inter, seq, ffn.TAG_X), seq * hidden).view(seq, hidden)
        y, launches = _run(ffn, e, x)
        assert launches >= 3
        xs = host(x)
        ref = np.stack([oe.forward(np.ascontiguousarray(xs[t])) for t in range(seq)])
        oracle.assert_close(y, ref, what=f"fallback {inter}x{hidden} seq {seq}")


@pytest.mark.parametrize("seq", [1, 4])
def test_decode_mxfp4(oracle, ffn, cuda, seq):
    from test_gpu_mx import mx_expert
    H, I = 4096, 2048
    e, oe = mx_expert(ffn, oracle, 90, I, H, cuda)
    x = ffn.gen_normal(ffn.path_key(90, 0, seq, ffn.TAG_X), seq * H).view(seq, H)
    y, launches = _run(ffn, e, x)
    assert launches == LAUNCHES
    xs = host(x)
    ref = np.stack([oe.forward(np.ascontiguousarray(xs[t])) for t in range(seq)])
    oracle.assert_close(y, ref, what=f"decode mxfp4 seq {seq}")


def test_decode_back_to_back(oracle, ffn, cuda):
    """Eight experts in a row on one stream, accumulated into one output: the
    next call's kernels start while the previous call's finish."""
    import torch
    H, I, seq = 4096, 2048, 1
    pairs = [_nvfp4(ffn, oracle, 20 + k, I, H) for k in range(8)]
    x = ffn.gen_normal(ffn.path_key(20, 0, 0, ffn.TAG_X), seq * H).view(seq, H)
    out = torch.zeros(seq, H, dtype=torch.float32, device=cuda)
    for k, (e, _) in enumerate(pairs):
        e.forward(x, out=out, weight=0.125 * (k + 1), accumulate=True)
    xs = host(x)[0]
    ref = np.zeros(H, dtype=np.float32)
    for k, (_, oe) in enumerate(pairs):
        ref = ref + np.float32(0.125 * (k + 1)) * oe.forward(np.ascontiguousarray(xs))
    oracle.assert_close(host(out)[0], ref, what="eight experts back to back")



def _ternary(ffn, oracle, seed, inter, hidden, cuda, core, bs, proj):
    from test_gpu_parity import oracle_ternary_expert, with_block_scales
    e = ffn.SwigluExpert.generate(ffn.FMT_TERNARY, seed, 0, 0, inter, hidden, with_core=core, proj_scale=proj)
    if bs:
        e = with_block_scales(e, seed * 10, cuda)
    return e, oracle_ternary_expert(oracle, e)


@pytest.mark.parametrize("seq", [1, 2])
@pytest.mark.parametrize("core,bs,proj", [(True, False, 1.0), (False, False, 1.0), (True, True, 1.0),
                                          (True, False, 2.5)])
def test_decode_ternary_config1(oracle, ffn, cuda, seq, core, bs, proj):
    """Config 1 shapes: ternary + rank-16 Q8 cores (gate/up z from the core
    kernel; the down core's sums split between the phases), the 106 GB
    format's U8 block scales, and tier_b_proj_scale on gate/up.  Two tokens
    and more run on the GEMV engine."""
    H, I = 4096, 2048
    e, oe = _ternary(ffn, oracle, 31, I, H, cuda, core, bs, proj)
    x = ffn.gen_normal(ffn.path_key(31, seq, int(core), ffn.TAG_X), seq * H).view(seq, H)
    y, launches = _run(ffn, e, x)
    if seq == 1:
        assert launches == (3 if core else 2)
    else:
        assert launches >= (5 if core else 3)
    xs = host(x)
    ref = np.stack([oe.forward(np.ascontiguousarray(xs[t])) for t in range(seq)])
    oracle.assert_close(y, ref, what=f"decode ternary seq {seq} core {core} bs {bs} proj {proj}")


def test_decode_ternary_accumulate(oracle, ffn, cuda):
    import torch
    H, I, seq = 4096, 2048, 1
    e, oe = _ternary(ffn, oracle, 32, I, H, cuda, True, False, 1.0)
    x = ffn.gen_normal(ffn.path_key(32, 0, 0, ffn.TAG_X), seq * H).view(seq, H)
    base = ffn.gen_normal(ffn.path_key(32, 1, 0, ffn.TAG_X), seq * H).view(seq, H)
    out = base.clone()
    e.forward(x, out=out, weight=-0.6, accumulate=True)
    xs, b = host(x), host(base)
    ref = np.stack([oe.forward(np.ascontiguousarray(xs[t])) for t in range(seq)])
    oracle.assert_close(host(out) - b, np.float32(-0.6) * ref, what="decode ternary accumulate")
    assert torch.isfinite(out).all()
