"""The allocation-free expert entry point (ffn_b200_expert_forward_noalloc).

It exists for callers that cannot give this library device scratch and must
not see it allocate: a plugin host that owns the device-memory budget, code
running during CUDA stream capture, decode loops that must not allocate.  It
keeps its scratch in a fixed 1 MiB device array.  This file is collected last
so that a run stopping at the first failure has run every other test first.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _noalloc(ffn, e, x, out, weight, accumulate):
    ee = e.cstruct()
    import torch
    rc = ffn.lib().ffn_b200_expert_forward_noalloc(
        e.inter, e.hidden, x.shape[0], C.byref(ee), x.data_ptr(), out.data_ptr(), float(weight),
        int(accumulate), C.c_void_p(torch.cuda.current_stream().cuda_stream))
    ffn.check(rc, "expert_forward_noalloc")
    return out


@pytest.mark.parametrize("fmt,seq", [(0, 1), (0, 6), (1, 3)])
def test_noalloc_matches_expert_forward_on_two_calls(oracle, ffn, cuda, fmt, seq):
    import torch
    H, I = 4096, 2048
    e = ffn.SwigluExpert.generate(fmt, 70, 0, fmt, I, H, with_core=True)
    for call in range(2):  # the shared scratch keeps the first call's contents
        x = ffn.gen_normal(ffn.path_key(70, call, seq, ffn.TAG_X), seq * H).view(seq, H)
        base = torch.full((seq, H), 0.5, device=cuda)
        want = e.forward(x, out=base.clone(), weight=0.75, accumulate=True)
        got = _noalloc(ffn, e, x, base.clone(), 0.75, True)
        torch.cuda.synchronize()
        oracle.assert_close(got.cpu().numpy(), want.cpu().numpy(),
                            what=f"noalloc fmt {fmt} seq {seq} call {call}")


def test_noalloc_rejects_shapes_beyond_its_scratch(ffn, cuda):
    import torch
    H, I, seq = 4096, 2048, 64  # needs ~1.6 MB of scratch, above the 1 MiB array
    e = ffn.SwigluExpert.generate(0, 71, 0, 0, I, H)
    x = torch.zeros(seq, H, device=cuda)
    out = torch.zeros(seq, H, device=cuda)
    ee = e.cstruct()
    rc = ffn.lib().ffn_b200_expert_forward_noalloc(I, H, seq, C.byref(ee), x.data_ptr(),
                                                   out.data_ptr(), 1.0, 0, None)
    assert rc == -1
    assert b"more than the fixed" in ffn.lib().ffn_b200_last_error()
    assert float(out.abs().max()) == 0.0  # nothing ran
