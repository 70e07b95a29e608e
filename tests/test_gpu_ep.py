"""NVLink peer exchange of the expert-parallel partial outputs
(ffn_b200_ep_*), two processes on two GPUs.  Skipped with fewer than 2 GPUs.

1. Exact sums: rank r's part holds (r + 1) * base (small integers), the
   residual holds another pattern; every rank must get residual + 3 * base,
   bit-exact, over several calls (epochs, both result buffers).
2. A two-layer MoE stack run expert-parallel through EpStack with the
   exchange equals the same stack on one GPU with every expert (tolerance of
   the path: summation order differs), and the same stack with the exchange
   fused into each layer (ffn_b200_ep_moe_layer) equals the unfused one bit
   for bit."""
import os
import socket

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import datetime
    import sys
    for p in (ROOT, os.path.join(ROOT, "flash1017-engine_b200"), os.path.join(ROOT, "oracle")):
        sys.path.insert(0, p)
    import numpy as np
    import torch
    import torch.distributed as dist

    import ffn_b200 as F
    from ep import EpStack, expert_range

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    res = {}
    try:
        T, H = 24, 512
        ex = F.EpExchange(rank, world, 64, H)
        base = torch.arange(T * H, device=dev, dtype=torch.float32).view(T, H) % 97
        resid = (torch.arange(T * H, device=dev, dtype=torch.float32).view(T, H) % 13) - 6
        out = torch.empty(T, H, device=dev)
        exact = True
        for call in range(5):
            ex.part[:T].copy_((rank + 1 + call) * base)
            ex.allreduce(T, resid, out)
            torch.cuda.synchronize()
            want = resid + sum((r + 1 + call) for r in range(world)) * base
            exact = exact and bool(torch.equal(out, want))
        res["exact"] = exact and ex.error() == 0

        # two-layer MoE stack: EP with the exchange vs every expert on one GPU
        E, I, Tm, K, L = 16, 256, 40, 6, 2
        lo, hi = expert_range(rank, world, E)
        allx = [[F.SwigluExpert.generate(F.FMT_NVFP4, 41, lay, e, I, H) for e in range(E)]
                for lay in range(L)]
        routers = [F.gen_normal(F.path_key(41, lay, 0, F.TAG_ROUTER), E * H, 0.02).view(E, H)
                   for lay in range(L)]
        nw = torch.ones(H, device=dev)
        loc = [F.MoeLayer([e if lo <= i < hi else None for i, e in enumerate(allx[lay])],
                          routers[lay], H, I, top_k=K, router_mode=F.ROUTER_EXACT, norm_w=nw,
                          expert_range=(lo, hi)) for lay in range(L)]
        full = [F.MoeLayer(allx[lay], routers[lay], H, I, top_k=K, router_mode=F.ROUTER_EXACT,
                           norm_w=nw) for lay in range(L)]
        x = F.gen_normal(F.path_key(41, 0, 0, F.TAG_X), Tm * H).view(Tm, H)

        def fn(lay):
            def run(x_in, o, residual):
                loc[lay].forward(x_in, out=o, residual=residual)
            return run

        stack = EpStack([fn(lay) for lay in range(L)], rank, world, exchange=ex)
        a, b = torch.empty_like(x), torch.empty_like(x)
        y = stack.forward(x, a, b)
        ref = x
        for lay in range(L):
            ref = full[lay].forward(ref, residual=ref)
        torch.cuda.synchronize()
        yy, rr = y.cpu().numpy().astype(np.float64), ref.cpu().numpy().astype(np.float64)
        res["max_rel"] = float(np.abs(yy - rr).max() / np.abs(rr).max())
        res["finite"] = bool(np.isfinite(yy).all())

        # the same stack with the exchange fused into each layer (ffn_b200_ep_moe_layer):
        # the same arithmetic as the part buffer + allreduce path, so equal bit for bit
        def fn_fused(lay):
            def run(x_in, o, residual):
                loc[lay].forward_ep(ex, x_in, o, residual=residual)
            return run

        fstack = EpStack([fn_fused(lay) for lay in range(L)], rank, world, exchange=ex, fused=True)
        c, d = torch.empty_like(x), torch.empty_like(x)
        yf = fstack.forward(x, c, d)
        torch.cuda.synchronize()
        res["fused_equal"] = bool(torch.equal(yf, y)) and ex.error() == 0
        ex.close()
    except Exception as e:  # reported to the parent
        res["error"] = repr(e)
    finally:
        q.put((rank, res))
        dist.destroy_process_group()


def test_ep_exchange_two_gpus():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(2):
            r, res = q.get(timeout=300)
            out[r] = res
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    for r in (0, 1):
        assert "error" not in out[r], out[r]
        assert out[r]["exact"], out[r]
        assert out[r]["finite"] and out[r]["max_rel"] <= 1e-3, out[r]
        assert out[r]["fused_equal"], out[r]
