"""Expert parallelism host logic (flash1017-engine_b200/ep.py) on CPU: two gloo
ranks, each owning half of the experts, run a two-layer MoE stack through
EpStack; the result must equal the single-process stack of the oracle
(x_{l+1} = x_l + moe_l(x_l)).  Each rank's layer is the oracle restricted to its
expert block, so what is tested is the partition, the residual on rank 0 only
and the per-layer sum all-reduce."""
import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
E, H, I, T, K, LAYERS, SEED = 8, 128, 64, 5, 2, 2, 11


def _problem(O):
    experts = [[O.gen_nvfp4_expert(SEED, lay, e, I, H) for e in range(E)] for lay in range(LAYERS)]
    routers = [O.gen_router(SEED, lay, E, H) for lay in range(LAYERS)]
    x = O.gen_hidden(SEED, T, H)
    return experts, routers, x


def _partial(O, experts, wr, x, lo, hi):
    """sum over the top-k experts of each token that lie in [lo, hi) of w * expert(x)."""
    logits = O.router_logits(wr, x)
    idx, wt, _, _ = O.route(logits, K, None, 1)
    out = np.zeros_like(x)
    for t in range(x.shape[0]):
        xt = np.ascontiguousarray(x[t])
        for k in range(K):
            e = int(idx[t, k])
            if lo <= e < hi:
                O.axpy(out[t], wt[t, k], experts[e].forward(xt))
    return out


def _rank_main(rank, world, port, q):
    for p in (ROOT, os.path.join(ROOT, "flash1017-engine_b200"), os.path.join(ROOT, "oracle")):
        sys.path.insert(0, p)
    import datetime

    import torch
    import torch.distributed as dist

    import oracle as O
    from ep import EpStack, expert_range

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        experts, routers, x = _problem(O)
        lo, hi = expert_range(rank, world, E)

        def layer(lay):
            def run(x_in, out, residual):
                xin = x_in.numpy()
                y = _partial(O, experts[lay], routers[lay], xin, lo, hi)
                if residual is not None:
                    y = y + residual.numpy()
                out.copy_(torch.from_numpy(y))
            return run

        ep = EpStack([layer(lay) for lay in range(LAYERS)], rank, world)
        xt = torch.from_numpy(x.copy())
        a, b = torch.empty_like(xt), torch.empty_like(xt)
        y = ep.forward(xt, a, b)
        q.put((rank, y.numpy().copy()))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_expert_range():
    from ep import expert_range
    assert [expert_range(r, 8, 384) for r in (0, 7)] == [(0, 48), (336, 384)]
    assert expert_range(0, 1, 384) == (0, 384)
    with pytest.raises(ValueError):
        expert_range(0, 5, 384)
    with pytest.raises(ValueError):
        expert_range(2, 2, 384)


def test_ep_stack_world2_matches_single_process(oracle):
    import torch.multiprocessing as mp

    O = oracle
    experts, routers, x = _problem(O)
    ref = x.copy()
    for lay in range(LAYERS):
        y, _, _ = O.moe_layer(experts[lay], routers[lay], ref, top_k=K, score_fn=1)
        ref = ref + y

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    outs = {}
    try:
        for _ in range(2):
            r, y = q.get(timeout=120)
            outs[r] = y
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    np.testing.assert_array_equal(outs[0], outs[1])  # every rank holds the full output
    O.assert_close(outs[0], ref, what="EP world 2 vs single process")
