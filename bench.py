#!/usr/bin/env python
"""bench.py -- MoE expert-FFN tokens/s on 1/2/4/8 B200 (benchmark config 4).

Workload: a 40-layer NVFP4 MoE-FFN stack (hidden 4096, intermediate 2048, 384
routed SwiGLU experts per layer, the reference's ffn_norm RMSNorm on the layer
input (weights 1, eps 1e-20, flash1017.rs:7637), fp32 router N(0, 0.02) on the
tensor cores, sigmoid top-6 with renormalised weights, residual add between
layers), one decode step of 256
tokens, seed 4, random-init weights from the library's seeded generator.
Experts are sharded expert-parallel: rank r of N owns experts
[r*384/N, (r+1)*384/N) of every layer; every rank routes all tokens (the
routing is replicated, so no count exchange is needed) and the per-layer
partial outputs are summed with one NCCL all-reduce.  A "step" is the full
40-layer pass over the 256 tokens; `value` is tokens/s for the whole job.

The stack holds 15,360 experts (~217 GB): on one GPU only the layers that fit
are resident and layer-step l streams the weights of resident layer
l % resident_layers.  Every layer's weights (>= 2.6 GB per rank) are far
larger than L2, so every layer-step reads its expert bytes from HBM, as the
full stack does; config.resident_layers records the number.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
                       [--workload config4|config3]
(N > 1 under torchrun, one rank per GPU).

--workload config3 measures benchmark config 3 instead: one NVFP4 MoE layer
over a prefill of 8192 tokens (bf16-valued N(0,1) hidden states, seed 3,
sigmoid top-6 of 384, no ffn_norm), which the library runs on its tensor-core
grouped GEMM; a step is one layer pass, the roofline is the gate/up GEMM's
TFLOP/s against the measured dense bf16 peak.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "flash1017-engine_b200")
ORACLE = os.path.join(ROOT, "oracle")
for _p in (PKG, ORACLE):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "MoE expert-FFN tokens/s (40-layer NVFP4 top-6/384 decode stack)"
UNIT = "tokens/s"
EXPERT_BYTES = lambda H, I: 3 * (I * H // 2 + I * H // 16)  # noqa: E731


def tern106_mat_bytes(rows, cols):
    """One matrix of the 106 GB format: codes, row scales, U8 block scales,
    rank-16 core (B rows x 16, A 16 x cols, two 16-float scale vectors)."""
    return rows * cols // 4 + 4 * rows + rows * cols // 64 + 16 * rows + 16 * cols + 128


METRIC106 = "MoE expert-FFN tokens/s (40-layer 106 GB-format ternary top-6/384 decode stack)"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["config4", "config3", "expert", "compress"], default="config4")
    ap.add_argument("--tokens", type=int, default=None)
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--experts", type=int, default=384)
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--inter", type=int, default=2048)
    ap.add_argument("--top-k", type=int, default=6)
    ap.add_argument("--seed", type=int, default=None)
    ap.add_argument("--max-resident", type=int, default=0,
                    help="cap on resident layers (0: as many as fit)")
    ap.add_argument("--cpu-seconds", type=float, default=12.0,
                    help="CPU-baseline sample length")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-subrecords", action="store_true",
                    help="config4 on one GPU: skip the configs 0-3 sub-records")
    ap.add_argument("--format", choices=["nvfp4", "ternary106", "ternary", "mxfp4", "mxfp8"],
                    default="nvfp4",
                    help="expert format: NVFP4 (the benchmark configs), the reference compressor's 106 GB "
                         "format (ternary + U8 block-64 scales + rank-16 Q8 core), config 1's "
                         "ternary + rank-16 core, MXFP4 (MTP experts), MXFP8 (shared expert); "
                         "config4 takes nvfp4 / ternary106, --workload expert all of them")
    ap.add_argument("--pool", type=int, default=64,
                    help="--workload expert: distinct experts cycled per step (> L2)")
    ap.add_argument("--exchange", choices=["p2p", "nccl"], default="p2p",
                    help="per-layer sum over ranks: NVLink peer exchange or NCCL all-reduce")
    ap.add_argument("--path", choices=["auto", "gemv", "fp4", "grouped"], default="auto",
                    help="MoE expert path: the layer's own choice (NVFP4 decode: block-scaled FP4 "
                         "tensor cores; prefill: grouped GEMM), the f16x2 GEMV slices, the FP4 "
                         "path, or the grouped GEMM")
    return ap.parse_args()


METRIC3 = "MoE expert-FFN prefill tokens/s (one NVFP4 top-6/384 layer, 8192 tokens)"


def metric_of(a):
    if a.workload == "config3":
        return METRIC3
    if a.workload == "expert":
        return (f"SwiGLU expert forwards/s ({a.format}, {a.tokens} token(s), rotating pool of "
                f"{a.pool} experts)")
    return METRIC106 if a.format == "ternary106" else METRIC


def base_config(a, world, resident):
    if a.workload == "config3":
        return {
            "workload": "config3: one NVFP4 MoE layer, prefill of 8192 tokens, top-6 of 384, " + (
                "block-scaled FP4 decode engine (six activation terms)" if getattr(a, "path", "auto") == "fp4"
                else "tensor-core grouped GEMM"),
            "hidden": a.hidden, "inter": a.inter, "experts": a.experts, "top_k": a.top_k,
            "tokens": a.tokens, "seed": a.seed,
            "router": "fp32 weights, tensor-core split-f16, sigmoid top-k; bf16-valued inputs",
            "parallelism": f"ep{world}",
            "l2": "no flush: each step streams the layer's 5.4 GB of expert weights (> 126 MB L2)",
        }
    wl = ("config4: 40-layer NVFP4 MoE-FFN stack, 256-token decode, top-6 of 384, expert-parallel"
          if a.format == "nvfp4" else
          "config4 shape with the 106 GB format: 40-layer ternary (U8 block-64 scales, rank-16 Q8 "
          "core) MoE-FFN stack, 256-token decode, top-6 of 384, expert-parallel")
    return {
        "workload": wl,
        "hidden": a.hidden, "inter": a.inter, "experts": a.experts, "top_k": a.top_k,
        "layers": a.layers, "tokens": a.tokens, "seed": a.seed,
        "router": "fp32 weights, tensor-core split-f16 (about fp32 accurate), sigmoid top-k",
        "ffn_norm": "RMSNorm, weight 1, eps 1e-20",
        "resident_layers": resident, "parallelism": f"ep{world}",
        "l2": "no flush: every layer-step streams >= 2.6 GB of expert weights (> 126 MB L2)",
    }


# --------------------------------------------------------------- CPU legs
class CpuSample:
    """The oracle (C restatement of the reference's Rayon CPU path) on a
    bounded sample of the workload: the first 4 tokens through the first 2
    layers (ffn_norm + router + top-6 + six SwiGLU experts + weighted combine
    per token, as the reference runs a decode step).  The experts the sample routes to
    are generated once, outside any timing."""

    N_TOK, N_LAY = 4, 2

    def __init__(self, a, threads: int):
        import numpy as np

        import oracle as O

        self.O, self.a, self.threads = O, a, threads
        self.n_lay = min(self.N_LAY, a.layers)
        O.set_threads(threads)
        H, I, E, K = a.hidden, a.inter, a.experts, a.top_k
        self.x = O.gen_hidden(a.seed, self.N_TOK, H)
        if a.workload == "config3":  # bf16 hidden states (round to nearest even, as torch), no ffn_norm
            u = self.x.view(np.uint32).astype(np.uint64)
            self.x = (((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)).view(np.float32)
        self.norm_w = np.ones(H, dtype=np.float32) if a.workload == "config4" else None
        self.routers, self.experts = [], {}
        xn = O.rms_norm(self.x, self.norm_w) if self.norm_w is not None else self.x
        for layer in range(self.n_lay):
            wr = O.gen_router(a.seed, layer, E, H)
            idx, _, _, _ = O.route(O.router_logits(wr, xn), K, None, 1)
            self.routers.append(wr)
            for e in set(idx.ravel().tolist()):
                self.experts[(layer, e)] = O.gen_nvfp4_expert(a.seed, layer, e, I, H)

    def first_layer_outputs(self):
        """The oracle's outputs of the sample tokens through the first layer
        (what the GPU's layer gives for the same tokens), for the parity figure
        of the CPU leg."""
        import numpy as np
        O, a = self.O, self.a
        wr = self.routers[0]
        outs = []
        for t in range(self.N_TOK):
            xt = np.ascontiguousarray(self.x[t])
            if self.norm_w is not None:
                xt = O.rms_norm(xt[None, :], self.norm_w)[0]
            idx, wt, _, _ = O.route(O.router_logits(wr, xt), a.top_k, None, 1)
            out = np.zeros(a.hidden, dtype=np.float32)
            for k in range(a.top_k):
                O.axpy(out, wt[0, k], self.experts[(0, int(idx[0, k]))].forward(xt))
            outs.append(out)
        return np.stack(outs)

    def run_once(self) -> int:
        """One pass over the sample; returns the token-layers computed."""
        import numpy as np
        O, a = self.O, self.a
        for layer in range(self.n_lay):
            wr = self.routers[layer]
            for t in range(self.N_TOK):
                xt = np.ascontiguousarray(self.x[t])
                if self.norm_w is not None:
                    xt = O.rms_norm(xt[None, :], self.norm_w)[0]
                idx, wt, _, _ = O.route(O.router_logits(wr, xt), a.top_k, None, 1)
                out = np.zeros(a.hidden, dtype=np.float32)
                for k in range(a.top_k):
                    O.axpy(out, wt[0, k], self.experts[(layer, int(idx[0, k]))].forward(xt))
        return self.n_lay * self.N_TOK

    def measure(self, seconds: float):
        """(tokens/s of the full stack, seconds, token-layers) over repeated passes."""
        t0 = time.perf_counter()
        n = 0
        while True:
            n += self.run_once()
            if time.perf_counter() - t0 >= seconds:
                break
        dt = time.perf_counter() - t0
        return 1.0 / (self.a.layers * dt / n), dt, n

    def describe(self, dt, n):
        return (f"oracle C restatement of the reference CPU path, {self.threads} threads, per-token "
                f"decode order (flash1017.rs:7259-7567): {n} token-layers ({self.N_TOK} tokens x "
                f"{self.n_lay} layers, repeated) in {dt:.1f} s, extrapolated to the {self.a.layers}-layer "
                f"stack from that sample")


def run_reference(a):
    """--impl reference: the reference's CPU algorithm (the oracle port; the
    Rust reference cannot be built here) timed on this host's cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    sample = CpuSample(a, threads)
    vals, tot_dt, tot_n = [], 0.0, 0
    for i in range(a.warmup + a.steps):
        v, dt, n = sample.measure(0.0)  # one pass over the sample per step
        if i >= a.warmup:
            vals.append(v)
            tot_dt += dt
            tot_n += n
    value = statistics.median(vals)
    desc = sample.describe(tot_dt, tot_n)
    line = {
        "impl": "reference", "metric": metric_of(a), "value": value, "unit": UNIT,
        "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": a.tokens / value * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": base_config(a, a.gpus, a.layers),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": desc},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clock/throttle samples of one GPU while running."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, bus_id: str):
        self.bus_id = bus_id
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", self.bus_id], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[0]))
                smax = float(f[1])
            except ValueError:
                continue
            for n, v in zip(names, f[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------------------- GPU arm
def run_ours(a):
    import torch

    import ffn_b200 as F
    from ep import EpStack, expert_range

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
    H, I, E, K, T, L = a.hidden, a.inter, a.experts, a.top_k, a.tokens, a.layers
    e_lo, e_hi = expert_range(rank, world, E)
    e_loc = e_hi - e_lo
    tern = a.format == "ternary106"
    fk = "ternary" if tern else "nvfp4"  # kernel kinds of the expert phases
    path = _path_code(a)
    fp4 = not tern and path in (0, 3)  # NVFP4 decode layers take the FP4 path under AUTO
    gu_kind, dn_kind = ("fp4_gateup", "fp4_down") if fp4 else (f"gateup_{fk}", f"down_{fk}")
    ebytes = (2 * tern106_mat_bytes(I, H) + tern106_mat_bytes(H, I)) if tern else EXPERT_BYTES(H, I)
    layer_bytes = e_loc * ebytes
    subs = None
    if world == 1 and not tern and not a.no_subrecords:
        # configs 0-3, measured before config 4 fills the HBM
        cs = 0.0 if a.no_cpu_baseline else min(3.0, a.cpu_seconds)
        subs = {"config0": _sub_expert(a, F, dev, "nvfp4", 0, cs),
                "config1": _sub_expert(a, F, dev, "ternary", 1, cs),
                "config2": _sub_layer(a, F, dev, 2, cs),
                "config3": _sub_layer(a, F, dev, 3, cs)}
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
    free, _ = torch.cuda.mem_get_info(dev)
    reserve = 4 << 30
    # NVFP4 layers on the FP4 path hold only their stage images (the same bytes;
    # the reference layout is generated into a scratch expert and packed); the
    # GEMV path keeps the reference layout
    images = not tern and path != F.PATH_GEMV
    per_layer = layer_bytes + 512 * e_loc
    resident = max(1, min(L, (free - reserve - L * E * H * 4) // per_layer))
    if a.max_resident:
        resident = min(resident, a.max_resident)
    if world > 1:  # every rank streams the same layer schedule
        t = torch.tensor([resident], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        resident = int(t.item())

    # ---- weights: one buffer per resident layer, carved per matrix
    n1, n1s = I * H // 2, I * H // 16
    tables = []
    buffers = []
    gen = torch.Generator(device=dev)
    gu_b = F.lib().ffn_b200_fp4_pack_bytes(I, H, 0)
    dn_b = F.lib().ffn_b200_fp4_pack_bytes(I, H, 1)
    scratch = torch.empty(3 * (n1 + n1s), dtype=torch.uint8, device=dev) if images else None
    for lay in range(resident):
        # the layer's stage images, one buffer carved per expert; or the reference layout
        buf = torch.empty(e_loc * (gu_b + dn_b) if images else layer_bytes + 512 * e_loc,
                          dtype=torch.uint8, device=dev)
        buffers.append(buf)
        experts = [None] * E
        off = 0

        def take(n, align=16):
            nonlocal off
            off = (off + align - 1) // align * align
            t = buf.narrow(0, off, n)
            off += n
            return t

        for j in range(e_loc):
            e = e_lo + j
            if images:
                experts[e] = packed_expert(F, a.seed, lay, e, I, H, scratch,
                                           buf.narrow(0, j * (gu_b + dn_b), gu_b),
                                           buf.narrow(0, j * (gu_b + dn_b) + gu_b, dn_b))
                continue
            mats = []
            for tag, (r, c) in zip((F.TAG_W1, F.TAG_W3, F.TAG_W2), ((I, H), (I, H), (H, I))):
                k = F.path_key(a.seed, lay, e, tag)
                if not tern:
                    w = buf.narrow(0, off, n1)
                    s = buf.narrow(0, off + n1, n1s)
                    off += n1 + n1s
                    F.check(F.lib().ffn_b200_gen_nvfp4(k, r, c, w.data_ptr(), s.data_ptr(),
                                                       F._stream()), "gen_nvfp4")
                    mats.append(F.Nvfp4Matrix(w, s, 1.0, r, c))
                    continue
                p = take(r * c // 4)
                rs = take(4 * r).view(torch.float32)
                bs = take(r * c // 64, 4)
                ca, cb = take(16 * c).view(torch.int8), take(16 * r).view(torch.int8)
                cas, cbs = take(64).view(torch.float32), take(64).view(torch.float32)
                F.check(F.lib().ffn_b200_gen_ternary(k, r, c, p.data_ptr(), rs.data_ptr(),
                                                     F._stream()), "gen_ternary")
                F.check(F.lib().ffn_b200_gen_core(k, r, c, ca.data_ptr(), cas.data_ptr(),
                                                  cb.data_ptr(), cbs.data_ptr(), F._stream()),
                        "gen_core")
                gen.manual_seed(k & 0x7FFFFFFFFFFFFFFF)
                bs.copy_(torch.randint(0, 256, (r * c // 64,), dtype=torch.uint8, device=dev,
                                       generator=gen))
                mats.append(F.TernaryMatrix(p, rs, r, c, core=(ca, cas, cb, cbs), bs=bs))
            experts[e] = F.SwigluExpert(F.FMT_TERNARY if tern else F.FMT_NVFP4, mats, I, H)
        tables.append((experts, F.expert_table(experts, dev)))
    routers = [F.gen_normal(F.path_key(a.seed, lay, 0, F.TAG_ROUTER), E * H, 0.02).view(E, H)
               for lay in range(L)]
    ws = F.Workspace(dev)
    norm_w = torch.ones(H, dtype=torch.float32, device=dev)
    layers = [F.MoeLayer(tables[lay % resident][0], routers[lay], H, I, top_k=K,
                         score_fn=F.SCORE_SIGMOID, expert_range=(e_lo, e_lo + e_loc),
                         table=tables[lay % resident][1], ws=ws, norm_w=norm_w,
                         norm_eps=1e-20, router_mode=F.ROUTER_TENSOR, path=path) for lay in range(L)]
    x0 = F.gen_normal(F.path_key(a.seed, 0, 0, F.TAG_X), T * H).view(T, H)
    xa = torch.empty_like(x0)
    xb = torch.empty_like(x0)
    topk = [torch.empty(T, K, dtype=torch.int32, device=dev) for _ in range(L)]
    torch.cuda.synchronize()

    capturing = [False]

    fused = [None]  # the exchange, while layers run fused with it

    def layer_fn(lay):
        def run(x_in, out, residual):
            idx = topk[lay] if capturing[0] else None
            if fused[0] is not None:
                layers[lay].forward_ep(fused[0], x_in, out, residual=residual, topk_idx=idx)
            else:
                layers[lay].forward(x_in, out=out, residual=residual, topk_idx=idx)
        return run

    exchange = None
    if world > 1 and a.exchange == "p2p":
        try:
            exchange = F.EpExchange(rank, world, T, H)
        except Exception as e:  # no peer access: NCCL all-reduce instead
            print(f"rank {rank}: NVLink peer exchange unavailable ({e}); using NCCL", file=sys.stderr)
        ok = torch.tensor([1 if exchange is not None else 0], device=dev)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        if not int(ok.item()) and exchange is not None:
            exchange.close()
            exchange = None
    ep = EpStack([layer_fn(lay) for lay in range(L)], rank, world, exchange=exchange,
                 fused=exchange is not None)
    fused[0] = exchange if ep.fused else None

    def stack(x_in, capture=False):
        capturing[0] = capture
        return ep.forward(x_in, xa, xb)

    def step():
        xa.copy_(x0)
        return stack(xa)

    # routing of the (deterministic) step -> experts hit per layer on this rank
    xa.copy_(x0)
    stack(xa, capture=True)
    torch.cuda.synchronize()
    if world > 1:  # the ranks enter the warm-up together
        dist.barrier()
    u_loc = []
    for lay in range(L):
        ids = torch.unique(topk[lay])
        u_loc.append(int(((ids >= e_lo) & (ids < e_lo + e_loc)).sum().item()))
    # gate/up kernel bytes per expert hit: NVFP4 weights + scales, or ternary
    # codes + row scales + block scales + the core's B rows (A is read by corez)
    gu_hit = 2 * (I * H // 4 + 4 * I + I * H // 64 + 16 * I) if tern else 2 * (n1 + n1s)
    gateup_bytes_step = sum(u * gu_hit for u in u_loc)
    weight_bytes_step = sum(u * ebytes for u in u_loc)

    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    if exchange is not None:  # a timed-out exchange wait: fall back to NCCL
        bad = torch.tensor([exchange.error()], device=dev)
        dist.all_reduce(bad, op=dist.ReduceOp.MAX)
        if int(bad.item()):
            print("peer exchange reported a timed-out wait; using NCCL", file=sys.stderr)
            ep.exchange = None
            ep.fused = False
            fused[0] = None
            for _ in range(a.warmup):
                step()
            torch.cuda.synchronize()
    exch_used = "nvlink-p2p" if ep.exchange is not None else ("nccl" if world > 1 else "none")
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(_bus_id(dev, local))
    if rank == 0:
        clocks.start()
        time.sleep(0.3)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    # live roofline: event pairs only around the expert GEMV kernels (fewer
    # event records between the kernels of the timed region)
    F.profile_kinds([gu_kind, dn_kind])
    F.profile_enable(True)
    n0 = F.launch_count()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record()
    for _ in range(a.steps):
        step()
    t_end.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    launches = F.launch_count() - n0
    F.profile_enable(False)
    prof = F.profile_read()
    clk = clocks.stop() if rank == 0 else None
    ms = t_start.elapsed_time(t_end)
    # per-kernel breakdown: one more (untimed) step with every kind timed
    F.profile_kinds(None)
    F.profile_enable(True)
    step()
    torch.cuda.synchronize()
    F.profile_enable(False)
    breakdown = F.profile_read()
    tt = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    ms = float(tt.item())
    ms_step = ms / a.steps
    value = T * a.steps / (ms * 1e-3)

    # ---- end to end through the public API with host buffers (the same event
    # pairs as in the timed region above, so the two numbers compare)
    x_host = x0.cpu().pin_memory()
    out_host = torch.empty_like(x_host).pin_memory()
    F.profile_kinds([gu_kind, dn_kind])
    F.profile_enable(True)
    for i in range(a.warmup + a.steps):
        if i == a.warmup:
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            e_start = torch.cuda.Event(enable_timing=True)
            e_end = torch.cuda.Event(enable_timing=True)
            e_start.record()
        xa.copy_(x_host, non_blocking=True)
        y = stack(xa)
        if rank == 0:
            out_host.copy_(y, non_blocking=True)
    e_end.record()
    torch.cuda.synchronize()
    F.profile_enable(False)
    e_ms = e_start.elapsed_time(e_end)
    te = torch.tensor([e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e = T * a.steps / (float(te.item()) * 1e-3)

    # ---- untimed checks.  (1) The timed TENSOR router's top-k sets against the
    # bit-exact EXACT router on layer 0's input.  (2) N > 1: the expert-parallel
    # output of the first two layers against the same two layers with every
    # expert on rank 0 (the part of the stack one GPU can hold).
    checks = {}
    if not tern:
        ex_layer = F.MoeLayer(tables[0][0], routers[0], H, I, top_k=K, score_fn=F.SCORE_SIGMOID,
                              expert_range=(e_lo, e_lo + e_loc), table=tables[0][1], ws=ws, norm_w=norm_w,
                              norm_eps=1e-20, router_mode=F.ROUTER_EXACT, path=path)
        ex_idx = torch.empty(T, K, dtype=torch.int32, device=dev)
        ex_layer.forward(x0, topk_idx=ex_idx)
        torch.cuda.synchronize()
        same = (torch.sort(ex_idx, 1).values == torch.sort(topk[0], 1).values).all(1)
        checks["router_tensor_vs_exact"] = {"layer": 0, "tokens": T, "same_top_k_set": int(same.sum().item())}
    if world > 1 and not tern:
        xe2 = torch.empty_like(x0)
        two = EpStack([layer_fn(lay) for lay in range(2)], rank, world, exchange=ep.exchange,
                      fused=ep.fused)
        y2 = two.forward(x0, xe2, torch.empty_like(x0))
        torch.cuda.synchronize()
        if rank == 0:
            cur = x0
            for lay in range(2):
                sc = torch.empty(3 * (n1 + n1s), dtype=torch.uint8, device=dev)
                full = [packed_expert(F, a.seed, lay, e, I, H, sc) for e in range(E)]
                lf = F.MoeLayer(full, routers[lay], H, I, top_k=K, score_fn=F.SCORE_SIGMOID, norm_w=norm_w,
                                norm_eps=1e-20, router_mode=F.ROUTER_TENSOR, path=path)
                cur = lf.forward(cur, residual=cur)
                del full, lf
            yy, rr = y2.double(), cur.double()
            err = float((yy - rr).abs().max() / rr.abs().max())
            cos = float((yy * rr).sum() / (yy.norm() * rr.norm()))
            checks["ep_vs_single_gpu"] = {"layers": 2, "max_rel_err": err, "cosine": cos,
                                          "ok": bool(err <= 1e-3 and cos >= 0.99999)}
            torch.cuda.empty_cache()
        dist.barrier()

    # ---- roofline of the dominant kernel (gate/up GEMV), live event timing
    gu_ms, gu_n = prof.get(gu_kind, (0.0, 0))
    peaks = _peaks()
    achieved = gateup_bytes_step * a.steps / (gu_ms * 1e-3) / 1e9 if gu_ms else None
    traffic = None if tern else _traffic_per_launch(gu_kind, gateup_bytes_step / L)
    kname = ("fp4_gemm_kernel<1> (tcgen05 kind::mxf4nvf4, gate+up)" if fp4 else
             f"phase_kernel<{'TERNARY' if tern else 'NVFP4'}, gate+up>")
    roof = {"bound": "hbm", "kernel": kname,
            "achieved": achieved, "peak": peaks[0], "unit": "GB/s",
            "frac": achieved / peaks[0] if achieved else None, "traffic": traffic,
            "peak_source": peaks[1],
            "algorithmic_bytes_per_launch": gateup_bytes_step / L,
            "launches": gu_n, "avg_launch_us": gu_ms * 1e3 / gu_n if gu_n else None}
    kernels = {k: {"us_per_launch_one_step": round(v[0] * 1e3 / v[1], 2), "launches": v[1]}
               for k, v in breakdown.items()}

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline and not tern:
        threads = os.cpu_count() or 1
        sample = CpuSample(a, threads)
        cv, dt, n = sample.measure(a.cpu_seconds)
        cpu = {"value": cv, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": sample.describe(dt, n)}

    if rank == 0:
        cfg = base_config(a, world, resident)
        cfg["exchange"] = exch_used
        cfg["expert_path"] = ("tcgen05 block-scaled FP4 (kind::mxf4nvf4), activations as 6 NVFP4 terms"
                              if fp4 else "warp GEMV slices, f16x2 activations")
        cfg["experts_hit_per_layer_rank0"] = u_loc
        cfg["weight_bytes_per_step_rank0"] = weight_bytes_step
        line = {
            "metric": metric_of(a), "value": value, "unit": UNIT, "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": ("ternary (block-64 U8 scales, rank-16 Q8 core) weights x f16x2 split "
                      "activations, f32 accumulate" if tern else
                      "nvfp4 weights x 6-term nvfp4 activations (tcgen05 block-scaled FP4 MMA), f32 "
                      "accumulate" if fp4 else
                      "nvfp4 weights x f16x2 split activations, f32 accumulate"),
            "data": "synthetic (seeded random-init weights and N(0,1) hidden states)",
            "config": cfg,
            "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": T * H * 4,
                    "d2h_bytes_per_step": T * H * 4},
            "gpu_launches": launches,
            "roofline": roof,
            "cpu_baseline": cpu,
            "clocks": clk,
            "kernels": kernels,
            "hbm_weight_gbs_rank0": weight_bytes_step / (ms_step * 1e-3) / 1e9,
        }
        if subs is not None:
            line["configs"] = subs
        line["checks"] = checks
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_prefill(a):
    """Config 3: one MoE layer over 8192 prefill tokens on the grouped GEMM."""
    import torch

    import ffn_b200 as F
    from ep import expert_range

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
    H, I, E, K, T = a.hidden, a.inter, a.experts, a.top_k, a.tokens
    e_lo, e_hi = expert_range(rank, world, E)
    fp4 = a.path == "fp4"  # the block-scaled FP4 decode engine instead of the grouped GEMM
    experts = [None] * E
    for e in range(e_lo, e_hi):
        experts[e] = F.SwigluExpert.generate(F.FMT_NVFP4, a.seed, 0, e, I, H)
        if fp4:
            experts[e].pack_fp4()
    wr = F.gen_normal(F.path_key(a.seed, 0, 0, F.TAG_ROUTER), E * H, 0.02).view(E, H)
    layer = F.MoeLayer(experts, wr, H, I, top_k=K, score_fn=F.SCORE_SIGMOID,
                       router_mode=F.ROUTER_TENSOR, expert_range=(e_lo, e_hi), path=_path_code(a))
    x0 = F.gen_normal(F.path_key(a.seed, 0, 0, F.TAG_X), T * H).view(T, H)
    x0 = x0.to(torch.bfloat16).to(torch.float32)  # config 3: bf16 hidden states
    out = torch.empty_like(x0)
    idx = torch.empty(T, K, dtype=torch.int32, device=dev)
    layer.forward(x0, out=out, topk_idx=idx)
    torch.cuda.synchronize()
    checks = None
    if fp4 and world == 1:
        # untimed: the FP4 path's layer output against the grouped GEMM's (whose
        # config-3 outputs the GPU tests pin to the oracle), all tokens
        ref_layer = F.MoeLayer(experts, wr, H, I, top_k=K, score_fn=F.SCORE_SIGMOID,
                               router_mode=F.ROUTER_TENSOR, expert_range=(e_lo, e_hi), path=F.PATH_GROUPED)
        ref = torch.empty_like(x0)
        ref_layer.forward(x0, out=ref, topk_idx=idx)
        torch.cuda.synchronize()
        err = float((out - ref).abs().max() / ref.abs().max())
        cos = float(torch.nn.functional.cosine_similarity(out.double().flatten(), ref.double().flatten(), dim=0))
        checks = {"fp4_vs_grouped": {"tokens": T, "max_rel_err": err, "cosine": cos}}
        del ref_layer, ref
    ids, cnt = torch.unique(idx, return_counts=True)
    local_pairs = int(cnt[(ids >= e_lo) & (ids < e_hi)].sum().item())

    def step():
        layer.forward(x0, out=out)
        if world > 1:
            dist.all_reduce(out)

    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(_bus_id(dev, local))
    if rank == 0:
        clocks.start()
        time.sleep(0.3)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    F.profile_enable(True)
    n0 = F.launch_count()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(a.steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    launches = F.launch_count() - n0
    F.profile_enable(False)
    prof = F.profile_read()
    clk = clocks.stop() if rank == 0 else None
    tt = torch.tensor([t0.elapsed_time(t1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    ms = float(tt.item())
    ms_step = ms / a.steps
    value = T * a.steps / (ms * 1e-3)

    # end to end: host x in, host out back, every step
    x_host = x0.cpu().pin_memory()
    out_host = torch.empty_like(x_host).pin_memory()
    xd = torch.empty_like(x0)
    F.profile_enable(True)
    for i in range(a.warmup + a.steps):
        if i == a.warmup:
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
        xd.copy_(x_host, non_blocking=True)
        layer.forward(xd, out=out)
        if world > 1:
            dist.all_reduce(out)
        if rank == 0:
            out_host.copy_(out, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    F.profile_enable(False)
    te = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e = T * a.steps / (float(te.item()) * 1e-3)

    # roofline: gate/up GEMM, algorithmic FLOPs of this rank's pairs
    gu_ms, gu_n = prof.get("fp4_gateup" if fp4 else "gemm_gateup", (0.0, 0))
    gu_flop = 2.0 * local_pairs * 2 * H * I
    peak, src = _tensor_peak()
    if fp4:
        peak, src = 9000.0, "nominal dense FP4 (9 PFLOP/s; no measured FP4 peak on this pool)"
    achieved = gu_flop * gu_n / (gu_ms * 1e-3) / 1e12 if gu_ms else None
    dn_ms, dn_n = prof.get("fp4_down" if fp4 else "gemm_down", (0.0, 0))
    dn_tf = 2.0 * local_pairs * H * I * dn_n / (dn_ms * 1e-3) / 1e12 if dn_ms else None
    roof = {"bound": "tensor",
            "kernel": ("fp4_gemm_kernel<1> (gate+up, tcgen05 kind::mxf4nvf4, six activation terms, "
                       "chunks of <= 8 tokens)" if fp4 else "grouped gemm_kernel<1> (gate+up, tcgen05 kind::f16)"),
            "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
            "frac": achieved / peak if achieved else None, "traffic": None, "peak_source": src,
            "algorithmic_flop_per_launch": gu_flop, "launches": gu_n,
            "avg_launch_us": gu_ms * 1e3 / gu_n if gu_n else None,
            "down_tflops": dn_tf,
            "fp4_dense_nominal_tflops": 9000.0,
            "note": ("FP4 x FP4 MMAs with the activations as six NVFP4 residual terms: the tensor "
                     "cores do six times the algorithmic FLOPs, and every <= 8-token chunk of an "
                     "expert streams the expert's weights again" if fp4 else
                     "f16 operands (weights dequantised exactly in TMEM); FP4 block-scaled MMA "
                     "needs FP4 activations: one term is outside the 1e-3 tolerance, six terms "
                     "cost six times the tensor work (--path fp4 measures that engine here)")}
    kernels = {k: {"ms": round(v[0], 3), "launches": v[1]} for k, v in prof.items()}
    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        threads = os.cpu_count() or 1
        sample = CpuSample(a, threads)
        cv, dt, n = sample.measure(a.cpu_seconds)
        cpu = {"value": cv, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": sample.describe(dt, n)}
    if rank == 0:
        cfg = base_config(a, world, 1)
        cfg["routed_pairs_rank0"] = local_pairs
        line = {
            "metric": METRIC3, "value": value, "unit": UNIT, "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": ("nvfp4 weights x 6-term nvfp4 activations (tcgen05 block-scaled FP4 MMA), f32 accumulate"
                      if fp4 else "nvfp4 weights dequantised to f16 x f16 activations, f32 accumulate"),
            "data": "synthetic (seeded random-init weights, bf16-valued N(0,1) hidden states)",
            "config": cfg,
            "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": T * H * 4,
                    "d2h_bytes_per_step": T * H * 4},
            "gpu_launches": launches, "roofline": roof, "cpu_baseline": cpu, "clocks": clk,
            "kernels": kernels,
            "tflops_layer": 2.0 * T * K * 3 * H * I / (ms_step * 1e-3) / 1e12,
        }
        if checks:
            line["checks"] = checks
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def _tensor_peak():
    try:
        d = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        return float(d["bf16_tflops"]), "measured dense bf16 burst (MEASURED_PEAKS.json bf16_tflops)"
    except (OSError, KeyError, ValueError):
        return 1590.0, "fallback (1.59 PFLOP/s)"


def _bus_id(dev, local):
    """nvidia-smi -i selector of this rank's GPU (its UUID when torch knows it)."""
    import torch
    try:
        uuid = str(torch.cuda.get_device_properties(dev).uuid)
        if uuid:
            return uuid if uuid.startswith("GPU-") else "GPU-" + uuid
    except Exception:
        pass
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        return vis.split(",")[local]
    return str(local)


def _peaks():
    try:
        d = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback (6.65 TB/s)"


def _traffic_per_launch(kind, alg_bytes_per_launch):
    """DRAM bytes per launch of the gate/up kernel `kind` from its committed
    ncu summary (profiles/<kind>.json: measured traffic / algorithmic bytes of
    the captured launch), scaled to this launch's algorithmic bytes; None when
    no capture of that kernel is committed."""
    name = {"gateup_nvfp4": "gateup_nvfp4.json", "fp4_gateup": "fp4_gateup_nvfp4.json"}.get(kind)
    if name is None:
        return None
    try:
        d = json.load(open(os.path.join(ROOT, "profiles", name)))
        return alg_bytes_per_launch * float(d["traffic_over_algorithmic"])
    except (OSError, KeyError, ValueError):
        return None


def packed_expert(F, seed, layer, expert, I, H, scratch, gu=None, dn=None):
    """An NVFP4 expert of the stack as the FP4 path holds it: the seeded
    reference layout generated into `scratch` (reused), packed into stage
    images (gu / dn, or new tensors); the expert keeps only the images and its
    global scales (its reference-layout pointers are NULL, so a layer of such
    experts runs only the FP4 path)."""
    n1, n1s = I * H // 2, I * H // 16
    mats = []
    off = 0
    for tag, (r, c) in zip((F.TAG_W1, F.TAG_W3, F.TAG_W2), ((I, H), (I, H), (H, I))):
        w, s = scratch.narrow(0, off, n1), scratch.narrow(0, off + n1, n1s)
        off += n1 + n1s
        F.check(F.lib().ffn_b200_gen_nvfp4(F.path_key(seed, layer, expert, tag), r, c, w.data_ptr(),
                                           s.data_ptr(), F._stream()), "gen_nvfp4")
        mats.append(F.Nvfp4Matrix(w, s, 1.0, r, c))
    ex = F.SwigluExpert(F.FMT_NVFP4, mats, I, H).pack_fp4(gu, dn)
    for m in ex.mats:
        m.w = m.s = None
    return ex


def _path_code(a):
    import ffn_b200 as F
    return {"auto": F.PATH_AUTO, "gemv": F.PATH_GEMV, "fp4": F.PATH_FP4,
            "grouped": F.PATH_GROUPED}[a.path]


# --------------------------------------------------------------- one expert
def _expert_mat_bytes(fmt, r, c):
    if fmt == "nvfp4":
        return r * c // 2 + r * c // 16
    if fmt == "mxfp4":
        return r * c // 2 + r * c // 32
    if fmt == "mxfp8":
        return r * c + ((r + 31) // 32) * (c // 32)
    if fmt == "ternary106":
        return tern106_mat_bytes(r, c)
    return r * c // 4 + 4 * r + 16 * r + 16 * c + 128  # ternary + rank-16 core (config 1)


def run_expert(a):
    """Benchmark configs 0 (NVFP4) and 1 (ternary + rank-16 core) and the other
    expert formats: one SwiGLU expert forward over `tokens` rows, cycling
    through a pool of distinct experts larger than L2 (a step = one pass over
    the pool); roofline = the expert's weight bytes over HBM."""
    import numpy as np
    import torch

    import ffn_b200 as F
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    H, I, T, P = a.hidden, a.inter, a.tokens, a.pool
    fmt = a.format
    shapes = ((I, H), (I, H), (H, I))
    ebytes = sum(_expert_mat_bytes(fmt, r, c) for r, c in shapes)
    gen = torch.Generator(device=dev)
    experts = []
    for e in range(P):
        keys = [F.path_key(a.seed, 0, e, tag) for tag in (F.TAG_W1, F.TAG_W3, F.TAG_W2)]
        if fmt == "nvfp4":
            experts.append(F.SwigluExpert.generate(F.FMT_NVFP4, a.seed, 0, e, I, H))
        elif fmt in ("ternary", "ternary106"):
            ex = F.SwigluExpert.generate(F.FMT_TERNARY, a.seed, 0, e, I, H, with_core=True)
            if fmt == "ternary106":
                for k, m in zip(keys, ex.mats):
                    gen.manual_seed(k & 0x7FFFFFFFFFFFFFFF)
                    m.bs = torch.randint(0, 256, (m.rows * m.cols // 64,), dtype=torch.uint8,
                                         device=dev, generator=gen)
            experts.append(ex)
        else:
            mats = []
            for k, (r, c) in zip(keys, shapes):
                gen.manual_seed(k & 0x7FFFFFFFFFFFFFFF)
                if fmt == "mxfp4":
                    w = torch.randint(0, 256, (r * c // 2,), dtype=torch.uint8, device=dev, generator=gen)
                    sc = torch.randint(110, 131, (r * c // 32,), dtype=torch.uint8, device=dev, generator=gen)
                    mats.append(F.Mxfp4Matrix(w, sc, F.Mxfp4Matrix.bias_for(sc), r, c))
                else:
                    w = torch.randint(0, 256, (r * c,), dtype=torch.uint8, device=dev, generator=gen)
                    w[(w & 0x7F) == 0x7F] = 0x38  # no E4M3 NaN codes
                    sc = torch.randint(118, 131, (((r + 31) // 32) * (c // 32),), dtype=torch.uint8,
                                       device=dev, generator=gen)
                    mats.append(F.Mxfp8Matrix(w, sc, F.Mxfp8Matrix.bias_for(sc), r, c))
            experts.append(F.SwigluExpert(F.FMT_MXFP4 if fmt == "mxfp4" else F.FMT_MXFP8, mats, I, H))
    x = F.gen_normal(F.path_key(a.seed, 0, 0, F.TAG_X), T * H).view(T, H)
    out = torch.zeros(T, H, dtype=torch.float32, device=dev)

    def step():
        for ex in experts:
            ex.forward(x, out=out, weight=1.0, accumulate=True)

    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    clocks = ClockSampler(_bus_id(dev, 0))
    clocks.start()
    time.sleep(0.3)
    n0 = F.launch_count()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t0.record()
    for _ in range(a.steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    launches = F.launch_count() - n0
    ms_eager = t0.elapsed_time(t1)
    # the same pass captured once in a CUDA graph and replayed: the library's
    # launches back to back, without the Python call overhead between them
    gms = _graph_ms(step, a.steps, a.warmup)
    clk = clocks.stop()
    ms = gms * a.steps if gms is not None else ms_eager
    fwd = P * a.steps
    value = fwd / (ms * 1e-3)
    us_fwd = ms * 1e3 / fwd
    # end to end: the step's x uploaded from pinned host memory, out read back
    x_host = x.cpu().pin_memory()
    o_host = torch.empty_like(x_host).pin_memory()
    for i in range(a.warmup + a.steps):
        if i == a.warmup:
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
        x.copy_(x_host, non_blocking=True)
        step()
        o_host.copy_(out, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    e2e = fwd / (e0.elapsed_time(e1) * 1e-3)
    # per-kernel breakdown of one step
    F.profile_kinds(None)
    F.profile_enable(True)
    step()
    torch.cuda.synchronize()
    F.profile_enable(False)
    kernels = {k: {"us_per_launch": round(v[0] * 1e3 / v[1], 2), "launches": v[1]}
               for k, v in F.profile_read().items()}
    peaks = _peaks()
    achieved = ebytes / (us_fwd * 1e-6) / 1e9
    cpu = None
    if not a.no_cpu_baseline:
        import oracle as O
        O.set_threads(os.cpu_count() or 1)
        e0h = experts[0]
        if fmt == "nvfp4":
            oe = O.Nvfp4Expert(I, H, tuple(m.w.cpu().numpy() for m in e0h.mats),
                               tuple(m.s.cpu().numpy() for m in e0h.mats),
                               tuple(m.gs for m in e0h.mats))
        elif fmt in ("ternary", "ternary106"):
            cores = tuple(O.Core(m.core[0].cpu().numpy(), m.core[1].cpu().numpy(),
                                 m.core[2].cpu().numpy(), m.core[3].cpu().numpy()) for m in e0h.mats)
            bs = tuple(m.bs.cpu().numpy() for m in e0h.mats) if fmt == "ternary106" else None
            oe = O.TernaryExpert(I, H, tuple(m.p.cpu().numpy() for m in e0h.mats),
                                 tuple(m.rs.cpu().numpy() for m in e0h.mats), cores, 1.0, bs)
        else:
            oe = O.MxExpert(3 if fmt == "mxfp4" else 4, I, H, tuple(m.w.cpu().numpy() for m in e0h.mats),
                            tuple(m.s.cpu().numpy() for m in e0h.mats))
        xs = x.cpu().numpy()
        n, c0 = 0, time.perf_counter()
        while time.perf_counter() - c0 < min(a.cpu_seconds, 6.0):
            for t in range(T):
                oe.forward(np.ascontiguousarray(xs[t]))
            n += 1
        dt = time.perf_counter() - c0
        cpu = {"value": n / dt, "unit": "expert forwards/s", "cores": os.cpu_count() or 1,
               "kind": "port", "sample": f"oracle expert forward over the same {T} token(s), {n} "
                                         f"repetitions in {dt:.1f} s"}
    line = {
        "metric": metric_of(a), "value": value, "unit": "expert forwards/s", "n_gpus": 1,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms / a.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None,
        "dtype": (f"{fmt} weights x f32 activations, f32 accumulate (CUDA-core decode kernels)"
                  if fmt in ("nvfp4", "mxfp4") and T <= 8 else
                  f"{fmt} weights x f16x2 split activations, f32 accumulate"),
        "data": "synthetic (seeded random-init weights and N(0,1) hidden states)",
        "config": {"workload": f"one SwiGLU expert ({fmt}), {T} token(s), pool of {P} experts "
                               f"({P * ebytes / 1e9:.2f} GB > 126 MB L2)",
                   "hidden": H, "inter": I, "tokens": T, "pool": P, "seed": a.seed,
                   "l2": "no flush: the pool exceeds L2, every forward reads its weights from HBM",
                   "timing": ("CUDA graph of one pass over the pool, replayed; eager calls: "
                              f"{ms_eager * 1e3 / fwd:.2f} us per forward") if gms is not None
                             else "eager calls"},
        "e2e": {"value": e2e, "unit": "expert forwards/s", "h2d_bytes_per_step": T * H * 4,
                "d2h_bytes_per_step": T * H * 4},
        "gpu_launches": launches,
        "roofline": {"bound": "hbm", "kernel": f"expert forward ({fmt}, all its launches)",
                     "achieved": achieved, "peak": peaks[0], "unit": "GB/s", "frac": achieved / peaks[0],
                     "traffic": None, "peak_source": peaks[1], "algorithmic_bytes_per_forward": ebytes,
                     "us_per_forward": us_fwd},
        "cpu_baseline": cpu,
        "clocks": clk,
        "kernels": kernels,
    }
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------- configs 0-3
# Sub-records of the default (config 4) run on one GPU: the other benchmark
# configurations measured in the same process, before config 4 fills the HBM,
# each with its own roofline, an oracle CPU sample and the parity of the
# sampled tokens against that sample's oracle outputs (the CPU leg, where the
# oracle serves as the checker).

def _event_ms(step, steps, warmup):
    """Device ms per step: CUDA events on the current stream, synchronised on both sides."""
    import torch
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    return t0.elapsed_time(t1) / steps


def _graph_ms(step, steps, warmup):
    """Device ms per step with step() captured once in a CUDA graph and replayed
    (the library's own launches, without the Python call overhead between
    them); None when the capture fails."""
    import torch
    try:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            step()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            step()
        ms = _event_ms(g.replay, steps, warmup)
        del g
        return ms
    except Exception:  # noqa: BLE001 -- capture unsupported: eager timing stands
        torch.cuda.synchronize()
        return None


def _cpu_rate(fn, seconds):
    """(calls/s, calls, seconds) of fn() repeated for about `seconds`."""
    t0 = time.perf_counter()
    n = 0
    while True:
        fn()
        n += 1
        dt = time.perf_counter() - t0
        if dt >= seconds:
            return n / dt, n, dt


def _parity(O, y, ref, what):
    e, c = O.max_rel_err(y, ref), O.cosine(y, ref)
    return {"checked": what, "max_rel_err": e, "cosine": c,
            "ok": bool(e <= O.REL_TOL and c >= O.COS_TOL),
            "tolerance": f"max|y-ref|/max|ref| <= {O.REL_TOL}, cosine >= {O.COS_TOL}"}


def _host(t):
    import numpy as np
    return np.ascontiguousarray(t.detach().cpu().numpy())


def _sub_expert(a, F, dev, fmt, seed, cpu_s):
    """Config 0 (NVFP4) or 1 (ternary + rank-16 core): one SwiGLU expert, one
    token, cycling through 64 distinct experts (906 / 424 MB, > L2)."""
    import torch
    H, I, pool = a.hidden, a.inter, 64
    tern = fmt == "ternary"
    experts = [F.SwigluExpert.generate(F.FMT_TERNARY if tern else F.FMT_NVFP4, seed, 0, e, I, H,
                                       **({"with_core": True} if tern else {})) for e in range(pool)]
    x = F.gen_normal(F.path_key(seed, 0, 0, F.TAG_X), H).view(1, H)
    out = torch.zeros(1, H, dtype=torch.float32, device=dev)

    def step():
        for ex in experts:
            ex.forward(x, out=out, weight=1.0, accumulate=True)

    us_eager = _event_ms(step, 20, 3) * 1e3 / pool
    gms = _graph_ms(step, 20, 3)
    us = gms * 1e3 / pool if gms is not None else us_eager
    ebytes = sum(_expert_mat_bytes(fmt, r, c) for r, c in ((I, H), (I, H), (H, I)))
    peak, src = _peaks()
    gbs = ebytes / (us * 1e-6) / 1e9
    rec = {"workload": f"config{1 if tern else 0}: one {'ternary + rank-16 Q8 core' if tern else 'NVFP4'} "
                       f"SwiGLU expert, batch-1 decode, H {H}, I {I}, seed {seed}, pool of {pool} experts",
           "metric": "expert forwards/s", "value": 1e6 / us, "us_per_forward": us,
           "timing": ("CUDA graph of one pass over the pool (64 ffn_b200_expert_forward calls), replayed"
                      if gms is not None else "eager calls"),
           "us_per_forward_eager": us_eager,
           "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                        "peak_source": src, "algorithmic_bytes_per_forward": ebytes}}
    y = _host(experts[0].forward(x))[0]
    if cpu_s > 0:
        import numpy as np
        import oracle as O  # the CPU leg: baseline and checker
        O.set_threads(os.cpu_count() or 1)
        e0 = experts[0]
        if tern:
            cores = tuple(O.Core(*(_host(t) for t in m.core)) for m in e0.mats)
            oe = O.TernaryExpert(I, H, tuple(_host(m.p) for m in e0.mats), tuple(_host(m.rs) for m in e0.mats),
                                 cores, e0.proj_scale)
        else:
            oe = O.Nvfp4Expert(I, H, tuple(_host(m.w) for m in e0.mats), tuple(_host(m.s) for m in e0.mats),
                               tuple(m.gs for m in e0.mats))
        xs = np.ascontiguousarray(_host(x)[0])
        rate, n, dt = _cpu_rate(lambda: oe.forward(xs), cpu_s)
        rec["cpu_baseline"] = {"value": rate, "unit": "expert forwards/s", "cores": os.cpu_count() or 1,
                               "kind": "port", "sample": f"oracle expert forward, 1 token, {n} calls in {dt:.1f} s"}
        rec["parity"] = _parity(O, y, oe.forward(xs), "expert 0, token 0, against the oracle")
    del experts
    torch.cuda.empty_cache()
    return rec


def _sub_layer(a, F, dev, cfg, cpu_s):
    """Config 2 (one NVFP4 MoE layer, 64-token decode, sigmoid top-6 of 384,
    seed 2: the block-scaled FP4 path) or config 3 (8192-token prefill,
    bf16-valued hidden states, seed 3: the grouped GEMM)."""
    import copy

    import torch
    H, I, E, K = a.hidden, a.inter, a.experts, a.top_k
    T, seed = (64, 2) if cfg == 2 else (8192, 3)
    experts = [F.SwigluExpert.generate(F.FMT_NVFP4, seed, 0, e, I, H) for e in range(E)]
    if cfg == 2:  # the decode layer runs on the FP4 path's stage images
        experts = [e.pack_fp4() for e in experts]
    wr = F.gen_normal(F.path_key(seed, 0, 0, F.TAG_ROUTER), E * H, 0.02).view(E, H)
    layer = F.MoeLayer(experts, wr, H, I, top_k=K, score_fn=F.SCORE_SIGMOID, router_mode=F.ROUTER_TENSOR)
    x = F.gen_normal(F.path_key(seed, 0, 0, F.TAG_X), T * H).view(T, H)
    if cfg == 3:
        x = x.to(torch.bfloat16).to(torch.float32)
    out = torch.empty_like(x)
    idx = torch.empty(T, K, dtype=torch.int32, device=dev)
    layer.forward(x, out=out, topk_idx=idx)
    torch.cuda.synchronize()
    hit = int(torch.unique(idx).numel())
    kinds = ("fp4_gateup", "fp4_down") if cfg == 2 else ("gemm_gateup", "gemm_down")
    F.profile_kinds(list(kinds))
    F.profile_enable(True)
    ms = _event_ms(lambda: layer.forward(x, out=out), 10 if cfg == 2 else 5, 3)
    F.profile_enable(False)
    prof = F.profile_read()
    F.profile_kinds(None)
    gu_ms, gu_n = prof.get(kinds[0], (0.0, 0))
    gu_us = gu_ms * 1e3 / gu_n if gu_n else None
    rec = {"workload": (f"config2: one NVFP4 MoE layer, decode batch of 64 tokens, sigmoid top-6 of {E}, "
                        f"seed 2, block-scaled FP4 path" if cfg == 2 else
                        f"config3: one NVFP4 MoE layer, prefill of 8192 bf16-valued tokens, top-6 of {E}, "
                        f"seed 3, tensor-core grouped GEMM"),
           "metric": "tokens/s", "value": T / (ms * 1e-3), "ms_per_layer": ms, "experts_hit": hit,
           "l2": "no flush: each pass streams the hit experts' weights (> 126 MB L2)"}
    if cfg == 2:
        peak, src = _peaks()
        gbs = hit * 2 * (I * H // 2 + I * H // 16) / (gu_us * 1e-6) / 1e9 if gu_us else None
        rec["roofline"] = {"bound": "hbm", "kernel": "fp4_gemm_kernel<1> (gate+up)", "achieved": gbs,
                           "peak": peak, "unit": "GB/s", "frac": gbs / peak if gbs else None,
                           "peak_source": src, "avg_launch_us": gu_us}
    else:
        peak, src = _tensor_peak()
        tf = 2.0 * T * K * 2 * H * I / (gu_us * 1e-6) / 1e12 if gu_us else None
        rec["roofline"] = {"bound": "tensor", "kernel": "grouped gemm_kernel<1> (gate+up, tcgen05 kind::f16)",
                           "achieved": tf, "peak": peak, "unit": "TFLOP/s", "frac": tf / peak if tf else None,
                           "peak_source": src, "avg_launch_us": gu_us,
                           "layer_tflops": 2.0 * T * K * 3 * H * I / (ms * 1e-3) / 1e12}
    if cpu_s > 0:
        import oracle as O  # the CPU leg: baseline and checker
        b = copy.copy(a)
        b.workload, b.tokens, b.seed, b.layers = ("config3" if cfg == 3 else "config2"), T, seed, 1
        sample = CpuSample(b, os.cpu_count() or 1)
        cv, dt, n = sample.measure(cpu_s)
        rec["cpu_baseline"] = {"value": cv, "unit": "tokens/s", "cores": os.cpu_count() or 1, "kind": "port",
                               "sample": sample.describe(dt, n)}
        got = _host(out)[: CpuSample.N_TOK]
        rec["parity"] = _parity(O, got, sample.first_layer_outputs(),
                                f"tokens 0-{CpuSample.N_TOK - 1} of the layer against the oracle")
    del experts, layer
    torch.cuda.empty_cache()
    return rec


def run_compress(a):
    """The 106 GB format's compressor (flash1017.rs:10377-10645) on the GPU: a
    step compresses every NVFP4 matrix of a pool of experts (gate, up, down of
    each) into ternary codes + block-64 scales + the rank-16 Q8 core."""
    import ctypes as C

    import numpy as np
    import torch

    import ffn_b200 as F
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    H, I, P = a.hidden, a.inter, a.pool
    shapes = ((I, H), (I, H), (H, I))
    experts = [F.SwigluExpert.generate(F.FMT_NVFP4, a.seed, 0, e, I, H) for e in range(P)]
    L = F.lib()
    jobs = []  # (matrix, rows, cols, outputs)
    for e, ex in enumerate(experts):
        for k, (m, (r, c)) in enumerate(zip(ex.mats, shapes)):
            outs = (torch.empty(r * c // 4, dtype=torch.uint8, device=dev),
                    torch.empty(r, dtype=torch.float32, device=dev),
                    torch.empty(r * c // 64, dtype=torch.uint8, device=dev),
                    torch.empty(r * 16, dtype=torch.int8, device=dev),
                    torch.empty(16, dtype=torch.float32, device=dev),
                    torch.empty(16 * c, dtype=torch.int8, device=dev),
                    torch.empty(16, dtype=torch.float32, device=dev))
            jobs.append((m, r, c, outs, 1000 * e + k))
    ws = torch.empty(max(L.ffn_b200_compress_ws_bytes(r, c) for r, c in shapes), dtype=torch.uint8,
                     device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    ptr = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731

    def step():
        for m, r, c, o, seed in jobs:
            rc = L.ffn_b200_compress_ternary_b64(r, c, ptr(m.w), ptr(m.s), float(m.gs), seed, *map(ptr, o),
                                                 ptr(ws), ws.numel(), C.c_void_p(stream))
            if rc:
                raise RuntimeError(L.ffn_b200_last_error().decode())

    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    clocks = ClockSampler(_bus_id(dev, 0))
    clocks.start()
    time.sleep(0.3)
    n0 = F.launch_count()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(a.steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    launches = F.launch_count() - n0
    clk = clocks.stop()
    ms = t0.elapsed_time(t1)
    n_exp = P * a.steps
    value = n_exp / (ms * 1e-3)
    in_b = sum(r * c // 2 + r * c // 16 for r, c in shapes)
    out_b = sum(r * c // 4 + r * 4 + r * c // 64 + 16 * (r + c) + 128 for r, c in shapes)
    achieved = (in_b + out_b) * n_exp / (ms * 1e-3) / 1e9
    # end to end: each matrix's NVFP4 bytes uploaded from pinned host memory, the outputs read back
    w_h = [m.w.cpu().pin_memory() for m, *_ in jobs]
    s_h = [m.s.cpu().pin_memory() for m, *_ in jobs]
    o_h = [[t.cpu().pin_memory() for t in o] for _, _, _, o, _ in jobs]
    for i in range(a.warmup + a.steps):
        if i == a.warmup:
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
        for j, (m, r, c, o, seed) in enumerate(jobs):
            m.w.copy_(w_h[j], non_blocking=True)
            m.s.copy_(s_h[j], non_blocking=True)
        step()
        for j, (_, _, _, o, _) in enumerate(jobs):
            for hdst, dsrc in zip(o_h[j], o):
                hdst.copy_(dsrc, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    e2e = n_exp / (e0.elapsed_time(e1) * 1e-3)
    peaks = _peaks()
    cpu = None
    if not a.no_cpu_baseline:
        import oracle as O
        m, r, c, _, seed = jobs[0]
        w0, s0 = m.w.cpu().numpy(), m.s.cpu().numpy()
        n, c0 = 0, time.perf_counter()
        while n == 0 or time.perf_counter() - c0 < min(a.cpu_seconds, 6.0):
            O.compress_ternary_b64(w0, s0, m.gs, r, c, seed)
            n += 1
        dt = time.perf_counter() - c0
        cpu = {"value": n / dt / 3, "unit": "expert compressions/s", "cores": 1, "kind": "port",
               "sample": f"oracle compression of one {r}x{c} matrix, {n} times in {dt:.1f} s "
                         f"(an expert = 3 matrices of that size)"}
    line = {
        "metric": f"106 GB-format expert compressions/s (3 NVFP4 matrices of {I}x{H} each)",
        "value": value, "unit": "expert compressions/s", "n_gpus": 1, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": ms / a.steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32 (bit-exact to the reference's f32 compressor)",
        "data": "synthetic (seeded random-init NVFP4 experts)",
        "config": {"workload": f"compressor: pool of {P} NVFP4 experts per step", "hidden": H, "inter": I,
                   "pool": P, "seed": a.seed,
                   "l2": "no flush: each matrix's workspace residual is written and read twice per call"},
        "e2e": {"value": e2e, "unit": "expert compressions/s", "h2d_bytes_per_step": in_b * P,
                "d2h_bytes_per_step": out_b * P},
        "gpu_launches": launches,
        "roofline": {"bound": "hbm", "kernel": "compressor (all its launches)", "achieved": achieved,
                     "peak": peaks[0], "unit": "GB/s", "frac": achieved / peaks[0], "traffic": None,
                     "peak_source": peaks[1], "algorithmic_bytes_per_expert": in_b + out_b},
        "cpu_baseline": cpu,
        "clocks": clk,
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    a = parse_args()
    if a.workload == "compress":
        if a.seed is None:
            a.seed = 5
        if a.pool == 64:
            a.pool = 8
        if a.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "--workload compress has no "
                              "reference arm; its cpu_baseline times the oracle"}))
            return 0
        return run_compress(a)
    if a.workload == "expert":
        for k, v in (("tokens", 1), ("layers", 1), ("seed", 0 if a.format == "nvfp4" else 1)):
            if getattr(a, k) is None:
                setattr(a, k, v)
        if a.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "--workload expert has no "
                              "reference arm; its cpu_baseline times the oracle"}))
            return 0
        return run_expert(a)
    if a.workload == "config3":
        for k, v in (("tokens", 8192), ("layers", 1), ("seed", 3)):
            if getattr(a, k) is None:
                setattr(a, k, v)
    else:
        for k, v in (("tokens", 256), ("layers", 40), ("seed", 4)):
            if getattr(a, k) is None:
                setattr(a, k, v)
    if a.impl == "reference":
        return run_reference(a)
    if a.workload == "config3":
        return run_prefill(a)
    return run_ours(a)


if __name__ == "__main__":
    sys.exit(main())
