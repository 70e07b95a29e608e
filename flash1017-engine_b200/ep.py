"""Expert parallelism of the MoE-FFN stack over the GPUs of one node.

Rank r of N owns the contiguous expert block [r*E/N, (r+1)*E/N) of every layer
(static EP, 48 of 384 experts per rank at N = 8).  Router weights are
replicated, so every rank computes the routing of every token itself and
knows, without a count exchange, which of its experts each token uses.  A
layer on rank r computes

    out_r[t] = sum over t's top-k experts e owned by r of w[t,e] * expert_e(x[t])
               (+ x[t], the residual, on rank 0 only)

and one sum all-reduce over the ranks gives every rank the full layer output
sum_r out_r = x + sum_e w * expert_e(x), the input of the next layer
(reference: the decode MoE block of crates/flash-core/src/flash1017.rs:7277-7567,
residual add as in flash1017.rs:4900-4905).  The all-reduce carries
tokens x hidden fp32 values per layer (4 MB at 256 tokens x 4096), which is
latency-bound on NVLink; the expert weights, 5.3 GB per layer, never move.

The collective is whatever torch.distributed backend the process group runs:
NCCL over NVLink on GPUs, gloo on CPU (the tests).
"""
from __future__ import annotations

from typing import Callable, Optional, Sequence, Tuple


def expert_range(rank: int, world: int, n_experts: int) -> Tuple[int, int]:
    """[begin, end) of the experts rank `rank` owns; n_experts % world == 0."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if n_experts % world:
        raise ValueError(f"{n_experts} experts do not divide over {world} ranks")
    per = n_experts // world
    return rank * per, (rank + 1) * per


# layer(x_in, out, residual_or_None) writes this rank's partial layer output
LayerFn = Callable[[object, object, Optional[object]], None]


class EpStack:
    """A stack of MoE layers run expert-parallel: per layer, this rank's partial
    output, then the sum over ranks.  The sum is either a torch.distributed
    all-reduce (residual added by rank 0) or, given `exchange` (an
    ffn_b200.EpExchange), the library's NVLink peer exchange, which reads every
    rank's partial from the exchange's shared `part` buffer and adds the
    residual itself; with fused=True each layer callable runs the layer and
    the exchange in one library call.  Every rank issues the same collectives
    in the same order."""

    def __init__(self, layers: Sequence[LayerFn], rank: int, world: int, group=None,
                 exchange=None, fused: bool = False):
        self.layers = list(layers)
        self.rank, self.world, self.group = rank, world, group
        self.exchange = exchange if world > 1 else None
        # fused: a layer callable runs the whole layer, exchange included
        # (ffn_b200.MoeLayer.forward_ep), given (x_in, out, residual=x_in)
        self.fused = fused and self.exchange is not None

    def forward(self, x, buf_a, buf_b, on_layer: Optional[Callable[[int], None]] = None):
        """Runs every layer on x (not modified); buf_a / buf_b are ping-pong
        buffers shaped like x.  Returns the buffer holding the stack output."""
        cur = x
        for i, layer in enumerate(self.layers):
            nxt = buf_a if cur is not buf_a else buf_b
            if self.fused:
                layer(cur, nxt, cur)
            elif self.exchange is not None:
                layer(cur, self.exchange.part, None)
                self.exchange.allreduce(cur.shape[0], cur, nxt)
            else:
                layer(cur, nxt, cur if self.rank == 0 else None)
            if self.world > 1 and self.exchange is None:
                import torch.distributed as dist

                dist.all_reduce(nxt, group=self.group)
            if on_layer is not None:
                on_layer(i)
            cur = nxt
        return cur
