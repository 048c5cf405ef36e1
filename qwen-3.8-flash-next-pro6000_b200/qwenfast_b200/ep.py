"""Expert parallelism for the decode MoE layer, one process per GPU.

Partition (the plan for the reference's single-GPU layer, ``serve/qwenfast/qf_a16moe.cu:852-922``, spread over
G GPUs): rank r holds the contiguous experts ``[r*E/G, (r+1)*E/G)``; the tokens and the router are replicated.
Every rank runs the router itself (identical ids everywhere: the kernels are deterministic), inside its MoE launch
(fused router) or as its own launch, then the MoE kernel in shard mode on its local experts. Each (token, top-k position) slot has exactly one owner, so the shards' slot
buffers sum exactly (every other rank contributes zeros); one all-reduce over NCCL / NVLink gives every rank the
full slot buffer and the combine kernel finishes the layer -- the same bits as one GPU. The shared expert runs on
one rank (``shared_rank``), whose slot buffer carries its output.

The collective is ``torch.distributed.all_reduce`` on the compute stream (capturable in a CUDA graph); the only
exchange of the path.
"""
from dataclasses import replace
from typing import Optional

import torch
import torch.distributed as dist

from . import ops


def shard_range(E: int, rank: int, world: int):
    """Contiguous expert range of ``rank`` among ``world`` ranks (E % world == 0, as in config 4)."""
    if world < 1 or not 0 <= rank < world:
        raise RuntimeError(f"shard_range: bad rank {rank} of {world}")
    if E % world != 0:
        raise RuntimeError(f"shard_range: {E} experts do not split over {world} ranks")
    per = E // world
    return rank * per, (rank + 1) * per


def shard_weights(lw: ops.MoELayerWeights, rank: int, world: int, shared_rank: int = 0) -> ops.MoELayerWeights:
    """This rank's part of a layer: its experts' kernel-layout weights (views), the full router and shared gate,
    and the shared expert's weights on ``shared_rank`` only. ``E`` stays the router's expert count."""
    lo, hi = shard_range(lw.E, rank, world)
    own_shared = rank == shared_rank
    return replace(lw, w13=lw.w13[lo:hi], s13=lw.s13[lo:hi], w2=lw.w2[lo:hi], s2=lw.s2[lo:hi],
                   sh_w13=lw.sh_w13 if own_shared else None, sh_w2=lw.sh_w2 if own_shared else None)


def slot_rows(M: int, topk: int) -> int:
    """Rows of the slot buffer: M*topk routed slots, then M shared rows."""
    return M * topk + M


def reduce_slots(slots: torch.Tensor, group=None) -> torch.Tensor:
    """Sum the shards' slot buffers in place on every rank (exact: each slot has one nonzero owner)."""
    dist.all_reduce(slots, op=dist.ReduceOp.SUM, group=group)
    return slots


def ep_layer_step(x: torch.Tensor, shard: ops.MoELayerWeights, topk: int, bufs: dict, rbufs, out: torch.Tensor,
                  rank: int, world: int, has_shared: Optional[bool] = None, group=None, renormalize: bool = True,
                  pdl: bool = True, fused: bool = True):
    """One expert-parallel decode layer-step on this rank: router (replicated; inside the MoE launch when
    ``fused``), local experts (shard mode), all-reduce of the slot buffer, combine. ``shard`` comes from
    ``shard_weights``; ``has_shared`` says whether the layer has a shared expert (on any rank; default: this rank
    holds w_gate). Returns (out, topk_w, topk_ids)."""
    M, H = x.shape
    lo, hi = shard_range(shard.E, rank, world)
    if has_shared is None:
        has_shared = shard.w_gate is not None
    route = {}
    if fused:
        tw = torch.empty(M, topk, dtype=torch.float32, device=x.device)
        ids = torch.empty(M, topk, dtype=torch.int32, device=x.device)
        route = dict(router_w=shard.router, renormalize=renormalize,
                     logits=torch.empty(M, shard.E, dtype=torch.bfloat16, device=x.device))
    else:
        tw, ids, _ = ops.router_topk(x, shard.router, topk, renormalize, rbufs[0], rbufs[1], pdl)
    ops.a16_moe_decode(x, ids, tw, shard.w13, shard.s13, None, shard.w2, shard.s2, None, shard.w_gate, None,
                       bufs["hbuf"], bufs["ybuf"], bufs["gl"], bufs["ctrl"], out, 4, None, bufs["pbuf"],
                       shard.sh_w13, None, shard.sh_w2, None, bufs["shbuf"], pdl=pdl, mode=1, expert_range=(lo, hi),
                       num_experts=shard.E, **route)
    slots = bufs["ybuf"][: slot_rows(M, topk) * H]
    if world > 1:
        reduce_slots(slots, group)
    ops.moe_combine(slots, x, shard.w_gate, has_shared, out, topk, pdl)
    return out, tw, ids
