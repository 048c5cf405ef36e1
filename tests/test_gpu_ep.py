"""Expert-parallel MoE on the GPU: the shard-mode kernel plus the combine kernel reproduce the
single-GPU layer bit for bit.

On one GPU the G shards run one after the other (each with its own scratch); their slot buffers are summed as the
all-reduce would (exact: one owner per slot) and combined. With two or more GPUs the same step runs as one process
per GPU over NCCL (ep.ep_layer_step)."""
import os
import socket

import pytest
import torch

from qwenfast_b200._lib import QF_MOE_CTRL_MIRROR
import torch.multiprocessing as mp

from qwenfast_b200 import ep, ops, synthetic
from qwenfast_b200.ops import MoELayerWeights

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def layer_on(dev, L):
    return MoELayerWeights.from_canonical(L["router"].to(dev), L["w13"].to(dev), L["s13"].to(dev), L["w2"].to(dev),
                                          L["s2"].to(dev), L["w_gate"].to(dev), L["sh_gu"].to(dev), L["sh_d"].to(dev))


@pytest.fixture(scope="module")
def cfg4(cuda):
    cfg = synthetic.CONFIGS[4]
    L = synthetic.make_moe_layer(cfg, device=cuda)
    return cfg, layer_on(cuda, L)


def full_layer(x, lw, topk):
    M, H = x.shape
    bufs = ops.moe_workspace(M, H, lw.I, topk, lw.Is, x.device)
    out = torch.empty_like(x)
    _, tw, ids, _ = ops.moe_layer_step(x, lw, topk, bufs, ops.router_bufs(x.device), out)
    return out, tw, ids


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("M", [1, 10, 64])
def test_shards_sum_to_the_full_layer(cfg4, cuda, world, M):
    cfg, lw = cfg4
    x = synthetic.make_tokens(cfg, M=M, device=cuda, seed=M)
    ref, tw, ids = full_layer(x, lw, cfg.topk)
    rows = ep.slot_rows(M, cfg.topk)
    total = torch.zeros(rows * cfg.H, dtype=torch.float32, device=cuda)
    owners = torch.zeros(rows, dtype=torch.int32, device=cuda)
    for r in range(world):
        sh = ep.shard_weights(lw, r, world)
        lo, hi = ep.shard_range(cfg.E, r, world)
        bufs = ops.moe_workspace(M, cfg.H, cfg.I, cfg.topk, cfg.Is, cuda)
        bufs["ybuf"].fill_(1.0)                       # every slot the shard does not own must come back zero
        ops.a16_moe_decode(x, ids, tw, sh.w13, sh.s13, None, sh.w2, sh.s2, None, sh.w_gate, None, bufs["hbuf"],
                           bufs["ybuf"], bufs["gl"], bufs["ctrl"], torch.empty_like(x), 4, None, bufs["pbuf"],
                           sh.sh_w13, None, sh.sh_w2, None, bufs["shbuf"], mode=1, expert_range=(lo, hi),
                           num_experts=cfg.E)
        torch.cuda.synchronize()
        assert ops.moe_error_word(bufs["ctrl"]) == 0
        assert int(bufs["ctrl"][:QF_MOE_CTRL_MIRROR].abs().sum().item()) == 0
        part = bufs["ybuf"][: rows * cfg.H]
        routed = part[: M * cfg.topk * cfg.H].view(M * cfg.topk, cfg.H)
        local = ((ids.view(-1) >= lo) & (ids.view(-1) < hi))
        assert not routed[~local].any()               # other shards' slots are exactly zero
        if r != 0:
            assert not part[M * cfg.topk * cfg.H:].any()
        owners += (part.view(rows, cfg.H) != 0).any(1).to(torch.int32)
        total += part.float()
    assert int(owners.max()) <= 1
    out = torch.empty_like(x)
    ops.moe_combine(total.to(torch.bfloat16), x, lw.w_gate, True, out, cfg.topk)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


def test_ep_layer_step_single_rank(cfg4, cuda):
    cfg, lw = cfg4
    x = synthetic.make_tokens(cfg, device=cuda, seed=2)
    ref, _, _ = full_layer(x, lw, cfg.topk)
    bufs = ops.moe_workspace(cfg.M, cfg.H, cfg.I, cfg.topk, cfg.Is, cuda)
    out = torch.empty_like(x)
    ep.ep_layer_step(x, ep.shard_weights(lw, 0, 1), cfg.topk, bufs, ops.router_bufs(cuda), out, 0, 1)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


def _nccl_worker(rank, world, port, result_dir):
    import sys
    for p in (ROOT, os.path.join(ROOT, "qwen-3.8-flash-next-pro6000_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import datetime
    import torch.distributed as dist
    from qwenfast_b200 import ep as epm, ops as o, synthetic as syn
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=dev, timeout=datetime.timedelta(seconds=60))
    try:
        cfg = syn.CONFIGS[4]
        L = syn.make_moe_layer(cfg, device=dev)
        lw = layer_on(dev, L)
        x = syn.make_tokens(cfg, device=dev)
        bufs = o.moe_workspace(cfg.M, cfg.H, cfg.I, cfg.topk, cfg.Is, dev)
        out = torch.empty_like(x)
        epm.ep_layer_step(x, epm.shard_weights(lw, rank, world), cfg.topk, bufs, o.router_bufs(dev), out, rank, world)
        torch.cuda.synchronize()
        res = {"out": out.cpu()}
        if rank == 0:
            res["ref"] = full_layer(x, lw, cfg.topk)[0].cpu()
        torch.save(res, os.path.join(result_dir, f"rank{rank}.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_ep_over_nccl(cuda, tmp_path):
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs two or more GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.start_processes(_nccl_worker, args=(world, port, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    ref = torch.load(os.path.join(tmp_path, "rank0.pt"))["ref"]
    for r in range(world):
        assert torch.equal(torch.load(os.path.join(tmp_path, f"rank{r}.pt"))["out"], ref)
