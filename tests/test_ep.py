"""Expert parallelism on the CPU: the partition, the slot-buffer exchange and the combine.

Each rank of a gloo process group computes only its contiguous experts' slot outputs (the CPU oracle stands in for
the shard-mode kernel), rank 0 adds the shared expert's rows, ``ep.reduce_slots`` sums the buffers, and the
combine of the sum must equal the single-process layer bit for bit -- the exactness the GPU path relies on (every
slot has one owner, so the sum adds only zeros to it)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from oracle import moe_ref, router_ref
from qwenfast_b200 import ep, synthetic

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_shard_range_partitions_the_experts():
    for E, world in ((16, 1), (16, 2), (16, 4), (512, 8), (512, 2)):
        covered = []
        for r in range(world):
            lo, hi = ep.shard_range(E, r, world)
            assert hi - lo == E // world
            covered.extend(range(lo, hi))
        assert covered == list(range(E))
    with pytest.raises(RuntimeError):
        ep.shard_range(10, 0, 4)
    with pytest.raises(RuntimeError):
        ep.shard_range(16, 4, 4)


def _layer(M=6, seed=3):
    cfg = synthetic.CONFIGS[0]
    L = synthetic.make_moe_layer(cfg, seed=seed)
    g = torch.Generator().manual_seed(seed + 1)
    Is = 128
    L["w_gate"] = (torch.randn(cfg.H, generator=g) * 0.02).to(torch.bfloat16)
    L["sh_gu"] = (torch.randn(2 * Is, cfg.H, generator=g) * 0.02).to(torch.bfloat16)
    L["sh_d"] = (torch.randn(cfg.H, Is, generator=g) * 0.02).to(torch.bfloat16)
    x = synthetic.make_tokens(cfg, M=M, seed=seed)
    return cfg, L, x


def _worker(rank, world, port, result_dir):
    import sys
    for p in (ROOT, os.path.join(ROOT, "qwen-3.8-flash-next-pro6000_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist
    from oracle import moe_ref as mr, router_ref as rr
    from qwenfast_b200 import ep as epm
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        cfg, L, x = _layer()
        M, H, k = x.shape[0], cfg.H, cfg.topk
        w, ids, _ = rr.router_topk(x, L["router"], k, True)        # replicated: identical on every rank
        lo, hi = epm.shard_range(cfg.E, rank, world)
        _, y = mr.moe_rounded(x, ids, w, L["w13"], L["s13"], L["w2"], L["s2"], expert_range=(lo, hi),
                              return_slots=True)
        slots = torch.zeros(epm.slot_rows(M, k), H)
        slots[: M * k] = y.float().reshape(M * k, H)
        if rank == 0:
            slots[M * k:] = mr.shared_expert_bf16(x, L["sh_gu"], L["sh_d"]).float()
        owned = (slots[: M * k].abs().sum(1) != 0).to(torch.int32)
        epm.reduce_slots(slots)
        dist.all_reduce(owned)
        out = mr.combine_slots(x, slots[: M * k].view(M, k, H), slots[M * k:].to(torch.bfloat16), L["w_gate"])
        torch.save({"out": out, "owned": owned, "ids": ids}, os.path.join(result_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_expert_parallel_combine_is_exact(world, tmp_path):
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    cfg, L, x = _layer()
    w, ids, _ = router_ref.router_topk(x, L["router"], cfg.topk, True)
    ref = moe_ref.moe_rounded(x, ids, w, L["w13"], L["s13"], L["w2"], L["s2"], w_gate=L["w_gate"],
                              shared_w=(L["sh_gu"], L["sh_d"]))
    for r in range(world):
        got = torch.load(os.path.join(tmp_path, f"rank{r}.pt"))
        assert torch.equal(got["ids"], ids)
        assert torch.equal(got["out"], ref)
        assert int(got["owned"].max()) <= 1       # no slot has two owners


def _fail_worker(rank, world, port, result_dir, how):
    """Rank 1 fails between steps -- it exits (``how == "exits"``) or stays alive without joining the exchange
    (``"stalls"``); rank 0 runs the slot exchange and must get an error within the process group's timeout."""
    import datetime
    import sys
    import time
    for p in (ROOT, os.path.join(ROOT, "qwen-3.8-flash-next-pro6000_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist
    from qwenfast_b200 import ep as epm
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=4))
    if rank == 1:
        if how == "stalls":
            time.sleep(10)
        os._exit(0)
    t0 = time.time()
    err = None
    try:
        epm.reduce_slots(torch.ones(epm.slot_rows(2, 4), 64))
    except Exception as e:   # gloo reports the lost peer or the timeout as a RuntimeError
        err = f"{type(e).__name__}: {e}"
    torch.save({"error": err, "elapsed": time.time() - t0}, os.path.join(result_dir, "rank0.pt"))
    os._exit(0)


@pytest.mark.parametrize("how", ["exits", "stalls"])
def test_a_failed_rank_is_reported_not_waited_for(how, tmp_path):
    """Failure detection on the host (gloo, CPU): the surviving rank's exchange raises instead of hanging."""
    mp.start_processes(_fail_worker, args=(2, _free_port(), str(tmp_path), how), nprocs=2, join=True,
                       start_method="spawn")
    got = torch.load(os.path.join(tmp_path, "rank0.pt"))
    assert got["error"] is not None
    assert got["elapsed"] < 30, got
