#!/usr/bin/env python3
"""Benchmark of the decode MoE layer-step on B200: router top-k + W4A16 routed experts + shared expert + combine.

Default workload: H=2048, 512 experts, top-10 renormalised, I=512 int4 group-128 experts,
bf16 shared expert (Is=512), M=10 tokens. A "step" is one layer-step: router + routed experts + shared expert +
combine in one launch (the fused layer-step of ops.moe_layer_step; us_router_kernel times the separate router op);
the timed loop replays a CUDA graph over L distinct synthetic layers (default 16, 13.6 GB of weights), so every
step streams its experts from HBM (each step touches ~157 MB, a full cycle ~2.5 GB >> 126 MB L2).

Output: one JSON line (rank 0). value = microseconds per layer-step (lower is better); roofline = the MoE kernel's
algorithmic bytes per launch / its CUDA-event launch time vs the measured HBM copy bandwidth; e2e = the same step
through the public ops with x in pinned host memory and out written to pinned host memory every step (one GPU: read
and written by the launch itself; expert parallelism: copy-engine transfers); cpu_baseline = the CPU oracle (a port
of the reference's torch dequant-and-matmul path) on this host.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--M 10] [--layers 16]
  python bench.py --sweep out.json      # config 2 (M sweep, Zipf routing) and config 3 (W8A8) extra records
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.join(ROOT, "qwen-3.8-flash-next-pro6000_b200")
for _p in (ROOT, PKG_ROOT):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "µs per MoE layer-step & achieved HBM GB/s at M=1–64, 1/2/4/8 B200"
UNIT = "us/layer-step"
PER_EXPERT_BYTES = None   # filled from the config: int4 weights + bf16 scales of gate_up and down


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=480)
    ap.add_argument("--warmup", type=int, default=48)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--M", type=int, default=0, help="tokens per layer-step (default: the config's: 10, or 64 for config 4)")
    ap.add_argument("--config", type=int, default=0,
                    help="1 or 4 (default: config 1 on one GPU, config 4 -- expert parallel, M=64, seed 7 -- on more)")
    ap.add_argument("--layers", type=int, default=16)
    ap.add_argument("--zipf", type=float, default=0.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-config4", action="store_true", help="skip the one-GPU config-4 record of the N=1 line")
    ap.add_argument("--sweep", default="")
    ap.add_argument("--sweep-configs", default="2,3,w8g",
                    help="which sweep records to take (comma list of 2, 3, nvfp4, w8g)")
    ap.add_argument("--sweep-n", default="2048,4096,8192,12288", help="config-3 weight row counts N to sweep")
    ap.add_argument("--timeline", default="", help="write the per-CTA item timeline of config-1 layer-steps here")
    ap.add_argument("--timeline-m", default="1,10", help="token counts of the timeline")
    return ap.parse_args()


def expert_bytes(H, I, group=128):
    return (2 * I * H + H * I) // 2 + 2 * (2 * I * H + H * I) // group


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def load_traffic(name):
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        return json.load(open(p)).get(name)
    return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index, self.rows, self.proc = index, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), "--query-gpu=" + self.Q,
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.rows.append(parts)

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in self.rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


# ------------------------------------------------------------------------------------------------ CPU legs
def cpu_layer(cfg, seed=0):
    """A CPU layer for the oracle whose experts are materialised lazily (only the routed ones are filled)."""
    import torch
    from qwenfast_b200 import synthetic
    g = torch.Generator().manual_seed(seed)
    H, E, I = cfg.H, cfg.E, cfg.I
    L = dict(router=(torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16),
             w_gate=(torch.randn(H, generator=g) * 0.02).to(torch.bfloat16),
             sh_gu=(torch.randn(2 * cfg.Is, H, generator=g) * 0.02).to(torch.bfloat16),
             sh_d=(torch.randn(H, cfg.Is, generator=g) * 0.02).to(torch.bfloat16),
             w13=torch.empty(E, 2 * I, H // 8, dtype=torch.int32), s13=torch.empty(E, 2 * I, H // 128, dtype=torch.bfloat16),
             w2=torch.empty(E, H, I // 8, dtype=torch.int32), s2=torch.empty(E, H, I // 128, dtype=torch.bfloat16),
             filled=set())

    def fill(ids):
        for e in set(ids.flatten().tolist()) - L["filled"]:
            ge = torch.Generator().manual_seed(seed * 100003 + e)
            L["w13"][e] = synthetic.random_int4_words((2 * I, H // 8), ge, "cpu")
            L["s13"][e] = synthetic.group_scales((2 * I, H // 128), ge, "cpu")
            L["w2"][e] = synthetic.random_int4_words((H, I // 8), ge, "cpu")
            L["s2"][e] = synthetic.group_scales((H, I // 128), ge, "cpu")
            L["filled"].add(e)
    L["fill"] = fill
    return L


def cpu_step(cfg, L, x):
    from oracle import moe_ref, router_ref
    w, ids, _ = router_ref.router_topk(x, L["router"], cfg.topk, True)
    L["fill"](ids)
    return moe_ref.moe_rounded(x, ids, w, L["w13"], L["s13"], L["w2"], L["s2"], w_gate=L["w_gate"],
                               shared_w=(L["sh_gu"], L["sh_d"]))


def host_threads() -> int:
    """CPU threads this process may really use: the affinity set, capped by the cgroup CPU quota (a container may
    see every core of its host but be allowed a few of them; more threads than that only thrash)."""
    try:
        n = len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        n = os.cpu_count() or 1
    try:
        with open("/sys/fs/cgroup/cpu.max") as f:
            quota, period = f.read().split()[:2]
        if quota != "max":
            n = min(n, max(1, int(int(quota) / int(period))))
    except (OSError, ValueError):
        pass
    return max(1, n)


def time_cpu(cfg, M, steps, warmup, budget_s):
    """Times the CPU oracle layer-step with every host thread it may use. Returns (us per step, steps timed,
    threads)."""
    import torch
    torch.set_num_threads(host_threads())
    from qwenfast_b200 import synthetic
    L = cpu_layer(cfg)
    xs = [synthetic.make_tokens(cfg, M=M, seed=s) for s in range(4)]
    for i in range(max(4, warmup)):     # at least one pass over the inputs: every routed expert is materialised
        cpu_step(cfg, L, xs[i % 4])
    n, t0 = 0, time.perf_counter()
    while n < steps and (n == 0 or time.perf_counter() - t0 < budget_s):
        cpu_step(cfg, L, xs[n % 4])
        n += 1
    dt = time.perf_counter() - t0
    return dt / n * 1e6, n, torch.get_num_threads()


def run_reference(args):
    rank, world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    from qwenfast_b200 import synthetic
    cfg_id = args.config or (4 if world > 1 else 1)
    cfg = synthetic.CONFIGS[cfg_id]
    M = args.M or cfg.M
    warm = max(4, args.warmup)   # at least one pass over the four inputs (every routed expert materialised)
    us, n, cores = time_cpu(cfg, M, args.steps, warm, budget_s=150.0)
    line = {"impl": "reference", "metric": METRIC, "value": us, "unit": UNIT, "n_gpus": args.gpus, "steps": n,
            "warmup": args.warmup, "warmup_run": warm, "ms_per_step": us / 1e3, "higher_is_better": False,
            "scaling": "strong" if world > 1 else "weak",
            "vs_baseline": None, "dtype": "bf16/int4 (fp32 accumulate)", "data": "synthetic",
            "config": {"workload": f"config{cfg_id} MoE layer-step M={M} (CPU oracle port of the reference torch path)",
                       "config_id": cfg_id, "H": cfg.H, "E": cfg.E, "I": cfg.I, "topk": cfg.topk, "Is": cfg.Is,
                       "M": M},
            "cpu_baseline": {"value": us, "unit": UNIT, "cores": cores, "kind": "port",
                             "sample": f"{n} layer-steps (router + routed experts + shared) on the host"},
            "e2e": {"value": us, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------------ GPU arm
def build_layers(cfg, nl, dev, zipf=0.0, seed_base=1000):
    import torch
    from qwenfast_b200 import synthetic
    from qwenfast_b200.ops import MoELayerWeights
    layers = []
    for l in range(nl):
        L = synthetic.make_moe_layer(cfg, device=dev, seed=seed_base + l, zipf_s=zipf)
        layers.append(MoELayerWeights.from_canonical(L["router"], L["w13"], L["s13"], L["w2"], L["s2"], L["w_gate"],
                                                     L["sh_gu"], L["sh_d"]))
        del L
    torch.cuda.synchronize()
    return layers


def workload_seeds(cfg_id):
    """(weight seed base, token seed base) of a bench workload: config 1 layers 1000 + l, config 4 (seed 7) 7000 + l
    and tokens 7100 + l -- one synthetic layer per slot of the cycled graph."""
    return (1000, 1000) if cfg_id == 1 else (7000, 7100)


def measure(cfg, cfg_id, M, NL, dev, args, rank, world, epar, zipf=0.0, timed_clocks=False, host_e2e=True):
    """One workload: NL synthetic layers cycled in CUDA graphs so that every step streams its experts from HBM.
    Times exactly args.steps layer-steps (reps of the NL-layer graph plus one graph of the remainder) after at least
    args.warmup untimed ones, then the kernel-only graphs (MoE launch, separate router op, collective) and the end-to-end
    loop through the public op with host buffers. Every rank runs the same sequence (the graphs hold collectives under
    expert parallelism). Returns a dict of measurements (rank-max device times)."""
    import torch
    import torch.distributed as dist
    from qwenfast_b200 import ep, ops, synthetic

    wseed, tseed = workload_seeds(cfg_id)
    layers = build_layers(cfg, NL, dev, zipf, wseed)
    shards = [ep.shard_weights(lw, rank, world) for lw in layers] if epar else layers
    lo, hi = ep.shard_range(cfg.E, rank, world)
    bufs = ops.moe_workspace(M, cfg.H, cfg.I, cfg.topk, cfg.Is, dev)
    rb = ops.router_bufs(dev)
    # independent N(0, 1) tokens per layer (chaining outputs into the next layer would correlate the tokens and
    # shrink the number of distinct experts below the configuration's)
    xs = [synthetic.make_tokens(cfg, M=M, device=dev, seed=tseed + l) for l in range(NL)]
    outs = [torch.empty_like(xs[0]) for _ in range(NL)]

    def layer_step(x, l, out, pdl=True):
        if epar:
            _, tw, ids = ep.ep_layer_step(x, shards[l], cfg.topk, bufs, rb, out, rank, world, has_shared=True,
                                          pdl=pdl)
        else:
            _, tw, ids, _ = ops.moe_layer_step(x, layers[l], cfg.topk, bufs, rb, out, pdl=pdl)
        return tw, ids

    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for _ in range(2):
            for l in range(NL):
                layer_step(xs[l], l, outs[l])
    torch.cuda.current_stream().wait_stream(stream)
    torch.cuda.synchronize()
    err = ops.moe_error_word(bufs["ctrl"])
    if err:
        raise RuntimeError(f"MoE kernel reported error word {err:#x}")

    steps = max(1, args.steps)
    rem = steps % NL
    g_full = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_full):
        tws = [layer_step(xs[l], l, outs[l]) for l in range(NL)]
    g_rem = None
    if rem:
        g_rem = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_rem):
            for l in range(rem):
                layer_step(xs[l], l, outs[l])
    ids_list = [t[1] for t in tws]
    # kernel-only graph of the layer-step launches (router inside, no collective or combine): the per-launch time of
    # the roofline's kernel
    r_tw = torch.empty(M, cfg.topk, dtype=torch.float32, device=dev)
    r_ids = torch.empty(M, cfg.topk, dtype=torch.int32, device=dev)
    r_lg = torch.empty(M, cfg.E, dtype=torch.bfloat16, device=dev)
    g_moe = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_moe):
        for l in range(NL):
            lw = shards[l]
            ops.a16_moe_decode(xs[l], r_ids, r_tw, lw.w13, lw.s13, None, lw.w2, lw.s2, None, lw.w_gate,
                               None, bufs["hbuf"], bufs["ybuf"], bufs["gl"], bufs["ctrl"], outs[l], 4, None,
                               bufs["pbuf"], lw.sh_w13, None, lw.sh_w2, None, bufs["shbuf"],
                               mode=1 if epar else 0, expert_range=(lo, hi), num_experts=cfg.E,
                               router_w=lw.router, logits=r_lg)
    g_coll = None
    if epar:
        slots = bufs["ybuf"][: ep.slot_rows(M, cfg.topk) * cfg.H]
        g_coll = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_coll):
            for l in range(NL):
                ep.reduce_slots(slots)
    g_router = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_router):
        for l in range(NL):
            ops.router_topk(xs[l], layers[l].router, cfg.topk, True, rb[0], rb[1])
    # the same layer-steps without programmatic dependent launch: each launch starts only after the previous one has
    # ended, so the difference to us_step is what the chain's overlap (the next launch's prologue -- router rows
    # requested, plan scratch cleared -- under the previous launch's tail) buys
    g_nopdl = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_nopdl):
        for l in range(NL):
            layer_step(xs[l], l, outs[l], pdl=False)

    def rank_max(v):
        if world > 1:
            t = torch.tensor([v], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t.item())
        return v

    def timed(fn):
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        ev0.record()
        fn()
        ev1.record()
        torch.cuda.synchronize()
        return rank_max(ev0.elapsed_time(ev1))

    reps, warm_reps = steps // NL, max(1, math.ceil(max(args.warmup, 3) / NL))

    def run_steps():
        for _ in range(reps):
            g_full.replay()
        if g_rem is not None:
            g_rem.replay()

    for _ in range(warm_reps):
        g_full.replay()
    torch.cuda.synchronize()
    clk = None
    if timed_clocks:
        # soak ~1 s under the same load first, so clocks settle and the sampler sees the timed regime; every rank
        # replays the same number of times
        t0 = time.perf_counter()
        g_full.replay()
        torch.cuda.synchronize()
        n_soak = max(1, min(2000, math.ceil(1.0 / max(rank_max(time.perf_counter() - t0), 1e-6))))
        with ClockSampler(int(os.environ.get("LOCAL_RANK", "0"))) as sampler:
            for i in range(n_soak):
                g_full.replay()
                if i % 8 == 7:
                    torch.cuda.synchronize()
            torch.cuda.synchronize()
            ms_full = timed(run_steps)
        clk = sampler.summary()
    else:
        ms_full = timed(run_steps)
    us_step = ms_full * 1e3 / steps
    res = dict(us_step=us_step, steps=steps, warmup_run=warm_reps * NL + (NL if timed_clocks else 0), clocks=clk)
    for name, g in (("us_moe", g_moe), ("us_router", g_router), ("us_coll", g_coll), ("us_step_no_pdl", g_nopdl)):
        if g is None:
            res[name] = None
            continue
        for _ in range(warm_reps):
            g.replay()
        res[name] = timed(lambda: [g.replay() for _ in range(max(1, reps))]) * 1e3 / (NL * max(1, reps))
    torch.cuda.synchronize()
    err = ops.moe_error_word(bufs["ctrl"])
    if err:
        raise RuntimeError(f"MoE kernel reported error word {err:#x}")

    # algorithmic bytes (counted from the routing each layer actually produced); with expert parallelism the MoE
    # kernel of this rank streams its own distinct experts (and the shared expert on rank 0)
    per_e = expert_bytes(cfg.H, cfg.I)
    U = [int(torch.unique(ids_list[l]).numel()) for l in range(NL)]
    U_loc = [int(torch.unique(ids_list[l][(ids_list[l] >= lo) & (ids_list[l] < hi)]).numel()) for l in range(NL)]
    shared_b = (3 * cfg.H * cfg.Is + cfg.H) * 2
    act_b = 2 * M * cfg.H * 2
    moe_b = [u * per_e + shared_b + act_b for u in U]
    loc_b = [u * per_e + (shared_b if rank == 0 else 0) + act_b for u in U_loc]
    router_b = cfg.E * cfg.H * 2 + M * cfg.H * 2
    res.update(U=U, moe_b=moe_b, step_b=statistics.mean(moe_b) + router_b,
               launch_b=statistics.mean(loc_b) + router_b)

    if host_e2e:
        # end to end through the public ops: pinned host x in, result out, every step. One GPU: the fused layer-step
        # reads x from pinned host memory itself (staged to device memory inside the launch) and writes out to pinned
        # host memory; expert parallelism: copy-engine transfers around the step.
        xh = xs[0].cpu().pin_memory()
        oh = torch.empty_like(xh).pin_memory()
        xd = torch.empty_like(xs[0])
        od = torch.empty_like(xs[0])

        def e2e_step(l):
            if epar:
                xd.copy_(xh, non_blocking=True)
                layer_step(xd, l, od)
                oh.copy_(od, non_blocking=True)
            else:
                ops.moe_layer_step(xh, layers[l], cfg.topk, bufs, rb, oh, x_stage=xd)

        for l in range(NL):
            e2e_step(l)
        torch.cuda.synchronize()
        n_e2e = min(steps, 4 * NL)
        res["e2e_us"] = timed(lambda: [e2e_step(i % NL) for i in range(n_e2e)]) * 1e3 / n_e2e
        res["e2e_steps"] = n_e2e
    del g_full, g_rem, g_moe, g_router, g_coll, g_nopdl
    return res


def run_ours(args):
    import torch
    import torch.distributed as dist
    from qwenfast_b200 import build as qbuild
    from qwenfast_b200 import synthetic

    rank, world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    qbuild.build()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=__import__("datetime").timedelta(seconds=120))
    # config 1 (M = 10) is the one-GPU headline; the expert-parallel runs measure config 4 (M = 64 replicated, seed 7,
    # E / N contiguous experts per rank), whose one-GPU baseline the N = 1 line carries as "config4"
    cfg_id = args.config or (4 if world > 1 else 1)
    cfg = synthetic.CONFIGS[cfg_id]
    M, NL = args.M or cfg.M, args.layers
    epar = world > 1
    r = measure(cfg, cfg_id, M, NL, dev, args, rank, world, epar, zipf=args.zipf, timed_clocks=True)
    peak, peak_kind = load_peaks()
    achieved = r["launch_b"] / (r["us_moe"] * 1e-6) / 1e9
    rank_frac = None
    if epar:
        # per-rank HBM fraction of the local MoE kernel
        mine = torch.tensor([achieved / peak], device=dev)
        allf = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(allf, mine)
        rank_frac = [round(float(t.item()), 4) for t in allf]
    c4 = None
    if world == 1 and cfg_id == 1 and not args.no_config4:
        cfg4 = synthetic.CONFIGS[4]
        torch.cuda.empty_cache()
        r4 = measure(cfg4, 4, cfg4.M, NL, dev, args, rank, world, False, host_e2e=False)
        c4 = {"workload": "config4 layer-step on one GPU (M=64 replicated tokens, seed 7, all 512 experts): the "
                          "single-GPU baseline of the expert-parallel scaling runs",
              "us_per_layer_step": r4["us_step"], "us_moe_kernel": r4["us_moe"],
              "unique_experts_mean": statistics.mean(r4["U"]),
              "hbm_frac_moe_kernel": r4["launch_b"] / (r4["us_moe"] * 1e-6) / 1e9 / peak}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        us_cpu, n_cpu, cores = time_cpu(cfg, M, steps=40, warmup=4, budget_s=20.0)
        cpu = {"value": us_cpu, "unit": UNIT, "cores": cores, "kind": "port",
               "sample": f"{n_cpu} config-{cfg_id} layer-steps (M={M}) of the CPU oracle, torch fp32 on {cores} threads"}

    if rank == 0:
        # the committed capture is of the config-1 one-GPU launch (profiles/moe_persistent_kernel_config1_M10.md);
        # other workloads have no capture of their own
        traffic = load_traffic("moe_persistent_kernel") if cfg_id == 1 and world == 1 else None
        if cfg_id == 1:
            wl = (f"config1 decode MoE layer-step (router top-10 + 512-expert W4A16 + bf16 shared expert + combine), "
                  f"M={M}")
        else:
            wl = (f"config4 decode MoE layer-step (M={M} tokens replicated, seed 7), expert-parallel over {world} GPUs "
                  f"({cfg.E // world} contiguous experts each, NCCL all-reduce of the slot buffer, then the combine)"
                  if epar else f"config4 decode MoE layer-step (M={M} tokens, seed 7) on one GPU")
        line = {
            "metric": METRIC, "value": r["us_step"], "unit": UNIT, "n_gpus": world, "steps": r["steps"],
            "warmup": args.warmup, "warmup_run": r["warmup_run"],
            "ms_per_step": r["us_step"] / 1e3, "higher_is_better": False, "scaling": "strong" if epar else "weak",
            "vs_baseline": None,
            "dtype": "bf16 activations, int4 experts, fp32 accumulate", "data": "synthetic",
            "config": {"workload": wl, "config_id": cfg_id,
                       "H": cfg.H, "E": cfg.E, "I": cfg.I, "topk": cfg.topk, "Is": cfg.Is, "M": M,
                       "layers_cycled": NL, "zipf_s": args.zipf,
                       "l2": f"weights cycled over {NL} layers (~{statistics.mean(r['moe_b']) * NL / 1e9:.1f} GB "
                             f"touched per cycle) > 126 MB L2; no flush",
                       "parallelism": f"ep{world}" if epar else "single GPU", "graph": "CUDA graph + PDL"},
            "hbm_gbs_step": r["step_b"] / (r["us_step"] * 1e-6) / 1e9,
            "unique_experts_mean": statistics.mean(r["U"]),
            "us_moe_kernel": r["us_moe"], "us_router_kernel": r["us_router"],
            "us_collective": r["us_coll"], "rank_hbm_frac": rank_frac,
            "pdl_chain": {"us_per_layer_step_pdl": r["us_step"], "us_per_layer_step_no_pdl": r["us_step_no_pdl"],
                          "note": "the same graph of layer-steps launched without programmatic dependent launch"},
            "nccl_ranks": dist.get_world_size() if epar else None,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_kind": peak_kind, "kernel": "moe_persistent_kernel (layer-step launch, router inside)",
                         "bytes_per_launch": r["launch_b"],
                         "traffic": traffic,
                         "traffic_source": ("profiles/traffic.json: ncu dram read + write bytes of one config-1 "
                                            "launch (M=10, one GPU)") if traffic is not None else
                                           "no ncu capture of this workload"},
            "e2e": {"value": r["e2e_us"], "unit": UNIT, "h2d_bytes_per_step": M * cfg.H * 2,
                    "d2h_bytes_per_step": M * cfg.H * 2, "steps": r["e2e_steps"]},
            # ours per step: the fused layer-step launch (+ the combine under expert parallelism; the all-reduce is
            # NCCL's)
            "gpu_launches": (2 if epar else 1) * r["steps"],
            "clocks": r["clocks"],
        }
        if c4:
            line["config4"] = c4
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_sweep(args):
    """Extra records (one GPU): config 2 -- the layer-step over M in {1..64} with Zipf-skewed routing across stacked
    layers --, config 3 -- the W8A8 GEMM (K=2048) over N and M --, "nvfp4" -- config-1 shapes on NVFP4 experts --
    and "w8g" -- the W8A16 group-128 GEMM over K in {2048, 2560, 6144}, N and M <= 16. Every record carries its algorithmic bytes and the
    fraction of the measured HBM bandwidth. Written to ``args.sweep`` as a JSON list; one summary line per record."""
    import torch
    from qwenfast_b200 import build as qbuild
    from qwenfast_b200 import formats, ops, synthetic

    qbuild.build()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peak, peak_kind = load_peaks()
    records = []

    def graph_time(fn, reps, warm=3):
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(warm):
                fn()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        for _ in range(warm):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    which = {int(c) if c.strip().isdigit() else c.strip() for c in args.sweep_configs.split(",") if c.strip()}
    # ---------------------------------------------------------------- config 2: M sweep, Zipf routing, 48 layers
    cfg = synthetic.CONFIGS[1]
    NL = max(args.layers, 48)
    zipf = args.zipf if args.zipf > 0 else 1.1
    layers = build_layers(cfg, NL, dev, zipf) if 2 in which else None
    per_e = expert_bytes(cfg.H, cfg.I)
    shared_b = (3 * cfg.H * cfg.Is + cfg.H) * 2
    for M in (1, 2, 4, 8, 16, 32, 64) if 2 in which else ():
        bufs = ops.moe_workspace(M, cfg.H, cfg.I, cfg.topk, cfg.Is, dev)
        rb = ops.router_bufs(dev)
        xs = [synthetic.make_tokens(cfg, M=M, device=dev, seed=7000 + l) for l in range(NL)]
        outs = [torch.empty_like(xs[0]) for _ in range(NL)]
        ids_l, tw_l = [None] * NL, [None] * NL

        def all_steps():
            for l in range(NL):
                _, tw, ids, _ = ops.moe_layer_step(xs[l], layers[l], cfg.topk, bufs, rb, outs[l])
                ids_l[l], tw_l[l] = ids, tw

        ms = graph_time(all_steps, reps=4)

        def moe_only():
            for l in range(NL):
                lw = layers[l]
                ops.a16_moe_decode(xs[l], ids_l[l], tw_l[l], lw.w13, lw.s13, None, lw.w2, lw.s2, None, lw.w_gate, None,
                                   bufs["hbuf"], bufs["ybuf"], bufs["gl"], bufs["ctrl"], outs[l], 4, None,
                                   bufs["pbuf"], lw.sh_w13, None, lw.sh_w2, None, bufs["shbuf"])

        ms_moe = graph_time(moe_only, reps=4)
        err = ops.moe_error_word(bufs["ctrl"])
        if err:
            raise RuntimeError(f"MoE kernel reported error word {err:#x} at M={M}")
        U = [int(torch.unique(ids_l[l]).numel()) for l in range(NL)]
        moe_b = statistics.mean(u * per_e + shared_b + 2 * M * cfg.H * 2 for u in U)
        us_step, us_moe = ms * 1e3 / NL, ms_moe * 1e3 / NL
        rec = {"config": 2, "M": M, "layers": NL, "zipf_s": zipf, "unique_experts_mean": statistics.mean(U),
               "us_per_layer_step": us_step, "us_moe_kernel": us_moe, "moe_bytes": moe_b,
               "achieved_gbs": moe_b / (us_moe * 1e-6) / 1e9, "peak_gbs": peak, "peak_kind": peak_kind}
        rec["frac"] = rec["achieved_gbs"] / peak
        # the layer-step is one launch (router inside): its bytes add the router weights and the router's x read
        rec["step_bytes"] = moe_b + cfg.E * cfg.H * 2 + M * cfg.H * 2
        rec["step_frac"] = rec["step_bytes"] / (us_step * 1e-6) / 1e9 / peak
        records.append(rec)
        print(json.dumps(rec), flush=True)
        del bufs, xs, outs
    del layers
    torch.cuda.empty_cache()

    # ---------------------------------------------------------------- config-1 shapes on NVFP4 experts
    if "nvfp4" in which:
        NL4 = 16
        lay4 = []
        for l in range(NL4):
            wp, sf, g13 = synthetic.make_nvfp4_experts(cfg.E, 2 * cfg.I, cfg.H, device=dev, seed=500 + l)
            wk13, sk13 = formats.repack_nvfp4(wp, sf, gated=True)
            wp, sf, g2 = synthetic.make_nvfp4_experts(cfg.E, cfg.H, cfg.I, device=dev, seed=900 + l)
            wk2, sk2 = formats.repack_nvfp4(wp, sf, gated=False)
            del wp, sf
            L = synthetic.make_moe_layer(synthetic.MoEConfig("nvfp4-shared", cfg.H, 16, 128, 4, 1, cfg.Is, 1300 + l),
                                         device=dev)   # the router and the bf16 shared expert only
            router = (torch.randn(cfg.E, cfg.H, device=dev, generator=torch.Generator(device=dev).manual_seed(l))
                      * 0.02).to(torch.bfloat16)
            lay4.append(dict(w13=wk13, s13=sk13, w2=wk2, s2=sk2, gs13=(1.0 / g13).to(torch.bfloat16),
                             gs2=(1.0 / g2).to(torch.bfloat16), router=router, w_gate=L["w_gate"],
                             sh13=formats.repack_bf16(L["sh_gu"], gated=True),
                             sh2=formats.repack_bf16(L["sh_d"], gated=False)))
            del L
        per_e4 = (2 * cfg.I * cfg.H + cfg.H * cfg.I) // 2 + (2 * cfg.I * cfg.H + cfg.H * cfg.I) // 16
        for M in (1, 10):
            bufs = ops.moe_workspace(M, cfg.H, cfg.I, cfg.topk, cfg.Is, dev)
            rb = ops.router_bufs(dev)
            xs = [synthetic.make_tokens(cfg, M=M, device=dev, seed=8000 + l) for l in range(NL4)]
            routes = [ops.router_topk(xs[l], lay4[l]["router"], cfg.topk, True, *rb) for l in range(NL4)]
            outs = [torch.empty_like(xs[0]) for _ in range(NL4)]

            def nvfp4_layers():
                for l, q in enumerate(lay4):
                    tw, ids, _ = routes[l]
                    ops.a16_moe_decode(xs[l], ids, tw, q["w13"], q["s13"], q["gs13"], q["w2"], q["s2"], q["gs2"],
                                       q["w_gate"], None, bufs["hbuf"], bufs["ybuf"], bufs["gl"], bufs["ctrl"],
                                       outs[l], 4, None, bufs["pbuf"], q["sh13"], None, q["sh2"], None,
                                       bufs["shbuf"], fmt="nvfp4")

            ms4 = graph_time(nvfp4_layers, reps=8)
            r_tw = torch.empty(M, cfg.topk, dtype=torch.float32, device=dev)
            r_ids = torch.empty(M, cfg.topk, dtype=torch.int32, device=dev)
            r_lg = torch.empty(M, cfg.E, dtype=torch.bfloat16, device=dev)

            def nvfp4_layer_steps():   # the router inside the launch (qf_moe_layer_decode_nvfp4)
                for l, q in enumerate(lay4):
                    ops.a16_moe_decode(xs[l], r_ids, r_tw, q["w13"], q["s13"], q["gs13"], q["w2"], q["s2"], q["gs2"],
                                       q["w_gate"], None, bufs["hbuf"], bufs["ybuf"], bufs["gl"], bufs["ctrl"],
                                       outs[l], 4, None, bufs["pbuf"], q["sh13"], None, q["sh2"], None,
                                       bufs["shbuf"], fmt="nvfp4", router_w=q["router"], logits=r_lg)

            ms4s = graph_time(nvfp4_layer_steps, reps=8)
            err = ops.moe_error_word(bufs["ctrl"])
            if err:
                raise RuntimeError(f"NVFP4 MoE kernel reported error word {err:#x} at M={M}")
            U = [int(torch.unique(routes[l][1]).numel()) for l in range(NL4)]
            b4 = statistics.mean(u * per_e4 + shared_b + 2 * M * cfg.H * 2 for u in U)
            us4 = ms4 * 1e3 / NL4
            rec = {"config": "1-nvfp4", "M": M, "layers": NL4, "unique_experts_mean": statistics.mean(U),
                   "us_moe_kernel": us4, "moe_bytes": b4, "achieved_gbs": b4 / (us4 * 1e-6) / 1e9,
                   "peak_gbs": peak, "peak_kind": peak_kind, "us_layer_step": ms4s * 1e3 / NL4,
                   "note": "NVFP4 experts (e2m1 + E4M3 group-16 scales), bf16 shared expert; us_moe_kernel with the "
                           "routing given, us_layer_step with the router inside the launch"}
            rec["frac"] = rec["achieved_gbs"] / peak
            records.append(rec)
            print(json.dumps(rec), flush=True)
            del bufs, xs, outs, routes
        del lay4
        torch.cuda.empty_cache()

    # ---------------------------------------------------------------- config 3: W8A8 GEMM, K = 2048
    K = synthetic.W8A8_K
    for N in [int(n) for n in args.sweep_n.split(",") if n.strip()] if 3 in which else ():
        copies = max(2, math.ceil(400e6 / (N * K)))   # > 3x the 126 MB L2 per cycle
        ws = []
        for c in range(copies):
            q, sw = synthetic.make_w8a8(N, K, device=dev, seed=10 + c)
            ws.append((formats.repack_w8(q), sw))   # load-time repack to the kernel layout
            del q
        for M in (1, 2, 4, 8, 10, 16):
            x = synthetic.make_w8a8_tokens(M, K, device=dev)
            xq = torch.empty(16 * K, dtype=torch.int8, device=dev)
            sx = torch.empty(M, dtype=torch.float32, device=dev)

            def gemms():
                for q, sw in ws:
                    ops.w8a8_gemm(x, q, sw, xq=xq, sx=sx)

            ms = graph_time(gemms, reps=8)
            if ops.w8a8_take_status():
                raise RuntimeError(f"W8A8 kernel reported a wait timeout at N={N} M={M}")
            us = ms * 1e3 / copies
            b = N * K + 4 * N + 2 * M * K + 2 * M * N
            rec = {"config": 3, "N": N, "K": K, "M": M, "us_per_gemm": us, "bytes": b,
                   "achieved_gbs": b / (us * 1e-6) / 1e9, "peak_gbs": peak, "peak_kind": peak_kind,
                   "l2": f"{copies} weight copies cycled (> L2)"}
            rec["frac"] = rec["achieved_gbs"] / peak
            records.append(rec)
            print(json.dumps(rec), flush=True)
        del ws
        torch.cuda.empty_cache()
    # ---------------------------------------------------------------- W8A16 group-128 GEMM (the dense projections)
    # the op the reference calls for every int8 dense projection (serve/overlays/sglang/srt/qwenfast.py:351-353):
    # canonical int8 weights + bf16 group-128 scales, M <= 16 rows
    for K in (2048, 2560, 6144) if "w8g" in which else ():
        for N in [int(n) for n in args.sweep_n.split(",") if n.strip()]:
            copies = max(2, math.ceil(400e6 / (N * K)))   # > 3x the 126 MB L2 per cycle
            g = torch.Generator(device=dev).manual_seed(N + K)
            ws = [(torch.randint(-127, 128, (N, K), generator=g, device=dev, dtype=torch.int32).to(torch.int8),
                   (torch.rand(N, K // 128, generator=g, device=dev) * 1e-3 + 1e-4).to(torch.bfloat16))
                  for _ in range(copies)]
            for M in (1, 4, 8, 16):
                x = torch.randn(M, K, generator=g, device=dev).to(torch.bfloat16)

                def gemms():
                    for q, s8 in ws:
                        ops.w8g_gemm(x, q, s8, 0, pdl=True)

                ms = graph_time(gemms, reps=8)
                if ops.w8g_take_status():
                    raise RuntimeError(f"W8A16 kernel reported a wait timeout at N={N} K={K} M={M}")
                us = ms * 1e3 / copies
                b = N * K + 2 * N * K // 128 + 2 * M * K + 2 * M * N
                rec = {"config": "w8g", "N": N, "K": K, "M": M, "us_per_gemm": us, "bytes": b,
                       "achieved_gbs": b / (us * 1e-6) / 1e9, "peak_gbs": peak, "peak_kind": peak_kind,
                       "l2": f"{copies} weight copies cycled (> L2)"}
                rec["frac"] = rec["achieved_gbs"] / peak
                records.append(rec)
                print(json.dumps(rec), flush=True)
            del ws
            torch.cuda.empty_cache()
    with open(args.sweep, "w") as f:
        json.dump(records, f, indent=1)


KIND_NAMES = {1: "GL", 2: "S1", 3: "G1", 4: "S1F", 5: "S2", 6: "G2", 7: "CB"}


def decode_timeline(dbg, sms):
    """The MoE kernel's timeline buffer (include/qwenfast_b200.h, ``dbg``) -> per-phase summary in us, relative to
    the earliest CTA entry: router + routing plan (median consumer start), per item kind the count, the span of
    starts, the median / max time from an item's start to its last stage retired, and when the last pipeline
    stopped."""
    d = dbg.view(-1, 32)[:sms].tolist()
    U = lambda v: (v & ((1 << 64) - 1)) >> 12
    t0 = min(U(row[31]) for row in d if row[31] != 0)
    ev = []
    for c, row in enumerate(d):
        for v in row[:31]:
            if v:
                tag = v & 0xFFF
                ev.append(((U(v) - t0) / 1e3, c, (tag >> 5) & 3, tag & 31))
    ev.sort()
    open_items, dur, starts = {}, {}, {}
    for t, c, vp, code in ev:
        if 1 <= code <= 7:
            open_items[(c, vp)] = (code, t)
            starts.setdefault(code, []).append(t)
        elif 17 <= code <= 23 and open_items.get((c, vp), (0,))[0] == code - 16:
            dur.setdefault(code - 16, []).append((t - open_items.pop((c, vp))[1], t))
    med = lambda v: sorted(v)[len(v) // 2]
    stops = [t for t, _, _, code in ev if code == 31]   # absent when a CTA's stamp slots ran out first
    out = dict(consumers_start_us=round(med([t for t, _, _, code in ev if code == 30]), 2),
               last_stop_us=round(max(stops), 2) if stops else None, kinds={})
    for k, st in sorted(starts.items()):
        dd = dur.get(k, [])
        out["kinds"][KIND_NAMES[k]] = dict(
            n=len(st), first_start_us=round(min(st), 2), last_start_us=round(max(st), 2),
            stages_us_median=round(med([a for a, _ in dd]), 2) if dd else None,
            stages_us_max=round(max(a for a, _ in dd), 2) if dd else None,
            last_stages_done_us=round(max(b for _, b in dd), 2) if dd else None)
    return out


def run_timeline(args):
    """Per-item timeline of the config-1 layer-step (router inside) at each M of ``--timeline-m``: the kernel's
    globaltimer stamps (every pipeline: item start, stages retired, start / stop), taken on one launch per run
    inside a CUDA graph of 8 layer-steps over 8 different layers (weights from HBM), without programmatic launch so
    that each launch starts after the previous one ended. Four runs per M; written to ``args.timeline`` (JSON) with a
    summary line per run."""
    import torch
    from qwenfast_b200 import ops, synthetic

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = synthetic.CONFIGS[1]
    NL = 8
    layers = build_layers(cfg, NL, dev)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    res = {}
    for M in [int(m) for m in args.timeline_m.split(",") if m.strip()]:
        xs = [synthetic.make_tokens(cfg, M=M, device=dev, seed=200 + i) for i in range(NL)]
        bufs = ops.moe_workspace(M, cfg.H, cfg.I, cfg.topk, cfg.Is, dev)
        out = torch.empty(M, cfg.H, dtype=torch.bfloat16, device=dev)
        tw = torch.empty(M, cfg.topk, dtype=torch.float32, device=dev)
        ids = torch.empty(M, cfg.topk, dtype=torch.int32, device=dev)
        lg = torch.empty(M, cfg.E, dtype=torch.bfloat16, device=dev)
        dbg = torch.zeros(ops.DBG_NUMEL, dtype=torch.int64, device=dev)

        def seq():
            for i, lw in enumerate(layers):
                ops.a16_moe_decode(xs[i], ids, tw, lw.w13, lw.s13, None, lw.w2, lw.s2, None, lw.w_gate, None,
                                   bufs["hbuf"], bufs["ybuf"], bufs["gl"], bufs["ctrl"], out, 4,
                                   dbg if i == NL // 2 else None, bufs["pbuf"], lw.sh_w13, None, lw.sh_w2, None,
                                   bufs["shbuf"], pdl=False, router_w=lw.router, logits=lg)

        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(3):
                seq()
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            seq()
        runs = []
        for _ in range(4):
            g.replay()
            dbg.zero_()
            g.replay()
            torch.cuda.synchronize()
            runs.append(decode_timeline(dbg.cpu(), sms))
        if ops.moe_error_word(bufs["ctrl"]) != 0:
            raise RuntimeError("timeline: the MoE kernel reported an error")
        res[M] = runs
        for r in runs:
            print(json.dumps(dict(M=M, **r)), flush=True)
        del g
    with open(args.timeline, "w") as f:
        json.dump(res, f, indent=1)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.timeline:
        run_timeline(args)
    elif args.sweep:
        run_sweep(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
