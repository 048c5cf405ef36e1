"""Seeded synthetic inputs of the benchmark configurations (there are no checkpoints or datasets here).

config 0  toy layer: H=256, E=16, I=128, top-4 renormalised, no shared expert, M=4, seed 0
config 1  Qwen3-Next-style decode layer: H=2048, E=512, I=512, top-10 renormalised, bf16 shared expert
          (Is=512, ~N(0, 0.02), sigmoid gate), M=10
config 2  config 1 shapes, M in {1..64}, 48 stacked layers, router skewed so expert load ~ Zipf(1.1)
config 3  W8A8 dense GEMM: K=2048, N in {2048, 4096, 8192, 12288}, M in {1, 2, 4, 8, 10, 16}
config 4  expert parallel: config-1 weights, seed 7, M=64 replicated on every rank
Distributions: activations bf16 ~N(0,1); router bf16 ~N(0, 0.02); int4 codes uniform in 0..15 (zero point 8);
group scales bf16(|N(0, 0.01)| + 1e-4); INT8 weights uniform in [-127, 127].
"""
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class MoEConfig:
    name: str
    H: int
    E: int
    I: int
    topk: int
    M: int
    Is: int
    seed: int
    renormalize: bool = True


CONFIGS = {
    0: MoEConfig("toy", 256, 16, 128, 4, 4, 0, 0),
    1: MoEConfig("qwen3-next-decode", 2048, 512, 512, 10, 10, 512, 0),
    4: MoEConfig("qwen3-next-ep", 2048, 512, 512, 10, 64, 512, 7),
}
SWEEP_M = (1, 2, 4, 8, 16, 32, 64)
W8A8_N = (2048, 4096, 8192, 12288)
W8A8_M = (1, 2, 4, 8, 10, 16)
W8A8_K = 2048


def _gen(device, seed):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def random_int4_words(shape, g, device) -> torch.Tensor:
    """int32 words whose eight nibbles are independent uniform codes in 0..15."""
    w = torch.randint(0, 2 ** 32, shape, generator=g, device=device, dtype=torch.int64)
    return torch.where(w >= 2 ** 31, w - 2 ** 32, w).to(torch.int32)


def group_scales(shape, g, device) -> torch.Tensor:
    return (torch.randn(shape, generator=g, device=device).abs() * 0.01 + 1e-4).to(torch.bfloat16)


def make_nvfp4_experts(E: int, N: int, K: int, device="cpu", seed: int = 0):
    """Synthetic NVFP4 experts (the reference's checkpoint format): uniform e2m1 codes uint8 [E, N, K/2], E4M3 group-16
    scales |N(0, 1)| * 2 + 1/64 [E, N, K/16], per-expert global values g in [100, 300) (the weight is
    e2m1 * scale / g)."""
    g = _gen(device, seed)
    wp = torch.randint(0, 256, (E, N, K // 2), generator=g, device=device, dtype=torch.int32).to(torch.uint8)
    sf = (torch.randn(E, N, K // 16, generator=g, device=device).abs() * 2 + 1.0 / 64).to(torch.float8_e4m3fn)
    gv = torch.rand(E, generator=g, device=device) * 200 + 100
    return wp, sf, gv


def make_moe_layer(cfg: MoEConfig, device="cpu", seed=None, zipf_s: float = 0.0) -> dict:
    """Canonical weights of one MoE layer. ``zipf_s > 0`` skews the router (config 2)."""
    g = _gen(device, cfg.seed if seed is None else seed)
    H, E, I = cfg.H, cfg.E, cfg.I
    router = torch.randn(E, H, generator=g, device=device) * 0.02
    if zipf_s > 0:
        router = zipf_router(router, zipf_s, g)
    d = dict(
        router=router.to(torch.bfloat16),
        w13=random_int4_words((E, 2 * I, H // 8), g, device),
        s13=group_scales((E, 2 * I, H // 128), g, device),
        w2=random_int4_words((E, H, I // 8), g, device),
        s2=group_scales((E, H, I // 128), g, device),
    )
    if cfg.Is:
        d["w_gate"] = (torch.randn(H, generator=g, device=device) * 0.02).to(torch.bfloat16)
        d["sh_gu"] = (torch.randn(2 * cfg.Is, H, generator=g, device=device) * 0.02).to(torch.bfloat16)
        d["sh_d"] = (torch.randn(H, cfg.Is, generator=g, device=device) * 0.02).to(torch.bfloat16)
    return d


def zipf_router(router: torch.Tensor, s: float, g) -> torch.Tensor:
    """Skew expert load toward a Zipf(s) profile by scaling router row e by (E / rank_e)^(0.41 s), rank_e a seeded
    permutation of 1..E: a larger row norm widens that expert's logit spread, so it lands in the top-k more often.
    With zero-mean tokens a linear router can put an expert in at most about half of the tokens' top-k, so the head
    of Zipf(1.1) cannot be reached; the exponent matches its top-50 share instead (about 0.73 of all selections at
    E = 512, top-10; the hottest experts then see roughly 40% of the tokens)."""
    E = router.shape[0]
    perm = torch.randperm(E, generator=g, device=router.device)
    rank = torch.empty(E, device=router.device)
    rank[perm] = torch.arange(1, E + 1, device=router.device, dtype=torch.float32)
    gain = (E / rank) ** (0.41 * s)
    return router * gain[:, None]


def make_tokens(cfg: MoEConfig, M=None, device="cpu", seed=None) -> torch.Tensor:
    g = _gen(device, (cfg.seed if seed is None else seed) + 1000)
    return torch.randn(cfg.M if M is None else M, cfg.H, generator=g, device=device).to(torch.bfloat16)


def make_w8a8(N: int, K: int = W8A8_K, device="cpu", seed: int = 3):
    g = _gen(device, seed)
    q = torch.randint(-127, 128, (N, K), generator=g, device=device, dtype=torch.int8)
    sw = torch.randn(N, generator=g, device=device).abs() * 0.01 + 1e-4
    return q, sw.float()


def make_w8a8_tokens(M: int, K: int = W8A8_K, device="cpu", seed: int = 4):
    g = _gen(device, seed)
    return torch.randn(M, K, generator=g, device=device).to(torch.bfloat16)
