"""Seeded synthetic inputs for the W13 workloads (no checkpoints, no datasets).

Distributions follow the workload definitions: FP8 weights N(0, 0.02)
quantized with 128x128 fp32 block scales, activations N(0, 1) bf16, uniform
top-k routing (distinct experts per token) or Zipf(s) skewed routing; INT4
weights uniform nibbles (signed range [-8, 7]) with |N(0, 0.01)| bf16 group-32
scales.  Weight quantization follows DeepGEMM's per_block_cast_to_fp8 as the
reference calls it (baselines/fp8-group-gemm/baseline_dsv3_decode.py:45-48):
amax per 128x128 block clamped at 1e-4, q = e4m3(w * 448/amax), scale = amax/448.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

SEED_WEIGHTS, SEED_ACTS, SEED_ROUTING = 1, 2, 3


@dataclass(frozen=True)
class W13Config:
    name: str
    E: int
    topk: int
    T: int
    K: int
    N: int
    routing: str = "uniform"   # or "zipf"
    zipf_s: float = 1.1
    quant: str = "fp8"         # or "int4"
    silu: bool = False

    @property
    def R(self) -> int:
        return self.T * self.topk


# The workload configurations (the five benchmark configurations, numbered 1-5)
CONFIGS = {
    "cpu_fp8": W13Config("cpu_fp8", E=8, topk=2, T=256, K=512, N=1024),
    "dsv3_decode": W13Config("dsv3_decode", E=256, topk=8, T=128, K=7168, N=4096),
    "dsv3_prefill": W13Config("dsv3_prefill", E=256, topk=8, T=8192, K=7168, N=4096,
                              routing="zipf"),
    "dsv3_prefill_silu": W13Config("dsv3_prefill_silu", E=256, topk=8, T=8192, K=7168, N=4096,
                                   routing="zipf", silu=True),
    "kimi_int4_decode": W13Config("kimi_int4_decode", E=384, topk=8, T=64, K=7168, N=4096,
                                  quant="int4"),
    "kimi_int4_decode_silu": W13Config("kimi_int4_decode_silu", E=384, topk=8, T=64, K=7168,
                                       N=4096, quant="int4", silu=True),
    # the reference's own Kimi TP8 shape (2I_r = 512, T in {1, 8}), fused SiLU
    "kimi_int4_tp8_t1": W13Config("kimi_int4_tp8_t1", E=384, topk=8, T=1, K=7168, N=512,
                                  quant="int4", silu=True),
    "kimi_int4_tp8_t8": W13Config("kimi_int4_tp8_t8", E=384, topk=8, T=8, K=7168, N=512,
                                  quant="int4", silu=True),
    "ep_prefill": W13Config("ep_prefill", E=256, topk=8, T=32768, K=7168, N=4096, routing="zipf"),
    # one EP=8 rank of the decode config (32 local experts, ~4 rows each): the
    # reference's own per-rank decode shape (tasks/fp8-group-gemm-dsv3-decode.yaml:14),
    # also the small case for ncu captures (0.94 GB of weights > L2)
    "dsv3_decode_rank": W13Config("dsv3_decode_rank", E=32, topk=8, T=16, K=7168, N=4096),
    # small FP8 prefill case for ncu captures (32 experts, 0.94 GB of weights)
    "dsv3_prefill_small": W13Config("dsv3_prefill_small", E=32, topk=8, T=2048, K=7168, N=4096,
                                    routing="zipf"),
    # small INT4 case for ncu captures (128 routed rows over ~70 active experts,
    # ~1.1 GB of weights > L2; the decode kernel's regime, like configuration 4)
    "kimi_int4_small": W13Config("kimi_int4_small", E=96, topk=8, T=16, K=7168, N=4096,
                                 quant="int4"),
}


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def routing(T: int, E: int, topk: int, kind: str = "uniform", zipf_s: float = 1.1,
            seed: int = SEED_ROUTING, device="cpu") -> torch.Tensor:
    """int32 [T, topk] of distinct experts per token."""
    g = _gen(seed, "cpu")
    if kind == "uniform":
        ids = torch.rand(T, E, generator=g).argsort(dim=1)[:, :topk]
    elif kind == "zipf":
        ranks = torch.arange(1, E + 1, dtype=torch.float64)
        p = ranks.pow(-zipf_s)
        p = p / p.sum()
        perm = torch.randperm(E, generator=g)            # rank -> expert
        pe = torch.empty(E, dtype=torch.float64)
        pe[perm] = p
        ids = torch.multinomial(pe.expand(T, E), topk, replacement=False, generator=g)
    else:
        raise ValueError(kind)
    return ids.to(torch.int32).contiguous().to(device)


def activations(T: int, K: int, seed: int = SEED_ACTS, device="cpu", scale: float = 1.0):
    g = _gen(seed, "cpu")
    return (torch.randn(T, K, generator=g) * scale).to(torch.bfloat16).to(device)


def ceil_pow2(s: torch.Tensor) -> torch.Tensor:
    """Smallest power of two >= s (positive normal float32), from the bits."""
    bits = s.float().contiguous().view(torch.int32)
    ex = (bits >> 23) + ((bits & 0x7FFFFF) != 0).to(torch.int32)
    return (ex << 23).view(torch.float32)


def per_block_cast_to_fp8(w: torch.Tensor, use_ue8m0: bool = False):
    """[..., N, K] float -> (e4m3 [..., N, K], f32 [..., N/128, K/128]).

    use_ue8m0 rounds each block scale up to a power of two (UE8M0) and divides
    by it exactly -- the weights of the block-scaled GEMM path."""
    *lead, N, K = w.shape
    v = w.float().reshape(*lead, N // 128, 128, K // 128, 128)
    amax = v.abs().amax(dim=(-3, -1), keepdim=True).clamp(min=1e-4)
    if use_ue8m0:
        sc = ceil_pow2(amax / 448.0)
        q = (v * torch.reciprocal(sc)).to(torch.float8_e4m3fn).reshape(*lead, N, K)
        s = sc.reshape(*lead, N // 128, K // 128)
    else:
        q = (v * (448.0 / amax)).to(torch.float8_e4m3fn).reshape(*lead, N, K)
        s = (amax / 448.0).reshape(*lead, N // 128, K // 128)
    return q, s.contiguous()


def fp8_weights(E: int, N: int, K: int, seed: int = SEED_WEIGHTS, device="cpu",
                std: float = 0.02, chunk: int = 8, use_ue8m0: bool = False, select=None):
    """Random-init FP8 expert weights, generated on `device` in expert chunks.

    `select` (a sequence of expert ids) keeps only those experts, in that
    order, with the values they have in the full E-expert set: every chunk is
    still drawn from the one generator, so an expert-parallel rank holding a
    shard sees exactly the weights a single GPU holding all E would."""
    keep = list(range(E)) if select is None else [int(e) for e in select]
    slot = {}
    for i, e in enumerate(keep):
        slot.setdefault(e, []).append(i)
    w_q = torch.empty(len(keep), N, K, dtype=torch.float8_e4m3fn, device=device)
    w_s = torch.empty(len(keep), N // 128, K // 128, dtype=torch.float32, device=device)
    g = _gen(seed, device)
    for e0 in range(0, E, chunk):
        e1 = min(E, e0 + chunk)
        w = torch.randn(e1 - e0, N, K, generator=g, device=device) * std
        if not any(e in slot for e in range(e0, e1)):
            del w
            continue
        q, s = per_block_cast_to_fp8(w, use_ue8m0)
        for e in range(e0, e1):
            for i in slot.get(e, ()):
                w_q[i] = q[e - e0]
                w_s[i] = s[e - e0]
        del w, q, s
    return w_q, w_s


def int4_weights(E: int, N: int, K: int, seed: int = SEED_WEIGHTS, device="cpu"):
    """Raw compressed-tensors INT4: int32 [E, K/8, N] (8 offset-8 nibbles
    along K, low nibble first) and bf16 scales [E, K/32, N] ~ |N(0, 0.01)|."""
    g = _gen(seed, device)
    raw = torch.randint(-(2**31), 2**31 - 1, (E, K // 8, N), dtype=torch.int32, generator=g,
                        device=device)
    scales = (torch.randn(E, K // 32, N, generator=g, device=device).abs() * 0.01).to(torch.bfloat16)
    return raw, scales
