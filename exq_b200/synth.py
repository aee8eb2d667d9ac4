"""Seeded synthetic inputs with the shapes and distributions of the
benchmark configurations (the reference measures on seeded synthetic tensors:
scripts/bench_int4.py:114-117, scripts/bench_sglang_integration.py:192-207).

Router: logits N(0, 1) [T, E] plus a per-expert Zipf(s) log-bias
``-s * ln(rank_e)`` with ``rank`` a seeded permutation of 1..E, then
softmax -> top-k -> renormalise (weights sum to 1 per token).
Weights: N(0, 0.02^2) (the 0.02 scale of bench_sglang_integration.py:193-203).
Activations: N(0, 1).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class MoEConfig:
    name: str
    n_experts: int
    top_k: int
    hidden: int
    inter: int
    act_dtype: torch.dtype
    n_shared: int = 0
    n_layers: int = 1
    tokens: tuple = (16,)


CONFIGS = {
    "olmoe": MoEConfig("OLMoE-1B-7B", 64, 8, 2048, 1024, torch.float16, tokens=(16,)),
    "qwen3": MoEConfig("Qwen3-30B-A3B", 128, 8, 2048, 768, torch.float16,
                       tokens=(1, 8, 32, 64, 128, 256)),
    "olmoe_mixed": MoEConfig("OLMoE-1B-7B mixed BF16/INT8/INT4", 64, 8, 2048, 1024,
                             torch.float16, n_layers=16, tokens=(64,)),
    "mixtral": MoEConfig("Mixtral-8x7B", 8, 2, 4096, 14336, torch.bfloat16, tokens=(256, 4096)),
    "dsv2_lite": MoEConfig("DeepSeek-V2-Lite", 64, 6, 2048, 1408, torch.bfloat16, n_shared=2,
                           n_layers=26, tokens=(64, 256)),
}


def zipf_ranks(n_experts: int, seed: int) -> torch.Tensor:
    """Seeded permutation: rank (1 = hottest) of every expert."""
    g = torch.Generator().manual_seed(seed * 7919 + 17)
    return torch.randperm(n_experts, generator=g) + 1


def zipf_router(n_tokens: int, n_experts: int, top_k: int, seed: int = 0, s: float = 1.1,
                device="cpu", ids_dtype=torch.int32):
    """(topk_ids [T, k], topk_weights f32 [T, k]) with Zipf-skewed routing."""
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn(n_tokens, n_experts, generator=g)
    ranks = zipf_ranks(n_experts, seed).float()
    logits = logits - s * torch.log(ranks)
    probs = torch.softmax(logits, dim=-1)
    w, ids = torch.topk(probs, top_k, dim=-1)
    w = w / w.sum(dim=-1, keepdim=True)
    return ids.to(ids_dtype).to(device), w.float().to(device)


def tier_plan(n_experts: int, seed: int = 0, bf16_frac: float = 0.10,
              int8_frac: float = 0.20) -> list[str]:
    """Tiers by expected Zipf frequency: hottest ``bf16_frac`` BF16, the next
    ``int8_frac`` INT8, the rest INT4 (64 experts -> 6 / 13 / 45)."""
    ranks = zipf_ranks(n_experts, seed)
    n_bf16 = int(round(bf16_frac * n_experts))
    n_int8 = int(round((bf16_frac + int8_frac) * n_experts)) - n_bf16
    out = []
    for r in ranks.tolist():
        if r <= n_bf16:
            out.append("BF16")
        elif r <= n_bf16 + n_int8:
            out.append("INT8")
        else:
            out.append("INT4")
    return out


def expert_weights(n_experts: int, inter: int, hidden: int, seed: int = 0,
                   dtype=torch.float16, device="cpu", std: float = 0.02):
    """(w13 [E, 2I, H], w2 [E, H, I]) ~ N(0, std^2)."""
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(seed + 1000)
    w13 = torch.randn(n_experts, 2 * inter, hidden, generator=g, device=dev, dtype=torch.float32)
    w13 = (w13 * std).to(dtype)
    w2 = torch.randn(n_experts, hidden, inter, generator=g, device=dev, dtype=torch.float32)
    w2 = (w2 * std).to(dtype)
    return w13, w2


def hidden_states(n_tokens: int, hidden: int, seed: int = 0, dtype=torch.float16,
                  device="cpu") -> torch.Tensor:
    g = torch.Generator().manual_seed(seed + 2000)
    return torch.randn(n_tokens, hidden, generator=g).to(dtype).to(device)


def touched_experts(topk_ids: torch.Tensor) -> list[int]:
    return sorted(set(topk_ids.reshape(-1).tolist()))


def expected_unique(n_tokens: int, n_experts: int, top_k: int, seed: int = 0) -> float:
    ids, _ = zipf_router(n_tokens, n_experts, top_k, seed)
    return float(len(touched_experts(ids)))


def int4_expert_bytes(hidden: int, inter: int, group: int = 128) -> int:
    return 3 * inter * hidden // 2 + 2 * (2 * inter * (hidden // group) + hidden * (inter // group))


__all__ = ["CONFIGS", "MoEConfig", "zipf_router", "tier_plan", "expert_weights",
           "hidden_states", "touched_experts", "int4_expert_bytes", "math"]
