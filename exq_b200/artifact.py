"""Compiled-artifact reader: the per-expert quant plan the grouped launch honours.

Drop-in for exq/kernels/exq_artifact.py (``load_exq_artifact``,
``ExpertProfile``, ``freq_to_block_m``) and the key helpers of
exq/model_utils.py:121-144.  The artifact JSON maps ``"layer:expert"`` to
``"BF16" | "INT8" | "INT4"`` under ``quant_assignments`` (written by
scripts/compile_model.py:91-97; ``quant_plan`` is the legacy key); missing
entries default to INT4 (exq_artifact.py:134-138).  Host-side only.
"""
from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

PRECISION_TO_INT = {"BF16": 0, "INT8": 1, "INT4": 2}
INT_TO_PRECISION = {v: k for k, v in PRECISION_TO_INT.items()}
_TIER_TO_BLOCK_M = {0: 128, 1: 64, 2: 32}
_TIER_TO_FREQ = {0: 0.15, 1: 0.05, 2: 0.01}


def freq_to_block_m(freq: float, tier: int) -> int:
    """BLOCK_M hint per (frequency, tier) (exq_artifact.py:39-45)."""
    if tier == 1:
        return 64 if freq >= 0.03 else 32
    return _TIER_TO_BLOCK_M[tier]


def parse_quant_key(key: str) -> tuple[int, int]:
    layer, index = key.split(":")
    return int(layer), int(index)


def format_quant_key(layer: int, index: int) -> str:
    return f"{layer}:{index}"


def quant_assignments(artifact: dict) -> dict[tuple[int, int], str]:
    """``{(layer, expert): precision}`` from an artifact dict."""
    raw = artifact.get("quant_assignments") or artifact.get("quant_plan", {})
    return {parse_quant_key(k): v for k, v in raw.items()}


def layer_tiers(artifact: dict, layer: int, n_experts: int) -> list[str]:
    """Tier name of every expert of one layer (INT4 when unassigned or unknown)."""
    qa = quant_assignments(artifact)
    out = []
    for e in range(n_experts):
        p = qa.get((layer, e), "INT4")
        out.append(p if p in PRECISION_TO_INT else "INT4")
    return out


@dataclass
class ExpertProfile:
    """Per-layer expert metadata in kernel-ready form (exq_artifact.py:48-93)."""

    n_layers: int
    n_experts_per_layer: int
    tiers: torch.Tensor     # int8 [L, E]: 0 BF16, 1 INT8, 2 INT4
    freqs: torch.Tensor     # float32 [L, E]
    block_m: torch.Tensor   # int32 [L, E]
    hot_mask: torch.Tensor  # bool [L, E]

    @property
    def n_experts_total(self) -> int:
        return self.n_layers * self.n_experts_per_layer

    def layer_profile(self, layer_idx: int) -> dict:
        return {"tiers": self.tiers[layer_idx], "freqs": self.freqs[layer_idx],
                "block_m": self.block_m[layer_idx], "hot_mask": self.hot_mask[layer_idx]}

    def hot_expert_count(self, layer_idx: int) -> int:
        return int(self.hot_mask[layer_idx].sum().item())

    def expected_memory_ratio(self) -> float:
        ratio = torch.tensor([1.0, 0.5, 0.25], device=self.tiers.device)
        return float(ratio[self.tiers.long()].mean().item())

    def precision_counts(self) -> dict[str, int]:
        return {name: int((self.tiers == code).sum().item())
                for code, name in INT_TO_PRECISION.items()}

    def block_m_distribution(self) -> dict[int, int]:
        vals, counts = torch.unique(self.block_m.flatten().cpu(), return_counts=True)
        return {int(v): int(c) for v, c in zip(vals.tolist(), counts.tolist())}

    def layer_tier_names(self, layer_idx: int) -> list[str]:
        return [INT_TO_PRECISION[int(t)] for t in self.tiers[layer_idx].tolist()]


def load_exq_artifact(artifact_path: str, profile_path: str | None = None,
                      device: str = "cuda") -> ExpertProfile:
    """Artifact (+ optional routing profile) -> ExpertProfile on ``device``
    (exq_artifact.py:96-192)."""
    with open(artifact_path, encoding="utf-8") as f:
        artifact = json.load(f)
    assignments = artifact.get("quant_assignments", {})
    if not assignments:
        raise ValueError(f"Artifact at {artifact_path} has no quant_assignments")
    keys = [parse_quant_key(k) for k in assignments]
    n_layers = max(k[0] for k in keys) + 1
    n_experts = max(k[1] for k in keys) + 1

    tiers = np.full((n_layers, n_experts), PRECISION_TO_INT["INT4"], dtype=np.int8)
    for (layer, e), prec in zip(keys, assignments.values()):
        tiers[layer, e] = PRECISION_TO_INT.get(prec, PRECISION_TO_INT["INT4"])

    freqs = np.zeros((n_layers, n_experts), dtype=np.float32)
    candidates = [profile_path]
    if profile_path is None:
        stem = Path(artifact_path).stem
        candidates += [str(Path("profiles") / f"{stem}.json"),
                       str(Path("profiles") / "olmoe-1b-7b-0924-256.json")]
    loaded = False
    for cand in candidates:
        if cand and Path(cand).exists():
            with open(cand, encoding="utf-8") as f:
                prof = json.load(f)
            for layer_str, layer_data in prof.get("layers", {}).items():
                layer = int(layer_str)
                if layer >= n_layers:
                    continue
                for stats in layer_data.get("expert_stats", []):
                    e = stats.get("expert_id", 0)
                    if e < n_experts:
                        freqs[layer, e] = float(stats.get("activation_freq", 0.0))
            loaded = True
            break
    if not loaded:
        freqs = np.vectorize(lambda t: _TIER_TO_FREQ[int(t)], otypes=[np.float32])(tiers)

    block_m = np.vectorize(freq_to_block_m, otypes=[np.int32])(freqs, tiers.astype(np.int64))
    return ExpertProfile(
        n_layers=n_layers,
        n_experts_per_layer=n_experts,
        tiers=torch.from_numpy(tiers).to(device),
        freqs=torch.from_numpy(np.asarray(freqs, dtype=np.float32)).to(device),
        block_m=torch.from_numpy(np.asarray(block_m, dtype=np.int32)).to(device),
        hot_mask=torch.from_numpy(tiers == PRECISION_TO_INT["BF16"]).to(device),
    )
