"""SGLang integration: drop-in for exq/runtime/sglang_backend.py.

``patch_sglang(artifact_path)`` replaces SGLang's
``UnquantizedFusedMoEMethod.forward_cuda`` (sglang_backend.py:183-210); layers
at or beyond the artifact's layer count fall through to SGLang's own kernel
(:83-85); re-patching clears the packed-weight cache (:197-199).

Differences from the reference, all on the data path:

* the artifact's per-expert precisions are honoured: each expert of a layer is
  packed to its ``quant_assignments`` tier (the reference packs every expert
  INT4, :40-45) and all tiers run in the same grouped launch;
* the layer runs as route -> gate_up(+gather) -> SiLU*mul -> down -> combine in
  four launches with no host synchronisation (the reference reads ``max_tok``
  back to the host every call, :121) and no per-call allocation beyond torch's
  caching allocator;
* fp16 and bf16 activations are both served, with fp32 / fp16 / bf16 router
  weights.
"""
from __future__ import annotations

import json
import logging
import time
import types

import torch

from .artifact import layer_tiers
from .experts import ExpertBank

logger = logging.getLogger(__name__)

# id(layer) -> packed bank + metadata (packed on first call, reused after)
_exq_packed_cache: dict[int, dict] = {}
_artifact_state: dict = {"artifact": {}}


def _get_or_pack(layer) -> dict:
    """Pack ``layer.w13_weight`` / ``w2_weight`` per the quant plan, once."""
    key = id(layer)
    if key in _exq_packed_cache:
        return _exq_packed_cache[key]
    t0 = time.perf_counter()
    w1 = layer.w13_weight
    w2 = layer.w2_weight
    act_dtype = w1.dtype if w1.dtype in (torch.float16, torch.bfloat16) else torch.float16
    n_experts = w1.shape[0]
    tiers = layer_tiers(_artifact_state["artifact"], int(getattr(layer, "layer_id", 0) or 0),
                        n_experts)
    # the reference quantises from fp16 copies of the weights (:41-42)
    bank = ExpertBank.from_dense(w1.to(torch.float16), w2.to(torch.float16), tiers,
                                 act_dtype=act_dtype)
    cache = {
        "bank": bank,
        "n_experts": n_experts,
        "inter2": w1.shape[1],
        "hidden": w1.shape[2],
        "tiers": tiers,
    }
    _exq_packed_cache[key] = cache
    logger.info("ExQ: packed layer %s in %.1fms", getattr(layer, "layer_id", "?"),
                (time.perf_counter() - t0) * 1000)
    return cache


def _combine_input(hidden_states: torch.Tensor):
    try:
        from sglang.srt.layers.moe.token_dispatcher.standard import StandardCombineInput
    except ImportError:
        return types.SimpleNamespace(hidden_states=hidden_states)
    return StandardCombineInput(hidden_states=hidden_states)


def _exq_forward_cuda(self_method, layer, dispatch_output, _original_forward_cuda,
                      _artifact_n_layers: int):
    """Replacement for UnquantizedFusedMoEMethod.forward_cuda (sglang_backend.py:65-158)."""
    layer_id = getattr(layer, "layer_id", None)
    if layer_id is None or layer_id >= _artifact_n_layers:
        return _original_forward_cuda(self_method, layer, dispatch_output)
    hidden = dispatch_output.hidden_states
    topk = dispatch_output.topk_output
    cache = _get_or_pack(layer)
    bank: ExpertBank = cache["bank"]
    if hidden.dtype != bank.act_dtype:
        hidden = hidden.to(bank.act_dtype)
    out = bank.forward(hidden, topk.topk_ids, topk.topk_weights)
    return _combine_input(out)


class ExQSGLangBackend:
    """Artifact metadata and the per-layer packed-weight cache (:163-180)."""

    def __init__(self, artifact_path: str):
        with open(artifact_path, encoding="utf-8") as f:
            artifact = json.load(f)
        qa = artifact.get("quant_assignments", {})
        layer_ids = {int(k.split(":")[0]) for k in qa}
        self.n_layers = max(layer_ids) + 1 if layer_ids else 0
        self.artifact_path = artifact_path
        self.artifact = artifact
        logger.info("ExQ SGLang backend: %d layers (%d assignments)", self.n_layers, len(qa))

    def clear_cache(self):
        _exq_packed_cache.clear()

    def cache_stats(self) -> dict:
        return {"n_layers_cached": len(_exq_packed_cache), "n_layers_in_artifact": self.n_layers}


def make_patched_forward(original, n_layers: int):
    def patched(self, layer, dispatch_output):
        return _exq_forward_cuda(self, layer, dispatch_output, original, n_layers)
    return patched


def patch_sglang(artifact_path: str) -> ExQSGLangBackend:
    """Route SGLang's unquantized fused-MoE forward through exq_b200 (:183-210)."""
    try:
        from sglang.srt.layers.quantization.unquant import UnquantizedFusedMoEMethod
    except ImportError as exc:
        raise ImportError("SGLang not installed: pip install sglang") from exc
    backend = ExQSGLangBackend(artifact_path)
    _artifact_state["artifact"] = backend.artifact
    if getattr(UnquantizedFusedMoEMethod, "_exq_patched", False):
        logger.warning("ExQ: re-patching SGLang (cache cleared)")
        _exq_packed_cache.clear()
        original = UnquantizedFusedMoEMethod._exq_original_forward_cuda
    else:
        original = UnquantizedFusedMoEMethod.forward_cuda
    UnquantizedFusedMoEMethod._exq_original_forward_cuda = original
    UnquantizedFusedMoEMethod.forward_cuda = make_patched_forward(original, backend.n_layers)
    UnquantizedFusedMoEMethod._exq_patched = True
    logger.info("ExQ: patched SGLang (%d layers covered)", backend.n_layers)
    return backend


def unpatch_sglang():
    """Restore SGLang's original forward_cuda (:213-225)."""
    try:
        from sglang.srt.layers.quantization.unquant import UnquantizedFusedMoEMethod
    except ImportError:
        return
    if not getattr(UnquantizedFusedMoEMethod, "_exq_patched", False):
        return
    UnquantizedFusedMoEMethod.forward_cuda = UnquantizedFusedMoEMethod._exq_original_forward_cuda
    UnquantizedFusedMoEMethod._exq_patched = False
    _exq_packed_cache.clear()
    logger.info("ExQ: SGLang patch removed")


def set_artifact(artifact: dict) -> None:
    """Install a quant plan without SGLang (library use and tests)."""
    _artifact_state["artifact"] = artifact
    _exq_packed_cache.clear()
