"""Drop-in for the reference's ``exq.kernels`` package (exq/kernels/__init__.py:1-21).

Same names, signatures, argument meaning and return conventions as
exq/kernels/moe_int4_kernel.py and exq/kernels/moe_grouped_gemm.py; the work
runs in the sm_100a library through its C ABI.  Differences a caller can see:

* tensors must be on a CUDA device (there is no CPU path);
* ``block_m`` / ``block_n`` / ``block_k`` are accepted and ignored: the kernels
  choose their own tiles;
* INT4 GEMMs support group size 128 only (K a multiple of 128);
  ``pack_int4_weights`` itself supports every group size the reference does;
* ``moe_int4_full_forward`` returns the layer output the reference intends
  (the shipped reference raises NameError at moe_int4_kernel.py:424);
* sorting is stable and every reduction runs in a fixed order, so outputs are
  bit-reproducible run to run.
"""
from __future__ import annotations

import torch

from . import _lib as L
from .artifact import ExpertProfile, load_exq_artifact  # noqa: F401  (re-export)
from .experts import ExpertBank, pack_int4

_DESC_CACHE: dict = {}


def pack_int4_weights(weights: torch.Tensor, group_size: int = 128):
    """[N, K] -> (u8 [N, K//2], fp16 [N, K//group]) (moe_int4_kernel.py:37-93)."""
    if weights.dim() != 2:
        raise ValueError("weights must be [N, K]")
    return pack_int4(weights, group_size)


def pack_experts_int4(expert_weights: torch.Tensor, group_size: int = 128):
    """[E, N, K] -> (u8 [E, N, K//2], fp16 [E, N, K//group]) (moe_int4_kernel.py:96-119)."""
    if expert_weights.dim() != 3:
        raise ValueError("expert_weights must be [n_experts, N, K]")
    return pack_int4(expert_weights, group_size)


def _single_proj_desc(tier: int, w: torch.Tensor, s: torch.Tensor | None) -> torch.Tensor:
    """Descriptor array for a one-projection bank (cached by pointers/shapes)."""
    key = (tier, w.data_ptr(), tuple(w.shape), tuple(w.stride()), w.device,
           None if s is None else (s.data_ptr(), tuple(s.shape), tuple(s.stride())))
    d = _DESC_CACHE.get(key)
    if d is None:
        import numpy as np
        e = w.shape[0]
        rows = np.zeros((e, 5), dtype=np.int64)
        rows[:, 0] = tier
        rows[:, 1] = w.data_ptr() + np.arange(e, dtype=np.int64) * w.stride(0) * w.element_size()
        if s is not None:
            rows[:, 2] = s.data_ptr() + np.arange(e, dtype=np.int64) * s.stride(0) * s.element_size()
        d = torch.from_numpy(rows).to(w.device)
        if len(_DESC_CACHE) > 64:
            _DESC_CACHE.clear()
        _DESC_CACHE[key] = d
    return d


def _grouped_gemm(desc, n_experts, n_rows, k, hidden_states, router_indices, out_dtype,
                  want_routing=False):
    dev = L.require_cuda(hidden_states, router_indices)
    x = hidden_states.contiguous()
    ids = router_indices.contiguous()
    t, topk = ids.shape
    n = t * topk
    out = torch.empty(n, n_rows, dtype=out_dtype, device=dev)
    ws = L.workspace(dev, L.lib().exq_moe_gemm_workspace_bytes(t, topk, n_experts))
    so = torch.empty(n, dtype=torch.int64, device=dev) if want_routing else None
    ends = torch.empty(n_experts + 1, dtype=torch.int32, device=dev) if want_routing else None
    L.check(L.lib().exq_moe_gemm(L.ptr(desc), n_experts, n_rows, k, L.ptr(x), L.tag(x), t,
                                 L.ptr(ids), L.tag(ids), topk, L.ptr(out), L.tag(out), L.ptr(so),
                                 L.ptr(ends), L.ptr(ws), ws.numel(), L.stream_of(dev)),
            "moe_gemm")
    return (out, so, ends) if want_routing else out


def moe_int4_forward(hidden_states: torch.Tensor, expert_packed: torch.Tensor,
                     expert_scales: torch.Tensor, router_indices: torch.Tensor, n_experts: int,
                     group_size: int = 128, block_m: int = 64, block_n: int = 128,
                     block_k: int = 32) -> torch.Tensor:
    """One INT4 projection; returns [T*k, N] fp16 in expert-sorted (stable) order
    (moe_int4_kernel.py:245-327)."""
    L.require_cuda(hidden_states, expert_packed, expert_scales, router_indices)
    _, k = hidden_states.shape
    e, n, k_packed = expert_packed.shape
    if k_packed != k // 2:
        raise ValueError(f"packed K={k_packed} != K//2={k // 2}")
    eff_group = k // expert_scales.shape[2]
    if eff_group != 128:
        raise NotImplementedError(f"INT4 GEMM supports group size 128 (got {eff_group})")
    if not (expert_packed.is_contiguous() and expert_scales.is_contiguous()):
        raise ValueError("packed weights and scales must be contiguous")
    desc = _single_proj_desc(L.TIER_INT4, expert_packed, expert_scales)
    return _grouped_gemm(desc, e, n, k, hidden_states, router_indices, torch.float16)


def moe_int4_full_forward(hidden_states: torch.Tensor, w13_packed: torch.Tensor,
                          w13_scales: torch.Tensor, w2_packed: torch.Tensor,
                          w2_scales: torch.Tensor, router_indices: torch.Tensor,
                          router_weights: torch.Tensor, n_experts: int, group_size: int = 128,
                          block_m: int = 64, block_n: int = 128, block_k: int = 32) -> torch.Tensor:
    """gate_up -> SiLU*mul -> down -> weighted combine; returns [T, H]
    (moe_int4_kernel.py:330-426) in the activation dtype."""
    bank = ExpertBank.from_int4_packed(w13_packed.contiguous(), w13_scales.contiguous(),
                                       w2_packed.contiguous(), w2_scales.contiguous(),
                                       act_dtype=hidden_states.dtype)
    if bank.n_routed != n_experts:
        raise ValueError("n_experts does not match the packed weights")
    return bank.forward(hidden_states, router_indices, router_weights)


def moe_grouped_gemm(hidden_states: torch.Tensor, expert_weights: torch.Tensor,
                     router_indices: torch.Tensor, n_experts: int, block_m: int = 64,
                     block_n: int = 64, block_k: int = 32) -> torch.Tensor:
    """16-bit grouped GEMM; returns [T*k, N] fp16 in sorted order
    (moe_grouped_gemm.py:173-227)."""
    L.require_cuda(hidden_states, expert_weights, router_indices)
    _, k = hidden_states.shape
    e, n, k2 = expert_weights.shape
    if k != k2:
        raise ValueError(f"K mismatch: hidden_states K={k}, expert_weights K={k2}")
    if k % 128:
        raise NotImplementedError("grouped GEMM needs K to be a multiple of 128")
    w = expert_weights
    if w.dtype != hidden_states.dtype:
        w = w.to(hidden_states.dtype)
    w = w.contiguous()
    desc = _single_proj_desc(L.TIER_BF16, w, None)
    # a converted temporary may be freed right after: the caching allocator
    # only reuses its memory for work queued later on the same stream
    return _grouped_gemm(desc, e, n, k, hidden_states, router_indices, torch.float16)


def sort_tokens_by_expert(router_indices: torch.Tensor, hidden_states: torch.Tensor,
                          n_experts: int):
    """(sort_order i64, sorted_hidden, expert_ends i32 [E+1], max_tok int)
    (moe_grouped_gemm.py:139-166).  ``max_tok`` needs one device->host read, as
    in the reference."""
    from . import exq_dispatch_cuda as D
    dev = L.require_cuda(router_indices, hidden_states)
    n = router_indices.numel()
    top_k = router_indices.shape[1]
    so = torch.empty(n, dtype=torch.int64, device=dev)
    se = torch.empty(n, dtype=torch.int64, device=dev)
    ends = torch.empty(n_experts + 1, dtype=torch.int32, device=dev)
    D.dispatch(router_indices, so, se, ends, n_experts)
    sorted_hidden = torch.empty(n, hidden_states.shape[1], dtype=hidden_states.dtype, device=dev)
    D.gather_hidden(hidden_states, so, sorted_hidden, top_k)
    max_tok = int((ends[1:] - ends[:-1]).max().item()) if n > 0 else 1
    return so, sorted_hidden, ends, max_tok


def unsort_output(sorted_output: torch.Tensor, router_indices: torch.Tensor,
                  router_weights: torch.Tensor) -> torch.Tensor:
    """Weighted top-k recombination of sorted rows (moe_grouped_gemm.py:234-260)."""
    from . import exq_dispatch_cuda as D
    dev = L.require_cuda(sorted_output, router_indices, router_weights)
    n = router_indices.numel()
    so = torch.empty(n, dtype=torch.int64, device=dev)
    se = torch.empty(n, dtype=torch.int64, device=dev)
    e = int(router_indices.max().item()) + 1 if n else 1
    ends = torch.empty(e + 1, dtype=torch.int32, device=dev)
    D.dispatch(router_indices, so, se, ends, e)
    out_dtype = torch.promote_types(sorted_output.dtype, router_weights.dtype)
    result = torch.empty(router_indices.shape[0], sorted_output.shape[1], dtype=out_dtype,
                         device=dev)
    D.combine(sorted_output, so, router_weights, result)
    return result


def router_topk(router_logits: torch.Tensor, top_k: int, renormalize: bool = True):
    """``(topk_ids int32 [T, k], topk_weights fp32 [T, k])`` from router logits
    ``[T, E]`` (fp32/fp16/bf16): softmax, the ``top_k`` largest probabilities
    (descending; equal ones by lower expert id), divided by their sum when
    ``renormalize``.  The routing the reference's generated layers compute
    (exq/codegen/triton_emitter.py:273-276), i.e. SGLang's ``topk_output``
    (exq/runtime/sglang_backend.py:88-90), in one kernel."""
    dev = L.require_cuda(router_logits)
    if router_logits.dim() != 2:
        raise ValueError("router_logits must be [T, E]")
    x = router_logits.contiguous()
    t, e = x.shape
    ids = torch.empty(t, top_k, dtype=torch.int32, device=dev)
    w = torch.empty(t, top_k, dtype=torch.float32, device=dev)
    L.check(L.lib().exq_router_topk(L.ptr(x), L.tag(x), t, e, int(top_k), int(bool(renormalize)),
                                    L.ptr(ids), L.ptr(w), L.stream_of(dev)), "router_topk")
    return ids, w


__all__ = [
    "router_topk",
    "moe_grouped_gemm",
    "sort_tokens_by_expert",
    "moe_int4_forward",
    "moe_int4_full_forward",
    "pack_experts_int4",
    "pack_int4_weights",
    "load_exq_artifact",
    "ExpertProfile",
    "unsort_output",
]
