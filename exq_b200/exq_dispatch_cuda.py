"""Drop-in for the reference's ``exq_dispatch_cuda`` extension module.

Same functions, argument meaning and output-argument convention as
exq/kernels/cuda_src/exq_dispatch.cu:312-318 (every function fills
caller-preallocated tensors and returns None), plus the two sgl_kernel steps
the SGLang backend calls (``moe_align_block_size``, ``silu_and_mul``,
exq/runtime/sglang_backend.py:79, :108-109, :140), so ``patch_sglang`` runs
without sgl_kernel.  Every call enqueues on torch's current CUDA stream and
goes through the C ABI of ``libexq_b200.so``; nothing falls back to the CPU.
Argument errors raise ``ValueError`` (the reference raised ``c10::Error`` from
``data_ptr<T>()``, surfacing as ``RuntimeError``).
"""
from __future__ import annotations

import torch

from . import _lib as L


def _contig(t: torch.Tensor, name: str) -> torch.Tensor:
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t


def dispatch(router_indices: torch.Tensor, sort_order: torch.Tensor,
             sorted_expert_ids: torch.Tensor, expert_ends: torch.Tensor, n_experts: int) -> None:
    """Stable sort of the flat top-k ids by expert (exq_dispatch.cu:99-149).

    ``sort_order`` / ``sorted_expert_ids`` int64 [T*k], ``expert_ends`` int32 [E+1].
    """
    dev = L.require_cuda(router_indices, sort_order, sorted_expert_ids, expert_ends)
    ids = router_indices.reshape(-1).contiguous()
    n = ids.numel()
    if sort_order.dtype != torch.int64 or sorted_expert_ids.dtype != torch.int64:
        raise ValueError("sort_order and sorted_expert_ids must be int64")
    if expert_ends.dtype != torch.int32 or expert_ends.numel() != n_experts + 1:
        raise ValueError("expert_ends must be int32 [n_experts + 1]")
    if sort_order.numel() != n or sorted_expert_ids.numel() != n:
        raise ValueError("sort_order / sorted_expert_ids must have T*k entries")
    L.check(L.lib().exq_dispatch(L.ptr(ids), L.tag(ids), n, int(n_experts),
                                 L.ptr(_contig(sort_order, "sort_order")),
                                 L.ptr(_contig(sorted_expert_ids, "sorted_expert_ids")),
                                 L.ptr(_contig(expert_ends, "expert_ends")), L.stream_of(dev)),
            "dispatch")


def build_ends_from_slots(sorted_slot_ids: torch.Tensor, flat_router: torch.Tensor,
                          expert_ends: torch.Tensor, sort_order: torch.Tensor, n_active: int,
                          n_experts: int) -> None:
    """``expert_ends`` and ``sort_order`` from align output (exq_dispatch.cu:181-229).

    ``sorted_slot_ids`` int32 [EM] (entries >= n_active are padding),
    ``flat_router`` int32 [n_active], ``expert_ends`` int32 [E+1] (no pre-zeroing
    needed), ``sort_order`` int64 [n_active].  One launch, no temporaries.
    """
    dev = L.require_cuda(sorted_slot_ids, flat_router, expert_ends, sort_order)
    if sorted_slot_ids.dtype != torch.int32 or flat_router.dtype != torch.int32:
        raise ValueError("sorted_slot_ids and flat_router must be int32")
    if expert_ends.dtype != torch.int32 or expert_ends.numel() != n_experts + 1:
        raise ValueError("expert_ends must be int32 [n_experts + 1]")
    if sort_order.dtype != torch.int64 or sort_order.numel() < n_active:
        raise ValueError("sort_order must be int64 with n_active entries")
    if flat_router.numel() < n_active:
        raise ValueError("flat_router has fewer than n_active entries")
    L.check(L.lib().exq_build_ends_from_slots(
        L.ptr(_contig(sorted_slot_ids, "sorted_slot_ids")), sorted_slot_ids.numel(),
        L.ptr(_contig(flat_router, "flat_router")), int(n_active), int(n_experts),
        L.ptr(_contig(expert_ends, "expert_ends")), L.ptr(_contig(sort_order, "sort_order")),
        L.stream_of(dev)), "build_ends_from_slots")


def gather_hidden(hidden: torch.Tensor, sort_order: torch.Tensor, out: torch.Tensor,
                  top_k: int) -> None:
    """``out[i] = hidden[sort_order[i] // top_k]`` (exq_dispatch.cu:234-260); fp16/bf16."""
    dev = L.require_cuda(hidden, sort_order, out)
    if hidden.dim() != 2 or hidden.stride(1) != 1:
        raise ValueError("hidden must be [T, H] with unit inner stride")
    if out.dtype != hidden.dtype or not out.is_contiguous():
        raise ValueError("out must be contiguous with hidden's dtype")
    if sort_order.dtype != torch.int64:
        raise ValueError("sort_order must be int64")
    n = sort_order.numel()
    if out.numel() != n * hidden.shape[1]:
        raise ValueError("out must be [len(sort_order), H]")
    L.check(L.lib().exq_gather_hidden(L.ptr(hidden), L.tag(hidden), hidden.shape[0],
                                      hidden.shape[1], hidden.stride(0),
                                      L.ptr(_contig(sort_order, "sort_order")), n, int(top_k),
                                      L.ptr(out), L.stream_of(dev)), "gather_hidden")


def combine(down_out: torch.Tensor, sort_order: torch.Tensor, router_weights: torch.Tensor,
            result: torch.Tensor) -> None:
    """``result[t] = sum_j w[t, j] * down_out[pos(t, j)]`` (exq_dispatch.cu:263-310).

    Deterministic fp32 sum in top-k order; weights fp32/fp16/bf16.
    """
    dev = L.require_cuda(down_out, sort_order, router_weights, result)
    if router_weights.dim() != 2:
        raise ValueError("router_weights must be [T, k]")
    t, k = router_weights.shape
    w = router_weights.contiguous()
    d = _contig(down_out, "down_out")
    h = d.shape[-1]
    if result.numel() != t * h or not result.is_contiguous():
        raise ValueError("result must be a contiguous [T, H]")
    if sort_order.dtype != torch.int64:
        raise ValueError("sort_order must be int64")
    n = sort_order.numel()
    ws = L.workspace(dev, L.lib().exq_combine_workspace_bytes(n))
    L.check(L.lib().exq_combine(L.ptr(d), L.tag(d), n, h, L.ptr(_contig(sort_order, "sort_order")),
                                L.ptr(w), L.tag(w), t, k, L.ptr(result), L.tag(result),
                                L.ptr(ws), ws.numel(), L.stream_of(dev)), "combine")


def moe_align_block_size(topk_ids: torch.Tensor, num_experts: int, block_size: int,
                         sorted_token_ids: torch.Tensor, experts_ids: torch.Tensor,
                         num_tokens_post_pad: torch.Tensor, cumsum_buffer: torch.Tensor,
                         pad_sorted_token_ids: bool = False) -> None:
    """sgl_kernel ``moe_align_block_size`` (exq/runtime/sglang_backend.py:102-109).

    Slots are written in ascending order inside each expert's padded range;
    ``experts_ids`` holds -1 for blocks past ``num_tokens_post_pad``;
    ``cumsum_buffer[num_experts + 1]`` receives the exclusive padded prefix.
    """
    dev = L.require_cuda(topk_ids, sorted_token_ids, experts_ids, num_tokens_post_pad,
                         cumsum_buffer)
    for name, tt in (("sorted_token_ids", sorted_token_ids), ("experts_ids", experts_ids),
                     ("num_tokens_post_pad", num_tokens_post_pad),
                     ("cumsum_buffer", cumsum_buffer)):
        if tt.dtype != torch.int32 or not tt.is_contiguous():
            raise ValueError(f"{name} must be a contiguous int32 tensor")
    if cumsum_buffer.numel() < num_experts + 1:
        raise ValueError("cumsum_buffer needs num_experts + 1 entries")
    ids = topk_ids.reshape(-1).contiguous()
    L.check(L.lib().exq_moe_align_block_size(
        L.ptr(ids), L.tag(ids), ids.numel(), int(num_experts), int(block_size),
        L.ptr(sorted_token_ids), sorted_token_ids.numel(), L.ptr(experts_ids),
        experts_ids.numel(), L.ptr(num_tokens_post_pad), L.ptr(cumsum_buffer),
        int(bool(pad_sorted_token_ids)), L.stream_of(dev)), "moe_align_block_size")


def silu_and_mul(input: torch.Tensor, out: torch.Tensor) -> None:
    """sgl_kernel ``silu_and_mul``: ``out = silu(x[:, :I]) * x[:, I:]`` (fp32 math)."""
    dev = L.require_cuda(input, out)
    x = _contig(input, "input")
    i2 = x.shape[-1]
    if i2 % 2:
        raise ValueError("input's last dimension must be even")
    m = x.numel() // i2
    if out.dtype != x.dtype or not out.is_contiguous() or out.numel() != m * (i2 // 2):
        raise ValueError("out must be contiguous [.., I] with input's dtype")
    L.check(L.lib().exq_silu_and_mul(L.ptr(x), L.ptr(out), L.tag(x), m, i2 // 2,
                                     L.stream_of(dev)), "silu_and_mul")
