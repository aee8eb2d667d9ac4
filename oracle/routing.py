"""Routing-metadata oracle: sort / align / ends / gather / combine (CPU, numpy).

Test infrastructure only: never imported by the shipped package.

Canonical forms.  Where the reference leaves an order to atomics
(``compact_via_expert_counter_kernel``, exq/kernels/cuda_src/exq_dispatch.cu
:160-178, and sgl_kernel's align scatter), this oracle emits the stable
ascending order: within an expert, slots appear in increasing flat-slot index.
That order is one of the outputs the reference may legally produce; tests of
reference-produced data compare per-expert segments as sets, tests of this
build compare exactly.
"""
from __future__ import annotations

import numpy as np


def sort_tokens_by_expert(router_indices: np.ndarray, n_experts: int):
    """Restates moe_grouped_gemm.py:139-166 (minus the hidden gather).

    Returns ``(sort_order i64 [n], ends i32 [E+1], max_tok)``: a stable argsort
    of the flat expert ids, the bincount prefix and the largest count (1 when
    there are no slots, :164).
    """
    flat = np.asarray(router_indices).reshape(-1).astype(np.int64)
    order = np.argsort(flat, kind="stable").astype(np.int64)
    counts = np.bincount(flat, minlength=n_experts)[:n_experts]
    ends = np.zeros(n_experts + 1, dtype=np.int32)
    ends[1:] = np.cumsum(counts).astype(np.int32)
    max_tok = int(counts.max()) if flat.size > 0 else 1
    return order, ends, max_tok


def dispatch(router_indices: np.ndarray, n_experts: int):
    """Restates ``exq_dispatch`` (exq_dispatch.cu:99-149).

    CUB's radix sort over the low ceil(log2(E+1)) bits is stable, so the
    permutation is exactly the stable argsort.  Returns
    ``(sort_order i64, sorted_expert_ids i64, expert_ends i32 [E+1])``.
    """
    order, ends, _ = sort_tokens_by_expert(router_indices, n_experts)
    flat = np.asarray(router_indices).reshape(-1).astype(np.int64)
    return order, flat[order], ends


def align_capacity(numel: int, num_experts: int, block_size: int):
    """Buffer sizes the caller allocates (exq/runtime/sglang_backend.py:102-106)."""
    max_padded = numel + num_experts * (block_size - 1)
    return max_padded, -(-max_padded // block_size)


def moe_align_block_size(topk_ids: np.ndarray, num_experts: int, block_size: int,
                         sorted_cap: int | None = None, pad_sorted: bool = True):
    """Restates the sgl_kernel ``moe_align_block_size`` contract.

    Called by exq/runtime/sglang_backend.py:102-109 with ``num_experts = E+1``
    and ``block_size = 16``.  Contract (also documented by the vLLM op
    docstring): count the flat slots per expert over ``num_experts`` buckets,
    round each count up to a multiple of ``block_size``, exclusive-scan the
    padded counts into ``cumsum`` (length ``num_experts + 1``), write each slot
    index into its expert's range (canonical ascending order here), fill every
    other position with the pad value ``numel``; ``expert_ids[b]`` is the
    expert that owns block ``b`` for blocks below ``num_tokens_post_pad /
    block_size`` and -1 beyond.
    """
    flat = np.asarray(topk_ids).reshape(-1).astype(np.int64)
    n = flat.size
    max_padded, max_blocks = align_capacity(n, num_experts, block_size)
    if sorted_cap is None:
        sorted_cap = max_padded
    counts = np.bincount(flat, minlength=num_experts)[:num_experts]
    padded = (counts + block_size - 1) // block_size * block_size
    cumsum = np.zeros(num_experts + 1, dtype=np.int32)
    cumsum[1:] = np.cumsum(padded)
    ntpp = int(cumsum[-1])
    sorted_ids = np.full(sorted_cap, n, dtype=np.int32)
    fill = np.array(cumsum[:-1], dtype=np.int64)
    for s in range(n):
        e = flat[s]
        sorted_ids[fill[e]] = s
        fill[e] += 1
    expert_ids = np.full(max_blocks, -1, dtype=np.int32)
    for e in range(num_experts):
        expert_ids[cumsum[e] // block_size: cumsum[e + 1] // block_size] = e
    return sorted_ids, expert_ids, np.array([ntpp], dtype=np.int32), cumsum


def build_ends_from_slots(sorted_slot_ids: np.ndarray, flat_router: np.ndarray,
                          n_active: int, n_experts: int):
    """Restates ``exq_build_ends_from_slots`` (exq_dispatch.cu:181-229).

    Histogram of the expert of every valid slot (slot < n_active, :92-95),
    inclusive scan into ``ends[1:]`` (:202-214), then compaction of the valid
    slots into ``sort_order`` at per-expert cursors (:160-178), here in stable
    order of appearance.
    """
    ids = np.asarray(sorted_slot_ids).reshape(-1).astype(np.int64)
    fr = np.asarray(flat_router).reshape(-1).astype(np.int64)
    valid = ids[ids < n_active]
    experts = fr[valid]
    counts = np.bincount(experts, minlength=n_experts)[:n_experts]
    ends = np.zeros(n_experts + 1, dtype=np.int32)
    ends[1:] = np.cumsum(counts)
    cursor = ends[:-1].astype(np.int64).copy()
    sort_order = np.zeros(n_active, dtype=np.int64)
    for s, e in zip(valid, experts):
        sort_order[cursor[e]] = s
        cursor[e] += 1
    return ends, sort_order


def gather_hidden(hidden: np.ndarray, sort_order: np.ndarray, top_k: int) -> np.ndarray:
    """Restates ``gather_hidden_vec_kernel`` (exq_dispatch.cu:234-260): a row copy."""
    return np.asarray(hidden)[np.asarray(sort_order, dtype=np.int64) // top_k]


def combine(down_out: np.ndarray, sort_order: np.ndarray, router_weights: np.ndarray,
            out_dtype=np.float16) -> np.ndarray:
    """Restates ``exq_combine`` (exq_dispatch.cu:263-310).

    ``result[t] = cast(sum_j w[t, j] * down[pos(t, j)])`` with fp32 products and
    an fp32 sum; the sum runs in top-k order j = 0..k-1 (the reference's atomics
    leave the order open).
    """
    down = np.asarray(down_out, dtype=np.float32)
    w = np.asarray(router_weights, dtype=np.float32)
    t, k = w.shape
    so = np.asarray(sort_order, dtype=np.int64)
    inv = np.empty_like(so)
    inv[so] = np.arange(so.size)
    acc = np.zeros((t, down.shape[1]), dtype=np.float32)
    for j in range(k):
        rows = inv[np.arange(t) * k + j]
        acc += w[:, j:j + 1] * down[rows]
    return acc.astype(out_dtype)


def silu_and_mul(x: np.ndarray, out_dtype=np.float16) -> np.ndarray:
    """sgl_kernel ``silu_and_mul``: ``silu(x[:, :I]) * x[:, I:]`` in fp32."""
    xf = np.asarray(x, dtype=np.float32)
    i = xf.shape[-1] // 2
    g, u = xf[..., :i], xf[..., i:]
    return (g / (np.float32(1.0) + np.exp(-g)) * u).astype(out_dtype)


def router_topk(logits, top_k: int, renormalize: bool = True):
    """Router top-k as the reference's generated MoE layers compute it
    (exq/codegen/triton_emitter.py:273-276): ``softmax`` over the experts in
    fp32, ``torch.topk`` of the probabilities, then the selected weights
    divided by their sum (the renormalisation; SGLang's ``topk_output`` that
    exq/runtime/sglang_backend.py:88-90 receives is the same computation).
    Returns (ids int64 [T, k], weights fp32 [T, k]), weights in descending
    order.  Equal probabilities are ordered by the lower expert id here (the
    reference leaves that to torch.topk)."""
    import torch
    p = torch.softmax(torch.as_tensor(logits).float(), dim=-1)
    t, e = p.shape
    # stable descending order: sort by (-p, expert)
    order = torch.argsort(-p, dim=-1, stable=True)[:, :top_k]
    w = torch.gather(p, 1, order)
    if renormalize:
        w = w / w.sum(dim=-1, keepdim=True)
    return order, w
