"""fp32 MoE-layer oracle (CPU, torch fp32 matmuls).

Test infrastructure only: never imported by the shipped package.  It is also
the CPU baseline that ``bench.py`` times (the reference's torch
dequant+matmul path).

Composition (each step cites the reference):
1. dequantise every expert to fp32 (scripts/bench_int4.py:62-78 for INT4,
   exq/eval/quant_shim.py:84-96 for INT8; BF16 weights as stored);
2. route: stable sort of the flat top-k ids (moe_grouped_gemm.py:139-166);
3. per expert, ``gate_up = x @ W13[e]^T`` (the Triton GEMM,
   moe_int4_kernel.py:124-240, output rounded to the activation dtype as the
   kernel's fp16 store does, :238-240);
4. ``mid = silu(gate) * up`` in fp32, rounded (sgl_kernel silu_and_mul,
   moe_int4_kernel.py:398-400);
5. ``down = mid @ W2[e]^T``, rounded (:402-420);
6. ``y[t] = sum_j w[t,j] * down[t,j]`` in fp32, rounded
   (exq_dispatch.cu:263-310; the top-k sum of moe_int4_kernel.py:423-426).
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from . import quant


def dequant_expert(tier: str, w13, w2):
    """One expert's (w13 [2I,H], w2 [H,I]) as fp32 torch tensors.

    ``w13``/``w2`` are ``(packed, scales)`` for INT4, ``(q, scales)`` for INT8,
    or a 16-bit array for BF16.
    """
    if tier == "INT4":
        a = quant.dequant_int4(*w13)
        b = quant.dequant_int4(*w2)
    elif tier == "INT8":
        a = quant.dequant_int8(*w13)
        b = quant.dequant_int8(*w2)
    elif tier == "BF16":
        a = _to_f32(w13)
        b = _to_f32(w2)
    else:
        raise ValueError(tier)
    return torch.as_tensor(np.asarray(a, dtype=np.float32)), torch.as_tensor(
        np.asarray(b, dtype=np.float32))


def _to_f32(x):
    if isinstance(x, torch.Tensor):
        return x.float().numpy()
    return np.asarray(x, dtype=np.float32)


def _round(x: torch.Tensor, dtype) -> torch.Tensor:
    return x if dtype is None else x.to(dtype).float()


def moe_layer(hidden: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor,
              w13_f32: list, w2_f32: list, act_dtype=torch.float16,
              round_intermediates: bool = True) -> torch.Tensor:
    """fp32 MoE layer; returns fp32 ``[T, H]`` (cast by the caller).

    ``w13_f32[e]`` / ``w2_f32[e]`` are the dequantised fp32 weights of expert e
    (``None`` for experts that cannot be routed to); ``w13_f32`` may instead be
    a callable ``e -> (w13, w2)`` that dequantises on demand (``w2_f32`` is
    then ignored).  With ``round_intermediates`` the activations are cast to
    fp16 and the gate_up, mid and down tensors are rounded to fp16, where and
    as the reference does whatever the model dtype: its GEMM loads the
    activations ``.to(tl.float16)`` (exq/kernels/moe_int4_kernel.py:199) and
    stores out1 / mid / out2 as fp16 (:386-410).  ``act_dtype`` is the dtype
    of the caller's hidden states (the output is cast to it by the caller).
    """
    rd = torch.float16 if round_intermediates else None
    x = _round(hidden.float(), rd)
    t, k = topk_ids.shape
    flat = topk_ids.reshape(-1).long()
    wts = topk_weights.reshape(-1).float()
    order = torch.argsort(flat, stable=True)
    y = torch.zeros(t, x.shape[1], dtype=torch.float32)
    sorted_e = flat[order]
    if order.numel() == 0:
        return y
    uniq, counts = torch.unique_consecutive(sorted_e, return_counts=True)
    start = 0
    for e, c in zip(uniq.tolist(), counts.tolist()):
        slots = order[start:start + c]
        start += c
        toks = slots // k
        xe = x[toks]
        if callable(w13_f32):
            we13, we2 = w13_f32(e)
        else:
            we13, we2 = w13_f32[e], w2_f32[e]
        gu = _round(xe @ we13.T, rd)
        inter = gu.shape[1] // 2
        g, u = gu[:, :inter], gu[:, inter:]
        mid = _round(g * torch.sigmoid(g) * u, rd)
        d = _round(mid @ we2.T, rd)
        y.index_add_(0, toks, d * wts[slots, None])
    return y


def moe_projection(hidden: torch.Tensor, topk_ids: torch.Tensor, w_f32: torch.Tensor):
    """One projection in expert-sorted order (``moe_int4_forward``,
    moe_int4_kernel.py:245-327): ``out[i] = x[sort_order[i] // k] @ W[e_i]^T``.

    ``w_f32``: [E, N, K] fp32, or a callable ``e -> [N, K]``.  Returns fp32
    ``[T*k, N]``.
    """
    k = topk_ids.shape[1]
    flat = topk_ids.reshape(-1).long()
    order = torch.argsort(flat, stable=True)
    x = hidden.float()[order // k]
    get = w_f32 if callable(w_f32) else (lambda e: w_f32[e])
    sorted_e = flat[order]
    if order.numel() == 0:
        return torch.empty(0, 0)
    uniq, counts = torch.unique_consecutive(sorted_e, return_counts=True)
    out = None
    start = 0
    for e, c in zip(uniq.tolist(), counts.tolist()):
        w = get(e)
        if out is None:
            out = torch.empty(order.numel(), w.shape[0], dtype=torch.float32)
        out[start:start + c] = x[start:start + c] @ w.T
        start += c
    return out


def rel_l2(y: torch.Tensor, y_ref: torch.Tensor) -> float:
    """``||y - y_ref||_2 / ||y_ref||_2`` in fp32 (the parity metric)."""
    y = y.float().cpu()
    y_ref = y_ref.float().cpu()
    den = torch.linalg.vector_norm(y_ref).item()
    return torch.linalg.vector_norm(y - y_ref).item() / max(den, 1e-30)


def max_diff_over_rms(y: torch.Tensor, y_ref: torch.Tensor) -> float:
    """The reference's own check, scripts/bench_int4.py:88-93."""
    y = y.float().cpu()
    y_ref = y_ref.float().cpu()
    rms = y_ref.pow(2).mean().sqrt().item()
    return (y - y_ref).abs().max().item() / max(rms, 1e-6)


def silu(x: torch.Tensor) -> torch.Tensor:
    return F.silu(x)
