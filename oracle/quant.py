"""Weight-tier oracle: INT4 / INT8 / BF16 packing and dequantisation (CPU, numpy).

Test infrastructure only: never imported by the shipped package.

INT4 (exq/kernels/moe_int4_kernel.py:37-93, pack_int4_weights)
    Per row, per group of ``group_size`` (128) consecutive K elements:
    ``scale = max(amax(|w|) / 7, eps_f32)`` computed in fp32 (:75-78),
    ``q = clamp(round_half_even(w / scale), -8, 7)`` (:80-81),
    nibble ``q + 8``; even K in the low nibble, odd K in the high nibble
    (:87-89); scales stored as fp16 (:91).  When ``K < group_size`` the group
    is the whole row (:63-64).
INT8 (exq/eval/quant_shim.py:84-96, quantize_tensor_int8)
    Per output row: ``scale = max(amax(|w|) / 127, eps_f32)``,
    ``q = clamp(round(w / scale), -128, 127)``.  The reference keeps the scale
    in fp32 and only simulates the tier; the packed INT8 tier of this build
    stores the scale as fp16 (the format the quant plan names), so this oracle
    returns the fp16 scale and dequantises with it.
BF16 / 16-bit tier
    Weights used as stored (exq/kernels/exq_artifact.py:25, tier 0).
"""
from __future__ import annotations

import numpy as np

F32_EPS = np.float32(np.finfo(np.float32).eps)


def pack_int4(w: np.ndarray, group_size: int = 128):
    """Restates ``pack_int4_weights`` (moe_int4_kernel.py:37-93).

    ``w``: [N, K] (any float dtype; promoted to fp32 exactly as the reference's
    ``weights.float()``).  Returns ``(packed u8 [N, K/2], scales f16 [N, K/gs])``.
    """
    w = np.asarray(w)
    if w.ndim != 2:
        raise ValueError("pack_int4 expects a [N, K] matrix")
    n, k = w.shape
    if k % 2 != 0:
        raise ValueError(f"K={k} must be divisible by 2 for INT4 packing")
    if k < group_size:
        group_size = k
    if k % group_size != 0:
        raise ValueError(f"K={k} must be divisible by group_size={group_size}")
    ng = k // group_size
    wf = w.astype(np.float32).reshape(n, ng, group_size)
    scale = np.abs(wf).max(axis=-1) / np.float32(7.0)
    scale = np.maximum(scale, F32_EPS).astype(np.float32)
    q = np.clip(np.rint(wf / scale[..., None]), -8, 7).astype(np.int8).reshape(n, k)
    lo = (q[:, 0::2] + 8).astype(np.uint8)
    hi = (q[:, 1::2] + 8).astype(np.uint8)
    packed = (lo | (hi << 4)).astype(np.uint8)
    return packed, scale.astype(np.float16)


def pack_experts_int4(w: np.ndarray, group_size: int = 128):
    """Restates ``pack_experts_int4`` (moe_int4_kernel.py:96-119): per-expert loop."""
    outs = [pack_int4(w[e], group_size) for e in range(w.shape[0])]
    return (np.stack([o[0] for o in outs]), np.stack([o[1] for o in outs]))


def unpack_int4_values(packed: np.ndarray) -> np.ndarray:
    """Nibbles back to signed integers in [-8, 7], original K order."""
    p = np.asarray(packed, dtype=np.uint8)
    lo = (p & 0x0F).astype(np.int8) - 8
    hi = ((p >> 4) & 0x0F).astype(np.int8) - 8
    out = np.empty(p.shape[:-1] + (p.shape[-1] * 2,), dtype=np.int8)
    out[..., 0::2] = lo
    out[..., 1::2] = hi
    return out


def dequant_int4(packed: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """fp32 dequantisation as scripts/bench_int4.py:62-78 does it.

    ``(nibble - 8) * scale`` with the fp16 scale promoted to fp32 and repeated
    over each group along K; works for [..., N, K/2] with scales [..., N, G].
    """
    q = unpack_int4_values(packed).astype(np.float32)
    k = q.shape[-1]
    gs = k // scales.shape[-1]
    s = np.repeat(np.asarray(scales, dtype=np.float32), gs, axis=-1)
    return q * s


def quant_int8(w: np.ndarray):
    """Per-output-row symmetric INT8 (quant_shim.py:84-96) -> (int8 [N,K], f16 [N])."""
    wf = np.asarray(w).astype(np.float32)
    scale = np.abs(wf).max(axis=-1) / np.float32(127.0)
    scale = np.maximum(scale, F32_EPS).astype(np.float32)
    q = np.clip(np.rint(wf / scale[..., None]), -128, 127).astype(np.int8)
    return q, scale.astype(np.float16)


def dequant_int8(q: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """``q * scale`` in fp32 with the stored fp16 scale (per output row)."""
    return np.asarray(q, dtype=np.float32) * np.asarray(scales, dtype=np.float32)[..., None]


def int4_bytes_per_expert(hidden: int, inter: int) -> int:
    """Nibble bytes of one expert's three projections (tests/test_stress.py:747-796)."""
    return 3 * hidden * inter // 2


def algorithmic_weight_bytes(prec: str, hidden: int, inter: int, group_size: int = 128) -> int:
    """Bytes one touched expert streams from HBM per layer call.

    INT4: nibbles ``3*I*H/2`` + fp16 group scales ``2*(2I*H/gs + H*I/gs)``
    (= 1.546875*I*H at gs=128).  INT8: ``3*I*H`` + fp16 row scales
    ``2*(2I + H)``.  BF16: ``6*I*H``.
    """
    if prec == "INT4":
        return 3 * inter * hidden // 2 + 2 * (2 * inter * (hidden // group_size)
                                               + hidden * (inter // group_size))
    if prec == "INT8":
        return 3 * inter * hidden + 2 * (2 * inter + hidden)
    if prec == "BF16":
        return 6 * inter * hidden
    raise ValueError(prec)
