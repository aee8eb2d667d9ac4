"""Packed expert weights of one MoE layer (any mix of BF16 / INT8 / INT4) and
its single-call forward.

An ``ExpertBank`` owns one contiguous tensor set per tier and a device array
of ``exq_expert_desc`` records (include/exq_b200.h) pointing into them, so a
layer whose experts follow a compiled quant plan (``quant_assignments``,
exq/kernels/exq_artifact.py:120-138) runs as one grouped launch per
projection.  Routed experts come first; ``n_shared`` always-on experts (e.g.
DeepSeek-V2's shared experts) follow and receive every token with weight 1.

HBM layout per tier (E_t experts of that tier, in expert order):
  INT4: w13 u8 [E_t, 2I, H/2], w13_scales f16 [E_t, 2I, H/128],
        w2 u8 [E_t, H, I/2],   w2_scales f16 [E_t, H, I/128]
  INT8: w13 i8 [E_t, 2I, H], w13_scales f16 [E_t, 2I], w2 i8 [E_t, H, I], w2_scales f16 [E_t, H]
  BF16: w13 [E_t, 2I, H], w2 [E_t, H, I] in the activation dtype
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib as L

TIER_NAMES = {"BF16": L.TIER_BF16, "INT8": L.TIER_INT8, "INT4": L.TIER_INT4}
GROUP = 128


def _desc_rows(tier: int, n: int, tensors, extra_rows=None):
    """int64 [n, 5] descriptor rows for experts 0..n-1 of one tier tensor set."""
    w13, s13, w2, s2 = tensors
    rows = np.zeros((n, 5), dtype=np.int64)
    rows[:, 0] = tier & 0xFFFFFFFF
    for j, t in enumerate((w13, s13, w2, s2)):
        if t is None:
            continue
        step = t.stride(0) * t.element_size()
        rows[:, 1 + j] = t.data_ptr() + np.arange(n, dtype=np.int64) * step
    return rows


def pack_int4(w: torch.Tensor, group_size: int = GROUP):
    """GPU INT4 packing of the last dimension (bit-exact with pack_int4_weights)."""
    dev = L.require_cuda(w)
    w = w.contiguous()
    k = w.shape[-1]
    if k % 2:
        raise ValueError(f"K={k} must be divisible by 2 for INT4 packing")
    gs = k if k < group_size else group_size
    if k % gs:
        raise ValueError(f"K={k} must be divisible by group_size={gs}. "
                         "Choose a group_size that divides K, or use group_size=K for a single group.")
    rows = w.numel() // k
    packed = torch.empty(*w.shape[:-1], k // 2, dtype=torch.uint8, device=dev)
    scales = torch.empty(*w.shape[:-1], k // gs, dtype=torch.float16, device=dev)
    L.check(L.lib().exq_pack_int4(L.ptr(w), L.tag(w), rows, k, int(group_size), L.ptr(packed),
                                  L.ptr(scales), L.stream_of(dev)), "pack_int4")
    return packed, scales


def quant_int8(w: torch.Tensor):
    """GPU INT8 tier: per-row symmetric, fp16 scale."""
    dev = L.require_cuda(w)
    w = w.contiguous()
    k = w.shape[-1]
    rows = w.numel() // k
    q = torch.empty(w.shape, dtype=torch.int8, device=dev)
    scales = torch.empty(w.shape[:-1], dtype=torch.float16, device=dev)
    L.check(L.lib().exq_quant_int8(L.ptr(w), L.tag(w), rows, k, L.ptr(q), L.ptr(scales),
                                   L.stream_of(dev)), "quant_int8")
    return q, scales


@dataclass
class ExpertBank:
    """Packed experts of one layer plus their device descriptor array."""

    hidden: int
    inter: int
    act_dtype: torch.dtype
    n_routed: int
    n_shared: int
    tiers: list  # per expert (routed then shared): "BF16" / "INT8" / "INT4"
    storage: dict = field(default_factory=dict)  # tier -> (w13, s13, w2, s2)
    desc: torch.Tensor | None = None  # int64 [E_total, 5] on device
    _ws: torch.Tensor | None = None

    @property
    def n_total(self) -> int:
        return self.n_routed + self.n_shared

    @property
    def device(self) -> torch.device:
        return self.desc.device

    # ------------------------------------------------------------ builders
    @classmethod
    def from_dense(cls, w13: torch.Tensor, w2: torch.Tensor, tiers=None,
                   act_dtype: torch.dtype = torch.float16, shared_w13: torch.Tensor | None = None,
                   shared_w2: torch.Tensor | None = None, shared_tier: str = "BF16"):
        """Quantise dense expert weights per tier on the GPU.

        ``w13`` [E, 2I, H], ``w2`` [E, H, I]; ``tiers`` a list of E tier names
        (default all INT4).  Optional shared experts ``shared_w13`` [S, 2I, H],
        ``shared_w2`` [S, H, I] in ``shared_tier``.
        """
        L.require_cuda(w13, w2, shared_w13, shared_w2)
        e, i2, h = w13.shape
        inter = i2 // 2
        if w2.shape != (e, h, inter):
            raise ValueError("w2 must be [E, H, I] matching w13 [E, 2I, H]")
        tiers = list(tiers) if tiers is not None else ["INT4"] * e
        if len(tiers) != e:
            raise ValueError("one tier per routed expert")
        all_w13, all_w2 = w13, w2
        n_shared = 0
        if shared_w13 is not None:
            n_shared = shared_w13.shape[0]
            all_w13 = torch.cat([w13, shared_w13.to(w13.dtype)], 0)
            all_w2 = torch.cat([w2, shared_w2.to(w2.dtype)], 0)
            tiers = tiers + [shared_tier] * n_shared
        bank = cls(hidden=h, inter=inter, act_dtype=act_dtype, n_routed=e, n_shared=n_shared,
                   tiers=tiers)
        for name in ("INT4", "INT8", "BF16"):
            sel = [i for i, t in enumerate(tiers) if t == name]
            if not sel:
                continue
            idx = torch.tensor(sel, device=w13.device)
            a, b = all_w13.index_select(0, idx), all_w2.index_select(0, idx)
            if name == "INT4":
                bank.storage[name] = (*pack_int4(a), *pack_int4(b))
            elif name == "INT8":
                bank.storage[name] = (*quant_int8(a), *quant_int8(b))
            else:
                bank.storage[name] = (a.to(act_dtype).contiguous(), None,
                                      b.to(act_dtype).contiguous(), None)
            bank.storage[name + "_index"] = sel
        bank._build_desc(w13.device)
        return bank

    @classmethod
    def from_int4_packed(cls, w13_packed, w13_scales, w2_packed, w2_scales,
                         act_dtype: torch.dtype = torch.float16):
        """Wrap already-packed INT4 tensors (reference format) without copying."""
        L.require_cuda(w13_packed, w13_scales, w2_packed, w2_scales)
        e, i2, h2 = w13_packed.shape
        h = h2 * 2
        inter = i2 // 2
        for t, shape in ((w13_packed, (e, i2, h // 2)), (w13_scales, (e, i2, h // GROUP)),
                         (w2_packed, (e, h, inter // 2)), (w2_scales, (e, h, inter // GROUP))):
            if tuple(t.shape) != shape:
                raise NotImplementedError(
                    f"expected {shape} for group size {GROUP}, got {tuple(t.shape)}")
            if not t.is_contiguous():
                raise ValueError("packed weights must be contiguous")
        bank = cls(hidden=h, inter=inter, act_dtype=act_dtype, n_routed=e, n_shared=0,
                   tiers=["INT4"] * e)
        bank.storage["INT4"] = (w13_packed, w13_scales, w2_packed, w2_scales)
        bank.storage["INT4_index"] = list(range(e))
        bank._build_desc(w13_packed.device)
        return bank

    def _build_desc(self, device):
        rows = np.zeros((self.n_total, 5), dtype=np.int64)
        rows[:, 0] = L.TIER_NONE & 0xFFFFFFFF
        for name, code in TIER_NAMES.items():
            if name not in self.storage:
                continue
            sel = self.storage[name + "_index"]
            rows[sel] = _desc_rows(code, len(sel), self.storage[name])
        self.desc = torch.from_numpy(rows).to(device)

    def weight_bytes(self, expert: int) -> int:
        """HBM bytes one call streams for this expert when it is touched."""
        h, i = self.hidden, self.inter
        t = self.tiers[expert]
        if t == "INT4":
            return 3 * i * h // 2 + 2 * (2 * i * (h // GROUP) + h * (i // GROUP))
        if t == "INT8":
            return 3 * i * h + 2 * (2 * i + h)
        return 6 * i * h

    # ------------------------------------------------------------ forward
    def workspace_bytes(self, n_tokens: int, top_k: int) -> int:
        return int(L.lib().exq_moe_layer_workspace_bytes(n_tokens, top_k, self.n_shared,
                                                          self.n_total, self.hidden, self.inter))

    def reserve(self, n_tokens: int, top_k: int) -> None:
        """Pre-size the cached workspace (call before CUDA-graph capture)."""
        need = self.workspace_bytes(n_tokens, top_k)
        if self._ws is None or self._ws.numel() < need:
            self._ws = L.workspace(self.device, need)

    def forward(self, hidden_states: torch.Tensor, topk_ids: torch.Tensor,
                topk_weights: torch.Tensor, out: torch.Tensor | None = None,
                workspace: torch.Tensor | None = None) -> torch.Tensor:
        """route -> gate_up -> SiLU*mul -> down -> weighted combine, in 4 launches."""
        dev = L.require_cuda(hidden_states, topk_ids, topk_weights)
        if hidden_states.dtype != self.act_dtype:
            raise ValueError(f"hidden_states must be {self.act_dtype}")
        x = hidden_states.contiguous()
        t = x.shape[0]
        if x.shape[1] != self.hidden:
            raise ValueError("hidden size mismatch")
        ids = topk_ids.contiguous()
        w = topk_weights.contiguous()
        if ids.dim() != 2 or ids.shape != w.shape or ids.shape[0] != t:
            raise ValueError("topk_ids / topk_weights must both be [T, k]")
        k = ids.shape[1]
        if out is None:
            out = torch.empty(t, self.hidden, dtype=self.act_dtype, device=dev)
        if workspace is None:
            self.reserve(t, k)
            workspace = self._ws
        L.check(L.lib().exq_moe_layer_forward(
            L.ptr(self.desc), self.n_routed, self.n_shared, self.hidden, self.inter, L.ptr(x),
            L.tag(x), t, L.ptr(ids), L.tag(ids), L.ptr(w), L.tag(w), k, L.ptr(out),
            L.ptr(workspace), workspace.numel(), L.stream_of(dev)), "moe_layer_forward")
        return out

    __call__ = forward
