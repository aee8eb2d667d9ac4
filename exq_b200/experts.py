"""Packed expert weights of one MoE layer (any mix of BF16 / INT8 / INT4) and
its single-call forward.

An ``ExpertBank`` owns one contiguous storage per tier plus a device array
``expert_slot`` (tier << 24 | index inside the tier storage), described to the
library by ``exq_moe_weights`` (include/exq_b200.h), so a layer whose experts
follow a compiled quant plan (``quant_assignments``,
exq/kernels/exq_artifact.py:120-138) runs as one grouped launch per
projection.  Routed experts come first; ``n_shared`` always-on experts (e.g.
DeepSeek-V2's shared experts) follow and receive every token with weight 1.

HBM layout per tier (n = experts in the tier; "permuted" = inside each octet
of k the order [0,4,1,5,2,6,3,7], the order the tcgen05 kernel consumes):
  INT4: w13 u8 [n, 2I, H/2], w2 u8 [n, H, I/2]  (reference nibble format)
        w13_scales f16 [n, H/128, 2I], w2_scales f16 [n, I/128, H]  (group-major)
  INT8: w13 i8 [n, 2I, H], w2 i8 [n, H, I] (permuted); scales f16 [n, 2I], [n, H]
  BF16: w13 f16 [n, 2I, H], w2 f16 [n, H, I] (permuted); 16-bit weights are held
        as fp16, the operand type of the kernel's matrix products
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import torch

from . import _lib as L

TIER_NAMES = {"BF16": L.TIER_BF16, "INT8": L.TIER_INT8, "INT4": L.TIER_INT4}
GROUP = 128
OCTET_PERM = (0, 4, 1, 5, 2, 6, 3, 7)
OCTET_INV = (0, 2, 4, 6, 1, 3, 5, 7)


class MoeWeightsC(C.Structure):
    """ctypes mirror of ``exq_moe_weights``."""
    _fields_ = [("n_routed", C.c_int32), ("n_shared", C.c_int32), ("hidden", C.c_int64),
                ("inter", C.c_int64), ("n_tier", C.c_int32 * 3), ("reserved", C.c_int32),
                ("w13", C.c_void_p * 3), ("w13_scales", C.c_void_p * 3), ("w2", C.c_void_p * 3),
                ("w2_scales", C.c_void_p * 3), ("expert_slot", C.c_void_p)]


def octet_permute(t: torch.Tensor) -> torch.Tensor:
    """Reorder every 8-element group of the last dimension to [0,4,1,5,2,6,3,7]."""
    k = t.shape[-1]
    idx = torch.tensor(OCTET_PERM, device=t.device)
    return t.reshape(*t.shape[:-1], k // 8, 8).index_select(-1, idx).reshape(t.shape).contiguous()


def octet_unpermute(t: torch.Tensor) -> torch.Tensor:
    k = t.shape[-1]
    idx = torch.tensor(OCTET_INV, device=t.device)
    return t.reshape(*t.shape[:-1], k // 8, 8).index_select(-1, idx).reshape(t.shape).contiguous()


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
    """GPU INT8 tier: per-row symmetric, fp16 scale (natural k order)."""
    dev = L.require_cuda(w)
    w = w.contiguous()
    k = w.shape[-1]
    rows = w.numel() // k
    q = torch.empty(w.shape, dtype=torch.int8, device=dev)
    scales = torch.empty(w.shape[:-1], dtype=torch.float16, device=dev)
    L.check(L.lib().exq_quant_int8(L.ptr(w), L.tag(w), rows, k, L.ptr(q), L.ptr(scales),
                                   L.stream_of(dev)), "quant_int8")
    return q, scales


def _int4_storage(packed13, scales13, packed2, scales2):
    return (packed13.contiguous(), scales13.transpose(-1, -2).contiguous(), packed2.contiguous(),
            scales2.transpose(-1, -2).contiguous())


@dataclass
class ExpertBank:
    """Packed experts of one layer in the tcgen05 storage format."""

    hidden: int
    inter: int
    act_dtype: torch.dtype
    n_routed: int
    n_shared: int
    tiers: list  # per expert (routed then shared): "BF16" / "INT8" / "INT4"
    storage: dict = field(default_factory=dict)  # tier -> (w13, s13, w2, s2)
    index: dict = field(default_factory=dict)    # tier -> expert ids in storage order
    expert_slot: torch.Tensor | None = None
    cstruct: MoeWeightsC | None = None
    _ws: torch.Tensor | None = None

    @property
    def n_total(self) -> int:
        return self.n_routed + self.n_shared

    @property
    def device(self) -> torch.device:
        return self.expert_slot.device

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
        if any(t not in TIER_NAMES for t in tiers):
            raise ValueError(f"unknown tier in {sorted(set(tiers))}")
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
                bank.storage[name] = _int4_storage(*pack_int4(a), *pack_int4(b))
            elif name == "INT8":
                qa, sa = quant_int8(a)
                qb, sb = quant_int8(b)
                bank.storage[name] = (octet_permute(qa), sa, octet_permute(qb), sb)
            else:
                bank.storage[name] = (octet_permute(a.to(torch.float16)), None,
                                      octet_permute(b.to(torch.float16)), None)
            bank.index[name] = sel
            del a, b
        bank._finalize(w13.device)
        return bank

    @classmethod
    def from_int4_packed(cls, w13_packed, w13_scales, w2_packed, w2_scales,
                         act_dtype: torch.dtype = torch.float16):
        """Wrap reference-format INT4 tensors (packed u8 + [E, N, K/128] scales).

        The packed weights are used in place; only the (1/32-size) scales are
        copied into the group-major order the kernel reads.
        """
        L.require_cuda(w13_packed, w13_scales, w2_packed, w2_scales)
        e, i2, h2 = w13_packed.shape
        h = h2 * 2
        inter = i2 // 2
        for t, shape in ((w13_packed, (e, i2, h // 2)), (w13_scales, (e, i2, h // GROUP)),
                         (w2_packed, (e, h, inter // 2)), (w2_scales, (e, h, inter // GROUP))):
            if tuple(t.shape) != shape:
                raise NotImplementedError(
                    f"expected {shape} for group size {GROUP}, got {tuple(t.shape)}")
        bank = cls(hidden=h, inter=inter, act_dtype=act_dtype, n_routed=e, n_shared=0,
                   tiers=["INT4"] * e)
        bank.storage["INT4"] = _int4_storage(w13_packed, w13_scales, w2_packed, w2_scales)
        bank.index["INT4"] = list(range(e))
        bank._finalize(w13_packed.device)
        return bank

    def _finalize(self, device):
        slot = [-1] * self.n_total
        for name, sel in self.index.items():
            for j, e in enumerate(sel):
                slot[e] = (TIER_NAMES[name] << 24) | j
        self.expert_slot = torch.tensor(slot, dtype=torch.int32, device=device)
        cs = MoeWeightsC()
        cs.n_routed, cs.n_shared = self.n_routed, self.n_shared
        cs.hidden, cs.inter = self.hidden, self.inter
        for name, code in TIER_NAMES.items():
            st = self.storage.get(name)
            cs.n_tier[code] = len(self.index.get(name, []))
            if st is None:
                continue
            w13, s13, w2, s2 = st
            cs.w13[code], cs.w2[code] = w13.data_ptr(), w2.data_ptr()
            cs.w13_scales[code] = s13.data_ptr() if s13 is not None else None
            cs.w2_scales[code] = s2.data_ptr() if s2 is not None else None
        cs.expert_slot = self.expert_slot.data_ptr()
        self.cstruct = cs

    @classmethod
    def merged(cls, first: "ExpertBank", second: "ExpertBank") -> "ExpertBank":
        """One bank whose routed experts are ``first``'s, then ``second``'s
        (ids offset by ``first.n_routed``); neither may hold shared experts.
        A tier only one of them holds is shared, not copied; a tier both hold
        is concatenated."""
        if first.n_shared or second.n_shared:
            raise ValueError("merged banks hold routed experts only")
        if (first.hidden, first.inter, first.act_dtype) != (second.hidden, second.inter,
                                                            second.act_dtype):
            raise ValueError("merged banks need the same hidden, inter and activation dtype")
        bank = cls(hidden=first.hidden, inter=first.inter, act_dtype=first.act_dtype,
                   n_routed=first.n_routed + second.n_routed, n_shared=0,
                   tiers=list(first.tiers) + list(second.tiers))
        for name in TIER_NAMES:
            a, b = first.storage.get(name), second.storage.get(name)
            ia = list(first.index.get(name, []))
            ib = [e + first.n_routed for e in second.index.get(name, [])]
            if a is None and b is None:
                continue
            if a is None or b is None:
                bank.storage[name] = a if b is None else b
            else:
                bank.storage[name] = tuple(None if x is None else torch.cat([x, y], 0)
                                           for x, y in zip(a, b))
            bank.index[name] = ia + ib
        bank._finalize(first.device)
        return bank

    # ------------------------------------------------------------ on-disk cache
    _CACHE_VERSION = 1

    def save(self, path) -> None:
        """Write the packed tiers (the HBM storage format, byte for byte) and
        the expert map to ``path`` (``torch.save``), so a later process loads
        them without re-packing (the reference re-packs every layer on its
        first call, exq/runtime/sglang_backend.py:32-60)."""
        storage = {name: tuple(None if t is None else t.detach().to("cpu") for t in st)
                   for name, st in self.storage.items() if st is not None}
        torch.save({"version": self._CACHE_VERSION, "hidden": self.hidden, "inter": self.inter,
                    "act_dtype": str(self.act_dtype).replace("torch.", ""),
                    "n_routed": self.n_routed, "n_shared": self.n_shared,
                    "tiers": list(self.tiers), "index": {k: list(v) for k, v in self.index.items()},
                    "storage": storage}, path)

    @classmethod
    def load(cls, path, device="cuda") -> "ExpertBank":
        """A bank written by ``save``, on ``device``."""
        d = torch.load(path, map_location="cpu", weights_only=True)
        if d.get("version") != cls._CACHE_VERSION:
            raise ValueError(f"{path}: not an expert-bank cache of version {cls._CACHE_VERSION}")
        bank = cls(hidden=d["hidden"], inter=d["inter"], act_dtype=getattr(torch, d["act_dtype"]),
                   n_routed=d["n_routed"], n_shared=d["n_shared"], tiers=list(d["tiers"]))
        dev = torch.device(device)
        bank.storage = {name: tuple(None if t is None else t.to(dev) for t in st)
                        for name, st in d["storage"].items()}
        bank.index = {k: list(v) for k, v in d["index"].items()}
        bank._finalize(dev)
        return bank

    # ------------------------------------------------------------ inspection
    def expert_reference_format(self, e: int):
        """Expert ``e`` in the reference's layouts: INT4 -> (packed, scales [N, K/128])
        per projection, INT8 -> (q natural order, row scales), BF16 -> fp16 tensors."""
        tier = self.tiers[e]
        j = self.index[tier].index(e)
        w13, s13, w2, s2 = self.storage[tier]
        if tier == "INT4":
            return tier, (w13[j], s13[j].transpose(0, 1)), (w2[j], s2[j].transpose(0, 1))
        if tier == "INT8":
            return tier, (octet_unpermute(w13[j]), s13[j]), (octet_unpermute(w2[j]), s2[j])
        return tier, octet_unpermute(w13[j]), octet_unpermute(w2[j])

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

    def _args(self, hidden_states, topk_ids, topk_weights, out, workspace):
        dev = L.require_cuda(hidden_states, topk_ids, topk_weights)
        if hidden_states.dtype not in (torch.float16, torch.bfloat16):
            raise ValueError("hidden_states must be fp16 or bf16")
        x = hidden_states.contiguous()
        t = x.shape[0]
        if x.dim() != 2 or x.shape[1] != self.hidden:
            raise ValueError("hidden_states must be [T, hidden]")
        ids = topk_ids.contiguous()
        w = topk_weights.contiguous()
        if ids.dim() != 2 or ids.shape != w.shape or ids.shape[0] != t:
            raise ValueError("topk_ids / topk_weights must both be [T, k]")
        k = ids.shape[1]
        if out is None:
            out = torch.empty(t, self.hidden, dtype=x.dtype, device=dev)
        if workspace is None:
            self.reserve(t, k)
            workspace = self._ws
        return dev, x, ids, w, k, out, workspace

    def forward(self, hidden_states: torch.Tensor, topk_ids: torch.Tensor,
                topk_weights: torch.Tensor, out: torch.Tensor | None = None,
                workspace: torch.Tensor | None = None) -> torch.Tensor:
        """The five stages route -> prep -> gate_up -> down -> weighted combine.

        Up to 16384 (token, expert) slots the route and prep stages are one
        fused launch, and gate_up, down and the combine are one GEMM launch
        that builds its tile list from the ids: two launches per call.  Above
        that, routing and the activation prep are separate launches (three)."""
        return self.forward_range(hidden_states, topk_ids, topk_weights, 0, 5, out, workspace)

    def forward_from_logits(self, hidden_states: torch.Tensor, router_logits: torch.Tensor,
                            top_k: int, renormalize: bool = True,
                            out: torch.Tensor | None = None) -> torch.Tensor:
        """The layer from router logits [T, n_routed] (fp32/fp16/bf16): the
        fused router top-k (softmax, top_k, optional renormalisation, as
        ``kernels.router_topk``) feeding the routing stage in one C call,
        ``exq_moe_layer_forward_from_logits``.  Up to 16384 slots that is three
        launches, the routing kernel chained programmatically after the
        router."""
        dev = L.require_cuda(hidden_states, router_logits)
        if hidden_states.dtype not in (torch.float16, torch.bfloat16):
            raise ValueError("hidden_states must be fp16 or bf16")
        x = hidden_states.contiguous()
        lg = router_logits.contiguous()
        t = x.shape[0]
        if x.dim() != 2 or x.shape[1] != self.hidden:
            raise ValueError("hidden_states must be [T, hidden]")
        if lg.dim() != 2 or lg.shape != (t, self.n_routed):
            raise ValueError(f"router_logits must be [T, {self.n_routed}]")
        need = int(L.lib().exq_moe_layer_from_logits_workspace_bytes(
            t, top_k, self.n_shared, self.n_total, self.hidden, self.inter))
        if self._ws is None or self._ws.numel() < need:
            self._ws = L.workspace(dev, need)
        if out is None:
            out = torch.empty(t, self.hidden, dtype=x.dtype, device=dev)
        L.check(L.lib().exq_moe_layer_forward_from_logits(
            C.byref(self.cstruct), L.ptr(x), L.tag(x), t, L.ptr(lg), L.tag(lg), int(top_k),
            int(bool(renormalize)), L.ptr(out), L.ptr(self._ws), self._ws.numel(),
            L.stream_of(dev)), "moe_layer_forward_from_logits")
        return out

    def forward_range(self, hidden_states, topk_ids, topk_weights, first: int, end: int,
                      out=None, workspace=None):
        dev, x, ids, w, k, out, workspace = self._args(hidden_states, topk_ids, topk_weights, out,
                                                      workspace)
        L.check(L.lib().exq_moe_layer_forward_range(
            C.byref(self.cstruct), L.ptr(x), L.tag(x), x.shape[0], L.ptr(ids), L.tag(ids), L.ptr(w),
            L.tag(w), k, L.ptr(out), L.ptr(workspace), workspace.numel(), L.stream_of(dev),
            first, end), "moe_layer_forward")
        return out

    __call__ = forward
