"""Two-tier expert store: hot experts in HBM, cold INT4 experts in host memory.

The reference's ``ExpertWeightCache`` (exq/runtime/__init__.py:35-106) keeps the
experts its compiled plan marks BF16 or INT8 on the GPU and the INT4 ones in
CPU memory, prefetching those by async copy on a side stream when the router
selects them (``prefetch``, ``sync_prefetches``, hit / miss statistics).

``OffloadedExpertBank`` does the same for an ``ExpertBank``:

* BF16 / INT8 experts and the shared experts stay in HBM (the bank's own
  storage);
* every INT4 expert's packed weights and scales live in pinned host memory,
  and an HBM pool of ``gpu_slots`` INT4 entries holds the ones in use;
* ``prefetch(experts)`` copies missing experts into free or least recently
  used pool entries on a copy stream (one ``cudaMemcpyAsync`` per tensor), the
  copies ordered after every kernel already queued on the compute stream (an
  evicted entry may still be read by one);
* ``forward`` makes the call's routed experts resident, points their
  ``expert_slot`` entries (tier << 24 | pool entry) at the pool, waits for the
  copies on the compute stream and runs the unchanged layer launch.

A pool large enough for every INT4 expert behaves as the resident bank; the
outputs are bit-identical to it (the same kernels read the same bytes).
"""
from __future__ import annotations

from collections import OrderedDict

import torch

from . import _lib as L
from .experts import ExpertBank, MoeWeightsC, TIER_NAMES


class SlotPool:
    """Least-recently-used assignment of experts to ``n_slots`` pool entries.

    ``assign(needed)`` returns ``(placement, loads)``: the entry of every
    needed expert, and the (expert, entry) pairs that must be copied in; the
    experts it evicted are in ``evicted``.
    Experts needed by the same call are never evicted for one another; more
    needed experts than entries raise ``ValueError``."""

    def __init__(self, n_slots: int):
        if n_slots < 1:
            raise ValueError("the pool needs at least one entry")
        self.n_slots = n_slots
        self.where: OrderedDict[int, int] = OrderedDict()   # expert -> entry, LRU first
        self.free = list(range(n_slots - 1, -1, -1))
        self.hits = 0
        self.misses = 0

    def assign(self, needed):
        needed = list(dict.fromkeys(int(e) for e in needed))
        if len(needed) > self.n_slots:
            raise ValueError(f"{len(needed)} experts needed at once, the pool holds "
                             f"{self.n_slots}")
        keep = set(needed)
        placement, loads = {}, []
        self.evicted = []
        for e in needed:
            if e in self.where:
                self.where.move_to_end(e)
                placement[e] = self.where[e]
                self.hits += 1
        for e in needed:
            if e in placement:
                continue
            self.misses += 1
            if self.free:
                slot = self.free.pop()
            else:
                victim = next(v for v in self.where if v not in keep)
                slot = self.where.pop(victim)
                self.evicted.append(victim)
            self.where[e] = slot
            placement[e] = slot
            loads.append((e, slot))
        return placement, loads

    def resident(self, e: int) -> bool:
        return e in self.where

    @property
    def stats(self) -> dict:
        n = self.hits + self.misses
        return {"gpu_slots": self.n_slots, "resident": len(self.where), "hits": self.hits,
                "misses": self.misses, "hit_rate": self.hits / n if n else 0.0}


class OffloadedExpertBank:
    """An ``ExpertBank`` whose INT4 experts live in pinned host memory, with
    an HBM pool of ``gpu_slots`` INT4 entries (see the module docstring).

    Built from a resident bank (``src``): its INT4 storage is copied to the
    host and released, and ``src`` itself is not usable afterwards (its other
    tiers are shared with this object)."""

    def __init__(self, src: ExpertBank, gpu_slots: int, copy_stream=None):
        if "INT4" not in src.storage:
            raise ValueError("the bank has no INT4 experts to offload")
        dev = src.device
        self.src = src
        self.device = dev
        self.int4_experts = list(src.index["INT4"])
        n4 = len(self.int4_experts)
        self.pool = SlotPool(min(gpu_slots, n4))
        w13, s13, w2, s2 = src.storage["INT4"]
        # host store: expert -> (w13, s13, w2, s2), pinned for async copies
        self.host = {}
        for j, e in enumerate(self.int4_experts):
            self.host[e] = tuple(t[j].to("cpu").pin_memory() for t in (w13, s13, w2, s2))
        n = self.pool.n_slots
        self.gpu = tuple(torch.empty((n,) + tuple(t.shape[1:]), dtype=t.dtype, device=dev)
                         for t in (w13, s13, w2, s2))
        # the layer's view: the pool as the INT4 tier, the other tiers as in src
        bank = ExpertBank(hidden=src.hidden, inter=src.inter, act_dtype=src.act_dtype,
                          n_routed=src.n_routed, n_shared=src.n_shared, tiers=list(src.tiers))
        bank.storage = {k: v for k, v in src.storage.items() if k != "INT4"}
        bank.index = {k: list(v) for k, v in src.index.items() if k != "INT4"}
        bank.storage["INT4"] = self.gpu
        bank.index["INT4"] = [-1] * n          # placeholder: entries are mapped per call
        self._slot_host = [-1] * src.n_total
        for name, sel in bank.index.items():
            if name == "INT4":
                continue
            for j, e in enumerate(sel):
                self._slot_host[e] = (TIER_NAMES[name] << 24) | j
        self.bank = bank
        self._build_cstruct()
        src.storage["INT4"] = None             # the HBM copy of the INT4 tier is released
        src.cstruct = None                     # src's layer view pointed at it
        del w13, s13, w2, s2
        self.copy_stream = copy_stream or torch.cuda.Stream(dev)
        self.bytes_copied = 0
        self._dirty = False      # expert_slot on the device differs from _slot_host
        self._pending = False    # copies queued since the compute stream last waited

    def _build_cstruct(self):
        b = self.bank
        b.expert_slot = torch.tensor(self._slot_host, dtype=torch.int32, device=self.device)
        cs = MoeWeightsC()
        cs.n_routed, cs.n_shared = b.n_routed, b.n_shared
        cs.hidden, cs.inter = b.hidden, b.inter
        for name, code in TIER_NAMES.items():
            st = b.storage.get(name)
            cs.n_tier[code] = len(b.index.get(name, []))
            if st is None:
                continue
            w13, s13, w2, s2 = st
            cs.w13[code], cs.w2[code] = w13.data_ptr(), w2.data_ptr()
            cs.w13_scales[code] = s13.data_ptr() if s13 is not None else None
            cs.w2_scales[code] = s2.data_ptr() if s2 is not None else None
        cs.expert_slot = b.expert_slot.data_ptr()
        b.cstruct = cs

    # ------------------------------------------------------------ residency
    def prefetch(self, experts) -> int:
        """Make these INT4 experts resident (ids of other tiers are ignored).
        Copies run on the copy stream after the compute stream's queued work;
        ``forward`` orders its launch after them.  Returns the bytes queued."""
        need = [int(e) for e in experts if int(e) in self.host]
        placement, loads = self.pool.assign(need)
        compute = torch.cuda.current_stream(self.device)
        queued = 0
        if loads:
            self.copy_stream.wait_stream(compute)   # an evicted entry may still be read
            with torch.cuda.stream(self.copy_stream):
                for e, slot in loads:
                    for dst, src in zip(self.gpu, self.host[e]):
                        dst[slot].copy_(src, non_blocking=True)
                        queued += src.numel() * src.element_size()
        for e in self.pool.evicted:
            self._slot_host[e] = -1
        for e, slot in loads:
            self._slot_host[e] = (TIER_NAMES["INT4"] << 24) | slot
        self._dirty = self._dirty or bool(loads)
        self.bytes_copied += queued
        self._pending = self._pending or bool(loads)
        return queued

    def sync_prefetches(self) -> None:
        """Order the compute stream after every copy queued so far."""
        if self._pending:
            torch.cuda.current_stream(self.device).wait_stream(self.copy_stream)
            self._pending = False

    @property
    def stats(self) -> dict:
        s = self.pool.stats
        s["bytes_copied"] = self.bytes_copied
        s["cpu_stored"] = len(self.host)
        return s

    # ------------------------------------------------------------ forward
    def forward(self, hidden_states: torch.Tensor, topk_ids: torch.Tensor,
                topk_weights: torch.Tensor, ids_host: torch.Tensor | None = None,
                out: torch.Tensor | None = None) -> torch.Tensor:
        """The layer on the two-tier store.  ``ids_host``: the routing ids on
        the host, when the caller has them (else ``topk_ids`` is read back,
        one synchronisation)."""
        ids_h = ids_host if ids_host is not None else topk_ids.to("cpu")
        self.prefetch(torch.unique(ids_h.reshape(-1)).tolist())
        if self._dirty:   # ordered on the compute stream after the kernels that read it
            slot = torch.tensor(self._slot_host, dtype=torch.int32).pin_memory()
            self.bank.expert_slot.copy_(slot, non_blocking=True)
            self._dirty = False
        self.sync_prefetches()
        return self.bank.forward(hidden_states, topk_ids, topk_weights, out)

    __call__ = forward
