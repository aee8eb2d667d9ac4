"""Expert parallelism for the MoE expert layer (one process per GPU, NCCL).

The reference has no expert-parallel path of its own: its layer runs whole on
one GPU (exq/runtime/sglang_backend.py:65-158).  This module shards the
routed experts of one layer across the ranks of a process group and moves
tokens to their experts with one all-to-all each way:

1. one kernel (``exq_ep_pack``) groups the (token, expert) slots of this
   rank's tokens by destination rank, copies their hidden rows into a send
   buffer and counts them; an all-to-all of the counts tells every rank what
   it receives (the step's one host synchronisation, for NCCL's split sizes;
   the shared experts, which every rank holds and runs on its own tokens,
   are computed while the host waits for the counts);
2. the rows and their expert index local to the destination go out in
   all-to-alls;
3. each rank runs its experts on the rows it received with the fused layer
   kernel (every received row is a token with one expert of weight 1);
4. the expert outputs return by the reverse all-to-all, in send order;
5. the owner of each token applies the router weights and sums its slots,
   plus the shared experts' output, in one kernel (``exq_ep_combine``).

Rank r owns routed experts [r*E/P, (r+1)*E/P).  Counts travel to the host
once per call to size the exchange, so a call is not CUDA-graph capturable.

The packing, the local expert compute and the combine are functions of the
layer (``pack_fn``, ``local_fn``, ``combine_fn``).  By default they are this
package's CUDA kernels; the multi-process CPU tests substitute the CPU oracle
to check the exchange logic on ``gloo`` ranks.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib as L


def shard_range(n_routed: int, world: int, rank: int) -> tuple[int, int]:
    """[lo, hi) of the routed experts rank ``rank`` owns."""
    if n_routed % world:
        raise ValueError(f"{n_routed} routed experts do not split evenly over {world} ranks")
    per = n_routed // world
    return rank * per, (rank + 1) * per


def _cuda_pack(hidden: torch.Tensor, topk_ids: torch.Tensor, per_rank: int, world: int):
    """(send_rows [T*k, H], send_ids [T*k] i32, slot_row [T*k] i32, counts [world] i32)
    with the slots grouped by destination rank (``exq_ep_pack``, one launch)."""
    t, k = topk_ids.shape
    dev = hidden.device
    ids = topk_ids.contiguous()
    send_rows = torch.empty(t * k, hidden.shape[1], dtype=hidden.dtype, device=dev)
    send_ids = torch.empty(t * k, dtype=torch.int32, device=dev)
    slot_row = torch.empty(t * k, dtype=torch.int32, device=dev)
    counts = torch.empty(world, dtype=torch.int32, device=dev)
    L.check(L.lib().exq_ep_pack(L.ptr(ids), L.tag(ids), t, k, per_rank, world,
                                L.ptr(hidden), L.tag(hidden), hidden.shape[1], L.ptr(send_rows),
                                L.ptr(send_ids), L.ptr(slot_row), L.ptr(counts),
                                L.stream_of(dev)), "ep_pack")
    return send_rows, send_ids, slot_row, counts


def _cuda_combine(back: torch.Tensor, slot_row: torch.Tensor, weights: torch.Tensor,
                  base: torch.Tensor | None) -> torch.Tensor:
    """y[t] = base[t] + sum_j w[t, j] * back[slot_row[t*k + j]] (``exq_ep_combine``)."""
    t, k = weights.shape
    w = weights.contiguous()
    y = torch.empty(t, back.shape[1], dtype=back.dtype, device=back.device)
    L.check(L.lib().exq_ep_combine(L.ptr(back), L.tag(back), L.ptr(slot_row), L.ptr(w),
                                   L.tag(w), t, k, back.shape[1],
                                   None if base is None else L.ptr(base), L.ptr(y),
                                   L.stream_of(back.device)), "ep_combine")
    return y


class ExpertParallelLayer:
    """One MoE layer whose routed experts are sharded over a process group.

    ``local_bank`` holds this rank's routed experts (``n_routed / world`` of
    them, as an :class:`exq_b200.ExpertBank`); ``shared_bank`` optionally holds
    the always-on shared experts (replicated on every rank).
    """

    def __init__(self, local_bank, n_routed: int, group=None, shared_bank=None,
                 local_fn=None, combine_fn=None, shared_fn=None, pack_fn=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.n_routed = n_routed
        self.lo, self.hi = shard_range(n_routed, self.world, self.rank)
        self.per_rank = self.hi - self.lo
        self.local_bank = local_bank
        self.shared_bank = shared_bank
        if local_bank is not None and getattr(local_bank, "n_routed", self.per_rank) != self.per_rank:
            raise ValueError(f"local bank holds {local_bank.n_routed} experts, rank {self.rank} "
                             f"owns {self.per_rank}")
        self._counts = None
        self.local_fn = local_fn or self._bank_rows
        self.combine_fn = combine_fn or _cuda_combine
        self.shared_fn = shared_fn or self._shared_rows
        self.pack_fn = pack_fn or _cuda_pack

    def _host_counts(self, device) -> torch.Tensor:
        """[2 * world] int64 host buffer for the send / receive counts (pinned
        when the layer runs on a GPU)."""
        if self._counts is None:
            self._counts = torch.empty(2 * self.world, dtype=torch.int64,
                                       pin_memory=device.type == "cuda")
        return self._counts

    # default compute: the fused layer kernel, one expert of weight 1 per row
    def _bank_rows(self, rows: torch.Tensor, local_ids: torch.Tensor) -> torch.Tensor:
        if rows.shape[0] == 0:
            return rows.new_empty(0, rows.shape[1])
        ones = torch.ones(rows.shape[0], 1, dtype=torch.float32, device=rows.device)
        return self.local_bank(rows, local_ids.view(-1, 1), ones)

    def _shared_rows(self, hidden: torch.Tensor) -> torch.Tensor | None:
        if self.shared_bank is None:
            return None
        s = self.shared_bank.n_routed
        ids = torch.arange(s, dtype=torch.int32, device=hidden.device).expand(hidden.shape[0], s)
        w = torch.ones(hidden.shape[0], s, dtype=torch.float32, device=hidden.device)
        return self.shared_bank(hidden, ids.contiguous(), w)

    def forward(self, hidden: torch.Tensor, topk_ids: torch.Tensor,
                topk_weights: torch.Tensor) -> torch.Tensor:
        """[T, H] output for this rank's T tokens (same dtype as ``hidden``).

        Expert ids out of range are dropped and flagged in the device status,
        as in the single-GPU layer."""
        if topk_ids.shape != topk_weights.shape or topk_ids.shape[0] != hidden.shape[0]:
            raise ValueError("topk_ids / topk_weights must be [T, k] for hidden [T, H]")
        t, k = topk_ids.shape
        h = hidden.shape[1]
        send_rows, send_ids, slot_row, send_counts = self.pack_fn(hidden.contiguous(), topk_ids,
                                                                  self.per_rank, self.world)
        send_counts = send_counts.to(torch.int64)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        # the one host sync of a step: the counts travel to pinned memory, and
        # the shared experts (independent of the exchange) run while the host waits
        counts = self._host_counts(hidden.device)
        counts[:self.world].copy_(send_counts, non_blocking=True)
        counts[self.world:].copy_(recv_counts, non_blocking=True)
        ready = torch.cuda.Event() if hidden.is_cuda else None
        if ready is not None:
            ready.record()
        shared = self.shared_fn(hidden)
        if ready is not None:
            ready.synchronize()
        sc, rc = counts[:self.world].tolist(), counts[self.world:].tolist()
        n_send = sum(sc)
        recv_rows = hidden.new_empty(sum(rc), h)
        recv_ids = torch.empty(sum(rc), dtype=torch.int32, device=hidden.device)
        dist.all_to_all_single(recv_rows, send_rows[:n_send], rc, sc, group=self.group)
        dist.all_to_all_single(recv_ids, send_ids[:n_send], rc, sc, group=self.group)

        out_rows = self.local_fn(recv_rows, recv_ids).contiguous()
        back = hidden.new_empty(max(n_send, 1), h)
        dist.all_to_all_single(back[:n_send], out_rows, sc, rc, group=self.group)
        return self.combine_fn(back, slot_row, topk_weights, shared)

    __call__ = forward


def build_rank_banks(w13: torch.Tensor, w2: torch.Tensor, world: int, rank: int, tiers=None,
                     act_dtype: torch.dtype = torch.float16, shared_w13=None, shared_w2=None,
                     shared_tier: str = "BF16"):
    """This rank's ExpertBank (its slice of the routed experts) and, when given,
    the shared-expert bank.  ``w13`` [E, 2I, H] / ``w2`` [E, H, I] on the GPU."""
    from .experts import ExpertBank
    L.require_cuda(w13, w2)
    lo, hi = shard_range(w13.shape[0], world, rank)
    local = ExpertBank.from_dense(w13[lo:hi], w2[lo:hi],
                                  None if tiers is None else list(tiers)[lo:hi],
                                  act_dtype=act_dtype)
    shared = None
    if shared_w13 is not None:
        shared = ExpertBank.from_dense(shared_w13, shared_w2, [shared_tier] * shared_w13.shape[0],
                                       act_dtype=act_dtype)
    return local, shared
