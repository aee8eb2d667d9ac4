"""Expert parallelism for the MoE expert layer (one process per GPU).

The reference has no expert-parallel path of its own: its layer runs whole on
one GPU (exq/runtime/sglang_backend.py:65-158).  This module shards the
routed experts of one layer across the ranks of a process group; rank r owns
routed experts [r*E/P, (r+1)*E/P).  Two exchanges move tokens to their experts.

Peer memory (``max_tokens`` given, GPUs of one node): every rank allocates one
buffer and maps the other ranks' buffers through CUDA IPC (``PeerExchange``).
A step is four kernels' worth of work on the caller's stream, with no NCCL and
no host synchronisation (so it can be captured in a CUDA graph):
1. ``exq_ep_dispatch`` groups this rank's (token, expert) slots by destination
   and stores each hidden row and local expert id straight into the
   destination's receive block over NVLink, then raises an arrival flag there;
2. ``exq_ep_expert_forward_shared`` puts the rank's own tokens into its own
   receive block (one row per token and shared expert), waits for every
   arrival flag, runs one layer launch over the received rows (local experts)
   and the own block (the shared experts, replicated on every rank), stores
   each received row's output back into its source's return block, raising a
   return flag there, and sums the shared experts' rows per token.  Without
   shared experts (or with ``fold_shared=False``) the shared experts run as a
   call of their own after the dispatch and ``exq_ep_expert_forward`` serves
   the received rows only;
3. ``exq_ep_combine_peer`` waits for every return flag, applies the router
   weights and sums each token's slots plus the shared output.
Each destination reserves ``max_tokens * top_k`` rows per source, so no
count exchange is needed; a call with more tokens is refused on the host.

NCCL (default): one kernel (``exq_ep_pack``) groups the slots by destination
rank into a send buffer and counts them; an all-to-all of the counts sizes the
exchange (one host synchronisation, during which the shared experts run);
all-to-alls move the rows and local ids, each rank runs its experts on what it
received, the outputs return by the reverse all-to-all, and ``exq_ep_combine``
applies the router weights.  The packing, the local expert compute and the
combine are functions of the layer (``pack_fn``, ``local_fn``, ``combine_fn``);
the multi-process CPU tests substitute the CPU oracle to check this exchange on
``gloo`` ranks.
"""
from __future__ import annotations

import ctypes as C

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
    # at least one row, so that an empty exchange still hands NCCL real buffers
    send_rows = torch.empty(max(t * k, 1), hidden.shape[1], dtype=hidden.dtype, device=dev)
    send_ids = torch.empty(max(t * k, 1), dtype=torch.int32, device=dev)
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


class PeerExchange:
    """This rank's expert-parallel buffer, mapped into every rank of the group.

    Collective: every rank of ``group`` constructs it with the same sizes.  The
    buffer holds ``world * capacity`` receive and return rows (``capacity``
    rows reserved per source rank) plus the arrival flags; ``peers`` is the
    device array of all ranks' buffer addresses as mapped in this process.
    ``close`` (also collective) unmaps and frees it."""

    def __init__(self, group, capacity: int, hidden: int, device: torch.device):
        lib = L.lib()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.capacity, self.hidden, self.device = capacity, hidden, device
        nbytes = int(lib.exq_ep_buffer_bytes(self.world, capacity, hidden))
        if nbytes == 0:
            raise ValueError(f"bad expert-parallel buffer sizes: {self.world} ranks, capacity "
                             f"{capacity}, hidden {hidden}")
        self.nbytes = nbytes
        self.ptr, self._mapped = None, []
        with torch.cuda.device(device):
            handle = (C.c_uint8 * 64)()
            err = None
            try:
                own = C.c_void_p()
                L.check(lib.exq_ep_ipc_alloc(nbytes, C.byref(own), handle), "ep_ipc_alloc")
                self.ptr = own.value
                L.check(lib.exq_ep_buffer_init(self.ptr, self.world, capacity, hidden,
                                               L.stream_of(device)), "ep_buffer_init")
                # every rank's buffer is initialised before its handle is
                # published, so no rank writes into a buffer still being cleared
                torch.cuda.synchronize(device)
            except Exception as e:  # noqa: BLE001 - reported to every rank below
                err = e
            self._agree(err)
            mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=device)
            every = torch.empty(self.world, 64, dtype=torch.uint8, device=device)
            dist.all_gather_into_tensor(every, mine, group=group)
            every = every.cpu()
            addrs = []
            try:
                for r in range(self.world):
                    if r == self.rank:
                        addrs.append(self.ptr)
                        continue
                    p = C.c_void_p()
                    h = (C.c_uint8 * 64)(*every[r].tolist())
                    L.check(lib.exq_ep_ipc_open(h, C.byref(p)), "ep_ipc_open")
                    self._mapped.append(p.value)
                    addrs.append(p.value)
            except Exception as e:  # noqa: BLE001
                err = e
            self._agree(err)
            self.peers = torch.tensor(addrs, dtype=torch.int64, device=device)

    def _agree(self, err) -> None:
        """Collective: every rank raises if any rank failed, so that no rank is
        left waiting for a peer that gave up."""
        ok = torch.tensor([0 if err else 1], dtype=torch.int32, device=self.device)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=self.group)
        if int(ok.item()) == 1:
            return
        lib = L.lib()
        for p in self._mapped:
            lib.exq_ep_ipc_close(p)
        if self.ptr is not None:
            lib.exq_ep_ipc_free(self.ptr)
        self._mapped, self.ptr = [], None
        why = f"{type(err).__name__}: {err}" if err else "failed on another rank"
        raise RuntimeError(f"peer-memory exchange unavailable on rank {self.rank}: {why}")

    def close(self) -> None:
        if self.ptr is None:
            return
        lib = L.lib()
        torch.cuda.synchronize(self.device)
        # no rank may still be writing into a buffer that is about to go
        flag = torch.zeros(1, device=self.device)
        dist.all_reduce(flag, group=self.group)
        torch.cuda.synchronize(self.device)
        with torch.cuda.device(self.device):
            for p in self._mapped:
                L.check(lib.exq_ep_ipc_close(p), "ep_ipc_close")
            L.check(lib.exq_ep_ipc_free(self.ptr), "ep_ipc_free")
        self._mapped, self.ptr = [], None


class ExpertParallelLayer:
    """One MoE layer whose routed experts are sharded over a process group.

    ``local_bank`` holds this rank's routed experts (``n_routed / world`` of
    them, as an :class:`exq_b200.ExpertBank`); ``shared_bank`` optionally holds
    the always-on shared experts (replicated on every rank).  With
    ``max_tokens`` (and ``top_k``) the layer exchanges over peer memory and a
    call takes at most ``max_tokens`` tokens of at most ``top_k`` experts;
    constructing it is then collective.  Without, it exchanges over NCCL.
    """

    def __init__(self, local_bank, n_routed: int, group=None, shared_bank=None,
                 local_fn=None, combine_fn=None, shared_fn=None, pack_fn=None,
                 max_tokens: int | None = None, top_k: int | None = None,
                 fold_shared: bool = True):
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
        self.peer = None
        self._ws = None
        self.fold = None
        if max_tokens is not None:
            if top_k is None or top_k <= 0 or max_tokens <= 0 or local_bank is None:
                raise ValueError("the peer exchange needs max_tokens > 0, top_k > 0 and a bank")
            if local_bank.n_shared:
                raise ValueError("the peer exchange's local bank holds routed experts only; "
                                 "pass the shared experts as shared_bank")
            self.peer = PeerExchange(group, max_tokens * top_k, local_bank.hidden,
                                     local_bank.device)
            # shared experts folded into the expert launch: one bank with the
            # local experts, then the shared ones, over the received rows and
            # this rank's own block (one row per token and shared expert)
            self.fold = None
            if (fold_shared and shared_bank is not None and shared_fn is None
                    and shared_bank.n_shared == 0 and shared_bank.n_routed <= top_k):
                from .experts import ExpertBank
                self.fold = ExpertBank.merged(local_bank, shared_bank)
            bank = self.fold or local_bank
            rows = (self.world + (1 if self.fold is not None else 0)) * self.peer.capacity
            # the layer's own workspace, sized once: a captured step keeps
            # pointing at it whatever else the bank is called on
            self._ws = L.workspace(local_bank.device, bank.workspace_bytes(rows, 1))

    def close(self) -> None:
        """Release the peer buffers (collective)."""
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def check_status(self) -> None:
        """Synchronise and raise if a kernel of this rank flagged an error since
        the last check; a wait on another rank that ran out (EXQ_DEV_TIMEOUT)
        means the peer exchange is out of step until ``reset`` (collective)."""
        st = L.read_device_status(self.local_bank.device if self.local_bank is not None
                                  else None, clear=True)
        if st & L.DEV_TIMEOUT:
            raise RuntimeError(f"rank {self.rank}: an expert-parallel wait on another rank ran "
                               f"out (device status {st:#x}); call reset() on every rank")
        if st:
            raise RuntimeError(f"rank {self.rank}: device status {st:#x}")

    def reset(self) -> None:
        """Re-initialise this rank's peer buffer after a timed-out step
        (collective: every rank calls it, and no rank's step is in flight)."""
        if self.peer is None:
            return
        px, dev = self.peer, self.peer.device
        torch.cuda.synchronize(dev)
        flag = torch.zeros(1, device=dev)
        dist.all_reduce(flag, group=self.group)   # every rank's kernels have drained
        torch.cuda.synchronize(dev)
        L.check(L.lib().exq_ep_buffer_init(px.ptr, self.world, px.capacity, px.hidden,
                                           L.stream_of(dev)), "ep_buffer_init")
        torch.cuda.synchronize(dev)
        dist.all_reduce(flag, group=self.group)   # every buffer is clear before any dispatch
        torch.cuda.synchronize(dev)

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
            return rows.new_empty(1, rows.shape[1])[:0]
        ones = torch.ones(rows.shape[0], 1, dtype=torch.float32, device=rows.device)
        return self.local_bank(rows, local_ids.view(-1, 1), ones)

    def _shared_rows(self, hidden: torch.Tensor) -> torch.Tensor | None:
        if self.shared_bank is None:
            return None
        s, t = self.shared_bank.n_routed, hidden.shape[0]
        # every token to every shared expert with weight 1: built once per
        # token count (no launches in a step, and stable for graph capture)
        cache = self.__dict__.setdefault("_shared_args", {})
        key = (t, hidden.device)
        if key not in cache:
            ids = torch.arange(s, dtype=torch.int32, device=hidden.device).expand(t, s).contiguous()
            cache[key] = (ids, torch.ones(t, s, dtype=torch.float32, device=hidden.device))
        ids, w = cache[key]
        return self.shared_bank(hidden, ids, w)

    def forward(self, hidden: torch.Tensor, topk_ids: torch.Tensor,
                topk_weights: torch.Tensor, check: bool = False,
                events: list | None = None) -> torch.Tensor:
        """[T, H] output for this rank's T tokens (same dtype as ``hidden``).

        Expert ids out of range are dropped and flagged in the device status,
        as in the single-GPU layer.  Every rank passes the same activation
        dtype: a rank runs its experts on the rows it receives in the dtype of
        its own ``hidden``.  ``check``: synchronise after the step and raise if
        a kernel flagged an error (``check_status``).  ``events``: five CUDA
        events recorded on the current stream around the peer exchange's
        phases (dispatch, shared experts, local expert stages with the wait
        for the arrivals, combine with the wait for the returns)."""
        if topk_ids.shape != topk_weights.shape or topk_ids.shape[0] != hidden.shape[0]:
            raise ValueError("topk_ids / topk_weights must be [T, k] for hidden [T, H]")
        if self.peer is not None:
            y = self._forward_peer(hidden, topk_ids, topk_weights, events)
            if check:
                self.check_status()
            return y
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
        n_recv = sum(rc)
        # buffers of at least one row: an empty exchange still passes NCCL real addresses
        recv_rows = hidden.new_empty(max(n_recv, 1), h)[:n_recv]
        recv_ids = torch.empty(max(n_recv, 1), dtype=torch.int32, device=hidden.device)[:n_recv]
        dist.all_to_all_single(recv_rows, send_rows[:n_send], rc, sc, group=self.group)
        dist.all_to_all_single(recv_ids, send_ids[:n_send], rc, sc, group=self.group)

        out_rows = self.local_fn(recv_rows, recv_ids).contiguous()
        back = hidden.new_empty(max(n_send, 1), h)
        dist.all_to_all_single(back[:n_send], out_rows, sc, rc, group=self.group)
        y = self.combine_fn(back, slot_row, topk_weights, shared)
        if check and y.is_cuda:
            self.check_status()
        return y

    def _forward_peer(self, hidden, topk_ids, topk_weights, events=None):
        px, bank, lib = self.peer, self.local_bank, L.lib()
        t, k = topk_ids.shape
        if t * k > px.capacity:
            raise ValueError(f"{t} tokens x top-{k} exceed the exchange's {px.capacity} rows "
                             "per rank (max_tokens * top_k)")
        dev = L.require_cuda(hidden, topk_ids, topk_weights)
        x, ids, w = hidden.contiguous(), topk_ids.contiguous(), topk_weights.contiguous()
        h = x.shape[1]
        # everything the three launches check, before the dispatch raises this
        # rank's flags on its peers (a later refusal would leave them waiting)
        if x.dtype not in (torch.float16, torch.bfloat16):
            raise ValueError("hidden must be fp16 or bf16")
        if w.dtype not in (torch.float32, torch.float16, torch.bfloat16):
            raise ValueError("topk_weights must be fp32, fp16 or bf16")
        if ids.dtype not in (torch.int32, torch.int64):
            raise ValueError("topk_ids must be int32 or int64")
        if h != px.hidden or h != bank.hidden:
            raise ValueError(f"hidden size {h} differs from the exchange's {px.hidden}")
        s = L.stream_of(dev)
        slot_row = torch.empty(t * k, dtype=torch.int32, device=dev)
        mark = (lambda i: events[i].record()) if events is not None else (lambda i: None)
        mark(0)
        L.check(lib.exq_ep_dispatch(L.ptr(ids), L.tag(ids), t, k, self.per_rank, self.world,
                                    self.rank, L.ptr(x), L.tag(x), h, px.capacity,
                                    L.ptr(px.peers), L.ptr(slot_row), s), "ep_dispatch")
        mark(1)
        ws = self._ws
        if self.fold is not None:
            shared = torch.empty(t, h, dtype=x.dtype, device=dev)
            mark(2)
            L.check(lib.exq_ep_expert_forward_shared(
                C.byref(self.fold.cstruct), L.tag(x), self.world, self.rank, px.capacity, px.ptr,
                L.ptr(px.peers), L.ptr(x), t, self.shared_bank.n_routed, L.ptr(shared),
                L.ptr(ws), ws.numel(), s), "ep_expert_forward_shared")
        else:
            shared = self.shared_fn(x)
            mark(2)
            L.check(lib.exq_ep_expert_forward(C.byref(bank.cstruct), L.tag(x), self.world,
                                              self.rank, px.capacity, px.ptr, L.ptr(px.peers),
                                              L.ptr(ws), ws.numel(), s), "ep_expert_forward")
        mark(3)
        y = torch.empty(t, h, dtype=x.dtype, device=dev)
        L.check(lib.exq_ep_combine_peer(px.ptr, self.world, px.capacity, h, L.tag(x),
                                        L.ptr(slot_row), L.ptr(w), L.tag(w), t, k,
                                        None if shared is None else L.ptr(shared), L.ptr(y), s),
                "ep_combine_peer")
        mark(4)
        return y

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
