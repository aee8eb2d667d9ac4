"""Workers for the expert-parallel tests (spawned as separate processes).

The CPU workers run the exchange of exq_b200.ep.ExpertParallelLayer on gloo
ranks with the CPU oracle as the local expert compute and the combine; the
GPU worker runs the real kernels over NCCL and compares with the full layer
on one GPU."""
import faulthandler
import os
import sys
import traceback

import torch
import torch.distributed as dist

from oracle import moe as OM

H, I, E, K = 64, 32, 8, 2


def _init(rank, world, port, backend):
    # a rank that is still running after 50 s prints every thread's stack, so
    # a stuck rank shows where it waits before the group timeout ends the test
    faulthandler.dump_traceback_later(50, exit=False)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group(backend, rank=rank, world_size=world, timeout=timedelta(seconds=60))


def _weights(seed=0):
    g = torch.Generator().manual_seed(seed)
    w13 = [torch.randn(2 * I, H, generator=g) * 0.05 for _ in range(E)]
    w2 = [torch.randn(H, I, generator=g) * 0.05 for _ in range(E)]
    return w13, w2


def _tokens(rank, t, case):
    g = torch.Generator().manual_seed(100 + rank)
    x = torch.randn(t, H, generator=g).to(torch.float16)
    if case == "one_rank":   # every slot to the experts of rank 0
        ids = torch.stack([torch.randperm(E // 2, generator=g)[:K] for _ in range(t)]) if t else \
            torch.zeros(0, K, dtype=torch.int64)
    else:
        ids = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(t)]) if t else \
            torch.zeros(0, K, dtype=torch.int64)
    w = torch.rand(t, K, generator=g)
    return x, ids, w / w.sum(-1, keepdim=True).clamp_min(1e-6)


def cpu_worker(rank, world, port, case, t_per_rank):
    from exq_b200.ep import ExpertParallelLayer
    _init(rank, world, port, "gloo")
    try:
        w13, w2 = _weights()
        t = t_per_rank[rank]
        x, ids, w = _tokens(rank, t, case)

        def local_fn(rows, local_ids):
            lo = rank * (E // world)
            if rows.shape[0] == 0:
                return rows.new_empty(0, H)
            gids = (local_ids.long() + lo).view(-1, 1)
            ones = torch.ones(rows.shape[0], 1)
            return OM.moe_layer(rows, gids, ones, w13, w2).to(rows.dtype)

        def pack_fn(hidden, topk_ids, per_rank, world_):
            # slots grouped by destination rank in ascending slot order
            t_, k_ = topk_ids.shape
            flat = topk_ids.reshape(-1).long()
            dest = flat // per_rank
            order = torch.sort(dest, stable=True).indices
            slot_row = torch.empty_like(order)
            slot_row[order] = torch.arange(order.numel())
            counts = torch.bincount(dest, minlength=world_).to(torch.int32)
            return (hidden[order // k_].contiguous(), (flat[order] % per_rank).to(torch.int32),
                    slot_row.to(torch.int32), counts)

        def combine_fn(back, slot_row, weights, base):
            t_, k_ = weights.shape
            y = torch.zeros(t_, back.shape[1])
            for j in range(k_):
                y += weights[:, j:j + 1].float() * back[slot_row.view(t_, k_)[:, j].long()].float()
            if base is not None:
                y += base.float()
            return y.to(back.dtype)

        layer = ExpertParallelLayer(None, E, local_fn=local_fn, combine_fn=combine_fn,
                                    shared_fn=lambda h: None, pack_fn=pack_fn)
        y = layer(x, ids, w)
        ref = OM.moe_layer(x, ids, w, w13, w2).to(torch.float16)
        assert y.shape == (t, H) and y.dtype == torch.float16
        if t:
            err = OM.rel_l2(y, ref)
            assert err < 1e-3, f"rank {rank}: rel-L2 {err:.2e}"
    finally:
        dist.destroy_process_group()


def _gpu_step_inputs(step, rank, world, t, case, e, h, k, dev):
    from exq_b200.synth import hidden_states, zipf_router
    seed = 10 * step + rank
    if t == 0:
        ids = torch.zeros(0, k, dtype=torch.int64)
        w = torch.zeros(0, k)
    elif case == "one_rank":   # every slot to the experts of rank 0
        g = torch.Generator().manual_seed(seed)
        ids = torch.stack([torch.randperm(e // world, generator=g)[:k] for _ in range(t)])
        w = torch.rand(t, k, generator=g)
    else:
        ids, w = zipf_router(t, e, k, seed=seed)
    x = hidden_states(max(t, 1), h, seed=seed)[:t].to(dev, torch.bfloat16)
    return x, ids.to(dev), w.to(dev)


def gpu_worker(rank, world, port, mode="nccl", max_tokens=64, shared=False):
    """EP on `world` GPUs vs the whole layer on one GPU (Mixtral-like, bf16),
    over four steps: spread routing, a rank with no tokens, every slot to rank
    0's experts, spread again.  mode "peer": the peer-memory exchange (receive
    area of world * max_tokens * top_k rows), also checked bit for bit against
    the NCCL exchange when world > 1.  shared: two always-on BF16 shared
    experts; the peer exchange then folds them into its expert launch, checked
    bit for bit against the same exchange with them run apart."""
    from exq_b200 import ExpertBank
    from exq_b200 import _lib as L
    from exq_b200.ep import ExpertParallelLayer, build_rank_banks
    from exq_b200.synth import expert_weights
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    _init(rank, world, port, "nccl")
    try:
        e, h, inter, k = 8, 512, 256, 2
        w13, w2 = expert_weights(e, inter, h, seed=0, device=dev)
        sw13 = sw2 = None
        if shared:
            sw13, sw2 = expert_weights(2, inter, h, seed=5, device=dev)
        local, sh = build_rank_banks(w13, w2, world, rank, act_dtype=torch.bfloat16,
                                     shared_w13=sw13, shared_w2=sw2)
        full = ExpertBank.from_dense(w13, w2, None, act_dtype=torch.bfloat16, shared_w13=sw13,
                                     shared_w2=sw2)
        apart = None
        if mode == "peer":
            layer = ExpertParallelLayer(local, e, shared_bank=sh, max_tokens=max_tokens, top_k=k)
            assert (layer.fold is not None) == shared
            if shared:
                apart = ExpertParallelLayer(local, e, shared_bank=sh, max_tokens=max_tokens,
                                            top_k=k, fold_shared=False)
            nccl = ExpertParallelLayer(local, e, shared_bank=sh) if world > 1 else None
        else:
            layer, nccl = ExpertParallelLayer(local, e, shared_bank=sh), None
        L.read_device_status(dev, clear=True)
        steps = [(48, "spread"), (0 if rank == 0 else 17, "spread"), (64, "one_rank"),
                 (48, "spread")]
        for step, (t, case) in enumerate(steps):
            x, ids, w = _gpu_step_inputs(step, rank, world, t, case, e, h, k, dev)
            y = layer(x, ids, w)
            assert y.shape == (t, h) and y.dtype == torch.bfloat16
            if nccl is not None:
                y2 = nccl(x, ids, w)
                assert torch.equal(y, y2), f"rank {rank} step {step}: peer != NCCL exchange"
            if apart is not None:
                y3 = apart(x, ids, w)
                assert torch.equal(y, y3), f"rank {rank} step {step}: folded != apart"
            if t:
                ref = full(x, ids, w)
                torch.cuda.synchronize(dev)
                err = OM.rel_l2(y.float().cpu(), ref.float().cpu())
                assert err < 5e-3, f"rank {rank} step {step}: rel-L2 {err:.2e} vs one GPU"
        torch.cuda.synchronize(dev)
        status = L.read_device_status(dev, clear=True)
        assert status == 0, f"rank {rank}: device status {status:#x}"
        if mode == "peer":
            layer.close()
            if apart is not None:
                apart.close()
        dist.barrier()
    except BaseException:
        # print before the process group teardown, which may abort the process
        traceback.print_exc()
        sys.stderr.flush()
        raise
    finally:
        dist.destroy_process_group()


def gpu_graph_worker(rank, world, port):
    """The peer-memory exchange captured in a CUDA graph: each replay with new
    inputs in the captured buffers equals an eager call bit for bit (the step
    counter lives on the device, so replays and eager calls interleave)."""
    from exq_b200 import _lib as L
    from exq_b200.ep import ExpertParallelLayer, build_rank_banks
    from exq_b200.synth import expert_weights
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    _init(rank, world, port, "nccl")
    try:
        e, h, inter, k, t = 8, 512, 256, 2, 40
        w13, w2 = expert_weights(e, inter, h, seed=0, device=dev)
        local, _ = build_rank_banks(w13, w2, world, rank, act_dtype=torch.bfloat16)
        layer = ExpertParallelLayer(local, e, max_tokens=64, top_k=k)
        x0, ids0, w0 = _gpu_step_inputs(0, rank, world, t, "spread", e, h, k, dev)
        xs, idss, ws = x0.clone(), ids0.clone(), w0.clone()
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            layer(xs, idss, ws)
        torch.cuda.current_stream(dev).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            ys = layer(xs, idss, ws)
        for step in range(1, 4):
            x, ids, w = _gpu_step_inputs(step, rank, world, t, "spread", e, h, k, dev)
            xs.copy_(x)
            idss.copy_(ids.to(idss.dtype))
            ws.copy_(w)
            graph.replay()
            ref = layer(x, ids, w)
            torch.cuda.synchronize(dev)
            assert torch.equal(ys, ref), f"rank {rank} replay {step} differs from the eager call"
        status = L.read_device_status(dev, clear=True)
        assert status == 0, f"rank {rank}: device status {status:#x}"
        del graph
        layer.close()
        dist.barrier()
    except BaseException:
        traceback.print_exc()
        sys.stderr.flush()
        raise
    finally:
        dist.destroy_process_group()


def agree_worker(rank, world, port):
    """PeerExchange setup failures are collective: a failure on one rank makes
    every rank raise, so no rank waits for a peer that gave up."""
    from exq_b200.ep import PeerExchange
    _init(rank, world, port, "gloo")
    try:
        px = PeerExchange.__new__(PeerExchange)
        px.group, px.world, px.rank = None, world, rank
        px.device, px._mapped, px.ptr = torch.device("cpu"), [], None
        px._agree(None)
        try:
            px._agree(ValueError("no peer access") if rank == 0 else None)
        except RuntimeError as e:
            assert ("no peer access" in str(e)) == (rank == 0), str(e)
        else:
            raise AssertionError(f"rank {rank} went on although rank 0 failed")
    finally:
        dist.destroy_process_group()


def gpu_timeout_worker(rank, world, port):
    """A device-side wait that runs out, on a one-rank peer exchange: a step
    whose expert stage never runs leaves the combine waiting for a return flag
    that nothing raises.  With a 2 ms limit the combine returns, the device
    status carries EXQ_DEV_TIMEOUT, the layer's status check raises, a step
    before the collective reset times out again (the buffer is marked failed),
    and after reset() a correct step matches the whole layer on one GPU."""
    from exq_b200 import ExpertBank
    from exq_b200 import _lib as L
    from exq_b200.ep import ExpertParallelLayer, build_rank_banks
    from exq_b200.synth import expert_weights
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    _init(rank, world, port, "nccl")
    try:
        e, h, inter, k, t = 8, 512, 256, 2, 24
        w13, w2 = expert_weights(e, inter, h, seed=0, device=dev)
        local, _ = build_rank_banks(w13, w2, world, rank, act_dtype=torch.bfloat16)
        full = ExpertBank.from_dense(w13, w2, None, act_dtype=torch.bfloat16)
        layer = ExpertParallelLayer(local, e, max_tokens=64, top_k=k)
        x, ids, w = _gpu_step_inputs(0, rank, world, t, "spread", e, h, k, dev)
        L.read_device_status(dev, clear=True)
        y = layer(x, ids, w, check=True)
        assert OM.rel_l2(y.float().cpu(), full(x, ids, w).float().cpu()) < 5e-3

        L.set_ep_wait_timeout(2_000_000)
        try:
            px, lib, s = layer.peer, L.lib(), L.stream_of(dev)
            ids32 = ids.to(torch.int32).contiguous()
            slot_row = torch.empty(t * k, dtype=torch.int32, device=dev)
            L.check(lib.exq_ep_dispatch(L.ptr(ids32), L.tag(ids32), t, k, e // world, world, rank,
                                        L.ptr(x), L.tag(x), h, px.capacity, L.ptr(px.peers),
                                        L.ptr(slot_row), s), "ep_dispatch")
            # no exq_ep_expert_forward: this step's return flag is never raised
            out = torch.full((t, h), 7.0, dtype=x.dtype, device=dev)
            wc = w.contiguous()
            L.check(lib.exq_ep_combine_peer(px.ptr, world, px.capacity, h, L.tag(x),
                                            L.ptr(slot_row), L.ptr(wc), L.tag(wc), t, k, None,
                                            L.ptr(out), s), "ep_combine_peer")
            torch.cuda.synchronize(dev)          # the kernel returned
            assert bool((out == 7.0).all()), "a timed-out combine must not write its output"
            try:
                layer.check_status()
            except RuntimeError as err:
                assert "ran out" in str(err), str(err)
            else:
                raise AssertionError("the timed-out wait was not reported")
            # out of step until reset: the next step's return is withheld
            layer(x, ids, w)
            torch.cuda.synchronize(dev)
            assert L.read_device_status(dev, clear=True) & L.DEV_TIMEOUT
        finally:
            L.set_ep_wait_timeout(0)
        layer.reset()
        x2, ids2, w2_ = _gpu_step_inputs(1, rank, world, t, "spread", e, h, k, dev)
        y2 = layer(x2, ids2, w2_, check=True)
        assert OM.rel_l2(y2.float().cpu(), full(x2, ids2, w2_).float().cpu()) < 5e-3
        layer.close()
        dist.barrier()
    except BaseException:
        traceback.print_exc()
        sys.stderr.flush()
        raise
    finally:
        dist.destroy_process_group()
