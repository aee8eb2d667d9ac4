"""Expert parallelism: the exchange logic on gloo ranks (CPU), the CUDA path
over NCCL and over peer memory (two GPUs), and the peer-memory path as a
one-rank group (one GPU)."""
import socket

import pytest
import torch
import torch.multiprocessing as mp

import _ep_helpers as EH


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("case,t_per_rank", [("spread", (5, 7)), ("one_rank", (6, 3)),
                                             ("spread", (4, 0))])
def test_ep_exchange_matches_single_process_oracle(case, t_per_rank):
    """Two gloo ranks: routing to both ranks, every slot to rank 0's experts
    (rank 1 receives nothing), and a rank with no tokens."""
    mp.spawn(EH.cpu_worker, args=(2, _free_port(), case, t_per_rank), nprocs=2, join=True)


def test_peer_exchange_setup_failure_is_collective():
    mp.spawn(EH.agree_worker, args=(2, _free_port()), nprocs=2, join=True)


def test_shard_range():
    from exq_b200.ep import shard_range
    assert shard_range(8, 2, 1) == (4, 8)
    assert shard_range(64, 8, 0) == (0, 8)
    with pytest.raises(ValueError):
        shard_range(6, 4, 0)


@pytest.mark.gpu
def test_ep_nccl_two_gpus_matches_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.spawn(EH.gpu_worker, args=(2, _free_port(), "nccl"), nprocs=2, join=True)


@pytest.mark.gpu
@pytest.mark.parametrize("max_tokens", [64, 2100, 8300])
def test_ep_peer_one_gpu_matches_single_gpu(max_tokens):
    """The peer-memory exchange with one rank: dispatch, flags, the local layer
    on the padded receive area, the return and the combine on one GPU.  With
    max_tokens 8300 the receive area (16600 rows) is above the fused routing
    limit, so the layer takes its separate route and prep kernels."""
    mp.spawn(EH.gpu_worker, args=(1, _free_port(), "peer", max_tokens), nprocs=1, join=True)


@pytest.mark.gpu
@pytest.mark.parametrize("max_tokens", [64, 2100, 4200])
def test_ep_peer_one_gpu_with_shared_experts_folded(max_tokens):
    """Two BF16 shared experts folded into the expert launch (own receive
    block): bit for bit the exchange with the shared experts run apart, and
    the whole layer on one GPU within tolerance (one-rank group)."""
    mp.spawn(EH.gpu_worker, args=(1, _free_port(), "peer", max_tokens, True), nprocs=1,
             join=True)


@pytest.mark.gpu
def test_ep_peer_two_gpus_with_shared_experts_folded():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.spawn(EH.gpu_worker, args=(2, _free_port(), "peer", 64, True), nprocs=2, join=True)


@pytest.mark.gpu
def test_ep_peer_step_replays_from_a_cuda_graph():
    """A peer-memory step captured once in a CUDA graph and replayed with new
    inputs equals the eager call (one-rank group, one GPU)."""
    mp.spawn(EH.gpu_graph_worker, args=(1, _free_port()), nprocs=1, join=True)


@pytest.mark.gpu
def test_ep_peer_two_gpus_matches_nccl_and_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.spawn(EH.gpu_worker, args=(2, _free_port(), "peer"), nprocs=2, join=True)


@pytest.mark.gpu
def test_ep_peer_wait_runs_out_and_recovers():
    """A wait on another rank that runs out (2 ms limit, a return flag that
    nothing raises) returns with EXQ_DEV_TIMEOUT, is reported by the layer's
    status check, and the exchange works again after reset() (one GPU)."""
    mp.spawn(EH.gpu_timeout_worker, args=(1, _free_port()), nprocs=1, join=True)
