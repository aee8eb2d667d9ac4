"""The two-tier expert store on the GPU: outputs bit-identical to the resident
bank (the same kernels read the same bytes), across calls that evict and
reload INT4 experts, with BF16 / INT8 experts and shared experts resident."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _banks(cuda, n_experts=16, shared=False):
    """Two identical banks from the same weights: one stays resident, one is
    offloaded (building the offloaded store releases its source's INT4 tier)."""
    from exq_b200 import ExpertBank
    from exq_b200.synth import CONFIGS, expert_weights, tier_plan
    c = CONFIGS["qwen3"]
    tiers = tier_plan(n_experts, seed=2)
    out = []
    for _ in range(2):
        w13, w2 = expert_weights(n_experts, c.inter, c.hidden, seed=8, device=cuda)
        sw13 = sw2 = None
        if shared:
            sw13, sw2 = expert_weights(1, c.inter, c.hidden, seed=9, device=cuda)
        out.append(ExpertBank.from_dense(w13, w2, tiers, act_dtype=torch.float16,
                                         shared_w13=sw13, shared_w2=sw2))
    return out[0], out[1], tiers, c


def _call_ids(tiers, pick_int4, others, t, k, seed):
    """[t, k] ids over a chosen set of INT4 experts plus some other-tier ones."""
    g = torch.Generator().manual_seed(seed)
    pool = list(pick_int4) + list(others)
    rows = [torch.tensor(pool)[torch.randperm(len(pool), generator=g)[:k]] for _ in range(t)]
    ids = torch.stack(rows).to(torch.int32)
    w = torch.softmax(torch.randn(t, k, generator=g), -1)
    return ids, w


@pytest.mark.parametrize("shared", [False, True])
def test_offloaded_bank_matches_resident_across_evictions(cuda, shared):
    from exq_b200.offload import OffloadedExpertBank
    from exq_b200.synth import hidden_states
    ref, src, tiers, c = _banks(cuda, shared=shared)
    int4 = [e for e, t in enumerate(tiers) if t == "INT4"]
    hot = [e for e, t in enumerate(tiers) if t != "INT4"]
    off = OffloadedExpertBank(src, gpu_slots=4)
    assert off.stats["cpu_stored"] == len(int4) and off.stats["gpu_slots"] == 4
    calls = [int4[0:4], int4[2:6], int4[0:2] + int4[8:10], int4[5:9], int4[0:4]]
    for i, pick in enumerate(calls):
        ids, w = _call_ids(tiers, pick, hot[:2], t=5, k=4, seed=i)
        x = hidden_states(5, c.hidden, seed=i).to(cuda)
        y = off(x, ids.to(cuda), w.to(cuda))
        y_ref = ref(x, ids.to(cuda), w.to(cuda))
        torch.cuda.synchronize()
        assert torch.equal(y, y_ref), i
    st = off.stats
    assert st["misses"] > 4 and st["hits"] > 0 and st["resident"] == 4
    assert st["bytes_copied"] == st["misses"] * ref.weight_bytes(int4[0])


def test_offloaded_bank_graph_of_resident_calls_and_errors(cuda):
    """A pool that holds every INT4 expert behaves as the resident bank; a
    call that needs more INT4 experts than the pool holds is refused."""
    from exq_b200.offload import OffloadedExpertBank
    from exq_b200.synth import hidden_states, zipf_router
    ref, src, tiers, c = _banks(cuda)
    n4 = sum(t == "INT4" for t in tiers)
    off = OffloadedExpertBank(src, gpu_slots=64)
    assert off.stats["gpu_slots"] == n4
    ids, w = zipf_router(32, 16, 8, seed=4)
    x = hidden_states(32, c.hidden, seed=4).to(cuda)
    y = off(x, ids.to(cuda), w.to(cuda), ids_host=ids)
    assert torch.equal(y, ref(x, ids.to(cuda), w.to(cuda)))
    small = OffloadedExpertBank(_banks(cuda)[1], gpu_slots=2)
    int4 = [e for e, t in enumerate(tiers) if t == "INT4"]
    bad = torch.tensor([int4[:3]], dtype=torch.int32)
    with pytest.raises(ValueError):
        small(x[:1], bad.to(cuda), torch.full((1, 3), 1 / 3, device=cuda))


def test_bank_cache_round_trip_on_gpu(cuda, tmp_path):
    """A mixed-tier bank with a shared expert, saved and loaded: the same
    outputs bit for bit."""
    from exq_b200 import ExpertBank
    from exq_b200.synth import hidden_states, zipf_router
    ref, _, tiers, c = _banks(cuda, shared=True)
    ref.save(tmp_path / "bank.pt")
    got = ExpertBank.load(tmp_path / "bank.pt", device=cuda)
    ids, w = zipf_router(24, 16, 8, seed=6)
    x = hidden_states(24, c.hidden, seed=6).to(cuda)
    assert torch.equal(got(x, ids.to(cuda), w.to(cuda)), ref(x, ids.to(cuda), w.to(cuda)))


def test_offloaded_bank_zero_tokens_and_prefetch_ahead(cuda):
    """No tokens; experts prefetched ahead of the call they serve count as
    hits in that call."""
    from exq_b200.offload import OffloadedExpertBank
    from exq_b200.synth import hidden_states
    ref, src, tiers, c = _banks(cuda)
    int4 = [e for e, t in enumerate(tiers) if t == "INT4"]
    off = OffloadedExpertBank(src, gpu_slots=3)
    y0 = off(torch.zeros(0, c.hidden, dtype=torch.float16, device=cuda),
             torch.zeros(0, 2, dtype=torch.int32, device=cuda),
             torch.zeros(0, 2, device=cuda))
    assert y0.shape == (0, c.hidden)
    off.prefetch(int4[:2])
    misses = off.stats["misses"]
    ids = torch.tensor([[int4[0], int4[1]]] * 3, dtype=torch.int32)
    w = torch.full((3, 2), 0.5)
    x = hidden_states(3, c.hidden, seed=1).to(cuda)
    y = off(x, ids.to(cuda), w.to(cuda), ids_host=ids)
    assert off.stats["misses"] == misses and off.stats["hits"] >= 2
    assert torch.equal(y, ref(x, ids.to(cuda), w.to(cuda)))
