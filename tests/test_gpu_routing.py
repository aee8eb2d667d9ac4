"""GPU parity: routing metadata, gather, combine, SiLU*mul and the packers
against the CPU oracle, through the C ABI.  Integer/byte outputs bit-exact."""
import numpy as np
import pytest
import torch

from conftest import golden
from oracle import quant as OQ
from oracle import routing as OR

pytestmark = pytest.mark.gpu

ALIGN_CASES = [(1, 8, 128), (7, 2, 8), (16, 8, 64), (256, 8, 128), (64, 6, 64), (0, 2, 4),
               (33, 6, 3), (4096, 2, 8), (513, 8, 256), (3, 1, 1)]


def _ids(t, k, e, seed, dtype=torch.int32):
    rng = np.random.default_rng(seed)
    return torch.from_numpy(rng.integers(0, e, size=(t, k))).to(dtype)


@pytest.mark.parametrize("t,k,e", ALIGN_CASES)
@pytest.mark.parametrize("ids_dtype", [torch.int32, torch.int64])
def test_moe_align_block_size_bit_exact(cuda, t, k, e, ids_dtype):
    from exq_b200 import exq_dispatch_cuda as D
    ids = _ids(t, k, e, t * 7 + k, ids_dtype)
    num_experts, bs = e + 1, 16
    cap, blocks = OR.align_capacity(ids.numel(), num_experts, bs)
    sorted_ids = torch.full((cap,), -7, dtype=torch.int32, device=cuda)
    expert_ids = torch.full((blocks,), -7, dtype=torch.int32, device=cuda)
    ntpp = torch.empty(1, dtype=torch.int32, device=cuda)
    cumsum = torch.empty(num_experts + 1, dtype=torch.int32, device=cuda)
    D.moe_align_block_size(ids.to(cuda), num_experts, bs, sorted_ids, expert_ids, ntpp, cumsum,
                           True)
    r_sorted, r_blocks, r_ntpp, r_cumsum = OR.moe_align_block_size(ids.numpy(), num_experts, bs)
    assert np.array_equal(sorted_ids.cpu().numpy(), r_sorted)
    assert np.array_equal(expert_ids.cpu().numpy(), r_blocks)
    assert int(ntpp.item()) == int(r_ntpp[0])
    assert np.array_equal(cumsum.cpu().numpy(), r_cumsum)


def test_moe_align_without_padding_leaves_caller_fill(cuda):
    from exq_b200 import exq_dispatch_cuda as D
    ids = _ids(5, 2, 4, 1)
    cap, blocks = OR.align_capacity(10, 5, 16)
    sorted_ids = torch.full((cap,), 12345, dtype=torch.int32, device=cuda)
    expert_ids = torch.empty(blocks, dtype=torch.int32, device=cuda)
    ntpp = torch.empty(1, dtype=torch.int32, device=cuda)
    cumsum = torch.empty(6, dtype=torch.int32, device=cuda)
    D.moe_align_block_size(ids.to(cuda), 5, 16, sorted_ids, expert_ids, ntpp, cumsum, False)
    r_sorted, _, _, _ = OR.moe_align_block_size(ids.numpy(), 5, 16)
    got = sorted_ids.cpu().numpy()
    assert np.array_equal(np.where(r_sorted == 10, 12345, r_sorted), got)


@pytest.mark.parametrize("t,k,e", ALIGN_CASES)
def test_build_ends_from_slots_bit_exact(cuda, t, k, e):
    from exq_b200 import exq_dispatch_cuda as D
    ids = _ids(t, k, e, t + 3 * k)
    n = ids.numel()
    r_sorted, _, _, _ = OR.moe_align_block_size(ids.numpy(), e + 1, 16)
    ends = torch.full((e + 1,), -1, dtype=torch.int32, device=cuda)   # not pre-zeroed
    so = torch.empty(n, dtype=torch.int64, device=cuda)
    D.build_ends_from_slots(torch.from_numpy(r_sorted).to(cuda), ids.reshape(-1).to(cuda), ends, so,
                            n, e)
    r_ends, r_so = OR.build_ends_from_slots(r_sorted, ids.numpy().reshape(-1), n, e)
    assert np.array_equal(ends.cpu().numpy(), r_ends)
    assert np.array_equal(so.cpu().numpy(), r_so)


def test_build_ends_from_atomics_ordered_align_output(cuda):
    """The reference's sgl align may order slots inside an expert arbitrarily:
    ends stay equal and every expert segment holds the same slot set."""
    from exq_b200 import exq_dispatch_cuda as D
    ids = _ids(200, 8, 32, 9)
    n = ids.numel()
    r_sorted, _, _, cums = OR.moe_align_block_size(ids.numpy(), 33, 16)
    rng = np.random.default_rng(0)
    shuffled = r_sorted.copy()
    for e in range(33):
        seg = shuffled[cums[e]:cums[e + 1]]
        rng.shuffle(seg)
        shuffled[cums[e]:cums[e + 1]] = seg
    ends = torch.empty(33, dtype=torch.int32, device=cuda)
    so = torch.empty(n, dtype=torch.int64, device=cuda)
    D.build_ends_from_slots(torch.from_numpy(shuffled).to(cuda), ids.reshape(-1).to(cuda), ends, so,
                            n, 32)
    r_ends, r_so = OR.build_ends_from_slots(shuffled, ids.numpy().reshape(-1), n, 32)
    got = so.cpu().numpy()
    assert np.array_equal(ends.cpu().numpy(), r_ends)
    assert np.array_equal(got, r_so)   # order of appearance, as the oracle states
    for e in range(32):
        assert sorted(got[r_ends[e]:r_ends[e + 1]]) == sorted(np.nonzero(ids.numpy().reshape(-1) == e)[0])


@pytest.mark.parametrize("t,k,e", ALIGN_CASES)
def test_dispatch_bit_exact(cuda, t, k, e):
    from exq_b200 import exq_dispatch_cuda as D
    ids = _ids(t, k, e, 5 * t + k, torch.int64)
    n = ids.numel()
    so = torch.empty(n, dtype=torch.int64, device=cuda)
    se = torch.empty(n, dtype=torch.int64, device=cuda)
    ends = torch.empty(e + 1, dtype=torch.int32, device=cuda)
    D.dispatch(ids.to(cuda), so, se, ends, e)
    r_so, r_se, r_ends = OR.dispatch(ids.numpy(), e)
    assert np.array_equal(so.cpu().numpy(), r_so)
    assert np.array_equal(se.cpu().numpy(), r_se)
    assert np.array_equal(ends.cpu().numpy(), r_ends)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("h", [2048, 96, 100])
def test_gather_hidden_bit_exact(cuda, dtype, h):
    from exq_b200 import exq_dispatch_cuda as D
    t, k = 37, 4
    x = torch.randn(t, h).to(dtype)
    ids = _ids(t, k, 16, 2)
    so, _, _ = OR.dispatch(ids.numpy(), 16)
    out = torch.empty(t * k, h, dtype=dtype, device=cuda)
    D.gather_hidden(x.to(cuda), torch.from_numpy(so).to(cuda), out, k)
    assert torch.equal(out.cpu(), x[torch.from_numpy(so) // k])


@pytest.mark.parametrize("wdt", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
def test_combine_bit_exact(cuda, wdt, dt):
    from exq_b200 import exq_dispatch_cuda as D
    t, k, h = 29, 8, 2048
    ids = _ids(t, k, 64, 4)
    so, _, _ = OR.dispatch(ids.numpy(), 64)
    down = torch.randn(t * k, h).to(dt)
    w = torch.softmax(torch.randn(t, k), -1).to(wdt)
    res = torch.empty(t, h, dtype=dt, device=cuda)
    D.combine(down.to(cuda), torch.from_numpy(so).to(cuda), w.to(cuda), res)
    ref = OR.combine(down.float().numpy(), so, w.float().numpy(), out_dtype=np.float32)
    ref = torch.from_numpy(ref).to(dt)
    assert torch.equal(res.cpu(), ref)


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
def test_silu_and_mul(cuda, dt):
    from exq_b200 import exq_dispatch_cuda as D
    x = (torch.randn(33, 2 * 768) * 3).to(dt)
    out = torch.empty(33, 768, dtype=dt, device=cuda)
    D.silu_and_mul(x.to(cuda), out)
    ref = torch.from_numpy(OR.silu_and_mul(x.float().numpy(), np.float32)).to(dt)
    torch.testing.assert_close(out.cpu().float(), ref.float(), rtol=8e-3, atol=1e-5)


def test_pack_int4_bit_exact_on_golden_and_large(cuda):
    from exq_b200 import pack_int4_weights
    g = golden("pack_int4.npz")
    for i in range(5):
        w = torch.from_numpy(g[f"w{i}"]).to(cuda)
        p, s = pack_int4_weights(w, int(g[f"gs{i}"]))
        assert np.array_equal(p.cpu().numpy(), g[f"packed{i}"]), i
        assert np.array_equal(s.cpu().numpy().view(np.uint16), g[f"scales{i}"].view(np.uint16)), i
    w = torch.from_numpy(g["w_edge"]).to(cuda)
    p, s = pack_int4_weights(w)
    assert np.array_equal(p.cpu().numpy(), g["packed_edge"])
    # a full Qwen3-shaped expert bank slice, bf16 input
    wl = (torch.randn(4, 1536, 2048) * 0.02).to(torch.bfloat16)
    from exq_b200 import pack_experts_int4
    p, s = pack_experts_int4(wl.to(cuda))
    rp, rs = OQ.pack_experts_int4(wl.float().numpy())
    assert np.array_equal(p.cpu().numpy(), rp)
    assert np.array_equal(s.cpu().numpy().view(np.uint16), rs.view(np.uint16))


def test_quant_int8_bit_exact(cuda):
    from exq_b200.experts import quant_int8
    w = (torch.randn(256, 2048) * 0.02).half()
    q, s = quant_int8(w.to(cuda))
    rq, rs = OQ.quant_int8(w.numpy())
    assert np.array_equal(q.cpu().numpy(), rq)
    assert np.array_equal(s.cpu().numpy().view(np.uint16), rs.view(np.uint16))


def test_sort_tokens_by_expert_api(cuda):
    from exq_b200 import sort_tokens_by_expert
    g = golden("routing.npz")
    for i in range(4):
        ids = torch.from_numpy(g[f"ids{i}"])
        x = torch.randn(ids.shape[0], 64).half()
        so, sh, ends, mt = sort_tokens_by_expert(ids.to(cuda), x.to(cuda), int(g[f"e{i}"]))
        assert np.array_equal(so.cpu().numpy(), g[f"sort_order{i}"])
        assert np.array_equal(ends.cpu().numpy(), g[f"ends{i}"])
        assert mt == int(g[f"max_tok{i}"])
        assert torch.equal(sh.cpu(), x[so.cpu() // ids.shape[1]])


def test_unsort_output_api(cuda):
    from exq_b200 import unsort_output
    g = golden("routing.npz")
    for i in range(4):
        got = unsort_output(torch.from_numpy(g[f"rows{i}"]).to(cuda),
                            torch.from_numpy(g[f"ids{i}"]).to(cuda),
                            torch.from_numpy(g[f"wts{i}"]).to(cuda))
        np.testing.assert_allclose(got.cpu().numpy(), g[f"unsort{i}"], rtol=1e-5, atol=1e-6)


def test_bad_expert_id_is_flagged_not_faulting(cuda):
    from exq_b200 import _lib as L
    from exq_b200 import exq_dispatch_cuda as D
    L.read_device_status(cuda, clear=True)
    ids = torch.tensor([[0, 1], [2, 99]], dtype=torch.int32, device=cuda)
    so = torch.empty(4, dtype=torch.int64, device=cuda)
    se = torch.empty(4, dtype=torch.int64, device=cuda)
    ends = torch.empty(5, dtype=torch.int32, device=cuda)
    D.dispatch(ids, so, se, ends, 4)
    assert L.read_device_status(cuda) & L.DEV_BAD_EXPERT_ID
    assert ends.cpu().tolist() == [0, 1, 2, 3, 3]   # the bad slot is dropped


ROUTER_CASES = [(1, 8, 2, torch.float32), (37, 64, 8, torch.bfloat16), (256, 128, 8, torch.float16),
                (4096, 8, 2, torch.bfloat16), (100, 160, 6, torch.float32), (9, 1024, 32, torch.float32),
                (3, 32, 32, torch.float16), (64, 60, 1, torch.float32)]


@pytest.mark.parametrize("t,e,k,dt", ROUTER_CASES)
@pytest.mark.parametrize("renorm", [True, False])
def test_router_topk_vs_oracle(cuda, t, e, k, dt, renorm):
    """Fused softmax -> top-k -> renormalise: ids exactly (descending, equal
    probabilities by lower expert id), weights within 2e-6 relative (CUDA's
    expf and a different summation order than torch's softmax)."""
    from exq_b200 import router_topk
    g = torch.Generator().manual_seed(t + 7 * e + k)
    logits = (torch.randn(t, e, generator=g) * 2).to(dt)
    ids, w = router_topk(logits.to(cuda), k, renorm)
    r_ids, r_w = OR.router_topk(logits.float(), k, renorm)
    assert ids.dtype == torch.int32 and w.dtype == torch.float32
    assert torch.equal(ids.cpu().long(), r_ids)
    torch.testing.assert_close(w.cpu(), r_w, rtol=2e-6, atol=1e-9)


def test_router_topk_ties_and_errors(cuda):
    from exq_b200 import router_topk
    logits = torch.tensor([[0.5, 1.0, 1.0, 0.2, 1.0], [3.0, 3.0, 3.0, 3.0, 3.0]], device=cuda)
    ids, w = router_topk(logits, 3, True)
    assert ids.tolist() == [[1, 2, 4], [0, 1, 2]]
    torch.testing.assert_close(w[1].cpu(), torch.full((3,), 1 / 3), rtol=1e-6, atol=0)
    with pytest.raises(ValueError):
        router_topk(logits, 6, True)            # top_k > n_experts
    with pytest.raises(ValueError):
        router_topk(torch.zeros(2, 1025, device=cuda), 2, True)
    e_ids, e_w = router_topk(torch.zeros(0, 8, device=cuda), 2, True)
    assert e_ids.shape == (0, 2) and e_w.shape == (0, 2)


@pytest.mark.parametrize("cfg,t", [("qwen3", 64), ("mixtral", 16), ("qwen3", 600)])
def test_layer_from_router_logits(cuda, cfg, t):
    """The layer fed by the fused router (one call: router, then the routing
    launch chained to it) equals the layer fed the oracle router's ids and
    weights (same ids; weights within an ulp).  T=600 (4800 slots) takes the
    separate routing kernel and activation prep after the router."""
    from _layer_helpers import oracle_layer
    from exq_b200 import ExpertBank
    from exq_b200.synth import CONFIGS, expert_weights, hidden_states
    from oracle import moe as OM
    c = CONFIGS[cfg]
    w13, w2 = expert_weights(c.n_experts, c.inter, c.hidden, seed=3, dtype=torch.float16,
                             device=cuda)
    bank = ExpertBank.from_dense(w13, w2, None, act_dtype=c.act_dtype)
    del w13, w2
    g = torch.Generator().manual_seed(t)
    logits = torch.randn(t, c.n_experts, generator=g)
    x = hidden_states(t, c.hidden, seed=t, dtype=c.act_dtype)
    y = bank.forward_from_logits(x.to(cuda), logits.to(cuda), c.top_k, True)
    r_ids, r_w = OR.router_topk(logits, c.top_k, True)
    ref = oracle_layer(bank, x, r_ids, r_w)
    assert OM.rel_l2(y, ref) < 5e-3
    y2 = bank(x.to(cuda), r_ids.to(cuda).int(), r_w.to(cuda))
    assert OM.rel_l2(y, y2) < 1e-5


def test_layer_from_logits_edges(cuda):
    """Zero tokens; bf16 logits without renormalisation (OLMoE-style routing)
    against the oracle router feeding the oracle layer."""
    from _layer_helpers import oracle_layer
    from exq_b200 import ExpertBank
    from exq_b200.synth import CONFIGS, expert_weights, hidden_states
    from oracle import moe as OM
    c = CONFIGS["olmoe"]
    w13, w2 = expert_weights(c.n_experts, c.inter, c.hidden, seed=4, dtype=torch.float16,
                             device=cuda)
    bank = ExpertBank.from_dense(w13, w2, None, act_dtype=torch.float16)
    del w13, w2
    y0 = bank.forward_from_logits(torch.zeros(0, c.hidden, dtype=torch.float16, device=cuda),
                                  torch.zeros(0, c.n_experts, device=cuda), c.top_k)
    assert y0.shape == (0, c.hidden)
    g = torch.Generator().manual_seed(12)
    logits = torch.randn(19, c.n_experts, generator=g).to(torch.bfloat16)
    x = hidden_states(19, c.hidden, seed=12)
    y = bank.forward_from_logits(x.to(cuda), logits.to(cuda), c.top_k, renormalize=False)
    r_ids, r_w = OR.router_topk(logits.float(), c.top_k, False)
    ref = oracle_layer(bank, x, r_ids, r_w)
    assert OM.rel_l2(y, ref) < 5e-3
    with pytest.raises(ValueError):
        bank.forward_from_logits(x.to(cuda), logits[:, :10].to(cuda), c.top_k)
