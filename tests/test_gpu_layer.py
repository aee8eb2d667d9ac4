"""GPU parity of the grouped expert GEMMs and the fused MoE layer.

Tolerance (north_star): relative L2 error <= 0.5 % against the reference's
own implementation (its Triton kernels, via the golden fixtures) or its torch
dequant+matmul path (the oracle), fp16/bf16 activations, fp32 accumulation.
"""
import numpy as np
import pytest
import torch

from _layer_helpers import oracle_layer
from conftest import golden
from oracle import moe as OM
from oracle import quant as OQ

pytestmark = pytest.mark.gpu
TOL = 5e-3   # 0.5 % relative L2


@pytest.mark.parametrize("name", ["small", "wide"])
def test_moe_int4_forward_matches_reference_triton(cuda, name):
    from exq_b200 import moe_int4_forward
    g = golden(f"int4_gemm_{name}.npz")
    out = moe_int4_forward(torch.from_numpy(g["hidden"]).to(cuda),
                           torch.from_numpy(g["packed"]).to(cuda),
                           torch.from_numpy(g["scales"]).to(cuda),
                           torch.from_numpy(g["ids"]).to(cuda), int(g["n_experts"]))
    assert out.dtype == torch.float16
    ref = torch.from_numpy(g["out"].astype(np.float32))
    assert OM.rel_l2(out, ref) < 1e-3
    w = torch.from_numpy(OQ.dequant_int4(g["packed"], g["scales"]))
    orc = OM.moe_projection(torch.from_numpy(g["hidden"]), torch.from_numpy(g["ids"]), w)
    assert OM.rel_l2(out, orc) < 1e-3


def test_moe_grouped_gemm_matches_reference_triton(cuda):
    from exq_b200 import moe_grouped_gemm
    g = golden("fp16_gemm.npz")
    out = moe_grouped_gemm(torch.from_numpy(g["hidden"]).to(cuda), torch.from_numpy(g["w"]).to(cuda),
                           torch.from_numpy(g["ids"]).to(cuda), 4)
    assert OM.rel_l2(out, torch.from_numpy(g["out"].astype(np.float32))) < 1e-3


@pytest.mark.parametrize("t,k,e,n,kd", [(1, 8, 128, 1536, 2048), (33, 8, 128, 1536, 2048),
                                        (40, 2, 4, 256, 512), (3, 1, 2, 4096, 14336)])
@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
def test_moe_int4_forward_shapes(cuda, t, k, e, n, kd, dt):
    from exq_b200 import moe_int4_forward, pack_experts_int4
    from exq_b200.synth import zipf_router
    w = (torch.randn(e, n, kd, device=cuda) * 0.02).half()
    p, s = pack_experts_int4(w)
    del w
    ids, _ = zipf_router(t, e, k, seed=t)
    x = torch.randn(t, kd).to(dt)
    out = moe_int4_forward(x.to(cuda), p, s, ids.to(cuda), e)
    ref = OM.moe_projection(x, ids, lambda i: torch.from_numpy(
        OQ.dequant_int4(p[i].cpu().numpy(), s[i].cpu().numpy())))
    assert OM.rel_l2(out, ref) < 2e-3


def test_full_forward_matches_reference_layer(cuda):
    from exq_b200 import moe_int4_full_forward
    g = golden("layer_int4.npz")
    y = moe_int4_full_forward(*(torch.from_numpy(g[n]).to(cuda) for n in
                                ("hidden", "p13", "s13", "p2", "s2", "ids", "wts")), 4)
    ref = torch.from_numpy(g["y"].astype(np.float32))
    assert OM.rel_l2(y, ref) < 2e-3
    assert OM.max_diff_over_rms(y, ref) < 0.01


def _bank(cfg_name, cuda, tiers=None, seed=0, n_experts=None):
    from exq_b200 import ExpertBank
    from exq_b200.synth import CONFIGS, expert_weights
    c = CONFIGS[cfg_name]
    e = n_experts or c.n_experts
    w13, w2 = expert_weights(e, c.inter, c.hidden, seed=seed, dtype=torch.float16, device=cuda)
    sw13 = sw2 = None
    if c.n_shared:
        sw13, sw2 = expert_weights(c.n_shared, c.inter, c.hidden, seed=seed + 99,
                                   dtype=torch.float16, device=cuda)
    return ExpertBank.from_dense(w13, w2, tiers, act_dtype=c.act_dtype, shared_w13=sw13,
                                 shared_w2=sw2), c


@pytest.mark.parametrize("cfg,t", [("olmoe", 16), ("qwen3", 1), ("qwen3", 8), ("qwen3", 64)])
def test_layer_int4_vs_oracle(cuda, cfg, t):
    from exq_b200.synth import hidden_states, zipf_router
    bank, c = _bank(cfg, cuda)
    ids, w = zipf_router(t, c.n_experts, c.top_k, seed=t)
    x = hidden_states(t, c.hidden, seed=t, dtype=c.act_dtype)
    y = bank(x.to(cuda), ids.to(cuda), w.to(cuda))
    ref = oracle_layer(bank, x, ids, w)
    assert OM.rel_l2(y, ref) < TOL


@pytest.mark.parametrize("wdt", [torch.float16, torch.bfloat16])
def test_layer_router_weight_dtypes(cuda, wdt):
    """The combine reads the router weights in the caller's dtype (fp32, fp16 or
    bf16), as the reference's combine does; a heavy expert (tiles of 64) and
    light ones in the same call."""
    from exq_b200.synth import hidden_states, zipf_router
    bank, c = _bank("qwen3", cuda, n_experts=32)
    ids, w = zipf_router(96, 32, 8, seed=31)
    x = hidden_states(96, c.hidden, seed=31)
    wq = w.to(wdt)
    y = bank(x.to(cuda), ids.to(cuda), wq.to(cuda))
    ref = oracle_layer(bank, x, ids, wq.float())
    assert OM.rel_l2(y, ref) < TOL
    y32 = bank(x.to(cuda), ids.to(cuda), wq.float().to(cuda))
    assert torch.equal(y, y32)  # the same weight values give the same bits


def test_layer_mixed_tiers_vs_oracle(cuda):
    """6 BF16 / 13 INT8 / 45 INT4 experts in one launch."""
    from exq_b200.synth import hidden_states, tier_plan, zipf_router
    tiers = tier_plan(64, seed=0)
    bank, c = _bank("olmoe_mixed", cuda, tiers=tiers)
    assert sorted(bank.storage) == ["BF16", "INT4", "INT8"]
    ids, w = zipf_router(64, 64, 8, seed=0)
    x = hidden_states(64, c.hidden, seed=0)
    y = bank(x.to(cuda), ids.to(cuda), w.to(cuda))
    ref = oracle_layer(bank, x, ids, w)
    assert OM.rel_l2(y, ref) < TOL
    used = {tiers[i] for i in set(ids.reshape(-1).tolist())}
    assert used == {"BF16", "INT8", "INT4"}


def test_layer_bf16_with_shared_experts_vs_oracle(cuda):
    """BASELINE config 5 shape: E64 top-6 I1408 INT4 + 2 shared BF16 experts, bf16."""
    from exq_b200.synth import hidden_states, zipf_router
    bank, c = _bank("dsv2_lite", cuda)
    assert bank.n_shared == 2 and bank.tiers[-2:] == ["BF16", "BF16"]
    ids, w = zipf_router(64, 64, 6, seed=5)
    x = hidden_states(64, c.hidden, seed=5, dtype=torch.bfloat16)
    y = bank(x.to(cuda), ids.to(cuda), w.to(cuda))
    assert y.dtype == torch.bfloat16
    ref = oracle_layer(bank, x, ids, w)
    assert OM.rel_l2(y, ref) < TOL


def test_layer_mixtral_long_k_vs_oracle(cuda):
    """BASELINE config 4 shape (E8 top-2 H4096 I14336, bf16), decode tokens."""
    from exq_b200.synth import hidden_states, zipf_router
    bank, c = _bank("mixtral", cuda)
    ids, w = zipf_router(8, 8, 2, seed=1)
    x = hidden_states(8, c.hidden, seed=1, dtype=torch.bfloat16)
    y = bank(x.to(cuda), ids.to(cuda), w.to(cuda))
    ref = oracle_layer(bank, x, ids, w)
    assert OM.rel_l2(y, ref) < TOL


@pytest.mark.parametrize("tiers", [None, "mixed"])
def test_layer_above_fused_routing_limit(cuda, tiers):
    """More than 16384 slots (Qwen3 shape, 2100 tokens x top-8 = 16800): the
    routing runs as the single-CTA sort plus the separate activation prep, the
    GEMM builds no tile list of its own; checked on a token sample, all tiers."""
    from exq_b200.synth import CONFIGS, hidden_states, tier_plan, zipf_router
    c0 = CONFIGS["qwen3"]
    bank, c = _bank("qwen3", cuda, tiers=tier_plan(c0.n_experts, seed=4) if tiers else None)
    ids, w = zipf_router(2100, 128, 8, seed=21)
    x = hidden_states(2100, c.hidden, seed=21)
    assert ids.numel() > 16384
    y = bank(x.to(cuda), ids.to(cuda), w.to(cuda)).cpu()
    sample = torch.tensor([0, 3, 1049, 1050, 2098, 2099])
    ref = oracle_layer(bank, x, ids, w, tokens=sample)
    assert OM.rel_l2(y[sample], ref) < TOL


def test_layer_full_size_sampled_tokens(cuda):
    """Qwen3 at 256 tokens (all 128 experts touched, hot experts > 32 rows):
    every token's output depends on that token only, so a sample of tokens is
    checked against the oracle at full size."""
    from exq_b200.synth import hidden_states, zipf_router
    bank, c = _bank("qwen3", cuda)
    ids, w = zipf_router(256, 128, 8, seed=11)
    x = hidden_states(256, c.hidden, seed=11)
    y = bank(x.to(cuda), ids.to(cuda), w.to(cuda)).cpu()
    counts = torch.bincount(ids.reshape(-1).long(), minlength=128)
    assert counts.max() > 32   # multi-tile experts are exercised
    sample = torch.tensor([0, 1, 17, 100, 128, 200, 254, 255])
    ref = oracle_layer(bank, x, ids, w, tokens=sample)
    assert OM.rel_l2(y[sample], ref) < TOL


def test_layer_full_size_exact_properties(cuda):
    """Size-independent properties at the full Qwen3 T=256 size, both exact:
    permuting tokens permutes the output rows (a token's result does not depend
    on which tokens share its expert tile), and halving every router weight
    halves the output (the weight multiplies an fp32 partial; halving is exact)."""
    from exq_b200.synth import hidden_states, zipf_router
    bank, c = _bank("qwen3", cuda)
    ids, w = zipf_router(256, 128, 8, seed=12)
    x = hidden_states(256, c.hidden, seed=12)
    x, ids, w = x.to(cuda), ids.to(cuda), w.to(cuda)
    y = bank(x, ids, w)
    perm = torch.randperm(256, generator=torch.Generator().manual_seed(5)).to(cuda)
    y_perm = bank(x[perm], ids[perm], w[perm])
    assert torch.equal(y_perm, y[perm])
    y_half = bank(x, ids, w * 0.5)
    # atol: one fp16 subnormal step, for outputs that halve into the subnormal range
    torch.testing.assert_close(y_half, y * 0.5, rtol=0, atol=6e-8)


def test_layer_deterministic_and_token_count_edges(cuda):
    from exq_b200.synth import hidden_states, zipf_router
    bank, c = _bank("qwen3", cuda, n_experts=16)
    ids, w = zipf_router(37, 16, 8, seed=2)
    x = hidden_states(37, c.hidden, seed=2).to(cuda)
    y1 = bank(x, ids.to(cuda), w.to(cuda))
    y2 = bank(x, ids.to(cuda), w.to(cuda))
    assert torch.equal(y1, y2)
    # zero tokens
    y0 = bank(x[:0], ids[:0].to(cuda), w[:0].to(cuda))
    assert y0.shape == (0, c.hidden)
    # every token to the same experts: one expert with 37*... rows > tile height
    same = torch.zeros_like(ids)
    same[:, 1:] = torch.arange(1, 8)
    ys = bank(x, same.to(cuda), w.to(cuda))
    ref = oracle_layer(bank, x.cpu(), same, w)
    assert OM.rel_l2(ys, ref) < TOL


def test_layer_back_to_back_calls_keep_their_own_tiles(cuda):
    """Calls launched back to back on one stream, with different routings on
    one cached workspace, each equal bit for bit the same call made alone: a
    kernel that starts before its predecessors finish (programmatic launch)
    must not read the previous call's tile list."""
    from exq_b200.synth import hidden_states, zipf_router
    bank, c = _bank("qwen3", cuda, n_experts=64)
    calls = []
    for i, t in enumerate([256, 3, 64, 1, 200, 17]):
        ids, w = zipf_router(t, 64, 8, seed=40 + i)
        x = hidden_states(t, c.hidden, seed=40 + i).to(cuda)
        calls.append((x, ids.to(cuda), w.to(cuda)))
    alone = []
    for args in calls:
        alone.append(bank(*args))
        torch.cuda.synchronize()
    for _ in range(20):
        outs = [bank(*args) for args in calls]
        torch.cuda.synchronize()
        for o, a in zip(outs, alone):
            assert torch.equal(o, a)


def test_layer_bad_expert_id_dropped_and_flagged(cuda):
    from exq_b200 import _lib as L
    from exq_b200.synth import hidden_states, zipf_router
    bank, c = _bank("qwen3", cuda, n_experts=8)
    ids, w = zipf_router(4, 8, 2, seed=3)
    x = hidden_states(4, c.hidden, seed=3)
    bad = ids.clone()
    bad[1, 1] = 1000
    L.read_device_status(cuda, clear=True)
    y = bank(x.to(cuda), bad.to(cuda), w.to(cuda))
    assert L.read_device_status(cuda) & L.DEV_BAD_EXPERT_ID
    w_drop = w.clone()
    w_drop[1, 1] = 0.0
    ref = oracle_layer(bank, x, ids, w_drop)
    assert OM.rel_l2(y, ref) < TOL


def test_sglang_forward_with_mock_layer(cuda):
    """The patched forward_cuda on a mock SGLang layer honours the artifact's
    per-expert tiers (sglang_backend.py:65-158 call shape)."""
    import types
    from exq_b200 import sglang_backend as B
    from exq_b200.synth import expert_weights, hidden_states, zipf_router
    e, h, i = 16, 2048, 768
    qa = {f"0:{j}": ("BF16" if j < 2 else "INT8" if j < 5 else "INT4") for j in range(e)}
    B.set_artifact({"quant_assignments": qa})
    w13, w2 = expert_weights(e, i, h, seed=4, device=cuda)
    layer = types.SimpleNamespace(w13_weight=w13, w2_weight=w2, layer_id=0)
    ids, w = zipf_router(24, e, 8, seed=4)
    x = hidden_states(24, h, seed=4)
    disp = types.SimpleNamespace(hidden_states=x.to(cuda), topk_output=types.SimpleNamespace(
        topk_ids=ids.to(cuda), topk_weights=w.to(cuda)))
    out = B._exq_forward_cuda(None, layer, disp, lambda *a: "fallthrough", 1)
    bank = B._get_or_pack(layer)["bank"]
    assert bank.tiers[:6] == ["BF16", "BF16", "INT8", "INT8", "INT8", "INT4"]
    ref = oracle_layer(bank, x, ids, w)
    assert OM.rel_l2(out.hidden_states, ref) < TOL
    layer2 = types.SimpleNamespace(w13_weight=w13, w2_weight=w2, layer_id=3)
    assert B._exq_forward_cuda(None, layer2, disp, lambda *a: "fallthrough", 1) == "fallthrough"


def _stage_runs(bank, x, ids, w):
    """The same call as one fused launch chain and as separately launched
    stages: (all stages, gate_up+down with the separate combine, every stage
    alone)."""
    fused = bank(x, ids, w)
    y_sep = torch.empty_like(fused)
    bank.forward_range(x, ids, w, 0, 4, out=y_sep)
    bank.forward_range(x, ids, w, 4, 5, out=y_sep)
    y_alone = torch.empty_like(fused)
    for s in range(5):
        bank.forward_range(x, ids, w, s, s + 1, out=y_alone)
    torch.cuda.synchronize()
    return fused, y_sep, y_alone


@pytest.mark.parametrize("cfg,t,tiers", [("qwen3", 1, None), ("qwen3", 8, None),
                                         ("qwen3", 256, None), ("dsv2_lite", 64, None),
                                         ("olmoe_mixed", 64, "mixed"), ("qwen3", 600, None)])
def test_fused_combine_bit_identical_to_separate_combine(cuda, cfg, t, tiers):
    """The top-k combine fused into the down items (a token's last arriving row
    block sums its slots in slot order) gives the same bits as the separate
    combine kernel, and gate_up + down in one launch the same bits as two."""
    from exq_b200.synth import CONFIGS, hidden_states, tier_plan, zipf_router
    c0 = CONFIGS[cfg]
    tl = tier_plan(c0.n_experts, seed=0) if tiers else None
    bank, c = _bank(cfg, cuda, tiers=tl)
    ids, w = zipf_router(t, c.n_experts, c.top_k, seed=70 + t)
    x = hidden_states(t, c.hidden, seed=70 + t, dtype=c.act_dtype).to(cuda)
    fused, y_sep, y_alone = _stage_runs(bank, x, ids.to(cuda), w.to(cuda))
    assert torch.equal(fused, y_sep)
    assert torch.equal(fused, y_alone)


def test_fused_combine_tokens_without_experts(cuda):
    """Tokens whose slots are all padding (-1) or all dropped (id past the
    experts) get a zero row; the other tokens match the oracle."""
    from exq_b200 import _lib as L
    from exq_b200.synth import hidden_states, zipf_router
    bank, c = _bank("qwen3", cuda, n_experts=16)
    ids, w = zipf_router(12, 16, 8, seed=9)
    x = hidden_states(12, c.hidden, seed=9)
    ids[3] = -1
    ids[7] = 99
    L.read_device_status(cuda, clear=True)
    y = bank(x.to(cuda), ids.to(cuda), w.to(cuda)).cpu()
    assert L.read_device_status(cuda, clear=True) & L.DEV_BAD_EXPERT_ID
    assert torch.count_nonzero(y[3]) == 0 and torch.count_nonzero(y[7]) == 0
    keep = torch.tensor([i for i in range(12) if i not in (3, 7)])
    ref = oracle_layer(bank, x, ids, w, tokens=keep)
    assert OM.rel_l2(y[keep], ref) < TOL
    _, y_sep, _ = _stage_runs(bank, x.to(cuda), ids.to(cuda), w.to(cuda))
    assert torch.equal(y, y_sep.cpu())


@pytest.mark.parametrize("t", [32, 128])
def test_layer_qwen3_decode_sizes_in_full(cuda, t):
    """BASELINE config 2 at T=32 and T=128: every token against the oracle."""
    from exq_b200.synth import hidden_states, zipf_router
    bank, c = _bank("qwen3", cuda)
    ids, w = zipf_router(t, c.n_experts, c.top_k, seed=t + 1)
    x = hidden_states(t, c.hidden, seed=t + 1)
    y = bank(x.to(cuda), ids.to(cuda), w.to(cuda))
    ref = oracle_layer(bank, x, ids, w)
    assert OM.rel_l2(y, ref) < TOL


def test_layer_mixtral_prefill_4096(cuda):
    """BASELINE config 4 prefill (E8 top-2 H4096 I14336, bf16, T=4096): 8192
    rows, 210 to 3109 per expert (Zipf), so every expert runs several token
    tiles in the large-call path.  A sample of tokens run as a call of their own must give the same
    rows bit for bit (a token's result does not depend on the other tokens in
    its tiles), and that small call is checked against the oracle."""
    from exq_b200.synth import hidden_states, zipf_router
    bank, c = _bank("mixtral", cuda)
    t = 4096
    ids, w = zipf_router(t, c.n_experts, c.top_k, seed=40)
    x = hidden_states(t, c.hidden, seed=40, dtype=torch.bfloat16)
    xd, idd, wd = x.to(cuda), ids.to(cuda), w.to(cuda)
    y = bank(xd, idd, wd)
    assert torch.bincount(ids.reshape(-1).long(), minlength=8).min() > 192   # 4+ tiles each
    sample = torch.tensor([0, 1, 2, 511, 1024, 2047, 2048, 3000, 4000, 4094, 4095])
    ys = bank(xd[sample.to(cuda)], idd[sample.to(cuda)], wd[sample.to(cuda)])
    assert torch.equal(ys, y[sample.to(cuda)])
    ref = oracle_layer(bank, x, ids, w, tokens=sample)
    assert OM.rel_l2(ys, ref) < TOL


@pytest.mark.parametrize("cfg,t,tiers", [("mixtral", 1024, None), ("olmoe_mixed", 2048, "mixed"),
                                         ("qwen3", 4096, None)])
def test_layer_128_token_tiles(cuda, cfg, t, tiers):
    """Calls averaging >= 128 rows per expert run 128-token tiles: Mixtral
    T=1024 (2048 slots, fused routing, the combine in the GEMM launch), OLMoE
    mixed tiers T=2048 and Qwen3 T=4096 (separate routing).  A token sample
    against the oracle, the sample run alone bit for bit (64-token tiles
    there), and the launch chain against separately launched stages."""
    from exq_b200.synth import CONFIGS, hidden_states, tier_plan, zipf_router
    c0 = CONFIGS[cfg]
    tl = tier_plan(c0.n_experts, seed=0) if tiers else None
    bank, c = _bank(cfg, cuda, tiers=tl)
    ids, w = zipf_router(t, c.n_experts, c.top_k, seed=90 + t)
    assert ids.numel() >= 128 * c.n_experts   # the 128-token tile rule
    x = hidden_states(t, c.hidden, seed=90 + t, dtype=c.act_dtype)
    xd, idd, wd = x.to(cuda), ids.to(cuda), w.to(cuda)
    y, y_sep, y_alone = _stage_runs(bank, xd, idd, wd)
    assert torch.equal(y, y_sep)
    assert torch.equal(y, y_alone)
    sample = torch.tensor([0, 1, 7, t // 3, t // 2, t - 2, t - 1])
    sd = sample.to(cuda)
    ys = bank(xd[sd], idd[sd], wd[sd])
    assert torch.equal(ys, y[sd])
    ref = oracle_layer(bank, x, ids, w, tokens=sample)
    assert OM.rel_l2(ys, ref) < TOL



@pytest.mark.parametrize("t,e", [(600, 128), (1800, 128), (1100, 16), (2048, 4)])
def test_layer_fused_routing_between_4096_and_16384_slots(cuda, t, e):
    """4096 < slots <= 16384: up to 512 rows per expert on average, the
    multi-CTA routing kernel with the gather (few buckets: per-warp aggregated
    counts) and the GEMM building its tile list from the ids; deeper experts
    (2048 tokens over 4 experts) the separate routing and gather kernels.  A
    token sample against the oracle, the sample alone bit for bit, and the
    launch chain against separately launched stages."""
    from exq_b200.synth import hidden_states, zipf_router
    bank, c = _bank("qwen3", cuda, n_experts=e)
    ids, w = zipf_router(t, e, 4 if e <= 16 else 8, seed=t)
    assert 4096 < ids.numel() <= 16384
    x = hidden_states(t, c.hidden, seed=t)
    xd, idd, wd = x.to(cuda), ids.to(cuda), w.to(cuda)
    y, y_sep, y_alone = _stage_runs(bank, xd, idd, wd)
    assert torch.equal(y, y_sep) and torch.equal(y, y_alone)
    sample = torch.tensor([0, 5, t // 2, t - 1])
    sd = sample.to(cuda)
    assert torch.equal(bank(xd[sd], idd[sd], wd[sd]), y[sd])
    ref = oracle_layer(bank, x, ids, w, tokens=sample)
    assert OM.rel_l2(y[sd], ref) < TOL
