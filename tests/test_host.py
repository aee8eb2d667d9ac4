"""CPU: the C-ABI library loads and exports its header; host-side validation,
the artifact reader, the synthetic generators and the SGLang patch logic."""
import ctypes as C
import json
import types

import numpy as np
import pytest
import torch

from exq_b200 import _lib as L
from exq_b200 import artifact as A
from exq_b200 import synth as S


def test_library_exports_every_header_symbol(lib_path):
    decl = L.header_declarations()
    assert decl, "no declarations parsed from include/exq_b200.h"
    assert sorted(decl) == L.exported_symbols()
    handle = C.CDLL(str(lib_path))
    for name in decl:
        assert hasattr(handle, name), name
    assert L.lib().exq_abi_version() == 1


def test_ctypes_bindings_match_header_arity():
    """Every function the header declares is bound in exq_b200._lib with as many
    arguments as the declaration has parameters (a stale binding would pass
    shifted arguments to the library)."""
    import re
    from pathlib import Path
    src = (Path(__file__).resolve().parent.parent / "include" / "exq_b200.h").read_text()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    decls = {}
    for m in re.finditer(r"EXQ_API\s+[\w\s\*]*?\b(exq_\w+)\s*\(([^;]*?)\)\s*;", src, flags=re.S):
        params = m.group(2).strip()
        decls[m.group(1)] = 0 if params in ("", "void") else params.count(",") + 1
    assert len(decls) >= 30
    for name, n in decls.items():
        assert name in L.SIGNATURES, f"{name} is declared but not bound"
        assert len(L.SIGNATURES[name][1]) == n, f"{name}: {n} parameters, bound with " \
            f"{len(L.SIGNATURES[name][1])}"


def test_status_strings(lib_path):
    for code in (0, -1, -2, -3, -4):
        assert L.lib().exq_status_string(code)


def test_invalid_arguments_rejected_on_host(lib_path):
    """Argument errors return EXQ_ERR_INVALID before any CUDA call is made."""
    lib = L.lib()
    # bad ids dtype
    assert lib.exq_moe_align_block_size(None, L.F32, 4, 5, 16, 1, 100, 1, 10, 1, 1, 1, None) == -1
    assert "int32/int64" in lib.exq_last_error().decode()
    # sorted_token_ids too small for numel + E*(bs-1)
    assert lib.exq_moe_align_block_size(1, L.I32, 8, 4, 16, 1, 10, 1, 10, 1, 1, 1, None) == -1
    assert lib.exq_gather_hidden(1, L.F32, 1, 8, 8, 1, 1, 1, 1, None) == -1
    assert lib.exq_combine(1, L.F16, 5, 8, 1, 1, L.F16, 2, 2, 1, L.F16, None, 0, None) == -1
    assert lib.exq_pack_int4(1, L.F16, 4, 7, 128, 1, 1, None) == -1
    assert lib.exq_pack_int4(1, L.F16, 4, 192, 128, 1, 1, None) == -1
    # unsupported group size for the GEMM
    assert lib.exq_moe_gemm(1, 4, 64, 96, 1, L.F16, 2, 1, L.I32, 2, 1, L.F16, None, None, 1,
                            1 << 20, None) == -2
    # workspace too small, unsupported inter, bad stage range
    from exq_b200.experts import MoeWeightsC
    need = lib.exq_moe_layer_workspace_bytes(4, 2, 0, 8, 256, 256)
    assert need > 0
    w = MoeWeightsC()
    w.n_routed, w.hidden, w.inter = 8, 256, 256
    w.n_tier[2] = 8
    w.w13[2] = w.w2[2] = w.w13_scales[2] = w.w2_scales[2] = 256
    w.expert_slot = 256
    assert lib.exq_moe_layer_forward(C.byref(w), 1, L.F16, 4, 1, L.I32, 1, L.F32, 2, 1, 1,
                                     need - 1, None) == -4
    w.inter = 96
    assert lib.exq_moe_layer_forward(C.byref(w), 1, L.F16, 4, 1, L.I32, 1, L.F32, 2, 1, 1,
                                     1 << 30, None) == -2
    w.inter = 256
    assert lib.exq_moe_layer_forward_range(C.byref(w), 1, L.F16, 4, 1, L.I32, 1, L.F32, 2, 1, 1,
                                           1 << 30, None, 3, 9) == -1


def test_ep_entry_points_validate_on_host(lib_path):
    """The expert-parallel entry points size their buffer with plain arithmetic
    and reject bad arguments before any CUDA call."""
    lib = L.lib()
    up = lambda v: (v + 255) // 256 * 256  # noqa: E731
    p, cap, h = 2, 512, 4096
    rows = p * cap
    rows_in = rows + cap   # the receive side also holds this rank's own block
    assert lib.exq_ep_buffer_bytes(p, cap, h) == (1024 + 2 * up(4 * rows_in) + up(rows_in * 2 * h)
                                                  + up(rows * 2 * h))
    for bad in [(0, cap, h), (65, cap, h), (p, 0, h), (p, cap, 7), (64, 1 << 25, h)]:
        assert lib.exq_ep_buffer_bytes(*bad) == 0
    assert lib.exq_ep_buffer_init(None, p, cap, h, None) == -1
    assert "buffer is null" in lib.exq_last_error().decode()
    assert lib.exq_ep_ipc_alloc(0, C.byref(C.c_void_p()), None) == -1
    assert lib.exq_ep_ipc_open(None, C.byref(C.c_void_p())) == -1
    assert lib.exq_ep_ipc_free(None) == 0 and lib.exq_ep_ipc_close(None) == 0
    peers = 256
    # rank outside the group
    assert lib.exq_ep_dispatch(1, L.I32, 4, 2, 4, p, p, 256, L.F16, h, cap, peers, 1, None) == -1
    assert "rank 2 of 2" in lib.exq_last_error().decode()
    # ids dtype, activation dtype, more slots than one call takes
    assert lib.exq_ep_dispatch(1, L.F32, 4, 2, 4, p, 0, 256, L.F16, h, cap, peers, 1, None) == -1
    assert lib.exq_ep_dispatch(1, L.I32, 4, 2, 4, p, 0, 256, L.F32, h, cap, peers, 1, None) == -1
    assert lib.exq_ep_dispatch(1, L.I32, 4097, 1, 4, p, 0, 256, L.F16, h, cap, peers, 1,
                               None) == -2
    # the local bank holds routed experts only
    from exq_b200.experts import MoeWeightsC
    w = MoeWeightsC()
    w.n_routed, w.n_shared, w.hidden, w.inter = 4, 1, h, 256
    assert lib.exq_ep_expert_forward(C.byref(w), L.F16, p, 0, cap, 256, peers, 256, 1 << 30,
                                     None) == -1
    assert "shared experts" in lib.exq_last_error().decode()
    assert lib.exq_ep_combine_peer(256, p, cap, h, L.F16, 1, 1, L.I32, 4, 2, None, 1, None) == -1


def test_workspace_sizes_grow_with_tokens(lib_path):
    lib = L.lib()
    a = lib.exq_moe_layer_workspace_bytes(1, 8, 0, 128, 2048, 768)
    b = lib.exq_moe_layer_workspace_bytes(256, 8, 0, 128, 2048, 768)
    assert 0 < a < b
    assert b >= 256 * 8 * (2048 * 4 + 768 * 2)


def test_artifact_reader(tmp_path):
    art = {"quant_assignments": {"0:0": "BF16", "0:1": "INT8", "0:3": "INT4", "1:2": "INT8",
                                 "1:0": "WEIRD"}}
    p = tmp_path / "a.json"
    p.write_text(json.dumps(art))
    prof = A.load_exq_artifact(str(p), device="cpu")
    assert prof.n_layers == 2 and prof.n_experts_per_layer == 4
    assert prof.tiers.tolist() == [[0, 1, 2, 2], [2, 2, 1, 2]]   # missing/unknown -> INT4
    assert prof.hot_mask.tolist()[0] == [True, False, False, False]
    assert prof.block_m.tolist()[0] == [128, 64, 32, 32]        # tier-derived freqs
    assert prof.precision_counts() == {"BF16": 1, "INT8": 2, "INT4": 5}
    assert A.layer_tiers(art, 0, 5) == ["BF16", "INT8", "INT4", "INT4", "INT4"]
    with pytest.raises(ValueError):
        (tmp_path / "b.json").write_text("{}")
        A.load_exq_artifact(str(tmp_path / "b.json"), device="cpu")


def test_artifact_reader_with_profile(tmp_path):
    art = {"quant_assignments": {"0:0": "INT8", "0:1": "INT8"}}
    prof_json = {"layers": {"0": {"expert_stats": [{"expert_id": 0, "activation_freq": 0.05},
                                                   {"expert_id": 1, "activation_freq": 0.01}]}}}
    (tmp_path / "a.json").write_text(json.dumps(art))
    (tmp_path / "p.json").write_text(json.dumps(prof_json))
    prof = A.load_exq_artifact(str(tmp_path / "a.json"), str(tmp_path / "p.json"), device="cpu")
    assert prof.block_m.tolist() == [[64, 32]]


def test_zipf_router_is_seeded_and_normalised():
    a_ids, a_w = S.zipf_router(32, 64, 8, seed=3)
    b_ids, b_w = S.zipf_router(32, 64, 8, seed=3)
    assert torch.equal(a_ids, b_ids) and torch.equal(a_w, b_w)
    torch.testing.assert_close(a_w.sum(-1), torch.ones(32))
    assert all(len(set(r)) == 8 for r in a_ids.tolist())
    # skew: the hottest expert is picked by most tokens
    hot = int((S.zipf_ranks(64, 3) == 1).nonzero()[0])
    assert (a_ids == hot).any(-1).float().mean() > 0.5


def test_tier_plan_counts():
    plan = S.tier_plan(64, seed=0)
    assert (plan.count("BF16"), plan.count("INT8"), plan.count("INT4")) == (6, 13, 45)


def test_sglang_patch_logic_with_fake_method(monkeypatch, tmp_path):
    """patch/unpatch and the layer fallthrough rule (sglang_backend.py:83-85,
    :197-199) against a fake SGLang module; no kernel is launched."""
    import sys
    from exq_b200 import sglang_backend as B

    class FakeMethod:
        def forward_cuda(self, layer, dispatch_output):
            return "original"

    mod = types.ModuleType("sglang.srt.layers.quantization.unquant")
    mod.UnquantizedFusedMoEMethod = FakeMethod
    for name in ("sglang", "sglang.srt", "sglang.srt.layers", "sglang.srt.layers.quantization"):
        monkeypatch.setitem(sys.modules, name, types.ModuleType(name))
    monkeypatch.setitem(sys.modules, "sglang.srt.layers.quantization.unquant", mod)
    art = tmp_path / "a.json"
    art.write_text(json.dumps({"quant_assignments": {"0:0": "INT4", "1:0": "INT8"}}))
    backend = B.patch_sglang(str(art))
    assert backend.n_layers == 2
    m = FakeMethod()
    # layer beyond the artifact and layer without id fall through to the original
    assert m.forward_cuda(types.SimpleNamespace(layer_id=5), None) == "original"
    assert m.forward_cuda(types.SimpleNamespace(), None) == "original"
    B.patch_sglang(str(art))   # re-patch keeps the true original
    assert m.forward_cuda(types.SimpleNamespace(layer_id=2), None) == "original"
    B.unpatch_sglang()
    assert FakeMethod.forward_cuda(m, None, None) == "original"
    assert not FakeMethod._exq_patched
