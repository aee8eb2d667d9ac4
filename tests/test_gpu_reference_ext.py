"""The dispatch rows checked against the reference's own CUDA extension.

``baseline/_ref/exq_src/build/exq_dispatch_cuda*.so`` is the reference's
``exq/kernels/cuda_src/exq_dispatch.cu`` compiled unmodified for sm_100 by
``bench.py --setup-reference`` (torch's extension builder, as the reference's
``setup_cuda.py`` builds it for sm_86).  The tests run both implementations on
the same device inputs:

- ``dispatch`` (exq_dispatch.cu:99-149, CUB stable radix sort): bit-exact;
- ``build_ends_from_slots`` (:181-229, atomic cursors): ``expert_ends`` equal,
  each expert's segment of ``sort_order`` equal as a set (the reference's
  atomics order slots inside a segment arbitrarily);
- ``gather_hidden`` (:234-260): bit-exact;
- ``combine`` (:263-310, fp32 ``atomicAdd`` then fp16): within one fp16 ulp
  of the reference (both sum the same fp32 products; only the order differs).

The align step the reference takes from sgl_kernel is not in the reference
tree; ``vllm._custom_ops.moe_align_block_size`` implements the same contract
and is used as a runtime cross-check where it loads.

Every test skips when the compiled extension (or vLLM) is absent.
"""
from __future__ import annotations

import importlib.util
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

REF_BUILD = Path(__file__).resolve().parents[1] / "baseline" / "_ref" / "exq_src" / "build"


@pytest.fixture(scope="module")
def ref_ext():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    so = sorted(REF_BUILD.glob("exq_dispatch_cuda*.so"))
    if not so:
        pytest.skip("reference extension not built (bench.py --setup-reference)")
    try:
        spec = importlib.util.spec_from_file_location("exq_dispatch_cuda", so[0])
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
    except Exception as e:  # noqa: BLE001 - the reason is the skip message
        pytest.skip(f"reference extension does not load: {type(e).__name__}: {e}")
    return mod


def _ids(t, k, e, seed, zipf=False):
    g = torch.Generator().manual_seed(seed)
    if zipf:
        from exq_b200.synth import zipf_router
        ids, _ = zipf_router(t, e, k, seed=seed)
        return ids.to(torch.int64)
    # distinct experts per token, like a router's top-k
    return torch.stack([torch.randperm(e, generator=g)[:k] for _ in range(t)]).to(torch.int64)


DISPATCH_CASES = [(1, 1, 4), (1, 8, 128), (3, 2, 8), (17, 6, 64), (256, 8, 128), (200, 2, 8),
                  (4096, 2, 8), (64, 8, 129)]


@pytest.mark.parametrize("t,k,e", DISPATCH_CASES)
def test_dispatch_matches_reference_extension(ref_ext, t, k, e):
    from exq_b200 import exq_dispatch_cuda as D
    dev = torch.device("cuda", 0)
    ids = _ids(t, k, e, 11 * t + k, zipf=(t >= 64)).to(dev)
    n = ids.numel()
    outs = []
    for impl in (ref_ext, D):
        so = torch.full((n,), -5, dtype=torch.int64, device=dev)
        se = torch.full((n,), -5, dtype=torch.int64, device=dev)
        ends = torch.full((e + 1,), -5, dtype=torch.int32, device=dev)
        impl.dispatch(ids, so, se, ends, e)
        outs.append((so, se, ends))
    torch.cuda.synchronize()
    for a, b in zip(*outs):
        assert torch.equal(a, b)


@pytest.mark.parametrize("t,k,e", [(1, 8, 128), (5, 2, 4), (256, 8, 128), (4096, 2, 8), (33, 6, 64)])
def test_build_ends_from_slots_matches_reference_extension(ref_ext, t, k, e):
    from exq_b200 import exq_dispatch_cuda as D
    dev = torch.device("cuda", 0)
    ids = _ids(t, k, e, 5 * t + e, zipf=True).to(dev)
    n = ids.numel()
    flat = ids.reshape(-1).to(torch.int32)
    # align output over E + 1 buckets with block 16, as the reference backend calls it
    nb, bs = e + 1, 16
    cap = n + nb * (bs - 1)
    sorted_ids = torch.empty(cap, dtype=torch.int32, device=dev)
    blocks = torch.empty((cap + bs - 1) // bs, dtype=torch.int32, device=dev)
    ntpp = torch.empty(1, dtype=torch.int32, device=dev)
    cums = torch.empty(nb + 1, dtype=torch.int32, device=dev)
    D.moe_align_block_size(ids, nb, bs, sorted_ids, blocks, ntpp, cums, True)
    res = []
    for impl in (ref_ext, D):
        ends = torch.zeros(e + 1, dtype=torch.int32, device=dev)
        so = torch.full((n,), -5, dtype=torch.int64, device=dev)
        impl.build_ends_from_slots(sorted_ids, flat, ends, so, n, e)
        res.append((ends.cpu(), so.cpu()))
    (re_, rso), (me, mso) = res
    assert torch.equal(re_, me)
    for x in range(e):
        a, b = int(me[x]), int(me[x + 1])
        assert sorted(rso[a:b].tolist()) == sorted(mso[a:b].tolist())
    # ours is the stable order: ascending slots inside each segment
    for x in range(e):
        seg = mso[int(me[x]):int(me[x + 1])].numpy()
        assert np.all(np.diff(seg) > 0)


@pytest.mark.parametrize("t,k,h", [(1, 8, 2048), (256, 8, 2048), (37, 2, 4096), (64, 6, 512)])
def test_gather_hidden_matches_reference_extension(ref_ext, t, k, h):
    from exq_b200 import exq_dispatch_cuda as D
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(t + h)
    hidden = torch.randn(t, h, generator=g, device=dev).half()
    so = torch.randperm(t * k, generator=g, device=dev).to(torch.int64)
    outs = []
    for impl in (ref_ext, D):
        out = torch.full((t * k, h), float("nan"), dtype=torch.float16, device=dev)
        impl.gather_hidden(hidden, so, out, k)
        outs.append(out)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])


def _fp16_ulp(x: torch.Tensor) -> torch.Tensor:
    a = x.abs().float().clamp_min(2.0 ** -14)
    return torch.exp2(torch.floor(torch.log2(a)) - 10)


@pytest.mark.parametrize("t,k,h", [(1, 8, 2048), (256, 8, 2048), (100, 2, 4096), (3, 6, 512)])
def test_combine_matches_reference_extension(ref_ext, t, k, h):
    from exq_b200 import exq_dispatch_cuda as D
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(3 * t + k)
    n = t * k
    down = torch.randn(n, h, generator=g, device=dev).half()
    so = torch.randperm(n, generator=g, device=dev).to(torch.int64)
    w = torch.softmax(torch.randn(t, k, generator=g, device=dev), -1).half()
    outs = []
    for impl in (ref_ext, D):
        y = torch.full((t, h), float("nan"), dtype=torch.float16, device=dev)
        impl.combine(down, so, w, y)
        outs.append(y)
    torch.cuda.synchronize()
    ref, got = outs
    assert torch.isfinite(got).all()
    diff = (got.float() - ref.float()).abs()
    assert bool((diff <= _fp16_ulp(ref)).all()), float(diff.max())


@pytest.mark.parametrize("t,k,e", [(1, 8, 128), (7, 2, 8), (256, 8, 128), (4096, 2, 8)])
def test_align_matches_vllm_op(t, k, e):
    """sgl_kernel's align contract, cross-checked against vLLM's CUDA op of the
    same contract: per-expert padded ranges, the same slot set in each range,
    pad value ``numel`` inside ranges, block owners and the padded total."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    try:
        from vllm import _custom_ops as ops
        torch.ops._moe_C.moe_align_block_size  # noqa: B018 - registered by the import
    except Exception as ex:  # noqa: BLE001 - the reason is the skip message
        pytest.skip(f"vLLM's align op does not load: {type(ex).__name__}: {ex}")
    from exq_b200 import exq_dispatch_cuda as D
    dev = torch.device("cuda", 0)
    ids = _ids(t, k, e, 7 * t + e, zipf=True).to(dev).to(torch.int32)
    n = ids.numel()
    nb, bs = e + 1, 16
    cap = n + nb * (bs - 1)   # the reference backend's capacity (sglang_backend.py:102)
    nblk = (cap + bs - 1) // bs
    v_sorted = torch.full((cap,), -3, dtype=torch.int32, device=dev)
    v_blocks = torch.full((nblk,), -3, dtype=torch.int32, device=dev)
    v_ntpp = torch.empty(1, dtype=torch.int32, device=dev)
    ops.moe_align_block_size(ids, nb, bs, v_sorted, v_blocks, v_ntpp, None)
    m_sorted = torch.full((cap,), -3, dtype=torch.int32, device=dev)
    m_blocks = torch.full((nblk,), -3, dtype=torch.int32, device=dev)
    m_ntpp = torch.empty(1, dtype=torch.int32, device=dev)
    cums = torch.empty(nb + 1, dtype=torch.int32, device=dev)
    D.moe_align_block_size(ids, nb, bs, m_sorted, m_blocks, m_ntpp, cums, True)
    torch.cuda.synchronize()
    ntpp = int(m_ntpp.item())
    assert ntpp == int(v_ntpp.item())
    assert torch.equal(m_blocks[:ntpp // bs].cpu(), v_blocks[:ntpp // bs].cpu())
    vs, ms, c = v_sorted.cpu().numpy(), m_sorted.cpu().numpy(), cums.cpu().numpy()
    for x in range(nb):
        a, b = int(c[x]), int(c[x + 1])
        mv, vv = ms[a:b], vs[a:b]
        assert sorted(mv[mv < n].tolist()) == sorted(vv[vv < n].tolist())
        assert np.all(vv[vv >= n] == n) and np.all(mv[mv >= n] == n)
