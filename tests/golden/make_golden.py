"""Generate the golden fixtures under tests/golden/ from the reference itself.

Run in a container that has the reference checkout (read-only), with
``$EXQ_REFERENCE`` set to its directory:

    EXQ_REFERENCE=<reference checkout> python tests/golden/make_golden.py

The reference's Python modules are loaded by file path (``exq/__init__.py``
imports a Rust extension that is not built here), its ``@triton.jit`` kernels
run on the CPU under ``TRITON_INTERPRET=1``, and every fixture is written as a
small ``.npz`` (inputs and reference outputs).  Seeds are fixed below, so a
re-run reproduces the same files.  Nothing at test time reads the reference.

Fixtures
  pack_int4.npz      pack_int4_weights on assorted shapes / dtypes / edge cases
                     (moe_int4_kernel.py:37-93), incl. K < group and all-zero rows
  quant_shim.npz     quantize_tensor_int8 / quantize_tensor_int4 outputs
                     (exq/eval/quant_shim.py:84-125)
  int4_gemm_*.npz    _moe_gemm_int4_kernel output in expert-sorted order
                     (moe_int4_kernel.py:124-240) with the reference's own sort
                     (moe_grouped_gemm.py:139-166)
  fp16_gemm.npz      _moe_gemm_kernel output (moe_grouped_gemm.py:47-132)
  layer_int4.npz     gate_up -> silu*mul -> down -> top-k combine composed from the
                     reference's Triton kernel and torch combine (moe_int4_kernel.py
                     :374-426, with the undefined ``top_k`` at :424 taken as
                     router_indices.shape[1])
  routing.npz        sort_tokens_by_expert / unsort_output / pytorch_moe_reference
"""
from __future__ import annotations

import importlib.util
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

if "EXQ_REFERENCE" not in os.environ:
    sys.exit("set EXQ_REFERENCE to the reference checkout's directory")
REF = Path(os.environ["EXQ_REFERENCE"])
OUT = Path(__file__).resolve().parent


def _load(name: str, rel: str):
    spec = importlib.util.spec_from_file_location(name, REF / rel)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def _np(t: torch.Tensor):
    if t.dtype == torch.bfloat16:
        return t.float().numpy()
    return t.numpy()


def _sort(router_indices: torch.Tensor, hidden: torch.Tensor, n_experts: int):
    """The reference's sort_tokens_by_expert (moe_grouped_gemm.py:139-166) on CPU.

    The reference hard-codes device="cuda" for ``expert_ends``; the calls are
    otherwise identical.
    """
    top_k = router_indices.shape[1]
    flat = router_indices.reshape(-1).long()
    sort_order = torch.argsort(flat, stable=True)
    sorted_ids = flat[sort_order]
    sorted_hidden = hidden[(sort_order // top_k).long()]
    counts = torch.bincount(sorted_ids, minlength=n_experts)
    ends = torch.zeros(n_experts + 1, dtype=torch.int32)
    ends[1:] = counts.cumsum(0).int()
    max_tok = int(counts.max().item()) if flat.numel() > 0 else 1
    return sort_order, sorted_hidden, ends, max_tok


def _int4_gemm(kmod, sorted_h, packed, scales, ends, n, k, max_tok, n_experts, gs=128):
    out = torch.zeros(sorted_h.shape[0], n, dtype=torch.float16)
    bm, bn = 64, 128
    grid = (n_experts, max((max_tok + bm - 1) // bm, 1), (n + bn - 1) // bn)
    kmod._moe_gemm_int4_kernel[grid](
        sorted_h, packed, scales, out, ends, N=n, K=k,
        stride_am=sorted_h.stride(0), stride_be=packed.stride(0), stride_bn=packed.stride(1),
        stride_se=scales.stride(0), stride_sn=scales.stride(1), stride_cm=out.stride(0),
        BLOCK_M=bm, BLOCK_N=bn, BLOCK_K=32, GROUP_SIZE=gs)
    return out


def make_pack(kmod):
    g = torch.Generator().manual_seed(1234)
    cases = {}
    shapes = [((64, 256), torch.float16, 0.02, 128), ((32, 384), torch.float16, 1.0, 128),
              ((16, 64), torch.float16, 0.02, 128), ((8, 256), torch.float32, 0.5, 64),
              ((24, 1024), torch.float16, 0.02, 128)]
    for i, (shape, dt, std, gs) in enumerate(shapes):
        w = (torch.randn(*shape, generator=g) * std).to(dt)
        p, s = kmod.pack_int4_weights(w, group_size=gs)
        cases[f"w{i}"] = _np(w)
        cases[f"gs{i}"] = np.array(gs)
        cases[f"packed{i}"] = _np(p)
        cases[f"scales{i}"] = _np(s)
    # edge cases: all-zero rows (eps clamp), one row of exact multiples of scale/2
    w = torch.zeros(4, 128, dtype=torch.float16)
    w[1] = torch.linspace(-1, 1, 128).half()
    w[2, ::2] = 7.0
    w[2, 1::2] = -0.5
    w[3] = torch.tensor([(j % 15 - 7) * 0.5 for j in range(128)]).half()
    p, s = kmod.pack_int4_weights(w)
    cases["w_edge"], cases["packed_edge"], cases["scales_edge"] = _np(w), _np(p), _np(s)
    np.savez_compressed(OUT / "pack_int4.npz", **cases)


def make_quant_shim(qmod):
    g = torch.Generator().manual_seed(99)
    w = (torch.randn(32, 256, generator=g) * 0.02).half()
    z = torch.zeros(4, 128, dtype=torch.float16)
    np.savez_compressed(OUT / "quant_shim.npz", w=_np(w), int8=_np(qmod.quantize_tensor_int8(w)),
                        int4=_np(qmod.quantize_tensor_int4(w)), zero=_np(z),
                        zero_int8=_np(qmod.quantize_tensor_int8(z)),
                        zero_int4=_np(qmod.quantize_tensor_int4(z)))


def make_int4_gemm(kmod, name, e, n, k, t, topk, seed):
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(e, n, k, generator=g) * 0.02).half()
    packed, scales = kmod.pack_experts_int4(w)
    hidden = torch.randn(t, k, generator=g).half()
    ids = torch.randint(0, e, (t, topk), generator=g)
    so, sh, ends, mt = _sort(ids, hidden, e)
    out = _int4_gemm(kmod, sh, packed, scales, ends, n, k, mt, e)
    np.savez_compressed(OUT / f"int4_gemm_{name}.npz", hidden=_np(hidden), ids=_np(ids),
                        packed=_np(packed), scales=_np(scales), sort_order=_np(so),
                        ends=_np(ends), out=_np(out), n_experts=np.array(e))


def make_fp16_gemm(gmod):
    g = torch.Generator().manual_seed(77)
    e, n, k, t, topk = 4, 128, 256, 6, 2
    w = (torch.randn(e, n, k, generator=g) * 0.05).half()
    hidden = torch.randn(t, k, generator=g).half()
    ids = torch.randint(0, e, (t, topk), generator=g)
    so, sh, ends, mt = _sort(ids, hidden, e)
    out = torch.zeros(t * topk, n, dtype=torch.float16)
    grid = (e, max((mt + 63) // 64, 1), (n + 63) // 64)
    gmod._moe_gemm_kernel[grid](sh, w, out, ends, N=n, K=k, stride_am=sh.stride(0),
                                stride_be=w.stride(0), stride_bn=w.stride(1),
                                stride_cm=out.stride(0), BLOCK_M=64, BLOCK_N=64, BLOCK_K=32,
                                expert_mask_ptr=0, USE_EXPERT_MASK=False)
    np.savez_compressed(OUT / "fp16_gemm.npz", hidden=_np(hidden), ids=_np(ids), w=_np(w),
                        out=_np(out))


def make_layer(kmod):
    g = torch.Generator().manual_seed(4242)
    e, h, inter, t, topk = 4, 256, 256, 6, 2
    w13 = (torch.randn(e, 2 * inter, h, generator=g) * 0.02).half()
    w2 = (torch.randn(e, h, inter, generator=g) * 0.02).half()
    hidden = torch.randn(t, h, generator=g).half()
    ids = torch.randint(0, e, (t, topk), generator=g)
    wts = torch.softmax(torch.randn(t, topk, generator=g), dim=-1).half()
    p13, s13 = kmod.pack_experts_int4(w13)
    p2, s2 = kmod.pack_experts_int4(w2)
    so, sh, ends, mt = _sort(ids, hidden, e)
    unsort = torch.argsort(so, stable=True)
    out1 = _int4_gemm(kmod, sh, p13, s13, ends, 2 * inter, h, mt, e)
    g_, u_ = out1.float()[:, :inter], out1.float()[:, inter:]
    mid = (g_ / (1 + torch.exp(-g_)) * u_).half()   # sgl_kernel silu_and_mul contract
    out2 = _int4_gemm(kmod, mid, p2, s2, ends, h, inter, mt, e)
    y = (out2[unsort].view(t, topk, h) * wts.unsqueeze(-1).to(out2.dtype)).sum(dim=1)
    np.savez_compressed(OUT / "layer_int4.npz", hidden=_np(hidden), ids=_np(ids), wts=_np(wts),
                        p13=_np(p13), s13=_np(s13), p2=_np(p2),
                        s2=_np(s2), gate_up=_np(out1), mid=_np(mid), down=_np(out2), y=_np(y))


def make_routing(gmod):
    g = torch.Generator().manual_seed(5)
    cases = {}
    for i, (t, topk, e) in enumerate([(7, 2, 4), (33, 8, 16), (1, 8, 128), (64, 6, 64)]):
        ids = torch.randint(0, e, (t, topk), generator=g)
        hidden = torch.randn(t, 8, generator=g).half()
        so, sh, ends, mt = _sort(ids, hidden, e)
        wts = torch.softmax(torch.randn(t, topk, generator=g), dim=-1)
        rows = torch.randn(t * topk, 8, generator=g)
        un = gmod.unsort_output(rows, ids, wts)
        cases.update({f"ids{i}": _np(ids), f"e{i}": np.array(e), f"sort_order{i}": _np(so),
                      f"ends{i}": _np(ends), f"max_tok{i}": np.array(mt), f"wts{i}": _np(wts),
                      f"rows{i}": _np(rows), f"unsort{i}": _np(un)})
    # naive per-token oracle of the reference (moe_grouped_gemm.py:267-290)
    ids = torch.randint(0, 4, (5, 2), generator=g)
    x = torch.randn(5, 32, generator=g)
    w = torch.randn(4, 16, 32, generator=g)
    rw = torch.softmax(torch.randn(5, 2, generator=g), dim=-1)
    ref = gmod.pytorch_moe_reference(x, w, ids, rw)
    cases.update({"naive_ids": _np(ids), "naive_x": _np(x), "naive_w": _np(w),
                  "naive_rw": _np(rw), "naive_out": _np(ref)})
    np.savez_compressed(OUT / "routing.npz", **cases)


def main():
    kmod = _load("_ref_moe_int4_kernel", "exq/kernels/moe_int4_kernel.py")
    gmod = _load("_ref_moe_grouped_gemm", "exq/kernels/moe_grouped_gemm.py")
    qmod = _load("_ref_quant_shim", "exq/eval/quant_shim.py")
    make_pack(kmod)
    make_quant_shim(qmod)
    make_int4_gemm(kmod, "small", 4, 256, 256, 5, 2, 11)
    make_int4_gemm(kmod, "wide", 6, 256, 384, 9, 3, 12)
    make_fp16_gemm(gmod)
    make_layer(kmod)
    make_routing(gmod)
    for f in sorted(OUT.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
