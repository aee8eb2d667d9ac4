"""exq_b200: the quantized MoE expert path of alityb/exq, rebuilt for B200 (sm_100a).

The public names mirror ``exq.kernels`` (exq/kernels/__init__.py:1-21); the
``exq_dispatch_cuda`` module mirrors the reference's CUDA extension; the
``sglang_backend`` module mirrors exq/runtime/sglang_backend.py.  All compute
runs in ``_lib/libexq_b200.so`` through the C ABI in ``include/exq_b200.h``.
"""
from .kernels import (  # noqa: F401
    ExpertProfile,
    load_exq_artifact,
    moe_grouped_gemm,
    moe_int4_forward,
    moe_int4_full_forward,
    pack_experts_int4,
    pack_int4_weights,
    router_topk,
    sort_tokens_by_expert,
    unsort_output,
)
from .experts import ExpertBank  # noqa: F401

__all__ = [
    "router_topk",
    "moe_grouped_gemm",
    "sort_tokens_by_expert",
    "moe_int4_forward",
    "moe_int4_full_forward",
    "pack_experts_int4",
    "pack_int4_weights",
    "load_exq_artifact",
    "ExpertProfile",
    "unsort_output",
    "ExpertBank",
]
