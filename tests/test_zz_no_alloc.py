"""exq_combine_noalloc: the combine entry point whose scratch is a static
device array inside the library (no allocation per call).  It must give the
same result as exq_combine with a caller workspace, on consecutive calls.

This file sorts last so the GPU test also runs after every other test has
used the library on the same device.
"""
import ctypes as C

import pytest
import torch

from exq_b200 import _lib as L

MAX_ACTIVE = 262144   # EXQ_COMBINE_NOALLOC_MAX_ACTIVE


def _noalloc(d, order, w, result):
    t, k = w.shape
    L.check(L.lib().exq_combine_noalloc(L.ptr(d), L.tag(d), order.numel(), d.shape[1],
                                        L.ptr(order), L.ptr(w), L.tag(w), t, k, L.ptr(result),
                                        L.tag(result), L.stream_of(d.device)),
            "combine_noalloc")


def test_noalloc_rejects_sizes_beyond_static_scratch(lib_path):
    """The size check runs before any CUDA call, so no GPU is needed."""
    lib = L.lib()
    n = MAX_ACTIVE + 8
    rc = lib.exq_combine_noalloc(1, L.F16, n, 64, 1, 1, L.F32, n // 8, 8, 1, L.F16, None)
    assert rc == -1
    assert "static scratch of 262144 slots" in lib.exq_last_error().decode()


@pytest.mark.gpu
@pytest.mark.parametrize("t,k,h,out_dtype", [(37, 8, 512, torch.float16),
                                             (4096, 8, 256, torch.bfloat16),
                                             (MAX_ACTIVE // 8, 8, 64, torch.float16)])
def test_noalloc_matches_workspace_combine(cuda, t, k, h, out_dtype):
    from exq_b200 import exq_dispatch_cuda as D
    g = torch.Generator().manual_seed(t + k + h)
    n = t * k
    down = torch.randn(n, h, generator=g).to(cuda, torch.float16)
    order = torch.randperm(n, generator=g).to(cuda)
    w = torch.rand(t, k, generator=g).to(cuda)
    ref = torch.empty(t, h, dtype=out_dtype, device=cuda)
    D.combine(down, order, w, ref)
    L.read_device_status(cuda, clear=True)
    outs = []
    for _ in range(2):   # two calls in a row reuse the same static scratch
        y = torch.full((t, h), float("nan"), dtype=out_dtype, device=cuda)
        _noalloc(down, order, w, y)
        outs.append(y)
    torch.cuda.synchronize(cuda)
    assert L.read_device_status(cuda) == 0
    for y in outs:
        # tolerance: exact; both entry points run the same kernels
        torch.testing.assert_close(y, ref, rtol=0, atol=0)
