"""mxq_linear_noalloc: the tensor-core linear for callers that may not
allocate device memory (an engine whose device memory belongs to its own pool
allocator, or a serving loop held to a no-allocation rule).  Its operand
scratch is a fixed 4 MiB array inside libmxq.so instead of the context
workspace.

The test calls it through the C-ABI twice in a row (the second call reuses
whatever the first left in the shared array) and checks both results against
the existing entry point, mxq_linear on the tensor-core path, within the
parity tolerance the other GPU tests use.  It creates its own context, so it
runs the same alone in a fresh process or after the rest of the suite (this
file is named to be collected last).
"""
import ctypes

import numpy as np
import pytest
import torch

from cpu_model_b200 import _lib, mx, synth

pytestmark = pytest.mark.gpu

REL_TOL = 1e-5


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300)


def noalloc(ctx, w, x):
    y = torch.empty((x.shape[0], w.n), dtype=torch.float32, device=x.device)
    ctx._bind()
    rc = ctx.lib.mxq_linear_noalloc(ctx.h, w.h, ctypes.c_void_p(x.data_ptr()), x.shape[0],
                                    ctypes.c_void_p(y.data_ptr()))
    _lib.check(rc, ctx.h)
    return y


@pytest.mark.parametrize("fmt,n,k,b", [(4, 384, 4096, 40), (8, 300, 2048, 130), (4, 1000, 11008, 9)])
def test_linear_noalloc_matches_linear(fmt, n, k, b):
    ctx = mx.MXContext(0)
    try:
        w, ws = synth.weights(fmt, n, k, -10, -4, 7 + n)
        W = mx.MXWeight(torch.from_numpy(w), torch.from_numpy(ws), fmt, n, k, ctx)
        x = torch.from_numpy(synth.normal((b, k), 11 + b)).cuda()
        ctx.set_path(mx.PATH_GEMM)
        ref = mx.mx_linear(x, W, ctx)
        ctx.set_path(mx.PATH_AUTO)
        y1 = noalloc(ctx, W, x)
        y2 = noalloc(ctx, W, x)
        ctx.synchronize()
        ref, y1, y2 = ref.cpu().numpy(), y1.cpu().numpy(), y2.cpu().numpy()
        assert rel_l2(y1, ref) <= REL_TOL
        assert rel_l2(y2, ref) <= REL_TOL
        W.close()
    finally:
        ctx.close()


def test_linear_noalloc_rejects_oversize():
    ctx = mx.MXContext(0)
    try:
        w, ws = synth.weights(8, 64, 8192, -10, -4, 3)
        W = mx.MXWeight(torch.from_numpy(w), torch.from_numpy(ws), 8, 64, 8192, ctx)
        x = torch.zeros((512, 8192), dtype=torch.float32, device="cuda")   # 8 MiB of operand > 4 MiB
        with pytest.raises(ValueError):
            noalloc(ctx, W, x)
        W.close()
    finally:
        ctx.close()
