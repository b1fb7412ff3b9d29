"""The host-buffer entry points (mxq_linear_host, mxq_linear_pair_host):
results equal the device-pointer calls bit for bit on every call -- the first
(plain launches), the second (which records a CUDA graph) and the replays --
with fresh inputs each call; a workspace reallocation in between and a
destroyed / re-created weight must not leave a stale graph behind."""
import ctypes

import numpy as np
import pytest
import torch

from cpu_model_b200 import _lib, mx, synth

pytestmark = pytest.mark.gpu


def host_pair(ctx, w1, w2, x):
    y = np.empty((x.shape[0], w2.n), np.float32)
    x = np.ascontiguousarray(x, np.float32)
    ctx._bind()
    _lib.check(ctx.lib.mxq_linear_pair_host(ctx.h, w1.h, w2.h, ctypes.c_void_p(x.ctypes.data), x.shape[0],
                                            ctypes.c_void_p(y.ctypes.data)), ctx.h)
    return y


def host_linear(ctx, w, x):
    y = np.empty((x.shape[0], w.n), np.float32)
    x = np.ascontiguousarray(x, np.float32)
    ctx._bind()
    _lib.check(ctx.lib.mxq_linear_host(ctx.h, w.h, ctypes.c_void_p(x.ctypes.data), x.shape[0],
                                       ctypes.c_void_p(y.ctypes.data)), ctx.h)
    return y


def weight(ctx, fmt, n, k, seed):
    w, ws = synth.weights(fmt, n, k, -8, -3, seed)
    return mx.MXWeight(torch.from_numpy(w), torch.from_numpy(ws), fmt, n, k, ctx)


@pytest.mark.parametrize("fmt", [4, 8])
def test_host_calls_match_device_calls_across_replays(fmt):
    ctx = mx.MXContext(0)
    try:
        n, k = 992, 2048
        W1, W2 = weight(ctx, fmt, n, k, 1), weight(ctx, fmt, k, n, 2)
        for b in (1, 3, 40, 1):                  # GEMV and GEMM paths; b=1 again after a bigger batch
            for it in range(4):                  # plain, capture, replay, replay
                x = synth.normal((b, k), 100 * b + it)
                yp = host_pair(ctx, W1, W2, x)
                yl = host_linear(ctx, W1, x)
                xd = torch.from_numpy(x).cuda()
                ref_p = mx.mx_linear_pair(xd, W1, W2, ctx).cpu().numpy()
                ref_l = mx.mx_linear(xd, W1, ctx).cpu().numpy()
                ctx.synchronize()
                assert np.array_equal(yp, ref_p), (b, it)
                assert np.array_equal(yl, ref_l), (b, it)
        # a destroyed weight's replacement (new data, maybe the same address)
        W1.close()
        W3 = weight(ctx, fmt, n, k, 3)
        x = synth.normal((1, k), 7)
        y = host_pair(ctx, W3, W2, x)
        ref = mx.mx_linear_pair(torch.from_numpy(x).cuda(), W3, W2, ctx).cpu().numpy()
        ctx.synchronize()
        assert np.array_equal(y, ref)
        W2.close()
        W3.close()
    finally:
        ctx.close()
