"""GPU parity of the operators around the MX linear layer, through libmxq.so's
C-ABI, against the CPU oracle on the same seeded inputs:

- mx_quantize_w (nn/tests/test_auto_generated.cpp:46): bytes, scales and
  w_sums bit-exact;
- mx_rank16_dot_ptrs in the reference's pointer-array form
  (nn/tests/autotest.hpp:126-136): bit-exact against the oracle's
  restatement of the kernel's summation order, and within 1e-5 of the
  exactly rounded dot;
- halting_step (nn/core/layers/halting.hpp:24-30): probabilities and ACT
  state bit-exact over several steps;
- HashedRouter::route (nn/tests/test_robustness.cpp:13-35): ids and scores
  bit-exact, the N = 31, K = 2 remainder case, the K > N error.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle
from cpu_model_b200 import mx, synth, _lib

pytestmark = pytest.mark.gpu

REL_TOL = 1e-5


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.linalg.norm(b)
    return np.linalg.norm(a - b) / (den if den > 0 else 1.0)


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def edge_weights(n, k, seed):
    w = synth.normal((n, k), seed) * np.float32(0.05)
    w[0, :32] = 0.0                                 # all-zero block
    w[1, 32:64] *= np.float32(1e-36)                # tiny block (exponent clamp)
    w[2, 0] = np.nan                                # non-finite blocks
    w[2, 40] = np.inf
    w[3, :32] = np.float32(0.5) * np.arange(-16, 16, dtype=np.float32) * np.float32(2.0 ** -4)   # ties
    w[4, 64:96] *= np.float32(1e30)                 # large block
    return w


# ---------------------------------------------------------- quantize_w ---
@pytest.mark.parametrize("fmt", [8, 4])
@pytest.mark.parametrize("n,k", [(8, 128), (300, 4096), (64, 11008)])
def test_quantize_w_bit_exact(ctx, fmt, n, k):
    w = edge_weights(n, k, 5 + n)
    d0, s0, z0 = oracle.quantize_w(fmt, w)
    d1, s1, z1 = mx.mx_quantize_w(cuda(w), fmt, ctx)
    ctx.synchronize()
    assert np.array_equal(host(s1), s0)
    assert np.array_equal(host(d1).view(d0.dtype), d0)
    assert np.array_equal(host(z1), z0)
    # the quantised weight runs through the linear like the oracle's bytes
    if n >= 64:
        W = mx.MXWeight(d1, s1, fmt, n, k, ctx)
        x = synth.normal((3, k), 9)
        xq, xs = oracle.quantize_x(x)
        ref = oracle.gemv(fmt, xq, xs, d0, s0, n, k)
        y = host(mx.mx_linear(cuda(x), W, ctx))
        ctx.synchronize()
        fin = np.isfinite(ref).all(0)
        assert rel_l2(y[:, fin], ref[:, fin]) <= REL_TOL
        W.close()


# ---------------------------------------------------- rank16_dot_ptrs ---
@pytest.mark.parametrize("fmt", [8, 4])
@pytest.mark.parametrize("k,b,nrows", [(1024, 1, 16), (4096, 3, 16), (2048, 2, 64), (96, 5, 7)])
def test_rank16_dot_ptrs_pointer_form(ctx, fmt, k, b, nrows):
    rows, scs, handles = [], [], []
    for j in range(nrows):
        w, ws = synth.weights(fmt, 1, k, -10, -4, 500 + j)
        rows.append(w)
        scs.append(ws)
        handles.append(mx.MXWeight(torch.from_numpy(w), torch.from_numpy(ws), fmt, 1, k, ctx))
    x = synth.normal((b, k), 77)
    xq, xs = oracle.quantize_x(x)
    a = mx.MXActivation(cuda(xq), cuda(xs))
    y = host(mx.mx_rank16_dot_ptrs(a, handles, ctx=ctx))
    ctx.synchronize()
    assert np.array_equal(y, oracle.rank16_dot_ptrs(fmt, xq, xs, rows, scs, k))
    ref = np.concatenate([oracle.gemv(fmt, xq, xs, rows[j], scs[j], 1, k) for j in range(nrows)], axis=1)
    assert rel_l2(y, ref) <= REL_TOL
    for h in handles:
        h.close()


def test_rank16_dot_ptrs_rejects_mixed_and_too_many(ctx):
    w8, s8 = synth.weights(8, 1, 128, -8, -3, 1)
    w4, s4 = synth.weights(4, 1, 128, -8, -3, 2)
    h8 = mx.MXWeight(torch.from_numpy(w8), torch.from_numpy(s8), 8, 1, 128, ctx)
    h4 = mx.MXWeight(torch.from_numpy(w4), torch.from_numpy(s4), 4, 1, 128, ctx)
    a = mx.mx_quantize_x(cuda(synth.normal((1, 128), 3)), ctx)
    with pytest.raises(ValueError):
        mx.mx_rank16_dot_ptrs(a, [h8, h4], ctx=ctx)
    with pytest.raises(ValueError):
        mx.mx_rank16_dot_ptrs(a, [h8] * 65, ctx=ctx)
    ctx.synchronize()
    h8.close()
    h4.close()


# --------------------------------------------------------- halting_step ---
@pytest.mark.parametrize("fmt", [8, 4])
def test_halting_step_bit_exact(ctx, fmt):
    k, b = 2048, 37
    w, ws = synth.weights(fmt, 1, k, -9, -6, 42)
    W = mx.MXWeight(torch.from_numpy(w), torch.from_numpy(ws), fmt, 1, k, ctx)
    state = mx.HaltingState(b)
    p_sum = np.zeros(b, np.float32)
    rem = np.zeros(b, np.float32)
    steps = np.zeros(b, np.uint64)
    halted_any = False
    for step in range(6):
        x = synth.normal((b, k), 100 + step)
        xq, xs = oracle.quantize_x(x)
        p1, h1 = mx.halting_step(mx.MXActivation(cuda(xq), cuda(xs)), W, -1.0, state, ctx)
        p0, h0 = oracle.halting_step(fmt, xq, xs, w, ws, k, -1.0, p_sum, rem, steps)
        assert np.array_equal(host(p1), p0)
        assert np.array_equal(host(h1), h0)
        assert np.array_equal(host(state.p_sum), p_sum) and np.array_equal(host(state.remainder), rem)
        assert np.array_equal(host(state.steps).astype(np.uint64), steps)
        halted_any |= bool(h0.any())
    assert halted_any
    ctx.synchronize()
    W.close()


def test_halting_step_rejects_multi_row(ctx):
    w, ws = synth.weights(8, 2, 64, -8, -3, 1)
    W = mx.MXWeight(torch.from_numpy(w), torch.from_numpy(ws), 8, 2, 64, ctx)
    a = mx.mx_quantize_x(cuda(synth.normal((1, 64), 2)), ctx)
    with pytest.raises(ValueError):
        mx.halting_step(a, W, 0.0, mx.HaltingState(1), ctx)
    ctx.synchronize()
    W.close()


# -------------------------------------------------------- HashedRouter ---
@pytest.mark.parametrize("t,d,e,k,h,seed", [(1, 1024, 31, 2, 8, 0), (64, 4096, 8, 2, 8, 7),
                                             (33, 2048, 1024, 16, 16, 3), (5, 96, 4, 4, 32, 11)])
def test_hashed_router_bit_exact(ctx, t, d, e, k, h, seed):
    x = synth.normal((t, d), 200 + t)
    if t > 2:
        x[1, :32] = 0.0
        x[2, 32:64] *= np.float32(1e-37)
    r = mx.HashedRouter(d, e, k, h, seed)
    idx, sc = r.route(cuda(x), ctx)
    i0, s0 = oracle.hashed_route(x, e, k, h, seed)
    assert np.array_equal(host(idx), i0) and np.array_equal(host(sc), s0)
    assert np.all(host(idx) >= 0) and np.all(host(idx) < e)
    for row in host(idx):
        assert len(set(row.tolist())) == k
    # the host-buffer form (the reference's call passes host memory)
    ih = np.empty((t, k), np.int32)
    sh = np.empty((t, k), np.int32)
    mx.check(ctx.lib.mxq_hashed_route_host(ctx.h, x.ctypes.data_as(ctypes.c_void_p), t, d, e, k, h, seed,
                                           ih.ctypes.data_as(ctypes.c_void_p), sh.ctypes.data_as(ctypes.c_void_p)),
             ctx.h)
    assert np.array_equal(ih, i0) and np.array_equal(sh, s0)


def test_hashed_router_remainder_and_bounds(ctx):
    """nn/tests/test_robustness.cpp:13-35: N = 31, K = 2 on x = 1 (d = 1024)
    yields two indices; K > N is an invalid argument."""
    r = mx.HashedRouter(1024, 31, 2, 8)
    idx, _ = r.route(torch.ones((1, 1024), dtype=torch.float32, device="cuda"), ctx)
    assert host(idx).shape == (1, 2)
    with pytest.raises(ValueError):
        mx.HashedRouter(1024, 10, 20, 8)
    out = torch.empty((1, 20), dtype=torch.int32, device="cuda")
    rc = ctx.lib.mxq_hashed_route(ctx.h, mx._ptr(torch.ones((1, 1024), device="cuda")), 1, 1024, 10, 20, 8, 0,
                                  mx._ptr(out), mx._ptr(out))
    assert rc == _lib.MXQ_ERR_INVALID_ARGUMENT
    ctx.synchronize()


# ------------------------------------------- online update / activation norm ---
@pytest.mark.parametrize("fmt,n,k", [(8, 200, 448), (4, 130, 1024)])
def test_update_gaussian_moment_bit_exact(ctx, fmt, n, k):
    """mx_update_gaussian_moment against the oracle: the tiled device weight,
    read back, equals the oracle's update of the MXINT8Tensor bytes; a large
    step saturates at the range ends."""
    w, ws = synth.weights(fmt, n, k, -9, -5, 90 + k)
    ws[3, 2] = 255                                      # a NaN block stays as it is
    W = mx.MXWeight(torch.from_numpy(w), torch.from_numpy(ws), fmt, n, k, ctx)
    g = synth.normal((n,), 91)
    x = synth.normal((k,), 92)
    cur = w
    for step in (0.37, -1e3):
        mx.mx_update_gaussian_moment(W, cuda(g), cuda(x), step, ctx)
        ctx.synchronize()
        cur = oracle.update_gaussian_moment(fmt, cur, ws, g, x, step)
        d, s = W.download()
        assert np.array_equal(d, cur) and np.array_equal(s, ws)
    vals = synth.unpack_int4(cur) if fmt == 4 else cur
    assert vals.min() == (-8 if fmt == 4 else -127) and vals.max() == (7 if fmt == 4 else 127)
    W.close()


@pytest.mark.parametrize("b,k", [(1, 32), (5, 4096), (3, 11008)])
def test_activation_norm_bit_exact(ctx, b, k):
    x = synth.normal((b, k), 93 + k)
    if k >= 64:
        x[0, 32:64] = 0.0
    xq, xs = oracle.quantize_x(x)
    nrm = host(mx.mx_compute_activation_norm(mx.MXActivation(cuda(xq), cuda(xs)), ctx))
    assert np.array_equal(nrm, oracle.activation_norm(xq, xs))
    deq = (xq.astype(np.float64) - 128) * np.exp2(xs.astype(np.float64) - 127).repeat(32, axis=1)
    assert np.allclose(nrm, np.linalg.norm(deq, axis=1), rtol=1e-6)


# ---------------------------------------------------- micro-expert pool ---
@pytest.mark.parametrize("fmt,router", [(4, "logits"), (8, "hashed")])
def test_micro_moe_reference_shape_bit_exact(ctx, fmt, router):
    """The reference's expert pool shape (nn/config/model_config.hpp:23-25):
    1024 routed 16-row experts, top-16, 2 shared, d 2048; routing by softmax
    top-k over logits or by the LSH HashedRouter (unit weights).  The layer is
    bit-identical to the oracle's restatement of its operation order."""
    E, S, D, K, T = 1024, 2, 2048, 16, 24
    wg, sg = synth.weights(fmt, (E + S) * 16, D, -9, -6, 71)
    wu, su = synth.weights(fmt, (E + S) * 16, D, -9, -6, 72)
    wd, sd = synth.weights(fmt, D, (E + S) * 16, -9, -6, 73)
    Wg, Wu, Wd = (mx.MXWeight(torch.from_numpy(a), torch.from_numpy(b), fmt, n, k, ctx)
                  for a, b, n, k in ((wg, sg, (E + S) * 16, D), (wu, su, (E + S) * 16, D), (wd, sd, D, (E + S) * 16)))
    x = synth.normal((T, D), 74)
    if router == "logits":
        logits = synth.normal((T, E), 75)
        idx_d, gate_d = mx.route_topk(cuda(logits), K, ctx)
        i0, g0 = oracle.route_topk(logits, K)
        assert np.array_equal(host(idx_d), i0) and np.array_equal(host(gate_d), g0)
    else:
        idx_d, _ = mx.HashedRouter(D, E, K, 16, seed=5).route(cuda(x), ctx)
        gate_d, g0 = None, None
        i0, _ = oracle.hashed_route(x, E, K, 16, 5)
        assert np.array_equal(host(idx_d), i0)
    y = host(mx.micro_moe(cuda(x), Wg, Wu, Wd, E, S, idx_d, gate_d, ctx))
    ctx.synchronize()
    ref = oracle.micro_moe(fmt, wg, sg, wu, su, wd, sd, E, S, x, i0, g0)
    assert np.all(np.isfinite(y)) and np.linalg.norm(y) > 0
    assert np.array_equal(y, ref)
    with pytest.raises(ValueError):                       # top-k beyond the pool
        mx.micro_moe(cuda(x), Wg, Wu, Wd, 8, E + S - 8, cuda(np.zeros((T, 9), np.int32)), None, ctx)
    ctx.synchronize()
    for W in (Wg, Wu, Wd):
        W.close()
