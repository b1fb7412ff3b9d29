"""GPU edge cases through libmxq.so's C-ABI: the GAE ring buffer against the
reference's own ReplayMemory outputs (committed fixtures), the reference's AMI
MX fixture values as known answers, and the failure path of the bounded
device waits (a wait that runs out is reported, and the context stays usable).
"""
import os

import numpy as np
import pytest
import torch

from oracle import oracle
from cpu_model_b200 import mx, synth, _lib

pytestmark = pytest.mark.gpu

REL_TOL = 1e-5
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


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


def ring_cases():
    d = np.load(os.path.join(GOLD, "gae_ring_reference.npz"))
    n = len({f.split("_")[0] for f in d.files})
    for i in range(n):
        p = "c%d_" % i
        yield {k[len(p):]: d[k] for k in d.files if k.startswith(p)}


# ------------------------------------------------------------- GAE ring ---
def test_gae_ring_matches_reference(ctx):
    """mxq_gae_ring on the reference's own ring contents: wrapped rings, a
    sweep cut to what is stored, 1500 environments (only the first 1024
    written, as in agentic_env/replay_memory.cpp:216-222); bit-exact over the
    whole ring."""
    for c in ring_cases():
        cap, size, cur, t, e = (int(v) for v in c["meta"])
        adv = torch.zeros(cap, dtype=torch.float32, device="cuda")
        ret = torch.zeros(cap, dtype=torch.float32, device="cuda")
        mx.fused_compute_gae_ring(cuda(c["r"]), cuda(c["v"]), cuda(c["d"]), cuda(c["nv"]), size, cur, t, e,
                                  adv, ret, 0.99, 0.95, ctx)
        ctx.synchronize()
        assert np.array_equal(host(adv), c["adv"]), (cap, size, cur, t, e)
        assert np.array_equal(host(ret), c["ret"]), (cap, size, cur, t, e)


def test_gae_ring_rejects_inconsistent_ring(ctx):
    z = torch.zeros(16, dtype=torch.float32, device="cuda")
    d = torch.zeros(16, dtype=torch.uint8, device="cuda")
    with pytest.raises(ValueError):      # cursor beyond the capacity
        mx.fused_compute_gae_ring(z, z, d, z, 16, 16, 2, 2, z.clone(), z.clone(), ctx=ctx)
    with pytest.raises(ValueError):      # a ring that is not full keeps cursor == size
        mx.fused_compute_gae_ring(z, z, d, z, 8, 3, 2, 2, z.clone(), z.clone(), ctx=ctx)
    ctx.synchronize()


def test_gae_linear_wide_envs(ctx):
    """mxq_gae over 1500 environments: the first 1024 equal the reference's
    output bit for bit; the reference stops at its MAX_ENVS and leaves the
    others at zero, where this entry point computes them (checked against
    the oracle)."""
    c = [c for c in ring_cases() if int(c["meta"][4]) > 1024][0]
    cap, size, cur, t, e = (int(v) for v in c["meta"])
    assert cur == 0 and size == cap == t * e          # the ring is exactly [T][E]
    r, v, d = (c[k].reshape(t, e) for k in ("r", "v", "d"))
    a, rt = mx.fused_compute_gae(cuda(r), cuda(v), cuda(d), cuda(c["nv"]), 0.99, 0.95, ctx)
    a, rt = host(a), host(rt)
    ref_a, ref_r = c["adv"].reshape(t, e), c["ret"].reshape(t, e)
    assert np.array_equal(a[:, :1024], ref_a[:, :1024]) and np.array_equal(rt[:, :1024], ref_r[:, :1024])
    o_a, o_r = oracle.gae(r, v, d, c["nv"], 0.99, 0.95)
    assert np.array_equal(a, o_a) and np.array_equal(rt, o_r)


# ------------------------------------------------------ AMI MX fixture ---
@pytest.mark.parametrize("seed", [0, 5, 126, 200])
def test_reference_ami_fixture_known_answers(ctx, seed):
    """The reference AMI harness's MX arguments (nn/tests/autotest.hpp:93-116):
    weights memset to seed % 127, weight and activation scale bytes 1,
    activation bytes 128 (q = 0), w_sums 0, at D = 1024.  Every per-block dot
    is 0 and so is every output; with activation bytes 129 (q = 1) each dot
    is 32 * (seed % 127) exactly, and the outputs, scaled by 2^(1-127) twice,
    are still 0 in fp32.  The 16-pointer form (:126-136) gives 16 zeros."""
    D = 1024
    wv = seed % 127
    w = np.full((D, D), wv, np.int8)
    ws = np.ones((D, D // 32), np.uint8)
    W = mx.MXWeight(torch.from_numpy(w), torch.from_numpy(ws), 8, D, D, ctx)
    for qbyte, dot in ((128, 0), (129, 32 * wv)):
        xq = np.full((1, D), qbyte, np.uint8)
        xs = np.ones((1, D // 32), np.uint8)
        a = mx.MXActivation(cuda(xq), cuda(xs))
        dots = host(mx.mx_block_dots(a, W, ctx))
        assert np.all(dots == dot)
        assert np.array_equal(oracle.block_dots(8, xq, w, D, D), dots)
        y = host(mx.mx_gemv(a, W, ctx))
        assert np.all(y == 0.0) and np.array_equal(y, oracle.gemv(8, xq, xs, w, ws, D, D))
        rows = cuda(np.arange(16, dtype=np.int32))
        y16 = host(mx.mx_rank16_dot_ptrs(a, W, rows, ctx))
        assert y16.shape == (1, 16) and np.all(y16 == 0.0)
    ctx.synchronize()
    W.close()


# ------------------------------------------------- bounded-wait failure ---
@pytest.mark.parametrize("fmt,n,k,b,sparse", [(8, 256, 512, 48, False), (4, 384, 1024, 200, False),
                                               (4, 256, 1024, 200, True)])
def test_bounded_wait_timeout_is_reported_and_context_recovers(ctx, fmt, n, k, b, sparse):
    """The tensor-core linear with its first activation copy withheld and a
    2 ms wait limit (mxq_debug_gemm_stall): its bounded waits run out, the
    kernel drains what it started and returns, the call reports
    MXQ_ERR_TIMEOUT, and the next calls on the same context are correct.
    The block-sparse case runs one row tile per CTA with two converter groups
    whose first k-tiles sit in different activation chunks, so one group
    issues MMAs before the other's wait runs out (the MMA drain path)."""
    w, ws = synth.weights(fmt, n, k, -8, -3, 31 + k)
    mask = np.ones(((n + 63) // 64, k // 64), np.uint8) if sparse else None
    W = mx.MXWeight(torch.from_numpy(w), torch.from_numpy(ws), fmt, n, k, ctx, block_mask=mask)
    x = synth.normal((b, k), 32 + b)
    xd = cuda(x)
    y = torch.empty((b, n), dtype=torch.float32, device="cuda")
    ctx._bind()
    rc = ctx.lib.mxq_debug_gemm_stall(ctx.h, W.h, mx._ptr(xd), b, mx._ptr(y), 2000)
    assert rc == _lib.MXQ_ERR_TIMEOUT, rc
    assert b"bounded wait" in ctx.lib.mxq_last_error(ctx.h)
    ctx.synchronize()                       # the status word was cleared
    xq, xs = oracle.quantize_x(x)
    ref = oracle.gemv(fmt, xq, xs, w, ws, n, k)
    for path in (mx.PATH_GEMM, mx.PATH_AUTO):
        ctx.set_path(path)
        try:
            y2 = host(mx.mx_linear(xd, W, ctx))
        finally:
            ctx.set_path(mx.PATH_AUTO)
        ctx.synchronize()
        assert rel_l2(y2, ref) <= REL_TOL
    with pytest.raises(ValueError):          # the limit is bounded on the host
        mx.check(ctx.lib.mxq_debug_gemm_stall(ctx.h, W.h, mx._ptr(xd), b, mx._ptr(y), 0), ctx.h)
    W.close()
