"""GPU parity for the block-sparse weights and the mixture-of-experts layer,
through libmxq.so's C-ABI, against the CPU oracle on the same seeded inputs.

Block-sparse weights are checked against the oracle's dense GEMV on the same
data with the masked-out 64x64 blocks zeroed; the MoE layer against the
oracle's mxo_moe (routing, per-expert SwiGLU MLP, fp64 combine).  fp32
outputs within relative L2 <= 1e-5; routing-dependent results are identical
across repeated calls.
"""
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


def bsr_weight(ctx, fmt, n, k, density, seed, emin=-8, emax=-3):
    w, ws = synth.weights(fmt, n, k, emin, emax, seed)
    mask = synth.block_mask(n, k, density, seed + 1000)
    W = mx.MXWeight(torch.from_numpy(w), torch.from_numpy(ws), fmt, n, k, ctx, block_mask=mask)
    return synth.apply_block_mask(fmt, w, mask), ws, mask, W


@pytest.mark.parametrize("fmt", [4, 8])
@pytest.mark.parametrize("n,k,b,density", [
    (384, 1024, 40, 0.25),     # typical
    (200, 2048, 9, 0.25),      # rows not a multiple of 64/128; small token tile
    (256, 4096, 300, 0.25),    # two token tiles of 256; few row tiles -> K split
    (512, 512, 64, 1.0),       # every block present (equals the dense weight)
    (256, 1024, 17, 0.05),     # very sparse: some row tiles store no tile at all
])
def test_bsr_linear_matches_masked_dense(ctx, fmt, n, k, b, density):
    wm, ws, mask, W = bsr_weight(ctx, fmt, n, k, density, 7 + n + k)
    x = synth.normal((b, k), 11 + b)
    xq, xs = oracle.quantize_x(x)
    ref = oracle.gemv(fmt, xq, xs, wm, ws, n, k)
    y = host(mx.mx_linear(cuda(x), W, ctx))
    ctx.synchronize()
    assert rel_l2(y, ref) <= REL_TOL
    # also through pre-quantised activations (mxq_gemv on the GEMM path)
    y2 = host(mx.mx_gemv(mx.MXActivation(cuda(xq), cuda(xs)), W, ctx))
    ctx.synchronize()
    assert np.array_equal(y, y2)
    W.close()


def test_bsr_all_blocks_masked_gives_zeros(ctx):
    n, k = 300, 512
    w, ws = synth.weights(4, n, k, -8, -3, 3)
    mask = np.zeros(((n + 63) // 64, k // 64), np.uint8)
    W = mx.MXWeight(torch.from_numpy(w), torch.from_numpy(ws), 4, n, k, ctx, block_mask=mask)
    y = host(mx.mx_linear(cuda(synth.normal((5, k), 4)), W, ctx))
    ctx.synchronize()
    assert np.all(y == 0.0)
    W.close()


def test_bsr_rejects_gemv_only_entries(ctx):
    _, _, _, W = bsr_weight(ctx, 8, 128, 256, 0.5, 5)
    a = mx.mx_quantize_x(cuda(synth.normal((2, 256), 6)), ctx)
    with pytest.raises(_lib.MXError):
        mx.mx_block_dots(a, W, ctx)
    ctx.synchronize()
    with pytest.raises(ValueError):   # k must be a multiple of 64
        w, ws = synth.weights(8, 64, 96, -8, -3, 1)
        mx.MXWeight(torch.from_numpy(w), torch.from_numpy(ws), 8, 64, 96, ctx,
                    block_mask=np.ones((1, 1), np.uint8))
    W.close()


def make_experts(ctx, fmt, e, d, f, density, seed, dense_every=0):
    """E experts: gate/up [F][D] and down [D][F], block-sparse (every
    `dense_every`-th expert uploaded dense, to mix both kinds)."""
    host_w, dev_w = [], []
    for j in range(e):
        mats = []
        for (n, k, s) in ((f, d, 0), (f, d, 1), (d, f, 2)):
            w, ws = synth.weights(fmt, n, k, -7, -3, seed + 10 * j + s)
            dense = dense_every and j % dense_every == 0
            mask = synth.block_mask(n, k, 1.0 if dense else density, seed + 10 * j + s + 500)
            wm = synth.apply_block_mask(fmt, w, mask)
            if dense:
                W = mx.MXWeight(torch.from_numpy(wm), torch.from_numpy(ws), fmt, n, k, ctx)
            else:
                W = mx.MXWeight(torch.from_numpy(w), torch.from_numpy(ws), fmt, n, k, ctx, block_mask=mask)
            mats.append((wm, ws, W))
        host_w.append((mats[0][0], mats[0][1], mats[1][0], mats[1][1], mats[2][0], mats[2][1]))
        dev_w.append((mats[0][2], mats[1][2], mats[2][2]))
    return host_w, dev_w


@pytest.mark.parametrize("fmt", [4, 8])
@pytest.mark.parametrize("t,d,f,e,k,density", [
    (48, 256, 512, 4, 2, 0.25),
    (130, 128, 256, 8, 2, 0.5),
    (20, 256, 384, 3, 1, 0.25),
])
def test_moe_matches_oracle(ctx, fmt, t, d, f, e, k, density):
    host_w, dev_w = make_experts(ctx, fmt, e, d, f, density, 100 + t, dense_every=3)
    x = synth.normal((t, d), 7)
    logits = synth.normal((t, e), 8)
    ref = oracle.moe(fmt, x, logits, d, f, k, host_w)
    assert np.linalg.norm(ref) > 0
    xd, ld = cuda(x), cuda(logits)
    g, u, dn = ([w[i] for w in dev_w] for i in range(3))
    y = host(mx.moe_swiglu(xd, ld, g, u, dn, k, ctx))
    ctx.synchronize()
    assert rel_l2(y, ref) <= REL_TOL
    y2 = host(mx.moe_swiglu(xd, ld, g, u, dn, k, ctx))
    ctx.synchronize()
    assert np.array_equal(y, y2)
    for ws in dev_w:
        for W in ws:
            W.close()


def test_moe_idle_experts_and_errors(ctx):
    """Experts that receive no token are skipped; k > E is rejected with the
    router's invalid-argument contract."""
    t, d, f, e, k = 16, 128, 256, 4, 1
    host_w, dev_w = make_experts(ctx, 4, e, d, f, 0.5, 300)
    x = synth.normal((t, d), 9)
    logits = synth.normal((t, e), 10)
    logits[:, 1] -= 100.0       # experts 1 and 3 never win
    logits[:, 3] -= 100.0
    ref = oracle.moe(4, x, logits, d, f, k, host_w)
    assert np.linalg.norm(ref) > 0
    g, u, dn = ([w[i] for w in dev_w] for i in range(3))
    y = host(mx.moe_swiglu(cuda(x), cuda(logits), g, u, dn, k, ctx))
    ctx.synchronize()
    assert rel_l2(y, ref) <= REL_TOL
    with pytest.raises(ValueError):
        mx.moe_swiglu(cuda(x), cuda(logits), g, u, dn, e + 1, ctx)
    ctx.synchronize()
    for ws in dev_w:
        for W in ws:
            W.close()
