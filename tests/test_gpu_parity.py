"""GPU parity tests: every call goes through libmxq.so (the C-ABI) and is
checked against the CPU oracle on the same seeded inputs.

Bars: quantised bytes, E8M0 scales, per-block int32 dots, routing and GAE are
bit-exact; fp32 linear outputs agree with the oracle's exactly-rounded
result within relative L2 error <= 1e-5 (REL_TOL).
"""
import numpy as np
import pytest
import torch

from oracle import oracle
from cpu_model_b200 import mx, synth

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


def weight(ctx, fmt, n, k, seed, emin=-10, emax=-4):
    w, ws = synth.weights(fmt, n, k, emin, emax, seed)
    return w, ws, mx.MXWeight(torch.from_numpy(w), torch.from_numpy(ws), fmt, n, k, ctx)


def edge_inputs(b, k, seed):
    x = synth.normal((b, k), seed)
    x[0, :32] = 0.0
    if k >= 96:
        x[0, 32:64] *= 1e-30
        x[0, 64:96] *= 1e30
    if b > 1 and k >= 64:
        x[1, 40] = 0.5 * 2.0 ** -6        # exact tie after scaling
        x[1, 33] = 127.0 * 2.0 ** -6
    return x


# ----------------------------------------------------------- quantisers ---
@pytest.mark.parametrize("b,k", [(1, 32), (3, 96), (5, 4096), (2, 11008)])
@pytest.mark.parametrize("act", [0, 1])
def test_quantize_bit_exact(ctx, b, k, act):
    x = edge_inputs(b, k, 10 + b)
    q, s = oracle.quantize_x(x, act)
    a = (mx.mx_quantize_x if act == 0 else mx.mx_fused_silu_quantize_x)(cuda(x), ctx)
    ctx.synchronize()
    assert np.array_equal(host(a.q), q)
    assert np.array_equal(host(a.s), s)


def test_quantize_nonfinite_blocks(ctx):
    x = synth.normal((2, 128), 3)
    x[0, 5] = np.inf
    x[1, 70] = np.nan
    q, s = oracle.quantize_x(x)
    a = mx.mx_quantize_x(cuda(x), ctx)
    assert np.array_equal(host(a.q), q) and np.array_equal(host(a.s), s)
    assert s[0, 0] == 255 and s[1, 2] == 255


@pytest.mark.parametrize("b,k", [(1, 64), (4, 11008)])
def test_swiglu_quantize_bit_exact(ctx, b, k):
    g = synth.normal((b, k), 21) * 4
    u = synth.normal((b, k), 22)
    q, s = oracle.swiglu_quantize(g, u)
    a = mx.fused_gated_silu_quantize(cuda(g), cuda(u), ctx)
    assert np.array_equal(host(a.q), q) and np.array_equal(host(a.s), s)


# ----------------------------------------------------------- block dots ---
@pytest.mark.parametrize("fmt", [8, 4])
@pytest.mark.parametrize("b,n,k", [(1, 1, 32), (3, 33, 96), (2, 300, 4096)])
def test_block_dots_bit_exact(ctx, fmt, b, n, k):
    w, ws, W = weight(ctx, fmt, n, k, 30 + n)
    xq, xs = oracle.quantize_x(synth.normal((b, k), 31))
    d = mx.mx_block_dots(mx.MXActivation(cuda(xq), cuda(xs)), W, ctx)
    assert np.array_equal(host(d), oracle.block_dots(fmt, xq, w, n, k))


def test_block_dots_extremes(ctx):
    """Largest |dot| per format: int8 127*127*32, int4 127*8*32."""
    for fmt, wv in ((8, -127), (4, -8)):
        n, k = 4, 64
        wvals = np.full((n, k), wv, np.int8)
        w = synth.pack_int4(wvals) if fmt == 4 else wvals
        ws = np.full((n, k // 32), 127, np.uint8)
        W = mx.MXWeight(torch.from_numpy(w), torch.from_numpy(ws), fmt, n, k, ctx)
        xq = np.full((2, k), 128 + 127, np.uint8)
        xq[1] = 1                                   # q = -127
        d = host(mx.mx_block_dots(mx.MXActivation(cuda(xq), cuda(np.full((2, 2), 127, np.uint8))), W, ctx))
        assert np.array_equal(d, oracle.block_dots(fmt, xq, w, n, k))
        assert abs(int(d[0, 0, 0])) == 127 * abs(wv) * 32


# --------------------------------------------------------------- GEMV ---
@pytest.mark.parametrize("fmt", [8, 4])
@pytest.mark.parametrize("b", [1, 2, 3, 4, 5, 8])
@pytest.mark.parametrize("n,k", [(1, 32), (33, 96), (1000, 4096), (256, 11008)])
def test_gemv_parity(ctx, fmt, b, n, k):
    w, ws, W = weight(ctx, fmt, n, k, 40 + n + k)
    x = edge_inputs(b, k, 41 + b)
    xq, xs = oracle.quantize_x(x)
    ref = oracle.gemv(fmt, xq, xs, w, ws, n, k)
    ctx.set_path(mx.PATH_GEMV)
    try:
        y = host(mx.mx_gemv(mx.MXActivation(cuda(xq), cuda(xs)), W, ctx))
        ctx.synchronize()
    finally:
        ctx.set_path(mx.PATH_AUTO)
    assert rel_l2(y, ref) <= REL_TOL


@pytest.mark.parametrize("fmt", [8, 4])
@pytest.mark.parametrize("b", [6, 12, 16])
@pytest.mark.parametrize("n,k", [(33, 96), (1000, 4096)])
def test_small_batch_mma_gemv_parity(ctx, fmt, b, n, k):
    """Batches 9-16 on the int8-MMA GEMV (batches 2-8 are covered above)."""
    w, ws, W = weight(ctx, fmt, n, k, 50 + n + k)
    x = edge_inputs(b, k, 51 + b)
    xq, xs = oracle.quantize_x(x)
    ref = oracle.gemv(fmt, xq, xs, w, ws, n, k)
    ctx.set_path(mx.PATH_GEMV)
    try:
        y = host(mx.mx_gemv(mx.MXActivation(cuda(xq), cuda(xs)), W, ctx))
        ctx.synchronize()
    finally:
        ctx.set_path(mx.PATH_AUTO)
    assert rel_l2(y, ref) <= REL_TOL


@pytest.mark.parametrize("b", [5, 12, 16])
def test_auto_path_small_batch_fp32(ctx, b):
    """fp32 rows through mx_linear in the automatic path: the MMA GEMV where
    the shape fits (up 4096 -> 11008), the tensor-core GEMM otherwise
    (down 11008 -> 4096 at batch > 8); both against the oracle."""
    for (n, k, seed) in [(11008, 4096, 61), (4096, 11008, 62)]:
        w, ws, W = weight(ctx, 4, n, k, seed, -8, -3)
        x = synth.normal((b, k), seed + b)
        xq, xs = oracle.quantize_x(x)
        y = host(mx.mx_linear(cuda(x), W, ctx))
        ctx.synchronize()
        rows = np.random.default_rng(seed).choice(n, 128, replace=False).astype(np.int32)
        ref = oracle.gather_dot(4, xq, xs, w, ws, k, rows)
        assert rel_l2(y[:, rows], ref) <= REL_TOL


# ---------------------------------------------------- tensor-core GEMM ---
@pytest.mark.parametrize("fmt", [8, 4])
@pytest.mark.parametrize("b", [1, 9, 16, 40, 64, 100, 256, 300])
@pytest.mark.parametrize("n,k", [(33, 96), (384, 4096), (256, 11008)])
def test_gemm_parity(ctx, fmt, b, n, k):
    w, ws, W = weight(ctx, fmt, n, k, 50 + n + k)
    x = edge_inputs(b, k, 51 + b)
    xq, xs = oracle.quantize_x(x)
    ref = oracle.gemv(fmt, xq, xs, w, ws, n, k)
    ctx.set_path(mx.PATH_GEMM)
    try:
        y = host(mx.mx_gemv(mx.MXActivation(cuda(xq), cuda(xs)), W, ctx))
        ctx.synchronize()
        y2 = host(mx.mx_linear(cuda(x), W, ctx))
        ctx.synchronize()
    finally:
        ctx.set_path(mx.PATH_AUTO)
    assert rel_l2(y, ref) <= REL_TOL
    assert np.array_equal(y, y2)


@pytest.mark.parametrize("fmt", [8, 4])
def test_gemm_extreme_weight_scales(ctx, fmt):
    """Weight scale bytes 245..249 (exponents 118..122): past the range where
    the converter folds the int4/int8 offset into one fma, so the two-step
    conversion runs; activations scaled by 2^-40 keep the products finite."""
    n, k, b = 384, 2048, 40
    w, ws, W = weight(ctx, fmt, n, k, 61, 118, 122)
    x = synth.normal((b, k), 62) * np.float32(2.0 ** -40)
    xq, xs = oracle.quantize_x(x)
    ref = oracle.gemv(fmt, xq, xs, w, ws, n, k)
    assert np.all(np.isfinite(ref))
    ctx.set_path(mx.PATH_GEMM)
    try:
        y = host(mx.mx_gemv(mx.MXActivation(cuda(xq), cuda(xs)), W, ctx))
        ctx.synchronize()
    finally:
        ctx.set_path(mx.PATH_AUTO)
    assert rel_l2(y, ref) <= REL_TOL


@pytest.mark.parametrize("fmt", [8, 4])
def test_decode_gemv_exact_scale_path(ctx, fmt):
    """Weight scale bytes 0..7 (exponents -127..-120, below the fast path's
    range) and one row whose first block scale is 0xFF (NaN): the decode
    GEMVs take their exact-scale path -- batch 1 (weight-resident), 2 (ring),
    5 (int8 MMA), on MX input and on fp32 rows.  Activations scaled by 2^40
    keep the products normal; NaN rows must match the oracle's."""
    n, k = 1000, 4096
    w, ws = synth.weights(fmt, n, k, -127, -120, 63)
    ws[3, 0] = 255
    W = mx.MXWeight(torch.from_numpy(w), torch.from_numpy(ws), fmt, n, k, ctx)
    for b in (1, 2, 5):
        x = synth.normal((b, k), 64 + b) * np.float32(2.0 ** 40)
        xq, xs = oracle.quantize_x(x)
        ref = oracle.gemv(fmt, xq, xs, w, ws, n, k)
        ctx.set_path(mx.PATH_GEMV)
        try:
            y_mx = host(mx.mx_gemv(mx.MXActivation(cuda(xq), cuda(xs)), W, ctx))
            y_f32 = host(mx.mx_linear(cuda(x), W, ctx))
            ctx.synchronize()
        finally:
            ctx.set_path(mx.PATH_AUTO)
        nan = np.isnan(ref)
        assert nan[:, 3].all() and nan.sum() == b
        for y in (y_mx, y_f32):
            assert np.array_equal(np.isnan(y), nan), b
            assert rel_l2(y[~nan], ref[~nan]) <= REL_TOL, b


def test_golden_fixture_on_gpu(ctx):
    import os
    d = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "mx_oracle.npz"))
    names = sorted({k.rsplit("_", 1)[0] for k in d.files if k.endswith("_shape")})
    for nm in names:
        fmt, b, n, k = (int(v) for v in d[nm + "_shape"])
        W = mx.MXWeight(torch.from_numpy(d[nm + "_w"]), torch.from_numpy(d[nm + "_ws"]), fmt, n, k, ctx)
        a = mx.mx_quantize_x(cuda(d[nm + "_x"]), ctx)
        assert np.array_equal(host(a.q), d[nm + "_xq"]) and np.array_equal(host(a.s), d[nm + "_xs"])
        assert np.array_equal(host(mx.mx_block_dots(a, W, ctx)), d[nm + "_dots"])
        for path in (mx.PATH_GEMV, mx.PATH_GEMM):
            if path == mx.PATH_GEMV and b > 8:
                continue
            ctx.set_path(path)
            try:
                y = host(mx.mx_gemv(a, W, ctx))
            finally:
                ctx.set_path(mx.PATH_AUTO)
            assert rel_l2(y, d[nm + "_y"]) <= REL_TOL, (nm, path)


# -------------------------------------------------- full-size workloads ---
def test_single_int8_linear_4096(ctx):
    """4096x4096 MX-int8 GEMV, exponents [-10,-4], x ~ N(0,1), batch 1,
    seed 0 (the reference's CPU-runnable linear)."""
    w, ws, W = weight(ctx, 8, 4096, 4096, 0, -10, -4)
    x = synth.normal((1, 4096), 0)
    xq, xs = oracle.quantize_x(x)
    ref = oracle.gemv(8, xq, xs, w, ws, 4096, 4096)
    y = host(mx.mx_linear(cuda(x), W, ctx))
    ctx.synchronize()
    assert rel_l2(y, ref) <= REL_TOL


@pytest.mark.parametrize("b", [1, 8, 64, 512])
def test_int4_mlp_pair_7b_shape(ctx, b):
    """MX-int4 up 4096->11008 then down 11008->4096 at batch 1/8/64/512.
    Stage-wise: up vs oracle (rows sampled at b=512), the requantised
    intermediate bit-exact against the oracle's quantiser applied to the GPU's
    own up output, down vs oracle on that intermediate."""
    wu, su, Wu = weight(ctx, 4, 11008, 4096, 1, -8, -3)
    wd, sd, Wd = weight(ctx, 4, 4096, 11008, 2, -8, -3)
    x = synth.normal((b, 4096), 3 + b)
    xq, xs = oracle.quantize_x(x)
    y1 = host(mx.mx_linear(cuda(x), Wu, ctx))
    ctx.synchronize()
    rows = np.arange(11008) if b <= 64 else np.random.default_rng(5).choice(11008, 96, replace=False).astype(np.int32)
    ref1 = oracle.gather_dot(4, xq, xs, wu, su, 4096, rows)
    assert rel_l2(y1[:, rows], ref1) <= REL_TOL
    hq, hs = oracle.quantize_x(y1)
    y2 = host(mx.mx_linear(cuda(y1), Wd, ctx))
    ctx.synchronize()
    rows2 = np.arange(4096) if b <= 64 else np.random.default_rng(6).choice(4096, 96, replace=False).astype(np.int32)
    ref2 = oracle.gather_dot(4, hq, hs, wd, sd, 11008, rows2)
    assert rel_l2(y2[:, rows2], ref2) <= REL_TOL
    yp = host(mx.mx_linear_pair(cuda(x), Wu, Wd, ctx))
    ctx.synchronize()
    assert np.array_equal(yp, y2)


@pytest.mark.parametrize("fmt,n,k", [(4, 22016, 4096), (4, 32000, 4096), (8, 12288, 2048), (4, 12288, 4096)])
def test_tall_batch1_linear_row_slices(ctx, fmt, n, k):
    """Batch-1 linears too tall for one co-resident launch (the 7B decoder's
    fused gate/up, LM head and QKV shapes) run as consecutive launches over
    128-row-tile slices; every row agrees with the oracle, fp32 and MX input."""
    w, ws, W = weight(ctx, fmt, n, k, 70 + n, -8, -3)
    x = synth.normal((1, k), 71)
    xq, xs = oracle.quantize_x(x)
    ref = oracle.gemv(fmt, xq, xs, w, ws, n, k)
    y = host(mx.mx_linear(cuda(x), W, ctx))
    y2 = host(mx.mx_gemv(mx.MXActivation(cuda(xq), cuda(xs)), W, ctx))
    ctx.synchronize()
    assert rel_l2(y, ref) <= REL_TOL
    assert rel_l2(y2, ref) <= REL_TOL
    W.close()


@pytest.mark.parametrize("fmt,k,m,n", [(4, 2048, 2048, 1024), (8, 1024, 1184, 2048), (4, 4096, 4096, 4096)])
def test_pair_mx_output_blocks_across_ctas(ctx, fmt, k, m, n):
    """Batch-1 pairs whose first projection has fewer than 32 rows a CTA, so
    one 32-row MX block of the intermediate is shared by two or three CTAs
    (the last of them to finish quantises it): the pair is bit-identical to
    two mxq_linear calls on the GPU's own intermediate, each vs the oracle."""
    w1, s1, W1 = weight(ctx, fmt, m, k, 80 + m, -8, -3)
    w2, s2, W2 = weight(ctx, fmt, n, m, 81 + n, -8, -3)
    x = synth.normal((1, k), 82)
    xd = cuda(x)
    yp = host(mx.mx_linear_pair(xd, W1, W2, ctx))
    for _ in range(3):                       # the block counters are left zero
        assert np.array_equal(host(mx.mx_linear_pair(xd, W1, W2, ctx)), yp)
    y1 = host(mx.mx_linear(xd, W1, ctx))
    y2 = host(mx.mx_linear(cuda(y1), W2, ctx))
    ctx.synchronize()
    assert np.array_equal(yp, y2)
    xq, xs = oracle.quantize_x(x)
    assert rel_l2(y1, oracle.gemv(fmt, xq, xs, w1, s1, m, k)) <= REL_TOL
    hq, hs = oracle.quantize_x(y1)
    assert rel_l2(y2, oracle.gemv(fmt, hq, hs, w2, s2, n, m)) <= REL_TOL
    W1.close()
    W2.close()


# ---------------------------------------------------- gather / MLP ---
@pytest.mark.parametrize("fmt", [8, 4])
def test_rank16_dot_ptrs(ctx, fmt):
    n, k = 1024, 2048
    w, ws, W = weight(ctx, fmt, n, k, 60)
    x = synth.normal((2, k), 61)
    xq, xs = oracle.quantize_x(x)
    rows = np.array([5, 1023, 0, 77, 77, 512, 3, 900, 1, 2, 4, 6, 8, 10, 12, 14], np.int32)
    ref = oracle.gather_dot(fmt, xq, xs, w, ws, k, rows)
    y = host(mx.mx_rank16_dot_ptrs(mx.MXActivation(cuda(xq), cuda(xs)), W, cuda(rows), ctx))
    assert rel_l2(y, ref) <= REL_TOL


def test_fixed_size_checks(ctx):
    """Shapes the API must reject (the reference throws invalid_argument)."""
    w, ws, W = weight(ctx, 8, 64, 64, 80)
    with pytest.raises(ValueError):
        mx.mx_linear(cuda(synth.normal((1, 96), 1)), W, ctx)
    with pytest.raises(ValueError):
        mx.MXWeight(torch.from_numpy(np.zeros((4, 48), np.int8)), torch.from_numpy(np.zeros((4, 1), np.uint8)),
                    8, 4, 48, ctx)
    with pytest.raises(ValueError):
        mx.mx_dot(mx.mx_quantize_x(cuda(synth.normal((1, 64), 2)), ctx), W, ctx)


# ------------------------------------------------------ routing / GAE ---
def test_misaligned_fp32_input_rejected(ctx):
    """fp32 inputs are read in 16-byte vectors: a device pointer off a
    16-byte boundary is refused on the host, before any launch, and the
    context stays usable."""
    n, k = 64, 256
    w, ws, W = weight(ctx, 8, n, k, 71)
    buf = torch.from_numpy(synth.normal((1, k + 4), 72)).reshape(-1).cuda()
    x_bad = buf[1:1 + k].view(1, k)
    assert x_bad.data_ptr() % 16 == 4
    with pytest.raises(ValueError):
        mx.mx_linear(x_bad, W, ctx)
    x_ok = buf[4:4 + k].view(1, k)
    assert x_ok.data_ptr() % 16 == 0
    y = host(mx.mx_linear(x_ok, W, ctx))
    ctx.synchronize()
    xq, xs = oracle.quantize_x(host(x_ok))
    assert rel_l2(y, oracle.gemv(8, xq, xs, w, ws, n, k)) <= REL_TOL


def test_route_topk_bit_exact(ctx):
    logits = synth.normal((4096, 8), 90)
    logits[7, 3] = logits[7, 5] = 9.0        # tie
    idx, gate = oracle.route_topk(logits, 2)
    gi, gg = mx.route_topk(cuda(logits), 2, ctx)
    assert np.array_equal(host(gi), idx) and np.array_equal(host(gg), gate)
    with pytest.raises(ValueError):
        mx.HashedRouter(1024, 10, 20)
    with pytest.raises(ValueError):
        mx.route_topk(cuda(logits), 9, ctx)


def test_gae_bit_exact(ctx):
    import os
    d = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "gae_reference.npz"))
    for case in ("kat", "rand"):
        a, r = mx.fused_compute_gae(cuda(d[case + "_r"]), cuda(d[case + "_v"]), cuda(d[case + "_d"]),
                                    cuda(d[case + "_nv"]), 0.99, 0.95, ctx)
        assert np.array_equal(host(a), d[case + "_adv"])
        assert np.array_equal(host(r), d[case + "_ret"])
    T, E = 512, 256
    g = synth.rng(91)
    rr = np.zeros((T, E), np.float32)
    done = np.zeros((T, E), np.uint8)
    done[-1] = 1
    rr[-1] = g.standard_normal(E, dtype=np.float32)
    v = g.standard_normal((T, E), dtype=np.float32)
    nv = np.zeros(E, np.float32)
    a0, r0 = oracle.gae(rr, v, done, nv, 0.99, 0.95)
    a1, r1 = mx.fused_compute_gae(cuda(rr), cuda(v), cuda(done), cuda(nv), 0.99, 0.95, ctx)
    assert np.array_equal(host(a1), a0) and np.array_equal(host(r1), r0)


@pytest.mark.parametrize("fmt", [8, 4])
@pytest.mark.parametrize("b", [1, 4, 16])
def test_repeat_calls_bit_identical(ctx, fmt, b):
    """Split-K reductions (streaming GEMV) and the GEMM are deterministic:
    repeated calls, interleaved with other shapes, give identical bits."""
    w, ws, W = weight(ctx, fmt, 2000, 4096, 95)
    w2, ws2, W2 = weight(ctx, fmt, 300, 11008, 96)
    x = cuda(synth.normal((b, 4096), 97))
    x2 = cuda(synth.normal((b, 11008), 98))
    ys = []
    for _ in range(4):
        ys.append(host(mx.mx_linear(x, W, ctx)))
        mx.mx_linear(x2, W2, ctx)
    ctx.synchronize()
    for y in ys[1:]:
        assert np.array_equal(y, ys[0])
