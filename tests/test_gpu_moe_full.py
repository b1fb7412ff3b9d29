"""GPU parity of the block-sparse MoE layer at its full benchmark shape --
4096 tokens, d 4096, 8 experts, top-2, SwiGLU FFN 14336, MX-int4 expert
matrices with 25 % of their 64x64 blocks present -- and of the gated MLP at
the contract's 1e-5 bar, through libmxq.so's C-ABI.

Stage-wise checks (the intermediate is requantised to MX, so one fp32
rounding difference in gate/up can move a byte by one step; each stage is
checked on the GPU's own input to it):
  routing       ids and gates bit-exact against the oracle;
  gate / up     the GPU's expert outputs against the oracle (sampled rows);
  down+combine  the oracle's SwiGLU requantisation of the GPU's gate/up,
                down projection and fp64 combine against the GPU layer's
                output, every output of a seeded sample of 64 tokens.
The per-expert gate/up outputs are those of the layer's own GEMMs: the same
kernel on the same gathered token rows, batch and tile choice (the layer's
slots follow token order), which is deterministic.
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


def masked(fmt, data, mask):
    """data with every masked-out 64x64 block zeroed (vectorised)."""
    per = 32 if fmt == 4 else 64
    n, kb = data.shape
    full = np.repeat(np.repeat(mask, 64, axis=0), per, axis=1)[:n, :kb]
    return np.where(full != 0, data, 0).astype(data.dtype)


def int4_matrix(n, k, emin, emax, seed):
    """Uniform int4 nibbles (any byte is two uniform nibbles in [-8, 7]) and
    E8M0 exponents uniform in [emin, emax]."""
    g = synth.rng(seed)
    data = g.integers(0, 256, size=(n, k // 2), dtype=np.uint8)
    sc = (g.integers(emin, emax + 1, size=(n, k // 32), dtype=np.int16) + 127).astype(np.uint8)
    return data, sc


def test_moe_config4_full_shape(ctx):
    T, D, F, E, K, dens = 4096, 4096, 14336, 8, 2, 0.25
    experts_host, experts_dev = [], []
    for e in range(E):
        hm, dm = [], []
        for j, (n, k) in enumerate(((F, D), (F, D), (D, F))):
            data, sc = int4_matrix(n, k, -8, -3, 9000 + 10 * e + j)
            mask = synth.block_mask(n, k, dens, 9500 + 10 * e + j)
            dm.append(mx.MXWeight(torch.from_numpy(data), torch.from_numpy(sc), 4, n, k, ctx, block_mask=mask))
            hm.append((masked(4, data, mask), sc))
        experts_host.append(hm)
        experts_dev.append(dm)
    x = synth.normal((T, D), 201)
    logits = synth.normal((T, E), 202)
    xd, ld = cuda(x), cuda(logits)
    gw, uw, dw = ([m[i] for m in experts_dev] for i in range(3))
    y = host(mx.moe_swiglu(xd, ld, gw, uw, dw, K, ctx))
    ctx.synchronize()
    assert np.all(np.isfinite(y))
    y2 = host(mx.moe_swiglu(xd, ld, gw, uw, dw, K, ctx))
    ctx.synchronize()
    assert np.array_equal(y, y2)                       # deterministic at full size

    # routing: bit-exact
    idx_d, gate_d = mx.route_topk(ld, K, ctx)
    idx, gate = host(idx_d), host(gate_d)
    i0, g0 = oracle.route_topk(logits, K)
    assert np.array_equal(idx, i0) and np.array_equal(gate, g0)

    # the layer's per-expert gate/up outputs (token order per expert)
    toks = [np.nonzero((idx == e).any(1))[0] for e in range(E)]
    G, U = [], []
    for e in range(E):
        rows = cuda(x[toks[e]])
        G.append(host(mx.mx_linear(rows, gw[e], ctx)))
        U.append(host(mx.mx_linear(rows, uw[e], ctx)))
    ctx.synchronize()

    rng = np.random.default_rng(17)
    sample = np.sort(rng.choice(T, 64, replace=False))
    frows = np.sort(rng.choice(F, 256, replace=False)).astype(np.int32)
    xq, xs = oracle.quantize_x(x[sample])
    # gate / up stage on sampled rows, every route of the sampled tokens
    got, ref = [], []
    for si, t in enumerate(sample):
        for j in range(K):
            e = idx[t, j]
            pos = np.searchsorted(toks[e], t)
            (wg, sg), (wu, su), _ = experts_host[e]
            for M, (w_, s_) in ((G[e], (wg, sg)), (U[e], (wu, su))):
                got.append(M[pos, frows])
                ref.append(oracle.gather_dot(4, xq[si:si + 1], xs[si:si + 1], w_, s_, D, frows)[0])
    assert rel_l2(np.array(got), np.array(ref)) <= REL_TOL

    # down + combine on the GPU's own gate/up
    yref = np.zeros((len(sample), D), np.float64)
    for j in range(K):
        for e in range(E):
            sel = np.nonzero(idx[sample, j] == e)[0]
            if sel.size == 0:
                continue
            pos = np.searchsorted(toks[e], sample[sel])
            hq, hs = oracle.swiglu_quantize(G[e][pos], U[e][pos])
            wd, sd = experts_host[e][2]
            out = oracle.gemv(4, hq, hs, wd, sd, D, F)
            yref[sel] += gate[sample[sel], j].astype(np.float64)[:, None] * out.astype(np.float64)
    assert rel_l2(y[sample], yref.astype(np.float32)) <= REL_TOL

    for dm in experts_dev:
        for W in dm:
            W.close()


@pytest.mark.parametrize("b", [1, 3, 24, 200])
def test_gated_mlp_step_stagewise(ctx, b):
    """gated_mlp_step at rel-L2 <= 1e-5: gate and up against the oracle, then
    the oracle's SwiGLU requantisation of the GPU's own gate/up and its down
    projection against the GPU's gated_mlp_step output."""
    d, f = 1024, 2816
    mats = []
    for j, (n, k) in enumerate(((f, d), (f, d), (d, f))):
        w, ws = synth.weights(4, n, k, -8, -3, 70 + j)
        mats.append((w, ws, mx.MXWeight(torch.from_numpy(w), torch.from_numpy(ws), 4, n, k, ctx)))
    (wg, sg, Wg), (wu, su, Wu), (wd, sd, Wd) = mats
    x = synth.normal((b, d), 73 + b)
    xdv = cuda(x)
    y = host(mx.gated_mlp_step(xdv, Wg, Wu, Wd, ctx))
    g = host(mx.mx_linear(xdv, Wg, ctx))
    u = host(mx.mx_linear(xdv, Wu, ctx))
    ctx.synchronize()
    xq, xs = oracle.quantize_x(x)
    assert rel_l2(g, oracle.gemv(4, xq, xs, wg, sg, f, d)) <= REL_TOL
    assert rel_l2(u, oracle.gemv(4, xq, xs, wu, su, f, d)) <= REL_TOL
    hq, hs = oracle.swiglu_quantize(g, u)
    # the library's own SwiGLU quantiser on the same gate/up: bit-exact
    a = mx.fused_gated_silu_quantize(cuda(g), cuda(u), ctx)
    assert np.array_equal(host(a.q), hq) and np.array_equal(host(a.s), hs)
    ref = oracle.gemv(4, hq, hs, wd, sd, d, f)
    assert rel_l2(y, ref) <= REL_TOL
    for m in mats:
        m[2].close()
