"""numpy wrapper of the CPU oracle (liboracle.so: mx_oracle.c +
mx_cpu_baseline.c).

TEST INFRASTRUCTURE ONLY: the checker for tests/, the smoke entry and the
CPU-baseline leg of bench.py.  The product (cpu_model_b200) never imports it.
Parity of the MX path against the reference is unpinned (the reference's MX
kernels are absent from its snapshot); the GAE restatement is pinned against
the reference's own compiled code (oracle/_ref) and its known-answer test.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")
REF_GAE = os.path.join(HERE, "_ref", "libref_gae.so")

_c = None


def build():
    subprocess.check_call(["make", "-s", "-C", HERE], stdout=subprocess.DEVNULL)


def lib():
    global _c
    if _c is None:
        srcs = [os.path.join(HERE, f) for f in ("mx_oracle.c", "mx_cpu_baseline.c", "mx_oracle.h")]
        if not os.path.exists(LIB) or any(os.path.getmtime(s) > os.path.getmtime(LIB) for s in srcs
                                           if os.path.exists(s)):
            build()
        _c = ctypes.CDLL(LIB)
        _c.mxo_e8m0_from_absmax.restype = ctypes.c_uint8
        _c.mxo_e8m0_from_absmax.argtypes = [ctypes.c_float, ctypes.c_int]
        _c.mxo_e8m0_decode.restype = ctypes.c_double
        _c.mxo_e8m0_decode.argtypes = [ctypes.c_uint8]
        _c.mxo_expf.restype = ctypes.c_float
        _c.mxo_expf.argtypes = [ctypes.c_float]
        _c.mxo_silu.restype = ctypes.c_float
        _c.mxo_silu.argtypes = [ctypes.c_float]
        _c.mxo_weight_at.restype = ctypes.c_int
        _c.mxo_route_topk.restype = ctypes.c_int
        _c.mxo_hashed_route.restype = ctypes.c_int
        _c.mxo_moe.restype = ctypes.c_int
        _c.mxb_gemv.restype = ctypes.c_int
        _c.mxb_max_threads.restype = ctypes.c_int
    return _c


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _sz(*v):
    return [ctypes.c_size_t(int(x)) for x in v]


def e8m0_from_absmax(m, qmax=127):
    return int(lib().mxo_e8m0_from_absmax(ctypes.c_float(m), qmax))


def e8m0_decode(s):
    return lib().mxo_e8m0_decode(ctypes.c_uint8(s))


def expf(x):
    return lib().mxo_expf(ctypes.c_float(x))


def silu(x):
    return lib().mxo_silu(ctypes.c_float(x))


def quantize_x(x, act=0):
    x = np.ascontiguousarray(x, dtype=np.float32)
    b, k = x.shape
    q = np.empty((b, k), np.uint8)
    s = np.empty((b, k // 32), np.uint8)
    lib().mxo_quantize_x(_p(x), *_sz(b, k), ctypes.c_int(act), _p(q), _p(s))
    return q, s


def swiglu_quantize(g, u):
    g = np.ascontiguousarray(g, dtype=np.float32)
    u = np.ascontiguousarray(u, dtype=np.float32)
    b, k = g.shape
    q = np.empty((b, k), np.uint8)
    s = np.empty((b, k // 32), np.uint8)
    lib().mxo_swiglu_quantize(_p(g), _p(u), *_sz(b, k), _p(q), _p(s))
    return q, s


def quantize_w(fmt, w):
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    data = np.zeros((n, k // 2), np.uint8) if fmt == 4 else np.zeros((n, k), np.int8)
    scales = np.empty((n, k // 32), np.uint8)
    sums = np.empty((n, k // 32), np.int32)
    lib().mxo_quantize_w(ctypes.c_int(fmt), _p(w), *_sz(n, k), _p(data), _p(scales), _p(sums))
    return data, scales, sums


def rank16_dot_ptrs(fmt, xq, xs, rows, row_scales, k):
    """rows: list of one-row weights (int8 [1][K] or int4 [1][K/2]) with
    their scales [1][K/32]; y [B][len(rows)] in the GPU's summation order."""
    xq = np.ascontiguousarray(xq, np.uint8)
    xs = np.ascontiguousarray(xs, np.uint8)
    b = xq.shape[0]
    rs = [np.ascontiguousarray(r) for r in rows]
    ss = [np.ascontiguousarray(x, np.uint8) for x in row_scales]
    rp = (ctypes.c_void_p * len(rs))(*[r.ctypes.data for r in rs])
    sp = (ctypes.c_void_p * len(ss))(*[x.ctypes.data for x in ss])
    y = np.empty((b, len(rs)), np.float32)
    lib().mxo_rank16_dot_ptrs(ctypes.c_int(fmt), _p(xq), _p(xs), rp, sp, *_sz(len(rs), b, k), _p(y))
    return y


def halting_step(fmt, xq, xs, w, ws, k, bias, p_sum, remainder, steps, eps=0.01):
    """ACT halting over B tokens; the state arrays (float32, float32, uint64)
    are updated in place.  Returns (p, halt)."""
    xq = np.ascontiguousarray(xq, np.uint8)
    b = xq.shape[0]
    p = np.empty(b, np.float32)
    h = np.empty(b, np.uint8)
    lib().mxo_halting_step(ctypes.c_int(fmt), _p(xq), _p(np.ascontiguousarray(xs, np.uint8)), _p(np.ascontiguousarray(w)),
                           _p(np.ascontiguousarray(ws, np.uint8)), *_sz(b, k), ctypes.c_float(bias), ctypes.c_float(eps),
                           _p(p_sum), _p(remainder), _p(steps), _p(p), _p(h))
    return p, h


def update_gaussian_moment(fmt, data, scales, g, x, step):
    """Returns the updated copy of data (MXINT8Tensor layout)."""
    out = np.array(data, copy=True)
    n = scales.shape[0]
    k = scales.shape[1] * 32
    lib().mxo_update_gaussian_moment(ctypes.c_int(fmt), _p(out), _p(np.ascontiguousarray(scales, np.uint8)),
                                     *_sz(n, k), _p(np.ascontiguousarray(g, np.float32)),
                                     _p(np.ascontiguousarray(x, np.float32)), ctypes.c_float(step))
    return out


def micro_moe(fmt, wg, sg, wu, su, wd, sd, n_routed, n_shared, x, idx, gate):
    """The micro-expert layer (mxo_micro_moe); idx/gate [T][k] (gate may be
    None = 1)."""
    x = np.ascontiguousarray(x, np.float32)
    t, d = x.shape
    idx = np.ascontiguousarray(idx, np.int32)
    k = idx.shape[1] if idx.ndim == 2 else 0
    y = np.empty((t, d), np.float32)
    g = None if gate is None else np.ascontiguousarray(gate, np.float32)
    c = lambda a: np.ascontiguousarray(a)
    lib().mxo_micro_moe(ctypes.c_int(fmt), _p(c(wg)), _p(c(sg)), _p(c(wu)), _p(c(su)), _p(c(wd)), _p(c(sd)),
                        *_sz(n_routed, n_shared, d), _p(x), _p(idx), _p(g) if g is not None else None,
                        *_sz(t, k), _p(y))
    return y


def activation_norm(xq, xs):
    xq = np.ascontiguousarray(xq, np.uint8)
    b, k = xq.shape
    out = np.empty(b, np.float32)
    lib().mxo_activation_norm(_p(xq), _p(np.ascontiguousarray(xs, np.uint8)), *_sz(b, k), _p(out))
    return out


def hashed_route(x, n_experts, top_k, n_hashes, seed):
    """(idx [T][top_k], score [T][top_k]) of the LSH router; ValueError for
    top_k > n_experts (the reference's invalid_argument)."""
    x = np.ascontiguousarray(x, np.float32)
    t, d = x.shape
    idx = np.empty((t, max(top_k, 1)), np.int32)
    sc = np.empty((t, max(top_k, 1)), np.int32)
    rc = lib().mxo_hashed_route(_p(x), *_sz(t, d, n_experts, top_k, n_hashes), ctypes.c_uint64(seed), _p(idx),
                                _p(sc))
    if rc != 0:
        raise ValueError("HashedRouter: top_k=%d must be in [1, n_experts=%d]" % (top_k, n_experts))
    return idx, sc


def block_dots(fmt, xq, w, n, k):
    xq = np.ascontiguousarray(xq, np.uint8)
    w = np.ascontiguousarray(w)
    b = xq.shape[0]
    out = np.empty((b, n, k // 32), np.int32)
    lib().mxo_block_dots(ctypes.c_int(fmt), _p(xq), _p(w), *_sz(b, n, k), _p(out))
    return out


def gemv(fmt, xq, xs, w, ws, n, k):
    xq = np.ascontiguousarray(xq, np.uint8)
    xs = np.ascontiguousarray(xs, np.uint8)
    w = np.ascontiguousarray(w)
    ws = np.ascontiguousarray(ws, np.uint8)
    b = xq.shape[0]
    y = np.empty((b, n), np.float32)
    lib().mxo_gemv(ctypes.c_int(fmt), _p(xq), _p(xs), _p(w), _p(ws), *_sz(b, n, k), _p(y))
    return y


def gather_dot(fmt, xq, xs, w, ws, k, rows):
    xq = np.ascontiguousarray(xq, np.uint8)
    xs = np.ascontiguousarray(xs, np.uint8)
    rows = np.ascontiguousarray(rows, np.int32)
    b = xq.shape[0]
    y = np.empty((b, rows.size), np.float32)
    lib().mxo_gather_dot(ctypes.c_int(fmt), _p(xq), _p(xs), _p(np.ascontiguousarray(w)),
                         _p(np.ascontiguousarray(ws, np.uint8)), ctypes.c_size_t(k), _p(rows),
                         *_sz(rows.size, b), _p(y))
    return y


def mlp_swiglu(fmt, x, d, f, wg, sg, wu, su, wd, sd):
    x = np.ascontiguousarray(x, np.float32)
    b = x.shape[0]
    y = np.empty((b, d), np.float32)
    mq = np.empty((b, f), np.uint8)
    ms = np.empty((b, f // 32), np.uint8)
    arrs = [np.ascontiguousarray(a) for a in (wg, sg, wu, su, wd, sd)]
    lib().mxo_mlp_swiglu(ctypes.c_int(fmt), _p(x), *_sz(b, d, f), *[_p(a) for a in arrs], _p(y), _p(mq), _p(ms))
    return y, mq, ms


def route_topk(logits, k):
    logits = np.ascontiguousarray(logits, np.float32)
    t, e = logits.shape
    idx = np.empty((t, max(k, 1)), np.int32)
    gate = np.empty((t, max(k, 1)), np.float32)
    rc = lib().mxo_route_topk(_p(logits), *_sz(t, e, k), _p(idx), _p(gate))
    if rc != 0:
        raise ValueError("top-k: k=%d must be in [1, %d]" % (k, e))
    return idx, gate


def gae(rewards, values, dones, next_values, gamma, lam):
    r = np.ascontiguousarray(rewards, np.float32)
    v = np.ascontiguousarray(values, np.float32)
    d = np.ascontiguousarray(dones, np.uint8)
    nv = np.ascontiguousarray(next_values, np.float32)
    t, e = r.shape
    adv = np.empty_like(r)
    ret = np.empty_like(r)
    lib().mxo_gae(_p(r), _p(v), _p(d), _p(nv), *_sz(t, e), ctypes.c_float(gamma), ctypes.c_float(lam),
                  _p(adv), _p(ret))
    return adv, ret


def gae_ring(rewards, values, dones, next_values, size, cursor, t, e, gamma, lam, adv, ret):
    """Ring-buffer GAE (mxo_gae_ring) over 1-D ring arrays of the capacity;
    adv/ret (float32, capacity) are updated in place and returned."""
    r = np.ascontiguousarray(rewards, np.float32)
    v = np.ascontiguousarray(values, np.float32)
    d = np.ascontiguousarray(dones, np.uint8)
    nv = np.ascontiguousarray(next_values, np.float32)
    assert adv.dtype == np.float32 and ret.dtype == np.float32 and adv.flags.c_contiguous and ret.flags.c_contiguous
    lib().mxo_gae_ring(_p(r), _p(v), _p(d), _p(nv), *_sz(r.size, size, cursor, t, e), ctypes.c_float(gamma),
                       ctypes.c_float(lam), _p(adv), _p(ret))
    return adv, ret


def ref_gae_ring(rewards_pushed, dones_pushed, values_latest, cap, t, e, next_values, gamma, lam):
    """The reference's own ReplayMemory (oracle/_ref/libref_gae.so): push the
    given items one by one into a ring of `cap` items (wrapping when more are
    pushed), write_values(len(values_latest)), fused_compute_gae(t, e).
    Returns the ring's (rewards, values, dones, advantages, returns, size,
    cursor)."""
    rp = np.ascontiguousarray(rewards_pushed, np.float32)
    dp = np.ascontiguousarray(dones_pushed, np.uint8)
    vl = np.ascontiguousarray(values_latest, np.float32)
    nv = np.ascontiguousarray(next_values, np.float32)
    out = {k: np.zeros(cap, np.float32) for k in ("r", "v", "adv", "ret")}
    d_out = np.zeros(cap, np.uint8)
    meta = np.zeros(2, np.uint64)
    L = ctypes.CDLL(REF_GAE)
    L.ref_gae_ring(_p(rp), _p(dp), *_sz(rp.size), _p(vl), *_sz(vl.size, cap, t, e), _p(nv), ctypes.c_float(gamma),
                   ctypes.c_float(lam), _p(out["r"]), _p(out["v"]), _p(d_out), _p(out["adv"]), _p(out["ret"]),
                   _p(meta))
    return out["r"], out["v"], d_out, out["adv"], out["ret"], int(meta[0]), int(meta[1])


def ref_gae_available():
    return os.path.exists(REF_GAE)


def ref_gae(rewards, values, dones, next_values, gamma, lam):
    """The reference's own ReplayMemory::fused_compute_gae, compiled from its
    sources into oracle/_ref/libref_gae.so."""
    r = np.ascontiguousarray(rewards, np.float32)
    v = np.ascontiguousarray(values, np.float32)
    d = np.ascontiguousarray(dones, np.uint8)
    nv = np.ascontiguousarray(next_values, np.float32)
    t, e = r.shape
    adv = np.empty_like(r)
    ret = np.empty_like(r)
    L = ctypes.CDLL(REF_GAE)
    L.ref_gae(_p(r.ravel()), _p(v.ravel()), _p(d.ravel()), _p(nv), *_sz(t, e), ctypes.c_float(gamma),
              ctypes.c_float(lam), _p(adv), _p(ret))
    return adv, ret


def policy_head(logits, actions):
    """(log_probs [R][C], action_logp [R], entropy [R]) of the PPO rollout head."""
    logits = np.ascontiguousarray(logits, np.float32)
    actions = np.ascontiguousarray(actions, np.float32)
    r, c = logits.shape
    lp = np.empty((r, c), np.float32)
    alp = np.empty(r, np.float32)
    ent = np.empty(r, np.float32)
    lib().mxo_policy_head(_p(logits), _p(actions), *_sz(r, c), _p(lp), _p(alp), _p(ent))
    return lp, alp, ent


def moe(fmt, x, logits, d, f, k, experts):
    """experts: list of (wg, sg, wu, su, wd, sd) dense-with-zero-blocks."""
    x = np.ascontiguousarray(x, np.float32)
    logits = np.ascontiguousarray(logits, np.float32)
    t, e = logits.shape
    y = np.empty((t, d), np.float32)
    cols = list(zip(*experts))
    arrs = [[np.ascontiguousarray(a) for a in col] for col in cols]
    ptrs = [(ctypes.c_void_p * e)(*[a.ctypes.data for a in col]) for col in arrs]
    rc = lib().mxo_moe(ctypes.c_int(fmt), _p(x), _p(logits), *_sz(t, d, f, e, k), *ptrs, _p(y))
    if rc != 0:
        raise ValueError("moe: bad top-k")
    return y


# ------------------------------------------------------ CPU baseline ---
def weight_sums(fmt, w, n, k):
    out = np.empty((n, k // 32), np.int32)
    lib().mxb_weight_sums(ctypes.c_int(fmt), _p(np.ascontiguousarray(w)), *_sz(n, k), _p(out))
    return out


def baseline_gemv(fmt, xq, xs, w, ws, wsums, n, k, threads=0):
    """Multi-threaded dpbusd restatement; returns (y, used_vnni)."""
    xq = np.ascontiguousarray(xq, np.uint8)
    b = xq.shape[0]
    y = np.empty((b, n), np.float32)
    used = lib().mxb_gemv(ctypes.c_int(fmt), _p(xq), _p(np.ascontiguousarray(xs, np.uint8)),
                          _p(np.ascontiguousarray(w)), _p(np.ascontiguousarray(ws, np.uint8)),
                          _p(np.ascontiguousarray(wsums, np.int32)), *_sz(b, n, k), _p(y),
                          ctypes.c_int(threads))
    return y, bool(used)


def max_threads():
    return lib().mxb_max_threads()


# ----------------------------------------------- dense decoder (numpy) ---
# The steps around the MX linears in cpu_model_b200's dense decoder, stated
# in float64 (the exactly rounded references the GPU's fp32 steps are held
# to).  The reference has no transformer; RMSNorm follows
# nn/core/normalization.cpp:16-47 (out = in * (1 / sqrt(sum(in^2) / n + eps))
# * weight).
def rmsnorm(x, g, eps):
    x = np.asarray(x, np.float64)
    inv = 1.0 / np.sqrt((x * x).sum(-1, keepdims=True) / x.shape[-1] + eps)
    return (x * inv * np.asarray(g, np.float64)).astype(np.float32)


def rope_table(max_ctx, theta, hd=128):
    """cos/sin [max_ctx][hd/2] computed in double, rounded once (the table
    the library builds on the host)."""
    j = np.arange(hd // 2, dtype=np.float64)
    p = np.arange(max_ctx, dtype=np.float64)[:, None]
    ang = p * np.power(float(theta), -2.0 * j / hd)[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def rope_rotate(x, pos, cos, sin):
    """x [..., n_heads, hd] float32 at positions pos [...] -> rotated, with
    the GPU's float32 operations (x1 c - x2 s, x2 c + x1 s)."""
    half = x.shape[-1] // 2
    c = cos[pos][..., None, :]
    s = sin[pos][..., None, :]
    x1, x2 = x[..., :half], x[..., half:]
    return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], axis=-1).astype(np.float32)


def bf16_round(x):
    """float32 -> nearest bfloat16 (ties to even), returned as float32."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def attention(q, k, v, qpos):
    """q [Tq][H][hd] at positions qpos [Tq]; k, v [Tk][H][hd] at positions
    0..Tk-1; causal softmax(q k^T / sqrt(hd)) v in float64 -> [Tq][H*hd]."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    hd = q.shape[-1]
    s = np.einsum("qhd,khd->hqk", q, k) / np.sqrt(hd)
    mask = np.arange(k.shape[0])[None, :] > np.asarray(qpos)[:, None]
    s = np.where(mask[None], -np.inf, s)
    s -= s.max(-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(-1, keepdims=True)
    o = np.einsum("hqk,khd->qhd", p, v)
    return o.reshape(q.shape[0], -1)


def silu_mul(g, u):
    g = np.asarray(g, np.float64)
    return g / (1.0 + np.exp(-g)) * np.asarray(u, np.float64)


def log_softmax_at(logits, target):
    x = np.asarray(logits, np.float64)
    m = x.max(-1, keepdims=True)
    lse = m[:, 0] + np.log(np.exp(x - m).sum(-1))
    return x[np.arange(x.shape[0]), target] - lse
