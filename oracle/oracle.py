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
