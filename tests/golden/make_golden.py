"""Generates the committed golden fixtures in this folder.

    python tests/golden/make_golden.py

gae_ring_reference.npz -- the same function on the reference's own ring
    buffer (ReplayMemory with capacity < items pushed, a sweep cut to what is
    stored, more than its MAX_ENVS = 1024 environments), through
    oracle/_ref's ref_gae_ring; the advantages/returns of the whole ring.

gae_reference.npz -- outputs of the REFERENCE's own
    nca::env::ReplayMemory::fused_compute_gae, compiled from its sources
    (agentic_env/replay_memory.cpp) into oracle/_ref/libref_gae.so by
    oracle/Makefile, on seeded inputs (plus the 2-env x 3-step case of
    agentic_env/test_memory.cpp:47-83).  These pin the GAE restatement.

mx_oracle.npz -- small MX cases (int8 and int4 weights, several batch sizes,
    edge blocks) computed by the CPU oracle.  The reference's MX kernels are
    absent from its snapshot, so these are self-fixtures of the restatement
    (parity unpinned): they freeze the contract so that a change to the oracle
    or to the GPU path is caught, and they travel to the GPU box.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle  # noqa: E402
from cpu_model_b200 import synth  # noqa: E402


def gae_cases():
    cases = {}
    # agentic_env/test_memory.cpp:47-83 (push order: env0, env1 per step)
    cases["kat_r"] = np.array([[1, 4], [2, 5], [3, 6]], np.float32)
    cases["kat_v"] = np.array([[10, 20], [9, 19], [8, 18]], np.float32)
    cases["kat_d"] = np.array([[0, 0], [0, 0], [1, 0]], np.uint8)
    cases["kat_nv"] = np.array([0, 17], np.float32)
    g = synth.rng(7)
    T, E = 64, 32
    cases["rand_r"] = g.standard_normal((T, E), dtype=np.float32)
    cases["rand_v"] = g.standard_normal((T, E), dtype=np.float32)
    cases["rand_d"] = (g.random((T, E)) < 0.05).astype(np.uint8)
    cases["rand_nv"] = g.standard_normal(E, dtype=np.float32)
    return cases


def make_gae():
    if not oracle.ref_gae_available():
        oracle.build()
    if not oracle.ref_gae_available():
        raise SystemExit("oracle/_ref/libref_gae.so missing: the reference sources are needed")
    c = gae_cases()
    out = dict(c)
    for name in ("kat", "rand"):
        adv, ret = oracle.ref_gae(c[name + "_r"], c[name + "_v"], c[name + "_d"], c[name + "_nv"], 0.99, 0.95)
        out[name + "_adv"] = adv
        out[name + "_ret"] = ret
    np.savez_compressed(os.path.join(HERE, "gae_reference.npz"), **out)


# (capacity, items pushed, rollout_steps T, envs E): a wrapped ring, a full
# ring with the cursor back at 0, a sweep cut to what is stored, more than the
# reference's MAX_ENVS = 1024 environments (the rest of the ring untouched),
# and a wrapped ring of wide rows
GAE_RING_CASES = [(100, 250, 10, 7), (64, 64, 8, 8), (50, 30, 10, 4), (3000, 3000, 2, 1500),
                  (1000, 1700, 5, 150)]


def make_gae_ring():
    """Outputs of the reference's own ReplayMemory ring: items pushed one by
    one (wrapping), the latest values written, fused_compute_gae(T, E)."""
    out = {}
    g = synth.rng(11)
    for i, (cap, npush, t, e) in enumerate(GAE_RING_CASES):
        rp = g.standard_normal(npush, dtype=np.float32)
        dp = (g.random(npush) < 0.1).astype(np.uint8)
        vl = g.standard_normal(min(t * e, min(npush, cap)), dtype=np.float32)
        nv = g.standard_normal(e, dtype=np.float32)
        r, v, d, adv, ret, size, cur = oracle.ref_gae_ring(rp, dp, vl, cap, t, e, nv, 0.99, 0.95)
        p = "c%d_" % i
        out.update({p + "r": r, p + "v": v, p + "d": d, p + "nv": nv, p + "adv": adv, p + "ret": ret,
                    p + "meta": np.array([cap, size, cur, t, e], np.int64)})
    np.savez_compressed(os.path.join(HERE, "gae_ring_reference.npz"), **out)


def make_mx():
    out = {}
    cases = [
        ("i8_b1", 8, 1, 64, 96, 0),
        ("i8_b3", 8, 3, 40, 160, 1),
        ("i4_b1", 4, 1, 64, 128, 2),
        ("i4_b5", 4, 5, 33, 96, 3),
        ("i4_b20", 4, 20, 130, 192, 4),
    ]
    for name, fmt, b, n, k, seed in cases:
        w, ws = synth.weights(fmt, n, k, -10, -4, seed)
        x = synth.normal((b, k), seed + 100)
        x[0, :32] = 0.0                      # an all-zero block
        if b > 1:
            x[1, 32:64] *= 1e-3              # a small-magnitude block
        xq, xs = oracle.quantize_x(x)
        out[name + "_w"] = w
        out[name + "_ws"] = ws
        out[name + "_x"] = x
        out[name + "_xq"] = xq
        out[name + "_xs"] = xs
        out[name + "_dots"] = oracle.block_dots(fmt, xq, w, n, k)
        out[name + "_y"] = oracle.gemv(fmt, xq, xs, w, ws, n, k)
        out[name + "_shape"] = np.array([fmt, b, n, k], np.int64)
    np.savez_compressed(os.path.join(HERE, "mx_oracle.npz"), **out)


if __name__ == "__main__":
    make_gae()
    make_gae_ring()
    make_mx()
    print("wrote", os.listdir(HERE))
