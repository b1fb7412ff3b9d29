"""The C++ boundary as a drop-in: tests/cpp/mx_dropin.cpp calls the reference's
MX operator interface in the reference's own call shapes (include/
nca_mx_linear.hpp over libmxq.so), and its outputs are checked against the
CPU oracle on the same inputs.

- test_dropin_program_builds (CPU): the program compiles and links with g++
  against the header, libmxq.so and the CUDA runtime.
- test_dropin_program_matches_oracle (GPU): it runs, and mx_gemv,
  mx_rank16_dot_ptrs (16 MXINT8Tensor pointers), gated_mlp_step, moe_swiglu,
  halting_step, HashedRouter::route and mx_quantize_w agree with the oracle
  (fp32 within rel-L2 1e-5 or bit-exact, as each operator's contract says).
"""
import os
import subprocess

import numpy as np
import pytest

from oracle import oracle
from cpu_model_b200 import synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "cpp", "mx_dropin.cpp")
LIBDIR = os.path.join(ROOT, "cpu_model_b200")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
REL_TOL = 1e-5


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.linalg.norm(b)
    return np.linalg.norm(a - b) / (den if den > 0 else 1.0)


def build(out_dir):
    from cpu_model_b200 import build as b
    b.build()
    exe = os.path.join(out_dir, "mx_dropin")
    cmd = ["g++", "-std=c++20", "-O1", "-I" + os.path.join(ROOT, "include"), "-I" + os.path.join(CUDA, "include"),
           SRC, "-o", exe, "-L" + LIBDIR, "-lmxq", "-L" + os.path.join(CUDA, "lib64"), "-lcudart",
           "-Wl,-rpath," + LIBDIR + ":" + os.path.join(CUDA, "lib64")]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_dropin_program_builds(tmp_path):
    assert os.path.exists(build(str(tmp_path)))


def write_inputs(d):
    B, K, N = 3, 1024, 512
    inp = {}
    inp["x"] = synth.normal((B, K), 1)
    inp["w8"], inp["w8s"] = synth.weights(8, N, K, -10, -4, 2)
    inp["r16"], inp["r16s"] = synth.weights(8, 16, K, -10, -4, 3)
    D, F = 512, 1024
    inp["mg"], inp["mgs"] = synth.weights(4, F, D, -8, -3, 4)
    inp["mu"], inp["mus"] = synth.weights(4, F, D, -8, -3, 5)
    inp["md"], inp["mds"] = synth.weights(4, D, F, -8, -3, 6)
    inp["xm"] = synth.normal((2, D), 7)       # no SwiGLU value within 1e-3 of a rounding tie
    E, T, DE, FE = 4, 32, 256, 256
    ex = [[synth.weights(4, n, k, -7, -3, 100 + 10 * e + j) for j, (n, k) in enumerate(((FE, DE), (FE, DE), (DE, FE)))]
          for e in range(E)]
    inp["experts"] = ex
    inp["xe"] = synth.normal((T, DE), 28)     # no SwiGLU value within 1e-4 of a rounding tie
    inp["le"] = synth.normal((T, E), 9)
    inp["wh"], inp["whs"] = synth.weights(8, 1, K, -9, -7, 10)
    inp["wq"] = synth.normal((64, 256), 11) * np.float32(0.1)
    inp["xq_in"] = synth.normal((1, 256), 12)
    files = {"x.f32": inp["x"], "w8.i8": inp["w8"], "w8.s": inp["w8s"], "rows16.i8": inp["r16"],
             "rows16.s": inp["r16s"], "mg.i4": inp["mg"], "mg.s": inp["mgs"], "mu.i4": inp["mu"],
             "mu.s": inp["mus"], "md.i4": inp["md"], "md.s": inp["mds"], "xm.f32": inp["xm"],
             "eg.i4": np.stack([e[0][0] for e in ex]), "eg.s": np.stack([e[0][1] for e in ex]),
             "eu.i4": np.stack([e[1][0] for e in ex]), "eu.s": np.stack([e[1][1] for e in ex]),
             "ed.i4": np.stack([e[2][0] for e in ex]), "ed.s": np.stack([e[2][1] for e in ex]),
             "xe.f32": inp["xe"], "le.f32": inp["le"], "wh.i8": inp["wh"], "wh.s": inp["whs"],
             "wq.f32": inp["wq"], "xq_in.f32": inp["xq_in"]}
    for name, arr in files.items():
        np.ascontiguousarray(arr).tofile(os.path.join(d, name))
    return inp


@pytest.mark.gpu
def test_dropin_program_matches_oracle(tmp_path):
    d = str(tmp_path)
    exe = build(d)
    inp = write_inputs(d)
    r = subprocess.run([exe, d], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    rd = lambda name, dt: np.fromfile(os.path.join(d, name), dt)
    B, K, N = 3, 1024, 512

    xq, xs = oracle.quantize_x(inp["x"])
    assert np.array_equal(rd("xq.u8", np.uint8).reshape(B, K), xq)
    y = rd("y_gemv.f32", np.float32).reshape(B, N)
    assert rel_l2(y, oracle.gemv(8, xq, xs, inp["w8"], inp["w8s"], N, K)) <= REL_TOL

    rows = [inp["r16"][j:j + 1] for j in range(16)]
    scs = [inp["r16s"][j:j + 1] for j in range(16)]
    y16 = rd("y_rank16.f32", np.float32).reshape(B, 16)
    assert np.array_equal(y16, oracle.rank16_dot_ptrs(8, xq, xs, rows, scs, K))

    D, F = 512, 1024
    ym = rd("y_mlp.f32", np.float32).reshape(2, D)
    ref, _, _ = oracle.mlp_swiglu(4, inp["xm"], D, F, inp["mg"], inp["mgs"], inp["mu"], inp["mus"], inp["md"],
                                  inp["mds"])
    assert rel_l2(ym, ref) <= REL_TOL

    T, DE, FE = 32, 256, 256
    host_w = [(e[0][0], e[0][1], e[1][0], e[1][1], e[2][0], e[2][1]) for e in inp["experts"]]
    ye = rd("y_moe.f32", np.float32).reshape(T, DE)
    assert rel_l2(ye, oracle.moe(4, inp["xe"], inp["le"], DE, FE, 2, host_w)) <= REL_TOL

    hal = rd("halting.f32", np.float32).reshape(3, 5)
    ps, rm, st = np.zeros(1, np.float32), np.zeros(1, np.float32), np.zeros(1, np.uint64)
    for s in range(3):
        p, h = oracle.halting_step(8, xq[:1], xs[:1], inp["wh"], inp["whs"], K, -2.0, ps, rm, st)
        assert np.array_equal(hal[s], np.array([p[0], ps[0], rm[0], float(st[0]), float(h[0])], np.float32))

    idx, _ = oracle.hashed_route(np.ones((1, 1024), np.float32), 31, 2, 8, 0)
    assert np.array_equal(rd("route.i32", np.int32), idx[0])

    dq, sq, _ = oracle.quantize_w(4, inp["wq"])
    xq2, xs2 = oracle.quantize_x(inp["xq_in"])
    yq = rd("y_quantw.f32", np.float32).reshape(1, 64)
    assert rel_l2(yq, oracle.gemv(4, xq2, xs2, dq, sq, 64, 256)) <= REL_TOL
