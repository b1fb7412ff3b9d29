// mx_dropin.cpp -- a C++ caller of the reference's MX operator interface,
// written the way the reference's own code calls it (free functions on
// MXUINT8Tensor / MXINT8Tensor containers, nn/tests/autotest.hpp:93-136;
// HashedRouter{Config}.route(x, idx), nn/tests/test_robustness.cpp:13-35;
// halting_step(x_q, w_halt, b, state, halt), nn/core/layers/halting.hpp:24-30),
// compiled against include/nca_mx_linear.hpp and linked with libmxq.so.
//
//   mx_dropin <dir>
//
// Reads the raw inputs tests/test_cpp_dropin.py wrote to <dir>, runs every
// operator on the calling thread's default context, and writes the raw
// outputs back to <dir> for the test to check against the CPU oracle.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "nca_mx_linear.hpp"

using nca::linalg::MXINT8Tensor;
using nca::linalg::MXUINT8Tensor;

static std::string g_dir;

static std::vector<uint8_t> load(const char* name) {
  std::string p = g_dir + "/" + name;
  FILE* f = std::fopen(p.c_str(), "rb");
  if (!f) throw std::runtime_error("missing input " + p);
  std::vector<uint8_t> v;
  uint8_t buf[1 << 16];
  size_t n;
  while ((n = std::fread(buf, 1, sizeof(buf), f)) > 0) v.insert(v.end(), buf, buf + n);
  std::fclose(f);
  return v;
}

static void store(const char* name, const void* p, size_t bytes) {
  std::string path = g_dir + "/" + name;
  FILE* f = std::fopen(path.c_str(), "wb");
  if (!f || std::fwrite(p, 1, bytes, f) != bytes) throw std::runtime_error("cannot write " + path);
  std::fclose(f);
}

static void ck(cudaError_t e) {
  if (e != cudaSuccess) throw std::runtime_error(cudaGetErrorString(e));
}

// device copy of a host buffer (freed at exit by the process)
template <typename T>
static T* dev(const std::vector<uint8_t>& h) {
  void* p = nullptr;
  ck(cudaMalloc(&p, h.size() ? h.size() : 16));
  ck(cudaMemcpy(p, h.data(), h.size(), cudaMemcpyHostToDevice));
  return static_cast<T*>(p);
}

template <typename T>
static T* dev_zero(size_t count) {
  void* p = nullptr;
  ck(cudaMalloc(&p, count * sizeof(T) + 16));
  ck(cudaMemset(p, 0, count * sizeof(T) + 16));
  return static_cast<T*>(p);
}

template <typename T>
static std::vector<T> host(const T* d, size_t count) {
  std::vector<T> v(count);
  ck(cudaDeviceSynchronize());
  ck(cudaMemcpy(v.data(), d, count * sizeof(T), cudaMemcpyDeviceToHost));
  return v;
}

// an activation of `batch` rows of K (device)
static MXUINT8Tensor activation(size_t batch, size_t k) {
  MXUINT8Tensor a;
  a.data = dev_zero<uint8_t>(batch * k);
  a.scales = dev_zero<uint8_t>(batch * k / 32);
  a.num_blocks = k / 32;
  a.batch = batch;
  return a;
}

int main(int argc, char** argv) {
  if (argc != 2) {
    std::fprintf(stderr, "usage: %s <dir>\n", argv[0]);
    return 2;
  }
  g_dir = argv[1];
  try {
    const auto& ctx = nca::linalg::default_context();
    const size_t B = 3, K = 1024, N = 512;

    // mx_quantize_x + mx_gemv on an int8 weight
    auto x = load("x.f32");                      // [B][K]
    float* xd = dev<float>(x);
    MXUINT8Tensor xa = activation(B, K);
    nca::linalg::mx_quantize_x(xd, xa);
    MXINT8Tensor w(ctx, MXQ_FMT_INT8, N, K, load("w8.i8").data(), load("w8.s").data(), false);
    float* y = dev_zero<float>(B * N);
    nca::linalg::mx_gemv(xa, w, y);
    auto yh = host(y, B * N);
    store("y_gemv.f32", yh.data(), yh.size() * 4);
    auto xq = host(xa.data, B * K);
    store("xq.u8", xq.data(), xq.size());

    // mx_rank16_dot_ptrs over 16 one-row weights (the pointer-array form)
    auto r16 = load("rows16.i8");                 // [16][K]
    auto r16s = load("rows16.s");                 // [16][K/32]
    std::vector<MXINT8Tensor> rows;
    for (size_t j = 0; j < 16; ++j)
      rows.emplace_back(ctx, MXQ_FMT_INT8, 1, K, r16.data() + j * K, r16s.data() + j * (K / 32), false);
    const MXINT8Tensor* ptrs[16];
    for (size_t j = 0; j < 16; ++j) ptrs[j] = &rows[j];
    float* y16 = dev_zero<float>(B * 16);
    nca::linalg::mx_rank16_dot_ptrs(xa, ptrs, y16);
    auto y16h = host(y16, B * 16);
    store("y_rank16.f32", y16h.data(), y16h.size() * 4);

    // gated_mlp_step on int4 gate/up [F][D] and down [D][F]
    const size_t D = 512, F = 1024, BM = 2;
    MXINT8Tensor g(ctx, MXQ_FMT_INT4, F, D, load("mg.i4").data(), load("mg.s").data(), false);
    MXINT8Tensor u(ctx, MXQ_FMT_INT4, F, D, load("mu.i4").data(), load("mu.s").data(), false);
    MXINT8Tensor dn(ctx, MXQ_FMT_INT4, D, F, load("md.i4").data(), load("md.s").data(), false);
    float* xm = dev<float>(load("xm.f32"));
    float* ym = dev_zero<float>(BM * D);
    nca::layers::gated_mlp_step(xm, BM, g, u, dn, ym);
    auto ymh = host(ym, BM * D);
    store("y_mlp.f32", ymh.data(), ymh.size() * 4);

    // moe_swiglu: E experts (dense int4, d 256, ffn 256), T tokens, top-2
    const size_t E = 4, T = 32, DE = 256, FE = 256;
    auto eg = load("eg.i4"), eu = load("eu.i4"), ed = load("ed.i4");
    auto egs = load("eg.s"), eus = load("eu.s"), eds = load("ed.s");
    std::vector<MXINT8Tensor> G, U, Dn;
    const size_t mb = FE * DE / 2, ms = FE * DE / 32;
    for (size_t e = 0; e < E; ++e) {
      G.emplace_back(ctx, MXQ_FMT_INT4, FE, DE, eg.data() + e * mb, egs.data() + e * ms, false);
      U.emplace_back(ctx, MXQ_FMT_INT4, FE, DE, eu.data() + e * mb, eus.data() + e * ms, false);
      Dn.emplace_back(ctx, MXQ_FMT_INT4, DE, FE, ed.data() + e * mb, eds.data() + e * ms, false);
    }
    std::vector<const MXINT8Tensor*> gp, up, dp;
    for (size_t e = 0; e < E; ++e) {
      gp.push_back(&G[e]);
      up.push_back(&U[e]);
      dp.push_back(&Dn[e]);
    }
    float* xe = dev<float>(load("xe.f32"));
    float* le = dev<float>(load("le.f32"));
    float* ye = dev_zero<float>(T * DE);
    nca::layers::moe_swiglu(gp, up, dp, xe, le, T, 2, ye);
    auto yeh = host(ye, T * DE);
    store("y_moe.f32", yeh.data(), yeh.size() * 4);
    bool threw = false;
    try {
      nca::layers::moe_swiglu(gp, up, dp, xe, le, T, E + 1, ye);
    } catch (const std::invalid_argument&) {
      threw = true;
    }
    if (!threw) throw std::runtime_error("moe_swiglu: k > E did not throw invalid_argument");

    // halting_step on token 0 of xa, three steps with a host state
    MXINT8Tensor wh(ctx, MXQ_FMT_INT8, 1, K, load("wh.i8").data(), load("wh.s").data(), false);
    MXUINT8Tensor x0 = xa;
    x0.batch = 1;
    nca::layers::HaltingState st;
    std::vector<float> hal;
    for (int s = 0; s < 3; ++s) {
      bool halt = false;
      const float p = nca::layers::halting_step(x0, wh, -2.0f, st, halt);
      hal.push_back(p);
      hal.push_back(st.p_sum);
      hal.push_back(st.remainder);
      hal.push_back((float)st.steps);
      hal.push_back(halt ? 1.0f : 0.0f);
    }
    store("halting.f32", hal.data(), hal.size() * 4);

    // HashedRouter: the remainder case and the top-k bound
    nca::linalg::HashedRouter router({1024, 31, 2, 8});
    std::vector<float> ones(1024, 1.0f);
    std::vector<size_t> idx;
    router.route(ones.data(), idx);
    if (idx.size() != 2) throw std::runtime_error("HashedRouter: expected 2 indices");
    std::vector<int32_t> idx32(idx.begin(), idx.end());
    store("route.i32", idx32.data(), idx32.size() * 4);
    threw = false;
    try {
      nca::linalg::HashedRouter bad({1024, 10, 20, 8});
    } catch (const std::invalid_argument&) {
      threw = true;
    }
    if (!threw) throw std::runtime_error("HashedRouter: top_k > n_experts did not throw");

    // mx_quantize_w into a shaped int4 weight, then a gemv through it
    const size_t NQ = 64, KQ = 256;
    float* wf = dev<float>(load("wq.f32"));     // [NQ][KQ]
    MXINT8Tensor wq(MXQ_FMT_INT4, NQ, KQ);
    nca::linalg::mx_quantize_w(wf, wq);
    float* xqf = dev<float>(load("xq_in.f32"));  // [1][KQ]
    MXUINT8Tensor xqa = activation(1, KQ);
    nca::linalg::mx_quantize_x(xqf, xqa);
    float* yq = dev_zero<float>(NQ);
    nca::linalg::mx_gemv(xqa, wq, yq);
    auto yqh = host(yq, NQ);
    store("y_quantw.f32", yqh.data(), yqh.size() * 4);

    ctx.synchronize();
    std::printf("dropin ok\n");
    return 0;
  } catch (const std::exception& e) {
    std::fprintf(stderr, "dropin failed: %s\n", e.what());
    return 1;
  }
}
