// mxq_api.cu -- the C-ABI (include/mxq.h): contexts, weight handles,
// workspace, regime selection and the small kernels (weight repack, top-k
// routing, GAE).  No exception crosses the boundary; every entry returns an
// MXQ_* status.
#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <cstdarg>
#include <new>
#include <string>
#include <vector>

#include "../../include/mxq.h"
#include "mxq_internal.h"

using namespace mxq;

struct mxq_context {
  int device = 0;
  cudaStream_t stream = nullptr;
  int path = MXQ_PATH_AUTO;
  uint32_t* status = nullptr;  // device status word (bounded waits that gave up)
  uint32_t* status_host = nullptr;  // pinned mirror, read after one stream sync
  uint64_t launches = 0;
  std::string err;
  // workspace (device)
  uint8_t* ws_q = nullptr;   size_t ws_q_bytes = 0;    // MX activation
  uint8_t* ws_s = nullptr;   size_t ws_s_bytes = 0;    // MX scales
  uint8_t* ws_op = nullptr;  size_t ws_op_bytes = 0;   // GEMM operand
  float* ws_f0 = nullptr;    size_t ws_f0_bytes = 0;   // fp32 intermediates
  float* ws_f1 = nullptr;    size_t ws_f1_bytes = 0;
  uint32_t* ws_cnt = nullptr; size_t ws_cnt_bytes = 0; // block counters of MX-output GEMVs (kept zero)
  float* ws_in = nullptr;    size_t ws_in_bytes = 0;   // host-call staging
  float* ws_out = nullptr;   size_t ws_out_bytes = 0;
  // MoE: routing bookkeeping, per-route expert outputs, pinned route counts
  int32_t* ws_moe = nullptr; size_t ws_moe_bytes = 0;
  float* ws_yr = nullptr;    size_t ws_yr_bytes = 0;
  int32_t* moe_counts_host = nullptr; size_t moe_counts_cap = 0;
  // MoE expert lanes: experts run round-robin on kMoeLanes streams, each with
  // its own operand and gate/up workspaces, forked from and joined to the
  // caller's stream (consecutive experts' GEMMs overlap their tails)
  static constexpr int kMoeLanes = 3;
  cudaStream_t moe_st[kMoeLanes] = {};
  cudaEvent_t moe_ev[kMoeLanes + 1] = {};
  uint8_t* ml_op[kMoeLanes] = {}; size_t ml_op_bytes[kMoeLanes] = {};
  float* ml_f0[kMoeLanes] = {};   size_t ml_f0_bytes[kMoeLanes] = {};
  float* ml_f1[kMoeLanes] = {};   size_t ml_f1_bytes[kMoeLanes] = {};
  // host-buffer entry points: pinned staging and one CUDA graph per
  // (call, weights, batch); ws_gen changes whenever a workspace moves, which
  // retires every captured graph
  uint64_t ws_gen = 1;
  cudaStream_t hstream = nullptr;   // private stream of the host-buffer calls (capturable)
  cudaEvent_t hevent = nullptr;
  // small host calls: mapped pinned buffers read and written by kernels, a
  // device sequence counter and the host's mirror of it
  uint32_t* seq_dev = nullptr;
  uint32_t host_seq = 0;
  float* pin_in = nullptr;  size_t pin_in_bytes = 0;
  float* pin_out = nullptr; size_t pin_out_bytes = 0;
  struct HostGraph {
    int kind;
    uint64_t w1, w2;
    size_t b;
    uint64_t gen;
    cudaStream_t stream;
    cudaGraphExec_t exec;   // null: capture failed, run uncaptured
    bool mapped;            // copies by kernels through mapped memory, completion by a flag
    uint64_t used;          // last call that used it (LRU)
  };
  // at most kMaxHostGraphs recorded calls; the least recently used goes
  static constexpr size_t kMaxHostGraphs = 64;
  std::vector<HostGraph> graphs;
  uint64_t graph_clock = 0;
};

struct mxq_weight_s {
  mxq_context* ctx = nullptr;
  uint64_t serial = 0;        // unique per created weight (graph cache keys)
  WeightView v{};
  uint8_t* data = nullptr;
  uint8_t* scales = nullptr;
  int32_t* tiles = nullptr;   // block-sparse: kt_ptr then kt_idx (device)
};

namespace {

thread_local std::string g_err;

int fail(mxq_context* c, int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  if (c) c->err = buf;
  g_err = buf;
  return code;
}

int cuda_fail(mxq_context* c, cudaError_t e, const char* what) {
  return fail(c, e == cudaErrorMemoryAllocation ? MXQ_ERR_OUT_OF_MEMORY : MXQ_ERR_CUDA,
              "%s: %s", what, cudaGetErrorString(e));
}

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) == cudaSuccess && prev != dev) cudaSetDevice(dev);
    else prev = -1;
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

template <typename T>
int ensure(mxq_context* c, T*& p, size_t& cap, size_t bytes, const char* what) {
  if (bytes <= cap) return MXQ_OK;
  ++c->ws_gen;
  if (p) cudaFree(p);
  p = nullptr;
  cap = 0;
  void* q = nullptr;
  cudaError_t e = cudaMalloc(&q, bytes);
  if (e != cudaSuccess) return cuda_fail(c, e, what);
  p = static_cast<T*>(q);
  cap = bytes;
  return MXQ_OK;
}

// A workspace of counters that the kernels using it leave zero: zeroed once
// when (re)allocated, in stream order before its first use.
int ensure_zeroed(mxq_context* c, uint32_t*& p, size_t& cap, size_t bytes, const char* what) {
  if (bytes <= cap) return MXQ_OK;
  if (int rc = ensure(c, p, cap, bytes, what)) return rc;
  const cudaError_t e = cudaMemsetAsync(p, 0, cap, c->stream);
  return e == cudaSuccess ? MXQ_OK : cuda_fail(c, e, what);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

uint64_t next_weight_serial() {
  static std::atomic<uint64_t> n{0};
  return ++n;
}

// Pinned host staging for the host-buffer entry points (moves bump ws_gen).
int ensure_pinned(mxq_context* c, float*& p, size_t& cap, size_t bytes, const char* what) {
  if (bytes <= cap) return MXQ_OK;
  ++c->ws_gen;
  if (p) cudaFreeHost(p);
  p = nullptr;
  cap = 0;
  void* q = nullptr;
  cudaError_t e = cudaHostAlloc(&q, bytes, cudaHostAllocMapped);
  if (e != cudaSuccess) return cuda_fail(c, e, what);
  p = static_cast<float*>(q);
  cap = bytes;
  return MXQ_OK;
}

// ------------------------------------------------------------ repack ---
__global__ void repack_kernel(const uint8_t* __restrict__ data,
                              const uint8_t* __restrict__ scales, int fmt, int N,
                              int K, int Npad, int Kpad, uint8_t* __restrict__ od,
                              uint8_t* __restrict__ os) {
  const int TB = fmt == 4 ? 32 : 64;
  const int KT = Kpad / kTileK;
  const long total = (long)Npad * KT;
  const int row_bytes = fmt == 4 ? K / 2 : K;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long)gridDim.x * blockDim.x) {
    const int n = (int)(i / KT), kt = (int)(i % KT);
    const long dst = (((long)(n / 128) * KT + kt) * 128 + (n % 128));
    for (int j = 0; j < TB; ++j) {
      const int byte = kt * TB + j;
      od[dst * TB + j] = (n < N && byte < row_bytes) ? data[(long)n * row_bytes + byte] : 0;
    }
    for (int h = 0; h < 2; ++h) {
      const int b = kt * 2 + h;
      os[dst * 2 + h] = (n < N && b < K / kBlock) ? scales[(long)n * (K / kBlock) + b] : 127;
    }
  }
}

// Block-sparse repack: one thread per (stored tile, row).  Stored tile ti
// holds k-tile tile_kt[ti] of row tile tile_rt[ti]; rows whose 64x64 block
// is masked out (or beyond N) are stored as zero weights with scale 127.
__global__ void repack_bsr_kernel(const uint8_t* __restrict__ data,
                                  const uint8_t* __restrict__ scales,
                                  const uint8_t* __restrict__ mask, int fmt, int N, int K,
                                  const int32_t* __restrict__ tile_rt, const int32_t* __restrict__ tile_kt,
                                  long ntiles, uint8_t* __restrict__ od, uint8_t* __restrict__ os) {
  const int TB = fmt == 4 ? 32 : 64;
  const int row_bytes = fmt == 4 ? K / 2 : K;
  const int KB = K / kTileK;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < ntiles * 128;
       i += (long)gridDim.x * blockDim.x) {
    const long ti = i / 128;
    const int r = (int)(i % 128);
    const int n = tile_rt[ti] * 128 + r, kt = tile_kt[ti];
    const bool keep = n < N && mask[(long)(n / 64) * KB + kt] != 0;
    for (int j = 0; j < TB; ++j)
      od[i * TB + j] = keep ? data[(long)n * row_bytes + (long)kt * TB + j] : 0;
    for (int h = 0; h < 2; ++h)
      os[i * 2 + h] = keep ? scales[(long)n * (K / kBlock) + kt * 2 + h] : 127;
  }
}

// Range of the weight scale bytes (selects the GEMV's fast scale path) and
// the largest finite one (sets the tensor-core path's exponent shift).
__global__ void scale_range_kernel(const uint8_t* __restrict__ s, size_t n, uint32_t* out) {
  uint32_t lo = 255, hi = 0, hif = 0;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const uint32_t v = s[i];
    lo = min(lo, v);
    hi = max(hi, v);
    if (v != 255u) hif = max(hif, v);
  }
  for (int o = 16; o > 0; o >>= 1) {
    lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
    hif = max(hif, __shfl_xor_sync(0xffffffffu, hif, o));
  }
  if ((threadIdx.x & 31) == 0) {
    atomicMin(&out[0], lo);
    atomicMax(&out[1], hi);
    atomicMax(&out[2], hif);
  }
}

// ------------------------------------------------------------ routing ---
__global__ void route_topk_kernel(const float* __restrict__ logits, int T, int E,
                                  int k, int32_t* __restrict__ idx,
                                  float* __restrict__ gate) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  const float* l = logits + (long)t * E;
  int32_t id[64];
  float ex[64];
  for (int j = 0; j < k; ++j) {
    int best = -1;
    for (int e = 0; e < E; ++e) {
      bool used = false;
      for (int p = 0; p < j; ++p) used |= id[p] == e;
      if (used) continue;
      if (best < 0 || l[e] > l[best]) best = e;
    }
    id[j] = best;
  }
  const float mx = l[id[0]];
  float den = 0.0f;
  for (int j = 0; j < k; ++j) {
    ex[j] = det_expf(__fsub_rn(l[id[j]], mx));
    den = __fadd_rn(den, ex[j]);
  }
  for (int j = 0; j < k; ++j) {
    idx[(long)t * k + j] = id[j];
    gate[(long)t * k + j] = __fdiv_rn(ex[j], den);
  }
}

// ---------------------------------------------------------------- GAE ---
// agentic_env/replay_memory.cpp:230-251: backward over t, one thread per env,
// the reference's float operations in the reference's order.
__global__ void gae_kernel(const float* __restrict__ r, const float* __restrict__ v,
                           const uint8_t* __restrict__ d, const float* __restrict__ nv,
                           int T, int E, float gamma, float gl,
                           float* __restrict__ adv, float* __restrict__ ret) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= E) return;
  float acc = 0.0f, vn = nv[k];
  for (int t = T - 1; t >= 0; --t) {
    const long i = (long)t * E + k;
    const float df = d[i] ? 0.0f : 1.0f;
    const float vt = v[i];
    const float delta = __fsub_rn(__fadd_rn(r[i], __fmul_rn(__fmul_rn(gamma, vn), df)), vt);
    acc = __fadd_rn(delta, __fmul_rn(__fmul_rn(gl, acc), df));
    adv[i] = acc;
    ret[i] = __fadd_rn(acc, vt);
    vn = vt;
  }
}

// The same sweep on the ReplayMemory ring (agentic_env/replay_memory.cpp:
// 210-251): items start at `start`, indices wrap once at `cap`, one thread
// per environment of the first `active`.
__global__ void gae_ring_kernel(const float* __restrict__ r, const float* __restrict__ v,
                                const uint8_t* __restrict__ d, const float* __restrict__ nv,
                                long cap, long start, int T, int E, int active, float gamma, float gl,
                                float* __restrict__ adv, float* __restrict__ ret) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= active) return;
  float acc = 0.0f, vn = nv[k];
  for (int t = T - 1; t >= 0; --t) {
    long i = start + (long)t * E + k;
    if (i >= cap) i -= cap;
    const float df = d[i] ? 0.0f : 1.0f;
    const float vt = v[i];
    const float delta = __fsub_rn(__fadd_rn(r[i], __fmul_rn(__fmul_rn(gamma, vn), df)), vt);
    acc = __fadd_rn(delta, __fmul_rn(__fmul_rn(gl, acc), df));
    adv[i] = acc;
    ret[i] = __fadd_rn(acc, vt);
    vn = vt;
  }
}

// ------------------------------------------------------- policy head ---
// training/ppo_trainer.cpp:64-66 and :77: one warp per row; max by shuffles,
// sums by a fixed shuffle tree (deterministic), exp by det_expf.
__device__ __forceinline__ float warp_sum_fixed(float v) {
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__global__ void policy_head_kernel(const float* __restrict__ x, const float* __restrict__ a, int rows,
                                   int cols, float* __restrict__ lp, float* __restrict__ alp,
                                   float* __restrict__ ent) {
  const int row = (int)(((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;                       // whole warps leave together
  const float* xr = x + (long)row * cols;
  const float* ar = a + (long)row * cols;
  float* lr = lp + (long)row * cols;
  float m = -3.402823466e38f;
  for (int j = lane; j < cols; j += 32) m = fmaxf(m, xr[j]);
  m = warp_max(m, 32);
  float s = 0.0f;
  for (int j = lane; j < cols; j += 32) s = __fadd_rn(s, det_expf(__fsub_rn(xr[j], m)));
  s = warp_sum_fixed(s);
  const float lse = __fadd_rn(m, logf(s));
  float sa = 0.0f, se = 0.0f;
  for (int j = lane; j < cols; j += 32) {
    const float l = __fsub_rn(xr[j], lse);
    lr[j] = l;
    sa = __fadd_rn(sa, __fmul_rn(l, ar[j]));
    se = __fsub_rn(se, __fmul_rn(det_expf(l), l));
  }
  sa = warp_sum_fixed(sa);
  se = warp_sum_fixed(se);
  if (lane == 0) {
    alp[row] = sa;
    ent[row] = se;
  }
}

// ------------------------------------------------- host-call transfers ---
// Small host calls move their data through mapped pinned memory with
// kernels: the input is read from host memory by one CTA, and the output,
// the status word and a fresh sequence number are written back by one CTA,
// the sequence number last, after a system-scope fence, so the host can
// poll for it instead of a stream synchronisation.
__global__ void host_in_kernel(float* __restrict__ dst, const float* __restrict__ src, size_t n) {
  for (size_t i = threadIdx.x; i < n / 4; i += blockDim.x)
    reinterpret_cast<float4*>(dst)[i] = reinterpret_cast<const float4*>(src)[i];
  for (size_t i = n / 4 * 4 + threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
}

__global__ void host_out_kernel(const float* __restrict__ src, float* dst, size_t n, const uint32_t* status,
                                uint32_t* status_host, uint32_t* seq_dev, volatile uint32_t* flag_host) {
  for (size_t i = threadIdx.x; i < n / 4; i += blockDim.x)
    reinterpret_cast<float4*>(dst)[i] = reinterpret_cast<const float4*>(src)[i];
  for (size_t i = n / 4 * 4 + threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
  __syncthreads();
  if (threadIdx.x == 0) {
    *status_host = *status;
    const uint32_t v = *seq_dev + 1;
    *seq_dev = v;
    __threadfence_system();
    *flag_host = v;
  }
}

int check_ctx(mxq_context* c) {
  return c ? MXQ_OK : fail(nullptr, MXQ_ERR_INVALID_ARGUMENT, "null context");
}

int check_weight(mxq_context* c, mxq_weight w) {
  if (!w || !w->data) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null weight handle");
  return MXQ_OK;
}

int use_gemv(mxq_context* c, size_t b, const mxq_weight_s* w) {
  if (w->v.kt_ptr) return 0;   // block-sparse: the GEMM walks the tile list
  if (c->path == MXQ_PATH_GEMV) return 1;
  if (c->path == MXQ_PATH_GEMM) return 0;
  return b <= (size_t)kGemvAutoBatch || bgemv_supported(w->v, (int)b);
}

// Batches the GEMV kernels take for this weight.
int gemv_batch_ok(const mxq_weight_s* w, size_t b) {
  return b <= (size_t)gemv_max_batch() || bgemv_supported(w->v, (int)b);
}

int after_launch(mxq_context* c, cudaError_t e, const char* what) {
  if (e != cudaSuccess) return cuda_fail(c, e, what);
  c->launches++;
  return MXQ_OK;
}

// launch_rgemv, counting every kernel it launched
static int rgemv_call(mxq_context* c, const GemvArgs& ga) {
  const int rc = after_launch(c, launch_rgemv(ga, c->stream, true), "gemv");
  if (rc == MXQ_OK) c->launches += (uint64_t)(rgemv_launches(ga) - 1);
  return rc;
}

// The batch-1 co-resident GEMV (mxq_cogemv.cu) takes this weight and input.
static bool gemv1_ok(const mxq_weight_s* w, bool inf32, bool qout) {
  return cogemv_supported(w->v, 1, inf32, qout);
}

// Decode GEMV straight from fp32 rows (quantised inside the kernel).  `next`
// (optional) is the weight the following call will read: its bytes are
// prefetched into L2 while this GEMV streams (cp.async-ring and weight-
// resident kernels), so the next layer starts warm.
int gemv_f32(mxq_context* c, mxq_weight w, const float* x, size_t b, float* y, mxq_weight next) {
  if (b == 1 && !gemv1_ok(w, true, false) && gemv1_ok(w, false, false)) {
    // batch 1, the fp32 row too long to stage next to the resident weights:
    // quantise it first, then the co-resident GEMV on MX input
    const int K = w->v.K;
    int rc;
    if ((rc = ensure(c, c->ws_q, c->ws_q_bytes, (size_t)K, "workspace q"))) return rc;
    if ((rc = ensure(c, c->ws_s, c->ws_s_bytes, (size_t)K / kBlock, "workspace s"))) return rc;
    QuantArgs qa{};
    qa.x = x;
    qa.B = 1;
    qa.K = K;
    qa.out_q = c->ws_q;
    qa.out_s = c->ws_s;
    if ((rc = after_launch(c, launch_quantize(qa, MXQ_ACT_NONE, c->stream, true), "quantize"))) return rc;
    GemvArgs ga{};
    ga.w = w->v;
    ga.xq = c->ws_q;
    ga.xs = c->ws_s;
    ga.y = y;
    ga.B = 1;
    return rgemv_call(c, ga);
  }
  if (bgemv_supported(w->v, (int)b)) {
    // small batch: MX-quantise the rows, then the MMA GEMV
    const int K = w->v.K;
    int rc;
    if ((rc = ensure(c, c->ws_q, c->ws_q_bytes, b * K, "workspace q"))) return rc;
    if ((rc = ensure(c, c->ws_s, c->ws_s_bytes, b * K / kBlock, "workspace s"))) return rc;
    QuantArgs qa{};
    qa.x = x;
    qa.B = (int)b;
    qa.K = K;
    qa.out_q = c->ws_q;
    qa.out_s = c->ws_s;
    if ((rc = after_launch(c, launch_quantize(qa, MXQ_ACT_NONE, c->stream, true), "quantize"))) return rc;
    GemvArgs ga{};
    ga.w = w->v;
    ga.xq = c->ws_q;
    ga.xs = c->ws_s;
    ga.y = y;
    ga.B = (int)b;
    return after_launch(c, launch_bgemv(ga, c->stream, true), "gemv");
  }
  GemvArgs ga{};
  ga.w = w->v;
  ga.xf = x;
  ga.y = y;
  ga.B = (int)b;
  if (next) {
    ga.pf_ptr = next->data;
    ga.pf_bytes = (size_t)next->v.Npad * next->v.Kpad / (next->v.fmt == 4 ? 2 : 1);
    ga.pf_ptr2 = next->scales;
    ga.pf_bytes2 = (size_t)next->v.Npad * next->v.Kpad / kBlock;
  }
  if (rgemv_supported(w->v, (int)b)) return rgemv_call(c, ga);
  return after_launch(c, launch_gemv(ga, c->stream, true), "gemv");
}

// fp32 x [B][K] (device) -> y [B][N] through quantise + GEMV or GEMM.
int linear_dev(mxq_context* c, mxq_weight w, const float* x, size_t b, float* y,
               int act) {
  const int K = w->v.K;
  int rc;
  if (use_gemv(c, b, w)) {
    if (!gemv_batch_ok(w, b))
      return fail(c, MXQ_ERR_INVALID_ARGUMENT, "GEMV path supports batch <= %d for this weight", gemv_max_batch());
    if (act == MXQ_ACT_NONE) return gemv_f32(c, w, x, b, y, nullptr);
    if ((rc = ensure(c, c->ws_q, c->ws_q_bytes, b * K, "workspace q"))) return rc;
    if ((rc = ensure(c, c->ws_s, c->ws_s_bytes, b * K / kBlock, "workspace s"))) return rc;
    QuantArgs qa{};
    qa.x = x;
    qa.B = (int)b;
    qa.K = K;
    qa.out_q = c->ws_q;
    qa.out_s = c->ws_s;
    if ((rc = after_launch(c, launch_quantize(qa, act, c->stream, true), "quantize"))) return rc;
    GemvArgs ga{};
    ga.w = w->v;
    ga.xq = c->ws_q;
    ga.xs = c->ws_s;
    ga.y = y;
    ga.B = (int)b;
    if (bgemv_supported(w->v, (int)b)) return after_launch(c, launch_bgemv(ga, c->stream, true), "gemv");
    return after_launch(c, launch_gemv(ga, c->stream, true), "gemv");
  }
  const int BN = gemm_pick_bn((int)b);
  const int Bpad = (int)((b + BN - 1) / BN * BN);
  if ((rc = ensure(c, c->ws_op, c->ws_op_bytes, (size_t)Bpad * w->v.Kpad * 2, "workspace operand")))
    return rc;
  QuantArgs qa{};
  qa.x = x;
  qa.B = (int)b;
  qa.K = K;
  qa.opnd = reinterpret_cast<__nv_bfloat16*>(c->ws_op);
  qa.Bpad = Bpad;
  qa.Kpad = w->v.Kpad;
  qa.BN = BN;
  qa.int4_order = w->v.fmt == 4;
  qa.shift = w->v.gemm_shift;
  if ((rc = after_launch(c, launch_quantize(qa, act, c->stream, true), "quantize"))) return rc;
  GemmArgs ga{};
  ga.w = w->v;
  ga.opnd = qa.opnd;
  ga.y = y;
  ga.B = (int)b;
  ga.Bpad = Bpad;
  ga.BN = BN;
  ga.status = c->status;
  return after_launch(c, launch_gemm(ga, c->stream, true), "gemm");
}

// MX activation (device) -> y
int gemv_dev(mxq_context* c, mxq_weight w, const uint8_t* xq, const uint8_t* xs,
             size_t b, float* y) {
  int rc;
  if (use_gemv(c, b, w)) {
    if (!gemv_batch_ok(w, b))
      return fail(c, MXQ_ERR_INVALID_ARGUMENT, "GEMV path supports batch <= %d for this weight", gemv_max_batch());
    GemvArgs ga{};
    ga.w = w->v;
    ga.xq = xq;
    ga.xs = xs;
    ga.y = y;
    ga.B = (int)b;
    if (bgemv_supported(w->v, (int)b)) return after_launch(c, launch_bgemv(ga, c->stream, true), "gemv");
    if (rgemv_supported(w->v, (int)b)) return rgemv_call(c, ga);
    return after_launch(c, launch_gemv(ga, c->stream, true), "gemv");
  }
  const int BN = gemm_pick_bn((int)b);
  const int Bpad = (int)((b + BN - 1) / BN * BN);
  if ((rc = ensure(c, c->ws_op, c->ws_op_bytes, (size_t)Bpad * w->v.Kpad * 2, "workspace operand")))
    return rc;
  QuantArgs qa{};
  qa.in_q = xq;
  qa.in_s = xs;
  qa.B = (int)b;
  qa.K = w->v.K;
  qa.opnd = reinterpret_cast<__nv_bfloat16*>(c->ws_op);
  qa.Bpad = Bpad;
  qa.Kpad = w->v.Kpad;
  qa.BN = BN;
  qa.int4_order = w->v.fmt == 4;
  qa.shift = w->v.gemm_shift;
  if ((rc = after_launch(c, launch_quantize(qa, 3, c->stream, true), "operand"))) return rc;
  GemmArgs ga{};
  ga.w = w->v;
  ga.opnd = qa.opnd;
  ga.y = y;
  ga.B = (int)b;
  ga.Bpad = Bpad;
  ga.BN = BN;
  ga.status = c->status;
  return after_launch(c, launch_gemm(ga, c->stream, true), "gemm");
}

}  // namespace

#define MXQ_TRY(...)                                                     \
  try {                                                                  \
    __VA_ARGS__                                                          \
  } catch (const std::bad_alloc&) {                                      \
    return fail(nullptr, MXQ_ERR_OUT_OF_MEMORY, "host allocation failed"); \
  } catch (...) {                                                        \
    return fail(nullptr, MXQ_ERR_CUDA, "unexpected exception");          \
  }

extern "C" {

int mxq_abi_version(void) { return 1; }

const char* mxq_last_error(mxq_ctx ctx) {
  return ctx ? ctx->err.c_str() : g_err.c_str();
}

int mxq_create(int device, mxq_ctx* out) {
  MXQ_TRY({
    if (!out) return fail(nullptr, MXQ_ERR_INVALID_ARGUMENT, "null output pointer");
    *out = nullptr;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaGetDeviceCount");
    if (device < 0 || device >= n)
      return fail(nullptr, MXQ_ERR_INVALID_ARGUMENT, "device %d out of range (%d devices)", device, n);
    DeviceGuard g(device);
    cudaDeviceProp prop;
    e = cudaGetDeviceProperties(&prop, device);
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaGetDeviceProperties");
    if (prop.major != 10)
      return fail(nullptr, MXQ_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a",
                  device, prop.major, prop.minor);
    auto* c = new mxq_context();
    c->device = device;
    e = cudaMalloc(&c->status, 4 * sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMemset(c->status, 0, 4 * sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaHostAlloc(&c->status_host, sizeof(uint32_t), cudaHostAllocDefault);
    if (e != cudaSuccess) {
      delete c;
      return cuda_fail(nullptr, e, "status word");
    }
    *out = c;
    return MXQ_OK;
  })
}

int mxq_destroy(mxq_ctx c) {
  MXQ_TRY({
    if (int rc = check_ctx(c)) return rc;
    DeviceGuard g(c->device);
    cudaStreamSynchronize(c->stream);
    cudaFree(c->status);
    cudaFreeHost(c->status_host);
    cudaFree(c->ws_q);
    cudaFree(c->ws_s);
    cudaFree(c->ws_op);
    cudaFree(c->ws_f0);
    cudaFree(c->ws_f1);
    cudaFree(c->ws_cnt);
    cudaFree(c->ws_in);
    cudaFree(c->ws_out);
    cudaFree(c->ws_moe);
    cudaFree(c->ws_yr);
    for (auto& g : c->graphs)
      if (g.exec) cudaGraphExecDestroy(g.exec);
    if (c->pin_in) cudaFreeHost(c->pin_in);
    if (c->pin_out) cudaFreeHost(c->pin_out);
    if (c->hstream) cudaStreamSynchronize(c->hstream), cudaStreamDestroy(c->hstream);
    if (c->hevent) cudaEventDestroy(c->hevent);
    if (c->seq_dev) cudaFree(c->seq_dev);
    if (c->moe_counts_host) cudaFreeHost(c->moe_counts_host);
    for (int l = 0; l < mxq_context::kMoeLanes; ++l) {
      if (c->moe_st[l]) cudaStreamSynchronize(c->moe_st[l]), cudaStreamDestroy(c->moe_st[l]);
      cudaFree(c->ml_op[l]);
      cudaFree(c->ml_f0[l]);
      cudaFree(c->ml_f1[l]);
    }
    for (auto& ev : c->moe_ev)
      if (ev) cudaEventDestroy(ev);
    delete c;
    return MXQ_OK;
  })
}

int mxq_set_stream(mxq_ctx c, void* s) {
  if (int rc = check_ctx(c)) return rc;
  c->stream = static_cast<cudaStream_t>(s);
  return MXQ_OK;
}

int mxq_set_path(mxq_ctx c, int path) {
  if (int rc = check_ctx(c)) return rc;
  if (path < MXQ_PATH_AUTO || path > MXQ_PATH_GEMM)
    return fail(c, MXQ_ERR_INVALID_ARGUMENT, "unknown path %d", path);
  c->path = path;
  return MXQ_OK;
}

int mxq_launch_count(mxq_ctx c, uint64_t* out) {
  if (int rc = check_ctx(c)) return rc;
  if (!out) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null output pointer");
  *out = c->launches;
  return MXQ_OK;
}

int mxq_reserve(mxq_ctx c, size_t max_batch, size_t max_k) {
  MXQ_TRY({
    if (int rc = check_ctx(c)) return rc;
    if (max_batch == 0 || max_k == 0 || max_k % kBlock)
      return fail(c, MXQ_ERR_INVALID_ARGUMENT, "reserve: batch and k must be > 0, k a multiple of 32");
    DeviceGuard g(c->device);
    const size_t kpad = (max_k + kTileK - 1) / kTileK * kTileK;
    const size_t bpad = (max_batch + 255) / 256 * 256;
    int rc;
    if ((rc = ensure(c, c->ws_q, c->ws_q_bytes, max_batch * max_k, "workspace q"))) return rc;
    if ((rc = ensure(c, c->ws_s, c->ws_s_bytes, max_batch * max_k / kBlock, "workspace s"))) return rc;
    if ((rc = ensure(c, c->ws_op, c->ws_op_bytes, bpad * kpad * 2, "workspace operand"))) return rc;
    if ((rc = ensure(c, c->ws_f0, c->ws_f0_bytes, max_batch * max_k * 4, "workspace f0"))) return rc;
    if ((rc = ensure(c, c->ws_f1, c->ws_f1_bytes, max_batch * max_k * 4, "workspace f1"))) return rc;
    if ((rc = ensure(c, c->ws_in, c->ws_in_bytes, max_batch * max_k * 4, "workspace in"))) return rc;
    if ((rc = ensure(c, c->ws_out, c->ws_out_bytes, max_batch * max_k * 4, "workspace out"))) return rc;
    return MXQ_OK;
  })
}

int mxq_synchronize(mxq_ctx c) {
  if (int rc = check_ctx(c)) return rc;
  DeviceGuard g(c->device);
  // one round trip: the status word rides the stream into pinned memory
  cudaError_t e = cudaMemcpyAsync(c->status_host, c->status, sizeof(uint32_t),
                                  cudaMemcpyDeviceToHost, c->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  if (e != cudaSuccess) return cuda_fail(c, e, "synchronize");
  const uint32_t st = *c->status_host;
  if (st) {
    // the status word a timed-out kernel left set
    cudaMemset(c->status, 0, 4 * sizeof(uint32_t));
    return fail(c, MXQ_ERR_TIMEOUT, "a device-side bounded wait gave up (status 0x%x)", st);
  }
  return MXQ_OK;
}

int mxq_weight_create(mxq_ctx c, int fmt, size_t n, size_t k, const void* data,
                      const uint8_t* scales, int on_device, mxq_weight* out) {
  MXQ_TRY({
    if (int rc = check_ctx(c)) return rc;
    if (!out || !data || !scales) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null pointer");
    *out = nullptr;
    if (fmt != MXQ_FMT_INT4 && fmt != MXQ_FMT_INT8)
      return fail(c, MXQ_ERR_INVALID_ARGUMENT, "unknown weight format %d", fmt);
    if (n == 0 || k == 0 || k % kBlock)
      return fail(c, MXQ_ERR_INVALID_ARGUMENT, "weight shape %zux%zu: K must be a positive multiple of 32", n, k);
    if (n > (1u << 24) || k > (1u << 24))
      return fail(c, MXQ_ERR_INVALID_ARGUMENT, "weight shape %zux%zu too large", n, k);
    DeviceGuard g(c->device);
    const int N = (int)n, K = (int)k;
    const int Npad = (N + 255) / 256 * 256;
    const int Kpad = (K + kTileK - 1) / kTileK * kTileK;
    const size_t src_bytes = fmt == 4 ? n * k / 2 : n * k;
    const size_t sc_bytes = n * k / kBlock;
    const size_t dst_bytes = (size_t)Npad * Kpad / (fmt == 4 ? 2 : 1);
    const size_t dsc_bytes = (size_t)Npad * Kpad / kBlock;
    auto* w = new mxq_weight_s();
    w->ctx = c;
    w->serial = next_weight_serial();
    cudaError_t e = cudaMalloc(&w->data, dst_bytes);
    if (e == cudaSuccess) e = cudaMalloc(&w->scales, dsc_bytes);
    const uint8_t* src_d = static_cast<const uint8_t*>(data);
    const uint8_t* src_s = scales;
    uint8_t* tmp = nullptr;
    if (e == cudaSuccess && !on_device) {
      e = cudaMalloc(&tmp, src_bytes + sc_bytes);
      if (e == cudaSuccess) e = cudaMemcpy(tmp, data, src_bytes, cudaMemcpyHostToDevice);
      if (e == cudaSuccess) e = cudaMemcpy(tmp + src_bytes, scales, sc_bytes, cudaMemcpyHostToDevice);
      src_d = tmp;
      src_s = tmp + src_bytes;
    }
    if (e == cudaSuccess) e = launch_repack(src_d, src_s, fmt, N, K, Npad, Kpad, w->data, w->scales, c->stream);
    uint32_t range[3] = {255, 0, 0};
    uint32_t* drange = nullptr;
    if (e == cudaSuccess) e = cudaMalloc(&drange, sizeof(range));
    if (e == cudaSuccess) e = cudaMemcpyAsync(drange, range, sizeof(range), cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = launch_scale_range(src_s, sc_bytes, drange, c->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(range, drange, sizeof(range), cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (drange) cudaFree(drange);
    if (tmp) cudaFree(tmp);
    if (e != cudaSuccess) {
      cudaFree(w->data);
      cudaFree(w->scales);
      delete w;
      return cuda_fail(c, e, "weight upload");
    }
    w->v.fmt = fmt;
    w->v.N = N;
    w->v.K = K;
    w->v.Npad = Npad;
    w->v.Kpad = Kpad;
    w->v.data = w->data;
    w->v.scales = w->scales;
    w->v.scale_lo = (int)range[0];
    w->v.scale_hi = (int)range[1];
    {
      // bf16 holds |q| * 2^n up to n = 120 (int8) / 124 (int4)
      const int emax = (int)range[2] - 127, lim = fmt == 8 ? 120 : 124;
      w->v.gemm_shift = emax > lim ? emax - lim : 0;
      w->v.gemm_fused = (int)range[2] - w->v.gemm_shift <= (fmt == 8 ? 231 : 246);
    }
    *out = w;
    return MXQ_OK;
  })
}

int mxq_weight_create_bsr(mxq_ctx c, int fmt, size_t n, size_t k, const void* data,
                          const uint8_t* scales, const uint8_t* block_mask, int on_device,
                          mxq_weight* out) {
  MXQ_TRY({
    if (int rc = check_ctx(c)) return rc;
    if (!out || !data || !scales || !block_mask) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null pointer");
    *out = nullptr;
    if (fmt != MXQ_FMT_INT4 && fmt != MXQ_FMT_INT8)
      return fail(c, MXQ_ERR_INVALID_ARGUMENT, "unknown weight format %d", fmt);
    if (n == 0 || k == 0 || k % kTileK)
      return fail(c, MXQ_ERR_INVALID_ARGUMENT, "block-sparse weight %zux%zu: K must be a positive multiple of 64", n, k);
    if (n > (1u << 24) || k > (1u << 24))
      return fail(c, MXQ_ERR_INVALID_ARGUMENT, "weight shape %zux%zu too large", n, k);
    DeviceGuard g(c->device);
    const int N = (int)n, K = (int)k;
    const int Npad = (N + 255) / 256 * 256, Kpad = K;
    const int T = Npad / 128, KB = K / kTileK, NB = (N + 63) / 64;
    // host-side tile list: a 128x64 tile is stored when either 64-row half
    // has its block present
    std::vector<int32_t> ptr(T + 1, 0), rt_of, kt_of;
    for (int rt = 0; rt < T; ++rt) {
      for (int kt = 0; kt < KB; ++kt) {
        bool any = false;
        for (int h = 0; h < 2; ++h) {
          const int br = rt * 2 + h;
          if (br < NB && block_mask[(size_t)br * KB + kt]) any = true;
        }
        if (any) {
          rt_of.push_back(rt);
          kt_of.push_back(kt);
        }
      }
      ptr[rt + 1] = (int32_t)rt_of.size();
    }
    const long ntiles = (long)rt_of.size();
    const int TB = fmt == 4 ? 32 : 64;
    const size_t src_bytes = fmt == 4 ? n * k / 2 : n * k;
    const size_t sc_bytes = n * k / kBlock;
    const size_t mask_bytes = (size_t)NB * KB;
    auto* w = new mxq_weight_s();
    w->ctx = c;
    w->serial = next_weight_serial();
    const size_t nt_alloc = ntiles > 0 ? (size_t)ntiles : 1;
    cudaError_t e = cudaMalloc(&w->data, nt_alloc * 128 * TB);
    if (e == cudaSuccess) e = cudaMalloc(&w->scales, nt_alloc * 256);
    if (e == cudaSuccess) e = cudaMalloc(&w->tiles, (T + 1 + nt_alloc) * sizeof(int32_t));
    uint8_t* tmp = nullptr;
    int32_t* dlist = nullptr;
    const size_t tmp_bytes = (on_device ? 0 : src_bytes + sc_bytes) + mask_bytes;
    if (e == cudaSuccess) e = cudaMalloc(&tmp, tmp_bytes);
    if (e == cudaSuccess) e = cudaMalloc(&dlist, 2 * nt_alloc * sizeof(int32_t));
    const uint8_t* src_d = static_cast<const uint8_t*>(data);
    const uint8_t* src_s = scales;
    uint8_t* dmask = tmp + (on_device ? 0 : src_bytes + sc_bytes);
    if (e == cudaSuccess && !on_device) {
      e = cudaMemcpy(tmp, data, src_bytes, cudaMemcpyHostToDevice);
      if (e == cudaSuccess) e = cudaMemcpy(tmp + src_bytes, scales, sc_bytes, cudaMemcpyHostToDevice);
      src_d = tmp;
      src_s = tmp + src_bytes;
    }
    if (e == cudaSuccess) e = cudaMemcpy(dmask, block_mask, mask_bytes, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(w->tiles, ptr.data(), (T + 1) * sizeof(int32_t), cudaMemcpyHostToDevice);
    if (e == cudaSuccess && ntiles > 0) {
      e = cudaMemcpy(w->tiles + T + 1, kt_of.data(), ntiles * sizeof(int32_t), cudaMemcpyHostToDevice);
      if (e == cudaSuccess) e = cudaMemcpy(dlist, rt_of.data(), ntiles * sizeof(int32_t), cudaMemcpyHostToDevice);
      if (e == cudaSuccess)
        e = cudaMemcpy(dlist + ntiles, kt_of.data(), ntiles * sizeof(int32_t), cudaMemcpyHostToDevice);
      if (e == cudaSuccess) {
        long ctas = (ntiles * 128 + 255) / 256;
        if (ctas > 148L * 32) ctas = 148L * 32;
        repack_bsr_kernel<<<(unsigned)ctas, 256, 0, c->stream>>>(src_d, src_s, dmask, fmt, N, K, dlist,
                                                                 dlist + ntiles, ntiles, w->data, w->scales);
        e = cudaGetLastError();
      }
    }
    uint32_t range[3] = {255, 0, 0};
    uint32_t* drange = nullptr;
    if (e == cudaSuccess) e = cudaMalloc(&drange, sizeof(range));
    if (e == cudaSuccess) e = cudaMemcpyAsync(drange, range, sizeof(range), cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess && ntiles > 0) e = launch_scale_range(w->scales, (size_t)ntiles * 256, drange, c->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(range, drange, sizeof(range), cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (drange) cudaFree(drange);
    if (dlist) cudaFree(dlist);
    if (tmp) cudaFree(tmp);
    if (e != cudaSuccess) {
      cudaFree(w->data);
      cudaFree(w->scales);
      cudaFree(w->tiles);
      delete w;
      return cuda_fail(c, e, "block-sparse weight upload");
    }
    if (ntiles == 0) range[0] = range[1] = range[2] = 127;
    w->v.fmt = fmt;
    w->v.N = N;
    w->v.K = K;
    w->v.Npad = Npad;
    w->v.Kpad = Kpad;
    w->v.data = w->data;
    w->v.scales = w->scales;
    w->v.scale_lo = (int)range[0];
    w->v.scale_hi = (int)range[1];
    {
      const int emax = (int)range[2] - 127, lim = fmt == 8 ? 120 : 124;
      w->v.gemm_shift = emax > lim ? emax - lim : 0;
      w->v.gemm_fused = (int)range[2] - w->v.gemm_shift <= (fmt == 8 ? 231 : 246);
    }
    w->v.kt_ptr = w->tiles;
    w->v.kt_idx = w->tiles + T + 1;
    w->v.nnz_tiles = (int)ntiles;
    *out = w;
    return MXQ_OK;
  })
}

int mxq_weight_destroy(mxq_weight w) {
  if (!w) return fail(nullptr, MXQ_ERR_INVALID_ARGUMENT, "null weight handle");
  DeviceGuard g(w->ctx->device);
  cudaFree(w->data);
  cudaFree(w->scales);
  if (w->tiles) cudaFree(w->tiles);
  delete w;
  return MXQ_OK;
}

int mxq_weight_download(mxq_weight w, void* data_host, uint8_t* scales_host) {
  MXQ_TRY({
    if (!w || !data_host || !scales_host) return fail(nullptr, MXQ_ERR_INVALID_ARGUMENT, "null pointer");
    if (w->v.kt_ptr) return fail(w->ctx, MXQ_ERR_UNSUPPORTED, "weight_download: block-sparse weights are not supported");
    DeviceGuard g(w->ctx->device);
    const WeightView& v = w->v;
    const int TB = v.fmt == 4 ? 32 : 64, KT = v.Kpad / kTileK;
    const size_t tb = (size_t)v.Npad * v.Kpad / (v.fmt == 4 ? 2 : 1), sb = (size_t)v.Npad * v.Kpad / kBlock;
    std::vector<uint8_t> td(tb), ts(sb);
    cudaError_t e = cudaStreamSynchronize(w->ctx->stream);
    if (e == cudaSuccess) e = cudaMemcpy(td.data(), v.data, tb, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemcpy(ts.data(), v.scales, sb, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(w->ctx, e, "weight_download");
    const size_t row_bytes = v.fmt == 4 ? (size_t)v.K / 2 : (size_t)v.K, nb = (size_t)v.K / kBlock;
    uint8_t* dd = static_cast<uint8_t*>(data_host);
    for (int n = 0; n < v.N; ++n)
      for (int kt = 0; kt < KT; ++kt) {
        const size_t src = (((size_t)(n / 128) * KT + kt) * 128 + (n % 128));
        for (int j = 0; j < TB; ++j) {
          const size_t byte = (size_t)kt * TB + j;
          if (byte < row_bytes) dd[(size_t)n * row_bytes + byte] = td[src * TB + j];
        }
        for (int hh = 0; hh < 2; ++hh) {
          const size_t b = (size_t)kt * 2 + hh;
          if (b < nb) scales_host[(size_t)n * nb + b] = ts[src * 2 + hh];
        }
      }
    return MXQ_OK;
  })
}

namespace {
struct MxqwHeader {
  char magic[4];
  uint32_t version, fmt, flags;
  uint64_t n, k;
};
static_assert(sizeof(MxqwHeader) == 32, "MXQW header layout");
}  // namespace

int mxq_weight_save(mxq_weight w, const char* path) {
  MXQ_TRY({
    if (!w || !path) return fail(nullptr, MXQ_ERR_INVALID_ARGUMENT, "null pointer");
    if (w->v.kt_ptr) return fail(w->ctx, MXQ_ERR_UNSUPPORTED, "weight_save: block-sparse weights are not supported");
    const size_t n = (size_t)w->v.N, k = (size_t)w->v.K;
    const size_t db = w->v.fmt == 4 ? n * k / 2 : n * k, sb = n * k / kBlock;
    std::vector<uint8_t> data(db), scales(sb);
    if (int rc = mxq_weight_download(w, data.data(), scales.data())) return rc;
    MxqwHeader h{{'M', 'X', 'Q', 'W'}, 1u, (uint32_t)w->v.fmt, 0u, n, k};
    FILE* f = std::fopen(path, "wb");
    if (!f) return fail(w->ctx, MXQ_ERR_INVALID_ARGUMENT, "weight_save: cannot open %s", path);
    const bool ok = std::fwrite(&h, sizeof(h), 1, f) == 1 && std::fwrite(data.data(), 1, db, f) == db &&
                    std::fwrite(scales.data(), 1, sb, f) == sb;
    const bool closed = std::fclose(f) == 0;
    if (!ok || !closed) return fail(w->ctx, MXQ_ERR_CUDA, "weight_save: write to %s failed", path);
    return MXQ_OK;
  })
}

int mxq_weight_load(mxq_ctx c, const char* path, mxq_weight* out) {
  MXQ_TRY({
    if (int rc = check_ctx(c)) return rc;
    if (!path || !out) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null pointer");
    *out = nullptr;
    FILE* f = std::fopen(path, "rb");
    if (!f) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "weight_load: cannot open %s", path);
    MxqwHeader h{};
    bool ok = std::fread(&h, sizeof(h), 1, f) == 1 && std::memcmp(h.magic, "MXQW", 4) == 0 && h.version == 1 &&
              (h.fmt == 4 || h.fmt == 8) && h.n > 0 && h.k > 0 && h.k % kBlock == 0 && h.n <= (1u << 24) &&
              h.k <= (1u << 24) && h.flags == 0;
    if (!ok) {
      std::fclose(f);
      return fail(c, MXQ_ERR_INVALID_ARGUMENT, "weight_load: %s is not an MXQW v1 dense weight", path);
    }
    const size_t db = h.fmt == 4 ? h.n * h.k / 2 : h.n * h.k, sb = h.n * h.k / kBlock;
    std::vector<uint8_t> data(db), scales(sb);
    ok = std::fread(data.data(), 1, db, f) == db && std::fread(scales.data(), 1, sb, f) == sb;
    std::fclose(f);
    if (!ok) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "weight_load: %s is truncated", path);
    return mxq_weight_create(c, (int)h.fmt, (size_t)h.n, (size_t)h.k, data.data(), scales.data(), 0, out);
  })
}

int mxq_weight_shape(mxq_weight w, int* fmt, size_t* n, size_t* k) {
  if (!w) return fail(nullptr, MXQ_ERR_INVALID_ARGUMENT, "null weight handle");
  if (fmt) *fmt = w->v.fmt;
  if (n) *n = (size_t)w->v.N;
  if (k) *k = (size_t)w->v.K;
  return MXQ_OK;
}

int mxq_quantize_x(mxq_ctx c, const float* x, size_t b, size_t k, int act,
                   uint8_t* q, uint8_t* s) {
  if (int rc = check_ctx(c)) return rc;
  if (!x || !q || !s) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null pointer");
  if (!aligned16(x)) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "fp32 input must be 16-byte aligned (it is read in 16-byte vectors)");
  if (b == 0 || k == 0 || k % kBlock)
    return fail(c, MXQ_ERR_INVALID_ARGUMENT, "quantize: K must be a positive multiple of 32");
  if (act != MXQ_ACT_NONE && act != MXQ_ACT_SILU)
    return fail(c, MXQ_ERR_INVALID_ARGUMENT, "unknown activation %d", act);
  DeviceGuard g(c->device);
  QuantArgs qa{};
  qa.x = x;
  qa.B = (int)b;
  qa.K = (int)k;
  qa.out_q = q;
  qa.out_s = s;
  return after_launch(c, launch_quantize(qa, act, c->stream, false), "quantize");
}

int mxq_swiglu_quantize(mxq_ctx c, const float* gate, const float* up, size_t b,
                        size_t k, uint8_t* q, uint8_t* s) {
  if (int rc = check_ctx(c)) return rc;
  if (!gate || !up || !q || !s) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null pointer");
  if (!aligned16(gate) || !aligned16(up)) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "fp32 input must be 16-byte aligned (it is read in 16-byte vectors)");
  if (b == 0 || k == 0 || k % kBlock)
    return fail(c, MXQ_ERR_INVALID_ARGUMENT, "quantize: K must be a positive multiple of 32");
  DeviceGuard g(c->device);
  QuantArgs qa{};
  qa.x = gate;
  qa.up = up;
  qa.B = (int)b;
  qa.K = (int)k;
  qa.out_q = q;
  qa.out_s = s;
  return after_launch(c, launch_quantize(qa, 2, c->stream, false), "swiglu quantize");
}

int mxq_gemv(mxq_ctx c, mxq_weight w, const uint8_t* xq, const uint8_t* xs,
             size_t b, float* y) {
  MXQ_TRY({
    if (int rc = check_ctx(c)) return rc;
    if (int rc = check_weight(c, w)) return rc;
    if (!xq || !xs || !y || b == 0) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null pointer or empty batch");
    if (!aligned16(xq)) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "activation must be 16-byte aligned");
    DeviceGuard g(c->device);
    return gemv_dev(c, w, xq, xs, b, y);
  })
}

static int reject_sparse(mxq_context* c, mxq_weight w, const char* what) {
  return w->v.kt_ptr ? fail(c, MXQ_ERR_UNSUPPORTED, "%s: not available for block-sparse weights", what) : MXQ_OK;
}

int mxq_gather_dot(mxq_ctx c, mxq_weight w, const uint8_t* xq, const uint8_t* xs,
                   size_t b, const int32_t* rows, size_t nrows, float* y) {
  if (int rc = check_ctx(c)) return rc;
  if (int rc = check_weight(c, w)) return rc;
  if (!xq || !xs || !rows || !y || b == 0 || nrows == 0)
    return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null pointer or empty input");
  if (int rc = reject_sparse(c, w, "gather_dot")) return rc;
  if (b > (size_t)gemv_max_batch())
    return fail(c, MXQ_ERR_INVALID_ARGUMENT, "gather_dot supports batch <= %d", gemv_max_batch());
  if (!aligned16(xq)) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "activation must be 16-byte aligned");
  DeviceGuard g(c->device);
  GemvArgs ga{};
  ga.w = w->v;
  ga.xq = xq;
  ga.xs = xs;
  ga.y = y;
  ga.B = (int)b;
  ga.rows = rows;
  ga.nrows = (int)nrows;
  return after_launch(c, launch_gemv(ga, c->stream, false), "gather_dot");
}

int mxq_block_dots(mxq_ctx c, mxq_weight w, const uint8_t* xq, size_t b, int32_t* dots) {
  if (int rc = check_ctx(c)) return rc;
  if (int rc = check_weight(c, w)) return rc;
  if (!xq || !dots || b == 0) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null pointer or empty batch");
  if (int rc = reject_sparse(c, w, "block_dots")) return rc;
  if (!aligned16(xq)) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "activation must be 16-byte aligned");
  DeviceGuard g(c->device);
  GemvArgs ga{};
  ga.w = w->v;
  ga.xq = xq;
  ga.B = (int)b;
  ga.block_dots = dots;
  return after_launch(c, launch_gemv(ga, c->stream, false), "block_dots");
}

int mxq_linear(mxq_ctx c, mxq_weight w, const float* x, size_t b, float* y) {
  MXQ_TRY({
    if (int rc = check_ctx(c)) return rc;
    if (int rc = check_weight(c, w)) return rc;
    if (!x || !y || b == 0) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null pointer or empty batch");
    if (!aligned16(x)) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "fp32 input must be 16-byte aligned (it is read in 16-byte vectors)");
    DeviceGuard g(c->device);
    return linear_dev(c, w, x, b, y, MXQ_ACT_NONE);
  })
}

int mxq_linear_pair(mxq_ctx c, mxq_weight w1, mxq_weight w2, const float* x,
                    size_t b, float* y) {
  MXQ_TRY({
    if (int rc = check_ctx(c)) return rc;
    if (int rc = check_weight(c, w1)) return rc;
    if (int rc = check_weight(c, w2)) return rc;
    if (!x || !y || b == 0) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null pointer or empty batch");
    if (!aligned16(x)) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "fp32 input must be 16-byte aligned (it is read in 16-byte vectors)");
    if (w2->v.K != w1->v.N)
      return fail(c, MXQ_ERR_INVALID_ARGUMENT, "pair shape mismatch: w1 N=%d, w2 K=%d", w1->v.N, w2->v.K);
    DeviceGuard g(c->device);
    int rc;
    if ((rc = ensure(c, c->ws_f0, c->ws_f0_bytes, b * w1->v.N * 4, "workspace mid"))) return rc;
    if (use_gemv(c, b, w1) && use_gemv(c, b, w2)) {
      if (b == 1 && gemv1_ok(w1, true, true) && gemv1_ok(w2, false, false)) {
        // batch 1, two co-resident GEMVs: the first also writes its output as
        // MX bytes, which the second reads (its weights stream meanwhile)
        const size_t m = (size_t)w1->v.N;
        if ((rc = ensure(c, c->ws_q, c->ws_q_bytes, m, "workspace q"))) return rc;
        if ((rc = ensure(c, c->ws_s, c->ws_s_bytes, m / kBlock, "workspace s"))) return rc;
        if ((rc = ensure_zeroed(c, c->ws_cnt, c->ws_cnt_bytes, m / kBlock * 4, "workspace counters"))) return rc;
        GemvArgs up{};
        up.w = w1->v;
        up.xf = x;
        up.y = c->ws_f0;
        up.B = 1;
        up.yq = c->ws_q;
        up.ys = c->ws_s;
        up.ycnt = c->ws_cnt;
        if ((rc = after_launch(c, launch_rgemv(up, c->stream, true), "gemv"))) return rc;
        GemvArgs dn{};
        dn.w = w2->v;
        dn.xq = c->ws_q;
        dn.xs = c->ws_s;
        dn.y = y;
        dn.B = 1;
        return after_launch(c, launch_rgemv(dn, c->stream, true), "gemv");
      }
      // decode: two launches; each GEMV quantises its fp32 input itself and
      // the first warms L2 with the second's weights while it streams
      if ((rc = gemv_f32(c, w1, x, b, c->ws_f0, w2))) return rc;
      return gemv_f32(c, w2, c->ws_f0, b, y, nullptr);
    }
    if ((rc = linear_dev(c, w1, x, b, c->ws_f0, MXQ_ACT_NONE))) return rc;
    return linear_dev(c, w2, c->ws_f0, b, y, MXQ_ACT_NONE);
  })
}

// Host-buffer calls: x_host -> pinned staging -> device, fn, device ->
// pinned staging -> y_host.  The first call of a (kind, weights, batch) runs
// as plain launches (sizing every workspace); the next one records the
// copies and launches into a CUDA graph, which later calls replay with one
// launch.  Any workspace move (ws_gen) or stream change retires the graph.
// The calls are synchronous, so they run on the context's private stream
// (capturable even when the caller's stream is the legacy default stream),
// after whatever the caller had queued on its own stream.
struct StreamSwap {
  mxq_context* c;
  cudaStream_t user;
  StreamSwap(mxq_context* cc, cudaStream_t s) : c(cc), user(cc->stream) { c->stream = s; }
  ~StreamSwap() { c->stream = user; }
};

static int host_call(mxq_context* c, int kind, uint64_t w1, uint64_t w2, size_t b, size_t in_elems,
                     size_t out_elems, const float* x_host, float* y_host,
                     int (*fn)(mxq_context*, void*, const float*, float*), void* arg) {
  if (!c->hstream) {
    cudaError_t e = cudaStreamCreateWithFlags(&c->hstream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->hevent, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaMalloc(&c->seq_dev, sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMemset(c->seq_dev, 0, sizeof(uint32_t));
    if (e != cudaSuccess) return cuda_fail(c, e, "host-call stream");
    c->host_seq = 0;
  }
  // order after the caller's queued work (nothing to order after when idle)
  cudaError_t ev = cudaStreamQuery(c->stream);
  if (ev == cudaErrorNotReady) {
    ev = cudaEventRecord(c->hevent, c->stream);
    if (ev == cudaSuccess) ev = cudaStreamWaitEvent(c->hstream, c->hevent, 0);
  }
  if (ev != cudaSuccess) return cuda_fail(c, ev, "host-call ordering");
  StreamSwap swap(c, c->hstream);
  int rc;
  const size_t in_bytes = in_elems * 4, out_bytes = out_elems * 4;
  const size_t out_pad = (out_bytes + 15) / 16 * 16;
  if ((rc = ensure(c, c->ws_in, c->ws_in_bytes, in_bytes, "workspace in"))) return rc;
  if ((rc = ensure(c, c->ws_out, c->ws_out_bytes, out_bytes, "workspace out"))) return rc;
  if ((rc = ensure_pinned(c, c->pin_in, c->pin_in_bytes, in_bytes, "pinned in"))) return rc;
  if ((rc = ensure_pinned(c, c->pin_out, c->pin_out_bytes, out_pad + 16, "pinned out"))) return rc;
  // pin_out: [y][status word][sequence flag]
  uint32_t* st_host = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(c->pin_out) + out_pad);
  uint32_t* flag_host = st_host + 1;
  const bool small = in_bytes + out_bytes <= ((size_t)1 << 20);
  mxq_context::HostGraph* hg = nullptr;
  for (auto& g : c->graphs)
    if (g.kind == kind && g.w1 == w1 && g.w2 == w2 && g.b == b) hg = &g;
  if (hg) hg->used = ++c->graph_clock;
  if (hg && (hg->gen != c->ws_gen || hg->stream != c->stream)) {
    if (hg->exec) cudaGraphExecDestroy(hg->exec);
    *hg = mxq_context::HostGraph{kind, w1, w2, b, 0, nullptr, nullptr, false, 0};
  }
  std::memcpy(c->pin_in, x_host, in_bytes);
  if (hg && hg->gen == c->ws_gen && hg->exec) {
    cudaError_t e = cudaSuccess;
    if (hg->mapped) {
      // one launch; completion seen through the mapped sequence flag
      const uint32_t expect = c->host_seq + 1;
      e = cudaGraphLaunch(hg->exec, c->stream);
      if (e != cudaSuccess) return cuda_fail(c, e, "graph launch");
      const auto t0 = std::chrono::steady_clock::now();
      for (uint32_t it = 0;; ++it) {
        if (__atomic_load_n(flag_host, __ATOMIC_ACQUIRE) == expect) break;
        if ((it & 1023u) == 1023u &&
            std::chrono::steady_clock::now() - t0 > std::chrono::seconds(2)) {
          e = cudaStreamSynchronize(c->stream);           // bounded: fall back to the stream
          c->host_seq = __atomic_load_n(flag_host, __ATOMIC_ACQUIRE);
          if (e != cudaSuccess) return cuda_fail(c, e, "host call");
          if (c->host_seq != expect) return fail(c, MXQ_ERR_CUDA, "host call: completion flag not seen");
          break;
        }
      }
      c->host_seq = expect;
    } else {
      // the graph ends with the status word's copy: one synchronisation
      e = cudaGraphLaunch(hg->exec, c->stream);
      if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
      if (e != cudaSuccess) return cuda_fail(c, e, "graph launch");
    }
    c->launches += 2;
    const uint32_t st = hg->mapped ? *st_host : *c->status_host;
    if (st) {
      cudaMemset(c->status, 0, 4 * sizeof(uint32_t));
      return fail(c, MXQ_ERR_TIMEOUT, "a device-side bounded wait gave up (status 0x%x)", st);
    }
    std::memcpy(y_host, c->pin_out, out_bytes);
    return MXQ_OK;
  }
  // plain launches (the first call of a key sizes every buffer it touches)
  const uint64_t gen0 = c->ws_gen;
  cudaError_t e = cudaMemcpyAsync(c->ws_in, c->pin_in, in_bytes, cudaMemcpyHostToDevice, c->stream);
  if (e != cudaSuccess) return cuda_fail(c, e, "copy in");
  if ((rc = fn(c, arg, c->ws_in, c->ws_out))) return rc;
  e = cudaMemcpyAsync(c->pin_out, c->ws_out, out_bytes, cudaMemcpyDeviceToHost, c->stream);
  if (e != cudaSuccess) return cuda_fail(c, e, "copy out");
  if ((rc = mxq_synchronize(c))) return rc;
  std::memcpy(y_host, c->pin_out, out_bytes);
  if (!hg) {
    if (c->graphs.size() >= mxq_context::kMaxHostGraphs) {
      auto lru = c->graphs.begin();
      for (auto it = c->graphs.begin(); it != c->graphs.end(); ++it)
        if (it->used < lru->used) lru = it;
      if (lru->exec) cudaGraphExecDestroy(lru->exec);
      c->graphs.erase(lru);
    }
    c->graphs.push_back(mxq_context::HostGraph{kind, w1, w2, b, 0, c->stream, nullptr, false, 0});
    hg = &c->graphs.back();
  }
  if (c->ws_gen == gen0 && hg->gen == 0) {
    // record the call for the next time
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    float* din = nullptr;
    float* dout = nullptr;
    uint32_t* dst_ = nullptr;
    bool good = !small || (cudaHostGetDevicePointer(reinterpret_cast<void**>(&din), c->pin_in, 0) == cudaSuccess &&
                           cudaHostGetDevicePointer(reinterpret_cast<void**>(&dout), c->pin_out, 0) == cudaSuccess);
    if (good && small) dst_ = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(dout) + out_pad);
    good = good && cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal) == cudaSuccess;
    if (good) {
      const uint64_t launches = c->launches;
      bool inner;
      if (small) {
        host_in_kernel<<<1, 1024, 0, c->stream>>>(c->ws_in, din, in_elems);
        inner = cudaGetLastError() == cudaSuccess;
        inner = inner && fn(c, arg, c->ws_in, c->ws_out) == MXQ_OK;
        host_out_kernel<<<1, 1024, 0, c->stream>>>(c->ws_out, dout, out_elems, c->status, dst_, c->seq_dev,
                                                   dst_ + 1);
        inner = inner && cudaGetLastError() == cudaSuccess;
      } else {
        inner = cudaMemcpyAsync(c->ws_in, c->pin_in, in_bytes, cudaMemcpyHostToDevice, c->stream) == cudaSuccess;
        inner = inner && fn(c, arg, c->ws_in, c->ws_out) == MXQ_OK;
        inner = inner && cudaMemcpyAsync(c->pin_out, c->ws_out, out_bytes, cudaMemcpyDeviceToHost,
                                         c->stream) == cudaSuccess;
        inner = inner && cudaMemcpyAsync(c->status_host, c->status, sizeof(uint32_t), cudaMemcpyDeviceToHost,
                                         c->stream) == cudaSuccess;
      }
      c->launches = launches;
      good = cudaStreamEndCapture(c->stream, &graph) == cudaSuccess && inner && graph && c->ws_gen == gen0;
    }
    if (good) good = cudaGraphInstantiate(&exec, graph, 0) == cudaSuccess;
    if (graph) cudaGraphDestroy(graph);
    (void)cudaGetLastError();
    hg->gen = c->ws_gen;
    hg->stream = c->stream;
    hg->exec = good ? exec : nullptr;
    hg->mapped = small;
    if (!good && exec) cudaGraphExecDestroy(exec);
  }
  return MXQ_OK;
}

struct LinArg { mxq_weight w; size_t b; };
struct PairArg { mxq_weight w1, w2; size_t b; };

int mxq_linear_host(mxq_ctx c, mxq_weight w, const float* x_host, size_t b, float* y_host) {
  MXQ_TRY({
    if (int rc = check_ctx(c)) return rc;
    if (int rc = check_weight(c, w)) return rc;
    if (!x_host || !y_host || b == 0) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null pointer or empty batch");
    DeviceGuard g(c->device);
    LinArg la{w, b};
    return host_call(c, 1, w->serial, 0, b, b * w->v.K, b * w->v.N, x_host, y_host,
                     [](mxq_context* cc, void* p, const float* xi, float* yo) {
                       auto* a = static_cast<LinArg*>(p);
                       return linear_dev(cc, a->w, xi, a->b, yo, MXQ_ACT_NONE);
                     }, &la);
  })
}

// ---------------------------------------------- column-sharded pair ---
// One rank's side of a batch-1 pair column-sharded over `world` GPUs.  The
// mailbox (device memory exported over CUDA IPC, opened by every other
// rank) holds, twice over (the device epoch's parity picks the half):
//   flags  [2 kinds][kMaxPeers] u32 at 0 (kind 0: first linear's rows
//          landed, kind 1: second's), written by the ranks over NVLink;
//   q      [2][n1] MX bytes of the intermediate, s [2][n1/32] its scales;
//   f      [2][n2] fp32 output rows.
// Local words (not exported): epoch, and one finished-CTA counter per role.
struct mxq_peers_s {
  mxq_context* ctx = nullptr;
  int rank = 0, world = 1;
  size_t n1 = 0, n2 = 0;
  uint8_t* mbox = nullptr;
  size_t off_q = 0, off_s = 0, off_f = 0, bytes = 0;
  uint8_t* base[kMaxPeers] = {};   // every rank's mailbox as mapped here
  bool opened[kMaxPeers] = {};
  uint32_t* local = nullptr;       // [0] epoch, [1] role-1 counter, [2] role-2 counter
  uint64_t wait_ns = kWaitLimitNs;
};

int mxq_peers_create(mxq_ctx c, int rank, int world, size_t n1, size_t n2, mxq_peers* out, void* handle_out) {
  MXQ_TRY({
    if (int rc = check_ctx(c)) return rc;
    if (!out || !handle_out) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null pointer");
    *out = nullptr;
    if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world)
      return fail(c, MXQ_ERR_INVALID_ARGUMENT, "peer group: rank %d of world %d (1..%d ranks)", rank, world, kMaxPeers);
    if (n1 == 0 || n2 == 0 || n1 % ((size_t)world * kBlock) || n2 % (size_t)world)
      return fail(c, MXQ_ERR_INVALID_ARGUMENT,
                  "peer group: n1=%zu must split into whole 32-row blocks per rank and n2=%zu into equal shards", n1, n2);
    DeviceGuard g(c->device);
    auto* P = new mxq_peers_s();
    P->ctx = c;
    P->rank = rank;
    P->world = world;
    P->n1 = n1;
    P->n2 = n2;
    P->off_q = 256;
    P->off_s = P->off_q + 2 * n1;
    P->off_f = (P->off_s + 2 * (n1 / kBlock) + 15) / 16 * 16;
    P->bytes = P->off_f + 2 * n2 * sizeof(float);
    cudaError_t e = cudaMalloc(&P->mbox, P->bytes);
    if (e == cudaSuccess) e = cudaMemset(P->mbox, 0, P->bytes);
    if (e == cudaSuccess) e = cudaMalloc(&P->local, 4 * sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMemset(P->local, 0, 4 * sizeof(uint32_t));
    cudaIpcMemHandle_t h{};
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, P->mbox);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
      cudaFree(P->mbox);
      cudaFree(P->local);
      delete P;
      return cuda_fail(c, e, "peer mailbox");
    }
    static_assert(sizeof(cudaIpcMemHandle_t) == MXQ_PEER_HANDLE_BYTES, "IPC handle size");
    std::memcpy(handle_out, &h, sizeof(h));
    P->base[rank] = P->mbox;
    *out = P;
    return MXQ_OK;
  })
}

int mxq_peers_connect(mxq_peers P, const void* handles) {
  MXQ_TRY({
    if (!P || !handles) return fail(nullptr, MXQ_ERR_INVALID_ARGUMENT, "null pointer");
    mxq_context* c = P->ctx;
    DeviceGuard g(c->device);
    for (int r = 0; r < P->world; ++r) {
      if (r == P->rank || P->base[r]) continue;
      cudaIpcMemHandle_t h;
      std::memcpy(&h, static_cast<const uint8_t*>(handles) + (size_t)r * sizeof(h), sizeof(h));
      void* p = nullptr;
      const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
      if (e != cudaSuccess) return cuda_fail(c, e, "open a peer's mailbox");
      P->base[r] = static_cast<uint8_t*>(p);
      P->opened[r] = true;
    }
    return MXQ_OK;
  })
}

int mxq_peers_set_wait_limit(mxq_peers P, uint32_t wait_us) {
  if (!P) return fail(nullptr, MXQ_ERR_INVALID_ARGUMENT, "null peer group");
  if (wait_us == 0 || wait_us > 10000000u)
    return fail(P->ctx, MXQ_ERR_INVALID_ARGUMENT, "peer wait limit must be in [1, 1e7] microseconds");
  P->wait_ns = (uint64_t)wait_us * 1000ull;
  return MXQ_OK;
}

int mxq_peers_destroy(mxq_peers P) {
  if (!P) return fail(nullptr, MXQ_ERR_INVALID_ARGUMENT, "null peer group");
  DeviceGuard g(P->ctx->device);
  cudaDeviceSynchronize();
  for (int r = 0; r < P->world; ++r)
    if (P->opened[r]) cudaIpcCloseMemHandle(P->base[r]);
  cudaFree(P->mbox);
  cudaFree(P->local);
  delete P;
  return MXQ_OK;
}

int mxq_linear_pair_sharded(mxq_ctx c, mxq_peers P, mxq_weight w1, mxq_weight w2, const float* x, float* y) {
  MXQ_TRY({
    if (int rc = check_ctx(c)) return rc;
    if (int rc = check_weight(c, w1)) return rc;
    if (int rc = check_weight(c, w2)) return rc;
    if (!P || !x || !y) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null pointer");
    if (P->ctx != c) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "peer group belongs to another context");
    for (int r = 0; r < P->world; ++r)
      if (!P->base[r]) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "peer group not connected (mxq_peers_connect)");
    if (!aligned16(x)) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "fp32 input must be 16-byte aligned (it is read in 16-byte vectors)");
    const size_t n1s = P->n1 / P->world, n2s = P->n2 / P->world;
    if ((size_t)w1->v.N != n1s || (size_t)w2->v.N != n2s || (size_t)w2->v.K != P->n1)
      return fail(c, MXQ_ERR_INVALID_ARGUMENT,
                  "sharded pair: shards must be %zu x K and %zu x %zu rows (got %d x %d, %d x %d)", n1s, n2s, P->n1,
                  w1->v.N, w1->v.K, w2->v.N, w2->v.K);
    if (!cogemv_supported(w1->v, 1, true, true) || !cogemv_supported(w2->v, 1, false, false))
      return fail(c, MXQ_ERR_UNSUPPORTED, "sharded pair: a shard does not fit the batch-1 co-resident GEMV");
    DeviceGuard g(c->device);
    int rc;
    if ((rc = ensure(c, c->ws_f0, c->ws_f0_bytes, n1s * 4, "workspace mid"))) return rc;
    if ((rc = ensure(c, c->ws_q, c->ws_q_bytes, n1s, "workspace q"))) return rc;
    if ((rc = ensure(c, c->ws_s, c->ws_s_bytes, n1s / kBlock, "workspace s"))) return rc;
    if ((rc = ensure_zeroed(c, c->ws_cnt, c->ws_cnt_bytes, n1s / kBlock * 4, "workspace counters"))) return rc;
    PeerArgs pa{};
    pa.world = P->world;
    pa.rank = P->rank;
    pa.epoch = P->local;
    pa.status = c->status;
    pa.wait_ns = P->wait_ns;
    auto flags = [&](int r, int kind) { return reinterpret_cast<uint32_t*>(P->base[r]) + kind * kMaxPeers; };
    // first linear: this rank's rows of the intermediate, as MX bytes, into every mailbox
    PeerArgs p1 = pa;
    p1.grid_cnt = P->local + 1;
    for (int r = 0; r < P->world; ++r) {
      p1.flag_out[r] = flags(r, 0) + P->rank;
      p1.q_out[r] = P->base[r] + P->off_q;
      p1.s_out[r] = P->base[r] + P->off_s;
    }
    p1.q_stride = P->n1;
    p1.s_stride = P->n1 / kBlock;
    p1.row_off = (int)(P->rank * n1s);
    GemvArgs up{};
    up.w = w1->v;
    up.xf = x;
    up.y = c->ws_f0;
    up.B = 1;
    up.yq = c->ws_q;
    up.ys = c->ws_s;
    up.ycnt = c->ws_cnt;
    if ((rc = after_launch(c, launch_cogemv_peer(up, p1, 1, c->stream, true), "sharded gemv 1"))) return rc;
    // second linear: waits for every rank's rows, reads the full MX
    // intermediate from the local mailbox, its fp32 rows into every mailbox
    PeerArgs p2 = pa;
    p2.grid_cnt = P->local + 2;
    p2.wait_flags = flags(P->rank, 0);
    p2.xq_base = P->mbox + P->off_q;
    p2.xs_base = P->mbox + P->off_s;
    p2.xq_stride = P->n1;
    p2.xs_stride = P->n1 / kBlock;
    for (int r = 0; r < P->world; ++r) {
      p2.flag_out[r] = flags(r, 1) + P->rank;
      p2.f_out[r] = reinterpret_cast<float*>(P->base[r] + P->off_f);
    }
    p2.f_stride = P->n2;
    p2.row_off = (int)(P->rank * n2s);
    // ... then its last CTA: every rank's output rows -> y, epoch advanced
    p2.done_flags = flags(P->rank, 1);
    p2.f_in = reinterpret_cast<const float*>(P->mbox + P->off_f);
    p2.f_in_stride = P->n2;
    p2.n_out = (int)P->n2;
    GemvArgs dn{};
    dn.w = w2->v;
    dn.B = 1;
    dn.y = y;
    return after_launch(c, launch_cogemv_peer(dn, p2, 2, c->stream, true), "sharded gemv 2");
  })
}

int mxq_debug_peer_stall(mxq_ctx c, mxq_peers P, mxq_weight w2, uint32_t wait_us) {
  MXQ_TRY({
    if (int rc = check_ctx(c)) return rc;
    if (int rc = check_weight(c, w2)) return rc;
    if (!P || P->ctx != c) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null or foreign peer group");
    if (P->world != 1) return fail(c, MXQ_ERR_UNSUPPORTED, "debug peer stall: one-rank groups only");
    if (wait_us == 0 || wait_us > 1000000u)
      return fail(c, MXQ_ERR_INVALID_ARGUMENT, "debug stall: wait limit must be in [1, 1e6] microseconds");
    if ((size_t)w2->v.N != P->n2 || (size_t)w2->v.K != P->n1 || !cogemv_supported(w2->v, 1, false, false))
      return fail(c, MXQ_ERR_INVALID_ARGUMENT, "debug peer stall: w2 must be n2 x n1");
    DeviceGuard g(c->device);
    // the second linear waiting on a flag word that nothing sets (local[3]);
    // its own flag goes to the same scratch word, its output to a scratch
    // buffer; a one-rank group needs no agreement with other ranks' epochs,
    // so it stays usable
    PeerArgs p2{};
    p2.world = 1;
    p2.rank = 0;
    p2.epoch = P->local;
    p2.grid_cnt = P->local + 2;
    p2.wait_flags = P->local + 3;
    p2.flag_out[0] = P->local + 3;
    p2.xq_base = P->mbox + P->off_q;
    p2.xs_base = P->mbox + P->off_s;
    p2.xq_stride = P->n1;
    p2.xs_stride = P->n1 / kBlock;
    p2.f_out[0] = reinterpret_cast<float*>(P->mbox + P->off_f);
    p2.f_stride = P->n2;
    p2.done_flags = P->local + 3;
    p2.f_in = reinterpret_cast<const float*>(P->mbox + P->off_f);
    p2.f_in_stride = P->n2;
    p2.n_out = (int)P->n2;
    p2.status = c->status;
    p2.wait_ns = (uint64_t)wait_us * 1000ull;
    float* scratch = nullptr;
    cudaError_t e = cudaMalloc(&scratch, P->n2 * sizeof(float));
    if (e != cudaSuccess) return cuda_fail(c, e, "debug peer stall");
    GemvArgs dn{};
    dn.w = w2->v;
    dn.B = 1;
    dn.y = scratch;
    int rc = after_launch(c, launch_cogemv_peer(dn, p2, 2, c->stream, false), "sharded gemv 2");
    const int st = rc ? rc : mxq_synchronize(c);
    cudaDeviceSynchronize();
    cudaFree(scratch);
    cudaMemset(P->local + 3, 0, sizeof(uint32_t));
    return st;
  })
}

int mxq_linear_pair_host(mxq_ctx c, mxq_weight w1, mxq_weight w2, const float* x_host,
                         size_t b, float* y_host) {
  MXQ_TRY({
    if (int rc = check_ctx(c)) return rc;
    if (int rc = check_weight(c, w1)) return rc;
    if (int rc = check_weight(c, w2)) return rc;
    if (!x_host || !y_host || b == 0) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null pointer or empty batch");
    if (w2->v.K != w1->v.N)
      return fail(c, MXQ_ERR_INVALID_ARGUMENT, "pair shape mismatch: w1 N=%d, w2 K=%d", w1->v.N, w2->v.K);
    DeviceGuard g(c->device);
    PairArg pa{w1, w2, b};
    return host_call(c, 2, w1->serial, w2->serial, b, b * w1->v.K, b * w2->v.N, x_host, y_host,
                     [](mxq_context* cc, void* p, const float* xi, float* yo) {
                       auto* a = static_cast<PairArg*>(p);
                       return mxq_linear_pair(cc, a->w1, a->w2, xi, a->b, yo);
                     }, &pa);
  })
}

int mxq_mlp_swiglu(mxq_ctx c, mxq_weight wg, mxq_weight wu, mxq_weight wd,
                   const float* x, size_t b, float* y) {
  MXQ_TRY({
    if (int rc = check_ctx(c)) return rc;
    if (int rc = check_weight(c, wg)) return rc;
    if (int rc = check_weight(c, wu)) return rc;
    if (int rc = check_weight(c, wd)) return rc;
    if (!x || !y || b == 0) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null pointer or empty batch");
    if (!aligned16(x)) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "fp32 input must be 16-byte aligned (it is read in 16-byte vectors)");
    if (wg->v.N != wu->v.N || wg->v.K != wu->v.K || wd->v.K != wg->v.N || wd->v.N != wg->v.K)
      return fail(c, MXQ_ERR_INVALID_ARGUMENT, "gated MLP shape mismatch");
    DeviceGuard g(c->device);
    const size_t F = wg->v.N;
    int rc;
    if ((rc = ensure(c, c->ws_f0, c->ws_f0_bytes, b * F * 4, "workspace gate"))) return rc;
    if ((rc = ensure(c, c->ws_f1, c->ws_f1_bytes, b * F * 4, "workspace up"))) return rc;
    if ((rc = linear_dev(c, wg, x, b, c->ws_f0, MXQ_ACT_NONE))) return rc;
    if ((rc = linear_dev(c, wu, x, b, c->ws_f1, MXQ_ACT_NONE))) return rc;
    // silu(gate) * up -> MX into ws_q (the gate/up GEMVs queued before have
    // consumed their quantised input; stream order makes the reuse safe)
    const size_t off_s = (b * F + 15) / 16 * 16;
    if ((rc = ensure(c, c->ws_q, c->ws_q_bytes, off_s + b * F / kBlock, "workspace mid"))) return rc;
    uint8_t* hq = c->ws_q;
    uint8_t* hs = c->ws_q + off_s;
    QuantArgs qa{};
    qa.x = c->ws_f0;
    qa.up = c->ws_f1;
    qa.B = (int)b;
    qa.K = (int)F;
    qa.out_q = hq;
    qa.out_s = hs;
    if ((rc = after_launch(c, launch_quantize(qa, 2, c->stream, true), "swiglu quantize"))) return rc;
    return gemv_dev(c, wd, hq, hs, b, y);
  })
}

int mxq_policy_head(mxq_ctx c, const float* logits, const float* actions, size_t rows,
                    size_t cols, float* log_probs, float* action_logp, float* entropy) {
  if (int rc = check_ctx(c)) return rc;
  if (!logits || !actions || !log_probs || !action_logp || !entropy)
    return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null pointer");
  if (cols == 0 || cols > (1u << 24) || rows > (1u << 28))
    return fail(c, MXQ_ERR_INVALID_ARGUMENT, "policy head: bad shape %zux%zu", rows, cols);
  if (rows == 0) return MXQ_OK;
  DeviceGuard g(c->device);
  const long threads = (long)rows * 32;
  policy_head_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, c->stream>>>(
      logits, actions, (int)rows, (int)cols, log_probs, action_logp, entropy);
  return after_launch(c, cudaGetLastError(), "policy_head");
}

// Expert layer operand: rows gathered from x (slot -> token row), quantised
// per 32-block into the tensor-core operand for weight w.
static int moe_operand(mxq_context* c, mxq_weight w, const float* x, const int32_t* gather, int b, int K,
                       int BN, int Bpad) {
  QuantArgs qa{};
  qa.x = x;
  qa.gather = gather;
  qa.B = b;
  qa.K = K;
  qa.opnd = reinterpret_cast<__nv_bfloat16*>(c->ws_op);
  qa.Bpad = Bpad;
  qa.Kpad = w->v.Kpad;
  qa.BN = BN;
  qa.int4_order = w->v.fmt == 4;
  qa.shift = w->v.gemm_shift;
  return after_launch(c, launch_quantize(qa, 0, c->stream, true), "moe operand");
}

static int moe_gemm(mxq_context* c, mxq_weight w, int b, int BN, int Bpad, float* y) {
  GemmArgs ga{};
  ga.w = w->v;
  ga.opnd = reinterpret_cast<const __nv_bfloat16*>(c->ws_op);
  ga.y = y;
  ga.B = b;
  ga.Bpad = Bpad;
  ga.BN = BN;
  ga.status = c->status;
  return after_launch(c, launch_gemm(ga, c->stream, true), "moe gemm");
}

// Expert-parallel MoE group: this rank's mailbox (flags [8] u32, then two
// halves of expert-output rows [max_routes][D] fp32, alternating by call)
// and every rank's as mapped here.
struct mxq_moe_group_s {
  mxq_context* ctx = nullptr;
  int rank = 0, world = 1;
  size_t max_routes = 0, D = 0;
  uint8_t* mbox = nullptr;
  size_t off_yr = 256, half_bytes = 0, bytes = 0;
  uint8_t* base[kMaxPeers] = {};
  bool opened[kMaxPeers] = {};
  uint32_t* local = nullptr;       // [0] exchanges completed, [1] grid counter
  uint64_t calls = 0;              // host: calls made (selects the half)
  uint64_t wait_ns = kWaitLimitNs;
};

static int moe_layer(mxq_context* c, const mxq_weight* w_gate, const mxq_weight* w_up, const mxq_weight* w_down,
                     int E, int e_lo, int n_local, const float* x, const float* logits, int T, int K, int D, int F,
                     float* y, mxq_moe_group_s* G);

int mxq_moe_swiglu(mxq_ctx c, const mxq_weight* w_gate, const mxq_weight* w_up,
                   const mxq_weight* w_down, size_t n_experts, const float* x,
                   const float* logits, size_t t, size_t k, float* y) {
  MXQ_TRY({
    if (int rc = check_ctx(c)) return rc;
    if (!w_gate || !w_up || !w_down || !x || !logits || !y || n_experts == 0)
      return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null pointer or no experts");
    if (!aligned16(x)) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "fp32 input must be 16-byte aligned (it is read in 16-byte vectors)");
    if (k == 0 || k > n_experts)
      return fail(c, MXQ_ERR_INVALID_ARGUMENT, "top-k: k=%zu must be in [1, n_experts=%zu]", k, n_experts);
    if (k > 64 || n_experts > 4096) return fail(c, MXQ_ERR_UNSUPPORTED, "top-k: k <= 64 and n_experts <= 4096");
    const int E = (int)n_experts;
    for (int e = 0; e < E; ++e) {
      if (int rc = check_weight(c, w_gate[e])) return rc;
      if (int rc = check_weight(c, w_up[e])) return rc;
      if (int rc = check_weight(c, w_down[e])) return rc;
    }
    const int D = w_gate[0]->v.K, F = w_gate[0]->v.N;
    for (int e = 0; e < E; ++e) {
      const WeightView &g = w_gate[e]->v, &u = w_up[e]->v, &d = w_down[e]->v;
      if (g.K != D || g.N != F || u.K != D || u.N != F || d.K != F || d.N != D)
        return fail(c, MXQ_ERR_INVALID_ARGUMENT,
                    "expert %d shapes: gate/up must be [%d][%d] and down [%d][%d]", e, F, D, D, F);
    }
    if (t == 0) return MXQ_OK;
    if (t > (1u << 24) || t * k > (1u << 26)) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "too many tokens");
    DeviceGuard g(c->device);
    return moe_layer(c, w_gate, w_up, w_down, E, 0, E, x, logits, (int)t, (int)k, D, F, y, nullptr);
  })
}

// The MoE layer after validation: routes and slots over all E experts, the
// expert GEMMs of experts [e_lo, e_lo + n_local) (weights w_*[0 .. n_local)),
// the combine.  With a group G, the expert outputs land in this rank's
// mailbox and one exchange copies this rank's slot rows to every other
// rank's mailbox before the combine.
static int moe_layer(mxq_context* c, const mxq_weight* w_gate, const mxq_weight* w_up, const mxq_weight* w_down,
                     int E, int e_lo, int n_local, const float* x, const float* logits, int T, int K, int D, int F,
                     float* y, mxq_moe_group_s* G) {
  {
    const int R = T * K;
    int rc;
    // bookkeeping: idx[R] gate[R] counts[E] offsets[E+1] slot_token[R] route_pos[R]
    const size_t moe_ints = (size_t)4 * R + 2 * E + 1;
    if ((rc = ensure(c, c->ws_moe, c->ws_moe_bytes, moe_ints * 4, "workspace moe"))) return rc;
    int32_t* idx = c->ws_moe;
    float* gate = reinterpret_cast<float*>(idx + R);
    int32_t* counts = idx + 2 * R;
    int32_t* offsets = counts + E;
    int32_t* slot_token = offsets + E + 1;
    int32_t* route_pos = slot_token + R;
    route_topk_kernel<<<(unsigned)((T + 127) / 128), 128, 0, c->stream>>>(logits, T, E, K, idx, gate);
    if ((rc = after_launch(c, cudaGetLastError(), "moe route"))) return rc;
    if ((rc = after_launch(c, launch_moe_assign(idx, T, K, E, counts, offsets, slot_token, route_pos,
                                                c->stream), "moe assign")))
      return rc;
    // the per-expert launches are sized on the host: one small read-back
    if ((size_t)E > c->moe_counts_cap) {
      if (c->moe_counts_host) cudaFreeHost(c->moe_counts_host);
      c->moe_counts_host = nullptr;
      c->moe_counts_cap = 0;
      if (cudaError_t e = cudaHostAlloc(&c->moe_counts_host, (size_t)E * 4, cudaHostAllocDefault))
        return cuda_fail(c, e, "moe counts");
      c->moe_counts_cap = (size_t)E;
    }
    if (cudaError_t e = cudaMemcpyAsync(c->moe_counts_host, counts, (size_t)E * 4, cudaMemcpyDeviceToHost,
                                        c->stream))
      return cuda_fail(c, e, "moe counts");
    if (cudaError_t e = cudaStreamSynchronize(c->stream)) return cuda_fail(c, e, "moe counts");
    int nmax = 0, off_lo = 0, off_hi = 0;
    for (int e = 0; e < E; ++e) {
      const int ne = c->moe_counts_host[e];
      if (e < e_lo) off_lo += ne;
      if (e < e_lo + n_local) off_hi += ne;
      if (e >= e_lo && e < e_lo + n_local) nmax = ne > nmax ? ne : nmax;
    }
    if (nmax > 0) {
      const int BNm = gemm_pick_bn(nmax);
      const size_t Bpm = (size_t)(nmax + BNm - 1) / BNm * BNm;
      int kmax = 0;
      for (int e = 0; e < n_local; ++e) {
        kmax = w_gate[e]->v.Kpad > kmax ? w_gate[e]->v.Kpad : kmax;
        kmax = w_up[e]->v.Kpad > kmax ? w_up[e]->v.Kpad : kmax;
        kmax = w_down[e]->v.Kpad > kmax ? w_down[e]->v.Kpad : kmax;
      }
      for (int l = 0; l < mxq_context::kMoeLanes; ++l) {
        if ((rc = ensure(c, c->ml_op[l], c->ml_op_bytes[l], Bpm * kmax * 2, "workspace operand"))) return rc;
        if ((rc = ensure(c, c->ml_f0[l], c->ml_f0_bytes[l], (size_t)nmax * F * 4, "workspace gate"))) return rc;
        if ((rc = ensure(c, c->ml_f1[l], c->ml_f1_bytes[l], (size_t)nmax * F * 4, "workspace up"))) return rc;
      }
      for (int l = 0; l < mxq_context::kMoeLanes; ++l)
        if (!c->moe_st[l]) {
          cudaError_t e = cudaStreamCreateWithFlags(&c->moe_st[l], cudaStreamNonBlocking);
          if (e != cudaSuccess) return cuda_fail(c, e, "moe lane stream");
        }
      for (auto& ev : c->moe_ev)
        if (!ev) {
          cudaError_t e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
          if (e != cudaSuccess) return cuda_fail(c, e, "moe lane event");
        }
    }
    float* yr = nullptr;
    if (G) {
      yr = reinterpret_cast<float*>(G->mbox + G->off_yr + (size_t)(G->calls & 1u) * G->half_bytes);
    } else {
      if ((rc = ensure(c, c->ws_yr, c->ws_yr_bytes, (size_t)R * D * 4, "workspace expert outputs"))) return rc;
      yr = c->ws_yr;
    }
    // fork the expert lanes off the caller's stream
    if (nmax > 0) {
      cudaError_t e = cudaEventRecord(c->moe_ev[mxq_context::kMoeLanes], c->stream);
      for (int l = 0; l < mxq_context::kMoeLanes && e == cudaSuccess; ++l)
        e = cudaStreamWaitEvent(c->moe_st[l], c->moe_ev[mxq_context::kMoeLanes], 0);
      if (e != cudaSuccess) return cuda_fail(c, e, "moe fork");
    }
    // an error return between the fork and the join still makes the
    // caller's stream wait for whatever the lanes have queued
    struct LaneJoinOnError {
      mxq_context* c;
      bool armed;
      ~LaneJoinOnError() {
        if (!armed) return;
        for (int l = 0; l < mxq_context::kMoeLanes; ++l)
          if (cudaEventRecord(c->moe_ev[l], c->moe_st[l]) == cudaSuccess)
            cudaStreamWaitEvent(c->stream, c->moe_ev[l], 0);
      }
    } join_guard{c, nmax > 0};
    // expert j (in id order, non-empty ones) runs on lane j % kMoeLanes with
    // that lane's workspaces; the swap below is undone on every exit
    struct LaneSwap {
      mxq_context* c;
      cudaStream_t st;
      uint8_t* op;
      float *f0, *f1;
      explicit LaneSwap(mxq_context* cc) : c(cc), st(cc->stream), op(cc->ws_op), f0(cc->ws_f0), f1(cc->ws_f1) {}
      void use(int l) {
        c->stream = c->moe_st[l];
        c->ws_op = c->ml_op[l];
        c->ws_f0 = c->ml_f0[l];
        c->ws_f1 = c->ml_f1[l];
      }
      ~LaneSwap() {
        c->stream = st;
        c->ws_op = op;
        c->ws_f0 = f0;
        c->ws_f1 = f1;
      }
    };
    int off = 0, lane_j = 0;
    for (int e = 0; e < E; ++e) {
      const int ne = c->moe_counts_host[e];
      if (e < e_lo || e >= e_lo + n_local) {   // another rank's expert: its slots stay in place
        off += ne;
        continue;
      }
      if (ne == 0) continue;
      const mxq_weight* wg = w_gate - e_lo;
      const mxq_weight* wu = w_up - e_lo;
      const mxq_weight* wdn = w_down - e_lo;
      LaneSwap lane(c);
      lane.use(lane_j++ % mxq_context::kMoeLanes);
      const int BN = gemm_pick_bn(ne), Bpad = (ne + BN - 1) / BN * BN;
      const WeightView &gv = wg[e]->v, &uv = wu[e]->v;
      if ((rc = moe_operand(c, wg[e], x, slot_token + off, ne, D, BN, Bpad))) return rc;
      if ((rc = moe_gemm(c, wg[e], ne, BN, Bpad, c->ws_f0))) return rc;
      if (uv.fmt != gv.fmt || uv.gemm_shift != gv.gemm_shift || uv.Kpad != gv.Kpad)
        if ((rc = moe_operand(c, wu[e], x, slot_token + off, ne, D, BN, Bpad))) return rc;
      if ((rc = moe_gemm(c, wu[e], ne, BN, Bpad, c->ws_f1))) return rc;
      // silu(gate) * up -> the down projection's operand
      QuantArgs qa{};
      qa.x = c->ws_f0;
      qa.up = c->ws_f1;
      qa.B = ne;
      qa.K = F;
      qa.opnd = reinterpret_cast<__nv_bfloat16*>(c->ws_op);
      qa.Bpad = Bpad;
      qa.Kpad = wdn[e]->v.Kpad;
      qa.BN = BN;
      qa.int4_order = wdn[e]->v.fmt == 4;
      qa.shift = wdn[e]->v.gemm_shift;
      if ((rc = after_launch(c, launch_quantize(qa, 2, c->stream, true), "moe swiglu"))) return rc;
      if ((rc = moe_gemm(c, wdn[e], ne, BN, Bpad, yr + (size_t)off * D))) return rc;
      off += ne;
    }
    // join: the combine on the caller's stream waits for every lane
    join_guard.armed = false;
    if (nmax > 0) {
      cudaError_t e = cudaSuccess;
      for (int l = 0; l < mxq_context::kMoeLanes && e == cudaSuccess; ++l) {
        e = cudaEventRecord(c->moe_ev[l], c->moe_st[l]);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(c->stream, c->moe_ev[l], 0);
      }
      if (e != cudaSuccess) return cuda_fail(c, e, "moe join");
    }
    if (G) {
      // this rank's slot rows [off_lo, off_hi) to the same rows of every other
      // rank's mailbox; then wait for every rank's
      TpGatherArgs a{};
      a.world = G->world;
      a.rank = G->rank;
      a.rows = off_hi - off_lo;
      a.skip_rank = G->rank;
      a.src = reinterpret_cast<const uint8_t*>(yr + (size_t)off_lo * D);
      a.row_bytes = (size_t)D * 4;
      a.dst_off = G->off_yr + (size_t)(G->calls & 1u) * G->half_bytes + (size_t)off_lo * D * 4;
      a.row_stride = (size_t)D * 4;
      a.rank_stride = 0;
      for (int r = 0; r < G->world; ++r) {
        a.base[r] = G->base[r];
        a.flag_out[r] = reinterpret_cast<uint32_t*>(G->base[r]) + G->rank;
      }
      a.wait_flags = reinterpret_cast<const uint32_t*>(G->mbox);
      a.seq = G->local;
      a.grid_cnt = G->local + 1;
      a.status = c->status;
      a.wait_ns = G->wait_ns;
      if ((rc = after_launch(c, launch_tp_gather(a, c->stream), "moe expert-output exchange"))) return rc;
      G->calls += 1;
    }
    return after_launch(c, launch_moe_combine(yr, gate, route_pos, T, D, K, y, c->stream), "moe combine");
  }
}

int mxq_moe_group_create(mxq_ctx c, int rank, int world, size_t max_tokens, size_t top_k, size_t d_model,
                         mxq_moe_group* out, void* handle_out) {
  MXQ_TRY({
    if (int rc = check_ctx(c)) return rc;
    if (!out || !handle_out) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null pointer");
    *out = nullptr;
    if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world)
      return fail(c, MXQ_ERR_INVALID_ARGUMENT, "moe group: rank %d of world %d (1..%d ranks)", rank, world, kMaxPeers);
    if (max_tokens == 0 || top_k == 0 || d_model == 0 || d_model % 4 || max_tokens * top_k > (1u << 26))
      return fail(c, MXQ_ERR_INVALID_ARGUMENT, "moe group: max_tokens, top_k > 0, d_model a multiple of 4");
    DeviceGuard g(c->device);
    auto* G = new mxq_moe_group_s();
    G->ctx = c;
    G->rank = rank;
    G->world = world;
    G->max_routes = max_tokens * top_k;
    G->D = d_model;
    G->half_bytes = (G->max_routes * d_model * 4 + 255) / 256 * 256;
    G->bytes = G->off_yr + 2 * G->half_bytes;
    cudaError_t e = cudaMalloc(&G->mbox, G->bytes);
    if (e == cudaSuccess) e = cudaMemset(G->mbox, 0, G->off_yr);
    if (e == cudaSuccess) e = cudaMalloc(&G->local, 4 * sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMemset(G->local, 0, 4 * sizeof(uint32_t));
    cudaIpcMemHandle_t h{};
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, G->mbox);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
      cudaFree(G->mbox);
      cudaFree(G->local);
      delete G;
      return cuda_fail(c, e, "moe group mailbox");
    }
    std::memcpy(handle_out, &h, sizeof(h));
    G->base[rank] = G->mbox;
    *out = G;
    return MXQ_OK;
  })
}

int mxq_moe_group_connect(mxq_moe_group G, const void* handles) {
  MXQ_TRY({
    if (!G || !handles) return fail(nullptr, MXQ_ERR_INVALID_ARGUMENT, "null pointer");
    mxq_context* c = G->ctx;
    DeviceGuard g(c->device);
    for (int r = 0; r < G->world; ++r) {
      if (r == G->rank || G->base[r]) continue;
      cudaIpcMemHandle_t h;
      std::memcpy(&h, static_cast<const uint8_t*>(handles) + (size_t)r * sizeof(h), sizeof(h));
      void* p = nullptr;
      const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
      if (e != cudaSuccess) return cuda_fail(c, e, "open a peer's moe mailbox");
      G->base[r] = static_cast<uint8_t*>(p);
      G->opened[r] = true;
    }
    return MXQ_OK;
  })
}

int mxq_moe_group_set_wait_limit(mxq_moe_group G, uint32_t wait_us) {
  if (!G) return fail(nullptr, MXQ_ERR_INVALID_ARGUMENT, "null moe group");
  if (wait_us == 0 || wait_us > 10000000u)
    return fail(G->ctx, MXQ_ERR_INVALID_ARGUMENT, "moe group wait limit must be in [1, 1e7] microseconds");
  G->wait_ns = (uint64_t)wait_us * 1000ull;
  return MXQ_OK;
}

int mxq_moe_group_destroy(mxq_moe_group G) {
  if (!G) return fail(nullptr, MXQ_ERR_INVALID_ARGUMENT, "null moe group");
  DeviceGuard g(G->ctx->device);
  cudaDeviceSynchronize();
  for (int r = 0; r < G->world; ++r)
    if (G->opened[r]) cudaIpcCloseMemHandle(G->base[r]);
  cudaFree(G->mbox);
  cudaFree(G->local);
  delete G;
  return MXQ_OK;
}

int mxq_moe_swiglu_sharded(mxq_ctx c, mxq_moe_group G, const mxq_weight* w_gate, const mxq_weight* w_up,
                           const mxq_weight* w_down, size_t n_experts, const float* x, const float* logits,
                           size_t t, size_t k, float* y) {
  MXQ_TRY({
    if (int rc = check_ctx(c)) return rc;
    if (!G || !w_gate || !w_up || !w_down || !x || !logits || !y || n_experts == 0)
      return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null pointer or no experts");
    if (G->ctx != c) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "moe group belongs to another context");
    for (int r = 0; r < G->world; ++r)
      if (!G->base[r]) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "moe group not connected (mxq_moe_group_connect)");
    if (!aligned16(x)) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "fp32 input must be 16-byte aligned (it is read in 16-byte vectors)");
    if (n_experts % (size_t)G->world)
      return fail(c, MXQ_ERR_INVALID_ARGUMENT, "expert-parallel moe: %zu experts do not split over %d ranks", n_experts,
                  G->world);
    if (k == 0 || k > n_experts)
      return fail(c, MXQ_ERR_INVALID_ARGUMENT, "top-k: k=%zu must be in [1, n_experts=%zu]", k, n_experts);
    if (k > 64 || n_experts > 4096) return fail(c, MXQ_ERR_UNSUPPORTED, "top-k: k <= 64 and n_experts <= 4096");
    const int E = (int)n_experts, El = E / G->world;
    for (int e = 0; e < El; ++e) {
      if (int rc = check_weight(c, w_gate[e])) return rc;
      if (int rc = check_weight(c, w_up[e])) return rc;
      if (int rc = check_weight(c, w_down[e])) return rc;
    }
    const int D = w_gate[0]->v.K, F = w_gate[0]->v.N;
    for (int e = 0; e < El; ++e) {
      const WeightView &g = w_gate[e]->v, &u = w_up[e]->v, &d = w_down[e]->v;
      if (g.K != D || g.N != F || u.K != D || u.N != F || d.K != F || d.N != D)
        return fail(c, MXQ_ERR_INVALID_ARGUMENT,
                    "expert %d shapes: gate/up must be [%d][%d] and down [%d][%d]", e, F, D, D, F);
    }
    if ((size_t)D != G->D) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "moe group sized for d_model %zu, experts have %d", G->D, D);
    if (t == 0) return MXQ_OK;
    if (t * k > G->max_routes)
      return fail(c, MXQ_ERR_INVALID_ARGUMENT, "moe group sized for %zu routes, got %zu tokens x top-%zu", G->max_routes,
                  t, k);
    DeviceGuard g(c->device);
    return moe_layer(c, w_gate, w_up, w_down, E, G->rank * El, El, x, logits, (int)t, (int)k, D, F, y, G);
  })
}

int mxq_debug_gemm_stall(mxq_ctx c, mxq_weight w, const float* x, size_t b, float* y, uint32_t wait_us) {
  MXQ_TRY({
    if (int rc = check_ctx(c)) return rc;
    if (int rc = check_weight(c, w)) return rc;
    if (!x || !y || b == 0) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null pointer or empty batch");
    if (!aligned16(x)) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "fp32 input must be 16-byte aligned (it is read in 16-byte vectors)");
    if (wait_us == 0 || wait_us > 1000000u)
      return fail(c, MXQ_ERR_INVALID_ARGUMENT, "debug stall: wait limit must be in [1, 1e6] microseconds");
    DeviceGuard g(c->device);
    const int BN = gemm_pick_bn((int)b);
    const int Bpad = (int)((b + BN - 1) / BN * BN);
    int rc;
    if ((rc = ensure(c, c->ws_op, c->ws_op_bytes, (size_t)Bpad * w->v.Kpad * 2, "workspace operand"))) return rc;
    QuantArgs qa{};
    qa.x = x;
    qa.B = (int)b;
    qa.K = w->v.K;
    qa.opnd = reinterpret_cast<__nv_bfloat16*>(c->ws_op);
    qa.Bpad = Bpad;
    qa.Kpad = w->v.Kpad;
    qa.BN = BN;
    qa.int4_order = w->v.fmt == 4;
    qa.shift = w->v.gemm_shift;
    if ((rc = after_launch(c, launch_quantize(qa, MXQ_ACT_NONE, c->stream, false), "quantize"))) return rc;
    GemmArgs ga{};
    ga.w = w->v;
    ga.opnd = qa.opnd;
    ga.y = y;
    ga.B = (int)b;
    ga.Bpad = Bpad;
    ga.BN = BN;
    ga.status = c->status;
    ga.splits = 1;
    ga.wait_ns = (uint64_t)wait_us * 1000ull;
    ga.withhold_x0 = 1;
    if ((rc = after_launch(c, launch_gemm(ga, c->stream, false), "gemm"))) return rc;
    return mxq_synchronize(c);
  })
}

int mxq_route_topk(mxq_ctx c, const float* logits, size_t t, size_t n_experts,
                   size_t k, int32_t* idx, float* gate) {
  if (int rc = check_ctx(c)) return rc;
  if (!logits || !idx || !gate) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null pointer");
  if (k == 0 || k > n_experts)
    return fail(c, MXQ_ERR_INVALID_ARGUMENT, "top-k: k=%zu must be in [1, n_experts=%zu]", k, n_experts);
  if (k > 64 || n_experts > 4096) return fail(c, MXQ_ERR_UNSUPPORTED, "top-k: k <= 64 and n_experts <= 4096");
  if (t == 0) return MXQ_OK;
  DeviceGuard g(c->device);
  route_topk_kernel<<<(unsigned)((t + 127) / 128), 128, 0, c->stream>>>(logits, (int)t, (int)n_experts,
                                                                     (int)k, idx, gate);
  return after_launch(c, cudaGetLastError(), "route_topk");
}

int mxq_gae(mxq_ctx c, const float* rewards, const float* values, const uint8_t* dones,
            const float* next_values, size_t t, size_t e, float gamma, float lambda,
            float* adv, float* ret) {
  if (int rc = check_ctx(c)) return rc;
  if (!rewards || !values || !dones || !next_values || !adv || !ret)
    return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null pointer");
  if (t == 0 || e == 0) return MXQ_OK;  // the reference returns early on an empty sweep
  DeviceGuard g(c->device);
  const float gl = gamma * lambda;
  gae_kernel<<<(unsigned)((e + 127) / 128), 128, 0, c->stream>>>(rewards, values, dones, next_values,
                                                                (int)t, (int)e, gamma, gl, adv, ret);
  return after_launch(c, cudaGetLastError(), "gae");
}

int mxq_quantize_w(mxq_ctx c, int fmt, const float* w, size_t n, size_t k, void* data, uint8_t* scales,
                   int32_t* w_sums) {
  if (int rc = check_ctx(c)) return rc;
  if (!w || !data || !scales) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null pointer");
  if (fmt != MXQ_FMT_INT4 && fmt != MXQ_FMT_INT8)
    return fail(c, MXQ_ERR_INVALID_ARGUMENT, "unknown weight format %d", fmt);
  if (n == 0 || k == 0 || k % kBlock)
    return fail(c, MXQ_ERR_INVALID_ARGUMENT, "quantize_w: K must be a positive multiple of 32");
  if (n > (1u << 24) || k > (1u << 24)) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "quantize_w: shape too large");
  DeviceGuard g(c->device);
  return after_launch(c, launch_quantize_w(fmt, w, (int)n, (int)k, static_cast<uint8_t*>(data), scales, w_sums,
                                           c->stream), "quantize_w");
}

int mxq_weight_quantize(mxq_ctx c, int fmt, size_t n, size_t k, const float* w, int on_device, mxq_weight* out) {
  MXQ_TRY({
    if (int rc = check_ctx(c)) return rc;
    if (!w || !out) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null pointer");
    *out = nullptr;
    if (fmt != MXQ_FMT_INT4 && fmt != MXQ_FMT_INT8)
      return fail(c, MXQ_ERR_INVALID_ARGUMENT, "unknown weight format %d", fmt);
    if (n == 0 || k == 0 || k % kBlock)
      return fail(c, MXQ_ERR_INVALID_ARGUMENT, "weight_quantize: K must be a positive multiple of 32");
    if (n > (1u << 24) || k > (1u << 24)) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "weight_quantize: shape too large");
    DeviceGuard g(c->device);
    // scratch: quantised bytes, scales, then (host input) the fp32 rows at a
    // 16-byte boundary
    const size_t data_bytes = fmt == 4 ? n * k / 2 : n * k, sc_bytes = n * k / kBlock;
    const size_t off = (data_bytes + sc_bytes + 15) / 16 * 16;
    const size_t in_bytes = on_device ? 0 : n * k * 4;
    uint8_t* tmp = nullptr;
    cudaError_t e = cudaMalloc(&tmp, off + in_bytes);
    if (e != cudaSuccess) return cuda_fail(c, e, "weight_quantize scratch");
    const float* src = w;
    if (!on_device) {
      float* staged = reinterpret_cast<float*>(tmp + off);
      e = cudaMemcpyAsync(staged, w, in_bytes, cudaMemcpyHostToDevice, c->stream);
      src = staged;
    }
    if (e == cudaSuccess) e = launch_quantize_w(fmt, src, (int)n, (int)k, tmp, tmp + data_bytes, nullptr, c->stream);
    if (e != cudaSuccess) {
      cudaStreamSynchronize(c->stream);
      cudaFree(tmp);
      return cuda_fail(c, e, "weight_quantize");
    }
    c->launches++;
    const int rc = mxq_weight_create(c, fmt, n, k, tmp, tmp + data_bytes, 1, out);
    cudaStreamSynchronize(c->stream);
    cudaFree(tmp);
    return rc;
  })
}

int mxq_halting_step_host(mxq_ctx c, mxq_weight w, const uint8_t* xq, const uint8_t* xs, float bias,
                          mxq_halting_state* state, float* p, uint8_t* should_halt) {
  MXQ_TRY({
    if (int rc = check_ctx(c)) return rc;
    if (!state || !p || !should_halt) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null pointer");
    DeviceGuard g(c->device);
    int rc;
    // device staging: [state 16 B][p 4 B][halt 1 B]
    if ((rc = ensure(c, c->ws_out, c->ws_out_bytes, 32, "workspace out"))) return rc;
    uint8_t* base = reinterpret_cast<uint8_t*>(c->ws_out);
    auto* dst = reinterpret_cast<mxq_halting_state*>(base);
    float* dp = reinterpret_cast<float*>(base + 16);
    uint8_t* dh = base + 20;
    cudaError_t e = cudaMemcpyAsync(dst, state, sizeof(mxq_halting_state), cudaMemcpyHostToDevice, c->stream);
    if (e != cudaSuccess) return cuda_fail(c, e, "copy in");
    if ((rc = mxq_halting_step(c, w, xq, xs, 1, bias, dst, dp, dh))) return rc;
    e = cudaMemcpyAsync(state, dst, sizeof(mxq_halting_state), cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(p, dp, 4, cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(should_halt, dh, 1, cudaMemcpyDeviceToHost, c->stream);
    if (e != cudaSuccess) return cuda_fail(c, e, "copy out");
    return mxq_synchronize(c);
  })
}

int mxq_rank16_dot_ptrs(mxq_ctx c, const mxq_weight* rows, size_t nrows, const uint8_t* xq, const uint8_t* xs,
                        size_t b, float* y) {
  if (int rc = check_ctx(c)) return rc;
  if (!rows || !xq || !xs || !y || b == 0 || nrows == 0)
    return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null pointer or empty input");
  if (nrows > (size_t)kRowPtrsMax)
    return fail(c, MXQ_ERR_INVALID_ARGUMENT, "rank16_dot_ptrs: at most %d weights per call", kRowPtrsMax);
  if (b > (1u << 20)) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "rank16_dot_ptrs: batch too large");
  if (!aligned16(xq)) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "activation must be 16-byte aligned");
  const WeightView* v[kRowPtrsMax];
  for (size_t j = 0; j < nrows; ++j) {
    if (int rc = check_weight(c, rows[j])) return rc;
    if (int rc = reject_sparse(c, rows[j], "rank16_dot_ptrs")) return rc;
    v[j] = &rows[j]->v;
    if (v[j]->fmt != v[0]->fmt || v[j]->K != v[0]->K)
      return fail(c, MXQ_ERR_INVALID_ARGUMENT, "rank16_dot_ptrs: weight %zu differs in format or K", j);
  }
  DeviceGuard g(c->device);
  return after_launch(c, launch_row_ptrs(v, (int)nrows, xq, xs, (int)b, y, c->stream), "rank16_dot_ptrs");
}

int mxq_halting_step(mxq_ctx c, mxq_weight w, const uint8_t* xq, const uint8_t* xs, size_t b, float bias,
                     mxq_halting_state* state, float* p, uint8_t* should_halt) {
  if (int rc = check_ctx(c)) return rc;
  if (int rc = check_weight(c, w)) return rc;
  if (!xq || !xs || !state || !p || !should_halt || b == 0)
    return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null pointer or empty batch");
  if (int rc = reject_sparse(c, w, "halting_step")) return rc;
  if (w->v.N != 1) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "halting_step: w_halt must have 1 row, has %d", w->v.N);
  if (b > (1u << 24)) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "halting_step: batch too large");
  if (!aligned16(xq)) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "activation must be 16-byte aligned");
  DeviceGuard g(c->device);
  return after_launch(c, launch_halting(w->v, xq, xs, (int)b, bias, MXQ_HALT_EPS, state, p, should_halt, c->stream),
                      "halting_step");
}

static int hashed_route_check(mxq_context* c, size_t t, size_t d, size_t n_experts, size_t top_k, size_t n_hashes) {
  if (top_k == 0 || top_k > n_experts)
    return fail(c, MXQ_ERR_INVALID_ARGUMENT, "HashedRouter: top_k (%zu) must be in [1, n_experts=%zu]", top_k,
                n_experts);
  if (top_k > 64 || n_experts > 65536) return fail(c, MXQ_ERR_UNSUPPORTED, "HashedRouter: top_k <= 64, n_experts <= 65536");
  if (n_hashes == 0 || n_hashes > 32) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "HashedRouter: n_hashes must be in [1, 32]");
  if (d == 0 || d % kBlock || d > (1u << 24)) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "HashedRouter: d must be a positive multiple of 32");
  if (t > (1u << 24)) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "HashedRouter: too many tokens");
  return MXQ_OK;
}

int mxq_hashed_route(mxq_ctx c, const float* x, size_t t, size_t d, size_t n_experts, size_t top_k,
                     size_t n_hashes, uint64_t seed, int32_t* idx, int32_t* score) {
  if (int rc = check_ctx(c)) return rc;
  if (!x || !idx || !score) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null pointer");
  if (int rc = hashed_route_check(c, t, d, n_experts, top_k, n_hashes)) return rc;
  if (t == 0) return MXQ_OK;
  DeviceGuard g(c->device);
  return after_launch(c, launch_hashed_route(x, (int)t, (int)d, (int)n_experts, (int)top_k, (int)n_hashes, seed,
                                             idx, score, c->stream), "hashed_route");
}

int mxq_hashed_route_host(mxq_ctx c, const float* x, size_t t, size_t d, size_t n_experts, size_t top_k,
                          size_t n_hashes, uint64_t seed, int32_t* idx, int32_t* score) {
  MXQ_TRY({
    if (int rc = check_ctx(c)) return rc;
    if (!x || !idx || !score) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null pointer");
    if (int rc = hashed_route_check(c, t, d, n_experts, top_k, n_hashes)) return rc;
    if (t == 0) return MXQ_OK;
    DeviceGuard g(c->device);
    int rc;
    const size_t in_bytes = t * d * 4, out_bytes = 2 * t * top_k * 4;
    if ((rc = ensure(c, c->ws_in, c->ws_in_bytes, in_bytes, "workspace in"))) return rc;
    if ((rc = ensure(c, c->ws_out, c->ws_out_bytes, out_bytes, "workspace out"))) return rc;
    int32_t* didx = reinterpret_cast<int32_t*>(c->ws_out);
    int32_t* dsc = didx + t * top_k;
    cudaError_t e = cudaMemcpyAsync(c->ws_in, x, in_bytes, cudaMemcpyHostToDevice, c->stream);
    if (e != cudaSuccess) return cuda_fail(c, e, "copy in");
    if ((rc = after_launch(c, launch_hashed_route(c->ws_in, (int)t, (int)d, (int)n_experts, (int)top_k,
                                                  (int)n_hashes, seed, didx, dsc, c->stream), "hashed_route")))
      return rc;
    e = cudaMemcpyAsync(idx, didx, t * top_k * 4, cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(score, dsc, t * top_k * 4, cudaMemcpyDeviceToHost, c->stream);
    if (e != cudaSuccess) return cuda_fail(c, e, "copy out");
    return mxq_synchronize(c);
  })
}

int mxq_update_gaussian_moment(mxq_ctx c, mxq_weight w, const float* g, const float* x, float step) {
  if (int rc = check_ctx(c)) return rc;
  if (int rc = check_weight(c, w)) return rc;
  if (!g || !x) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null pointer");
  if (int rc = reject_sparse(c, w, "update_gaussian_moment")) return rc;
  if (!(step == step) || step - step != 0.0f) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "update: step must be finite");
  DeviceGuard g_(c->device);
  // every cached host-call graph stays valid: the weight's buffers do not move
  return after_launch(c, launch_moment_update(w->v, g, x, step, w->data, c->stream), "update_gaussian_moment");
}

int mxq_activation_norm(mxq_ctx c, const uint8_t* xq, const uint8_t* xs, size_t b, size_t k, float* norms) {
  if (int rc = check_ctx(c)) return rc;
  if (!xq || !xs || !norms || b == 0) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null pointer or empty batch");
  if (k == 0 || k % kBlock || k > (1u << 24) || b > (1u << 24))
    return fail(c, MXQ_ERR_INVALID_ARGUMENT, "activation_norm: K a positive multiple of 32");
  DeviceGuard g(c->device);
  return after_launch(c, launch_act_norm(xq, xs, (int)b, (int)k, norms, c->stream), "activation_norm");
}

int mxq_micro_moe(mxq_ctx c, mxq_weight wg, mxq_weight wu, mxq_weight wd, size_t n_routed, size_t n_shared,
                  const float* x, const int32_t* idx, const float* gate, size_t t, size_t k, float* y) {
  if (int rc = check_ctx(c)) return rc;
  if (int rc = check_weight(c, wg)) return rc;
  if (int rc = check_weight(c, wu)) return rc;
  if (int rc = check_weight(c, wd)) return rc;
  if (!x || !y || (k > 0 && !idx)) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null pointer");
  if (int rc = reject_sparse(c, wg, "micro_moe")) return rc;
  if (int rc = reject_sparse(c, wu, "micro_moe")) return rc;
  if (int rc = reject_sparse(c, wd, "micro_moe")) return rc;
  if (k > n_routed) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "micro_moe: top_k (%zu) exceeds n_experts (%zu)", k, n_routed);
  if (k > 64 || n_shared > 8 || k + n_shared == 0)
    return fail(c, MXQ_ERR_INVALID_ARGUMENT, "micro_moe: top_k <= 64, n_shared <= 8, at least one expert");
  const size_t E = n_routed + n_shared;
  const WeightView &g = wg->v, &u = wu->v, &d = wd->v;
  if ((size_t)g.N != E * 16 || (size_t)u.N != E * 16 || g.K != u.K || (size_t)d.K != E * 16 || d.N != g.K)
    return fail(c, MXQ_ERR_INVALID_ARGUMENT,
                "micro_moe: gate/up pools must be [%zu][D], down [D][%zu] (16 rows per expert)", E * 16, E * 16);
  if (E % 2) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "micro_moe: the expert count (routed + shared) must be even");
  if (t == 0) return MXQ_OK;
  if (t > (1u << 24)) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "micro_moe: too many tokens");
  DeviceGuard g_(c->device);
  return after_launch(c, launch_micro_moe(g, u, d, (int)n_routed, (int)n_shared, x, idx, gate, (int)t, (int)k, y,
                                          c->stream), "micro_moe");
}

int mxq_gae_ring(mxq_ctx c, const float* rewards, const float* values, const uint8_t* dones,
                 const float* next_values, size_t capacity, size_t size, size_t cursor, size_t t,
                 size_t e, float gamma, float lambda, float* adv, float* ret) {
  if (int rc = check_ctx(c)) return rc;
  if (!rewards || !values || !dones || !next_values || !adv || !ret)
    return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null pointer");
  if (capacity == 0 || size > capacity || cursor >= capacity || capacity > ((size_t)1 << 40))
    return fail(c, MXQ_ERR_INVALID_ARGUMENT, "gae ring: need size <= capacity, cursor < capacity");
  if (size < capacity && cursor != size % capacity)
    return fail(c, MXQ_ERR_INVALID_ARGUMENT, "gae ring: a ring that is not full has cursor == size");
  // agentic_env/replay_memory.cpp:205-213: empty sweep, truncation to what is stored
  size_t total = t * e;
  if (t == 0 || e == 0 || size == 0) return MXQ_OK;
  if (total > size) {
    t = size / e;
    total = t * e;
  }
  if (t == 0) return MXQ_OK;
  if (t > (size_t)INT32_MAX || e > (size_t)INT32_MAX) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "gae ring: too large");
  const size_t start = (capacity + cursor - total) % capacity;
  const int active = (int)(e > 1024 ? 1024 : e);   // the reference's MAX_ENVS
  DeviceGuard g(c->device);
  const float gl = gamma * lambda;
  gae_ring_kernel<<<(unsigned)((active + 127) / 128), 128, 0, c->stream>>>(
      rewards, values, dones, next_values, (long)capacity, (long)start, (int)t, (int)e, active, gamma, gl, adv, ret);
  return after_launch(c, cudaGetLastError(), "gae ring");
}

}  // extern "C"

namespace mxq {
cudaStream_t ctx_stream(mxq_context* c) { return c->stream; }
void ctx_set_stream_raw(mxq_context* c, cudaStream_t s) { c->stream = s; }
int ctx_fail(mxq_context* c, int code, const char* msg) { return fail(c, code, "%s", msg); }
int ctx_cuda_fail(mxq_context* c, cudaError_t e, const char* what) { return cuda_fail(c, e, what); }
uint32_t* ctx_status_word(mxq_context* c) { return c->status; }
int ctx_device(mxq_context* c) { return c->device; }
void ctx_add_launches(mxq_context* c, uint64_t n) { c->launches += n; }
uint64_t ctx_ws_gen(mxq_context* c) { return c->ws_gen; }
uint64_t ctx_launches(mxq_context* c) { return c->launches; }
void ctx_set_launches(mxq_context* c, uint64_t n) { c->launches = n; }
const WeightView* weight_view(mxq_weight w) { return w ? &w->v : nullptr; }

cudaError_t launch_scale_range(const uint8_t* scales, size_t count, uint32_t* out2, cudaStream_t st) {
  size_t ctas = (count + 255) / 256;
  if (ctas > 1024) ctas = 1024;
  if (ctas < 1) ctas = 1;
  scale_range_kernel<<<(unsigned)ctas, 256, 0, st>>>(scales, count, out2);
  return cudaGetLastError();
}

cudaError_t launch_repack(const uint8_t* data, const uint8_t* scales, int fmt, int N, int K,
                          int Npad, int Kpad, uint8_t* od, uint8_t* os, cudaStream_t st) {
  const long total = (long)Npad * (Kpad / kTileK);
  long ctas = (total + 255) / 256;
  if (ctas > 148L * 64) ctas = 148L * 64;
  repack_kernel<<<(unsigned)ctas, 256, 0, st>>>(data, scales, fmt, N, K, Npad, Kpad, od, os);
  return cudaGetLastError();
}
}  // namespace mxq

// ------------------------------------------------ linear without allocation
// mxq_linear_noalloc: the tensor-core linear (quantiser -> bf16 operand ->
// tcgen05 GEMM) with its operand scratch in a fixed device array instead of
// the context workspace, for callers that may not allocate device memory.
#include <mutex>

namespace {

// Operand scratch: Bpad x Kpad bf16 values.  Every GPU that loads this
// library holds it until the process exits.
constexpr size_t kNoallocScratchBytes = (size_t)4 << 20;   // 4 MiB
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoallocScratchBytes];

constexpr int kNoallocMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kNoallocMaxDevices] = {};

// Device address of g_noalloc_scratch on the context's device, looked up once
// per device with that device current.  In host code the symbol's name is
// only a host-side stand-in, so the kernels get this address instead.
int noalloc_scratch(mxq_context* c, void** out) {
  if (c->device < 0 || c->device >= kNoallocMaxDevices)
    return fail(c, MXQ_ERR_UNSUPPORTED, "mxq_linear_noalloc: device %d beyond %d", c->device, kNoallocMaxDevices);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_addr[c->device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) return cuda_fail(c, e, "mxq_linear_noalloc: scratch address");
    g_noalloc_addr[c->device] = p;
  }
  *out = g_noalloc_addr[c->device];
  return MXQ_OK;
}

}  // namespace

extern "C" int mxq_linear_noalloc(mxq_ctx c, mxq_weight w, const float* x, size_t b, float* y) {
  MXQ_TRY({
    if (int rc = check_ctx(c)) return rc;
    if (int rc = check_weight(c, w)) return rc;
    if (!x || !y || b == 0) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "null pointer or empty batch");
    if (!aligned16(x)) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "fp32 input must be 16-byte aligned (it is read in 16-byte vectors)");
    if (b > (size_t)(1 << 20)) return fail(c, MXQ_ERR_INVALID_ARGUMENT, "mxq_linear_noalloc: batch %zu too large", b);
    DeviceGuard g(c->device);   // the scratch address is per device: look it up with the device current
    const int BN = gemm_pick_bn((int)b);
    const size_t Bpad = (b + BN - 1) / BN * BN;
    const size_t need = Bpad * (size_t)w->v.Kpad * 2;
    if (need > kNoallocScratchBytes)
      return fail(c, MXQ_ERR_INVALID_ARGUMENT,
                  "mxq_linear_noalloc: batch %zu x K %d needs %zu bytes of scratch, more than the fixed %zu",
                  b, w->v.K, need, kNoallocScratchBytes);
    void* scratch = nullptr;
    if (int rc = noalloc_scratch(c, &scratch)) return rc;
    // the quantiser writes every element of the Bpad x Kpad operand (padding
    // included), so nothing left in the shared array from an earlier call is read
    QuantArgs qa{};
    qa.x = x;
    qa.B = (int)b;
    qa.K = w->v.K;
    qa.opnd = static_cast<__nv_bfloat16*>(scratch);
    qa.Bpad = (int)Bpad;
    qa.Kpad = w->v.Kpad;
    qa.BN = BN;
    qa.int4_order = w->v.fmt == 4;
    qa.shift = w->v.gemm_shift;
    if (int rc = after_launch(c, launch_quantize(qa, MXQ_ACT_NONE, c->stream, true), "quantize")) return rc;
    GemmArgs ga{};
    ga.w = w->v;
    ga.opnd = qa.opnd;
    ga.y = y;
    ga.B = (int)b;
    ga.Bpad = (int)Bpad;
    ga.BN = BN;
    ga.status = c->status;
    return after_launch(c, launch_gemm(ga, c->stream, true), "gemm");
  })
}
