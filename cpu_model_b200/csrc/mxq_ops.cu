// mxq_ops.cu -- the small MX operators around the linear layer:
//   mx_quantize_w   fp32 weight rows -> int8 / packed int4 + E8M0 + w_sums
//                   (nn/tests/test_auto_generated.cpp:46; training/fidelity_test.cpp:60-61);
//   halting_step    1-row MX dot + bias -> sigmoid -> ACT halting state
//                   (nn/core/layers/halting.hpp:16-30);
//   mx_rank16_dot_ptrs  dots against rows held by separate weight handles
//                   (nn/tests/test_auto_generated.cpp:55; pointer array
//                   nn/tests/autotest.hpp:126-136);
//   HashedRouter::route  LSH (sign-of-projection) top-K expert selection
//                   (nn/tests/test_robustness.cpp:13-35; "Rank-16 VNNI LSH
//                   router", nn/docs/job.md:11).
//
// The dot products here are one warp per (token, row): lane l takes the
// 32-element blocks l, l+32, ... in order, forms each block's exact int32 dot
// (dp4a), scales it by 2^e_x then 2^e_w in fp32 and adds it to its running
// sum; the 32 lane sums are combined by a fixed xor-butterfly.  The oracle
// restates exactly this order, so these results are bit-identical to it.
#include "../../include/mxq.h"
#include "mxq_internal.h"

namespace mxq {

namespace {

// int4 word (8 nibbles, element 2i low) -> two words of 16*w in natural order
__device__ __forceinline__ void nib_x16(uint32_t w, uint32_t& n0, uint32_t& n1) {
  const uint32_t lo = (w << 4) & 0xF0F0F0F0u;
  const uint32_t hi = w & 0xF0F0F0F0u;
  n0 = __byte_perm(lo, hi, 0x5140);
  n1 = __byte_perm(lo, hi, 0x7362);
}

// Byte offset of block b of row r in the tiled layout (data: TB bytes per row
// per 64-K tile, the block's half of it; scales: 2 bytes per row per tile).
__device__ __forceinline__ size_t tiled_row(int r, int kt, int KT) {
  return ((size_t)(r >> 7) * KT + kt) * 128 + (r & 127);
}

// Exact int32 dot of activation block (32 u8 = q+128) with weight block b of
// row r.
__device__ __forceinline__ int block_dot(const WeightView& w, int r, int b, const uint8_t* xblk) {
  const int KT = w.Kpad / kTileK;
  const size_t tr = tiled_row(r, b >> 1, KT);
  const uint4 x0 = *reinterpret_cast<const uint4*>(xblk);
  const uint4 x1 = *reinterpret_cast<const uint4*>(xblk + 16);
  const uint32_t xs[8] = {x0.x ^ 0x80808080u, x0.y ^ 0x80808080u, x0.z ^ 0x80808080u, x0.w ^ 0x80808080u,
                          x1.x ^ 0x80808080u, x1.y ^ 0x80808080u, x1.z ^ 0x80808080u, x1.w ^ 0x80808080u};
  int d = 0;
  if (w.fmt == 8) {
    const uint8_t* p = w.data + tr * 64 + (b & 1) * 32;
    const uint4 w0 = *reinterpret_cast<const uint4*>(p);
    const uint4 w1 = *reinterpret_cast<const uint4*>(p + 16);
    const uint32_t ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) d = __dp4a((int)xs[i], (int)ww[i], d);
  } else {
    const uint4 wq = *reinterpret_cast<const uint4*>(w.data + tr * 32 + (b & 1) * 16);
    const uint32_t wv[4] = {wq.x, wq.y, wq.z, wq.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t n0, n1;
      nib_x16(wv[i], n0, n1);
      d = __dp4a((int)xs[2 * i], (int)n0, d);
      d = __dp4a((int)xs[2 * i + 1], (int)n1, d);
    }
    d /= 16;   // exact: every product carried the factor 16
  }
  return d;
}

__device__ __forceinline__ uint32_t weight_scale(const WeightView& w, int r, int b) {
  return w.scales[tiled_row(r, b >> 1, w.Kpad / kTileK) * 2 + (b & 1)];
}

__device__ __forceinline__ float butterfly_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// sum_b 2^e_w,b * (2^e_x,b * dot_b) in the lane order described above
__device__ __forceinline__ float row_dot(const WeightView& w, int r, const uint8_t* xq, const uint8_t* xs,
                                         int lane) {
  const int nb = w.K / kBlock;
  float acc = 0.0f;
  for (int b = lane; b < nb; b += 32) {
    const int d = block_dot(w, r, b, xq + (size_t)b * kBlock);
    const float t = __fmul_rn(__fmul_rn((float)d, e8m0_to_float(xs[b])), e8m0_to_float(weight_scale(w, r, b)));
    acc = __fadd_rn(acc, t);
  }
  return butterfly_sum(acc);
}

// ------------------------------------------------------- mx_quantize_w ---
// One warp per (row, 32-element block), lane = element: block max, the E8M0
// exponent for QMAX (127 int8 / 7 int4), round-half-to-even, clamp to
// [-QMAX, QMAX]; a block holding a NaN/inf gets scale 0xFF and zeros.
template <int QMAX>
__global__ void __launch_bounds__(256) quantize_w_kernel(const float* __restrict__ w, int N, int K,
                                                         uint8_t* __restrict__ data, uint8_t* __restrict__ scales,
                                                         int32_t* __restrict__ wsums) {
  const int lane = threadIdx.x & 31;
  const long warp = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long nwarps = ((long)gridDim.x * blockDim.x) >> 5;
  const int nb = K / kBlock;
  for (long blk = warp; blk < (long)N * nb; blk += nwarps) {
    const long n = blk / nb;
    const int b = (int)(blk % nb);
    const float v = w[n * K + (long)b * kBlock + lane];
    const float av = fabsf(v);
    const bool nonfinite = !(av <= 3.402823466e38f);
    const bool any_nf = __any_sync(0xffffffffu, nonfinite);
    const float m = warp_max(nonfinite ? 0.0f : av, 32);
    int q = 0;
    uint32_t sb;
    if (any_nf) {
      sb = 255;
    } else if (m == 0.0f) {
      sb = 0;
    } else {
      const int e = e8m0_exponent<QMAX>(m);
      sb = (uint32_t)(e + 127);
      q = quant_value(v, e);
      q = q > QMAX ? QMAX : (q < -QMAX ? -QMAX : q);
    }
    if (QMAX == 127) {
      data[n * K + (long)b * kBlock + lane] = (uint8_t)(int8_t)q;
    } else {
      const int hi = __shfl_down_sync(0xffffffffu, q, 1);
      if ((lane & 1) == 0)
        data[n * (K / 2) + ((long)b * kBlock + lane) / 2] = (uint8_t)((q & 0xF) | ((hi & 0xF) << 4));
    }
    int s = q;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) {
      scales[n * nb + b] = (uint8_t)sb;
      if (wsums) wsums[n * nb + b] = s;
    }
  }
}

// -------------------------------------------------------- halting_step ---
// ACT halting (Graves 2016) on a 1-row MX weight: p = sigmoid(w . x + b);
// steps += 1; if p_sum + p >= 1 - eps the token halts, remainder = 1 - p_sum
// and p_sum becomes 1; otherwise p_sum += p.  One warp per token.
__global__ void halting_kernel(WeightView w, const uint8_t* __restrict__ xq, const uint8_t* __restrict__ xs,
                               int B, float bias, float eps, mxq_halting_state* __restrict__ st,
                               float* __restrict__ p_out, uint8_t* __restrict__ halt_out) {
  const int lane = threadIdx.x & 31;
  const int t = (int)(((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  if (t >= B) return;
  const float z = __fadd_rn(row_dot(w, 0, xq + (size_t)t * w.K, xs + (size_t)t * (w.K / kBlock), lane), bias);
  if (lane != 0) return;
  const float p = __fdiv_rn(1.0f, __fadd_rn(1.0f, det_expf(-z)));
  mxq_halting_state s = st[t];
  s.steps += 1;
  const bool halt = __fadd_rn(s.p_sum, p) >= __fsub_rn(1.0f, eps);
  if (halt) {
    s.remainder = __fsub_rn(1.0f, s.p_sum);
    s.p_sum = 1.0f;
  } else {
    s.p_sum = __fadd_rn(s.p_sum, p);
  }
  st[t] = s;
  p_out[t] = p;
  halt_out[t] = halt ? 1 : 0;
}

// -------------------------------------------------- rank16_dot_ptrs ---
// Row 0 of each weight: its tiled data and scales (the tile padding of K is
// the same for every row, so only the pointers differ).
struct RowPtrs {
  const uint8_t* data[kRowPtrsMax];
  const uint8_t* scales[kRowPtrsMax];
};

// y[t][j] = row 0 of weight j dotted with activation t; one warp per (t, j).
__global__ void row_ptrs_kernel(RowPtrs rp, int nrows, int fmt, int K, int Kpad, const uint8_t* __restrict__ xq,
                                const uint8_t* __restrict__ xs, int B, float* __restrict__ y) {
  const int lane = threadIdx.x & 31;
  const long wid = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (wid >= (long)B * nrows) return;
  const int t = (int)(wid / nrows), j = (int)(wid % nrows);
  WeightView w{};
  w.fmt = fmt;
  w.K = K;
  w.Kpad = Kpad;
  w.data = rp.data[j];
  w.scales = rp.scales[j];
  const float v = row_dot(w, 0, xq + (size_t)t * K, xs + (size_t)t * (K / kBlock), lane);
  if (lane == 0) y[(size_t)t * nrows + j] = v;
}

// ---------------------------------------------------- hashed router ---
// splitmix64 finaliser: the hyperplanes and the expert codes are generated
// from it, so the router stores no weights.
__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Hyperplane h's sign at element i: bit (i % 64) of mix64(seed, h, i / 64).
__device__ __forceinline__ int plane_sign(uint64_t seed, int h, int i) {
  const uint64_t r = mix64(seed ^ ((uint64_t)(h + 1) << 40) ^ (uint64_t)(i >> 6));
  return ((r >> (i & 63)) & 1ull) ? 1 : -1;
}

// One warp per token.  Per 32-element block (lane = element): quantise as
// mx_quantize_x does (exact bytes), then for every hyperplane the block's
// exact int dot with the +-1 signs (a warp sum), scaled by 2^e_x; lane h keeps
// hyperplane h's projection, added in block order.  Code bit h = projection
// h > 0.  Expert e's code is mix64(seed ^ 0xC0DEC0DE ^ (e << 20)) masked to
// H bits;
// score = H - popcount(code(x) ^ code_e); top-K by descending score, ties to
// the lower expert id.
__global__ void hashed_route_kernel(const float* __restrict__ x, int T, int D, int E, int K, int H,
                                    uint64_t seed, int32_t* __restrict__ idx, int32_t* __restrict__ score) {
  const int lane = threadIdx.x & 31;
  const int t = (int)(((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  if (t >= T) return;
  float proj = 0.0f;                 // lane h < H: hyperplane h
  const int nb = D / kBlock;
  for (int b = 0; b < nb; ++b) {
    const float v = x[(size_t)t * D + (size_t)b * kBlock + lane];
    const float av = fabsf(v);
    const bool nonfinite = !(av <= 3.402823466e38f);
    const bool any_nf = __any_sync(0xffffffffu, nonfinite);
    const float m = warp_max(nonfinite ? 0.0f : av, 32);
    if (any_nf || m == 0.0f) continue;    // a zero block adds nothing; a non-finite one is skipped
    const int e = e8m0_exponent<127>(m);
    const int q = quant_value(v, e);
    const float sx = pow2_exact(e);
    for (int h = 0; h < H; ++h) {
      const int d = __reduce_add_sync(0xffffffffu, q * plane_sign(seed, h, b * kBlock + lane));
      if (lane == h) proj = __fadd_rn(proj, __fmul_rn((float)d, sx));
    }
  }
  const uint32_t bit = (lane < H && proj > 0.0f) ? 1u : 0u;
  const uint32_t code = __ballot_sync(0xffffffffu, bit);
  if (lane != 0) return;
  const uint32_t mask = H == 32 ? 0xffffffffu : ((1u << H) - 1u);
  // top-K: repeated selection over the experts (K <= 64)
  int32_t chosen[64];
  for (int j = 0; j < K; ++j) {
    int best = -1, bs = -1;
    for (int ex = 0; ex < E; ++ex) {
      bool used = false;
      for (int p = 0; p < j; ++p) used |= chosen[p] == ex;
      if (used) continue;
      const uint32_t ce = (uint32_t)mix64(seed ^ 0xC0DEC0DEull ^ ((uint64_t)ex << 20)) & mask;
      const int s = H - __popc((code ^ ce) & mask);
      if (s > bs) {
        bs = s;
        best = ex;
      }
    }
    chosen[j] = best;
    idx[(size_t)t * K + j] = best;
    score[(size_t)t * K + j] = bs;
  }
}

// ------------------------------------------------ Gaussian moment update ---
// One thread per 16-byte piece of the tiled weight: every element w (int8,
// or an int4 nibble) of row n, column k becomes
//   clamp(rint(w + ((step * g[n]) * x[k]) * 2^-e), -QMAX, QMAX)
// with e the element's E8M0 block exponent (kept), QMAX 127 (int8) or 8 / 7
// (int4: [-8, 7]).  Padding rows and columns stay zero; a NaN-scale block
// (0xFF) is left as it is.
template <int WFMT>
__global__ void moment_update_kernel(WeightView w, const float* __restrict__ g, const float* __restrict__ x,
                                     float step, uint8_t* __restrict__ data) {
  constexpr int TB = WFMT == 4 ? 32 : 64;
  const int KT = w.Kpad / kTileK;
  const long pieces = (long)(w.Npad / 128) * KT * 128 * (TB / 16);
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < pieces; i += (long)gridDim.x * blockDim.x) {
    const int p = (int)(i % (TB / 16));
    const long tr = i / (TB / 16);                 // tiled row index ((rt * KT + kt) * 128 + row)
    const int row = (int)(tr % 128), kt = (int)((tr / 128) % KT), rt = (int)(tr / (128L * KT));
    const int n = rt * 128 + row;
    if (n >= w.N) continue;
    uint4 v = *reinterpret_cast<const uint4*>(data + tr * TB + p * 16);
    uint8_t* b = reinterpret_cast<uint8_t*>(&v);
    const float gn = __fmul_rn(step, g[n]);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int k0 = kt * kTileK + (WFMT == 4 ? (p * 16 + j) * 2 : p * 16 + j);
#pragma unroll
      for (int h = 0; h < (WFMT == 4 ? 2 : 1); ++h) {
        const int k = k0 + h;
        if (k >= w.K) continue;
        const uint32_t s = w.scales[tr * 2 + ((k % kTileK) >> 5)];
        if (s == 255u) continue;
        const int old = WFMT == 4 ? (((int)(b[j] >> (4 * h)) & 0xF) ^ 8) - 8 : (int)(int8_t)b[j];
        const float delta = __fmul_rn(__fmul_rn(gn, x[k]), pow2_exact(127 - (int)s));
        int q = __float2int_rn(__fadd_rn((float)old, delta));
        const int lo = WFMT == 4 ? -8 : -127, hi = WFMT == 4 ? 7 : 127;
        q = q < lo ? lo : (q > hi ? hi : q);
        if (WFMT == 4) b[j] = (uint8_t)((b[j] & (h ? 0x0F : 0xF0)) | ((q & 0xF) << (4 * h)));
        else b[j] = (uint8_t)(int8_t)q;
      }
    }
    *reinterpret_cast<uint4*>(data + tr * TB + p * 16) = v;
  }
}

// ------------------------------------------------ activation norm ---
// ||x||_2 of an MX activation row: per block the exact int sum of q^2,
// times 2^(2 e) in fp32, summed in the lanes-then-butterfly order.
__global__ void act_norm_kernel(const uint8_t* __restrict__ xq, const uint8_t* __restrict__ xs, int B, int K,
                                float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int t = (int)(((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  if (t >= B) return;
  const int nb = K / kBlock;
  float acc = 0.0f;
  for (int b = lane; b < nb; b += 32) {
    const uint8_t* q = xq + (size_t)t * K + (size_t)b * kBlock;
    int ss = 0;
#pragma unroll 8
    for (int i = 0; i < kBlock; ++i) {
      const int v = (int)q[i] - 128;
      ss += v * v;
    }
    const float sc = e8m0_to_float(xs[(size_t)t * nb + b]);
    acc = __fadd_rn(acc, __fmul_rn(__fmul_rn((float)ss, sc), sc));
  }
  acc = butterfly_sum(acc);
  if (lane == 0) out[t] = __fsqrt_rn(acc);
}

// ------------------------------------------------ micro-expert layer ---
// The reference's expert pool (1024 micro-experts of 16 rows, top-16 routed
// plus 2 shared, nn/config/model_config.hpp:23-25; 16-row slices of the
// gate/up matrices, training/fidelity_test.cpp:57-59).  Expert e owns rows
// 16e .. 16e+15 of the gate and up pools [(E_r + E_s) * 16][D] and columns
// 16e .. 16e+15 of the down pool [D][(E_r + E_s) * 16]; shared experts are
// e = E_r .. E_r + E_s - 1.  Per token (one CTA of 256 threads):
//   x -> MX (quantize_kernel's arithmetic) in shared memory;
//   the 16 gate and 16 up rows of each chosen expert: row dots in the fixed
//   lane order (one warp per row);
//   h = det_swiglu(g, u) * gate weight (1 for shared experts), placed in the
//   32-element blocks of the down pool's K (expert e's 16 values are half of
//   block e / 2; a block's other half is 0 unless its expert is chosen too),
//   each block MX-quantised;
//   y[j] = sum over the chosen blocks in ascending order of
//   (dot * 2^e_h) * 2^e_w, fp32.
constexpr int kMicroMaxSel = 64 + 8;   // routed k <= 64, shared <= 8

__global__ void __launch_bounds__(256) micro_moe_kernel(WeightView wg, WeightView wu, WeightView wd, int n_routed,
                                                        int n_shared, const float* __restrict__ x,
                                                        const int32_t* __restrict__ idx,
                                                        const float* __restrict__ gate, int k,
                                                        float* __restrict__ y) {
  extern __shared__ __align__(16) uint8_t sm[];
  const int D = wg.K, t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nsel = k + n_shared;
  uint8_t* xq = sm;                                     // [D] u8
  uint8_t* xs = xq + D;                                 // [D/32]
  float* hv = reinterpret_cast<float*>(sm + ((D + D / 32 + 15) / 16) * 16);   // [nsel][32]: g then u
  int* sel = reinterpret_cast<int*>(hv + nsel * 32);    // [nsel] expert ids
  float* wsel = reinterpret_cast<float*>(sel + nsel);   // [nsel] weights
  int* blk = reinterpret_cast<int*>(wsel + nsel);       // [nsel] distinct blocks, ascending
  int* nblk = blk + nsel;
  uint8_t* hq = reinterpret_cast<uint8_t*>(nblk + 4);   // [nsel][32] (16-byte aligned below)
  hq = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(hq) + 15) & ~(uintptr_t)15);
  uint8_t* hs = hq + nsel * 32;                         // [nsel]
  // 1. the token's x to MX bytes
  for (int b = warp; b < D / kBlock; b += 8) {
    const float v = x[(size_t)t * D + b * kBlock + lane];
    const float av = fabsf(v);
    const bool nonfinite = !(av <= 3.402823466e38f);
    const bool any_nf = __any_sync(0xffffffffu, nonfinite);
    const float m = warp_max(nonfinite ? 0.0f : av, 32);
    int q = 0;
    uint32_t sb = 0;
    if (any_nf) sb = 255;
    else if (m != 0.0f) {
      const int e = e8m0_exponent<127>(m);
      sb = (uint32_t)(e + 127);
      q = quant_value(v, e);
    }
    xq[b * kBlock + lane] = (uint8_t)(q + 128);
    if (lane == 0) xs[b] = (uint8_t)sb;
  }
  if (tid < nsel) {
    int e = tid < k ? idx[(size_t)t * k + tid] : n_routed + (tid - k);
    if (tid < k) e = e < 0 ? 0 : (e >= n_routed ? n_routed - 1 : e);   // ids outside the pool: clamped
    sel[tid] = e;
    wsel[tid] = tid < k ? (gate ? gate[(size_t)t * k + tid] : 1.0f) : 1.0f;
  }
  __syncthreads();
  // 2. gate and up rows of the chosen experts, one warp per row
  for (int r = warp; r < nsel * 32; r += 8) {
    const int s = r >> 5, j = r & 31;                   // j < 16: gate row j, else up row j - 16
    const int row = sel[s] * 16 + (j & 15);
    const float v = row_dot(j < 16 ? wg : wu, row, xq, xs, lane);
    if (lane == 0) hv[s * 32 + j] = v;
  }
  // the distinct down blocks, ascending (one thread; at most nsel entries)
  if (tid == 0) {
    int n = 0;
    for (int s2 = 0; s2 < nsel; ++s2) {
      const int b = sel[s2] >> 1;
      int pos = 0;
      while (pos < n && blk[pos] < b) ++pos;
      if (pos < n && blk[pos] == b) continue;
      for (int q2 = n; q2 > pos; --q2) blk[q2] = blk[q2 - 1];
      blk[pos] = b;
      ++n;
    }
    *nblk = n;
  }
  __syncthreads();
  // 3. h per block (one warp per block, lane = element) -> MX
  const int nb = *nblk;
  for (int i = warp; i < nb; i += 8) {
    const int e = blk[i] * 2 + (lane >> 4), slot = lane & 15;
    float v = 0.0f;
    for (int s2 = 0; s2 < nsel; ++s2)
      if (sel[s2] == e) v = __fmul_rn(det_swiglu(hv[s2 * 32 + slot], hv[s2 * 32 + 16 + slot]), wsel[s2]);
    const float av = fabsf(v);
    const bool nonfinite = !(av <= 3.402823466e38f);
    const bool any_nf = __any_sync(0xffffffffu, nonfinite);
    const float m = warp_max(nonfinite ? 0.0f : av, 32);
    int q = 0;
    uint32_t sb = 0;
    if (any_nf) sb = 255;
    else if (m != 0.0f) {
      const int ee = e8m0_exponent<127>(m);
      sb = (uint32_t)(ee + 127);
      q = quant_value(v, ee);
    }
    hq[i * 32 + lane] = (uint8_t)(q + 128);
    if (lane == 0) hs[i] = (uint8_t)sb;
  }
  __syncthreads();
  // 4. down: one thread per output row, the chosen blocks in ascending order
  for (int j = tid; j < wd.N; j += 256) {
    float acc = 0.0f;
    for (int i = 0; i < nb; ++i) {
      const int d = block_dot(wd, j, blk[i], hq + i * 32);
      acc = __fadd_rn(acc, __fmul_rn(__fmul_rn((float)d, e8m0_to_float(hs[i])),
                                     e8m0_to_float(weight_scale(wd, j, blk[i]))));
    }
    y[(size_t)t * wd.N + j] = acc;
  }
}

}  // namespace

size_t micro_moe_smem(int D, int nsel) {
  return (size_t)((D + D / 32 + 15) / 16) * 16 + (size_t)nsel * 32 * 4 + (size_t)nsel * 4 * 3 + 16 + 16 +
         (size_t)nsel * 33 + 16;
}

cudaError_t launch_micro_moe(const WeightView& wg, const WeightView& wu, const WeightView& wd, int n_routed,
                             int n_shared, const float* x, const int32_t* idx, const float* gate, int T, int k,
                             float* y, cudaStream_t st) {
  if (k + n_shared > kMicroMaxSel) return cudaErrorInvalidValue;
  const size_t smem = micro_moe_smem(wg.K, k + n_shared);
  static SmemAttr smem_attr;
  if (cudaError_t e = smem_attr.ensure(micro_moe_kernel, smem)) return e;
  micro_moe_kernel<<<(unsigned)T, 256, smem, st>>>(wg, wu, wd, n_routed, n_shared, x, idx, gate, k, y);
  return cudaGetLastError();
}

cudaError_t launch_moment_update(const WeightView& w, const float* g, const float* x, float step, uint8_t* data,
                                 cudaStream_t st) {
  const long pieces = (long)(w.Npad / 128) * (w.Kpad / kTileK) * 128 * ((w.fmt == 4 ? 32 : 64) / 16);
  long ctas = (pieces + 255) / 256;
  if (ctas > 148L * 16) ctas = 148L * 16;
  if (w.fmt == 4) moment_update_kernel<4><<<(unsigned)ctas, 256, 0, st>>>(w, g, x, step, data);
  else moment_update_kernel<8><<<(unsigned)ctas, 256, 0, st>>>(w, g, x, step, data);
  return cudaGetLastError();
}

cudaError_t launch_act_norm(const uint8_t* xq, const uint8_t* xs, int B, int K, float* out, cudaStream_t st) {
  const long threads = (long)B * 32;
  act_norm_kernel<<<(unsigned)((threads + 127) / 128), 128, 0, st>>>(xq, xs, B, K, out);
  return cudaGetLastError();
}

cudaError_t launch_quantize_w(int fmt, const float* w, int N, int K, uint8_t* data, uint8_t* scales,
                              int32_t* wsums, cudaStream_t st) {
  const long blocks = (long)N * (K / kBlock);
  long ctas = (blocks + 7) / 8;
  if (ctas > 148L * 16) ctas = 148L * 16;
  if (ctas < 1) ctas = 1;
  if (fmt == 8) quantize_w_kernel<127><<<(unsigned)ctas, 256, 0, st>>>(w, N, K, data, scales, wsums);
  else quantize_w_kernel<7><<<(unsigned)ctas, 256, 0, st>>>(w, N, K, data, scales, wsums);
  return cudaGetLastError();
}

cudaError_t launch_halting(const WeightView& w, const uint8_t* xq, const uint8_t* xs, int B, float bias,
                           float eps, mxq_halting_state* st, float* p, uint8_t* halt, cudaStream_t s) {
  const long threads = (long)B * 32;
  halting_kernel<<<(unsigned)((threads + 127) / 128), 128, 0, s>>>(w, xq, xs, B, bias, eps, st, p, halt);
  return cudaGetLastError();
}

cudaError_t launch_row_ptrs(const WeightView* const* ws, int nrows, const uint8_t* xq, const uint8_t* xs, int B,
                            float* y, cudaStream_t s) {
  if (nrows <= 0 || nrows > kRowPtrsMax) return cudaErrorInvalidValue;
  RowPtrs rp{};
  for (int j = 0; j < nrows; ++j) {
    rp.data[j] = ws[j]->data;
    rp.scales[j] = ws[j]->scales;
  }
  const long threads = (long)B * nrows * 32;
  row_ptrs_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(rp, nrows, ws[0]->fmt, ws[0]->K, ws[0]->Kpad,
                                                                   xq, xs, B, y);
  return cudaGetLastError();
}

cudaError_t launch_hashed_route(const float* x, int T, int D, int E, int K, int H, uint64_t seed, int32_t* idx,
                                int32_t* score, cudaStream_t s) {
  const long threads = (long)T * 32;
  hashed_route_kernel<<<(unsigned)((threads + 127) / 128), 128, 0, s>>>(x, T, D, E, K, H, seed, idx, score);
  return cudaGetLastError();
}

}  // namespace mxq
