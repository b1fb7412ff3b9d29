// mxq_moe.cu -- block-sparse mixture-of-experts plumbing around the
// tensor-core GEMM: route bookkeeping and the weighted combine.
//
// The reference's MoE runs gathered expert rows (mx_rank16_dot_ptrs,
// nn/tests/test_auto_generated.cpp:55, 16-row micro-experts sliced at
// training/fidelity_test.cpp:57-59); the layer built here is the top-k SwiGLU
// expert layer with 64x64 block-sparse expert matrices.  Every step is
// deterministic: slots are assigned in token order, the combine sums a
// token's k expert outputs in routing order.
#include "mxq_internal.h"

namespace mxq {

namespace {

constexpr int kAssignThreads = 256;

// Block-wide exclusive prefix sum of 0/1 flags (deterministic).
__device__ __forceinline__ int block_excl_scan(int flag, int* warp_sums, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned m = __ballot_sync(0xffffffffu, flag);
  const int within = __popc(m & ((1u << lane) - 1u));
  if (lane == 0) warp_sums[warp] = __popc(m);
  __syncthreads();
  int before = 0, all = 0;
  for (int w = 0; w < kAssignThreads / 32; ++w) {
    const int v = warp_sums[w];
    if (w < warp) before += v;
    all += v;
  }
  __syncthreads();
  *total = all;
  return before + within;
}

// One CTA per expert: how many routes chose it.
__global__ void __launch_bounds__(kAssignThreads) moe_count_kernel(const int32_t* __restrict__ idx,
                                                                  int routes, int32_t* __restrict__ counts) {
  __shared__ int warp_sums[kAssignThreads / 32];
  const int e = blockIdx.x;
  int n = 0;
  for (int base = 0; base < routes; base += kAssignThreads) {
    const int r = base + threadIdx.x;
    const int flag = r < routes && idx[r] == e;
    int total;
    block_excl_scan(flag, warp_sums, &total);
    n += total;
  }
  if (threadIdx.x == 0) counts[e] = n;
}

// One CTA per expert: slots of expert e start at offset(e) = sum of the
// earlier experts' counts and follow token order.  slot_token[pos] = token
// row to gather; route_pos[r] = slot position of route r.
__global__ void __launch_bounds__(kAssignThreads) moe_assign_kernel(const int32_t* __restrict__ idx,
                                                                   int routes, int k,
                                                                   const int32_t* __restrict__ counts,
                                                                   int32_t* __restrict__ offsets,
                                                                   int32_t* __restrict__ slot_token,
                                                                   int32_t* __restrict__ route_pos) {
  __shared__ int warp_sums[kAssignThreads / 32];
  const int e = blockIdx.x;
  int off = 0;
  for (int j = 0; j < e; ++j) off += counts[j];
  if (threadIdx.x == 0) {
    offsets[e] = off;
    if (e == (int)gridDim.x - 1) offsets[e + 1] = off + counts[e];
  }
  int n = 0;
  for (int base = 0; base < routes; base += kAssignThreads) {
    const int r = base + threadIdx.x;
    const int flag = r < routes && idx[r] == e;
    int total;
    const int before = block_excl_scan(flag, warp_sums, &total);
    if (flag) {
      const int p = off + n + before;
      slot_token[p] = r / k;
      route_pos[r] = p;
    }
    n += total;
  }
}

// y[t][d] = sum_j gate[t][j] * yr[route_pos[t*k+j]][d], j in routing order.
__global__ void moe_combine_kernel(const float* __restrict__ yr, const float* __restrict__ gate,
                                   const int32_t* __restrict__ route_pos, int T, int D, int k,
                                   float* __restrict__ y) {
  const long total = (long)T * D;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int t = (int)(i / D), d = (int)(i % D);
    float acc = 0.0f;
    for (int j = 0; j < k; ++j) {
      const int r = t * k + j;
      acc = __fmaf_rn(gate[r], yr[(long)route_pos[r] * D + d], acc);
    }
    y[i] = acc;
  }
}

}  // namespace

cudaError_t launch_moe_assign(const int32_t* idx, int T, int k, int E, int32_t* counts,
                              int32_t* offsets, int32_t* slot_token, int32_t* route_pos,
                              cudaStream_t st) {
  moe_count_kernel<<<E, kAssignThreads, 0, st>>>(idx, T * k, counts);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  moe_assign_kernel<<<E, kAssignThreads, 0, st>>>(idx, T * k, k, counts, offsets, slot_token, route_pos);
  return cudaGetLastError();
}

cudaError_t launch_moe_combine(const float* yr, const float* gate, const int32_t* route_pos, int T,
                               int D, int k, float* y, cudaStream_t st) {
  long ctas = ((long)T * D + 255) / 256;
  if (ctas > 148L * 16) ctas = 148L * 16;
  if (ctas < 1) ctas = 1;
  moe_combine_kernel<<<(unsigned)ctas, 256, 0, st>>>(yr, gate, route_pos, T, D, k, y);
  return cudaGetLastError();
}

}  // namespace mxq
