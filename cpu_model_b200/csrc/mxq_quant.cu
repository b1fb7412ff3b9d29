// mxq_quant.cu -- activation quantisers (mx_quantize_x,
// mx_fused_silu_quantize_x, fused_gated_silu_quantize; reference residue
// nn/core/layers/ssm.cpp:164-177 and :234-260) and the conversion of an MX
// activation into the tensor-core operand of the GEMM path.
//
// One warp owns one 32-element block at a time (lane = element): a coalesced
// 128-byte load, a 5-step shuffle max, the E8M0 exponent from the max's
// bits, and round-half-to-even quantisation -- the same float operations as
// the CPU oracle, so bytes agree exactly.
//
// The GEMM operand is bf16 q * 2^e (exact: |q| <= 127 needs 7 significand
// bits), laid out as [token tile][k tile][BN rows x 128 B] with the 128-byte
// swizzle already applied, so the GEMM moves each tile with one 1-D bulk
// copy.  For int4 weights the eight K slots of each 16-byte chunk hold
// elements {0,2,4,6,1,3,5,7}: the order in which the GEMM's int4 unpack
// produces weights (the dot product is invariant to a shared permutation).
#include "mxq_internal.h"

namespace mxq {

// in-group position -> slot, for the int4 operand order
__device__ __forceinline__ int int4_slot(int j) { return (j >> 1) + ((j & 1) << 2); }

// q * 2^(s - 127 + shift) for the bf16 GEMM operand (exact when in range;
// NaN for scale 0xFF; a zero q stays zero whatever the exponent).
__device__ __forceinline__ float operand_value(int q, uint32_t s, int shift) {
  if (s == 255u) return __int_as_float(0x7fc00000);
  if (q == 0) return 0.0f;
  const int n = (int)s - 127 + shift;
  if (n > 127) return q > 0 ? __int_as_float(0x7f800000) : __int_as_float(0xff800000);
  return __fmul_rn((float)q, pow2_exact(n));
}

__device__ __forceinline__ int nf_zero(int q, uint32_t sb) { return sb == 255u ? 0 : q; }

template <int MODE>
__global__ void __launch_bounds__(256) quantize_kernel(QuantArgs a) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // Dependents may launch now: the kernels that follow (GEMVs, the GEMM)
  // stream their weights before their own griddepcontrol.wait and read this
  // kernel's output only after it, which waits for this grid to complete.
  // Everything before this kernel is complete once its own wait returns.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int lane = threadIdx.x & 31;
  const long warp = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long nwarps = ((long)gridDim.x * blockDim.x) >> 5;
  const int kb = a.K / kBlock;
  const int rows = a.opnd ? a.Bpad : a.B;
  const int kbp = a.opnd ? a.Kpad / kBlock : kb;
  const long total = (long)rows * kbp;
  for (long blk = warp; blk < total; blk += nwarps) {
    const int t = (int)(blk / kbp);
    const int b = (int)(blk % kbp);
    const bool valid = t < a.B && b < kb;  // warp-uniform
    int q = 0;
    uint32_t sb = 0;
    if (valid) {
      const long idx = (long)t * a.K + (long)b * kBlock + lane;
      if (MODE == 3) {
        q = (int)a.in_q[idx] - 128;
        sb = a.in_s[(long)t * kb + b];
      } else {
        float v;
        if (MODE == 0) v = a.x[a.gather ? (long)a.gather[t] * a.K + (long)b * kBlock + lane : idx];
        else if (MODE == 1) v = det_silu(a.x[idx]);
        else v = det_swiglu(a.x[idx], a.up[idx]);
        const float av = fabsf(v);
        const bool nonfinite = !(av <= 3.402823466e38f);
        const bool any_nf = __any_sync(0xffffffffu, nonfinite);
        const float m = warp_max(nonfinite ? 0.0f : av, 32);
        if (any_nf) {
          sb = 255;
          q = 0;
        } else if (m == 0.0f) {
          sb = 0;
          q = 0;
        } else {
          const int e = e8m0_exponent<127>(m);
          sb = (uint32_t)(e + 127);
          q = quant_value(v, e);
        }
      }
      if (a.out_q) a.out_q[idx] = (uint8_t)(q + 128);
      if (a.out_s && lane == 0) a.out_s[(long)t * kb + b] = (uint8_t)sb;
    }
    if (a.opnd) {
      const float f = valid ? operand_value(q, sb, a.shift) : 0.0f;
      const int k = b * kBlock + lane;
      const int kt = k / kTileK;
      const int kin = k % kTileK;
      const int chunk = kin >> 3;
      const int slot = a.int4_order ? int4_slot(kin & 7) : (kin & 7);
      const long tile = (long)(t / a.BN) * (a.Kpad / kTileK) + kt;
      const long off = tile * (long)a.BN * 128 + sw128_offset(t % a.BN, chunk) + slot * 2;
      *reinterpret_cast<__nv_bfloat16*>(reinterpret_cast<uint8_t*>(a.opnd) + off) =
          __float2bfloat16_rn(f);
    }
  }
}

// Operand-only form (no MX bytes requested): one thread per 16-byte output
// chunk (8 consecutive K of one token row), 4 threads per 32-element block
// (block max over 2 shuffle steps), each chunk written whole -- 8 lanes fill
// a 128-byte row of a swizzled tile.  Same arithmetic as quantize_kernel, so
// the operand bytes are identical.
template <int MODE>
__global__ void __launch_bounds__(256) operand_kernel(QuantArgs a) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // Dependents may launch now: the kernels that follow (GEMVs, the GEMM)
  // stream their weights before their own griddepcontrol.wait and read this
  // kernel's output only after it, which waits for this grid to complete.
  // Everything before this kernel is complete once its own wait returns.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int kb = a.K / kBlock;
  const long cpr = a.Kpad / 8;                          // chunks per token row
  const long total = (long)a.Bpad * cpr;                // multiple of 4 (Kpad % 64 == 0)
  for (long base = (long)blockIdx.x * blockDim.x; base < total; base += (long)gridDim.x * blockDim.x) {
    const long gidx = base + threadIdx.x;               // whole warps iterate together
    const bool in = gidx < total;
    const int t = in ? (int)(gidx / cpr) : 0;
    const int kc = in ? (int)(gidx % cpr) : 0;
    const int k0 = kc * 8, b = k0 / kBlock;
    const bool valid = in && t < a.B && b < kb;         // uniform over the block's 4 lanes
    float v[8];
    int qv[8];
    uint32_t sb = 0;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      v[e] = 0.0f;
      qv[e] = 0;
    }
    if (valid) {
      const long idx = (long)t * a.K + k0;
      if (MODE == 3) {
        const uint2 qq = *reinterpret_cast<const uint2*>(a.in_q + idx);
        const uint32_t w2[2] = {qq.x, qq.y};
#pragma unroll
        for (int e = 0; e < 8; ++e) qv[e] = (int)((w2[e >> 2] >> (8 * (e & 3))) & 0xFFu) - 128;
        sb = a.in_s[(long)t * kb + b];
      } else {
        const float* src = MODE == 0 && a.gather ? a.x + (long)a.gather[t] * a.K + k0 : a.x + idx;
        const float4 x0 = *reinterpret_cast<const float4*>(src);
        const float4 x1 = *reinterpret_cast<const float4*>(src + 4);
        v[0] = x0.x; v[1] = x0.y; v[2] = x0.z; v[3] = x0.w;
        v[4] = x1.x; v[5] = x1.y; v[6] = x1.z; v[7] = x1.w;
        if (MODE == 1) {
#pragma unroll
          for (int e = 0; e < 8; ++e) v[e] = det_silu(v[e]);
        } else if (MODE == 2) {
          const float4 u0 = *reinterpret_cast<const float4*>(a.up + idx);
          const float4 u1 = *reinterpret_cast<const float4*>(a.up + idx + 4);
          const float u[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
          for (int e = 0; e < 8; ++e) v[e] = det_swiglu(v[e], u[e]);
        }
      }
    }
    if (MODE != 3) {
      float m = 0.0f;
      bool nf = false;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float av = fabsf(v[e]);
        const bool bad = !(av <= 3.402823466e38f);
        nf |= bad;
        m = fmaxf(m, bad ? 0.0f : av);
      }
#pragma unroll
      for (int o = 1; o < 4; o <<= 1) {
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        nf |= __shfl_xor_sync(0xffffffffu, (int)nf, o) != 0;
      }
      if (valid) {
        if (nf) {
          sb = 255;
        } else if (m != 0.0f) {
          const int e = e8m0_exponent<127>(m);
          sb = (uint32_t)(e + 127);
#pragma unroll
          for (int q = 0; q < 8; ++q) qv[q] = quant_value(v[q], e);
        }
      }
    }
    if (in) {
      __nv_bfloat16 o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float f = valid ? operand_value(nf_zero(qv[e], sb), sb, a.shift) : 0.0f;
        const int slot = a.int4_order ? int4_slot(e) : e;
        o[slot] = __float2bfloat16_rn(f);
      }
      const int kt = k0 / kTileK, chunk = (k0 % kTileK) >> 3;
      const long tile = (long)(t / a.BN) * (a.Kpad / kTileK) + kt;
      const long off = tile * (long)a.BN * 128 + sw128_offset(t % a.BN, chunk);
      *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(a.opnd) + off) = *reinterpret_cast<const uint4*>(o);
    }
  }
}

cudaError_t launch_quantize(const QuantArgs& a, int mode, cudaStream_t st,
                            bool pdl) {
  const int rows = a.opnd ? a.Bpad : a.B;
  const int kbp = a.opnd ? a.Kpad / kBlock : a.K / kBlock;
  const long blocks = (long)rows * kbp;
  long ctas = (blocks + 7) / 8;
  if (ctas > 148L * 16) ctas = 148L * 16;
  if (ctas < 1) ctas = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ctas);
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  const bool x16 = (reinterpret_cast<uintptr_t>(a.x) & 15u) == 0 && (reinterpret_cast<uintptr_t>(a.up) & 15u) == 0 &&
                   (reinterpret_cast<uintptr_t>(a.in_q) & 7u) == 0;
  if (a.opnd && !a.out_q && !a.out_s && x16) {
    const long chunks = (long)a.Bpad * (a.Kpad / 8);
    long octas = (chunks + 255) / 256;
    if (octas > 148L * 8) octas = 148L * 8;
    if (octas < 1) octas = 1;
    cfg.gridDim = dim3((unsigned)octas);
    switch (mode) {
      case 0: return cudaLaunchKernelEx(&cfg, operand_kernel<0>, a);
      case 1: return cudaLaunchKernelEx(&cfg, operand_kernel<1>, a);
      case 2: return cudaLaunchKernelEx(&cfg, operand_kernel<2>, a);
      case 3: return cudaLaunchKernelEx(&cfg, operand_kernel<3>, a);
    }
    return cudaErrorInvalidValue;
  }
  switch (mode) {
    case 0: return cudaLaunchKernelEx(&cfg, quantize_kernel<0>, a);
    case 1: return cudaLaunchKernelEx(&cfg, quantize_kernel<1>, a);
    case 2: return cudaLaunchKernelEx(&cfg, quantize_kernel<2>, a);
    case 3: return cudaLaunchKernelEx(&cfg, quantize_kernel<3>, a);
  }
  return cudaErrorInvalidValue;
}

}  // namespace mxq
