// mxq_gemv.cu -- decode-regime MX GEMV (batch <= 8): mx_gemv / mx_dot /
// mx_rank16_dot / mx_rank16_dot_ptrs of the reference
// (nn/tests/test_auto_generated.cpp:51-56; VNNI design nn/user.md:17).
//
// HBM-bound design.  Weights are read once, 16 bytes per lane per k-tile,
// straight from the tiled layout: for int4 a warp covers 16 rows x 32 bytes
// (512 contiguous bytes) per k-tile, two lanes per row, each lane one whole
// 32-element block; for int8, 8 rows x 64 bytes, four lanes per row.  The
// eight warps of a CTA split K; loads are double-buffered in registers
// (two batches of 4 k-tiles in flight per warp) and the first batch is
// issued before the programmatic-dependent-launch wait, so weight streaming
// overlaps the producer of the activations.  Activations (signed int8 and
// the block scale as a float) are staged once per warp in shared memory;
// lanes of a warp read them as broadcasts.
//
// Per block: int4 nibbles are widened to int8 in place as 16*w
// ((w << 4) & 0xF0F0F0F0 and w & 0xF0F0F0F0, re-interleaved with two
// byte-permutes), eight dp4a give 16 * sum(q_x * q_w) exactly, and the block
// scale 2^(e_x + e_w - 4) folds the factor 16 back out.  The int32 block dot
// is exact, as in the reference's dpbusd path; the fp32 sum over blocks runs
// in k order per lane and is combined across lanes and warps in a fixed
// order (deterministic).
#include "mxq_internal.h"

namespace mxq {

namespace {

constexpr int kGemvWarps = 8;
constexpr int kGemvU = 4;

// Shared memory per warp: NB x S x 64 activation bytes + NB x S x 2 float
// scales, rounded to 16 bytes so every warp's slice stays 16-byte aligned.
__host__ __device__ constexpr int gemv_warp_bytes(int nb, int s) {
  return (nb * s * 72 + 15) / 16 * 16;
}

__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// int4 word (8 nibbles, element 2i low) -> two words of 16*w in natural order
__device__ __forceinline__ void unpack_int4_x16(uint32_t w, uint32_t& n0,
                                                uint32_t& n1) {
  const uint32_t lo = (w << 4) & 0xF0F0F0F0u;  // 16*e0,16*e2,16*e4,16*e6
  const uint32_t hi = w & 0xF0F0F0F0u;         // 16*e1,16*e3,16*e5,16*e7
  n0 = __byte_perm(lo, hi, 0x5140);
  n1 = __byte_perm(lo, hi, 0x7362);
}

// 16 * (32-element block dot) for int4 weights in `w`, activations in x[8].
__device__ __forceinline__ int dot16_int4(const uint32_t (&n)[8],
                                          const uint4& x0, const uint4& x1) {
  int d = 0;
  d = __dp4a((int)x0.x, (int)n[0], d);
  d = __dp4a((int)x0.y, (int)n[1], d);
  d = __dp4a((int)x0.z, (int)n[2], d);
  d = __dp4a((int)x0.w, (int)n[3], d);
  d = __dp4a((int)x1.x, (int)n[4], d);
  d = __dp4a((int)x1.y, (int)n[5], d);
  d = __dp4a((int)x1.z, (int)n[6], d);
  d = __dp4a((int)x1.w, (int)n[7], d);
  return d;
}

__device__ __forceinline__ void unpack_block_int4(const uint4& w,
                                                  uint32_t (&n)[8]) {
  unpack_int4_x16(w.x, n[0], n[1]);
  unpack_int4_x16(w.y, n[2], n[3]);
  unpack_int4_x16(w.z, n[4], n[5]);
  unpack_int4_x16(w.w, n[6], n[7]);
}

// Half-block (16 elements) int8 dot.
__device__ __forceinline__ int dot_int8_half(const uint4& w, const uint4& x) {
  int d = 0;
  d = __dp4a((int)x.x, (int)w.x, d);
  d = __dp4a((int)x.y, (int)w.y, d);
  d = __dp4a((int)x.z, (int)w.z, d);
  d = __dp4a((int)x.w, (int)w.w, d);
  return d;
}

__device__ __forceinline__ uint4 xor80(uint4 v) {
  v.x ^= 0x80808080u;
  v.y ^= 0x80808080u;
  v.z ^= 0x80808080u;
  v.w ^= 0x80808080u;
  return v;
}

// weight block scale: 2^(s - 127 - shift), NaN for 0xFF
template <int SHIFT>
__device__ __forceinline__ float wscale(uint32_t s) {
  return s == 255u ? __int_as_float(0x7fc00000)
                   : pow2_exact((int)s - 127 - SHIFT);
}

template <int WFMT, int NB, bool GATHER, bool INF32>
__global__ void __launch_bounds__(256, 2) gemv_kernel(GemvArgs a) {
  constexpr int LPR = WFMT == 4 ? 2 : 4;  // lanes per row
  constexpr int ROWS = 32 / LPR;          // rows per warp (and per CTA)
  constexpr int TB = WFMT == 4 ? 32 : 64; // bytes per row per k-tile
  constexpr int U = kGemvU;
  constexpr int SHIFT = WFMT == 4 ? 4 : 0;
  extern __shared__ __align__(16) uint8_t smem[];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KT = a.w.Kpad / kTileK;
  const int S = (KT + kGemvWarps - 1) / kGemvWarps;
  const int kt0 = min(KT, warp * S);
  const int kt1 = min(KT, kt0 + S);
  const int nkt = kt1 - kt0;
  const int rloc = lane / LPR, sub = lane % LPR;

  int col = blockIdx.x * ROWS + rloc;  // output column
  int row;
  bool row_ok;
  if (GATHER) {
    row = col < a.nrows ? a.rows[col] : -1;
    row_ok = row >= 0 && row < a.w.N;
  } else {
    row = col;
    row_ok = row < a.w.Npad;
  }
  const int rr = row_ok ? row : 0;
  const size_t tile_stride = (size_t)128 * TB;  // bytes between k-tiles
  const uint8_t* wbase = a.w.data +
                         ((size_t)(rr / 128) * KT * 128 + (rr % 128)) * TB +
                         sub * 16 + (size_t)kt0 * tile_stride;
  const uint8_t* sbase = a.w.scales +
                         ((size_t)(rr / 128) * KT * 128 + (rr % 128)) * 2 +
                         (WFMT == 4 ? sub : (sub >> 1)) + (size_t)kt0 * 256;

  uint4 wa[U], wb[U];
  uint32_t sa[U], sbv[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    if (u < nkt) {
      wa[u] = ldg_stream(wbase + u * tile_stride);
      sa[u] = __ldg(sbase + u * 256);
    }
  }
  if (a.pf_bytes && threadIdx.x == 0) {
    // warm L2 with this CTA's share of the next layer's weights: their HBM
    // reads overlap this kernel instead of waiting for the next launch
    prefetch_l2_share(a.pf_ptr, a.pf_bytes, blockIdx.x, gridDim.x);
    prefetch_l2_share(a.pf_ptr2, a.pf_bytes2, blockIdx.x, gridDim.x);
  }

  asm volatile("griddepcontrol.wait;" ::: "memory");

  // ---- stage this warp's activation slice: signed int8 + float scales
  const int per_warp = gemv_warp_bytes(NB, S);
  uint8_t* act = smem + warp * per_warp;
  float* fa = reinterpret_cast<float*>(act + NB * S * 64);
  const int kb = a.w.K / kBlock;
  if (INF32) {
    // fp32 rows quantised here with quantize_kernel's arithmetic (bytes are
    // identical): 8 lanes per 32-element block, one float4 each, all of a
    // batch's loads in flight before use
    constexpr int QB = 6;
    const int nblk = nkt * 2;
    const int items = NB * nblk * 8;
    for (int base = lane; base < items; base += 32 * QB) {
      float4 v[QB];
#pragma unroll
      for (int i = 0; i < QB; ++i) {
        const int c = base + i * 32;
        const int t = c / (nblk * 8), bl = (c / 8) % nblk, part = c % 8;
        const int b = kt0 * 2 + bl;
        v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (c < items && t < a.B && b < kb)
          v[i] = *reinterpret_cast<const float4*>(a.xf + (size_t)t * a.w.K + b * kBlock + part * 4);
      }
#pragma unroll
      for (int i = 0; i < QB; ++i) {
        const int c = base + i * 32;          // 8-lane groups share (t, block)
        const int t = c / (nblk * 8), bl = (c / 8) % nblk, part = c % 8;
        const int b = kt0 * 2 + bl;
        const float e4[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
        float m = 0.0f;
        bool nf = false;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float av = fabsf(e4[e]);
          nf |= !(av <= 3.402823466e38f);
          m = fmaxf(m, nf ? 0.0f : av);
        }
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) {
          m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
          nf |= __shfl_xor_sync(0xffffffffu, (int)nf, o) != 0;
        }
        if (c < items) {
          uint32_t sb = 0;
          int e = 0;
          const bool live = t < a.B && b < kb;
          if (live) {
            if (nf) sb = 255;
            else if (m != 0.0f) { e = e8m0_exponent<127>(m); sb = (uint32_t)(e + 127); }
          }
          uint32_t packed = 0;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int q = (sb != 0 && sb != 255) ? quant_value(e4[k], e) : 0;
            packed |= ((uint32_t)q & 0xFFu) << (8 * k);
          }
          *reinterpret_cast<uint32_t*>(act + t * S * 64 + bl * kBlock + part * 4) = packed;
          if (part == 0) fa[t * S * 2 + bl] = live ? e8m0_to_float(sb) : 0.0f;
        }
      }
    }
  } else {
#pragma unroll
    for (int t = 0; t < NB; ++t) {
      if (t < a.B) {
        for (int c = lane; c < nkt * 4; c += 32) {
          const int k = kt0 * kTileK + c * 16;
          uint4 v = make_uint4(0, 0, 0, 0);
          if (k < a.w.K)
            v = xor80(*reinterpret_cast<const uint4*>(a.xq + (size_t)t * a.w.K + k));
          *reinterpret_cast<uint4*>(act + t * S * 64 + c * 16) = v;
        }
        for (int bb = lane; bb < nkt * 2; bb += 32) {
          const int b = kt0 * 2 + bb;
          fa[t * S * 2 + bb] = b < kb ? e8m0_to_float(a.xs[(size_t)t * kb + b]) : 0.0f;
        }
      } else {
        for (int c = lane; c < nkt * 4; c += 32)
          *reinterpret_cast<uint4*>(act + t * S * 64 + c * 16) = make_uint4(0, 0, 0, 0);
        for (int bb = lane; bb < nkt * 2; bb += 32) fa[t * S * 2 + bb] = 0.0f;
      }
    }
  }
  __syncwarp();

  float acc[NB];
#pragma unroll
  for (int t = 0; t < NB; ++t) acc[t] = 0.0f;

  auto compute = [&](const uint4& w, uint32_t s, int j) {
    // j = k-tile index within this warp's slice
    const float fw = wscale<SHIFT>(s);
    if (WFMT == 4) {
      uint32_t n[8];
      unpack_block_int4(w, n);
#pragma unroll
      for (int t = 0; t < NB; ++t) {
        const uint4* xp = reinterpret_cast<const uint4*>(act + t * S * 64 + j * 64 + sub * 32);
        const uint4 x0 = xp[0], x1 = xp[1];
        const int d = dot16_int4(n, x0, x1);
        const float f = fa[t * S * 2 + j * 2 + sub];
        acc[t] = __fmaf_rn((float)d, __fmul_rn(f, fw), acc[t]);
      }
    } else {
#pragma unroll
      for (int t = 0; t < NB; ++t) {
        const uint4 x = *reinterpret_cast<const uint4*>(act + t * S * 64 + j * 64 + sub * 16);
        const int d = dot_int8_half(w, x);
        const float f = fa[t * S * 2 + j * 2 + (sub >> 1)];
        acc[t] = __fmaf_rn((float)d, __fmul_rn(f, fw), acc[t]);
      }
    }
  };

  for (int base = 0; base < nkt; base += 2 * U) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = base + U + u;
      if (j < nkt) {
        wb[u] = ldg_stream(wbase + j * tile_stride);
        sbv[u] = __ldg(sbase + j * 256);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (base + u < nkt) compute(wa[u], sa[u], base + u);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = base + 2 * U + u;
      if (j < nkt) {
        wa[u] = ldg_stream(wbase + j * tile_stride);
        sa[u] = __ldg(sbase + j * 256);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (base + U + u < nkt) compute(wb[u], sbv[u], base + U + u);
  }

  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

#pragma unroll
  for (int t = 0; t < NB; ++t) {
#pragma unroll
    for (int o = LPR / 2; o > 0; o >>= 1)
      acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], o);
  }
  float* partial = reinterpret_cast<float*>(smem + kGemvWarps * per_warp);
  if (sub == 0) {
#pragma unroll
    for (int t = 0; t < NB; ++t)
      partial[(warp * ROWS + rloc) * NB + t] = row_ok ? acc[t] : 0.0f;  // bad gathered ids give 0
  }
  __syncthreads();
  const int ncols = GATHER ? a.nrows : a.w.N;
  for (int i = threadIdx.x; i < ROWS * NB; i += blockDim.x) {
    const int r = i % ROWS, t = i / ROWS;
    const int c = blockIdx.x * ROWS + r;
    if (t < a.B && c < ncols) {
      float s = 0.0f;
#pragma unroll
      for (int w = 0; w < kGemvWarps; ++w) s += partial[(w * ROWS + r) * NB + t];
      a.y[(size_t)t * ncols + c] = s;
    }
  }
}

// Debug/parity kernel: every int32 block dot, through the same unpack and
// dp4a sequence as the GEMV.  One thread per (token, row, block).
template <int WFMT>
__global__ void block_dots_kernel(GemvArgs a) {
  const int kb = a.w.K / kBlock;
  const long total = (long)a.B * a.w.N * kb;
  const int KT = a.w.Kpad / kTileK;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long)gridDim.x * blockDim.x) {
    const int b = (int)(i % kb);
    const int n = (int)((i / kb) % a.w.N);
    const int t = (int)(i / ((long)kb * a.w.N));
    const int kt = b / 2, h = b % 2;
    const size_t rowoff = ((size_t)(n / 128) * KT + kt) * 128 + (n % 128);
    const uint8_t* xp = a.xq + (size_t)t * a.w.K + b * kBlock;
    const uint4 x0 = xor80(*reinterpret_cast<const uint4*>(xp));
    const uint4 x1 = xor80(*reinterpret_cast<const uint4*>(xp + 16));
    int d;
    if (WFMT == 4) {
      const uint4 w = *reinterpret_cast<const uint4*>(a.w.data + rowoff * 32 + h * 16);
      uint32_t nn[8];
      unpack_block_int4(w, nn);
      d = dot16_int4(nn, x0, x1) >> 4;
    } else {
      const uint8_t* wp = a.w.data + rowoff * 64 + h * 32;
      d = dot_int8_half(*reinterpret_cast<const uint4*>(wp), x0) +
          dot_int8_half(*reinterpret_cast<const uint4*>(wp + 16), x1);
    }
    a.block_dots[i] = d;
  }
}

template <int WFMT, int NB, bool GATHER, bool INF32>
cudaError_t launch_t(const GemvArgs& a, cudaStream_t st, bool pdl) {
  constexpr int LPR = WFMT == 4 ? 2 : 4;
  constexpr int ROWS = 32 / LPR;
  const int KT = a.w.Kpad / kTileK;
  const int S = (KT + kGemvWarps - 1) / kGemvWarps;
  const size_t smem = (size_t)kGemvWarps * gemv_warp_bytes(NB, S) +
                      (size_t)kGemvWarps * ROWS * NB * 4;
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  static SmemAttr smem_attr;
  if (cudaError_t e = smem_attr.ensure(gemv_kernel<WFMT, NB, GATHER, INF32>, smem)) return e;
  const int ncols = GATHER ? a.nrows : a.w.Npad;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((ncols + ROWS - 1) / ROWS));
  cfg.blockDim = dim3(kGemvWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gemv_kernel<WFMT, NB, GATHER, INF32>, a);
}

template <int WFMT, bool GATHER, bool INF32>
cudaError_t launch_fmt(const GemvArgs& a, cudaStream_t st, bool pdl) {
  switch (a.B) {
    case 1: return launch_t<WFMT, 1, GATHER, INF32>(a, st, pdl);
    case 2: return launch_t<WFMT, 2, GATHER, INF32>(a, st, pdl);
    case 3: return launch_t<WFMT, 3, GATHER, INF32>(a, st, pdl);
    case 4: return launch_t<WFMT, 4, GATHER, INF32>(a, st, pdl);
    case 5: case 6: return launch_t<WFMT, 6, GATHER, INF32>(a, st, pdl);
    case 7: case 8: return launch_t<WFMT, 8, GATHER, INF32>(a, st, pdl);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

int gemv_max_batch() { return 8; }

cudaError_t launch_gemv(const GemvArgs& a, cudaStream_t st, bool pdl) {
  if (a.block_dots) {
    const long total = (long)a.B * a.w.N * (a.w.K / kBlock);
    long ctas = (total + 255) / 256;
    if (ctas > 148L * 32) ctas = 148L * 32;
    if (ctas < 1) ctas = 1;
    if (a.w.fmt == 4) block_dots_kernel<4><<<(unsigned)ctas, 256, 0, st>>>(a);
    else block_dots_kernel<8><<<(unsigned)ctas, 256, 0, st>>>(a);
    return cudaGetLastError();
  }
  if (a.B < 1 || a.B > gemv_max_batch()) return cudaErrorInvalidValue;
  if (a.rows) return a.w.fmt == 4 ? launch_fmt<4, true, false>(a, st, pdl) : launch_fmt<8, true, false>(a, st, pdl);
  if (a.xf) return a.w.fmt == 4 ? launch_fmt<4, false, true>(a, st, pdl) : launch_fmt<8, false, true>(a, st, pdl);
  return a.w.fmt == 4 ? launch_fmt<4, false, false>(a, st, pdl) : launch_fmt<8, false, false>(a, st, pdl);
}

}  // namespace mxq
