// mxq_bgemv.cu -- small-batch decode GEMV (3 <= batch <= 16) on the int8
// matrix-multiply-accumulate: the reference's mx_gemv / mx_quad_dot /
// mx_rank16_dot family (nn/tests/test_auto_generated.cpp:51-56) for a few
// tokens at once, HBM-bound like the batch-1 kernels.
//
// At batch 1 the dp4a kernels spend ~28 warp instructions per 512 weight
// bytes; with dp4a every further token adds ~13 per 16 bytes and lane, so
// batch 8 would cost ~4x the instructions of batch 1.  Here one
// mma.sync.m16n8k32 (s8 x s8 -> s32) computes a 16-row x 8-token x 32-K
// block product -- exactly one MX block, so its int32 results are the exact
// per-block dots of the contract -- and the per-block scales 2^(e_w + e_x)
// are applied to the four int32 results a lane holds (i2f, fmul, ffma).
// Batch 8 then costs about twice batch 1.
//
// K order inside a block is free (one scale per block), so a lane's
// fragment words come straight from the tiled weight layout: lane (g, t)
// takes word t (int4: 8 nibbles) of rows g and g+8 of each block; for int4
// the low nibbles (shifted up) fill the k-slots 4t..4t+3 and the high
// nibbles 16+4t..16+4t+3, both as 16*w, and the activation is stored with
// each 8-element group's even elements first so the B fragment reads the
// matching bytes; for int8 a lane takes bytes 8t..8t+7 of the row's block.
//
// Work split: 16-row units in contiguous balanced ranges per CTA (one CTA
// per SM), the K range dealt to the 16 warps in contiguous k-tile runs.  A
// warp streams its (unit, k-tile) stages -- 16 rows x 32 (64) bytes plus the
// 32 scale bytes -- through a private shared-memory ring of 6 stages with
// cp.async, the first ring's worth issued before the kernel waits for its
// predecessor.  Accumulators stay in registers per unit; after the last
// stage each warp parks its partial sums in its own shared-memory region and
// the CTA adds the 16 warps' values in warp order: deterministic, no
// cross-CTA reduction.
//
// Input: an MX activation (u8 q+128 bytes and E8M0 scales).  fp32 callers
// quantise first (quantize_kernel), which gives the same bytes.
#include "mxq_internal.h"

namespace mxq {

namespace {

constexpr int kBW = 16;                // warps per CTA
constexpr int kBT = kBW * 32;
// ring stages per warp (deeper rings, 8-14 stages, measured no faster: the
// kernel is not bound by the bytes in flight)
constexpr int kRings[1] = {6};
constexpr int kMaxUnits = 8;           // 16-row units per CTA (register accumulators)

template <int WFMT>
struct BCfg {
  static constexpr int TB = WFMT == 4 ? 32 : 64;     // bytes per row per k-tile
  static constexpr int S = TB + 16;                  // padded row stride in a stage (conflict-free reads)
  static constexpr int SB = 16 * S + 32;             // stage: 16 rows, then 32 scale bytes
  static constexpr int SHIFT = WFMT == 4 ? 4 : 0;    // int4 products come out x16
};

__device__ __forceinline__ void bcp16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void bcommit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bwait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void mma_s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                       uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

struct BGeom {
  int KT;      // k-tiles
  int kts;     // k-tiles of the largest warp slice
  int U;       // 16-row units
};

template <int WFMT>
__host__ __device__ __forceinline__ BGeom bgeom(const WeightView& w) {
  BGeom g;
  g.KT = w.Kpad / kTileK;
  g.kts = (g.KT + kBW - 1) / kBW;
  g.U = (w.N + 15) / 16;
  return g;
}

// shared memory: per warp one region -- its ring of R stages, then its
// activation slice [kts*2 blocks][NT tokens][32 B] and the block scales
// [kts*2][NT] floats; the region holds the warp's partial sums at the end
template <int WFMT, int NT>
__host__ __device__ __forceinline__ int bact_bytes(const BGeom& g) {
  return g.kts * 2 * NT * (32 + 4);
}

template <int WFMT, int NT>
__host__ __device__ __forceinline__ int bwarp_bytes(const BGeom& g, int R) {
  return R * BCfg<WFMT>::SB + bact_bytes<WFMT, NT>(g);
}

template <int WFMT, int NT, int kBR, bool FAST>
__global__ void __launch_bounds__(kBT, 1) bgemv_kernel(GemvArgs a) {
  using C = BCfg<WFMT>;
  constexpr int NM = NT / 8;                              // MMAs per block (8 tokens each)
  extern __shared__ __align__(16) uint8_t smem[];
  const BGeom g = bgeom<WFMT>(a.w);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gq = lane >> 2, tq = lane & 3;                // fragment row group / thread in group
  const int G = gridDim.x;
  const int u_lo = (int)((long)blockIdx.x * g.U / G);
  const int nu = (int)((long)(blockIdx.x + 1) * g.U / G) - u_lo;   // <= kMaxUnits (host check)
  const int kt0 = warp * g.KT / kBW;
  const int nkt = (warp + 1) * g.KT / kBW - kt0;
  const int Q = nu * nkt;                                 // stages of this warp

  const int wbytes = bwarp_bytes<WFMT, NT>(g, kBR);
  uint8_t* ring = smem + warp * wbytes;
  const uint32_t ring_s = smem_u32(ring);
  uint8_t* act = ring + kBR * C::SB;
  float* fa = reinterpret_cast<float*>(act + g.kts * 2 * NT * 32);

  // stages in order (unit, k-tile), k-tile fastest; the issue cursor walks
  // them incrementally.  Lane L copies 16 B (int4) / 32 B (int8) of row L/2,
  // lanes 0-1 the 32 scale bytes.
  const int r_ld = lane >> 1, h_ld = lane & 1;
  int iq = 0, iu = u_lo, ikt = kt0;
  auto issue = [&](int slot) {
    if (iq < Q) {
      const int row0 = iu * 16;
      const size_t tile = (size_t)(row0 >> 7) * g.KT + ikt;
      const uint8_t* src = a.w.data + (tile * 128 + (row0 & 127) + r_ld) * C::TB + h_ld * (C::TB / 2);
      const uint32_t dst = ring_s + slot * C::SB + r_ld * C::S + h_ld * (C::TB / 2);
      bcp16(dst, src);
      if (WFMT == 8) bcp16(dst + 16, src + 16);
      if (lane < 2)
        bcp16(ring_s + slot * C::SB + 16 * C::S + lane * 16, a.w.scales + (tile * 128 + (row0 & 127)) * 2 + lane * 16);
      ++iq;
      if (++ikt == kt0 + nkt) { ikt = kt0; ++iu; }
    }
    bcommit();
  };
#pragma unroll 1
  for (int s = 0; s < kBR; ++s) issue(s);
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");

  // ---- this warp's activation slice: signed bytes (int4 weights: each
  // 8-group even elements first), layout [block][token][32 B]; scales [block][token]
  const int K = a.w.K, kb = K / kBlock, B = a.B;
  {
    const int chunks = NT * g.kts * 4;                    // 16-byte chunks (token, 16 K)
    constexpr int QB = 6;
    for (int base = lane; base < chunks; base += 32 * QB) {
      uint4 v[QB];
#pragma unroll
      for (int i = 0; i < QB; ++i) {
        const int c = base + i * 32;
        const int t = c / (g.kts * 4), cc = c % (g.kts * 4);
        const int k = kt0 * kTileK + cc * 16;
        v[i] = make_uint4(0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u);
        if (c < chunks && t < B && cc < nkt * 4 && k < K)
          v[i] = *reinterpret_cast<const uint4*>(a.xq + (size_t)t * K + k);
      }
#pragma unroll
      for (int i = 0; i < QB; ++i) {
        const int c = base + i * 32;
        if (c < chunks) {
          const int t = c / (g.kts * 4), cc = c % (g.kts * 4);
          uint4 x = v[i];
          x.x ^= 0x80808080u; x.y ^= 0x80808080u; x.z ^= 0x80808080u; x.w ^= 0x80808080u;
          if (WFMT == 4)
            x = make_uint4(__byte_perm(x.x, x.y, 0x6420), __byte_perm(x.x, x.y, 0x7531),
                           __byte_perm(x.z, x.w, 0x6420), __byte_perm(x.z, x.w, 0x7531));
          *reinterpret_cast<uint4*>(act + ((cc >> 1) * NT + t) * 32 + (cc & 1) * 16) = x;
        }
      }
    }
    for (int c = lane; c < g.kts * 2 * NT; c += 32) {
      const int bl = c / NT, t = c % NT;
      const int b = kt0 * 2 + bl;
      fa[c] = (t < B && bl < nkt * 2 && b < kb) ? e8m0_to_float(a.xs[(size_t)t * kb + b]) : 0.0f;
    }
  }
  __syncwarp();

  float acc[kMaxUnits][NM][4];
#pragma unroll
  for (int u = 0; u < kMaxUnits; ++u)
#pragma unroll
    for (int m = 0; m < NM; ++m)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[u][m][i] = 0.0f;

  int slot = 0;                                           // ring slot of the next stage
#pragma unroll
  for (int u = 0; u < kMaxUnits; ++u) {
    if (u < nu) {
#pragma unroll 1
      for (int j = 0; j < nkt; ++j) {
        bwait<kBR - 1>();
        __syncwarp();
        const uint8_t* st = ring + slot * C::SB;
        // weight scales of rows gq, gq+8 (both blocks of the k-tile)
        const uint32_t sr0 = *reinterpret_cast<const uint16_t*>(st + 16 * C::S + gq * 2);
        const uint32_t sr1 = *reinterpret_cast<const uint16_t*>(st + 16 * C::S + (gq + 8) * 2);
#pragma unroll
        for (int b = 0; b < 2; ++b) {
          uint32_t a0, a1, a2, a3;
          if (WFMT == 4) {
            const uint32_t w0 = *reinterpret_cast<const uint32_t*>(st + gq * C::S + b * 16 + 4 * tq);
            const uint32_t w1 = *reinterpret_cast<const uint32_t*>(st + (gq + 8) * C::S + b * 16 + 4 * tq);
            const uint32_t mk = 0xF0F0F0F0u;
            a0 = (w0 << 4) & mk;
            a1 = (w1 << 4) & mk;
            a2 = w0 & mk;
            a3 = w1 & mk;
          } else {
            const uint2 w0 = *reinterpret_cast<const uint2*>(st + gq * C::S + b * 32 + 8 * tq);
            const uint2 w1 = *reinterpret_cast<const uint2*>(st + (gq + 8) * C::S + b * 32 + 8 * tq);
            a0 = w0.x;
            a1 = w1.x;
            a2 = w0.y;
            a3 = w1.y;
          }
          const uint32_t s0 = (sr0 >> (8 * b)) & 0xFFu, s1 = (sr1 >> (8 * b)) & 0xFFu;
          float f0, f1;
          if (FAST) {
            f0 = __int_as_float((int)((s0 - C::SHIFT) << 23));
            f1 = __int_as_float((int)((s1 - C::SHIFT) << 23));
          } else {
            f0 = s0 == 255u ? __int_as_float(0x7fc00000) : pow2_exact((int)s0 - 127 - C::SHIFT);
            f1 = s1 == 255u ? __int_as_float(0x7fc00000) : pow2_exact((int)s1 - 127 - C::SHIFT);
          }
          const int bl = j * 2 + b;
#pragma unroll
          for (int m = 0; m < NM; ++m) {
            const uint2 xb = *reinterpret_cast<const uint2*>(act + (bl * NT + m * 8 + gq) * 32 + 8 * tq);
            const float2 fx = *reinterpret_cast<const float2*>(fa + bl * NT + m * 8 + 2 * tq);
            int d[4];
            mma_s8(d, a0, a1, a2, a3, xb.x, xb.y);
            acc[u][m][0] = __fmaf_rn((float)d[0], __fmul_rn(f0, fx.x), acc[u][m][0]);
            acc[u][m][1] = __fmaf_rn((float)d[1], __fmul_rn(f0, fx.y), acc[u][m][1]);
            acc[u][m][2] = __fmaf_rn((float)d[2], __fmul_rn(f1, fx.x), acc[u][m][2]);
            acc[u][m][3] = __fmaf_rn((float)d[3], __fmul_rn(f1, fx.y), acc[u][m][3]);
          }
        }
        __syncwarp();                                     // every lane is done with the slot
        issue(slot);                                      // the stage kBR ahead
        slot = slot + 1 == kBR ? 0 : slot + 1;
      }
    }
  }
  bwait<0>();
  __syncwarp();
  // park the partial sums in this warp's region: [unit][16 rows][NT tokens]
  float* part = reinterpret_cast<float*>(ring);
#pragma unroll
  for (int u = 0; u < kMaxUnits; ++u)
    if (u < nu)
#pragma unroll
      for (int m = 0; m < NM; ++m) {
        const int t0 = m * 8 + 2 * tq;
        part[(u * 16 + gq) * NT + t0] = acc[u][m][0];
        part[(u * 16 + gq) * NT + t0 + 1] = acc[u][m][1];
        part[(u * 16 + gq + 8) * NT + t0] = acc[u][m][2];
        part[(u * 16 + gq + 8) * NT + t0 + 1] = acc[u][m][3];
      }
  __syncthreads();
  // y = sum over the 16 warps, in warp order
  for (int e = threadIdx.x; e < nu * 16 * NT; e += kBT) {
    const int t = e % NT, r = e / NT;
    const int n = u_lo * 16 + r;
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < kBW; ++w) s += reinterpret_cast<const float*>(smem + w * wbytes)[r * NT + t];
    if (t < B && n < a.w.N) a.y[(size_t)t * a.w.N + n] = s;
  }
}

int bsms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  }
  return n;
}

// ring depth for this shape: one that fits shared memory and whose region
// holds the partial sums; 0 when none does
template <int WFMT, int NT>
int bring(const WeightView& w) {
  const BGeom g = bgeom<WFMT>(w);
  const int G = g.U < bsms() ? g.U : bsms();
  const int max_nu = (g.U + G - 1) / G;
  if (max_nu > kMaxUnits) return 0;
  for (int R : kRings) {
    const size_t wb = (size_t)bwarp_bytes<WFMT, NT>(g, R);
    if (wb * kBW <= 220 * 1024 && (size_t)max_nu * 16 * NT * 4 <= wb) return R;
  }
  return 0;
}

template <int WFMT, int NT, int R, bool FAST>
cudaError_t blaunch_t(const GemvArgs& a, cudaStream_t st, bool pdl) {
  const BGeom g = bgeom<WFMT>(a.w);
  const size_t smem = (size_t)kBW * bwarp_bytes<WFMT, NT>(g, R);
  static SmemAttr smem_attr;
  if (cudaError_t e = smem_attr.ensure(bgemv_kernel<WFMT, NT, R, FAST>, smem)) return e;
  const int grid = g.U < bsms() ? g.U : bsms();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kBT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, bgemv_kernel<WFMT, NT, R, FAST>, a);
}

template <int WFMT, int NT, bool FAST>
cudaError_t blaunch_r(const GemvArgs& a, cudaStream_t st, bool pdl) {
  switch (bring<WFMT, NT>(a.w)) {
    case 6: return blaunch_t<WFMT, NT, 6, FAST>(a, st, pdl);
  }
  return cudaErrorInvalidValue;
}

template <int WFMT, int NT>
cudaError_t blaunch(const GemvArgs& a, cudaStream_t st, bool pdl) {
  return a.w.scale_lo >= (WFMT == 4 ? 5 : 1) && a.w.scale_hi <= 254 ? blaunch_r<WFMT, NT, true>(a, st, pdl)
                                                                      : blaunch_r<WFMT, NT, false>(a, st, pdl);
}

}  // namespace

bool bgemv_supported(const WeightView& w, int B) {
  if (B < kBgemvMinBatch || B > kBgemvMaxBatch || w.kt_ptr) return false;
  if (w.fmt == 4) return (B <= 8 ? bring<4, 8>(w) : bring<4, 16>(w)) > 0;
  return (B <= 8 ? bring<8, 8>(w) : bring<8, 16>(w)) > 0;
}

cudaError_t launch_bgemv(const GemvArgs& a, cudaStream_t st, bool pdl) {
  if (!bgemv_supported(a.w, a.B) || !a.xq || !a.xs || a.xf || a.rows || a.block_dots) return cudaErrorInvalidValue;
  if (a.w.fmt == 4) return a.B <= 8 ? blaunch<4, 8>(a, st, pdl) : blaunch<4, 16>(a, st, pdl);
  return a.B <= 8 ? blaunch<8, 8>(a, st, pdl) : blaunch<8, 16>(a, st, pdl);
}

}  // namespace mxq
