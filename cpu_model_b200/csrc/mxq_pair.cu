// mxq_pair.cu -- the decode (batch 1) linear pair in ONE kernel: y =
// W2 . quant(W1 . quant(x)), the 7B MLP's up and down projections
// (mxq_linear_pair; the reference's mx_gemv, nn/tests/test_auto_generated.cpp:56,
// called twice with the MX requantisation between, nn/core/layers/ssm.cpp:164-177).
//
// Why one kernel.  A batch-1 GEMV is a pure weight stream, ~3.3 us of HBM per
// 24 MB projection at the copy rate, but as two launches each SM's ingest
// idles while a launch computes, drains and hands over to the next (one
// register-resident CTA per SM cannot share the SM with its successor).  Here
// each CTA issues BOTH of its weight shares before it waits for anything:
//   up   (W1): into registers, up to kRounds 16-byte loads a thread;
//   down (W2): into shared memory, 16-byte cp.async copies of exactly its rows
//        ([k-tile][row][TB bytes]), plus the rows' E8M0 bytes of both layers
//        (8-byte copies, [k-tile][row][2]).
// So the whole pair's weights (~330 KB per SM for the 7B shape) are in flight
// from the first microsecond and the SM's ingest never waits on compute.
// Then: quantise x (per warp, its K-slice), up dot products from registers,
// the CTA's rows of y1 to global memory, a bounded grid-wide barrier, each
// warp quantises its K-slice of y1, down dot products from shared memory, y.
//
// Arithmetic order is exactly the weight-resident GEMV's (mxq_rgemv.cu): the
// same 4-row groups, the same contiguous K runs per warp and lane mapping,
// the same fma order, lane fold and warp-order sum, so the pair's y1 and y are
// bit-identical to two rgemv_res_kernel launches.
//
// Co-residency: one CTA per SM, grid <= the SM count (checked on the host
// against the occupancy calculator), so every CTA of the grid is resident
// when the barrier is reached; the barrier still gives up after the wait
// limit, records the timeout in the status word and skips the down phase.
#include "mxq_internal.h"

namespace mxq {

namespace {

constexpr int kPWarps = 16;
constexpr int kPThreads = kPWarps * 32;
constexpr int kRounds = 24;      // register rounds of the up share
constexpr int kGB = 4;           // 4-row groups per activation load

template <int WFMT>
struct PC {
  static constexpr int TB = WFMT == 4 ? 32 : 64;   // bytes per row per k-tile
  static constexpr int TPL = TB / 16;              // lanes per row per k-tile
  static constexpr int LPK = 4 * TPL;              // lanes per k-tile of a 4-row group
  static constexpr int KPL = 32 / LPK;             // k-tiles per warp load
  static constexpr int SHIFT = WFMT == 4 ? 4 : 0;  // int4 dots come out x16
};

// Per-layer geometry, identical on host and device.
struct LGeom {
  int KT, NL, kts, G4;   // k-tiles, warp loads per group, largest warp k-tiles, 4-row groups
};

template <int WFMT>
__host__ __device__ __forceinline__ LGeom lgeom(const WeightView& w) {
  using C = PC<WFMT>;
  LGeom g;
  g.KT = w.Kpad / kTileK;
  g.NL = (g.KT + C::KPL - 1) / C::KPL;
  g.kts = (g.NL + kPWarps - 1) / kPWarps * C::KPL;
  g.G4 = (w.N + 3) / 4;
  return g;
}

// Shared-memory plan (bytes), the same on host and device.
struct PPlan {
  int r1, r2;          // rows per CTA (max) of W1, W2
  int off_w2, off_s1, off_s2, off_act, off_part, total;
  int per_warp;        // activation slice bytes per warp (max of the layers)
};

__host__ __device__ __forceinline__ int ceil16(int v) { return (v + 15) / 16 * 16; }

template <int WFMT>
__host__ __device__ PPlan pplan(const WeightView& w1, const WeightView& w2, int G) {
  const LGeom g1 = lgeom<WFMT>(w1), g2 = lgeom<WFMT>(w2);
  PPlan p;
  p.r1 = (g1.G4 + G - 1) / G * 4;
  p.r2 = (g2.G4 + G - 1) / G * 4;
  const int slice = (g1.kts > g2.kts ? g1.kts : g2.kts) * kTileK;
  p.per_warp = ceil16(slice + slice / kBlock * 4);
  p.off_w2 = 0;
  p.off_s1 = ceil16(g2.KT * p.r2 * PC<WFMT>::TB);
  p.off_s2 = p.off_s1 + ceil16(g1.KT * p.r1 * 2);
  p.off_act = p.off_s2 + ceil16(g2.KT * p.r2 * 2);
  p.off_part = p.off_act + kPWarps * p.per_warp;
  // partial sums: [warp][group][4 rows] for the up rows, then the down rows
  p.total = p.off_part + kPWarps * (p.r1 / 4 + p.r2 / 4) * 4 * 4;
  return p;
}

__device__ __forceinline__ uint4 ldg_nc(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ void cpa16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cpa8(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds8(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u8 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Copy the E8M0 bytes of rows [n0, n0 + rows) for every k-tile into
// S[kt][row][2], `stride` rows per k-tile (8-byte pieces: rows come in whole
// 4-row groups, so every piece is 8-byte aligned on both sides and never
// crosses a row tile).
__device__ __forceinline__ void stage_scales(const WeightView& w, int KT, int n0, int rows, int stride,
                                             uint32_t dst) {
  const int pieces = rows / 4;
  for (int c = threadIdx.x; c < KT * pieces; c += kPThreads) {
    const int kt = c / pieces, p = c % pieces;
    const int n = n0 + p * 4;
    const size_t src = (((size_t)(n >> 7) * KT + kt) * 128 + (n & 127)) * 2;
    cpa8(dst + (uint32_t)((kt * stride + p * 4) * 2), w.scales + src);
  }
}

// This warp's K-slice of an fp32 row, MX-quantised exactly as quantize_kernel
// does, into act (int8, int4 layouts store each 8-group even elements first)
// and fa (block scales as floats).  8-lane groups share a 32-element block.
// The loads of NB rounds are issued before any of them is used, so a slice
// costs one memory round trip per NB rounds, not one per round.
template <int WFMT, bool CG, int NB>
__device__ __forceinline__ void quant_slice(const float* x, int K, int kt0, int nblk, int8_t* act, float* fa,
                                            int lane) {
  const int kb = K / kBlock;
  for (int base = lane; base < nblk * 8; base += 32 * NB) {
    float4 vv[NB];
#pragma unroll
    for (int u = 0; u < NB; ++u) {
      const int c = base + 32 * u;
      const int b = kt0 * 2 + c / 8;
      vv[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (c < nblk * 8 && b < kb) {
        const float4* src = reinterpret_cast<const float4*>(x + b * kBlock + (c % 8) * 4);
        vv[u] = CG ? __ldcg(src) : *src;
      }
    }
#pragma unroll
    for (int u = 0; u < NB; ++u) {
      const int c = base + 32 * u;          // warp-uniform: nblk * 8 is a multiple of 32
      if (c - lane >= nblk * 8) break;
      const int bl = c / 8, p4 = c % 8;
      const int b = kt0 * 2 + bl;
      const bool live = b < kb;
      const float e4[4] = {vv[u].x, vv[u].y, vv[u].z, vv[u].w};
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
      uint32_t s8 = 0;
      int e = 0;
      if (live) {
        if (nf) s8 = 255;
        else if (m != 0.0f) { e = e8m0_exponent<127>(m); s8 = (uint32_t)(e + 127); }
      }
      uint32_t packed = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int q = (s8 != 0 && s8 != 255) ? quant_value(e4[k], e) : 0;
        packed |= ((uint32_t)q & 0xFFu) << (8 * k);
      }
      if (WFMT == 4) {
        const uint32_t other = __shfl_xor_sync(0xffffffffu, packed, 1);
        packed = (p4 & 1) ? __byte_perm(other, packed, 0x7531) : __byte_perm(packed, other, 0x6420);
      }
      *reinterpret_cast<uint32_t*>(act + bl * kBlock + p4 * 4) = packed;
      if (p4 == 0) fa[bl] = live ? e8m0_to_float(s8) : 0.0f;
    }
  }
}

// One 16-byte weight piece against the activation: 16 * (or 1 *) the exact
// int32 dot, and the weight block scale as a float (2^(s-127-SHIFT)).
template <int WFMT, bool FAST>
__device__ __forceinline__ float piece(const uint4& w, uint32_t s, const uint4& x0, const uint4& x1, int& d) {
  using C = PC<WFMT>;
  int d0, d1;
  if (WFMT == 4) {
    const uint32_t m = 0xF0F0F0F0u;
    d0 = __dp4a((int)((w.x << 4) & m), (int)x0.x, 0);
    d1 = __dp4a((int)(w.x & m), (int)x0.y, 0);
    d0 = __dp4a((int)((w.y << 4) & m), (int)x0.z, d0);
    d1 = __dp4a((int)(w.y & m), (int)x0.w, d1);
    d0 = __dp4a((int)((w.z << 4) & m), (int)x1.x, d0);
    d1 = __dp4a((int)(w.z & m), (int)x1.y, d1);
    d0 = __dp4a((int)((w.w << 4) & m), (int)x1.z, d0);
    d1 = __dp4a((int)(w.w & m), (int)x1.w, d1);
  } else {
    d0 = __dp4a((int)x0.x, (int)w.x, 0);
    d1 = __dp4a((int)x0.y, (int)w.y, 0);
    d0 = __dp4a((int)x0.z, (int)w.z, d0);
    d1 = __dp4a((int)x0.w, (int)w.w, d1);
  }
  d = d0 + d1;
  return FAST ? __int_as_float((int)((s - C::SHIFT) << 23))
              : (s == 255u ? __int_as_float(0x7fc00000) : pow2_exact((int)s - 127 - C::SHIFT));
}

// Fold the 4 groups' lane sums of a warp (transpose reduction) and park each
// row's warp total in part[warp][group][4].
template <int WFMT>
__device__ __forceinline__ void fold_store(float (&acc)[kGB], int lane, int warp, int bi, int ng, int maxg,
                                           int rr, float* part) {
  constexpr int LA = 1, LB = WFMT == 4 ? 8 : 2, LC = 16;
  const bool bA = (lane & LA) != 0, bB = (lane & LB) != 0;
  const float s0 = bA ? acc[0] : acc[2], s1 = bA ? acc[1] : acc[3];
  float k0 = bA ? acc[2] : acc[0], k1 = bA ? acc[3] : acc[1];
  k0 += __shfl_xor_sync(0xffffffffu, s0, LA);
  k1 += __shfl_xor_sync(0xffffffffu, s1, LA);
  const float sx = bB ? k0 : k1;
  float k = bB ? k1 : k0;
  k += __shfl_xor_sync(0xffffffffu, sx, LB);
  k += __shfl_xor_sync(0xffffffffu, k, LC);
  const int gi = bi * kGB + (bA ? 2 : 0) + (bB ? 1 : 0);
  if (!(lane & LC) && gi < ng) part[(warp * maxg + gi) * 4 + rr] = k;
#pragma unroll
  for (int gg = 0; gg < kGB; ++gg) acc[gg] = 0.0f;
}

// Grid-wide barrier on {count, flag} (one launch at a time per context):
// the CTA's stores are ordered before its thread 0 by the CTA barrier; thread
// 0 fences and arrives; the last CTA to arrive resets the count and advances
// the flag; the others poll the flag with a time limit.  Returns false
// (status set) on timeout.  `arrive` false (test hook) skips the arrival.
__device__ bool grid_barrier(uint32_t* bar, uint32_t nctas, uint32_t* status, uint64_t lim, bool arrive) {
  __syncthreads();
  __shared__ int ok_s;
  if (threadIdx.x == 0) {
    int ok = 1;
    uint32_t* count = bar;
    uint32_t* flag = bar + 1;
    const uint32_t gen = ld_acquire(flag);
    __threadfence();
    if (arrive && atomicAdd(count, 1u) == nctas - 1) {
      atomicExch(count, 0u);
      __threadfence();
      atomicExch(flag, gen + 1u);
    } else {
      const uint64_t t0 = globaltimer_ns();
      for (uint32_t it = 0;; ++it) {
        if (ld_acquire(flag) != gen) break;
        if ((it & 15u) == 15u && globaltimer_ns() - t0 > lim) {
          atomicOr(status, kStatusTimeout);
          ok = 0;
          break;
        }
      }
    }
    __threadfence();
    ok_s = ok;
  }
  __syncthreads();
  return ok_s != 0;
}

template <int WFMT, bool FAST>
__global__ void __launch_bounds__(kPThreads, 1) pair_kernel(PairArgs a) {
  using C = PC<WFMT>;
  extern __shared__ __align__(16) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x;
  const PPlan P = pplan<WFMT>(a.w1, a.w2, G);
  const LGeom g1 = lgeom<WFMT>(a.w1), g2 = lgeom<WFMT>(a.w2);
  const uint32_t sb = smem_u32(smem);
  const uint64_t lim = a.wait_ns ? a.wait_ns : kWaitLimitNs;
  // lane -> (k-tile within a load, row within a group, 16-byte sub-slice)
  const int kto = lane / C::LPK;
  const int rr = (lane % C::LPK) / C::TPL;
  const int sub = lane % C::TPL;
  const int bh = WFMT == 4 ? sub : (sub >> 1);

  // rows of this CTA in each layer (whole 4-row groups)
  const int a_lo = (int)((long)blockIdx.x * g1.G4 / G), a_ng = (int)((long)(blockIdx.x + 1) * g1.G4 / G) - a_lo;
  const int b_lo = (int)((long)blockIdx.x * g2.G4 / G), b_ng = (int)((long)(blockIdx.x + 1) * g2.G4 / G) - b_lo;
  // K runs of this warp in each layer
  const int a_l0 = warp * g1.NL / kPWarps, a_nl = (warp + 1) * g1.NL / kPWarps - a_l0;
  const int b_l0 = warp * g2.NL / kPWarps, b_nl = (warp + 1) * g2.NL / kPWarps - b_l0;
  const int a_kt0 = a_l0 * C::KPL, b_kt0 = b_l0 * C::KPL;
  const int a_nr = (a_ng + kGB - 1) / kGB * a_nl * kGB;   // register rounds (<= kRounds, host-checked)

  // ---- 1. every weight byte of both layers in flight
  uint4 wv[kRounds];
  uint32_t vmask = 0;
  {
    int ibi = 0, ili = 0;
#pragma unroll
    for (int r = 0; r < kRounds; ++r) {
      const int gg = r % kGB;
      const int gi = ibi * kGB + gg;
      wv[r] = make_uint4(0, 0, 0, 0);
      if (r < a_nr && gi < a_ng && a_kt0 + ili * C::KPL + kto < g1.KT) {
        const int n = (a_lo + gi) * 4 + rr;
        const size_t rowoff = ((size_t)(n >> 7) * g1.KT + a_kt0 + ili * C::KPL + kto) * 128 + (n & 127);
        wv[r] = ldg_nc(a.w1.data + rowoff * C::TB + sub * 16);
        vmask |= 1u << r;
      }
      if (gg == kGB - 1 && ++ili == a_nl) { ili = 0; ++ibi; }
    }
  }
  {
    // copy group 1: the E8M0 bytes of both layers' rows; group 2: W2 rows
    // [b_lo*4, +b_ng*4) of every k-tile, TB bytes per row, 16-byte copies
    stage_scales(a.w1, g1.KT, a_lo * 4, a_ng * 4, P.r1, sb + P.off_s1);
    stage_scales(a.w2, g2.KT, b_lo * 4, b_ng * 4, P.r2, sb + P.off_s2);
    asm volatile("cp.async.commit_group;" ::: "memory");
    const int rows = b_ng * 4, per_kt = rows * C::TPL;
    for (int c = threadIdx.x; c < g2.KT * per_kt; c += kPThreads) {
      const int kt = c / per_kt, q = c % per_kt;
      const int n = b_lo * 4 + q / C::TPL;
      const size_t src = (((size_t)(n >> 7) * g2.KT + kt) * 128 + (n & 127)) * C::TB + (q % C::TPL) * 16;
      cpa16(sb + P.off_w2 + (uint32_t)((kt * P.r2 * C::TPL + q) * 16), a.w2.data + src);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");

  int8_t* act = reinterpret_cast<int8_t*>(smem + P.off_act + warp * P.per_warp);
  float* part = reinterpret_cast<float*>(smem + P.off_part);
  const int maxg1 = P.r1 / 4, maxg2 = P.r2 / 4;

  // ---- 2. up: quantise x's K-slice, dot products from registers
  const int a_nblk = g1.kts * 2;
  float* fa = reinterpret_cast<float*>(act + g1.kts * kTileK);
  quant_slice<WFMT, false, 2>(a.x, a.w1.K, a_kt0, a_nblk, act, fa, lane);
  asm volatile("cp.async.wait_group 1;" ::: "memory");   // every thread's scale copies have landed
  __syncthreads();
  {
    const int8_t* xrow = act + kto * kTileK + (WFMT == 4 ? sub * 32 : sub * 16);
    const float* frow = fa + kto * 2 + bh;
    float acc[kGB] = {0.0f, 0.0f, 0.0f, 0.0f};
    int li = 0, bi = 0;
#pragma unroll
    for (int r0 = 0; r0 < kRounds; r0 += kGB) {
      if (r0 < a_nr) {
        const int j = li * C::KPL;
        const float fx = frow[j * 2];
        const uint4 x0 = *reinterpret_cast<const uint4*>(xrow + j * kTileK);
        const uint4 x1 = WFMT == 4 ? *reinterpret_cast<const uint4*>(xrow + j * kTileK + 16) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int gg = 0; gg < kGB; ++gg) {
          const int r = r0 + gg;
          const int rl = (bi * kGB + gg) * 4 + rr;                       // row within the CTA
          uint32_t s = 127u;
          if ((vmask >> r) & 1u) s = lds8(sb + P.off_s1 + (uint32_t)(((a_kt0 + j + kto) * P.r1 + rl) * 2 + bh));
          int d;
          const float fw = piece<WFMT, FAST>(wv[r], s, x0, x1, d);
          acc[gg] = __fmaf_rn((float)d, __fmul_rn(fx, fw), acc[gg]);
        }
        if (++li == a_nl) {
          fold_store<WFMT>(acc, lane, warp, bi, a_ng, maxg1, rr, part);
          li = 0;
          ++bi;
        }
      }
    }
    if (a_nl == 0)
      for (int e = lane; e < a_ng * 4; e += 32) part[(warp * maxg1 + e / 4) * 4 + e % 4] = 0.0f;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < a_ng * 4; e += kPThreads) {
    const int gi = e / 4, r4 = e % 4;
    const int n = (a_lo + gi) * 4 + r4;
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < kPWarps; ++w) s += part[(w * maxg1 + gi) * 4 + r4];
    if (n < a.w1.N) a.y1[n] = s;
  }

  // ---- 3. every CTA's y1 rows are written
  const bool ok = grid_barrier(a.bar, (uint32_t)G, a.status, lim, !(a.withhold_arrive && blockIdx.x == 0));
  asm volatile("cp.async.wait_all;" ::: "memory");       // this thread's W2 copies, on every path
  __syncthreads();

  // ---- 4. down: quantise y1's K-slice, dot products from shared memory
  if (ok) {
    const int b_nblk = g2.kts * 2;
    float* fb = reinterpret_cast<float*>(act + g2.kts * kTileK);
    quant_slice<WFMT, true, 8>(a.y1, a.w2.K, b_kt0, b_nblk, act, fb, lane);
    __syncwarp();
    const int8_t* xrow = act + kto * kTileK + (WFMT == 4 ? sub * 32 : sub * 16);
    const float* frow = fb + kto * 2 + bh;
    const int nbk = (b_ng + kGB - 1) / kGB;
    float acc[kGB] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 1
    for (int bi = 0; bi < nbk; ++bi) {
#pragma unroll 1
      for (int li = 0; li < b_nl; ++li) {
        const int j = li * C::KPL;
        const int kt = b_kt0 + j + kto;
        const float fx = frow[j * 2];
        const uint4 x0 = *reinterpret_cast<const uint4*>(xrow + j * kTileK);
        const uint4 x1 = WFMT == 4 ? *reinterpret_cast<const uint4*>(xrow + j * kTileK + 16) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int gg = 0; gg < kGB; ++gg) {
          const int gi = bi * kGB + gg;
          const int rl = gi * 4 + rr;
          uint4 w = make_uint4(0, 0, 0, 0);
          uint32_t s = 127u;
          if (gi < b_ng && kt < g2.KT) {
            w = lds128(sb + P.off_w2 + (uint32_t)(((kt * P.r2 + rl) * C::TPL + sub) * 16));
            s = lds8(sb + P.off_s2 + (uint32_t)((kt * P.r2 + rl) * 2 + bh));
          }
          int d;
          const float fw = piece<WFMT, FAST>(w, s, x0, x1, d);
          acc[gg] = __fmaf_rn((float)d, __fmul_rn(fx, fw), acc[gg]);
        }
      }
      fold_store<WFMT>(acc, lane, warp, bi, b_ng, maxg2, rr, part + kPWarps * maxg1 * 4);
    }
    if (b_nl == 0)
      for (int e = lane; e < b_ng * 4; e += 32) part[kPWarps * maxg1 * 4 + (warp * maxg2 + e / 4) * 4 + e % 4] = 0.0f;
    __syncthreads();
    const float* p2 = part + kPWarps * maxg1 * 4;
    for (int e = threadIdx.x; e < b_ng * 4; e += kPThreads) {
      const int gi = e / 4, r4 = e % 4;
      const int n = (b_lo + gi) * 4 + r4;
      float s = 0.0f;
#pragma unroll
      for (int w = 0; w < kPWarps; ++w) s += p2[(w * maxg2 + gi) * 4 + r4];
      if (n < a.w2.N) a.y[n] = s;
    }
  }
}

int g_psms = 0;
int psms() {
  if (g_psms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&g_psms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || g_psms <= 0)
      g_psms = 148;
  }
  return g_psms;
}

template <int WFMT>
int pair_grid(const WeightView& w1, const WeightView& w2) {
  const LGeom g1 = lgeom<WFMT>(w1), g2 = lgeom<WFMT>(w2);
  int G = psms();
  if (g1.G4 < G) G = g1.G4;
  if (g2.G4 < G) G = g2.G4;
  return G;
}

template <int WFMT>
bool pair_ok_t(const WeightView& w1, const WeightView& w2) {
  if (w1.kt_ptr || w2.kt_ptr || w1.N != w2.K) return false;
  const int G = pair_grid<WFMT>(w1, w2);
  if (G < 1) return false;
  const LGeom g1 = lgeom<WFMT>(w1), g2 = lgeom<WFMT>(w2);
  const int rounds = ((g1.G4 + G - 1) / G + kGB - 1) / kGB * kGB * ((g1.NL + kPWarps - 1) / kPWarps);
  const PPlan P = pplan<WFMT>(w1, w2, G);
  return rounds <= kRounds && g1.kts <= 32 && g2.kts <= 32 && P.total <= 210 * 1024;
}

template <int WFMT, bool FAST>
cudaError_t launch_pair_t(const PairArgs& a, cudaStream_t st, bool pdl) {
  const int G = pair_grid<WFMT>(a.w1, a.w2);
  const PPlan P = pplan<WFMT>(a.w1, a.w2, G);
  static SmemAttr smem_attr;
  if (cudaError_t e = smem_attr.ensure(pair_kernel<WFMT, FAST>, (size_t)P.total)) return e;
  // the grid barrier needs every CTA resident at once: one per SM
  int occ = 0;
  if (cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, pair_kernel<WFMT, FAST>, kPThreads,
                                                                    (size_t)P.total))
    return e;
  if (occ < 1 || G > psms() * occ) return cudaErrorInvalidConfiguration;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)G);
  cfg.blockDim = dim3(kPThreads);
  cfg.dynamicSmemBytes = (size_t)P.total;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, pair_kernel<WFMT, FAST>, a);
}

template <int WFMT>
cudaError_t launch_pair_f(const PairArgs& a, cudaStream_t st, bool pdl) {
  constexpr int lo = WFMT == 4 ? 5 : 1;
  const bool fast = a.w1.scale_lo >= lo && a.w1.scale_hi <= 254 && a.w2.scale_lo >= lo && a.w2.scale_hi <= 254;
  return fast ? launch_pair_t<WFMT, true>(a, st, pdl) : launch_pair_t<WFMT, false>(a, st, pdl);
}

}  // namespace

bool pair_supported(const WeightView& w1, const WeightView& w2) {
  if (w1.fmt != w2.fmt) return false;
  return w1.fmt == 4 ? pair_ok_t<4>(w1, w2) : pair_ok_t<8>(w1, w2);
}

cudaError_t launch_pair(const PairArgs& a, cudaStream_t st, bool pdl) {
  if (!pair_supported(a.w1, a.w2) || !a.bar || !a.status || !a.y1) return cudaErrorInvalidValue;
  return a.w1.fmt == 4 ? launch_pair_f<4>(a, st, pdl) : launch_pair_f<8>(a, st, pdl);
}

}  // namespace mxq
