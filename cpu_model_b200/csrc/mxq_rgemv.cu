// mxq_rgemv.cu -- persistent decode GEMVs (batch <= 4): the HBM-bound mx_gemv
// of the reference (nn/tests/test_auto_generated.cpp:56; dpbusd design
// nn/user.md:17).  Two kernels: the cp.async-ring kernel below (batches 2-4,
// and batch 1 when the weight-resident kernel further down does not fit the
// shape) and the weight-resident batch-1 kernel.
//
// One CTA per SM, 16 warps, one wave: fixed per-CTA costs (activation
// staging, pipeline ramp) are paid once per launch, not once per wave.
//
// Work split.  Output rows are taken in groups of 4; each CTA owns a
// contiguous, balanced range of groups (ranges differ by one group: for a
// 7B MLP 18-19 groups of the up projection, 6-7 of the down projection per
// CTA).  Inside a CTA the 16 warps split K; a warp streams its K-slice of
// every group it owns from HBM into a ring of shared-memory slots private to
// each thread (cp.async, 8 rounds in flight, issued before the kernel waits
// for its predecessor), and reads back only what it loaded.  In the
// tiled weight layout a group's k-tile is 128 (int4) or 256 (int8)
// contiguous bytes, so one warp round covers 4 (2) k-tiles of the group in
// full 128-byte lines.  Partial sums stay inside the CTA: each warp folds its
// lanes with shuffles, writes one value per row to shared memory, and after
// the last group the CTA adds the 16 warps' values in warp order -- no
// cross-CTA reduction, deterministic results.
//
// Activations (an MX activation, or fp32 rows quantised here with
// quantize_kernel's arithmetic -- identical bytes) are staged once per warp
// for its K-slice as signed int8 plus a float block scale.  int4 nibbles are
// widened to int8 in place (16*w by a shift and a mask, re-interleaved with
// two byte-permutes), eight dp4a give the exact int32 block dot (x16), and
// 2^(e_x + e_w - 4) scales it into the fp32 sum.
#include "mxq_internal.h"


namespace mxq {

namespace {

constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
// Weight loads land in a per-thread ring of kRing 16-byte slots in shared
// memory (cp.async, slot-major so a warp's accesses are contiguous), with
// the 4-byte words holding their scale bytes beside them: 8 rounds (80 KB per
// CTA, so two consecutive kernels' CTAs share an SM) are in flight from the
// first instruction.
template <int NB>
struct RRing {
  static constexpr int R = 8;
  static constexpr int BYTES = R * kThreads * (16 + 4);
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}

template <int WFMT>
struct RCfg {
  static constexpr int TB = WFMT == 4 ? 32 : 64;   // bytes per row per k-tile
  static constexpr int TPL = TB / 16;              // lanes per row per k-tile (2 / 4)
  static constexpr int LPK = 4 * TPL;              // lanes per k-tile of a 4-row group (8 / 16)
  static constexpr int KPL = 32 / LPK;             // k-tiles per warp load (4 / 2)
  static constexpr int SHIFT = WFMT == 4 ? 4 : 0;  // int4 dots come out x16
};

__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// geometry shared by host and device
struct RGeom {
  int KT;      // k-tiles
  int kts;     // k-tiles per warp (multiple of KPL)
  int nload;   // warp loads per group
  int G4;      // 4-row groups
};

template <int WFMT>
__host__ __device__ __forceinline__ RGeom rgeom(const WeightView& w) {
  using C = RCfg<WFMT>;
  RGeom g;
  g.KT = w.Kpad / kTileK;
  const int per = (g.KT + kWarps - 1) / kWarps;
  g.kts = (per + C::KPL - 1) / C::KPL * C::KPL;
  g.nload = g.kts / C::KPL;
  g.G4 = (w.N + 3) / 4;
  return g;
}

template <int WFMT, int NB, bool FAST, bool INF32>
__global__ void __launch_bounds__(kThreads, 2) rgemv_kernel(GemvArgs a) {
  using C = RCfg<WFMT>;
  extern __shared__ __align__(16) uint8_t smem[];
  const RGeom g = rgeom<WFMT>(a.w);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x;
  const int g_lo = (int)((long)blockIdx.x * g.G4 / G);
  const int g_hi = (int)((long)(blockIdx.x + 1) * g.G4 / G);
  const int ng = g_hi - g_lo;
  const int kt0 = warp * g.kts;

  // lane -> (k-tile within a load, row within the group, sub-slice)
  const int kto = lane / C::LPK;
  const int rr = (lane % C::LPK) / C::TPL;
  const int sub = lane % C::TPL;
  const int bh = WFMT == 4 ? sub : (sub >> 1);   // block within the k-tile

  // shared memory: per warp its activation slice, then the partial sums
  const int slice = g.kts * kTileK;                      // activation bytes per token
  const int per_warp = (NB * slice + NB * g.kts * 2 * 4 + 15) / 16 * 16;
  constexpr int kRing = RRing<NB>::R;
  constexpr int kRingBytes = RRing<NB>::BYTES;
  int8_t* act = reinterpret_cast<int8_t*>(smem + kRingBytes + warp * per_warp);
  float* fa = reinterpret_cast<float*>(act + NB * slice);
  float* part = reinterpret_cast<float*>(smem + kRingBytes + kWarps * per_warp);   // [warp][group][4 rows][NB]
  const int max_ng = (g.G4 + G - 1) / G;

  // The lane streams the sequence (group gi, load li) with li fastest; two
  // cursors walk it -- one issuing loads, one computing -- by pointer bumps,
  // with the row address recomputed once per group.
  const int Q = ng * g.nload;
  const size_t kstep_w = (size_t)C::KPL * 128 * C::TB;   // next load of the same row
  const size_t kstep_s = (size_t)C::KPL * 256;
  uint32_t kmask = 0;                                    // loads whose k-tile exists
  for (int li = 0; li < g.nload && li < 32; ++li)
    if (kt0 + li * C::KPL + kto < g.KT) kmask |= 1u << li;
  struct Cursor {
    int gi, li;
    const uint8_t* wp;
    const uint8_t* sp;
  };
  auto row_base = [&](Cursor& cu) {
    const int n = (g_lo + cu.gi) * 4 + rr;
    const size_t rowoff = ((size_t)(n >> 7) * g.KT + kt0 + kto) * 128 + (n & 127);
    cu.wp = a.w.data + rowoff * C::TB + sub * 16;
    cu.sp = a.w.scales + rowoff * 2 + bh;
  };
  auto step = [&](Cursor& cu) {
    if (++cu.li == g.nload) {
      cu.li = 0;
      ++cu.gi;
      row_base(cu);
    } else {
      cu.wp += kstep_w;
      cu.sp += kstep_s;
    }
  };
  Cursor ic{0, 0, nullptr, nullptr};
  row_base(ic);
  int issued = 0;

  const uint32_t ring_w = smem_u32(smem);
  const uint32_t ring_s = ring_w + kRing * kThreads * 16;
  const int tid = threadIdx.x;
  // the scale byte's position in its aligned 4-byte word (rows of a lane
  // keep one parity; the scale array starts 4-byte aligned)
  const int ssub = (2 * (rr & 1) + bh) & 3;
  // one round: this thread's next load (if any) into ring slot `slot`; a
  // group is committed every round, so the wait depth below stays constant
  auto issue_one = [&](int slot) {
    if (issued < Q) {
      if ((kmask >> ic.li) & 1u) {
        cp_async16(ring_w + (uint32_t)(slot * kThreads + tid) * 16u, ic.wp);
        cp_async4(ring_s + (uint32_t)(slot * kThreads + tid) * 4u,
                  reinterpret_cast<const void*>(reinterpret_cast<uintptr_t>(ic.sp) & ~(uintptr_t)3));
      }
      step(ic);
      ++issued;
    }
    cp_async_commit();
  };
  // the weights do not depend on the previous kernel: the whole ring is in
  // flight before the wait for it
#pragma unroll 1
  for (int r = 0; r < kRing; ++r) issue_one(r);
  // Two CTAs fit on an SM: let the next kernel on the stream launch now, so
  // its CTAs start their own weight stream while this one finishes (its
  // griddepcontrol.wait still waits for this whole grid to complete).
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (a.pf_bytes && threadIdx.x == 0) {
    prefetch_l2_share(a.pf_ptr, a.pf_bytes, blockIdx.x, gridDim.x);
    prefetch_l2_share(a.pf_ptr2, a.pf_bytes2, blockIdx.x, gridDim.x);
  }

  asm volatile("griddepcontrol.wait;" ::: "memory");

  // ---- stage this warp's K-slice of the activation
  const int kb = a.w.K / kBlock;
  const int nblk = g.kts * 2;
  if (INF32) {
    constexpr int QB = 4;
    const int items = NB * nblk * 8;   // float4 chunks, 8 per block
    for (int base = lane; base < items; base += 32 * QB) {
      float4 v[QB];
#pragma unroll
      for (int i = 0; i < QB; ++i) {
        const int c = base + i * 32;
        const int t = c / (nblk * 8), bl = (c / 8) % nblk, p4 = c % 8;
        const int b = kt0 * 2 + bl;
        v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (c < items && t < a.B && b < kb)
          v[i] = *reinterpret_cast<const float4*>(a.xf + (size_t)t * a.w.K + b * kBlock + p4 * 4);
      }
#pragma unroll
      for (int i = 0; i < QB; ++i) {
        const int c = base + i * 32;          // 8-lane groups share (t, block)
        const int t = c / (nblk * 8), bl = (c / 8) % nblk, p4 = c % 8;
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
          uint32_t s8 = 0;
          int e = 0;
          const bool live = t < a.B && b < kb;
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
          *reinterpret_cast<uint32_t*>(act + t * slice + bl * kBlock + p4 * 4) = packed;
          if (p4 == 0) fa[t * nblk + bl] = live ? e8m0_to_float(s8) : 0.0f;
        }
      }
    }
  } else {
    for (int t = 0; t < NB; ++t) {
      for (int c = lane; c < g.kts * 4; c += 32) {
        const int k = kt0 * kTileK + c * 16;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (t < a.B && k < a.w.K) {
          v = *reinterpret_cast<const uint4*>(a.xq + (size_t)t * a.w.K + k);
          v.x ^= 0x80808080u; v.y ^= 0x80808080u; v.z ^= 0x80808080u; v.w ^= 0x80808080u;
        }
        *reinterpret_cast<uint4*>(act + t * slice + c * 16) = v;
      }
      for (int bb = lane; bb < nblk; bb += 32) {
        const int b = kt0 * 2 + bb;
        fa[t * nblk + bb] = (t < a.B && b < kb) ? e8m0_to_float(a.xs[(size_t)t * kb + b]) : 0.0f;
      }
    }
  }
  __syncwarp();

  float acc[NB];
#pragma unroll
  for (int t = 0; t < NB; ++t) acc[t] = 0.0f;
  int cgi = 0, cli = 0;                                 // compute cursor
  const int8_t* xrow = act + kto * kTileK + (WFMT == 4 ? sub * 32 : sub * 16);
  const float* frow = fa + kto * 2 + bh;

  auto compute = [&](const uint4& w, uint32_t s) {
    const int j = cli * C::KPL;                       // k-tile offset of this load (minus kto)
    float fw;
    if (FAST) fw = __int_as_float((int)((s - C::SHIFT) << 23));
    else fw = s == 255u ? __int_as_float(0x7fc00000) : pow2_exact((int)s - 127 - C::SHIFT);
    if (WFMT == 4) {
      uint32_t n[8];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t ww = k == 0 ? w.x : (k == 1 ? w.y : (k == 2 ? w.z : w.w));
        const uint32_t lo = (ww << 4) & 0xF0F0F0F0u, hi = ww & 0xF0F0F0F0u;
        n[2 * k] = __byte_perm(lo, hi, 0x5140);
        n[2 * k + 1] = __byte_perm(lo, hi, 0x7362);
      }
#pragma unroll
      for (int t = 0; t < NB; ++t) {
        const uint4* xp = reinterpret_cast<const uint4*>(xrow + t * slice + j * kTileK);
        const uint4 x0 = xp[0], x1 = xp[1];
        int d0 = __dp4a((int)x0.x, (int)n[0], 0);
        int d1 = __dp4a((int)x0.y, (int)n[1], 0);
        d0 = __dp4a((int)x0.z, (int)n[2], d0);
        d1 = __dp4a((int)x0.w, (int)n[3], d1);
        d0 = __dp4a((int)x1.x, (int)n[4], d0);
        d1 = __dp4a((int)x1.y, (int)n[5], d1);
        d0 = __dp4a((int)x1.z, (int)n[6], d0);
        d1 = __dp4a((int)x1.w, (int)n[7], d1);
        acc[t] = __fmaf_rn((float)(d0 + d1), __fmul_rn(frow[t * nblk + j * 2], fw), acc[t]);
      }
    } else {
#pragma unroll
      for (int t = 0; t < NB; ++t) {
        const uint4 x = *reinterpret_cast<const uint4*>(xrow + t * slice + j * kTileK);
        int d0 = __dp4a((int)x.x, (int)w.x, 0);
        int d1 = __dp4a((int)x.y, (int)w.y, 0);
        d0 = __dp4a((int)x.z, (int)w.z, d0);
        d1 = __dp4a((int)x.w, (int)w.w, d1);
        acc[t] = __fmaf_rn((float)(d0 + d1), __fmul_rn(frow[t * nblk + j * 2], fw), acc[t]);
      }
    }
    if (++cli == g.nload) {
      // group done: fold the lanes of each row (k-tiles x sub-slices), keep
      // the row's warp total in shared memory
#pragma unroll
      for (int t = 0; t < NB; ++t) {
#pragma unroll
        for (int o = 1; o < C::TPL; o <<= 1) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], o);
#pragma unroll
        for (int o = C::LPK; o < 32; o <<= 1) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], o);
      }
      if (kto == 0 && sub == 0)
#pragma unroll
        for (int t = 0; t < NB; ++t) part[((warp * max_ng + cgi) * 4 + rr) * NB + t] = acc[t];
#pragma unroll
      for (int t = 0; t < NB; ++t) acc[t] = 0.0f;
      cli = 0;
      ++cgi;
    }
  };

  // every lane runs the same number of steps (Q is CTA-uniform), so the
  // shuffles above are never divergent
#pragma unroll 1
  for (int q = 0; q < Q; ++q) {
    cp_async_wait<kRing - 1>();                     // round q has landed
    const int slot = q % kRing;
    uint4 w = make_uint4(0, 0, 0, 0);
    uint32_t sc = 127;
    if ((kmask >> cli) & 1u) {
      w = lds128(ring_w + (uint32_t)(slot * kThreads + tid) * 16u);
      sc = (lds32(ring_s + (uint32_t)(slot * kThreads + tid) * 4u) >> (8 * ssub)) & 0xFFu;
    }
    compute(w, sc);
    issue_one(slot);                                // refill the slot just read
  }
  cp_async_wait<0>();

  __syncthreads();
  // y = sum over the 16 warps, in warp order
  for (int e = threadIdx.x; e < ng * 4 * NB; e += kThreads) {
    const int t = e % NB, row = e / NB;          // row within this CTA's range
    const int gi = row / 4, r4 = row % 4;
    const int n = (g_lo + gi) * 4 + r4;
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s += part[((w * max_ng + gi) * 4 + r4) * NB + t];
    if (t < a.B && n < a.w.N) a.y[(size_t)t * a.w.N + n] = s;
  }
}

// ---------------------------------------------------------------------------
// Weight-resident decode GEMV (batch 1).  The ring kernel above keeps only 8
// of a CTA's ~20 rounds in flight before it must wait for its predecessor;
// the rest stream after the wait with their HBM latency exposed (timestamped
// traces of the 7B up projection: ~6.5 us of an ~8.5 us launch period were
// spent in the loop after the wait).  Here one CTA per SM holds its whole
// share in registers: every weight load (up to kResRounds 16-byte loads a
// thread, 96 registers) and the 256-byte scale blocks of the row tiles it
// touches (16-byte cp.async into shared memory) are issued before
// griddepcontrol.wait.  The activation row is then copied into shared memory
// with one round of cp.async and quantised there, and the dot products run
// from registers.  For int4 weights each 8-element group of the activation
// is stored even elements first, so a weight word's low nibbles (shifted up)
// and high nibbles (masked) are 16*w bytes that meet their activations
// without byte permutes; 4 groups share each activation load and their lanes
// are folded together by a transpose reduction.  The K range is dealt to the
// 16 warps in contiguous runs of whole loads whose lengths differ by at most
// one (the down projection's 43 loads go 3,3,...,2).
constexpr int kResRounds = 24;

struct ResGeom {
  int KT, NL, kts, G4;   // k-tiles, loads per group, k-tiles of the largest warp slice, 4-row groups
};

template <int WFMT>
__host__ __device__ __forceinline__ ResGeom res_geom(const WeightView& w) {
  using C = RCfg<WFMT>;
  ResGeom g;
  g.KT = w.Kpad / kTileK;
  g.NL = (g.KT + C::KPL - 1) / C::KPL;
  g.kts = (g.NL + kWarps - 1) / kWarps * C::KPL;
  g.G4 = (w.N + 3) / 4;
  return g;
}

template <int WFMT>
int res_rounds(const WeightView& w, int ctas) {
  const ResGeom g = res_geom<WFMT>(w);
  const int max_ng = (g.G4 + ctas - 1) / ctas;
  return (max_ng + 3) / 4 * 4 * ((g.NL + kWarps - 1) / kWarps);
}

template <int WFMT>
size_t res_smem_bytes(const WeightView& w, bool inf32, int ctas) {
  const ResGeom g = res_geom<WFMT>(w);
  const int per_warp = (g.kts * kTileK + g.kts * 2 * 4 + 15) / 16 * 16;
  const int max_ng = (g.G4 + ctas - 1) / ctas;
  const size_t xin = ((size_t)w.K * (inf32 ? 4 : 1) + 15) / 16 * 16;
  return (size_t)2 * g.KT * 256 + xin + (size_t)kWarps * per_warp + (size_t)kWarps * max_ng * 4 * 4;
}

template <int WFMT, bool FAST, bool INF32>
__global__ void __launch_bounds__(kThreads, 1) rgemv_res_kernel(GemvArgs a) {
  using C = RCfg<WFMT>;
  constexpr int GB = 4, RMAX = kResRounds;
  extern __shared__ __align__(16) uint8_t smem[];
  const ResGeom g = res_geom<WFMT>(a.w);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int G = gridDim.x;
  const int g_lo = (int)((long)blockIdx.x * g.G4 / G);
  const int ng = (int)((long)(blockIdx.x + 1) * g.G4 / G) - g_lo;
  const int nbk = (ng + GB - 1) / GB;
  const int l_lo = warp * g.NL / kWarps;
  const int nload = (warp + 1) * g.NL / kWarps - l_lo;
  const int kt0 = l_lo * C::KPL;
  const int nr = nbk * nload * GB;                       // <= RMAX (checked by the host)
  const int kto = lane / C::LPK;
  const int rr = (lane % C::LPK) / C::TPL;
  const int sub = lane % C::TPL;
  const int bh = WFMT == 4 ? sub : (sub >> 1);
  uint32_t kmask = 0;
  for (int li = 0; li < nload && li < 32; ++li)
    if (kt0 + li * C::KPL + kto < g.KT) kmask |= 1u << li;

  // shared memory: the 256-byte scale blocks [2 row tiles][KT] of the (at
  // most two) row tiles this CTA's rows touch, the activation input, then per
  // warp its quantised K-slice, then the partial sums
  const int K = a.w.K;
  const int slice = g.kts * kTileK;
  const int nblk = g.kts * 2;
  const int per_warp = (slice + nblk * 4 + 15) / 16 * 16;
  const int max_ng = (g.G4 + G - 1) / G;
  const uint32_t sc_base = smem_u32(smem);
  const int rt0 = (g_lo * 4) >> 7;                          // first row tile of this CTA
  const int nrt = (((g_lo + ng) * 4 - 1) >> 7) - rt0 + 1;   // 1 or 2 (ng * 4 <= 96 rows)
  uint8_t* xin = smem + 2 * g.KT * 256;
  const int xin_bytes = (K * (INF32 ? 4 : 1) + 15) / 16 * 16;
  int8_t* act = reinterpret_cast<int8_t*>(xin + xin_bytes + warp * per_warp);
  float* fa = reinterpret_cast<float*>(act + slice);
  float* part = reinterpret_cast<float*>(xin + xin_bytes + kWarps * per_warp);

  // ---- every weight load of this thread, before the wait
  uint4 wv[RMAX];
  uint32_t vmask = 0;                                    // rounds that were loaded
  {
    int ibi = 0, ili = 0;
#pragma unroll
    for (int r = 0; r < RMAX; ++r) {
      const int gg = r % GB;
      const int gi = ibi * GB + gg;
      wv[r] = make_uint4(0, 0, 0, 0);
      if (r < nr && gi < ng && ((kmask >> ili) & 1u)) {
        const int n = (g_lo + gi) * 4 + rr;
        const size_t rowoff = ((size_t)(n >> 7) * g.KT + kt0 + ili * C::KPL + kto) * 128 + (n & 127);
        wv[r] = ldg_stream(a.w.data + rowoff * C::TB + sub * 16);
        vmask |= 1u << r;
      }
      if (gg == GB - 1 && ++ili == nload) { ili = 0; ++ibi; }
    }
    // the scale blocks: contiguous [KT][256 B] per row tile, 16-byte copies
    const int per_rt = g.KT * 16;
    for (int c = tid; c < nrt * per_rt; c += kThreads) {
      const int part_ = c / per_rt, cc = c % per_rt;
      cp_async16(sc_base + (uint32_t)(part_ * per_rt + cc) * 16u,
                 a.w.scales + ((size_t)(rt0 + part_) * g.KT * 256 + (size_t)cc * 16));
    }
    cp_async_commit();
  }
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (a.pf_bytes && threadIdx.x == 0) {
    prefetch_l2_share(a.pf_ptr, a.pf_bytes, blockIdx.x, gridDim.x);
    prefetch_l2_share(a.pf_ptr2, a.pf_bytes2, blockIdx.x, gridDim.x);
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");

  // ---- the activation row into shared memory (one round of copies), and
  // this lane's MX block scales into registers meanwhile
  const int kb = K / kBlock;
  if (INF32) {
    for (int c = tid; c < K / 4; c += kThreads) cp_async16(smem_u32(xin) + c * 16, a.xf + c * 4);
  } else {
    for (int c = tid; c < K / 16; c += kThreads) cp_async16(smem_u32(xin) + c * 16, a.xq + c * 16);
  }
  cp_async_commit();
  float fxs[2] = {0.0f, 0.0f};
  if (!INF32) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int bb = lane + 32 * i, b = kt0 * 2 + bb;
      if (bb < nblk && b < kb) fxs[i] = e8m0_to_float(a.xs[b]);
    }
  }
  cp_async_wait<0>();
  __syncthreads();

  // ---- quantise this warp's K-slice (quantize_kernel's arithmetic)
  if (INF32) {
    const float* xf = reinterpret_cast<const float*>(xin);
    for (int c = lane; c < nblk * 8; c += 32) {            // 8-lane groups share a block
      const int bl = c / 8, p4 = c % 8;
      const int b = kt0 * 2 + bl;
      const bool live = b < kb;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (live) v = *reinterpret_cast<const float4*>(xf + b * kBlock + p4 * 4);
      const float e4[4] = {v.x, v.y, v.z, v.w};
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
      if (WFMT == 4) {   // lanes p4 = 2j, 2j+1 hold the two halves of an 8-group
        const uint32_t other = __shfl_xor_sync(0xffffffffu, packed, 1);
        packed = (p4 & 1) ? __byte_perm(other, packed, 0x7531) : __byte_perm(packed, other, 0x6420);
      }
      *reinterpret_cast<uint32_t*>(act + bl * kBlock + p4 * 4) = packed;
      if (p4 == 0) fa[bl] = live ? e8m0_to_float(s8) : 0.0f;
    }
  } else {
    for (int c = lane; c < g.kts * 4; c += 32) {
      const int k = kt0 * kTileK + c * 16;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (k < K) {
        v = *reinterpret_cast<const uint4*>(xin + k);
        v.x ^= 0x80808080u; v.y ^= 0x80808080u; v.z ^= 0x80808080u; v.w ^= 0x80808080u;
        if (WFMT == 4)
          v = make_uint4(__byte_perm(v.x, v.y, 0x6420), __byte_perm(v.x, v.y, 0x7531),
                         __byte_perm(v.z, v.w, 0x6420), __byte_perm(v.z, v.w, 0x7531));
      }
      *reinterpret_cast<uint4*>(act + c * 16) = v;
    }
#pragma unroll
    for (int i = 0; i < 2; ++i)
      if (lane + 32 * i < nblk) fa[lane + 32 * i] = fxs[i];
  }
  __syncwarp();

  // ---- dot products from registers
  const int8_t* xrow = act + kto * kTileK + (WFMT == 4 ? sub * 32 : sub * 16);
  const float* frow = fa + kto * 2 + bh;
  // lane bits that separate the lanes of one row: sub-slice bits, then the
  // k-tile bits (int4: 1, 8, 16; int8: 1, 2, 16)
  constexpr int LA = 1, LB = WFMT == 4 ? 8 : 2, LC = 16;
  const bool bA = (lane & LA) != 0, bB = (lane & LB) != 0;
  // this lane's scale byte for group gi at load li (row tile, k-tile, row, block)
  auto scale_at = [&](int gi, int li_) -> uint32_t {
    const int n = (g_lo + gi) * 4 + rr;
    const int off = (((n >> 7) - rt0) * g.KT + kt0 + li_ * C::KPL + kto) * 256 + (n & 127) * 2 + bh;
    uint32_t v;
    asm volatile("ld.shared.u8 %0, [%1];" : "=r"(v) : "r"(sc_base + (uint32_t)off));
    return v;
  };
  float acc[GB] = {0.0f, 0.0f, 0.0f, 0.0f};
  int li = 0, bi = 0;
#pragma unroll
  for (int r0 = 0; r0 < RMAX; r0 += GB) {
    if (r0 < nr) {                                       // warp-uniform
      const int j = li * C::KPL;
      // the block's 4 groups are 16 consecutive rows: when they lie in one
      // row tile their scale bytes sit 8 bytes apart from one base
      const int nb = (g_lo + bi * GB) * 4;               // first row of the block
      const bool one_tile = (nb >> 7) == ((nb + 4 * GB - 1) >> 7);
      const uint32_t sbase = sc_base + (uint32_t)((((nb >> 7) - rt0) * g.KT + kt0 + j + kto) * 256 +
                                                  ((nb & 127) + rr) * 2 + bh);
      const float fx = frow[j * 2];
      uint4 x0, x1 = make_uint4(0, 0, 0, 0);
      x0 = *reinterpret_cast<const uint4*>(xrow + j * kTileK);
      if (WFMT == 4) x1 = *reinterpret_cast<const uint4*>(xrow + j * kTileK + 16);
#pragma unroll
      for (int gg = 0; gg < GB; ++gg) {
        const int r = r0 + gg;
        uint32_t s = 127u;
        if ((vmask >> r) & 1u) {
          if (one_tile) asm volatile("ld.shared.u8 %0, [%1];" : "=r"(s) : "r"(sbase + 8u * gg));
          else s = scale_at(bi * GB + gg, li);
        }
        const uint4 w = wv[r];
        int d0, d1;
        float fw;
        if (WFMT == 4) {
          fw = FAST ? __int_as_float((int)((s - C::SHIFT) << 23))
                    : (s == 255u ? __int_as_float(0x7fc00000) : pow2_exact((int)s - 127 - C::SHIFT));
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
          fw = FAST ? __int_as_float((int)(s << 23)) : (s == 255u ? __int_as_float(0x7fc00000) : pow2_exact((int)s - 127));
          d0 = __dp4a((int)x0.x, (int)w.x, 0);
          d1 = __dp4a((int)x0.y, (int)w.y, 0);
          d0 = __dp4a((int)x0.z, (int)w.z, d0);
          d1 = __dp4a((int)x0.w, (int)w.w, d1);
        }
        acc[gg] = __fmaf_rn((float)(d0 + d1), __fmul_rn(fx, fw), acc[gg]);
      }
      if (++li == nload) {
        // fold the lanes of each row for the 4 groups at once: after the LA
        // and LB halving steps each lane holds one group
        const float s0 = bA ? acc[0] : acc[2], s1 = bA ? acc[1] : acc[3];
        float k0 = bA ? acc[2] : acc[0], k1 = bA ? acc[3] : acc[1];
        k0 += __shfl_xor_sync(0xffffffffu, s0, LA);
        k1 += __shfl_xor_sync(0xffffffffu, s1, LA);
        const float sx = bB ? k0 : k1;
        float k = bB ? k1 : k0;
        k += __shfl_xor_sync(0xffffffffu, sx, LB);
        k += __shfl_xor_sync(0xffffffffu, k, LC);
        const int gi = bi * GB + (bA ? 2 : 0) + (bB ? 1 : 0);
        if (!(lane & LC) && gi < ng) part[(warp * max_ng + gi) * 4 + rr] = k;
#pragma unroll
        for (int gg = 0; gg < GB; ++gg) acc[gg] = 0.0f;
        li = 0;
        ++bi;
      }
    }
  }
  // warps without loads (K shorter than 16 loads) still own zero partials
  if (nload == 0)
    for (int e = lane; e < ng * 4; e += 32) part[(warp * max_ng + e / 4) * 4 + e % 4] = 0.0f;

  __syncthreads();
  // y = sum over the 16 warps, in warp order
  for (int e = threadIdx.x; e < ng * 4; e += kThreads) {
    const int gi = e / 4, r4 = e % 4;
    const int n = (g_lo + gi) * 4 + r4;
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s += part[(w * max_ng + gi) * 4 + r4];
    if (n < a.w.N) a.y[n] = s;
  }
}

int g_sms = 0;

int sms() {
  if (g_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || g_sms <= 0)
      g_sms = 148;
  }
  return g_sms;
}

template <int WFMT>
size_t smem_bytes(const WeightView& w, int nb) {
  const RGeom g = rgeom<WFMT>(w);
  const int per_warp = (nb * g.kts * kTileK + nb * g.kts * 2 * 4 + 15) / 16 * 16;
  const int G = sms();
  const int max_ng = (g.G4 + G - 1) / G;
  const size_t ring = nb <= 2 ? RRing<1>::BYTES : RRing<4>::BYTES;
  return ring + (size_t)kWarps * per_warp + (size_t)kWarps * max_ng * 4 * nb * 4;
}

template <int WFMT, int NB, bool FAST, bool INF32>
cudaError_t launch_t(const GemvArgs& a, cudaStream_t st, bool pdl) {
  const size_t smem = smem_bytes<WFMT>(a.w, NB);
  if (smem > 220 * 1024) return cudaErrorInvalidValue;
  static SmemAttr smem_attr;
  if (cudaError_t e = smem_attr.ensure(rgemv_kernel<WFMT, NB, FAST, INF32>, smem)) return e;
  const int G4 = (a.w.N + 3) / 4;
  const int grid = G4 < sms() ? G4 : sms();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, rgemv_kernel<WFMT, NB, FAST, INF32>, a);
}

template <int WFMT, bool FAST, bool INF32>
cudaError_t launch_nb(const GemvArgs& a, cudaStream_t st, bool pdl) {
  switch (a.B) {
    case 1: return launch_t<WFMT, 1, FAST, INF32>(a, st, pdl);
    case 2: return launch_t<WFMT, 2, FAST, INF32>(a, st, pdl);
    case 3: return launch_t<WFMT, 3, FAST, INF32>(a, st, pdl);
    case 4: return launch_t<WFMT, 4, FAST, INF32>(a, st, pdl);
  }
  return cudaErrorInvalidValue;
}

template <int WFMT, bool INF32>
cudaError_t launch_fast(const GemvArgs& a, cudaStream_t st, bool pdl) {
  // fast scale path when every weight scale byte is in [SHIFT+1, 254]
  return a.w.scale_lo >= (WFMT == 4 ? 5 : 1) && a.w.scale_hi <= 254 ? launch_nb<WFMT, true, INF32>(a, st, pdl)
                                                                      : launch_nb<WFMT, false, INF32>(a, st, pdl);
}


template <int WFMT, bool FAST, bool INF32>
cudaError_t launch_res_t(const GemvArgs& a, cudaStream_t st, bool pdl) {
  const int G4 = (a.w.N + 3) / 4;
  const int grid = G4 < sms() ? G4 : sms();
  const size_t smem = res_smem_bytes<WFMT>(a.w, INF32, grid);
  static SmemAttr smem_attr;
  if (cudaError_t e = smem_attr.ensure(rgemv_res_kernel<WFMT, FAST, INF32>, smem)) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, rgemv_res_kernel<WFMT, FAST, INF32>, a);
}

template <int WFMT, bool INF32>
cudaError_t launch_res(const GemvArgs& a, cudaStream_t st, bool pdl) {
  return a.w.scale_lo >= (WFMT == 4 ? 5 : 1) && a.w.scale_hi <= 254 ? launch_res_t<WFMT, true, INF32>(a, st, pdl)
                                                                      : launch_res_t<WFMT, false, INF32>(a, st, pdl);
}

// The weight-resident kernel takes batch 1 when a thread's share fits its
// registers, the warp slices hold at most 64 MX blocks and everything it
// stages fits shared memory.
template <int WFMT>
bool res_ok(const WeightView& w, int B, bool inf32) {
  if (B != 1 || w.kt_ptr) return false;
  const int G4 = (w.N + 3) / 4;
  const int ctas = G4 < sms() ? G4 : sms();
  const ResGeom g = res_geom<WFMT>(w);
  return res_rounds<WFMT>(w, ctas) <= kResRounds && g.kts <= 32 &&
         res_smem_bytes<WFMT>(w, inf32, ctas) <= 200 * 1024;
}
}  // namespace

int rgemv_launches(const GemvArgs& a) {
  const bool f32 = a.xf != nullptr;
  if (cogemv_supported(a.w, a.B, f32, a.yq != nullptr)) return 1;
  const int parts = a.yq ? 0 : cogemv_row_parts(a.w, a.B, f32);
  return parts ? parts : 1;
}

bool rgemv_supported(const WeightView& w, int B) {
  if (B < 1 || B > kRgemvMaxBatch) return false;
  const size_t smem = w.fmt == 4 ? smem_bytes<4>(w, B) : smem_bytes<8>(w, B);
  return smem <= 220 * 1024;
}

cudaError_t launch_rgemv(const GemvArgs& a, cudaStream_t st, bool pdl) {
  if (!rgemv_supported(a.w, a.B) || a.rows || a.block_dots) return cudaErrorInvalidValue;
  const bool f32 = a.xf != nullptr;
  // batch 1: two launches resident per SM where the shape fits (mxq_cogemv.cu)
  if (cogemv_supported(a.w, a.B, f32, a.yq != nullptr)) return launch_cogemv(a, st, pdl);
  if (a.yq) return cudaErrorInvalidValue;
  if (const int parts = cogemv_row_parts(a.w, a.B, f32)) return launch_cogemv_rows(a, parts, st, pdl);
  if (a.w.fmt == 4 && res_ok<4>(a.w, a.B, f32)) return f32 ? launch_res<4, true>(a, st, pdl) : launch_res<4, false>(a, st, pdl);
  if (a.w.fmt == 8 && res_ok<8>(a.w, a.B, f32)) return f32 ? launch_res<8, true>(a, st, pdl) : launch_res<8, false>(a, st, pdl);
  if (a.w.fmt == 4) return f32 ? launch_fast<4, true>(a, st, pdl) : launch_fast<4, false>(a, st, pdl);
  return f32 ? launch_fast<8, true>(a, st, pdl) : launch_fast<8, false>(a, st, pdl);
}

}  // namespace mxq
