// mxq_cogemv.cu -- batch-1 decode GEMV with two consecutive launches resident
// on every SM: the HBM-bound mx_gemv of the reference
// (nn/tests/test_auto_generated.cpp:56; dpbusd design nn/user.md:17) for
// decode chains (an MLP pair, layer after layer).
//
// A weight-resident GEMV that fills an SM (one 512-thread CTA at 128
// registers) cannot start the next launch's weight stream until it exits, so
// each SM's ingest idles while the CTA computes and across the launch
// boundary.  Here a CTA is 256 threads at <= 128 registers and <= 113 KB of
// shared memory, so two fit an SM: the CTA issues every weight load of its
// share -- 24 rounds of 16 bytes a thread into registers, the rest into
// shared memory with cp.async -- and the scale bytes of its rows, and waits
// for its predecessor; the next launch is let in (griddepcontrol.
// launch_dependents) before or after the activation lands, and while this
// CTA computes, the next launch's CTA on the same SM streams its weights.
//
// Work split.  Output rows are taken in groups of 4, a contiguous balanced
// range of groups per CTA.  A quad is (block of 4 groups, warp load): the
// four rounds of a quad read the same k-tiles of four groups and share one
// activation load.  Quads are ordered block-major and dealt to the 8 warps
// in contiguous runs; a warp folds its lanes per block (after its last load
// of the block or at the end of its run) into a per-warp partial, and the
// CTA adds the 8 warps' partials of each row in warp order: no cross-CTA
// reduction, deterministic results.
//
// Arithmetic per 16-byte round (int4: one MX block of one row).  The nibble
// t in [-8, 7] is read as u = t + 8 in [0, 15] by one LOP3 ((w ^ 0x88..) &
// mask): low nibbles as u, high nibbles as 16u, so dp4a.u32.s32 needs no
// shifts; 16 * dot = 16 * sum(x u_lo) + sum(x 16 u_hi) - 128 * sum(x).  The
// block's -128 * sum(x) and the float conversion constant 1.5 * 2^23 are
// folded into the chain's start value, so 16 * d_lo + d_hi is the bit
// pattern of the float 1.5 * 2^23 + 16 * dot (exact: |16 dot| < 2^22) and one
// subtraction gives the exact integer dot as a float.  int8 weights use
// dp4a.s32.s32 with the same start value.
//
// Optional MX output (GemvArgs::yq): the CTA quantises the 32-row blocks its
// rows cover with quantize_kernel's arithmetic and writes u8 q+128 and the
// E8M0 byte, so the next linear of a pair reads MX bytes.  Blocks inside the
// CTA's rows are quantised from its own values; a block shared with
// neighbouring CTAs is quantised by the last of them to finish (each writes
// its fp32 rows, fences, and counts itself in on the block's counter; the
// one that completes the count reads the block back from L2 and resets the
// counter).
#include "mxq_internal.h"

namespace mxq {

namespace {

constexpr int kCoWarps = 8;
constexpr int kCoThreads = kCoWarps * 32;
constexpr int kCoReg = 24;                  // 16-byte weight rounds per thread in registers
constexpr size_t kCoSmemMax = 113 * 1024;   // two CTAs per SM (228 KB less 1 KB per CTA)
constexpr int kMagic = 0x4B400000;          // 1.5 * 2^23 as float bits
constexpr float kMagicF = 12582912.0f;

template <int WFMT>
struct CoCfg {
  static constexpr int TB = WFMT == 4 ? 32 : 64;   // bytes per row per k-tile
  static constexpr int TPL = TB / 16;              // lanes per row per k-tile (2 / 4)
  static constexpr int LPK = 4 * TPL;              // lanes per k-tile of a 4-row group (8 / 16)
  static constexpr int KPL = 32 / LPK;             // k-tiles per warp load (4 / 2)
  static constexpr int SHIFT = WFMT == 4 ? 4 : 0;  // int4 dots come out x16
};

// Geometry shared by host and device.
struct CoGeom {
  int KT;       // k-tiles
  int NL;       // warp loads per group (NL * KPL >= KT)
  int G4;       // 4-row groups
  int max_ng;   // most groups of one CTA
  int QW;       // most quads of one warp
  int SR;       // shared-memory weight rounds per thread
  int SS;       // scale bytes per k-tile (8 per group, 16-byte multiple)
  // shared-memory offsets (bytes)
  int off_sc, off_xin, off_act, off_fab, off_part, off_yv, off_flag, total;
};

template <int WFMT>
__host__ __device__ __forceinline__ CoGeom co_geom(const WeightView& w, int G, bool inf32, bool qout) {
  using C = CoCfg<WFMT>;
  CoGeom g;
  g.KT = w.Kpad / kTileK;
  g.NL = (g.KT + C::KPL - 1) / C::KPL;
  g.G4 = (w.N + 3) / 4;
  g.max_ng = (g.G4 + G - 1) / G;
  const int max_nq = (g.max_ng + 3) / 4 * g.NL;
  g.QW = (max_nq + kCoWarps - 1) / kCoWarps;
  g.SR = 4 * g.QW > kCoReg ? 4 * g.QW - kCoReg : 0;
  g.SS = (g.max_ng * 8 + 15) / 16 * 16;
  const int nlk = g.NL * C::KPL;                      // k-tiles an activation load can reach
  int off = g.SR * kCoThreads * 16;
  g.off_sc = off;
  off += g.KT * g.SS;
  g.off_xin = off;
  if (inf32) off += (w.K * 4 + 15) / 16 * 16;
  g.off_act = off;
  off += nlk * kTileK;
  g.off_fab = off;
  off += nlk * 2 * 8;
  g.off_part = off;
  off += (kCoWarps * g.max_ng * 4 * 4 + 15) / 16 * 16;
  g.off_yv = off;
  if (qout) off += (g.max_ng * 4 * 4 + 15) / 16 * 16;
  g.off_flag = off;
  off += 16;
  g.total = off;
  return g;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async8(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds8(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u8 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
// unsigned bytes of a times signed bytes of b, plus c
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// MX quantisation of one 32-element block held one value per lane
// (quantize_kernel's arithmetic); returns q, sets the E8M0 byte.
__device__ __forceinline__ int quant_lane(float v, uint32_t& sb) {
  const float av = fabsf(v);
  const bool nonfinite = !(av <= 3.402823466e38f);
  const bool any_nf = __any_sync(0xffffffffu, nonfinite);
  const float m = warp_max(nonfinite ? 0.0f : av, 32);
  if (any_nf) { sb = 255; return 0; }
  if (m == 0.0f) { sb = 0; return 0; }
  const int e = e8m0_exponent<127>(m);
  sb = (uint32_t)(e + 127);
  return quant_value(v, e);
}

// CTA owning 4-row group q (g_lo(c) = floor(c * G4 / G)).
__device__ __forceinline__ int owner_cta(int q, int G4, int G) {
  return (int)(((long long)(q + 1) * G - 1) / G4);
}

// --- peer mailboxes (column-sharded linears across GPUs) -----------------
// Publishes this launch's mailbox stores and sets every rank's flag: the
// peers are other GPUs (system scope), or with one rank this GPU itself.
__device__ __forceinline__ void publish_flags(const PeerArgs& p, uint32_t ep) {
  if (p.world == 1) {
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
    st_release_gpu(p.flag_out[0], ep);
  } else {
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    for (int r = 0; r < p.world; ++r) st_release_sys(p.flag_out[r], ep);
  }
}
// ROLE 0: a plain GEMV.  ROLE 1: the first linear of a column-sharded pair
// (fp32 input, MX output written into every rank's mailbox at this rank's
// rows, then this rank's flag set on every rank).  ROLE 2: the second
// linear (waits for every rank's flag, reads the full MX activation from the
// local mailbox, writes its fp32 rows into every rank's mailbox, sets flags;
// its last CTA then waits for every rank's rows and copies the whole output
// to y).
template <int WFMT, bool FAST, bool INF32, bool QOUT, int ROLE>
__global__ void __launch_bounds__(kCoThreads, 2) cogemv_kernel(GemvArgs a, PeerArgs p) {
  static_assert(ROLE == 0 || (ROLE == 1 && INF32 && QOUT) || (ROLE == 2 && !INF32 && !QOUT), "role");
  using C = CoCfg<WFMT>;
  extern __shared__ __align__(16) uint8_t smem[];
  const int G = gridDim.x;
  const CoGeom g = co_geom<WFMT>(a.w, G, INF32, QOUT);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int g_lo = (int)((long long)blockIdx.x * g.G4 / G);
  const int ng = (int)((long long)(blockIdx.x + 1) * g.G4 / G) - g_lo;
  const int nq = (ng + 3) / 4 * g.NL;
  const int q_lo = warp * nq / kCoWarps;
  const int nqw = (warp + 1) * nq / kCoWarps - q_lo;
  const int kto = lane / C::LPK;
  const int rr = (lane % C::LPK) / C::TPL;
  const int sub = lane % C::TPL;
  const int bh = WFMT == 4 ? sub : (sub >> 1);   // MX block of the lane within its k-tile
  const uint32_t sm = smem_u32(smem);
  const uint32_t w_sm = sm + (uint32_t)tid * 16u;            // slot s at + s * kCoThreads * 16
  const uint32_t sc_sm = sm + (uint32_t)g.off_sc;
  float* part = reinterpret_cast<float*>(smem + g.off_part);

  // ---- every weight round of this warp, before the wait
  uint4 wv[kCoReg];
  {
    int bi = q_lo / g.NL, li = q_lo % g.NL;
#pragma unroll
    for (int j = 0; j < kCoReg / 4; ++j) {
      const int kt = li * C::KPL + kto;
#pragma unroll
      for (int gg = 0; gg < 4; ++gg) {
        const int gi = bi * 4 + gg;
        wv[4 * j + gg] = make_uint4(0, 0, 0, 0);
        if (j < nqw && gi < ng && kt < g.KT) {
          const int n = (g_lo + gi) * 4 + rr;
          wv[4 * j + gg] = ldg_stream(a.w.data + (((size_t)(n >> 7) * g.KT + kt) * 128 + (n & 127)) * C::TB + sub * 16);
        }
      }
      if (++li == g.NL) { li = 0; ++bi; }
    }
#pragma unroll 1
    for (int j = kCoReg / 4; j < nqw; ++j) {
      const int kt = li * C::KPL + kto;
#pragma unroll
      for (int gg = 0; gg < 4; ++gg) {
        const int gi = bi * 4 + gg;
        const bool ok = gi < ng && kt < g.KT;
        const int n = (g_lo + (ok ? gi : 0)) * 4 + rr;
        const uint8_t* src = a.w.data + (((size_t)(n >> 7) * g.KT + (ok ? kt : 0)) * 128 + (n & 127)) * C::TB + sub * 16;
        // invalid rounds are zero-filled (no global read)
        cp_async16(w_sm + (uint32_t)((4 * j + gg - kCoReg) * kCoThreads * 16), src, ok ? 16u : 0u);
      }
      if (++li == g.NL) { li = 0; ++bi; }
    }
    // scale bytes of this CTA's rows: 8 bytes (4 rows x 2 blocks) per (k-tile, group)
    for (int c = tid; c < ng * g.KT; c += kCoThreads) {
      const int kt = c / ng, gi = c % ng;
      const int n = (g_lo + gi) * 4;
      cp_async8(sc_sm + (uint32_t)(kt * g.SS + gi * 8),
                a.w.scales + (((size_t)(n >> 7) * g.KT + kt) * 128 + (n & 127)) * 2);
    }
    cp_async_commit();
  }
  for (int e = tid; e < kCoWarps * g.max_ng * 4; e += kCoThreads) part[e] = 0.0f;
  // The next launch may take this SM's other slot and stream its own weights
  // while this one computes (its griddepcontrol.wait still waits for this
  // whole grid).  With a small activation (<= 8 KB) it is let in now; with a
  // larger one only once the activation has landed, so that the next
  // launch's weight requests do not queue ahead of it (measured on the 7B
  // MLP shapes: 4 KB MX rows 6.0 vs 6.4 us a launch, 11 KB MX and 16 KB fp32
  // rows 6.7 vs 6.9 and 6.9 vs 7.1 us).
  const bool early = a.w.K * (INF32 ? 4 : 1) <= 8192;
  if (early) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");

  // this call's epoch (peer roles): parity selects the mailbox half
  uint32_t ep = 0;
  const uint8_t* xq_in = a.xq;
  const uint8_t* xs_in = a.xs;
  if (ROLE != 0) {
    ep = *reinterpret_cast<volatile const uint32_t*>(p.epoch) + 1u;
    if (ROLE == 2) {
      xq_in = p.xq_base + (size_t)(ep & 1u) * p.xq_stride;
      xs_in = p.xs_base + (size_t)(ep & 1u) * p.xs_stride;
      int* okf = reinterpret_cast<int*>(smem + g.off_flag) + 2;
      if (tid == 0) okf[0] = peer_wait(p.wait_flags, p.world, ep, p.wait_ns, p.status);
      __syncthreads();
    }
  }

  // ---- the activation row
  const int K = a.w.K;
  const int kb = K / kBlock;
  const int nlk = g.NL * C::KPL;
  uint8_t* act = smem + g.off_act;
  uint2* fab = reinterpret_cast<uint2*>(smem + g.off_fab);   // per MX block: (float scale, int start value)
  if (INF32) {
    for (int c = tid; c < K / 4; c += kCoThreads) cp_async16(sm + g.off_xin + c * 16, a.xf + c * 4, 16u);
  } else {
    for (int c = tid; c < K / 16; c += kCoThreads) cp_async16(sm + g.off_act + c * 16, xq_in + c * 16, 16u);
  }
  cp_async_commit();
  // MX input: the scale bytes of the (at most kXsRegs) blocks this thread
  // converts below, loaded while the copies fly
  constexpr int kXsRegs = 4;
  uint32_t xsr[kXsRegs] = {0u, 0u, 0u, 0u};
  if (!INF32) {
#pragma unroll
    for (int k = 0; k < kXsRegs; ++k) {
      const int c = tid + k * kCoThreads, blk = c >> 1;
      if (!(c & 1) && blk < kb) xsr[k] = __ldcg(xs_in + blk);
    }
  }
  cp_async_wait_all();
  __syncthreads();
  if (!early) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (INF32) {
    // 8 lanes per block, 4 values a lane (quantize_kernel's arithmetic)
    const float* xf = reinterpret_cast<const float*>(smem + g.off_xin);
    const int p4 = lane & 7;
    for (int blk = warp * 4 + (lane >> 3); blk - (lane >> 3) < nlk * 2; blk += kCoWarps * 4) {
      const bool in = blk < nlk * 2;
      const bool live = blk < kb;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (live) v = *reinterpret_cast<const float4*>(xf + blk * kBlock + p4 * 4);
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
      int qs = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int q = (s8 != 0 && s8 != 255) ? quant_value(e4[k], e) : 0;
        qs += q;
        packed |= ((uint32_t)q & 0xFFu) << (8 * k);
      }
      if (WFMT == 4) {   // lanes p4 = 2j, 2j+1 hold the two halves of an 8-group
        const uint32_t other = __shfl_xor_sync(0xffffffffu, packed, 1);
        packed = (p4 & 1) ? __byte_perm(other, packed, 0x7531) : __byte_perm(packed, other, 0x6420);
      }
#pragma unroll
      for (int o = 4; o > 0; o >>= 1) qs += __shfl_xor_sync(0xffffffffu, qs, o);
      if (in) {
        *reinterpret_cast<uint32_t*>(act + blk * kBlock + p4 * 4) = packed;
        if (p4 == 0)
          fab[blk] = make_uint2(__float_as_uint(live ? e8m0_to_float(s8) : 0.0f),
                                (uint32_t)(kMagic - (WFMT == 4 ? 128 * qs : 0)));
      }
    }
  } else {
    // MX bytes: to signed (and int4 even-first order) in place; 16 bytes a
    // thread, the two threads of a block add their sums
    auto conv = [&](int k, uint32_t sb_pre, bool pre) {
      const int c = tid + k * kCoThreads;
      const bool in = c < nlk * 4;   // every lane takes the shuffle below
      uint4 v = make_uint4(0, 0, 0, 0);
      if (c * 16 < K) {
        v = *reinterpret_cast<const uint4*>(act + c * 16);
        v.x ^= 0x80808080u; v.y ^= 0x80808080u; v.z ^= 0x80808080u; v.w ^= 0x80808080u;
      }
      int qs = dp4a_ss(v.x, 0x01010101u, 0);
      qs = dp4a_ss(v.y, 0x01010101u, qs);
      qs = dp4a_ss(v.z, 0x01010101u, qs);
      qs = dp4a_ss(v.w, 0x01010101u, qs);
      if (WFMT == 4)
        v = make_uint4(__byte_perm(v.x, v.y, 0x6420), __byte_perm(v.x, v.y, 0x7531),
                       __byte_perm(v.z, v.w, 0x6420), __byte_perm(v.z, v.w, 0x7531));
      if (in) *reinterpret_cast<uint4*>(act + c * 16) = v;
      qs += __shfl_xor_sync(0xffffffffu, qs, 1);   // chunks c and c ^ 1 are lanes l and l ^ 1
      if (in && !(c & 1)) {
        const int blk = c >> 1;
        const uint32_t sb = pre ? sb_pre : (blk < kb ? (uint32_t)__ldcg(xs_in + blk) : 0u);
        fab[blk] = make_uint2(__float_as_uint(blk < kb ? e8m0_to_float(sb) : 0.0f),
                              (uint32_t)(kMagic - (WFMT == 4 ? 128 * qs : 0)));
      }
    };
#pragma unroll
    for (int k = 0; k < kXsRegs; ++k)
      if ((tid - lane) + k * kCoThreads < nlk * 4) conv(k, xsr[k], true);   // warp-uniform
#pragma unroll 1
    for (int k = kXsRegs; (tid - lane) + k * kCoThreads < nlk * 4; ++k) conv(k, 0u, false);
  }
  __syncthreads();

  // ---- dot products: register quads, then shared-memory quads
  const uint32_t act_lane = sm + (uint32_t)(g.off_act + kto * kTileK + (WFMT == 4 ? sub * 32 : sub * 16));
  const uint32_t fab_lane = sm + (uint32_t)(g.off_fab + (kto * 2 + bh) * 8);
  const uint32_t sc_lane = sc_sm + (uint32_t)(kto * g.SS + rr * 2 + bh);
  constexpr int LA = 1, LB = WFMT == 4 ? 8 : 2, LC = 16;
  const bool bA = (lane & LA) != 0, bB = (lane & LB) != 0;
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  int bi = q_lo / g.NL, li = q_lo % g.NL;

  auto fold = [&]() {
    // lanes of one row differ in bits LA, LB, LC; after the LA and LB halving
    // steps each lane holds one group of the block
    const float s0 = bA ? acc[0] : acc[2], s1 = bA ? acc[1] : acc[3];
    float k0 = bA ? acc[2] : acc[0], k1 = bA ? acc[3] : acc[1];
    k0 += __shfl_xor_sync(0xffffffffu, s0, LA);
    k1 += __shfl_xor_sync(0xffffffffu, s1, LA);
    const float sx = bB ? k0 : k1;
    float k = bB ? k1 : k0;
    k += __shfl_xor_sync(0xffffffffu, sx, LB);
    k += __shfl_xor_sync(0xffffffffu, k, LC);
    const int gi = bi * 4 + (bA ? 2 : 0) + (bB ? 1 : 0);
    if (!(lane & LC) && gi < ng) part[(warp * g.max_ng + gi) * 4 + rr] = k;
#pragma unroll
    for (int gg = 0; gg < 4; ++gg) acc[gg] = 0.0f;
  };

  auto quad = [&](const uint4 (&w)[4]) {
    const int kt = li * C::KPL + kto;
    const bool kok = kt < g.KT;
    const uint32_t koff = (uint32_t)(li * C::KPL);
    const uint4 x0 = lds128(act_lane + koff * kTileK);
    uint4 x1 = make_uint4(0, 0, 0, 0);
    if (WFMT == 4) x1 = lds128(act_lane + koff * kTileK + 16);
    const uint2 fb = lds64(fab_lane + koff * 16);
    const float fx = __uint_as_float(fb.x);
    const int start = (int)fb.y;
    const uint32_t sq = sc_lane + koff * (uint32_t)g.SS + (uint32_t)(bi * 32);
#pragma unroll
    for (int gg = 0; gg < 4; ++gg) {
      const bool ok = kok && bi * 4 + gg < ng;
      const uint32_t s = ok ? lds8(sq + gg * 8) : 127u;
      float fw;
      if (FAST) fw = __int_as_float((int)((s - C::SHIFT) << 23));
      else fw = s == 255u ? __int_as_float(0x7fc00000) : pow2_exact((int)s - 127 - C::SHIFT);
      int r;
      if (WFMT == 4) {
        const uint32_t o = 0x88888888u, ml = 0x0F0F0F0Fu, mh = 0xF0F0F0F0u;
        int d0 = dp4a_us((w[gg].x ^ o) & ml, x0.x, 0);
        int d1 = dp4a_us((w[gg].x ^ o) & mh, x0.y, start);
        d0 = dp4a_us((w[gg].y ^ o) & ml, x0.z, d0);
        d1 = dp4a_us((w[gg].y ^ o) & mh, x0.w, d1);
        d0 = dp4a_us((w[gg].z ^ o) & ml, x1.x, d0);
        d1 = dp4a_us((w[gg].z ^ o) & mh, x1.y, d1);
        d0 = dp4a_us((w[gg].w ^ o) & ml, x1.z, d0);
        d1 = dp4a_us((w[gg].w ^ o) & mh, x1.w, d1);
        r = d0 * 16 + d1;
      } else {
        int d0 = dp4a_ss(x0.x, w[gg].x, 0);
        int d1 = dp4a_ss(x0.y, w[gg].y, start);
        d0 = dp4a_ss(x0.z, w[gg].z, d0);
        d1 = dp4a_ss(x0.w, w[gg].w, d1);
        r = d0 + d1;
      }
      acc[gg] = __fmaf_rn(__fsub_rn(__int_as_float(r), kMagicF), __fmul_rn(fx, fw), acc[gg]);
    }
    if (++li == g.NL) {
      fold();
      li = 0;
      ++bi;
    }
  };

#pragma unroll
  for (int j = 0; j < kCoReg / 4; ++j) {
    if (j < nqw) {   // warp-uniform
      const uint4 w4[4] = {wv[4 * j], wv[4 * j + 1], wv[4 * j + 2], wv[4 * j + 3]};
      quad(w4);
    }
  }
#pragma unroll 1
  for (int j = kCoReg / 4; j < nqw; ++j) {
    const uint32_t base = w_sm + (uint32_t)((4 * j - kCoReg) * kCoThreads * 16);
    const uint4 w4[4] = {lds128(base), lds128(base + kCoThreads * 16), lds128(base + 2 * kCoThreads * 16),
                         lds128(base + 3 * kCoThreads * 16)};
    quad(w4);
  }
  if (nqw > 0 && li != 0) fold();   // the run ended inside a block

  __syncthreads();
  // y = sum over the 8 warps, in warp order
  const int N = a.w.N;
  float* yv = reinterpret_cast<float*>(smem + g.off_yv);
  for (int e = tid; e < ng * 4; e += kCoThreads) {
    const int n = g_lo * 4 + e;
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < kCoWarps; ++w) s += part[w * g.max_ng * 4 + e];
    if (n < N) {
      if (ROLE == 2) {
        const size_t o = (size_t)(ep & 1u) * p.f_stride + p.row_off + n;
        for (int r = 0; r < p.world; ++r) p.f_out[r][o] = s;
      } else {
        a.y[n] = s;
      }
    }
    if (QOUT) yv[e] = s;
  }
  // MX bytes out: local, or (ROLE 1) into every rank's mailbox at this rank's rows
  auto put_q = [&](int i, uint8_t v) {
    if (ROLE == 1) {
      const size_t o = (size_t)(ep & 1u) * p.q_stride + p.row_off + i;
      for (int r = 0; r < p.world; ++r) p.q_out[r][o] = v;
    } else {
      a.yq[i] = v;
    }
  };
  auto put_s = [&](int b, uint8_t v) {
    if (ROLE == 1) {
      const size_t o = (size_t)(ep & 1u) * p.s_stride + p.row_off / kBlock + b;
      for (int r = 0; r < p.world; ++r) p.s_out[r][o] = v;
    } else {
      a.ys[b] = v;
    }
  };
  const int R0 = g_lo * 4, R1 = min((g_lo + ng) * 4, N);
  if (QOUT && R1 > R0) {
    // MX bytes of the 32-row blocks this CTA's rows touch (N is a multiple of 32)
    const int b0 = R0 / kBlock, b1 = (R1 - 1) / kBlock;
    __syncthreads();   // every row of y written by this CTA ...
    int* flag = reinterpret_cast<int*>(smem + g.off_flag);
    if (tid < 2) {
      __threadfence();   // ... is visible GPU-wide before the CTA counts itself in
      const int b = tid == 0 ? b0 : b1;
      const bool shared_blk = b * kBlock < R0 || b * kBlock + kBlock > R1;
      int last = 0;
      if (shared_blk && (tid == 0 || b1 != b0)) {
        const int c_first = owner_cta(b * kBlock / 4, g.G4, G);
        const int c_last = owner_cta((b * kBlock + kBlock - 1) / 4, g.G4, G);
        const unsigned old = atomicAdd(&a.ycnt[b], 1u);
        last = old == (unsigned)(c_last - c_first);
      }
      flag[tid] = last;
    }
    __syncthreads();
    for (int b = b0 + warp; b <= b1; b += kCoWarps) {
      const bool inside = b * kBlock >= R0 && b * kBlock + kBlock <= R1;
      const bool mine = inside || (b == b0 && flag[0]) || (b == b1 && b1 != b0 && flag[1]);
      if (!mine) continue;   // warp-uniform
      float v;
      if (inside) {
        v = yv[b * kBlock - R0 + lane];
      } else {
        __threadfence();
        v = __ldcg(a.y + b * kBlock + lane);
      }
      uint32_t sb = 0;
      const int q = quant_lane(v, sb);
      put_q(b * kBlock + lane, (uint8_t)(q + 128));
      if (lane == 0) {
        put_s(b, (uint8_t)sb);
        if (!inside) a.ycnt[b] = 0u;   // every contributor has counted itself in
      }
    }
  }
  if (ROLE != 0) {
    // the last CTA of the grid to finish publishes this rank's rows: the CTA
    // barrier orders every thread's mailbox stores before thread 0's
    // GPU-scope fence and count; the last CTA's one release at system scope
    // is cumulative over every store it has observed through the counts, so
    // the peers see all of them before the flag
    int* lastf = reinterpret_cast<int*>(smem + g.off_flag) + 3;
    __syncthreads();
    if (tid == 0) {
      __threadfence();
      const unsigned old = atomicAdd(p.grid_cnt, 1u);
      const int last = old == (unsigned)G - 1u;
      if (last) {
        *p.grid_cnt = 0u;
        publish_flags(p, ep);
      }
      *lastf = last;
    }
    if (ROLE == 2) {
      // the same CTA then waits for every rank's rows, copies the whole
      // output out of the local mailbox and advances the epoch
      __syncthreads();
      if (*lastf) {   // CTA-uniform
        int* okf = reinterpret_cast<int*>(smem + g.off_flag) + 2;
        if (tid == 0) okf[0] = peer_wait(p.done_flags, p.world, ep, p.wait_ns, p.status);
        __syncthreads();
        const float* src = p.f_in + (size_t)(ep & 1u) * p.f_in_stride;
        for (int i = tid; i < p.n_out; i += kCoThreads) a.y[i] = __ldcg(src + i);
        __syncthreads();
        if (tid == 0) *p.epoch = ep;
      }
    }
  }
}

int co_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  }
  return n;
}

template <int WFMT, bool FAST, bool INF32, bool QOUT, int ROLE>
struct CoKernel {
  static cudaError_t prepare(size_t smem) {
    static SmemAttr attr;
    static bool carve[SmemAttr::kMaxDevices] = {};
    auto fn = cogemv_kernel<WFMT, FAST, INF32, QOUT, ROLE>;
    if (cudaError_t e = attr.ensure(fn, smem)) return e;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= SmemAttr::kMaxDevices) dev = 0;
    if (!carve[dev]) {
      // two CTAs of up to 113 KB share an SM: the largest shared carveout
      if (cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout,
                                               (int)cudaSharedmemCarveoutMaxShared))
        return e;
      carve[dev] = true;
    }
    return cudaSuccess;
  }
  static cudaError_t launch(const GemvArgs& a, const PeerArgs& pa, cudaStream_t st, bool pdl) {
    const int G4 = (a.w.N + 3) / 4;
    const int grid = G4 < co_sms() ? G4 : co_sms();
    const CoGeom g = co_geom<WFMT>(a.w, grid, INF32, QOUT);
    if (cudaError_t e = prepare((size_t)g.total)) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kCoThreads);
    cfg.dynamicSmemBytes = (size_t)g.total;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, cogemv_kernel<WFMT, FAST, INF32, QOUT, ROLE>, a, pa);
  }
};

template <int WFMT, bool INF32, bool QOUT, int ROLE = 0>
cudaError_t launch_co_fast(const GemvArgs& a, cudaStream_t st, bool pdl, const PeerArgs& pa = PeerArgs{}) {
  const bool fast = a.w.scale_lo >= (WFMT == 4 ? 5 : 1) && a.w.scale_hi <= 254;
  return fast ? CoKernel<WFMT, true, INF32, QOUT, ROLE>::launch(a, pa, st, pdl)
              : CoKernel<WFMT, false, INF32, QOUT, ROLE>::launch(a, pa, st, pdl);
}

template <int WFMT>
cudaError_t launch_co_t(const GemvArgs& a, cudaStream_t st, bool pdl) {
  const bool f32 = a.xf != nullptr, q = a.yq != nullptr;
  if (f32) return q ? launch_co_fast<WFMT, true, true>(a, st, pdl) : launch_co_fast<WFMT, true, false>(a, st, pdl);
  return q ? launch_co_fast<WFMT, false, true>(a, st, pdl) : launch_co_fast<WFMT, false, false>(a, st, pdl);
}

}  // namespace

bool cogemv_supported(const WeightView& w, int B, bool inf32, bool qout) {
  if (B != 1 || w.kt_ptr || w.N <= 0 || w.K <= 0) return false;
  if (qout && w.N % kBlock) return false;
  const int G4 = (w.N + 3) / 4;
  const int grid = G4 < co_sms() ? G4 : co_sms();
  const size_t total = w.fmt == 4 ? (size_t)co_geom<4>(w, grid, inf32, qout).total
                                  : (size_t)co_geom<8>(w, grid, inf32, qout).total;
  return total <= kCoSmemMax;
}

cudaError_t launch_cogemv(const GemvArgs& a, cudaStream_t st, bool pdl) {
  if (!cogemv_supported(a.w, a.B, a.xf != nullptr, a.yq != nullptr) || a.rows || a.block_dots)
    return cudaErrorInvalidValue;
  if (a.yq && (!a.ys || !a.ycnt)) return cudaErrorInvalidValue;
  return a.w.fmt == 4 ? launch_co_t<4>(a, st, pdl) : launch_co_t<8>(a, st, pdl);
}

// Rows [rt0 * 128, rt0 * 128 + n) of a dense weight as a weight of its own:
// the tiled layout keeps each 128-row tile's k-tiles together, so a slice at
// tile boundaries is a pointer offset.
static WeightView row_slice(const WeightView& w, int rt0, int n) {
  WeightView v = w;
  const size_t kt = (size_t)w.Kpad / kTileK;
  v.data = w.data + (size_t)rt0 * kt * 128 * (w.fmt == 4 ? 32 : 64);
  v.scales = w.scales + (size_t)rt0 * kt * 128 * 2;
  v.N = n;
  v.Npad = (n + 127) / 128 * 128;
  return v;
}

int cogemv_row_parts(const WeightView& w, int B, bool inf32) {
  if (B != 1 || w.kt_ptr || cogemv_supported(w, B, inf32, false)) return 0;
  const int tiles = (w.N + 127) / 128;
  for (int parts = 2; parts <= 8 && parts <= tiles; ++parts) {
    const int per = (tiles + parts - 1) / parts;
    if (cogemv_supported(row_slice(w, 0, per * 128 < w.N ? per * 128 : w.N), 1, inf32, false)) return parts;
  }
  return 0;
}

cudaError_t launch_cogemv_rows(const GemvArgs& a, int parts, cudaStream_t st, bool pdl) {
  if (parts < 2 || a.yq || a.rows || a.block_dots || a.B != 1) return cudaErrorInvalidValue;
  const int tiles = (a.w.N + 127) / 128;
  const int per = (tiles + parts - 1) / parts;
  for (int rt = 0; rt < tiles; rt += per) {
    const int n = ((rt + per) * 128 < a.w.N ? (rt + per) * 128 : a.w.N) - rt * 128;
    GemvArgs p = a;
    p.w = row_slice(a.w, rt, n);
    p.y = a.y + (size_t)rt * 128;
    if (!cogemv_supported(p.w, 1, a.xf != nullptr, false)) return cudaErrorInvalidValue;
    if (cudaError_t e = p.w.fmt == 4 ? launch_co_t<4>(p, st, pdl) : launch_co_t<8>(p, st, pdl)) return e;
  }
  return cudaSuccess;
}

cudaError_t launch_cogemv_peer(const GemvArgs& a, const PeerArgs& pa, int role, cudaStream_t st, bool pdl) {
  if (pa.world < 1 || pa.world > kMaxPeers || !pa.epoch || !pa.grid_cnt) return cudaErrorInvalidValue;
  if (role == 1) {
    if (!a.xf || !a.yq || !a.ys || !a.ycnt || !a.y || !cogemv_supported(a.w, 1, true, true)) return cudaErrorInvalidValue;
    return a.w.fmt == 4 ? launch_co_fast<4, true, true, 1>(a, st, pdl, pa) : launch_co_fast<8, true, true, 1>(a, st, pdl, pa);
  }
  if (role == 2) {
    if (a.xf || a.yq || !a.y || !pa.wait_flags || !pa.done_flags || !pa.xq_base || !pa.f_in || pa.n_out <= 0 ||
        !cogemv_supported(a.w, 1, false, false))
      return cudaErrorInvalidValue;
    return a.w.fmt == 4 ? launch_co_fast<4, false, false, 2>(a, st, pdl, pa)
                        : launch_co_fast<8, false, false, 2>(a, st, pdl, pa);
  }
  return cudaErrorInvalidValue;
}

}  // namespace mxq
