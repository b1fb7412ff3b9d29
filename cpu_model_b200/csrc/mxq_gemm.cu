// mxq_gemm.cu -- tensor-core MX GEMM for the prefill / rollout / MoE regime
// (batch > 4): the batched mx_gemv of the reference
// (nn/tests/test_auto_generated.cpp:56), on tcgen05 with TMEM accumulators.
//
// Why bf16 operands on kind::f16 rather than kind::i8: the MX contract scales
// every 32-element K block by its own 2^(e_x + e_w), different per (row,
// block) and per (token, block).  With kind::i8 each K=32 MMA would need its
// own int32 accumulator drained through tcgen05.ld and scaled on CUDA cores:
// one convert + one FMA per output per 32 MACs, which at 8k int8 MAC/clk/SM
// against 128 FP32 lanes/clk/SM caps the tensor pipe near a quarter of its
// rate.  Instead both operands are pre-scaled exactly: q_x * 2^e_x and
// q_w * 2^e_w are exact in bf16 (7-bit magnitudes), every product is exact in
// fp32, and the tensor core's fp32 accumulation applies the block scales for
// free.  The per-block int32 dots remain available bit-exactly through the
// GEMV's dp4a path (mxq_block_dots).
//
// Orientation: the UMMA M dimension (128 TMEM lanes) is the weight rows,
// N is the token tile (16..256), so one kernel spans small and large batches.
// Grid: (row tiles, token tiles, K splits).  When the row tiles alone leave
// SMs idle (the 4096-row down projection has 32 of them on 148 SMs) the K
// range is split over a thread-block cluster of S CTAs; each CTA parks its
// fp32 partial tile in its own shared memory and, after a cluster barrier,
// sums one slice of the tile over all S partials in rank order through
// distributed shared memory (deterministic, no global workspace).
//
// Warp roles (4 role warps + kConvWarps converter warps):
//   warp 0      raw producer: 1-D bulk copies of packed weight tiles + scales
//               (int4: 4 KB + 256 B per 128x64 tile) into the raw ring;
//   warp 1      TMEM owner and single-thread MMA issuer (4 x K=16 per tile);
//   warp 2      operand producer: bulk copy of the pre-swizzled bf16
//               activation tile (BN x 128 B) into the operand ring;
//   warps 4..   converters: unpack int4/int8 -> bf16, apply 2^e_w, write the
//               128B-swizzled K-major tile, fence to the async proxy; then
//               the epilogue (tcgen05.ld -> fp32 stores, coalesced by row,
//               or -> the shared partial tile when K is split).
// Every mbarrier wait is bounded; a wait that gives up sets the status word.
// Every thread reaches both cluster barriers whatever happened before.
#include "mxq_internal.h"

namespace mxq {

namespace {

constexpr int kRoleWarps = 4;
constexpr int kConvWarps = 16;
constexpr int kGemmThreads = (kRoleWarps + kConvWarps) * 32;
constexpr int kMaxSplits = 8;   // portable cluster size

// Three rings.  raw: packed weight tiles + scales streamed from HBM (sized
// to cover HBM latency at the k-tile rate); w: converted bf16 weight tiles
// (on-chip hand-off to the MMA); x: bf16 activation tiles (mostly L2 hits
// shared by every row tile; deep, so their latency stays hidden).
// The converter warps form NG groups; group g converts k-tiles i = g mod NG,
// so NG tiles are in conversion at once (one tile's convert -> fence ->
// hand-off chain is latency-bound).  RS and WS are multiples of NG: every
// ring stage is then always refilled by the same group, in order, which keeps
// the mbarrier parity waits unambiguous.
// MT = 1 or 2 weight row tiles (128 rows each) per CTA: with MT = 2 every
// activation tile feeds twice the weight rows, halving the operand traffic
// per MMA (the per-SM copy engine, not HBM or the tensor pipe, bounds the
// kernel).  The NG converter groups split as MT row tiles x GPR k-phases;
// each group keeps its own accumulator.
template <int WFMT, int BN, int MT>
struct Cfg {
  static constexpr int NG = BN <= 64 ? 4 : 2;
  static constexpr int GW = kConvWarps / NG;             // warps per group
  static constexpr int GT = GW * 32;
  static constexpr int GPR = NG / MT;                    // groups per row tile
  static constexpr int KPS = MT == 1 ? NG : (WFMT == 8 ? 2 : 4);   // k-tiles per chunk and row tile
  static constexpr int TPG = KPS / GPR;                  // k-tiles per group per chunk
  static constexpr int WSG = (MT == 2 && NG == 2) ? 2 : 1;         // weight stages per group
  static constexpr int TB = WFMT == 4 ? 32 : 64;
  static constexpr int RAW_W = 128 * TB;                 // packed weights of one k-tile
  static constexpr int RAW_CHUNK = MT * KPS * RAW_W;     // [MT][KPS][RAW_W]; scales read per thread
  static constexpr int RAW_TARGET = MT == 2 ? 64 * 1024
                                  : (WFMT == 8 ? (BN <= 64 ? 68 * 1024 : 34 * 1024)
                                               : (BN <= 64 ? 48 * 1024 : (BN <= 128 ? 40 * 1024 : 26 * 1024)));
  static constexpr int RSC = RAW_TARGET / RAW_CHUNK < 2 ? 2 : RAW_TARGET / RAW_CHUNK;
  static constexpr int W_TILE = 128 * 128;
  static constexpr int WS = NG * WSG;
  static constexpr int X_TILE = BN * 128;
  // activation chunks of XK k-tiles, about 32 KB per copy
  static constexpr int XK = X_TILE >= 32768 ? 1 : 32768 / X_TILE;
  static constexpr int X_CHUNK = XK * X_TILE;
  static constexpr int BUDGET = 222 * 1024;
  static constexpr int XS_FIT = (BUDGET - 2048 - RSC * RAW_CHUNK - WS * W_TILE) / X_CHUNK;
  static constexpr int XSC = XS_FIT > 8 ? 8 : XS_FIT;
  // one accumulator of BN columns per group
  static constexpr int ACC_COLS = NG * BN;
  static constexpr int TMEM_COLS = ACC_COLS <= 32 ? 32 : (ACC_COLS <= 64 ? 64 : (ACC_COLS <= 128 ? 128 : (ACC_COLS <= 256 ? 256 : 512)));
  static constexpr size_t OP_BYTES = (size_t)WS * W_TILE + (size_t)XSC * X_CHUNK;
  static constexpr size_t SMEM = 1024 + OP_BYTES + (size_t)RSC * RAW_CHUNK + 1024;
  // converter work per k-tile: 32-bit words of packed weights per thread,
  // and the 16-byte bf16 chunks they become
  static constexpr int WORDS = 128 * TB / 4 / GT;
  static constexpr int NCH = WFMT == 4 ? WORDS : WORDS / 2;
  static_assert(MT == 1 || MT == 2, "row tiles per CTA");
  static_assert(NG % MT == 0 && KPS % GPR == 0, "group split");
  // parity safety: any XSC consecutive activation chunks hold a tile of every group
  static_assert(XSC >= 2 && XSC * XK >= GPR, "activation ring");
  static_assert(ACC_COLS <= 512, "tensor memory");
  static_assert(SMEM <= 227 * 1024, "shared memory");
  // mbarriers (raw, activation, weight stages, accumulator, MMA drains) + TMEM slot
  static_assert((2 * RSC + 2 * XSC + WS + 1 + NG) * 8 + 4 <= 1024, "barrier area");
  static_assert(WORDS == 4 || WORDS == 8 || WORDS == 16, "converter split");
  // the split-K partial tile [BN][128] fp32 (one row tile at a time) reuses the w and x rings
  static_assert((size_t)BN * 128 * 4 <= OP_BYTES, "partial tile");
};

// 2^(s - 127 - shift) as a bf16 pair (subnormals down to 2^-133, zero
// below; NaN for scale 0xFF).
__device__ __forceinline__ uint32_t bf16x2_scale(uint32_t s, int shift) {
  const int n = (int)s - 127 - shift;
  const uint32_t h = s == 255u ? 0x7FC0u
                   : n >= -126 ? (uint32_t)(n + 127) << 7
                   : n >= -133 ? 1u << (n + 133) : 0u;
  return h | (h << 16);
}

// 2^(s - 127 - shift) as fp32 (NaN for scale 0xFF).
__device__ __forceinline__ float f32_scale(uint32_t s, int shift) {
  return s == 255u ? __int_as_float(0x7fc00000) : pow2_exact((int)s - 127 - shift);
}

// int4: 8 nibbles -> four bf16x2 (slot order e0,e2,e4,e6,e1,e3,e5,e7),
// each w * 2^e exactly.  PRMT builds bf16 128 + (w + 8) (exponent byte 0x43);
// FUSED: one fma v*s - 136*s (exact: both products are exact and so is the
// result; needs 136*s finite in bf16, i.e. scale byte <= 246); otherwise
// (v - 136) * s in two steps.
template <bool FUSED>
__device__ __forceinline__ uint4 cvt_int4_word(uint32_t w, __nv_bfloat162 sc, __nv_bfloat162 nb) {
  const uint32_t lo = (w ^ 0x88888888u) & 0x0F0F0F0Fu;
  const uint32_t hi = ((w >> 4) ^ 0x08888888u) & 0x0F0F0F0Fu;
  const uint32_t C = 0x43434343u;
  uint32_t p[4] = {__byte_perm(lo, C, 0x4140), __byte_perm(lo, C, 0x4342),
                   __byte_perm(hi, C, 0x4140), __byte_perm(hi, C, 0x4342)};
  uint4 r;
  uint32_t* rr = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&p[i]);
    if (FUSED) {
      v = __hfma2(v, sc, nb);
    } else {
      v = __hmul2(__hsub2(v, nb), sc);
    }
    rr[i] = *reinterpret_cast<uint32_t*>(&v);
  }
  return r;
}

// int8: 4 signed bytes -> two bf16x2 in natural order, w * 2^e exactly.
// PRMT builds the fp32 2^23 + (w + 128); FUSED: fma(v, s, -(2^23+128)*s)
// (exact; needs that product finite, scale byte <= 231).
template <bool FUSED>
__device__ __forceinline__ uint2 cvt_int8_word(uint32_t w, float sc, float nb) {
  const uint32_t wx = w ^ 0x80808080u;
  const uint32_t M = 0x4B000000u;
  float f[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float v = __uint_as_float(__byte_perm(wx, M, 0x7540 + i));
    f[i] = FUSED ? __fmaf_rn(v, sc, nb) : __fmul_rn(__fsub_rn(v, 8388736.0f), sc);
  }
  __nv_bfloat162 a = __floats2bfloat162_rn(f[0], f[1]);
  __nv_bfloat162 b = __floats2bfloat162_rn(f[2], f[3]);
  return make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
}

// One thread's share of one 128x64 k-tile, converted into registers: WORDS
// consecutive 32-bit words of one row (int4: 4 words per 32-element scale
// block; int8: 8), giving NCH 16-byte bf16 chunks starting at chunk c0 of the
// row (int4: word i -> chunk i; int8: words 2j, 2j+1 -> chunk j).
template <int WFMT, int WORDS, int NCH, bool FUSED>
__device__ __forceinline__ void convert_share(const uint8_t* raw, uint32_t sc2, int row, int w0,
                                              int shift, uint4 (&out)[NCH]) {
  if (WFMT == 4) {
#pragma unroll
    for (int q = 0; q < WORDS; q += 4) {
      const uint32_t sb = bf16x2_scale((sc2 >> (8 * ((w0 + q) >> 2))) & 0xFFu, shift);
      const __nv_bfloat162 sc = *reinterpret_cast<const __nv_bfloat162*>(&sb);
      const __nv_bfloat162 nb = FUSED ? __hmul2(__floats2bfloat162_rn(-136.0f, -136.0f), sc)
                                      : __floats2bfloat162_rn(136.0f, 136.0f);
      const uint4 v = *reinterpret_cast<const uint4*>(raw + row * 32 + (w0 + q) * 4);
      out[q + 0] = cvt_int4_word<FUSED>(v.x, sc, nb);
      out[q + 1] = cvt_int4_word<FUSED>(v.y, sc, nb);
      out[q + 2] = cvt_int4_word<FUSED>(v.z, sc, nb);
      out[q + 3] = cvt_int4_word<FUSED>(v.w, sc, nb);
    }
  } else {
#pragma unroll
    for (int q = 0; q < WORDS; q += 4) {
      const float sc = f32_scale((sc2 >> (8 * ((w0 + q) >> 3))) & 0xFFu, shift);
      const float nb = FUSED ? -8388736.0f * sc : 0.0f;
      const uint4 v = *reinterpret_cast<const uint4*>(raw + row * 64 + (w0 + q) * 4);
      const uint2 c0 = cvt_int8_word<FUSED>(v.x, sc, nb), c1 = cvt_int8_word<FUSED>(v.y, sc, nb);
      const uint2 c2 = cvt_int8_word<FUSED>(v.z, sc, nb), c3 = cvt_int8_word<FUSED>(v.w, sc, nb);
      out[q / 2 + 0] = make_uint4(c0.x, c0.y, c1.x, c1.y);
      out[q / 2 + 1] = make_uint4(c2.x, c2.y, c3.x, c3.y);
    }
  }
}

__device__ __forceinline__ uint32_t ldg_u16(const uint16_t* p) {
  unsigned short v;
  asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

template <int WFMT, int BN, int MT>
__global__ void __launch_bounds__(kGemmThreads, 1) gemm_tc_kernel(GemmArgs a) {
  using C = Cfg<WFMT, BN, MT>;
  constexpr int WS = C::WS;
  constexpr int XSC = C::XSC;
  constexpr int RSC = C::RSC;
  constexpr int KPS = C::KPS;
  constexpr int XK = C::XK;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the 128B-swizzled operand tiles
  const uint32_t base_u32 = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (base_u32 & 1023)) & 1023);
  uint8_t* w_ring = smem;                                    // WS x W_TILE
  uint8_t* x_ring = w_ring + WS * C::W_TILE;                 // XSC x X_CHUNK
  uint8_t* raw_ring = smem + C::OP_BYTES;                    // RSC x RAW_CHUNK
  uint64_t* bars = reinterpret_cast<uint64_t*>(raw_ring + RSC * C::RAW_CHUNK);
  uint64_t* raw_full = bars;
  uint64_t* raw_empty = raw_full + RSC;
  uint64_t* x_full = raw_empty + RSC;
  uint64_t* x_empty = x_full + XSC;
  uint64_t* w_empty = x_empty + XSC;
  uint64_t* acc_full = w_empty + WS;
  uint64_t* mma_done = acc_full + 1;                         // [NG] error-path MMA drains
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + C::NG);
  float* part = reinterpret_cast<float*>(w_ring);            // split-K partial [BN][128]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rt0 = blockIdx.x * MT;  // first 128-row weight tile
  const int nt = blockIdx.y;       // token tile
  const int S = gridDim.z;         // K splits (= cluster size)
  const int KT = a.w.Kpad / kTileK;                         // k-tiles of the operand
  // stored k-tiles of the row tile(s): all KT (dense) or the block-sparse
  // list (block-sparse weights run with MT = 1)
  const bool sparse = MT == 1 && a.w.kt_ptr != nullptr;
  const int tbase = sparse ? a.w.kt_ptr[rt0] : rt0 * KT;
  const int ntot = sparse ? a.w.kt_ptr[rt0 + 1] - tbase : KT;
  const int kb = (int)blockIdx.z * ntot / S;
  const int nk = ((int)blockIdx.z + 1) * ntot / S - kb;    // k-tiles of this CTA (may be 0)
  const int nch = (nk + KPS - 1) / KPS;                      // chunks (the last may be short)
  const int gpr_active = nk < C::GPR ? nk : C::GPR;          // groups per row tile with k-tiles
  const int ngrp = MT * gpr_active;
  uint32_t* status = a.status;
  const uint64_t lim = a.wait_ns ? a.wait_ns : kWaitLimitNs;

  if (threadIdx.x == 0) {
    for (int i = 0; i < RSC; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], kConvWarps);
    }
    for (int i = 0; i < XSC; ++i) {
      mbar_init(&x_full[i], 1);
      mbar_init(&x_empty[i], XK * MT);
    }
    for (int i = 0; i < WS; ++i) mbar_init(&w_empty[i], 1);
    mbar_init(acc_full, ngrp > 0 ? ngrp : 1);
    for (int i = 0; i < C::NG; ++i) mbar_init(&mma_done[i], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc(tmem_slot, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  bool eok = false;                // converter warps: every wait before the epilogue succeeded
  // Chunks of KPS consecutive k-tiles (per row tile) and XK activation tiles
  // move as one bulk copy each: large copies stream far better than per-tile
  // ones.  The producer warps run their loops warp-uniformly (every lane
  // waits, the elected lane issues the copies).  Warp 1 owns the TMEM
  // allocation.
  if (warp == 0) {
    // ------------------------------------------------ raw weight producer
    bool ok = true;
    int issued = 0;                       // chunks whose copies were issued
    for (int c = 0; c < nch && ok; ++c) {
      const int st = c % RSC;
      if (c >= RSC) ok = mbar_wait(&raw_empty[st], ((c / RSC) - 1) & 1, status, lim);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      issued = c + 1;
      if (elect_one()) {
        const int nt_c = nk - c * KPS < KPS ? nk - c * KPS : KPS;
        uint8_t* dst = raw_ring + st * C::RAW_CHUNK;
        mbar_arrive_expect_tx(&raw_full[st], (uint32_t)(MT * nt_c * C::RAW_W));
#pragma unroll
        for (int r = 0; r < MT; ++r) {
          const int tb = sparse ? tbase : (rt0 + r) * KT;
          bulk_g2s(dst + r * KPS * C::RAW_W, a.w.data + ((size_t)tb + kb + (size_t)c * KPS) * C::RAW_W,
                   (uint32_t)(nt_c * C::RAW_W), &raw_full[st]);
        }
      }
      __syncwarp();
    }
    // drain: the last issued copies have landed before shared memory is
    // released -- on the error path too (each wait is bounded; the phase
    // waited on is the latest one of its stage)
    for (int c = issued - (issued < RSC ? issued : RSC); c < issued; ++c)
      (void)mbar_wait(&raw_full[c % RSC], (c / RSC) & 1, status, lim);
  } else if (warp == 2) {
    // ------------------------------------------- activation tile producer
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const uint8_t* xsrc =
        reinterpret_cast<const uint8_t*>(a.opnd) + ((size_t)nt * KT + kb) * C::X_TILE;
    const int nxc = (nk + XK - 1) / XK;
    bool ok = true;
    int issued = 0;
    for (int c = 0; c < nxc && ok; ++c) {
      const int st = c % XSC;
      if (c >= XSC) ok = mbar_wait(&x_empty[st], ((c / XSC) - 1) & 1, status, lim);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      issued = c + 1;
      if (c == 0 && a.withhold_x0) continue;   // test hook: this chunk never arrives
      if (elect_one()) {
        const int nt_c = nk - c * XK < XK ? nk - c * XK : XK;
        mbar_arrive_expect_tx(&x_full[st], (uint32_t)(nt_c * C::X_TILE));
        if (!sparse) {
          bulk_g2s(x_ring + st * C::X_CHUNK, xsrc + (size_t)c * C::X_CHUNK, (uint32_t)(nt_c * C::X_TILE),
                   &x_full[st]);
        } else {
          // the stored k-tiles are not contiguous in K: one copy per tile
          const uint8_t* xrow = reinterpret_cast<const uint8_t*>(a.opnd) + (size_t)nt * KT * C::X_TILE;
          for (int j = 0; j < nt_c; ++j) {
            const int kx = a.w.kt_idx[tbase + kb + c * XK + j];
            bulk_g2s(x_ring + st * C::X_CHUNK + j * C::X_TILE, xrow + (size_t)kx * C::X_TILE, C::X_TILE,
                     &x_full[st]);
          }
        }
      }
      __syncwarp();
    }
    for (int c = issued - (issued < XSC ? issued : XSC); c < issued; ++c)
      if (c != 0 || !a.withhold_x0) (void)mbar_wait(&x_full[c % XSC], (c / XSC) & 1, status, lim);
  } else if (warp >= kRoleWarps) {
    // ----------------------------- converter groups: convert, issue MMAs
    // Group g serves row tile r = g / GPR and takes the k-tiles j = p, p+GPR,
    // ... (p = g % GPR) of every chunk, issuing their MMAs into its own
    // accumulator (TMEM columns g*BN ..), so each accumulator sums its tiles
    // in a fixed order.  Per tile: convert into registers, wait for the
    // group's weight stage, store, fence to the async proxy, group barrier,
    // then one elected lane of the group's issuing warp waits for the
    // activation chunk and issues 4 MMAs.  The raw chunk is released once
    // per chunk by every converter warp.  Every warp of a group passes the
    // group barrier once per tile whatever happened, so a timed-out wait
    // cannot strand the others.
    const int cw = warp - kRoleWarps;
    const int grp = cw / C::GW;
    const int r = grp / C::GPR, ph = grp % C::GPR;
    const int gt = (cw % C::GW) * 32 + lane;           // thread within the group
    const bool issuer = (cw % C::GW) == (grp & 3);     // spread over the SM's 4 schedulers
    constexpr int WPR = C::TB / 4;                     // words per row
    const int row = (gt * C::WORDS) / WPR, w0 = (gt * C::WORDS) % WPR;
    const int c0 = WFMT == 4 ? w0 : w0 / 2;
    const int shift = a.w.gemm_shift;
    const bool fused = a.w.gemm_fused != 0;
    const uint32_t idesc = idesc_bf16(128, BN);
    const uint64_t xdesc = sw128_kmajor_desc(smem_u32(x_ring));
    // this thread's row's two E8M0 bytes per k-tile, straight from global
    // memory (2 bytes per row per tile; a bulk copy of them would cost as
    // much as a weight chunk), one tile ahead
    const int tb_r = sparse ? tbase : (rt0 + r) * KT;
    const uint16_t* srow = reinterpret_cast<const uint16_t*>(a.w.scales) + ((size_t)tb_r + kb) * 128 + row;
    uint32_t sc_next = ph < nk ? ldg_u16(srow + (size_t)ph * 128) : 0u;
    const uint32_t acc = tmem + (uint32_t)(grp * BN);
    int ntile = 0;                                     // tiles this group has issued
    bool mma_issued = false;                           // this (issuer) warp issued an MMA
    bool ok = true;
    for (int c = 0; c < nch; ++c) {
      const int rs = c % RSC;
      if (ok) ok = mbar_wait(&raw_full[rs], (c / RSC) & 1, status, lim);
      ok = __all_sync(0xffffffffu, ok);
      const uint8_t* raw = raw_ring + rs * C::RAW_CHUNK + r * KPS * C::RAW_W;
#pragma unroll 1
      for (int t = 0; t < C::TPG; ++t) {
        const int j = ph + t * C::GPR;
        const int i = c * KPS + j;                     // this group's k-tile
        const bool has = i < nk;                       // group-uniform
        const uint32_t sc2 = sc_next;
        if (i + C::GPR < nk) sc_next = ldg_u16(srow + (size_t)(i + C::GPR) * 128);
        uint4 out[C::NCH];
        if (ok && has) {
          if (fused)
            convert_share<WFMT, C::WORDS, C::NCH, true>(raw + j * C::RAW_W, sc2, row, w0, shift, out);
          else
            convert_share<WFMT, C::WORDS, C::NCH, false>(raw + j * C::RAW_W, sc2, row, w0, shift, out);
        }
        if (t == C::TPG - 1) {
          __syncwarp();
          if (ok && lane == 0) mbar_arrive(&raw_empty[rs]);
        }
        const int ws = grp * C::WSG + (ntile % C::WSG);
        if (ok && has && ntile >= C::WSG) ok = mbar_wait(&w_empty[ws], ((ntile / C::WSG) - 1) & 1, status, lim);
        ok = __all_sync(0xffffffffu, ok);
        uint8_t* wt = w_ring + ws * C::W_TILE;
        if (ok && has) {
#pragma unroll
          for (int q = 0; q < C::NCH; ++q)
            *reinterpret_cast<uint4*>(wt + sw128_offset(row, c0 + q)) = out[q];
          // each writer makes its stores visible to the tensor core's async proxy
          fence_proxy_async_smem();
        }
        named_bar_sync(1 + grp, C::GT);
        if (issuer && has) {
          const int cx = i / XK, xs = cx % XSC;
          if (ok) ok = mbar_wait(&x_full[xs], (cx / XSC) & 1, status, lim);
          ok = __all_sync(0xffffffffu, ok);
          if (ok) {
            tc_fence_after();
            const uint64_t wd = sw128_kmajor_desc(smem_u32(wt));
            const uint64_t xd = xdesc + (uint64_t)((xs * C::X_CHUNK + (i % XK) * C::X_TILE) >> 4);
            if (elect_one()) {
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                mma_bf16_ss(acc, wd + 2 * kk, xd + 2 * kk, idesc, (ntile != 0 || kk != 0) ? 1u : 0u);
              mma_commit(&w_empty[ws]);
              mma_commit(&x_empty[xs]);
            }
            __syncwarp();
            mma_issued = true;
          }
        }
        if (has) ++ntile;
      }
    }
    if (issuer && ok && ph < gpr_active) {
      if (elect_one()) mma_commit(acc_full);
      __syncwarp();
    }
    // error path: MMAs this warp issued finish before the CTA frees shared
    // and tensor memory (the commit tracks the issuing lane's MMAs)
    if (issuer && mma_issued && !ok) {
      if (elect_one()) mma_commit(&mma_done[grp]);
      __syncwarp();
      (void)mbar_wait(&mma_done[grp], 0, status, lim);
    }
    if (ngrp > 0) ok = ok && mbar_wait(acc_full, 0, status, lim);
    eok = __all_sync(0xffffffffu, ok);
  }

  // ---------------------------------------------------------- epilogue
  // Row tile r's result is the sum of its GPR group accumulators in group
  // order (a CTA with no stored k-tiles -- an all-zero row tile of a
  // block-sparse weight, or an empty split -- writes zeros).  Warp w reads
  // TMEM lanes 32*(w%4)..; with MT = 2 half of the converter warps take each
  // row tile.  With a K split, each row tile's partial goes through shared
  // memory and is reduced over the cluster before the next row tile.
  const bool epi = warp >= kRoleWarps;
#pragma unroll 1
  for (int rr = 0; rr < MT; ++rr) {
    if (epi) {
      constexpr int NH = kConvWarps / 4 / MT;          // warps per lane quarter per row tile
      constexpr int CPG = BN / NH >= 8 ? BN / NH : 8;
      const int q = warp & 3, hh = (warp - kRoleWarps) >> 2;
      const int wr = hh / NH, h = hh % NH;             // row tile and column group of this warp
      const int trow = q * 32 + lane;
      const int row_g = (rt0 + rr) * 128 + trow;
      const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
      tc_fence_after();
      if (wr == rr && h * CPG < BN && eok) {
#pragma unroll 1
        for (int cc = h * CPG; cc < (h + 1) * CPG; cc += 8) {
          float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          for (int g = 0; g < gpr_active; ++g) {
            uint32_t v[8];
            tmem_ld8(lane_base + (uint32_t)((rr * C::GPR + g) * BN + cc), v);
            tmem_ld_wait();
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) f[jj] = g == 0 ? __uint_as_float(v[jj]) : f[jj] + __uint_as_float(v[jj]);
          }
          if (S > 1) {
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) part[(cc + jj) * 128 + trow] = f[jj];
          } else {
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) {
              const int tok = nt * BN + cc + jj;
              if (tok < a.B && row_g < a.w.N) a.y[(size_t)tok * a.w.N + row_g] = f[jj];
            }
          }
        }
      }
    }
    if (S > 1) {
      // ------------------------------------- split-K reduction over DSMEM
      __syncwarp();
      cluster_sync_all();                       // all partial tiles written
      const uint32_t rank = cluster_ctarank();
      const int tb = (int)rank * BN / S, te = ((int)rank + 1) * BN / S;
      const uint32_t pbase = smem_u32(part);
      uint32_t src[kMaxSplits];
#pragma unroll
      for (int s2 = 0; s2 < kMaxSplits; ++s2) src[s2] = s2 < S ? mapa_shared(pbase, (uint32_t)s2) : 0u;
      const int n4 = (te - tb) * 32;            // float4 per token row of 128
      for (int i = threadIdx.x; i < n4; i += kGemmThreads) {
        const int tok = tb + (i >> 5), r4 = (i & 31) * 4;
        const uint32_t off = (uint32_t)(tok * 128 + r4) * 4u;
        float4 sum = ld_dsmem_f4(src[0] + off);
#pragma unroll
        for (int s2 = 1; s2 < kMaxSplits; ++s2) {
          if (s2 < S) {
            const float4 v = ld_dsmem_f4(src[s2] + off);
            sum.x += v.x; sum.y += v.y; sum.z += v.z; sum.w += v.w;
          }
        }
        const int gtok = nt * BN + tok, grow = (rt0 + rr) * 128 + r4;
        if (gtok < a.B) {
          float* yr = a.y + (size_t)gtok * a.w.N;
          if (grow + 0 < a.w.N) yr[grow + 0] = sum.x;
          if (grow + 1 < a.w.N) yr[grow + 1] = sum.y;
          if (grow + 2 < a.w.N) yr[grow + 2] = sum.z;
          if (grow + 3 < a.w.N) yr[grow + 3] = sum.w;
        }
      }
      cluster_sync_all();                       // peers are done reading this CTA
    }
  }

  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// How many CTAs of one K-split cluster size can be resident at once (cached
// per kernel instance; 0 if the query fails).
template <int WFMT, int BN, int MT>
int max_clusters(int S) {
  using C = Cfg<WFMT, BN, MT>;
  static int cache[kMaxSplits + 1] = {};
  if (cache[S] != 0) return cache[S] < 0 ? 0 : cache[S];
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1, 1, (unsigned)S);
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = C::SMEM;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = (unsigned)S;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, gemm_tc_kernel<WFMT, BN, MT>, &cfg) != cudaSuccess || n <= 0) {
    (void)cudaGetLastError();
    cache[S] = -1;
    return 0;
  }
  cache[S] = n;
  return n;
}

// Pick the K split: minimise waves x (k-tiles per CTA + fixed per-CTA cost),
// the fixed cost (prologue, pipeline fill, epilogue) counted as 4 k-tiles,
// plus the shared-memory reduction when split (grows with the tile width).
template <int WFMT, int BN, int MT>
int pick_splits(int units, int KT) {
  int best = 1;
  long best_cost = -1;
  for (int S = 1; S <= kMaxSplits; ++S) {
    if (S > 1 && KT / S < 4) break;
    const int mc = max_clusters<WFMT, BN, MT>(S);
    if (mc <= 0) continue;
    const long waves = (units + mc - 1) / mc;
    const long overhead = 4 + (S > 1 ? MT * (1 + BN / 128) : 0);
    const long cost = waves * (MT * ((KT + S - 1) / S) + overhead);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = S;
    }
  }
  return best;
}

template <int WFMT, int BN, int MT>
cudaError_t launch_t(const GemmArgs& a, cudaStream_t st, bool pdl) {
  using C = Cfg<WFMT, BN, MT>;
  static SmemAttr smem_attr;
  if (cudaError_t e = smem_attr.ensure(gemm_tc_kernel<WFMT, BN, MT>, (size_t)C::SMEM)) return e;
  const int T = a.w.Npad / (128 * MT), NT = a.Bpad / BN;
  // k-tiles per row tile: all of K, or the block-sparse average
  const int KT = a.w.kt_ptr ? (a.w.nnz_tiles + T - 1) / T : a.w.Kpad / kTileK;
  const int S = a.splits > 0 ? (a.splits < KT ? a.splits : (KT > 0 ? KT : 1))
                             : pick_splits<WFMT, BN, MT>(T * NT, KT > 0 ? KT : 1);
  if (S > kMaxSplits) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)T, (unsigned)NT, (unsigned)S);
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (S > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = (unsigned)S;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, gemm_tc_kernel<WFMT, BN, MT>, a);
}

// Two row tiles per CTA for dense weights once the token tile is wide
// enough that the activation operand dominates the per-CTA traffic;
// block-sparse weights keep one (their row tiles store different k-tiles).
template <int WFMT, int BN>
cudaError_t launch_mt(const GemmArgs& a, cudaStream_t st, bool pdl) {
  if (BN >= 64 && a.w.kt_ptr == nullptr) return launch_t<WFMT, BN, 2>(a, st, pdl);
  return launch_t<WFMT, BN, 1>(a, st, pdl);
}

template <int WFMT>
cudaError_t launch_fmt(const GemmArgs& a, cudaStream_t st, bool pdl) {
  switch (a.BN) {
    case 16: return launch_t<WFMT, 16, 1>(a, st, pdl);
    case 32: return launch_t<WFMT, 32, 1>(a, st, pdl);
    case 64: return launch_mt<WFMT, 64>(a, st, pdl);
    case 128: return launch_mt<WFMT, 128>(a, st, pdl);
    case 256: return launch_mt<WFMT, 256>(a, st, pdl);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

int gemm_pick_bn(int B) {
  if (B <= 16) return 16;
  if (B <= 32) return 32;
  if (B <= 64) return 64;
  if (B <= 128) return 128;
  return 256;
}

cudaError_t launch_gemm(const GemmArgs& a, cudaStream_t st, bool pdl) {
  if (a.Bpad % a.BN != 0 || a.w.Npad % 128 != 0 || a.splits < 0 || a.splits > kMaxSplits)
    return cudaErrorInvalidValue;
  return a.w.fmt == 4 ? launch_fmt<4>(a, st, pdl) : launch_fmt<8>(a, st, pdl);
}

}  // namespace mxq
