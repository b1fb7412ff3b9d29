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
template <int WFMT, int BN>
struct Cfg {
  static constexpr int NG = BN <= 64 ? 4 : 2;
  static constexpr int GW = kConvWarps / NG;             // warps per group
  static constexpr int GT = GW * 32;
  static constexpr int TB = WFMT == 4 ? 32 : 64;
  static constexpr int RAW_W = 128 * TB;
  static constexpr int RAW_STAGE = RAW_W + 256;
  static constexpr int RAW_TARGET = WFMT == 8 ? (BN <= 64 ? 68 * 1024 : 34 * 1024)
                                              : (BN <= 64 ? 64 * 1024 : (BN <= 128 ? 40 * 1024 : 26 * 1024));
  static constexpr int RS = RAW_TARGET / RAW_STAGE / NG * NG;
  static constexpr int W_TILE = 128 * 128;
  static constexpr int WS = 4;
  static constexpr int X_TILE = BN * 128;
  static constexpr int BUDGET = 222 * 1024;
  static constexpr int XS_FIT = (BUDGET - 2048 - RS * RAW_STAGE - WS * W_TILE) / X_TILE;
  static constexpr int XS = XS_FIT > 16 ? 16 : XS_FIT;
  static constexpr int TMEM_COLS = BN <= 32 ? 32 : (BN <= 64 ? 64 : (BN <= 128 ? 128 : 256));
  static constexpr size_t OP_BYTES = (size_t)WS * W_TILE + (size_t)XS * X_TILE;
  static constexpr size_t SMEM = 1024 + OP_BYTES + (size_t)RS * RAW_STAGE + 1024;
  // converter work per k-tile: 32-bit words of packed weights per thread
  static constexpr int WORDS = 128 * TB / 4 / GT;
  static_assert(XS >= 3 && RS >= NG && RS % NG == 0 && WS % NG == 0, "ring depths");
  static_assert(SMEM <= 227 * 1024, "shared memory");
  static_assert(WORDS == 4 || WORDS == 8 || WORDS == 16, "converter split");
  // the split-K partial tile [BN][128] fp32 reuses the w and x rings
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

// One thread's share of one 128x64 k-tile: WORDS consecutive 32-bit words of
// one row (int4: 4 words per 32-element scale block, 8 per row; int8: 8 per
// block, 16 per row), converted and stored to the swizzled bf16 tile.
template <int WFMT, int WORDS, bool FUSED>
__device__ __forceinline__ void convert_share(const uint8_t* raw, const uint8_t* rsc, uint8_t* wt,
                                              int row, int w0, int shift) {
  if (WFMT == 4) {
    // 32 bytes per row; word i -> output chunk i
#pragma unroll
    for (int q = 0; q < WORDS; q += 4) {
      const uint32_t sb = bf16x2_scale(rsc[row * 2 + ((w0 + q) >> 2)], shift);
      const __nv_bfloat162 sc = *reinterpret_cast<const __nv_bfloat162*>(&sb);
      const __nv_bfloat162 nb = FUSED ? __hmul2(__floats2bfloat162_rn(-136.0f, -136.0f), sc)
                                      : __floats2bfloat162_rn(136.0f, 136.0f);
      const uint4 v = *reinterpret_cast<const uint4*>(raw + row * 32 + (w0 + q) * 4);
      const uint32_t words[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 o = cvt_int4_word<FUSED>(words[i], sc, nb);
        *reinterpret_cast<uint4*>(wt + sw128_offset(row, w0 + q + i)) = o;
      }
    }
  } else {
    // 64 bytes per row; word pair (2j, 2j+1) -> chunk j
#pragma unroll
    for (int q = 0; q < WORDS; q += 4) {
      const float sc = f32_scale(rsc[row * 2 + ((w0 + q) >> 3)], shift);
      const float nb = FUSED ? -8388736.0f * sc : 0.0f;
      const uint4 v = *reinterpret_cast<const uint4*>(raw + row * 64 + (w0 + q) * 4);
      const uint2 c0 = cvt_int8_word<FUSED>(v.x, sc, nb), c1 = cvt_int8_word<FUSED>(v.y, sc, nb);
      const uint2 c2 = cvt_int8_word<FUSED>(v.z, sc, nb), c3 = cvt_int8_word<FUSED>(v.w, sc, nb);
      const int ch = (w0 + q) >> 1;
      *reinterpret_cast<uint4*>(wt + sw128_offset(row, ch)) = make_uint4(c0.x, c0.y, c1.x, c1.y);
      *reinterpret_cast<uint4*>(wt + sw128_offset(row, ch + 1)) = make_uint4(c2.x, c2.y, c3.x, c3.y);
    }
  }
}

template <int WFMT, int BN>
__global__ void __launch_bounds__(kGemmThreads, 1) gemm_tc_kernel(GemmArgs a) {
  using C = Cfg<WFMT, BN>;
  constexpr int WS = C::WS;
  constexpr int XS = C::XS;
  constexpr int RS = C::RS;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the 128B-swizzled operand tiles
  const uint32_t base_u32 = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (base_u32 & 1023)) & 1023);
  uint8_t* w_ring = smem;                                    // WS x W_TILE
  uint8_t* x_ring = w_ring + WS * C::W_TILE;                 // XS x X_TILE
  uint8_t* raw_ring = smem + C::OP_BYTES;                    // RS x RAW_STAGE
  uint64_t* bars = reinterpret_cast<uint64_t*>(raw_ring + RS * C::RAW_STAGE);
  uint64_t* raw_full = bars;
  uint64_t* raw_empty = raw_full + RS;
  uint64_t* x_full = raw_empty + RS;
  uint64_t* x_empty = x_full + XS;
  uint64_t* w_full = x_empty + XS;
  uint64_t* w_empty = w_full + WS;
  uint64_t* acc_full = w_empty + WS;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  float* part = reinterpret_cast<float*>(w_ring);            // split-K partial [BN][128]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rt = blockIdx.x;       // 128-row weight tile
  const int nt = blockIdx.y;       // token tile
  const int S = gridDim.z;         // K splits (= cluster size)
  const int KT = a.w.Kpad / kTileK;
  const int kb = (int)blockIdx.z * KT / S;
  const int nk = ((int)blockIdx.z + 1) * KT / S - kb;
  uint32_t* status = a.status;

  if (threadIdx.x == 0) {
    for (int i = 0; i < RS; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], C::GW);
    }
    for (int i = 0; i < XS; ++i) {
      mbar_init(&x_full[i], 1);
      mbar_init(&x_empty[i], 1);
    }
    for (int i = 0; i < WS; ++i) {
      mbar_init(&w_full[i], C::GW);
      mbar_init(&w_empty[i], 1);
    }
    mbar_init(acc_full, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc(tmem_slot, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Role warps 0-2 run their loops warp-uniformly (every lane waits, the
  // elected lane issues the copies / MMAs), so the tcgen05 and bulk-copy
  // operands stay warp-uniform.
  if (warp == 0) {
    // ------------------------------------------------ raw weight producer
    const uint8_t* wsrc = a.w.data + ((size_t)rt * KT + kb) * C::RAW_W;
    const uint8_t* ssrc = a.w.scales + ((size_t)rt * KT + kb) * 256;
    bool ok = true;
    int r = 0;
    uint32_t ph = 0;
    for (int i = 0; i < nk && ok; ++i) {
      if (i >= RS) ok = mbar_wait(&raw_empty[r], ph ^ 1u, status);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      if (elect_one()) {
        uint8_t* dst = raw_ring + r * C::RAW_STAGE;
        mbar_arrive_expect_tx(&raw_full[r], C::RAW_STAGE);
        bulk_g2s(dst, wsrc + (size_t)i * C::RAW_W, C::RAW_W, &raw_full[r]);
        bulk_g2s(dst + C::RAW_W, ssrc + (size_t)i * 256, 256, &raw_full[r]);
      }
      __syncwarp();
      if (++r == RS) { r = 0; ph ^= 1u; }
    }
    // drain: the last issued copies have landed before shared memory is released
    for (int i = nk - (nk < RS ? nk : RS); i < nk && ok; ++i)
      ok = mbar_wait(&raw_full[i % RS], (i / RS) & 1, status);
  } else if (warp == 2) {
    // ------------------------------------------- activation tile producer
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const uint8_t* xsrc =
        reinterpret_cast<const uint8_t*>(a.opnd) + ((size_t)nt * KT + kb) * C::X_TILE;
    bool ok = true;
    int s = 0;
    uint32_t ph = 0;
    for (int i = 0; i < nk && ok; ++i) {
      if (i >= XS) ok = mbar_wait(&x_empty[s], ph ^ 1u, status);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      if (elect_one()) {
        mbar_arrive_expect_tx(&x_full[s], C::X_TILE);
        bulk_g2s(x_ring + s * C::X_TILE, xsrc + (size_t)i * C::X_TILE, C::X_TILE, &x_full[s]);
      }
      __syncwarp();
      if (++s == XS) { s = 0; ph ^= 1u; }
    }
    for (int i = nk - (nk < XS ? nk : XS); i < nk && ok; ++i)
      ok = mbar_wait(&x_full[i % XS], (i / XS) & 1, status);
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    const uint32_t idesc = idesc_bf16(128, BN);
    // descriptor start-address field is address >> 4: stage and K offsets
    // add to the prebuilt descriptors directly
    const uint64_t wdesc = sw128_kmajor_desc(smem_u32(w_ring));
    const uint64_t xdesc = sw128_kmajor_desc(smem_u32(x_ring));
    bool ok = true;
    int s = 0, sx = 0;
    uint32_t ph = 0, phx = 0;
    for (int i = 0; i < nk && ok; ++i) {
      ok = mbar_wait(&w_full[s], ph, status) && mbar_wait(&x_full[sx], phx, status);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const uint64_t wd = wdesc + (uint64_t)((s * C::W_TILE) >> 4);
      const uint64_t xd = xdesc + (uint64_t)((sx * C::X_TILE) >> 4);
      if (elect_one()) {
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_bf16_ss(tmem, wd + 2 * kk, xd + 2 * kk, idesc, (i | kk) != 0 ? 1u : 0u);
        mma_commit(&w_empty[s]);
        mma_commit(&x_empty[sx]);
      }
      __syncwarp();
      if (++s == WS) { s = 0; ph ^= 1u; }
      if (++sx == XS) { sx = 0; phx ^= 1u; }
    }
    if (ok && elect_one()) mma_commit(acc_full);
    __syncwarp();
  } else if (warp >= kRoleWarps) {
    // ------------------------------------------ converters, then epilogue
    const int cw = warp - kRoleWarps;
    const int grp = cw / C::GW;
    const int gt = (cw % C::GW) * 32 + lane;           // thread within the group
    constexpr int WPR = C::TB / 4;                     // words per row
    const int row = (gt * C::WORDS) / WPR, w0 = (gt * C::WORDS) % WPR;
    const int shift = a.w.gemm_shift;
    const bool fused = a.w.gemm_fused != 0;
    bool ok = true;
    for (int i = grp; i < nk && ok; i += C::NG) {
      const int r = i % RS, s = i % WS;
      ok = mbar_wait(&raw_full[r], (i / RS) & 1, status);
      if (ok && i >= WS) ok = mbar_wait(&w_empty[s], ((i / WS) - 1) & 1, status);
      ok = __all_sync(0xffffffffu, ok);   // keep each warp's lanes together
      if (!ok) break;
      const uint8_t* raw = raw_ring + r * C::RAW_STAGE;
      uint8_t* wt = w_ring + s * C::W_TILE;
      if (fused)
        convert_share<WFMT, C::WORDS, true>(raw, raw + C::RAW_W, wt, row, w0, shift);
      else
        convert_share<WFMT, C::WORDS, false>(raw, raw + C::RAW_W, wt, row, w0, shift);
      // each writer makes its stores visible to the tensor core's async
      // proxy; after the warp converges one lane arrives for all 32
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&raw_empty[r]);
        mbar_arrive(&w_full[s]);
      }
    }
    // epilogue
    if (ok) ok = mbar_wait(acc_full, 0, status);
    ok = __all_sync(0xffffffffu, ok);     // tcgen05.ld is warp-collective
    tc_fence_after();
    if (ok) {
      // warp w reads TMEM lanes 32*(w%4)..; the column range is split over
      // the kConvWarps/4 warps that share a lane quarter
      constexpr int NH = kConvWarps / 4;
      constexpr int CPG = BN / NH >= 8 ? BN / NH : 8;
      const int q = warp & 3, h = (warp - kRoleWarps) >> 2;
      const int trow = q * 32 + lane;
      const int row_g = rt * 128 + trow;
      const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
      if (h * CPG < BN) {
#pragma unroll 1
        for (int c = h * CPG; c < (h + 1) * CPG; c += 8) {
          uint32_t v[8];
          tmem_ld8(lane_base + (uint32_t)c, v);
          tmem_ld_wait();
          if (S > 1) {
#pragma unroll
            for (int j = 0; j < 8; ++j) part[(c + j) * 128 + trow] = __uint_as_float(v[j]);
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const int tok = nt * BN + c + j;
              if (tok < a.B && row_g < a.w.N) a.y[(size_t)tok * a.w.N + row_g] = __uint_as_float(v[j]);
            }
          }
        }
      }
    }
  }

  if (S > 1) {
    // ---------------------------------------- split-K reduction over DSMEM
    __syncwarp();
    cluster_sync_all();                         // all partial tiles written
    const uint32_t rank = cluster_ctarank();
    const int tb = (int)rank * BN / S, te = ((int)rank + 1) * BN / S;
    const uint32_t pbase = smem_u32(part);
    uint32_t src[kMaxSplits];
#pragma unroll
    for (int s = 0; s < kMaxSplits; ++s) src[s] = s < S ? mapa_shared(pbase, (uint32_t)s) : 0u;
    const int n4 = (te - tb) * 32;              // float4 per token row of 128
    for (int i = threadIdx.x; i < n4; i += kGemmThreads) {
      const int tok = tb + (i >> 5), r4 = (i & 31) * 4;
      const uint32_t off = (uint32_t)(tok * 128 + r4) * 4u;
      float4 acc = ld_dsmem_f4(src[0] + off);
#pragma unroll
      for (int s = 1; s < kMaxSplits; ++s) {
        if (s < S) {
          const float4 v = ld_dsmem_f4(src[s] + off);
          acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
        }
      }
      const int gtok = nt * BN + tok, grow = rt * 128 + r4;
      if (gtok < a.B) {
        float* yr = a.y + (size_t)gtok * a.w.N;
        if (grow + 0 < a.w.N) yr[grow + 0] = acc.x;
        if (grow + 1 < a.w.N) yr[grow + 1] = acc.y;
        if (grow + 2 < a.w.N) yr[grow + 2] = acc.z;
        if (grow + 3 < a.w.N) yr[grow + 3] = acc.w;
      }
    }
    cluster_sync_all();                         // peers are done reading this CTA
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
template <int WFMT, int BN>
int max_clusters(int S) {
  using C = Cfg<WFMT, BN>;
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
  if (cudaOccupancyMaxActiveClusters(&n, gemm_tc_kernel<WFMT, BN>, &cfg) != cudaSuccess || n <= 0) {
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
template <int WFMT, int BN>
int pick_splits(int units, int KT) {
  int best = 1;
  long best_cost = -1;
  for (int S = 1; S <= kMaxSplits; ++S) {
    if (S > 1 && KT / S < 4) break;
    const int mc = max_clusters<WFMT, BN>(S);
    if (mc <= 0) continue;
    const long waves = (units + mc - 1) / mc;
    const long overhead = 4 + (S > 1 ? 1 + BN / 128 : 0);
    const long cost = waves * ((KT + S - 1) / S + overhead);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = S;
    }
  }
  return best;
}

template <int WFMT, int BN>
cudaError_t launch_t(const GemmArgs& a, cudaStream_t st, bool pdl) {
  using C = Cfg<WFMT, BN>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<WFMT, BN>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)C::SMEM);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  const int T = a.w.Npad / 128, NT = a.Bpad / BN, KT = a.w.Kpad / kTileK;
  const int S = a.splits > 0 ? (a.splits < KT ? a.splits : KT) : pick_splits<WFMT, BN>(T * NT, KT);
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
  return cudaLaunchKernelEx(&cfg, gemm_tc_kernel<WFMT, BN>, a);
}

template <int WFMT>
cudaError_t launch_fmt(const GemmArgs& a, cudaStream_t st, bool pdl) {
  switch (a.BN) {
    case 16: return launch_t<WFMT, 16>(a, st, pdl);
    case 32: return launch_t<WFMT, 32>(a, st, pdl);
    case 64: return launch_t<WFMT, 64>(a, st, pdl);
    case 128: return launch_t<WFMT, 128>(a, st, pdl);
    case 256: return launch_t<WFMT, 256>(a, st, pdl);
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
