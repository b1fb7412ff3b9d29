// mxq_gemm.cu -- tensor-core MX GEMM for the prefill / rollout / MoE regime
// (batch > 8): the batched mx_gemv of the reference
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
// Warp roles (384 threads):
//   warp 0      raw producer: 1-D bulk copies of packed weight tiles + scales
//               (int4: 4 KB + 256 B per 128x64 tile) into an 8-deep raw ring;
//   warp 1      TMEM owner and single-thread MMA issuer (4 x K=16 per tile);
//   warp 2      operand producer: bulk copy of the pre-swizzled bf16
//               activation tile (BN x 128 B) into the operand ring;
//   warps 4-11  converters: unpack int4/int8 -> bf16, apply 2^e_w, write the
//               128B-swizzled K-major tile, fence to the async proxy; then
//               the epilogue (tcgen05.ld -> fp32 stores, coalesced by row).
// Every mbarrier wait is bounded; a wait that gives up sets the status word.
#include "mxq_internal.h"

namespace mxq {

namespace {

constexpr int kGemmThreads = 384;
constexpr uint32_t kWaitLimit = 1u << 22;

// Raw (packed weight) ring sized by bytes in flight: small token tiles are
// HBM-streaming (deep ring, ~100 KB per SM); large ones are MMA-bound.
template <int WFMT, int BN>
struct Cfg {
  static constexpr int TB = WFMT == 4 ? 32 : 64;
  static constexpr int RAW_W = 128 * TB;
  static constexpr int RAW_STAGE = RAW_W + 256;
  static constexpr int RAW_TARGET = BN <= 64 ? 104 * 1024 : (BN <= 128 ? 64 * 1024 : 36 * 1024);
  static constexpr int RS = RAW_TARGET / RAW_STAGE;
  static constexpr int W_TILE = 128 * 128;
  static constexpr int X_TILE = BN * 128;
  static constexpr int OP_STAGE = W_TILE + X_TILE;
  static constexpr int BUDGET = 222 * 1024;
  static constexpr int OS_FIT = (BUDGET - 2048 - RS * RAW_STAGE) / OP_STAGE;
  static constexpr int OS = OS_FIT > 4 ? 4 : OS_FIT;
  static constexpr int TMEM_COLS = BN <= 32 ? 32 : (BN <= 64 ? 64 : (BN <= 128 ? 128 : 256));
  static constexpr size_t SMEM = 1024 + (size_t)OS * OP_STAGE + (size_t)RS * RAW_STAGE + 1024;
  static_assert(OS >= 2 && RS >= 4, "rings too shallow");
};

__device__ __forceinline__ uint32_t bf16x2_scale(uint32_t s) {
  const uint32_t h = s == 0u ? 0x0040u : (s == 255u ? 0x7FC0u : (s << 7));
  return h | (h << 16);
}

// int4: 8 nibbles -> four bf16x2 (slot order e0,e2,e4,e6,e1,e3,e5,e7),
// each w * 2^e exactly: (128 + (w+8)) - 136 = w, then times the scale.
__device__ __forceinline__ uint4 cvt_int4_word(uint32_t w, __nv_bfloat162 sc) {
  const uint32_t wx = w ^ 0x88888888u;
  const uint32_t lo = wx & 0x0F0F0F0Fu;
  const uint32_t hi = (wx >> 4) & 0x0F0F0F0Fu;
  const uint32_t C = 0x43434343u;
  uint32_t p[4] = {__byte_perm(lo, C, 0x4140), __byte_perm(lo, C, 0x4342),
                   __byte_perm(hi, C, 0x4140), __byte_perm(hi, C, 0x4342)};
  const __nv_bfloat162 off = __floats2bfloat162_rn(136.0f, 136.0f);
  uint4 r;
  uint32_t* rr = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&p[i]);
    v = __hmul2(__hsub2(v, off), sc);
    rr[i] = *reinterpret_cast<uint32_t*>(&v);
  }
  return r;
}

// int8: 4 signed bytes -> two bf16x2 in natural order, w * 2^e exactly.
__device__ __forceinline__ uint2 cvt_int8_word(uint32_t w, float sc) {
  const uint32_t wx = w ^ 0x80808080u;
  const uint32_t M = 0x4B000000u;
  float f[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t bits = __byte_perm(wx, M, 0x7540 + i);  // 2^23 + (b + 128)
    f[i] = __fmul_rn(__fsub_rn(__uint_as_float(bits), 8388736.0f), sc);
  }
  __nv_bfloat162 a = __floats2bfloat162_rn(f[0], f[1]);
  __nv_bfloat162 b = __floats2bfloat162_rn(f[2], f[3]);
  return make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
}

template <int WFMT, int BN>
__global__ void __launch_bounds__(kGemmThreads, 1) gemm_tc_kernel(GemmArgs a) {
  using C = Cfg<WFMT, BN>;
  constexpr int OS = C::OS;
  constexpr int RS = C::RS;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the 128B-swizzled operand tiles
  const uint32_t base_u32 = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (base_u32 & 1023)) & 1023);
  uint8_t* op_ring = smem;                                   // OS x OP_STAGE
  uint8_t* raw_ring = op_ring + OS * C::OP_STAGE;            // RS x RAW_STAGE
  uint64_t* bars = reinterpret_cast<uint64_t*>(raw_ring + RS * C::RAW_STAGE);
  uint64_t* raw_full = bars;
  uint64_t* raw_empty = raw_full + RS;
  uint64_t* x_full = raw_empty + RS;
  uint64_t* w_full = x_full + OS;
  uint64_t* op_empty = w_full + OS;
  uint64_t* acc_full = op_empty + OS;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rt = blockIdx.x;       // 128-row weight tile
  const int nt = blockIdx.y;       // token tile
  const int KT = a.w.Kpad / kTileK;
  uint32_t* status = a.status;

  if (threadIdx.x == 0) {
    for (int i = 0; i < RS; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], 256);
    }
    for (int i = 0; i < OS; ++i) {
      mbar_init(&x_full[i], 1);
      mbar_init(&w_full[i], 256);
      mbar_init(&op_empty[i], 1);
    }
    mbar_init(acc_full, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc(tmem_slot, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------ raw weight producer
    if (lane == 0) {
      const uint8_t* wsrc = a.w.data + (size_t)rt * KT * C::RAW_W;
      const uint8_t* ssrc = a.w.scales + (size_t)rt * KT * 256;
      bool ok = true;
      for (int kt = 0; kt < KT && ok; ++kt) {
        const int r = kt % RS;
        if (kt >= RS) ok = mbar_wait(&raw_empty[r], ((kt / RS) - 1) & 1, status, kWaitLimit);
        if (!ok) break;
        uint8_t* dst = raw_ring + r * C::RAW_STAGE;
        mbar_arrive_expect_tx(&raw_full[r], C::RAW_STAGE);
        bulk_g2s(dst, wsrc + (size_t)kt * C::RAW_W, C::RAW_W, &raw_full[r]);
        bulk_g2s(dst + C::RAW_W, ssrc + (size_t)kt * 256, 256, &raw_full[r]);
      }
      // drain: the last issued copies have landed before shared memory is released
      for (int kt = KT - (KT < RS ? KT : RS); kt < KT && ok; ++kt)
        ok = mbar_wait(&raw_full[kt % RS], (kt / RS) & 1, status, kWaitLimit);
    }
  } else if (warp == 2) {
    // ------------------------------------------- activation tile producer
    if (lane == 0) {
      asm volatile("griddepcontrol.wait;" ::: "memory");
      const uint8_t* xsrc = reinterpret_cast<const uint8_t*>(a.opnd) + (size_t)nt * KT * C::X_TILE;
      bool ok = true;
      for (int kt = 0; kt < KT && ok; ++kt) {
        const int s = kt % OS;
        if (kt >= OS) ok = mbar_wait(&op_empty[s], ((kt / OS) - 1) & 1, status, kWaitLimit);
        if (!ok) break;
        uint8_t* dst = op_ring + s * C::OP_STAGE + C::W_TILE;
        mbar_arrive_expect_tx(&x_full[s], C::X_TILE);
        bulk_g2s(dst, xsrc + (size_t)kt * C::X_TILE, C::X_TILE, &x_full[s]);
      }
      for (int kt = KT - (KT < OS ? KT : OS); kt < KT && ok; ++kt)
        ok = mbar_wait(&x_full[kt % OS], (kt / OS) & 1, status, kWaitLimit);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16(128, BN);
      bool ok = true;
      for (int kt = 0; kt < KT && ok; ++kt) {
        const int s = kt % OS;
        const uint32_t par = (kt / OS) & 1;
        ok = mbar_wait(&w_full[s], par, status, kWaitLimit) &&
             mbar_wait(&x_full[s], par, status, kWaitLimit);
        if (!ok) break;
        tc_fence_after();
        const uint32_t wa = smem_u32(op_ring + s * C::OP_STAGE);
        const uint32_t xa = wa + C::W_TILE;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_bf16_ss(tmem, sw128_kmajor_desc(wa + kk * 32), sw128_kmajor_desc(xa + kk * 32),
                      idesc, (kt | kk) != 0 ? 1u : 0u);
        mma_commit(&op_empty[s]);
      }
      if (ok) mma_commit(acc_full);
    }
  } else if (warp >= 4) {
    // ------------------------------------------ converters, then epilogue
    const int ct = threadIdx.x - 128;  // 0..255
    bool ok = true;
    for (int kt = 0; kt < KT && ok; ++kt) {
      const int r = kt % RS, s = kt % OS;
      ok = mbar_wait(&raw_full[r], (kt / RS) & 1, status, kWaitLimit);
      if (ok && kt >= OS) ok = mbar_wait(&op_empty[s], ((kt / OS) - 1) & 1, status, kWaitLimit);
      ok = __all_sync(0xffffffffu, ok);   // keep each warp's lanes together
      if (!ok) break;
      const uint8_t* raw = raw_ring + r * C::RAW_STAGE;
      const uint8_t* rsc = raw + C::RAW_W;
      uint8_t* wt = op_ring + s * C::OP_STAGE;
      if (WFMT == 4) {
        const int row = ct >> 1, hh = ct & 1;
        const uint4 v = *reinterpret_cast<const uint4*>(raw + row * 32 + hh * 16);
        const uint32_t sc = bf16x2_scale(rsc[row * 2 + hh]);
        const __nv_bfloat162 s2 = *reinterpret_cast<const __nv_bfloat162*>(&sc);
        const uint32_t words[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int wi = 0; wi < 4; ++wi) {
          const uint4 o = cvt_int4_word(words[wi], s2);
          *reinterpret_cast<uint4*>(wt + sw128_offset(row, hh * 4 + wi)) = o;
        }
      } else {
#pragma unroll
        for (int rep = 0; rep < 2; ++rep) {
          const int u = ct + rep * 256;
          const int row = u >> 2, qd = u & 3;
          const uint4 v = *reinterpret_cast<const uint4*>(raw + row * 64 + qd * 16);
          const float sc = e8m0_to_float(rsc[row * 2 + (qd >> 1)]);
          const uint2 c0 = cvt_int8_word(v.x, sc), c1 = cvt_int8_word(v.y, sc);
          const uint2 c2 = cvt_int8_word(v.z, sc), c3 = cvt_int8_word(v.w, sc);
          *reinterpret_cast<uint4*>(wt + sw128_offset(row, qd * 2)) = make_uint4(c0.x, c0.y, c1.x, c1.y);
          *reinterpret_cast<uint4*>(wt + sw128_offset(row, qd * 2 + 1)) = make_uint4(c2.x, c2.y, c3.x, c3.y);
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(&raw_empty[r]);
      mbar_arrive(&w_full[s]);
    }
    // epilogue
    if (ok) ok = mbar_wait(acc_full, 0, status, kWaitLimit);
    ok = __all_sync(0xffffffffu, ok);     // tcgen05.ld is warp-collective
    tc_fence_after();
    if (ok) {
      const int q = warp & 3, h = (warp - 4) >> 2;
      const int row = rt * 128 + q * 32 + lane;
      const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
      for (int c = h * (BN / 2); c < (h + 1) * (BN / 2); c += 8) {
        uint32_t v[8];
        tmem_ld8(lane_base + (uint32_t)c, v);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int tok = nt * BN + c + j;
          if (tok < a.B && row < a.w.N) a.y[(size_t)tok * a.w.N + row] = __uint_as_float(v[j]);
        }
      }
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
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(a.w.Npad / 128), (unsigned)(a.Bpad / BN));
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
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
  if (a.Bpad % a.BN != 0 || a.w.Npad % 128 != 0) return cudaErrorInvalidValue;
  return a.w.fmt == 4 ? launch_fmt<4>(a, st, pdl) : launch_fmt<8>(a, st, pdl);
}

}  // namespace mxq
