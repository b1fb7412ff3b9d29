// mxq_common.cuh -- device helpers shared by the MX kernels (sm_100a).
//
// Numeric contract (identical to the CPU oracle, which is its checker):
//   E8M0 byte s encodes 2^(s-127); 0xFF is NaN.
//   Block exponent e = smallest integer with max|v| <= QMAX * 2^e, clamped to
//   e >= -127; all-zero block -> byte 0; non-finite block -> 0xFF.
//   q = round-half-to-even(v * 2^-e); activations are stored as u8 q+128
//   (nn/core/layers/ssm.cpp:170-177 with the rounding of the AVX-512 path,
//   nn/core/layers/ssm.cpp:249).
//   int4 weights: two's complement nibbles, element 2i in the low nibble.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

namespace mxq {

constexpr int kBlock = 32;           // MX block (K elements per E8M0 scale)
constexpr int kTileRows = 128;       // weight rows per tile in the tiled layout
constexpr int kTileK = 64;           // K elements per tile in the tiled layout

// Device status word bits (written by bounded waits that gave up).
constexpr uint32_t kStatusTimeout = 1u;
// Default limit of a bounded device wait (wall time, %globaltimer).
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// ------------------------------------------------------------ powers of 2 --

// 2^n as float for n in [-149, 127], exact (denormals included).
__device__ __forceinline__ float pow2_exact(int n) {
  return n >= -126 ? __int_as_float((n + 127) << 23)
                   : __int_as_float(1u << (n + 149));
}

// E8M0 byte -> float scale 2^(s-127) (exact; NaN for 0xFF).
__device__ __forceinline__ float e8m0_to_float(uint32_t s) {
  return s == 255u ? __int_as_float(0x7fc00000) : pow2_exact((int)s - 127);
}

// Smallest e with m <= qmax * 2^e for finite m > 0, from the float's bits.
// qmax = 127 = 1.984375 * 2^6 and qmax = 7 = 1.75 * 2^2; m = 1.f * 2^k:
// e = k - c when 1.f <= qmax / 2^c, else k - c + 1.  Denormal m give
// k < -126 and are clamped to -127 like every other tiny block.
template <int QMAX>
__device__ __forceinline__ int e8m0_exponent(float m) {
  static_assert(QMAX == 127 || QMAX == 7, "qmax");
  const uint32_t bits = __float_as_uint(m);
  const int kexp = (int)((bits >> 23) & 0xFF);
  if (kexp == 0) return -127;  // zero (handled by caller) or denormal
  const int k = kexp - 127;
  const uint32_t frac = bits & 0x7FFFFF;
  int e;
  if (QMAX == 127) e = k - 6 + (frac > 0x7E0000u ? 1 : 0);
  else             e = k - 2 + (frac > 0x600000u ? 1 : 0);
  return e < -127 ? -127 : e;
}

// Quantise one value with a block exponent (e in [-127, 126]); returns q.
__device__ __forceinline__ int quant_value(float v, int e) {
  const float inv = __int_as_float((127 - e) << 23);  // 2^-e, normal
  return __float2int_rn(__fmul_rn(v, inv));
}

// ------------------------------------------------ exp / SiLU (bit-exact) --
// exp(x) by Cody-Waite reduction (ln2 = hi + lo, hi exactly representable)
// and the degree-7 Taylor polynomial of e^r on |r| <= ln2/2 in Horner form
// with fused multiply-adds; 2^n applied through the exponent field.  Each
// step is one IEEE round-to-nearest operation, so the CPU oracle (compiled
// without contraction, using fmaf) produces the same bits.
__device__ __forceinline__ float det_expf(float x) {
  const float LOG2E = 1.44269504088896341f;
  const float LN2_HI = 6.93145751953125e-1f;
  const float LN2_LO = 1.42860682030941723212e-6f;
  if (x != x) return x;
  if (x > 88.72283935546875f) return __int_as_float(0x7f800000);
  if (x < -103.972084045410f) return 0.0f;
  const float t = __fmul_rn(x, LOG2E);
  const float nf = rintf(t);
  const int n = (int)nf;
  float r = __fmaf_rn(-nf, LN2_HI, x);
  r = __fmaf_rn(-nf, LN2_LO, r);
  float p = 1.0f / 5040.0f;
  p = __fmaf_rn(p, r, 1.0f / 720.0f);
  p = __fmaf_rn(p, r, 1.0f / 120.0f);
  p = __fmaf_rn(p, r, 1.0f / 24.0f);
  p = __fmaf_rn(p, r, 1.0f / 6.0f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  if (n > 127) {
    p = __fmul_rn(p, __int_as_float((n - 1 + 127) << 23));
    p = __fmul_rn(p, 2.0f);
  } else if (n < -126) {
    p = __fmul_rn(p, __int_as_float((n + 64 + 127) << 23));
    p = __fmul_rn(p, __int_as_float((-64 + 127) << 23));
  } else {
    p = __fmul_rn(p, __int_as_float((n + 127) << 23));
  }
  return p;
}

__device__ __forceinline__ float det_silu(float x) {
  const float e = det_expf(-x);
  return __fdiv_rn(x, __fadd_rn(1.0f, e));
}

__device__ __forceinline__ float det_swiglu(float g, float u) {
  return __fmul_rn(det_silu(g), u);
}

// ------------------------------------------------------- warp reductions --
__device__ __forceinline__ float warp_max(float v, int width) {
  for (int o = width / 2; o > 0; o >>= 1)
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// --------------------------------------------------- mbarrier / async ops --
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(count));
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar,
                                                      uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: a thread whose phase has not completed
// sleeps in hardware (woken when the phase completes, or after hint_ns)
// instead of spinning and taking issue slots from the warps doing work.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// One lane of a converged warp (the issuing lane for single-thread async
// instructions inside warp-uniform loops).
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait: polls with the suspend hint and gives up once `limit_ns` of
// wall time have passed, records the timeout in the device status word and
// returns false.  Every wait in the pipelines below goes through this, so a
// broken invariant ends the kernel instead of hanging the GPU.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* status,
                                          uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 0; it < (1u << 26); ++it) {   // also capped in polls
    if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
    if (globaltimer_ns() - t0 > limit_ns) break;
  }
  if (status) atomicOr(status, kStatusTimeout);
  return false;
}

// --- flags in peer memory (mailboxes over NVLink) ------------------------
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Bounded wait until every rank's flag has reached this call's epoch (the
// flags are written over NVLink by the other GPUs).  Returns 0, with the
// timeout recorded in the status word, once `limit_ns` have passed.
__device__ inline int peer_wait(const uint32_t* flags, int world, uint32_t ep, uint64_t limit_ns, uint32_t* status) {
  const uint64_t t0 = globaltimer_ns();
  for (int r = 0; r < world; ++r) {
    for (uint32_t it = 0;; ++it) {
      if ((int)(ld_acquire_sys(flags + r) - ep) >= 0) break;
      if (it > (1u << 26) || globaltimer_ns() - t0 > limit_ns) {
        if (status) atomicOr(status, kStatusTimeout);
        return 0;
      }
      __nanosleep(100);
    }
  }
  return 1;
}

// The same wait over every rank's flag but `skip`'s (a rank's own flag, which
// only its own kernel would set).
__device__ inline int peer_wait_others(const uint32_t* flags, int world, int skip, uint32_t ep, uint64_t limit_ns,
                                       uint32_t* status) {
  const uint64_t t0 = globaltimer_ns();
  for (int r = 0; r < world; ++r) {
    if (r == skip) continue;
    for (uint32_t it = 0;; ++it) {
      if ((int)(ld_acquire_sys(flags + r) - ep) >= 0) break;
      if (it > (1u << 26) || globaltimer_ns() - t0 > limit_ns) {
        if (status) atomicOr(status, kStatusTimeout);
        return 0;
      }
      __nanosleep(100);
    }
  }
  return 1;
}

// 1-D bulk copy global -> shared, completing bytes on an mbarrier.
// Both addresses 16-byte aligned and bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src,
                                         uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1], %2, [%3];" ::"r"(smem_u32(dst_smem)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// One CTA's slice of an L2 prefetch (bulk prefetch wants 16-byte multiples).
__device__ __forceinline__ void prefetch_l2_share(const void* p, size_t bytes, int cta, int ctas) {
  if (!p || !bytes) return;
  const size_t chunk = ((bytes + ctas - 1) / ctas + 15) / 16 * 16;
  const size_t lo = (size_t)cta * chunk;
  if (lo >= bytes) return;
  size_t n = bytes - lo < chunk ? bytes - lo : chunk;
  const uint8_t* q = static_cast<const uint8_t*>(p) + lo;
  while (n) {
    const uint32_t piece = (uint32_t)(n > 65536 ? 65536 : n);
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(q), "r"(piece) : "memory");
    q += piece;
    n -= piece;
  }
}


// ------------------------------------------------- clusters / DSMEM --
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Every thread of every CTA in the cluster must call this (a hardware
// barrier; CTAs of one cluster are always co-scheduled).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// Shared-memory address of the same variable in cluster CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}

__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// ------------------------------------------------------------- tcgen05 --
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile(
      "tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
          smem_u32(dst_smem)),
      "r"(ncols)
      : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(
                   taddr),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, bf16 inputs, fp32 accumulate.
__device__ __forceinline__ void mma_bf16_ss(uint32_t tmem_d, uint64_t adesc,
                                            uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(
          tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
      "[%0];" ::"r"(smem_u32(bar))
      : "memory");
}

// 32 lanes x 8 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]),
        "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle,
// rows of 128 bytes, 8-row atoms 1024 bytes apart.
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);   // start address
  d |= (uint64_t)1 << 16;                   // leading byte offset (unused)
  d |= (uint64_t)(1024 >> 4) << 32;         // stride byte offset
  d |= (uint64_t)1 << 46;                   // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                   // SWIZZLE_128B
  return d;
}

// Instruction descriptor: bf16 x bf16 -> fp32, both K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
  return (1u << 4)                      // D format f32
         | (1u << 7)                    // A bf16
         | (1u << 10)                   // B bf16
         | ((uint32_t)(N >> 3) << 17)   // N
         | ((uint32_t)(M >> 4) << 24);  // M
}

// Byte offset of (row, 16-byte chunk) inside a 128B-swizzled K-major tile.
__host__ __device__ __forceinline__ uint32_t sw128_offset(uint32_t row,
                                                          uint32_t chunk) {
  return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

}  // namespace mxq
