/*
 * mx_cpu_baseline.c -- multi-threaded CPU restatement of the reference's
 * removed AVX-512 VNNI MX GEMV (nn/core/simd/avx512_vnni.hpp, absent from the
 * snapshot; design described in nn/user.md:17 and
 * research_paper/HARDWARE_SATURATION.md:7-13): _mm512_dpbusd_epi32 over u8
 * activations (q+128) and s8 weights, two 32-element blocks per instruction,
 * each block's sum minus 128 * w_sum, scaled by 2^(e_x + e_w) and summed in
 * fp32.  OpenMP over output rows.
 *
 * TEST INFRASTRUCTURE / BASELINE ONLY: timed beside the GPU as the reference
 * CPU arm; never part of the product path.
 */
#include <stdint.h>
#include <stddef.h>
#include <string.h>
#include <omp.h>
#include <immintrin.h>

#define BLK 32

static inline float pow2f_i(int e)
{
    union { uint32_t u; float f; } v;
    if (e < -126 || e > 127) return e < 0 ? 0.0f : __builtin_inff();
    v.u = (uint32_t)(e + 127) << 23;
    return v.f;
}

/* Unpack one 16-byte int4 block (element 2i low nibble of byte i) into 32
 * signed bytes. */
static inline void unpack_int4_scalar(const uint8_t* src, int8_t* dst)
{
    for (int i = 0; i < 16; ++i) {
        int lo = src[i] & 0xF, hi = src[i] >> 4;
        dst[2 * i] = (int8_t)(lo >= 8 ? lo - 16 : lo);
        dst[2 * i + 1] = (int8_t)(hi >= 8 ? hi - 16 : hi);
    }
}

/* w_sums[n][b] = sum of the block's signed weights (the dpbusd correction). */
void mxb_weight_sums(int fmt, const void* w, size_t N, size_t K, int32_t* w_sums)
{
    size_t nb = K / BLK;
#pragma omp parallel for schedule(static)
    for (size_t n = 0; n < N; ++n) {
        int8_t tmp[BLK];
        for (size_t b = 0; b < nb; ++b) {
            const int8_t* p;
            if (fmt == 8) {
                p = (const int8_t*)w + n * K + b * BLK;
            } else {
                unpack_int4_scalar((const uint8_t*)w + n * (K / 2) + b * 16, tmp);
                p = tmp;
            }
            int32_t s = 0;
            for (int i = 0; i < BLK; ++i) s += p[i];
            w_sums[n * nb + b] = s;
        }
    }
}

/* 32 signed int4 weights of block b of row n (16 bytes) -> 32 int8 lanes. */
__attribute__((target("avx2,avx512f,avx512bw,avx512vl,avx512vnni")))
static inline __m256i load_w_block(int fmt, const void* w, size_t K, size_t n, size_t b)
{
    if (fmt == 8) return _mm256_loadu_si256((const __m256i*)((const int8_t*)w + n * K + b * BLK));
    const __m128i lo_mask = _mm_set1_epi8(0x0F);
    const __m256i eight = _mm256_set1_epi8(8);
    __m128i p = _mm_loadu_si128((const __m128i*)((const uint8_t*)w + n * (K / 2) + b * 16));
    __m128i lo = _mm_and_si128(p, lo_mask);
    __m128i hi = _mm_and_si128(_mm_srli_epi16(p, 4), lo_mask);
    __m256i v = _mm256_set_m128i(_mm_unpackhi_epi8(lo, hi), _mm_unpacklo_epi8(lo, hi));
    return _mm256_sub_epi8(_mm256_xor_si256(v, eight), eight);
}

__attribute__((target("avx2,avx512f,avx512bw,avx512vl,avx512vnni")))
static inline int32_t hsum8(__m256i d)
{
    __m128i s4 = _mm_add_epi32(_mm256_castsi256_si128(d), _mm256_extracti128_si256(d, 1));
    s4 = _mm_add_epi32(s4, _mm_shuffle_epi32(s4, 0x4E));
    s4 = _mm_add_epi32(s4, _mm_shuffle_epi32(s4, 0xB1));
    return _mm_cvtsi128_si32(s4);
}

/* Two blocks per _mm512_dpbusd_epi32 (u8 activations x s8 weights, 64 bytes
 * each); the low and high eight int32 lanes are the two blocks' dpbusd sums. */
__attribute__((target("avx2,avx512f,avx512bw,avx512vl,avx512vnni")))
static void gemv_vnni(int fmt, const uint8_t* xq, const uint8_t* xs,
                      const void* w, const uint8_t* ws, const int32_t* w_sums,
                      size_t B, size_t N, size_t K, float* y)
{
    size_t nb = K / BLK;
#pragma omp parallel for schedule(static)
    for (size_t n = 0; n < N; ++n) {
        for (size_t r = 0; r < B; ++r) {
            const uint8_t* x = xq + r * K;
            const uint8_t* sx = xs + r * nb;
            float acc = 0.0f;
            size_t b = 0;
            for (; b + 2 <= nb; b += 2) {
                __m512i vw = _mm512_inserti64x4(_mm512_castsi256_si512(load_w_block(fmt, w, K, n, b)),
                                                load_w_block(fmt, w, K, n, b + 1), 1);
                __m512i vx = _mm512_loadu_si512((const void*)(x + b * BLK));
                __m512i d = _mm512_dpbusd_epi32(_mm512_setzero_si512(), vx, vw);
                int32_t d0 = hsum8(_mm512_castsi512_si256(d)) - 128 * w_sums[n * nb + b];
                int32_t d1 = hsum8(_mm512_extracti64x4_epi64(d, 1)) - 128 * w_sums[n * nb + b + 1];
                acc += (float)d0 * pow2f_i((int)sx[b] + (int)ws[n * nb + b] - 254);
                acc += (float)d1 * pow2f_i((int)sx[b + 1] + (int)ws[n * nb + b + 1] - 254);
            }
            for (; b < nb; ++b) {
                __m256i vx = _mm256_loadu_si256((const __m256i*)(x + b * BLK));
                __m256i d = _mm256_dpbusd_epi32(_mm256_setzero_si256(), vx, load_w_block(fmt, w, K, n, b));
                int32_t dot = hsum8(d) - 128 * w_sums[n * nb + b];
                acc += (float)dot * pow2f_i((int)sx[b] + (int)ws[n * nb + b] - 254);
            }
            y[r * N + n] = acc;
        }
    }
}

static void gemv_portable(int fmt, const uint8_t* xq, const uint8_t* xs,
                          const void* w, const uint8_t* ws, const int32_t* w_sums,
                          size_t B, size_t N, size_t K, float* y)
{
    size_t nb = K / BLK;
#pragma omp parallel for schedule(static)
    for (size_t n = 0; n < N; ++n) {
        int8_t tmp[BLK];
        for (size_t r = 0; r < B; ++r) {
            const uint8_t* x = xq + r * K;
            float acc = 0.0f;
            for (size_t b = 0; b < nb; ++b) {
                const int8_t* p;
                if (fmt == 8) {
                    p = (const int8_t*)w + n * K + b * BLK;
                } else {
                    unpack_int4_scalar((const uint8_t*)w + n * (K / 2) + b * 16, tmp);
                    p = tmp;
                }
                int32_t d = 0;
                for (int i = 0; i < BLK; ++i) d += (int32_t)x[b * BLK + i] * p[i];
                d -= 128 * w_sums[n * nb + b];
                acc += (float)d * pow2f_i((int)xs[r * nb + b] + (int)ws[n * nb + b] - 254);
            }
            y[r * N + n] = acc;
        }
    }
}

/* Returns 1 when the VNNI kernel ran, 0 for the portable loop. */
int mxb_gemv(int fmt, const uint8_t* xq, const uint8_t* xs, const void* w,
             const uint8_t* ws, const int32_t* w_sums, size_t B, size_t N,
             size_t K, float* y, int nthreads)
{
    if (nthreads > 0) omp_set_num_threads(nthreads);
    if (__builtin_cpu_supports("avx512vnni") && __builtin_cpu_supports("avx512vl")) {
        gemv_vnni(fmt, xq, xs, w, ws, w_sums, B, N, K, y);
        return 1;
    }
    gemv_portable(fmt, xq, xs, w, ws, w_sums, B, N, K, y);
    return 0;
}

int mxb_max_threads(void) { return omp_get_max_threads(); }
