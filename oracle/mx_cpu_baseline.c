/*
 * mx_cpu_baseline.c -- multi-threaded CPU restatement of the reference's
 * removed AVX-512 VNNI MX GEMV (nn/core/simd/avx512_vnni.hpp, absent from the
 * snapshot; design described in nn/user.md:17 and
 * research_paper/HARDWARE_SATURATION.md:7-13): _mm512_dpbusd_epi32 over u8
 * activations (q+128) and s8 weights, two 32-element blocks per instruction,
 * each block scaled by 2^(e_x + e_w) in fp32 vector lanes with the
 * 128 * w_sum correction per block.  OpenMP over output rows.
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
 * each).  The 16 int32 lanes are converted to float and multiplied by their
 * block's scale 2^(e_x + e_w) into a float accumulator vector; the w_sums
 * correction (-128 * w_sum * scale per block) goes into a scalar; one
 * horizontal sum per output. */
__attribute__((target("avx2,avx512f,avx512bw,avx512vl,avx512vnni")))
static void gemv_vnni(int fmt, const uint8_t* xq, const uint8_t* xs,
                      const void* w, const uint8_t* ws, const int32_t* w_sums,
                      size_t B, size_t N, size_t K, float* y)
{
    size_t nb = K / BLK;
    const __m256i lo_mask = _mm256_set1_epi8(0x0F);
    const __m512i eight = _mm512_set1_epi8(8);
#pragma omp parallel for schedule(static)
    for (size_t n = 0; n < N; ++n) {
        const int32_t* zs = w_sums + n * nb;
        const uint8_t* sw = ws + n * nb;
        for (size_t r = 0; r < B; ++r) {
            const uint8_t* x = xq + r * K;
            const uint8_t* sx = xs + r * nb;
            __m512 acc = _mm512_setzero_ps();
            float corr = 0.0f;
            size_t b = 0;
            for (; b + 2 <= nb; b += 2) {
                __m512i vw, vx = _mm512_loadu_si512((const void*)(x + b * BLK));
                __mmask16 second;
                if (fmt == 8) {
                    /* natural order: lanes 0-7 block b, 8-15 block b+1 */
                    vw = _mm512_loadu_si512((const void*)((const int8_t*)w + n * K + b * BLK));
                    second = 0xFF00;
                } else {
                    /* [b:0-15 | b+1:0-15 | b:16-31 | b+1:16-31]; x's 16-byte
                     * chunks reordered to match: lanes 4-7 and 12-15 block b+1 */
                    __m256i p = _mm256_loadu_si256((const __m256i*)((const uint8_t*)w + n * (K / 2) + b * 16));
                    __m256i lo = _mm256_and_si256(p, lo_mask);
                    __m256i hi = _mm256_and_si256(_mm256_srli_epi16(p, 4), lo_mask);
                    vw = _mm512_inserti64x4(_mm512_castsi256_si512(_mm256_unpacklo_epi8(lo, hi)),
                                            _mm256_unpackhi_epi8(lo, hi), 1);
                    vw = _mm512_sub_epi8(_mm512_xor_si512(vw, eight), eight);
                    vx = _mm512_shuffle_i64x2(vx, vx, _MM_SHUFFLE(3, 1, 2, 0));
                    second = 0xF0F0;
                }
                const __m512i d = _mm512_dpbusd_epi32(_mm512_setzero_si512(), vx, vw);
                const float s0 = pow2f_i((int)sx[b] + (int)sw[b] - 254);
                const float s1 = pow2f_i((int)sx[b + 1] + (int)sw[b + 1] - 254);
                const __m512 sc = _mm512_mask_blend_ps(second, _mm512_set1_ps(s0), _mm512_set1_ps(s1));
                acc = _mm512_fmadd_ps(_mm512_cvtepi32_ps(d), sc, acc);
                corr += (float)(-128 * zs[b]) * s0 + (float)(-128 * zs[b + 1]) * s1;
            }
            float tail = 0.0f;
            for (; b < nb; ++b) {
                __m256i vx = _mm256_loadu_si256((const __m256i*)(x + b * BLK));
                __m256i d = _mm256_dpbusd_epi32(_mm256_setzero_si256(), vx, load_w_block(fmt, w, K, n, b));
                tail += (float)(hsum8(d) - 128 * zs[b]) * pow2f_i((int)sx[b] + (int)sw[b] - 254);
            }
            y[r * N + n] = _mm512_reduce_add_ps(acc) + corr + tail;
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
