/*
 * mx_oracle.c -- CPU restatement of the reference's MX linear path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker).  Built with -ffp-contract=off so
 * that every float operation below is evaluated exactly as written; the GPU
 * kernels evaluate the quantiser's float steps with the same IEEE operations
 * (explicit round-to-nearest intrinsics), so quantised bytes agree bit for
 * bit.  See mx_oracle.h for the numeric conventions and reference citations.
 */
#include "mx_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------- E8M0 --- */

/* nn/core/layers/ssm.cpp:170 calls extract_e8m0(max_abs); its body is not in
 * the snapshot.  Here: the smallest integer e with max_abs <= qmax * 2^e, found
 * with exact double comparisons (qmax * 2^e is exact in double). */
uint8_t mxo_e8m0_from_absmax(float max_abs, int qmax)
{
    if (!(max_abs == max_abs) || isinf(max_abs)) return 0xFF;
    if (max_abs == 0.0f) return 0;
    double m = (double)max_abs;
    int e = (int)floor(log2(m / (double)qmax)) - 2;
    while (m > ldexp((double)qmax, e)) ++e;
    if (e < -127) e = -127;
    if (e > 127) e = 127;
    return (uint8_t)(e + 127);
}

/* nn/core/layers/ssm.cpp:171 decode_e8m0_scale: byte -> 2^(byte-127). */
double mxo_e8m0_decode(uint8_t s)
{
    if (s == 0xFF) return NAN;
    return ldexp(1.0, (int)s - 127);
}

/* ------------------------------------------------------ exp and SiLU --- */

/* exp(x) by Cody-Waite argument reduction (ln2 split into an exactly
 * representable high part and a correction, as in the fdlibm expf design)
 * followed by the degree-7 Taylor polynomial of e^r on |r| <= ln2/2,
 * evaluated by Horner's rule with fused multiply-adds.  2^n is applied by
 * building the IEEE exponent directly.  Every step is a single IEEE
 * operation so the GPU evaluates the same sequence to the same bits. */
static float pow2i(int n) /* 2^n for n in [-126, 127] */
{
    union { uint32_t u; float f; } v;
    v.u = (uint32_t)(n + 127) << 23;
    return v.f;
}

float mxo_expf(float x)
{
    const float LOG2E = 1.44269504088896341f;
    const float LN2_HI = 6.93145751953125e-1f;
    const float LN2_LO = 1.42860682030941723212e-6f;
    if (x != x) return x;
    if (x > 88.72283935546875f) return INFINITY;
    if (x < -103.972084045410f) return 0.0f;
    float t = x * LOG2E;
    float nf = rintf(t);
    int n = (int)nf;
    float r = fmaf(-nf, LN2_HI, x);
    r = fmaf(-nf, LN2_LO, r);
    float p = 1.0f / 5040.0f;
    p = fmaf(p, r, 1.0f / 720.0f);
    p = fmaf(p, r, 1.0f / 120.0f);
    p = fmaf(p, r, 1.0f / 24.0f);
    p = fmaf(p, r, 1.0f / 6.0f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    if (n > 127) {
        p = p * pow2i(n - 1);
        p = p * 2.0f;
    } else if (n < -126) {
        p = p * pow2i(n + 64);
        p = p * pow2i(-64);
    } else {
        p = p * pow2i(n);
    }
    return p;
}

/* SiLU as in nn/core/layers/ssm.cpp:159 (y / (1 + exp(-y))). */
float mxo_silu(float x)
{
    float e = mxo_expf(-x);
    float d = 1.0f + e;
    return x / d;
}

/* ----------------------------------------------------------- quantise --- */

/* One 32-element block: v[32] -> 32 bytes (q+128) + scale byte.
 * Follows nn/core/layers/ssm.cpp:164-177 with round-half-to-even
 * (the _mm512_cvtps_epi32 behaviour of nn/core/layers/ssm.cpp:249). */
static void quantize_block(const float* v, uint8_t* q, uint8_t* s)
{
    float max_abs = 0.0f;
    int finite = 1;
    for (int i = 0; i < MXO_BLOCK; ++i) {
        float a = fabsf(v[i]);
        if (!(a == a) || isinf(a)) finite = 0;
        else if (a > max_abs) max_abs = a;
    }
    if (!finite) {
        *s = 0xFF;
        memset(q, 128, MXO_BLOCK);
        return;
    }
    uint8_t sb = mxo_e8m0_from_absmax(max_abs, 127);
    *s = sb;
    int e = (int)sb - 127;
    float inv = pow2i(-e); /* e in [-127, 122] for finite float input */
    for (int i = 0; i < MXO_BLOCK; ++i) {
        float val = rintf(v[i] * inv);
        float c = val + 128.0f;
        if (c < 0.0f) c = 0.0f;
        if (c > 255.0f) c = 255.0f;
        q[i] = (uint8_t)c;
    }
}

void mxo_quantize_x(const float* x, size_t B, size_t K, int act,
                    uint8_t* q, uint8_t* s)
{
    float buf[MXO_BLOCK];
    size_t nb = K / MXO_BLOCK;
    for (size_t r = 0; r < B; ++r)
        for (size_t b = 0; b < nb; ++b) {
            const float* src = x + r * K + b * MXO_BLOCK;
            for (int i = 0; i < MXO_BLOCK; ++i)
                buf[i] = act == 1 ? mxo_silu(src[i]) : src[i];
            quantize_block(buf, q + r * K + b * MXO_BLOCK, s + r * nb + b);
        }
}

void mxo_swiglu_quantize(const float* gate, const float* up, size_t B, size_t K,
                         uint8_t* q, uint8_t* s)
{
    float buf[MXO_BLOCK];
    size_t nb = K / MXO_BLOCK;
    for (size_t r = 0; r < B; ++r)
        for (size_t b = 0; b < nb; ++b) {
            size_t o = r * K + b * MXO_BLOCK;
            for (int i = 0; i < MXO_BLOCK; ++i)
                buf[i] = mxo_silu(gate[o + i]) * up[o + i];
            quantize_block(buf, q + o, s + r * nb + b);
        }
}

/* ------------------------------------------------------------ weights --- */

int mxo_weight_at(int fmt, const void* data, size_t K, size_t n, size_t k)
{
    if (fmt == MXO_FMT_INT8) return ((const int8_t*)data)[n * K + k];
    uint8_t byte = ((const uint8_t*)data)[n * (K / 2) + k / 2];
    int nib = (k & 1) ? (byte >> 4) : (byte & 0xF);
    return nib >= 8 ? nib - 16 : nib;
}

void mxo_quantize_w(int fmt, const float* w, size_t N, size_t K,
                    void* data, uint8_t* scales, int32_t* w_sums)
{
    int qmax = fmt == MXO_FMT_INT8 ? 127 : 7;
    size_t nb = K / MXO_BLOCK;
    if (fmt == MXO_FMT_INT4) memset(data, 0, N * K / 2);
    for (size_t n = 0; n < N; ++n)
        for (size_t b = 0; b < nb; ++b) {
            const float* v = w + n * K + b * MXO_BLOCK;
            float max_abs = 0.0f;
            int finite = 1;
            for (int i = 0; i < MXO_BLOCK; ++i) {
                float a = fabsf(v[i]);
                if (!(a == a) || isinf(a)) finite = 0;
                else if (a > max_abs) max_abs = a;
            }
            if (!finite) {
                /* a block holding a NaN/inf: scale 0xFF, zero values (the
                 * activation quantiser's convention) */
                scales[n * nb + b] = 0xFF;
                if (fmt == MXO_FMT_INT8) memset((int8_t*)data + n * K + b * MXO_BLOCK, 0, MXO_BLOCK);
                if (w_sums) w_sums[n * nb + b] = 0;
                continue;
            }
            uint8_t sb = mxo_e8m0_from_absmax(max_abs, qmax);
            scales[n * nb + b] = sb;
            float inv = pow2i(127 - (int)sb);
            int32_t sum = 0;
            for (int i = 0; i < MXO_BLOCK; ++i) {
                int qv = (int)rintf(v[i] * inv);
                if (qv > qmax) qv = qmax;
                if (qv < -qmax) qv = -qmax;
                sum += qv;
                size_t k = b * MXO_BLOCK + i;
                if (fmt == MXO_FMT_INT8) {
                    ((int8_t*)data)[n * K + k] = (int8_t)qv;
                } else {
                    uint8_t* p = (uint8_t*)data + n * (K / 2) + k / 2;
                    uint8_t nib = (uint8_t)(qv & 0xF);
                    *p |= (k & 1) ? (uint8_t)(nib << 4) : nib;
                }
            }
            if (w_sums) w_sums[n * nb + b] = sum;
        }
}

/* --------------------------------------------------------------- dots --- */

/* The VNNI contract: dpbusd(u8 = q+128, s8 w) - 128 * w_sum == sum q*w.
 * The restatement computes sum q*w directly (identical integer). */
static int32_t block_dot(int fmt, const uint8_t* xq, const void* w, size_t K,
                         size_t n, size_t b)
{
    int32_t acc = 0;
    const uint8_t* x = xq + b * MXO_BLOCK;
    if (fmt == MXO_FMT_INT8) {
        const int8_t* wr = (const int8_t*)w + n * K + b * MXO_BLOCK;
        for (int i = 0; i < MXO_BLOCK; ++i) acc += ((int32_t)x[i] - 128) * (int32_t)wr[i];
    } else {
        const uint8_t* wr = (const uint8_t*)w + n * (K / 2) + b * (MXO_BLOCK / 2);
        for (int i = 0; i < MXO_BLOCK / 2; ++i) {
            int lo = wr[i] & 0xF, hi = wr[i] >> 4;
            lo = lo >= 8 ? lo - 16 : lo;
            hi = hi >= 8 ? hi - 16 : hi;
            acc += ((int32_t)x[2 * i] - 128) * lo + ((int32_t)x[2 * i + 1] - 128) * hi;
        }
    }
    return acc;
}

void mxo_block_dots(int fmt, const uint8_t* xq, const void* w, size_t B,
                    size_t N, size_t K, int32_t* out)
{
    size_t nb = K / MXO_BLOCK;
    for (size_t r = 0; r < B; ++r)
        for (size_t n = 0; n < N; ++n)
            for (size_t b = 0; b < nb; ++b)
                out[(r * N + n) * nb + b] = block_dot(fmt, xq + r * K, w, K, n, b);
}

static float row_dot(int fmt, const uint8_t* xq, const uint8_t* xs,
                     const void* w, const uint8_t* ws, size_t K, size_t n)
{
    size_t nb = K / MXO_BLOCK;
    double acc = 0.0;
    for (size_t b = 0; b < nb; ++b) {
        uint8_t sx = xs[b], sw = ws[n * nb + b];
        int32_t d = block_dot(fmt, xq, w, K, n, b);
        if (sx == 0xFF || sw == 0xFF) { acc = NAN; continue; }
        acc += ldexp((double)d, (int)sx + (int)sw - 254);
    }
    return (float)acc;
}

void mxo_gemv(int fmt, const uint8_t* xq, const uint8_t* xs, const void* w,
              const uint8_t* ws, size_t B, size_t N, size_t K, float* y)
{
    size_t nb = K / MXO_BLOCK;
    /* rows are independent: the threads change no result */
    #pragma omp parallel for schedule(static) collapse(2)
    for (size_t r = 0; r < B; ++r)
        for (size_t n = 0; n < N; ++n)
            y[r * N + n] = row_dot(fmt, xq + r * K, xs + r * nb, w, ws, K, n);
}

void mxo_gather_dot(int fmt, const uint8_t* xq, const uint8_t* xs,
                    const void* w, const uint8_t* ws, size_t K,
                    const int32_t* rows, size_t nrows, size_t B, float* y)
{
    size_t nb = K / MXO_BLOCK;
    #pragma omp parallel for schedule(static) collapse(2)
    for (size_t r = 0; r < B; ++r)
        for (size_t j = 0; j < nrows; ++j)
            y[r * nrows + j] = row_dot(fmt, xq + r * K, xs + r * nb, w, ws, K,
                                       (size_t)rows[j]);
}

/* ------------------------------------ fixed-order fp32 row dots ------- */

/* 2^n for n in [-149, 127], exact (denormals included). */
static float pow2x(int n) { return ldexpf(1.0f, n); }

static float e8m0_f32(uint8_t s) { return s == 0xFF ? NAN : pow2x((int)s - 127); }

/* The GPU's one-warp row dot: lane l sums, in fp32 and block order, the
 * terms (d_b * 2^e_x,b) * 2^e_w,b of blocks b = l, l+32, ...; the 32 lane sums
 * are combined by the xor-butterfly v_l += v_(l^o), o = 16, 8, 4, 2, 1. */
static float lane_tree_dot(int fmt, const uint8_t* xq, const uint8_t* xs, const void* w,
                           const uint8_t* ws, size_t K, size_t n)
{
    size_t nb = K / MXO_BLOCK;
    float v[32];
    for (int l = 0; l < 32; ++l) v[l] = 0.0f;
    for (size_t b = 0; b < nb; ++b) {
        int32_t d = block_dot(fmt, xq, w, K, n, b);
        float t = ((float)d * e8m0_f32(xs[b])) * e8m0_f32(ws[n * nb + b]);
        v[b % 32] = v[b % 32] + t;
    }
    for (int o = 16; o > 0; o >>= 1) {
        float u[32];
        for (int l = 0; l < 32; ++l) u[l] = v[l] + v[l ^ o];
        for (int l = 0; l < 32; ++l) v[l] = u[l];
    }
    return v[0];
}

void mxo_rank16_dot_ptrs(int fmt, const uint8_t* xq, const uint8_t* xs,
                         const void* const* rows, const uint8_t* const* row_scales,
                         size_t nrows, size_t B, size_t K, float* y)
{
    size_t nb = K / MXO_BLOCK;
    for (size_t r = 0; r < B; ++r)
        for (size_t j = 0; j < nrows; ++j)
            y[r * nrows + j] = lane_tree_dot(fmt, xq + r * K, xs + r * nb, rows[j], row_scales[j], K, 0);
}

/* ACT halting (Graves 2016) over B tokens with the GPU's operation order. */
void mxo_halting_step(int fmt, const uint8_t* xq, const uint8_t* xs, const void* w,
                      const uint8_t* ws, size_t B, size_t K, float bias, float eps,
                      float* p_sum, float* remainder, uint64_t* steps, float* p, uint8_t* halt)
{
    size_t nb = K / MXO_BLOCK;
    for (size_t r = 0; r < B; ++r) {
        float z = lane_tree_dot(fmt, xq + r * K, xs + r * nb, w, ws, K, 0) + bias;
        float pr = 1.0f / (1.0f + mxo_expf(-z));
        steps[r] += 1;
        int h = p_sum[r] + pr >= 1.0f - eps;
        if (h) {
            remainder[r] = 1.0f - p_sum[r];
            p_sum[r] = 1.0f;
        } else {
            p_sum[r] = p_sum[r] + pr;
        }
        p[r] = pr;
        halt[r] = (uint8_t)h;
    }
}

/* mx_update_gaussian_moment as the library states it: w = clamp(rint(w +
 * ((step * g[n]) * x[k]) * 2^-e), lo, hi), scales kept, blocks with scale
 * 0xFF untouched; data in the MXINT8Tensor layout, updated in place. */
void mxo_update_gaussian_moment(int fmt, void* data, const uint8_t* scales, size_t N, size_t K,
                                const float* g, const float* x, float step)
{
    size_t nb = K / MXO_BLOCK;
    int lo = fmt == MXO_FMT_INT4 ? -8 : -127, hi = fmt == MXO_FMT_INT4 ? 7 : 127;
    for (size_t n = 0; n < N; ++n) {
        float gn = step * g[n];
        for (size_t k = 0; k < K; ++k) {
            uint8_t s = scales[n * nb + k / MXO_BLOCK];
            if (s == 0xFF) continue;
            int old = mxo_weight_at(fmt, data, K, n, k);
            float delta = (gn * x[k]) * pow2x(127 - (int)s);
            float r = rintf((float)old + delta);
            int q = r < (float)lo ? lo : (r > (float)hi ? hi : (int)r);
            if (fmt == MXO_FMT_INT8) {
                ((int8_t*)data)[n * K + k] = (int8_t)q;
            } else {
                uint8_t* p = (uint8_t*)data + n * (K / 2) + k / 2;
                *p = (k & 1) ? (uint8_t)((*p & 0x0F) | ((q & 0xF) << 4)) : (uint8_t)((*p & 0xF0) | (q & 0xF));
            }
        }
    }
}

/* ||dequant(x_b)||_2 in the GPU's order (lanes, then the butterfly). */
void mxo_activation_norm(const uint8_t* xq, const uint8_t* xs, size_t B, size_t K, float* out)
{
    size_t nb = K / MXO_BLOCK;
    for (size_t r = 0; r < B; ++r) {
        float v[32];
        for (int l = 0; l < 32; ++l) v[l] = 0.0f;
        for (size_t b = 0; b < nb; ++b) {
            int32_t ss = 0;
            for (int i = 0; i < MXO_BLOCK; ++i) {
                int q = (int)xq[r * K + b * MXO_BLOCK + i] - 128;
                ss += q * q;
            }
            float sc = e8m0_f32(xs[r * nb + b]);
            v[b % 32] = v[b % 32] + ((float)ss * sc) * sc;
        }
        for (int o = 16; o > 0; o >>= 1) {
            float u[32];
            for (int l = 0; l < 32; ++l) u[l] = v[l] + v[l ^ o];
            for (int l = 0; l < 32; ++l) v[l] = u[l];
        }
        out[r] = sqrtf(v[0]);
    }
}

/* The micro-expert layer in the GPU's operation order (see mxq_micro_moe):
 * per token, x quantised; each chosen expert's 16 gate and 16 up row dots by
 * lane_tree_dot; h = silu(g) * u * weight placed in the down pool's 32-blocks
 * and quantised; y[j] = sum over the chosen blocks, ascending, of
 * (d * 2^e_h) * 2^e_w in fp32.  Pools in the MXINT8Tensor layout. */
void mxo_micro_moe(int fmt, const void* wg, const uint8_t* sg, const void* wu, const uint8_t* su,
                   const void* wd, const uint8_t* sd, size_t n_routed, size_t n_shared, size_t D,
                   const float* x, const int32_t* idx, const float* gate, size_t T, size_t k, float* y)
{
    size_t E = n_routed + n_shared, nsel = k + n_shared, KD = E * 16;
    size_t rb = fmt == MXO_FMT_INT4 ? D / 2 : D;          /* bytes per pool row */
    uint8_t* xq = (uint8_t*)malloc(D);
    uint8_t* xs = (uint8_t*)malloc(D / 32);
    float* hv = (float*)malloc(nsel * 32 * sizeof(float));
    int* sel = (int*)malloc(nsel * sizeof(int));
    float* wsel = (float*)malloc(nsel * sizeof(float));
    int* blk = (int*)malloc(nsel * sizeof(int));
    uint8_t* hq = (uint8_t*)malloc(nsel * 32);
    uint8_t* hs = (uint8_t*)malloc(nsel);
    float blkv[32];
    for (size_t t = 0; t < T; ++t) {
        mxo_quantize_x(x + t * D, 1, D, 0, xq, xs);
        for (size_t s = 0; s < nsel; ++s) {
            int e = s < k ? idx[t * k + s] : (int)(n_routed + (s - k));
            if (s < k) e = e < 0 ? 0 : (e >= (int)n_routed ? (int)n_routed - 1 : e);
            sel[s] = e;
            wsel[s] = s < k ? (gate ? gate[t * k + s] : 1.0f) : 1.0f;
            for (int j = 0; j < 16; ++j) {
                size_t row = (size_t)e * 16 + j;
                const uint8_t* pg = (const uint8_t*)wg + row * rb;
                const uint8_t* pu = (const uint8_t*)wu + row * rb;
                hv[s * 32 + j] = lane_tree_dot(fmt, xq, xs, pg, sg + row * (D / 32), D, 0);
                hv[s * 32 + 16 + j] = lane_tree_dot(fmt, xq, xs, pu, su + row * (D / 32), D, 0);
            }
        }
        size_t nb = 0;
        for (size_t s = 0; s < nsel; ++s) {
            int b = sel[s] >> 1;
            size_t pos = 0;
            while (pos < nb && blk[pos] < b) ++pos;
            if (pos < nb && blk[pos] == b) continue;
            for (size_t q = nb; q > pos; --q) blk[q] = blk[q - 1];
            blk[pos] = b;
            ++nb;
        }
        for (size_t i = 0; i < nb; ++i) {
            for (int l = 0; l < 32; ++l) {
                int e = blk[i] * 2 + (l >> 4), slot = l & 15;
                float v = 0.0f;
                for (size_t s = 0; s < nsel; ++s)
                    if (sel[s] == e) v = (mxo_silu(hv[s * 32 + slot]) * hv[s * 32 + 16 + slot]) * wsel[s];
                blkv[l] = v;
            }
            mxo_quantize_x(blkv, 1, 32, 0, hq + i * 32, hs + i);
        }
        for (size_t j = 0; j < D; ++j) {
            float acc = 0.0f;
            for (size_t i = 0; i < nb; ++i) {
                int32_t d = 0;
                for (int l = 0; l < 32; ++l)
                    d += ((int32_t)hq[i * 32 + l] - 128) * mxo_weight_at(fmt, wd, KD, j, (size_t)blk[i] * 32 + l);
                acc = acc + ((float)d * e8m0_f32(hs[i])) * e8m0_f32(sd[j * (KD / 32) + blk[i]]);
            }
            y[t * D + j] = acc;
        }
    }
    free(xq); free(xs); free(hv); free(sel); free(wsel); free(blk); free(hq); free(hs);
}

/* splitmix64 finaliser (the router's hyperplane and code generator) */
static uint64_t mix64(uint64_t z)
{
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

int mxo_hashed_route(const float* x, size_t T, size_t D, size_t E, size_t K, size_t H,
                     uint64_t seed, int32_t* idx, int32_t* score)
{
    if (K == 0 || K > E || H == 0 || H > 32 || D % MXO_BLOCK) return -1;
    size_t nb = D / MXO_BLOCK;
    uint8_t q[MXO_BLOCK], sb;
    uint32_t mask = H == 32 ? 0xFFFFFFFFu : ((1u << H) - 1u);
    for (size_t t = 0; t < T; ++t) {
        float proj[32] = {0};
        for (size_t b = 0; b < nb; ++b) {
            const float* xb = x + t * D + b * MXO_BLOCK;
            int any = 0;
            for (int i = 0; i < MXO_BLOCK; ++i) any |= xb[i] != 0.0f;
            quantize_block(xb, q, &sb);
            if (!any || sb == 0xFF) continue;   /* a zero block adds nothing; a non-finite one is skipped */
            float sx = pow2x((int)sb - 127);
            for (size_t h = 0; h < H; ++h) {
                int32_t d = 0;
                for (int i = 0; i < MXO_BLOCK; ++i) {
                    size_t k = b * MXO_BLOCK + i;
                    uint64_t rr = mix64(seed ^ ((uint64_t)(h + 1) << 40) ^ (uint64_t)(k >> 6));
                    int sg = ((rr >> (k & 63)) & 1ull) ? 1 : -1;
                    d += ((int32_t)q[i] - 128) * sg;
                }
                proj[h] = proj[h] + (float)d * sx;
            }
        }
        uint32_t code = 0;
        for (size_t h = 0; h < H; ++h)
            if (proj[h] > 0.0f) code |= 1u << h;
        int32_t chosen[64];
        for (size_t j = 0; j < K; ++j) {
            int best = -1, bs = -1;
            for (size_t e = 0; e < E; ++e) {
                int used = 0;
                for (size_t p2 = 0; p2 < j; ++p2) used |= chosen[p2] == (int32_t)e;
                if (used) continue;
                uint32_t ce = (uint32_t)mix64(seed ^ 0xC0DEC0DEull ^ ((uint64_t)e << 20)) & mask;
                int sc = (int)H - __builtin_popcount((code ^ ce) & mask);
                if (sc > bs) { bs = sc; best = (int)e; }
            }
            chosen[j] = best;
            idx[t * K + j] = best;
            score[t * K + j] = bs;
        }
    }
    return 0;
}

/* ---------------------------------------------------------------- MLP --- */

static void mlp_from_q(int fmt, const uint8_t* xq, const uint8_t* xs, size_t B,
                       size_t D, size_t F, const void* wg, const uint8_t* sg,
                       const void* wu, const uint8_t* su, const void* wd,
                       const uint8_t* sd, float* y, uint8_t* mid_q,
                       uint8_t* mid_s)
{
    float* g = (float*)malloc(B * F * sizeof(float));
    float* u = (float*)malloc(B * F * sizeof(float));
    uint8_t* hq = mid_q ? mid_q : (uint8_t*)malloc(B * F);
    uint8_t* hs = mid_s ? mid_s : (uint8_t*)malloc(B * F / MXO_BLOCK);
    mxo_gemv(fmt, xq, xs, wg, sg, B, F, D, g);
    mxo_gemv(fmt, xq, xs, wu, su, B, F, D, u);
    mxo_swiglu_quantize(g, u, B, F, hq, hs);
    mxo_gemv(fmt, hq, hs, wd, sd, B, D, F, y);
    free(g);
    free(u);
    if (!mid_q) free(hq);
    if (!mid_s) free(hs);
}

void mxo_mlp_swiglu(int fmt, const float* x, size_t B, size_t D, size_t F,
                    const void* wg, const uint8_t* sg, const void* wu,
                    const uint8_t* su, const void* wd, const uint8_t* sd,
                    float* y, uint8_t* mid_q, uint8_t* mid_s)
{
    uint8_t* xq = (uint8_t*)malloc(B * D);
    uint8_t* xs = (uint8_t*)malloc(B * D / MXO_BLOCK);
    mxo_quantize_x(x, B, D, 0, xq, xs);
    mlp_from_q(fmt, xq, xs, B, D, F, wg, sg, wu, su, wd, sd, y, mid_q, mid_s);
    free(xq);
    free(xs);
}

/* ------------------------------------------------------------ routing --- */

int mxo_route_topk(const float* logits, size_t T, size_t E, size_t k,
                   int32_t* idx, float* gate)
{
    if (k == 0 || k > E || k > 64) return -1;
    for (size_t t = 0; t < T; ++t) {
        const float* l = logits + t * E;
        int32_t* id = idx + t * k;
        for (size_t j = 0; j < k; ++j) {
            int best = -1;
            for (size_t e = 0; e < E; ++e) {
                int used = 0;
                for (size_t p = 0; p < j; ++p) used |= id[p] == (int32_t)e;
                if (used) continue;
                if (best < 0 || l[e] > l[best]) best = (int)e;
            }
            id[j] = best;
        }
        /* softmax over the chosen logits; the first is the maximum */
        float mx = l[id[0]];
        float ex[64];
        float den = 0.0f;
        for (size_t j = 0; j < k; ++j) {
            ex[j] = mxo_expf(l[id[j]] - mx);
            den = den + ex[j];
        }
        for (size_t j = 0; j < k; ++j) gate[t * k + j] = ex[j] / den;
    }
    return 0;
}

/* ---------------------------------------------------------------- MoE --- */

int mxo_moe(int fmt, const float* x, const float* logits, size_t T, size_t D,
            size_t F, size_t E, size_t k, const void* const* wg,
            const uint8_t* const* sg, const void* const* wu,
            const uint8_t* const* su, const void* const* wd,
            const uint8_t* const* sd, float* y)
{
    int32_t* idx = (int32_t*)malloc(T * k * sizeof(int32_t));
    float* gate = (float*)malloc(T * k * sizeof(float));
    if (mxo_route_topk(logits, T, E, k, idx, gate) != 0) {
        free(idx);
        free(gate);
        return -1;
    }
    uint8_t* xq = (uint8_t*)malloc(D);
    uint8_t* xs = (uint8_t*)malloc(D / MXO_BLOCK);
    float* out = (float*)malloc(D * sizeof(float));
    double* acc = (double*)malloc(D * sizeof(double));
    for (size_t t = 0; t < T; ++t) {
        mxo_quantize_x(x + t * D, 1, D, 0, xq, xs);
        for (size_t d = 0; d < D; ++d) acc[d] = 0.0;
        for (size_t j = 0; j < k; ++j) {
            int e = idx[t * k + j];
            mlp_from_q(fmt, xq, xs, 1, D, F, wg[e], sg[e], wu[e], su[e], wd[e],
                       sd[e], out, NULL, NULL);
            for (size_t d = 0; d < D; ++d)
                acc[d] += (double)gate[t * k + j] * (double)out[d];
        }
        for (size_t d = 0; d < D; ++d) y[t * D + d] = (float)acc[d];
    }
    free(idx);
    free(gate);
    free(xq);
    free(xs);
    free(out);
    free(acc);
    return 0;
}

/* ------------------------------------------------------- policy head --- */

/* training/ppo_trainer.cpp:64-66 (log_softmax, action log-probability) and
 * :77 (entropy), one row at a time. */
void mxo_policy_head(const float* logits, const float* actions, size_t rows,
                     size_t cols, float* log_probs, float* action_logp,
                     float* entropy)
{
    for (size_t r = 0; r < rows; ++r) {
        const float* x = logits + r * cols;
        const float* a = actions + r * cols;
        float* lp = log_probs + r * cols;
        float m = x[0];
        for (size_t j = 1; j < cols; ++j) m = x[j] > m ? x[j] : m;
        float s = 0.0f;
        for (size_t j = 0; j < cols; ++j) s = s + mxo_expf(x[j] - m);
        const float lse = m + logf(s);
        float alp = 0.0f, ent = 0.0f;
        for (size_t j = 0; j < cols; ++j) {
            lp[j] = x[j] - lse;
            alp = alp + lp[j] * a[j];
            ent = ent - mxo_expf(lp[j]) * lp[j];
        }
        action_logp[r] = alp;
        entropy[r] = ent;
    }
}

/* ---------------------------------------------------------------- GAE --- */

/* agentic_env/replay_memory.cpp:204-253, same operation order per element. */
/* ReplayMemory::fused_compute_gae on the ring buffer itself
 * (agentic_env/replay_memory.cpp:204-253): the latest T*E items ending at
 * the write cursor (T cut to size/E when fewer are stored), at most the
 * first 1024 environments (the reference's MAX_ENVS), indices wrapping at
 * the capacity.  Entries outside that window are not written. */
void mxo_gae_ring(const float* rewards, const float* values, const uint8_t* dones,
                  const float* next_values, size_t cap, size_t size, size_t cursor,
                  size_t T, size_t E, float gamma, float lambda, float* adv, float* ret)
{
    size_t total = T * E;
    if (total == 0 || size == 0) return;
    if (total > size) {
        T = size / E;
        total = T * E;
    }
    size_t start = (cap + cursor - total) % cap;
    size_t active = E > 1024 ? 1024 : E;
    float gl = gamma * lambda;
    float* acc = (float*)calloc(active ? active : 1, sizeof(float));
    float* vn = (float*)malloc((active ? active : 1) * sizeof(float));
    memcpy(vn, next_values, active * sizeof(float));
    for (size_t tt = T; tt-- > 0;) {
        for (size_t k = 0; k < active; ++k) {
            size_t i = start + tt * E + k;
            if (i >= cap) i -= cap;
            float done_f = dones[i] ? 0.0f : 1.0f;
            float delta = rewards[i] + gamma * vn[k] * done_f - values[i];
            acc[k] = delta + gl * acc[k] * done_f;
            adv[i] = acc[k];
            ret[i] = acc[k] + values[i];
            vn[k] = values[i];
        }
    }
    free(acc);
    free(vn);
}

void mxo_gae(const float* rewards, const float* values, const uint8_t* dones,
             const float* next_values, size_t T, size_t E, float gamma,
             float lambda, float* adv, float* ret)
{
    float gl = gamma * lambda;
    float* acc = (float*)calloc(E, sizeof(float));
    float* vn = (float*)malloc(E * sizeof(float));
    memcpy(vn, next_values, E * sizeof(float));
    for (size_t tt = T; tt-- > 0;) {
        for (size_t k = 0; k < E; ++k) {
            size_t i = tt * E + k;
            float done_f = dones[i] ? 0.0f : 1.0f;
            float delta = rewards[i] + gamma * vn[k] * done_f - values[i];
            acc[k] = delta + gl * acc[k] * done_f;
            adv[i] = acc[k];
            ret[i] = acc[k] + values[i];
            vn[k] = values[i];
        }
    }
    free(acc);
    free(vn);
}
