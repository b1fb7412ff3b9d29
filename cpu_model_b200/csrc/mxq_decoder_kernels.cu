// mxq_decoder_kernels.cu -- the non-linear steps of the dense decoder that
// the MX linears plug into (mxq_decoder.cu): token embedding, RMSNorm
// (nn/core/normalization.cpp:16-47: out = in * (1 / sqrt(sum(in^2) / n +
// eps)) * weight), rotary position embedding with K/V written to a bf16 cache,
// causal attention for whole prompts (tiled, online softmax) and for one new
// token per sequence (split over the context, then combined), SwiGLU,
// residual adds, per-token log-probabilities.
//
// Every reduction runs in a fixed order and exp is the library's
// deterministic det_expf, so a forward pass is bit-reproducible.
#include "mxq_internal.h"

namespace mxq {

namespace {

// Every kernel here waits for its predecessor's results (programmatic
// dependent launch) and lets its own dependents launch at once: the MX
// linear that follows streams its weights while this kernel runs, and reads
// this kernel's output only after its own wait.
#define DK_PDL_PROLOGUE()                                   \
  asm volatile("griddepcontrol.wait;" ::: "memory");        \
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory")

// ------------------------------------------------------------ embedding ---
__global__ void embed_kernel(const int32_t* __restrict__ tok, const float* __restrict__ table, int R, int d,
                             int vocab, float* __restrict__ h) {
  DK_PDL_PROLOGUE();
  const int r = blockIdx.x;
  if (r >= R) return;
  int t = tok[r];
  t = t < 0 ? 0 : (t >= vocab ? vocab - 1 : t);
  const float4* src = reinterpret_cast<const float4*>(table + (size_t)t * d);
  float4* dst = reinterpret_cast<float4*>(h + (size_t)r * d);
  for (int i = threadIdx.x; i < d / 4; i += blockDim.x) dst[i] = src[i];
}

// --------------------------------------------------------------- RMSNorm ---
// One CTA of 1024 threads per row, each thread a few float4 chunks held in
// registers (one pass over memory), the square sum in a fixed tree: the
// per-thread chunks in order, the 32 lanes by a xor-butterfly, the 32 warps
// in order.  kNormVec chunks per thread cover d <= 16384.
constexpr int kNormThreads = 1024, kNormVec = 4;

__device__ __forceinline__ float norm_block_sum(float s, float* ws) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
  if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = s;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int w = 0; w < kNormThreads / 32; ++w) tot = __fadd_rn(tot, ws[w]);
  return tot;
}

// RESID: h += y first (written back), then out = RMSNorm(h) * g.  y's row r
// is `nparts` partial sums of d values side by side (y + r * y_ld), added
// in order before the residual (one part: h + y).
template <bool RESID>
__global__ void __launch_bounds__(kNormThreads) norm_kernel(float* __restrict__ h, const float* __restrict__ y,
                                                            const float* __restrict__ g, int d, float eps,
                                                            float* __restrict__ out, int nparts, size_t y_ld) {
  DK_PDL_PROLOGUE();
  __shared__ float ws[kNormThreads / 32];
  const int r = blockIdx.x, d4 = d / 4;
  float4* hr = reinterpret_cast<float4*>(h + (size_t)r * d);
  const float4* yr = reinterpret_cast<const float4*>(y + (size_t)r * y_ld);
  float4 v[kNormVec];
  float s = 0.0f;
#pragma unroll
  for (int u = 0; u < kNormVec; ++u) {
    const int i = threadIdx.x + u * kNormThreads;
    v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (i < d4) {
      v[u] = hr[i];
      if (RESID) {
        float4 b = yr[i];
        for (int q = 1; q < nparts; ++q) {
          const float4 c = yr[(size_t)q * d4 + i];
          b.x = __fadd_rn(b.x, c.x);
          b.y = __fadd_rn(b.y, c.y);
          b.z = __fadd_rn(b.z, c.z);
          b.w = __fadd_rn(b.w, c.w);
        }
        v[u].x = __fadd_rn(v[u].x, b.x);
        v[u].y = __fadd_rn(v[u].y, b.y);
        v[u].z = __fadd_rn(v[u].z, b.z);
        v[u].w = __fadd_rn(v[u].w, b.w);
        hr[i] = v[u];
      }
    }
    s = __fmaf_rn(v[u].x, v[u].x, s);
    s = __fmaf_rn(v[u].y, v[u].y, s);
    s = __fmaf_rn(v[u].z, v[u].z, s);
    s = __fmaf_rn(v[u].w, v[u].w, s);
  }
  const float tot = norm_block_sum(s, ws);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)d), eps)));
  float4* o = reinterpret_cast<float4*>(out + (size_t)r * d);
  const float4* g4 = reinterpret_cast<const float4*>(g);
#pragma unroll
  for (int u = 0; u < kNormVec; ++u) {
    const int i = threadIdx.x + u * kNormThreads;
    if (i < d4) {
      const float4 gg = g4[i];
      o[i] = make_float4(__fmul_rn(__fmul_rn(v[u].x, inv), gg.x), __fmul_rn(__fmul_rn(v[u].y, inv), gg.y),
                         __fmul_rn(__fmul_rn(v[u].z, inv), gg.z), __fmul_rn(__fmul_rn(v[u].w, inv), gg.w));
    }
  }
}

// The exchange of the tensor-parallel decoder's partial sums fused into the
// residual + RMSNorm (ExchNormArgs).  Waits only on the other GPUs' flags:
// a rank's own CTAs never wait on each other, and with at most one CTA a
// row and kExchNormMaxRows rows every CTA of the grid fits on the GPU at
// once, so each rank's flag is set whatever the others do.
__global__ void __launch_bounds__(kNormThreads) exch_norm_kernel(ExchNormArgs a) {
  DK_PDL_PROLOGUE();
  __shared__ float ws[kNormThreads / 32];
  __shared__ uint32_t next_s;
  __shared__ int ok_s;
  const int r = blockIdx.x, d4 = a.d / 4;
  if (threadIdx.x == 0) next_s = *a.seq + 1u;     // read before this CTA arrives on the counter
  const float4* yo = reinterpret_cast<const float4*>(a.y_own + (size_t)r * a.d);
  float4 own[kNormVec];
  const size_t row_off = a.slot_off + ((size_t)r * a.world + a.rank) * a.d * 4;
#pragma unroll
  for (int u = 0; u < kNormVec; ++u) {
    const int i = threadIdx.x + u * kNormThreads;
    own[u] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (i < d4) {
      own[u] = yo[i];
      for (int q = 0; q < a.world; ++q)
        if (q != a.rank) *reinterpret_cast<float4*>(a.base[q] + row_off + (size_t)i * 16) = own[u];
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t next = next_s;
    __threadfence();
    const unsigned old = atomicAdd(a.grid_cnt, 1u);
    if (old == gridDim.x - 1u) {
      *a.grid_cnt = 0u;
      if (a.world > 1) {
        asm volatile("fence.acq_rel.sys;" ::: "memory");
        for (int q = 0; q < a.world; ++q)
          if (q != a.rank) st_release_sys(a.flag_out[q], next);
      }
      *a.seq = next;
    }
    ok_s = a.world == 1 ||
           peer_wait_others(a.wait_flags, a.world, a.rank, next, a.wait_ns ? a.wait_ns : kWaitLimitNs, a.status);
  }
  __syncthreads();
  // partial sums in rank order (this rank's from registers), then the residual
  float4* hr = reinterpret_cast<float4*>(a.h + (size_t)r * a.d);
  const float4* mb = reinterpret_cast<const float4*>(a.base[a.rank] + a.slot_off + (size_t)r * a.world * a.d * 4);
  float4 v[kNormVec];
  float s = 0.0f;
#pragma unroll
  for (int u = 0; u < kNormVec; ++u) {
    const int i = threadIdx.x + u * kNormThreads;
    v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (i < d4) {
      float4 b = a.rank == 0 ? own[u] : __ldcg(mb + i);
      for (int q = 1; q < a.world; ++q) {
        const float4 c = q == a.rank ? own[u] : __ldcg(mb + (size_t)q * d4 + i);
        b.x = __fadd_rn(b.x, c.x);
        b.y = __fadd_rn(b.y, c.y);
        b.z = __fadd_rn(b.z, c.z);
        b.w = __fadd_rn(b.w, c.w);
      }
      if (!ok_s) b = make_float4(0.f, 0.f, 0.f, 0.f);   // a timed-out exchange: the status word reports it
      v[u] = hr[i];
      v[u].x = __fadd_rn(v[u].x, b.x);
      v[u].y = __fadd_rn(v[u].y, b.y);
      v[u].z = __fadd_rn(v[u].z, b.z);
      v[u].w = __fadd_rn(v[u].w, b.w);
      hr[i] = v[u];
    }
    s = __fmaf_rn(v[u].x, v[u].x, s);
    s = __fmaf_rn(v[u].y, v[u].y, s);
    s = __fmaf_rn(v[u].z, v[u].z, s);
    s = __fmaf_rn(v[u].w, v[u].w, s);
  }
  const float tot = norm_block_sum(s, ws);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)a.d), a.eps)));
  float4* o = reinterpret_cast<float4*>(a.out + (size_t)r * a.d);
  const float4* g4 = reinterpret_cast<const float4*>(a.g);
#pragma unroll
  for (int u = 0; u < kNormVec; ++u) {
    const int i = threadIdx.x + u * kNormThreads;
    if (i < d4) {
      const float4 gg = g4[i];
      o[i] = make_float4(__fmul_rn(__fmul_rn(v[u].x, inv), gg.x), __fmul_rn(__fmul_rn(v[u].y, inv), gg.y),
                         __fmul_rn(__fmul_rn(v[u].z, inv), gg.z), __fmul_rn(__fmul_rn(v[u].w, inv), gg.w));
    }
  }
}

// ----------------------------------------------------------- residual ---
__global__ void add_kernel(float* __restrict__ h, const float* __restrict__ y, size_t n4) {
  DK_PDL_PROLOGUE();
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
    float4 a = reinterpret_cast<float4*>(h)[i];
    const float4 b = reinterpret_cast<const float4*>(y)[i];
    a.x = __fadd_rn(a.x, b.x);
    a.y = __fadd_rn(a.y, b.y);
    a.z = __fadd_rn(a.z, b.z);
    a.w = __fadd_rn(a.w, b.w);
    reinterpret_cast<float4*>(h)[i] = a;
  }
}

// ------------------------------------------------------------- SwiGLU ---
// gu [R][2F] holds gate | up; act [R][F] = silu(gate) * up.
__global__ void swiglu_kernel(const float* __restrict__ gu, int R, int F, float* __restrict__ act) {
  DK_PDL_PROLOGUE();
  const size_t n = (size_t)R * F;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / F, j = i % F;
    act[i] = det_swiglu(gu[r * 2 * F + j], gu[r * 2 * F + F + j]);
  }
}

// ------------------------------------------------------ RoPE + K/V cache ---
// qkv [R][3d] rows b * T + t (token t of sequence b at position pos0 + t,
// pos0 read from the device when pos_dev is set).  Rotary embedding on the
// two halves of each head (x1, x2) -> (x1 c - x2 s, x2 c + x1 s) with the
// cos/sin table [max_ctx][hd/2]; q is rotated in place, k and v go to the
// cache [B][H][max_ctx][hd] as bf16.
__global__ void rope_kv_kernel(float* __restrict__ qkv, int T, int d, int H, int hd, int pos0,
                               const int32_t* __restrict__ pos_dev, const float* __restrict__ cs, int max_ctx,
                               __nv_bfloat16* __restrict__ kc, __nv_bfloat16* __restrict__ vc, int R) {
  DK_PDL_PROLOGUE();
  const int half = hd / 2;
  const long total = (long)R * H * half;
  const int p0 = pos_dev ? *pos_dev : pos0;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int j = (int)(i % half);
    const int h = (int)((i / half) % H);
    const int r = (int)(i / ((long)half * H));
    const int b = r / T, t = r % T, pos = p0 + t;
    const float c = cs[((size_t)pos * half + j) * 2], s = cs[((size_t)pos * half + j) * 2 + 1];
    float* row = qkv + (size_t)r * 3 * d;
    float* q = row + h * hd;
    const float q1 = q[j], q2 = q[j + half];
    q[j] = __fsub_rn(__fmul_rn(q1, c), __fmul_rn(q2, s));
    q[j + half] = __fadd_rn(__fmul_rn(q2, c), __fmul_rn(q1, s));
    const float* k = row + d + h * hd;
    const float k1 = k[j], k2 = k[j + half];
    const size_t cb = (((size_t)b * H + h) * max_ctx + pos) * hd;
    kc[cb + j] = __float2bfloat16_rn(__fsub_rn(__fmul_rn(k1, c), __fmul_rn(k2, s)));
    kc[cb + j + half] = __float2bfloat16_rn(__fadd_rn(__fmul_rn(k2, c), __fmul_rn(k1, s)));
    const float* v = row + 2 * d + h * hd;
    vc[cb + j] = __float2bfloat16_rn(v[j]);
    vc[cb + j + half] = __float2bfloat16_rn(v[j + half]);
  }
}

// ------------------------------------------------- prompt attention ---
// Causal attention for T tokens per sequence at positions pos0 .. pos0+T-1,
// keys 0 .. own position from the cache.  One CTA of 256 threads per (64
// queries, head, sequence); 64-key tiles; thread (ty, tx) = (tid / 16,
// tid % 16) owns score rows 4ty.. and columns 4tx.., output rows 4ty.. and
// dims 8tx..; online softmax (running max and sum per row, exp by
// det_expf); the output is the head's slice of att [R][d].
constexpr int kQB = 64, kKB = 64, kHD = 128;

__global__ void __launch_bounds__(256) attn_prompt_kernel(const float* __restrict__ qkv, int T, int d, int H,
                                                          int pos0, const __nv_bfloat16* __restrict__ kc,
                                                          const __nv_bfloat16* __restrict__ vc, int max_ctx,
                                                          float scale, float* __restrict__ att) {
  DK_PDL_PROLOGUE();
  extern __shared__ __align__(16) float sm[];
  float* Qt = sm;                          // [hd][kQB]      queries, transposed, pre-scaled
  float* Kt = Qt + kHD * kQB;              // [hd][kKB + 4]  keys, transposed
  float* V = Kt + kHD * (kKB + 4);         // [kKB][hd]
  float* P = V + kKB * kHD;                // [kQB][kKB + 4] probabilities
  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const int q0 = qb * kQB;                 // first query (token index within the sequence)
  const int nq = T - q0 < kQB ? T - q0 : kQB;
  for (int e = tid; e < kQB * kHD; e += 256) {
    const int i = e / kHD, dd = e % kHD;
    const float v = i < nq ? qkv[((size_t)b * T + q0 + i) * 3 * d + h * kHD + dd] : 0.0f;
    Qt[dd * kQB + i] = __fmul_rn(v, scale);
  }
  float m[4], l[4], o[4][8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -3.402823466e38f;
    l[i] = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) o[i][j] = 0.0f;
  }
  const size_t cbase = ((size_t)b * H + h) * max_ctx * kHD;
  const int last_key = pos0 + q0 + nq - 1;          // keys 0 .. last_key
  const int nkb = last_key / kKB + 1;
  for (int kb = 0; kb < nkb; ++kb) {
    __syncthreads();                                 // previous tile consumed
    for (int e = tid; e < kKB * kHD / 8; e += 256) {
      const int c = e / (kHD / 8), d8 = (e % (kHD / 8)) * 8;
      const int key = kb * kKB + c;
      uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
      if (key <= last_key) {
        kv = *reinterpret_cast<const uint4*>(kc + cbase + (size_t)key * kHD + d8);
        vv = *reinterpret_cast<const uint4*>(vc + cbase + (size_t)key * kHD + d8);
      }
      const __nv_bfloat16* kb16 = reinterpret_cast<const __nv_bfloat16*>(&kv);
      const __nv_bfloat16* vb16 = reinterpret_cast<const __nv_bfloat16*>(&vv);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        Kt[(d8 + u) * (kKB + 4) + c] = __bfloat162float(kb16[u]);
        V[c * kHD + d8 + u] = __bfloat162float(vb16[u]);
      }
    }
    __syncthreads();
    // scores: rows 4ty+i, columns 4tx+j
    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.0f;
#pragma unroll 4
    for (int dd = 0; dd < kHD; ++dd) {
      const float4 qv = *reinterpret_cast<const float4*>(Qt + dd * kQB + 4 * ty);
      const float4 kv = *reinterpret_cast<const float4*>(Kt + dd * (kKB + 4) + 4 * tx);
      const float qa[4] = {qv.x, qv.y, qv.z, qv.w}, ka[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) s[i][j] = __fmaf_rn(qa[i], ka[j], s[i][j]);
    }
    // causal mask, online softmax per row (the 16 threads of a row group are
    // lanes 16 apart in no case: tid = ty * 16 + tx, so they are one half-warp)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int qpos = pos0 + q0 + 4 * ty + i;
      float mx = -3.402823466e38f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int key = kb * kKB + 4 * tx + j;
        if (key > qpos) s[i][j] = -3.402823466e38f;
        mx = fmaxf(mx, s[i][j]);
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float mnew = fmaxf(m[i], mx);
      const float corr = det_expf(__fsub_rn(m[i], mnew));
      float rs = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int key = kb * kKB + 4 * tx + j;
        const float p = key > qpos ? 0.0f : det_expf(__fsub_rn(s[i][j], mnew));
        P[(4 * ty + i) * (kKB + 4) + 4 * tx + j] = p;
        rs = __fadd_rn(rs, p);
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) rs = __fadd_rn(rs, __shfl_xor_sync(0xffffffffu, rs, off));
      l[i] = __fadd_rn(__fmul_rn(l[i], corr), rs);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[i][j] = __fmul_rn(o[i][j], corr);
      m[i] = mnew;
    }
    __syncthreads();
    // o += P V: rows 4ty+i, dims 8tx+j
#pragma unroll 4
    for (int c = 0; c < kKB; ++c) {
      const float4 v0 = *reinterpret_cast<const float4*>(V + c * kHD + 8 * tx);
      const float4 v1 = *reinterpret_cast<const float4*>(V + c * kHD + 8 * tx + 4);
      const float va[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float p = P[(4 * ty + i) * (kKB + 4) + c];
#pragma unroll
        for (int j = 0; j < 8; ++j) o[i][j] = __fmaf_rn(p, va[j], o[i][j]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int qi = 4 * ty + i;
    if (qi < nq) {
      float* dst = att + ((size_t)b * T + q0 + qi) * d + h * kHD + 8 * tx;
#pragma unroll
      for (int j = 0; j < 8; ++j) dst[j] = __fdiv_rn(o[i][j], l[i]);
    }
  }
}

// ------------------------------------------------- one-token attention ---
// The new token of each sequence (position pos = *pos_dev) against keys
// 0 .. pos, split into chunks of kDC keys: one CTA of 256 threads per
// (chunk, head, sequence).  Scores: one key per thread (its bf16 row in
// 16-byte loads, q from shared memory).  Output: warp w takes keys 32w ..
// 32w+31 of the chunk, lane l dims 4l .. 4l+3 (one 8-byte load per key, a
// 256-byte row per warp and key), and the 8 warps' partial outputs are added
// in warp order.  Each CTA writes (max, sum, o[hd]) for its chunk; the last
// CTA of a (sequence, head) to finish (a counter, reset by that CTA) combines
// the chunks in chunk order, so the result does not depend on which CTA it is.
constexpr int kDC = 256;

__global__ void __launch_bounds__(256) attn_decode_kernel(const float* __restrict__ qkv, int d, int H,
                                                          const int32_t* __restrict__ pos_dev,
                                                          const __nv_bfloat16* __restrict__ kc,
                                                          const __nv_bfloat16* __restrict__ vc, int max_ctx,
                                                          float scale, int nch, float* __restrict__ part,
                                                          uint32_t* __restrict__ done, float* __restrict__ att) {
  DK_PDL_PROLOGUE();
  __shared__ float q[kHD];
  __shared__ float p[kDC];
  __shared__ float red[8];
  __shared__ float4 po[8][kHD / 4];
  __shared__ int last;
  const int ch = blockIdx.x, h = blockIdx.y, b = blockIdx.z, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nkeys = *pos_dev + 1;
  const int used = (nkeys + kDC - 1) / kDC;
  if (ch >= used) return;                               // chunk past the context (CTA-uniform)
  const int c0 = ch * kDC, c1 = c0 + kDC < nkeys ? c0 + kDC : nkeys;
  float* out = part + (((size_t)b * H + h) * nch + ch) * (kHD + 2);
  if (tid < kHD) q[tid] = __fmul_rn(qkv[(size_t)b * 3 * d + h * kHD + tid], scale);
  __syncthreads();
  const size_t cbase = ((size_t)b * H + h) * max_ctx * kHD;
  // scores, one key per thread
  const int c = c0 + tid;
  float s = -3.402823466e38f;
  if (c < c1) {
    const uint4* kr = reinterpret_cast<const uint4*>(kc + cbase + (size_t)c * kHD);
    uint4 kv[kHD / 8];
#pragma unroll
    for (int u = 0; u < kHD / 8; ++u) kv[u] = kr[u];
    s = 0.0f;
#pragma unroll
    for (int u = 0; u < kHD / 8; ++u) {
      const __nv_bfloat16* k16 = reinterpret_cast<const __nv_bfloat16*>(&kv[u]);
#pragma unroll
      for (int e = 0; e < 8; ++e) s = __fmaf_rn(q[u * 8 + e], __bfloat162float(k16[e]), s);
    }
  }
  float mx = s;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  mx = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) mx = fmaxf(mx, red[w]);
  const float e = c < c1 ? det_expf(__fsub_rn(s, mx)) : 0.0f;
  p[tid] = e;
  float sum = e;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
  __syncthreads();                                      // p written, red[] read
  if (lane == 0) red[warp] = sum;
  // o partial of this warp's 32 keys, dims 4 lane .. 4 lane + 3
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  const int k0 = c0 + warp * 32, k1 = k0 + 32 < c1 ? k0 + 32 : c1;
#pragma unroll 8
  for (int cc = k0; cc < k1; ++cc) {
    const uint2 vv = *reinterpret_cast<const uint2*>(vc + cbase + (size_t)cc * kHD + 4 * lane);
    const __nv_bfloat16* v16 = reinterpret_cast<const __nv_bfloat16*>(&vv);
    const float pc = p[cc - c0];
    acc.x = __fmaf_rn(pc, __bfloat162float(v16[0]), acc.x);
    acc.y = __fmaf_rn(pc, __bfloat162float(v16[1]), acc.y);
    acc.z = __fmaf_rn(pc, __bfloat162float(v16[2]), acc.z);
    acc.w = __fmaf_rn(pc, __bfloat162float(v16[3]), acc.w);
  }
  po[warp][lane] = acc;
  __syncthreads();
  if (tid < kHD) {
    float o = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) o = __fadd_rn(o, reinterpret_cast<const float*>(po[w])[tid]);
    out[2 + tid] = o;
  }
  if (tid == 0) {
    float tot = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) tot = __fadd_rn(tot, red[w]);
    out[0] = mx;
    out[1] = tot;
  }
  // the last chunk of this (sequence, head) to finish combines
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const uint32_t prev = atomicAdd(&done[b * H + h], 1u);
    last = prev == (uint32_t)used - 1;
    if (last) done[b * H + h] = 0u;                     // ready for the next step
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  if (tid < kHD) {
    const volatile float* pp = part + ((size_t)b * H + h) * nch * (kHD + 2);
    float M = -3.402823466e38f;
    for (int cc = 0; cc < used; ++cc) M = fmaxf(M, pp[cc * (kHD + 2)]);
    float L = 0.0f, a = 0.0f;
    for (int cc = 0; cc < used; ++cc) {
      const float w = det_expf(__fsub_rn(pp[cc * (kHD + 2)], M));
      L = __fmaf_rn(w, pp[cc * (kHD + 2) + 1], L);
      a = __fmaf_rn(w, pp[cc * (kHD + 2) + 2 + tid], a);
    }
    att[(size_t)b * d + h * kHD + tid] = __fdiv_rn(a, L);
  }
}

__global__ void pos_advance_kernel(int32_t* pos, int by) {
  DK_PDL_PROLOGUE();
  if (threadIdx.x == 0 && blockIdx.x == 0) *pos += by;
}

// ------------------------------------------------------- log-probs ---
// Per row r of logits [R][ld] (the first V columns the vocabulary):
// logp[r] = logits[r][target[r]] - logsumexp(logits[r][0..V)); one CTA of
// 256 threads per row, fixed reduction order.
__global__ void __launch_bounds__(256) logprob_kernel(const float* __restrict__ logits, int ld, int V,
                                                      const int32_t* __restrict__ target,
                                                      float* __restrict__ logp) {
  DK_PDL_PROLOGUE();
  __shared__ float red[8];
  const int r = blockIdx.x, tid = threadIdx.x;
  const float* x = logits + (size_t)r * ld;
  float mx = -3.402823466e38f;
  for (int j = tid; j < V; j += 256) mx = fmaxf(mx, x[j]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((tid & 31) == 0) red[tid >> 5] = mx;
  __syncthreads();
  mx = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) mx = fmaxf(mx, red[w]);
  __syncthreads();
  float s = 0.0f;
  for (int j = tid; j < V; j += 256) s = __fadd_rn(s, det_expf(__fsub_rn(x[j], mx)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
  if ((tid & 31) == 0) red[tid >> 5] = s;
  __syncthreads();
  if (tid == 0) {
    float tot = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) tot = __fadd_rn(tot, red[w]);
    int t = target[r];
    t = t < 0 ? 0 : (t >= V ? V - 1 : t);
    logp[r] = __fsub_rn(__fsub_rn(x[t], mx), logf(tot));
  }
}

// column `col` of a [R][ld] matrix -> out [R]
__global__ void column_kernel(const float* __restrict__ x, int R, int ld, int col, float* __restrict__ out) {
  DK_PDL_PROLOGUE();
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r < R) out[r] = x[(size_t)r * ld + col];
}

// rows r * T + T - 1 (the last token of each sequence) of x [B*T][n] -> y [B][n]
__global__ void last_rows_kernel(const float* __restrict__ x, int B, int T, int n, float* __restrict__ y) {
  DK_PDL_PROLOGUE();
  const int b = blockIdx.y;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    y[(size_t)b * n + i] = x[((size_t)b * T + T - 1) * n + i];
}

// seeded synthetic MX weights on the device: uniform bytes (int4: two
// uniform nibbles in [-8, 7]; int8: uniform in [-127, 127]) and E8M0
// exponents uniform in [emin, emax]; fp32 N(0, 1)-like table values by a
// sum of uniforms (Irwin-Hall, 12 terms)
__device__ __forceinline__ uint64_t smix(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__global__ void synth_bytes_kernel(uint8_t* __restrict__ out, size_t n, uint64_t seed, int fmt) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const uint64_t r = smix(seed ^ (i * 0xD1B54A32D192ED03ull));
    out[i] = fmt == 4 ? (uint8_t)(r & 0xFF) : (uint8_t)(int8_t)((int)(r % 255) - 127);
  }
}

__global__ void synth_scales_kernel(uint8_t* __restrict__ out, size_t n, uint64_t seed, int emin, int emax) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const uint64_t r = smix(seed ^ 0x5CA1E5ull ^ (i * 0xD1B54A32D192ED03ull));
    out[i] = (uint8_t)(127 + emin + (int)(r % (uint64_t)(emax - emin + 1)));
  }
}

__global__ void synth_normal_kernel(float* __restrict__ out, size_t n, uint64_t seed, float sd) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    float s = -6.0f;
    for (int k = 0; k < 12; ++k) {
      const uint64_t r = smix(seed ^ ((i * 12 + k) * 0xD1B54A32D192ED03ull));
      s += (float)(r >> 40) * (1.0f / 16777216.0f);
    }
    out[i] = s * sd;
  }
}

__global__ void fill_kernel(float* __restrict__ out, size_t n, float v) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) out[i] = v;
}

// <<<grid, block, smem, stream>>> with the programmatic-dependent-launch
// attribute.
template <typename... P, typename... A>
cudaError_t pdl_launch(void (*k)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, A... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, static_cast<P>(args)...);
}

unsigned grid_for(size_t n, unsigned threads) {
  size_t g = (n + threads - 1) / threads;
  if (g > 148u * 32u) g = 148u * 32u;
  return (unsigned)(g ? g : 1);
}

}  // namespace

// ------------------------------------------------------------ launchers ---
cudaError_t dk_embed(const int32_t* tok, const float* table, int R, int d, int vocab, float* h, cudaStream_t s) {
  return pdl_launch(embed_kernel, dim3(R), dim3(256), 0, s, tok, table, R, d, vocab, h);
}
cudaError_t dk_rmsnorm(const float* x, const float* g, int R, int d, float eps, float* y, cudaStream_t s) {
  if (d % 4 || d / 4 > kNormThreads * kNormVec) return cudaErrorInvalidValue;
  return pdl_launch(norm_kernel<false>, dim3(R), dim3(kNormThreads), 0, s, const_cast<float*>(x),
                    static_cast<const float*>(nullptr), g, d, eps, y, 1, (size_t)d);
}
cudaError_t dk_add(float* h, const float* y, size_t n, cudaStream_t s) {
  return pdl_launch(add_kernel, dim3(grid_for(n / 4, 256)), dim3(256), 0, s, h, y, n / 4);
}
cudaError_t dk_add_rmsnorm(float* h, const float* y, const float* g, int R, int d, float eps, float* out,
                           cudaStream_t s) {
  if (d % 4 || d / 4 > kNormThreads * kNormVec) return cudaErrorInvalidValue;
  return pdl_launch(norm_kernel<true>, dim3(R), dim3(kNormThreads), 0, s, h, y, g, d, eps, out, 1, (size_t)d);
}
cudaError_t dk_exchange_add_rmsnorm(const ExchNormArgs& a, cudaStream_t s) {
  if (a.d % 4 || a.d / 4 > kNormThreads * kNormVec || a.R < 1 || a.R > kExchNormMaxRows || a.world < 1 ||
      a.world > kMaxPeers || a.rank < 0 || a.rank >= a.world || a.slot_off % 16 || !a.seq || !a.grid_cnt ||
      !a.wait_flags)
    return cudaErrorInvalidValue;
  for (int q = 0; q < a.world; ++q)
    if (!a.base[q] || !a.flag_out[q] || (reinterpret_cast<uintptr_t>(a.base[q]) & 15u)) return cudaErrorInvalidValue;
  return pdl_launch(exch_norm_kernel, dim3(a.R), dim3(kNormThreads), 0, s, a);
}
cudaError_t dk_add_parts_rmsnorm(float* h, const float* y, int nparts, const float* g, int R, int d, float eps,
                                 float* out, cudaStream_t s) {
  if (d % 4 || d / 4 > kNormThreads * kNormVec || nparts < 1) return cudaErrorInvalidValue;
  return pdl_launch(norm_kernel<true>, dim3(R), dim3(kNormThreads), 0, s, h, y, g, d, eps, out, nparts,
                    (size_t)nparts * d);
}
cudaError_t dk_swiglu(const float* gu, int R, int F, float* act, cudaStream_t s) {
  return pdl_launch(swiglu_kernel, dim3(grid_for((size_t)R * F, 256)), dim3(256), 0, s, gu, R, F, act);
}
cudaError_t dk_rope_kv(float* qkv, int R, int T, int d, int H, int pos0, const int32_t* pos_dev, const float* cs,
                       int max_ctx, __nv_bfloat16* kc, __nv_bfloat16* vc, cudaStream_t s) {
  const size_t n = (size_t)R * H * (d / H / 2);
  return pdl_launch(rope_kv_kernel, dim3(grid_for(n, 256)), dim3(256), 0, s, qkv, T, d, H, d / H, pos0, pos_dev, cs,
                    max_ctx, kc, vc, R);
}
size_t dk_attn_prompt_smem() {
  return (size_t)(kHD * kQB + kHD * (kKB + 4) + kKB * kHD + kQB * (kKB + 4)) * sizeof(float);
}
cudaError_t dk_attn_prompt(const float* qkv, int B, int T, int d, int H, int pos0, const __nv_bfloat16* kc,
                           const __nv_bfloat16* vc, int max_ctx, float* att, cudaStream_t s) {
  static SmemAttr smem_attr;
  const size_t smem = dk_attn_prompt_smem();
  if (cudaError_t e = smem_attr.ensure(attn_prompt_kernel, smem)) return e;
  const dim3 grid((unsigned)((T + kQB - 1) / kQB), (unsigned)H, (unsigned)B);
  return pdl_launch(attn_prompt_kernel, grid, dim3(256), smem, s, qkv, T, d, H, pos0, kc, vc, max_ctx,
                    1.0f / sqrtf((float)kHD), att);
}
int dk_decode_chunks(int max_ctx) { return (max_ctx + kDC - 1) / kDC; }
cudaError_t dk_attn_decode(const float* qkv, int B, int d, int H, const int32_t* pos_dev, const __nv_bfloat16* kc,
                           const __nv_bfloat16* vc, int max_ctx, float* part, uint32_t* done, float* att,
                           cudaStream_t s) {
  const int nch = dk_decode_chunks(max_ctx);
  return pdl_launch(attn_decode_kernel, dim3((unsigned)nch, (unsigned)H, (unsigned)B), dim3(256), 0, s, qkv, d, H,
                    pos_dev, kc, vc, max_ctx, 1.0f / sqrtf((float)kHD), nch, part, done, att);
}
cudaError_t dk_pos_advance(int32_t* pos, int by, cudaStream_t s) {
  return pdl_launch(pos_advance_kernel, dim3(1), dim3(32), 0, s, pos, by);
}
cudaError_t dk_logprob(const float* logits, int R, int ld, int V, const int32_t* target, float* logp, cudaStream_t s) {
  return pdl_launch(logprob_kernel, dim3(R), dim3(256), 0, s, logits, ld, V, target, logp);
}
cudaError_t dk_column(const float* x, int R, int ld, int col, float* out, cudaStream_t s) {
  return pdl_launch(column_kernel, dim3((R + 255) / 256), dim3(256), 0, s, x, R, ld, col, out);
}
cudaError_t dk_last_rows(const float* x, int B, int T, int n, float* y, cudaStream_t s) {
  return pdl_launch(last_rows_kernel, dim3((unsigned)((n + 255) / 256), (unsigned)B), dim3(256), 0, s, x, B, T, n, y);
}
cudaError_t dk_synth_weight(uint8_t* data, size_t data_bytes, uint8_t* scales, size_t nscales, int fmt, int emin,
                            int emax, uint64_t seed, cudaStream_t s) {
  synth_bytes_kernel<<<grid_for(data_bytes, 256), 256, 0, s>>>(data, data_bytes, seed, fmt);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  synth_scales_kernel<<<grid_for(nscales, 256), 256, 0, s>>>(scales, nscales, seed, emin, emax);
  return cudaGetLastError();
}
cudaError_t dk_synth_normal(float* out, size_t n, uint64_t seed, float sd, cudaStream_t s) {
  synth_normal_kernel<<<grid_for(n, 256), 256, 0, s>>>(out, n, seed, sd);
  return cudaGetLastError();
}
cudaError_t dk_fill(float* out, size_t n, float v, cudaStream_t s) {
  fill_kernel<<<grid_for(n, 256), 256, 0, s>>>(out, n, v);
  return cudaGetLastError();
}

}  // namespace mxq
