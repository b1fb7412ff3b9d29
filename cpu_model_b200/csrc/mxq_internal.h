// mxq_internal.h -- launch interfaces shared between the C-ABI layer
// (mxq_api.cu) and the kernel translation units.
#pragma once
#include <cstdint>
#include <mutex>
#include <cuda_runtime.h>
#include "../../include/mxq.h"
#include "mxq_common.cuh"

namespace mxq {

// Weight tiles in HBM (both GEMV and GEMM read this layout):
//   data  : [Npad/128][Kpad/64][128 rows][TB bytes]   TB = 32 (int4) / 64 (int8)
//   scales: [Npad/128][Kpad/64][128 rows][2]          E8M0 per 32-K block
// Rows >= N and K >= K are zero weights with scale byte 127 (1.0).
struct WeightView {
  int fmt;        // 4 or 8
  int N, K;       // logical shape (rows, reduction length)
  int Npad, Kpad; // Npad multiple of 256, Kpad multiple of 64
  const uint8_t* data;
  const uint8_t* scales;
  int scale_lo, scale_hi;  // range of the logical weight scale bytes
  // Tensor-core path: weights enter the bf16 operand as q*2^(e-gemm_shift)
  // and activations as q*2^(e+gemm_shift), so the largest finite weight
  // scale still fits bf16 (0 unless a weight exponent exceeds 120 / 124).
  int gemm_shift;
  // The converter's one-fma form needs its offset term (136 or 2^23+128
  // times the scale) finite: every finite scale byte minus gemm_shift
  // <= 246 (int4) / 231 (int8).  A NaN scale byte gives NaN on either form.
  int gemm_fused;
  // Block-sparse weights (mxq_weight_create_bsr): row tile rt keeps only the
  // k-tiles kt_idx[kt_ptr[rt] .. kt_ptr[rt+1]), stored compactly in that
  // order (data [tile][128][TB], scales [tile][128][2]).  Null when dense.
  const int32_t* kt_ptr;
  const int32_t* kt_idx;
  int nnz_tiles;
};

// The largest dynamic shared memory already allowed for one kernel, per
// device: cudaFuncSetAttribute applies to the current device only, so a
// process with contexts on several devices sets it once on each.  The value
// only grows (a smaller request never lowers it), under a lock, so threads
// launching the same kernel cannot leave it below what one of them needs.
struct SmemAttr {
  static constexpr int kMaxDevices = 64;
  size_t bytes[kMaxDevices] = {};
  std::mutex mu;
  template <typename F>
  cudaError_t ensure(F* fn, size_t smem) {
    if (smem <= 48 * 1024) return cudaSuccess;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) dev = -1;
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && bytes[dev] >= smem) return cudaSuccess;
    const size_t want = dev >= 0 && bytes[dev] > smem ? bytes[dev] : smem;
    const cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)want);
    if (e == cudaSuccess && dev >= 0) bytes[dev] = want;
    return e;
  }
};

struct QuantArgs {
  const float* x;        // fp32 input [B][K] (modes 0-2; gate for mode 2)
  const int32_t* gather; // optional (mode 0): source row of x per output row (MoE dispatch)
  const float* up;       // up projection (mode 2)
  const uint8_t* in_q;   // MX input (mode 3)
  const uint8_t* in_s;
  int B, K;
  uint8_t* out_q;        // optional MX output [B][K] (u8 = q + 128)
  uint8_t* out_s;        // optional scales [B][K/32]
  __nv_bfloat16* opnd;   // optional GEMM operand (tiled, swizzled)
  int Bpad, Kpad, BN;
  int int4_order;        // operand K order for int4 weights
  int shift;             // operand exponent shift (WeightView::gemm_shift)
};

// mode: 0 = plain, 1 = SiLU, 2 = SwiGLU(x, up), 3 = MX input -> operand
cudaError_t launch_quantize(const QuantArgs& a, int mode, cudaStream_t st, bool pdl);

struct GemvArgs {
  WeightView w;
  const uint8_t* xq;     // MX activations [B][K] ...
  const uint8_t* xs;     // [B][K/32]
  const float* xf;       // ... or fp32 rows [B][K], quantised in the kernel
  const void* pf_ptr;    // optional: bytes to prefetch into L2 (next layer's
  size_t pf_bytes;       //   weights and scales), spread over the CTAs
  const void* pf_ptr2;
  size_t pf_bytes2;
  float* y;              // [B][N]   (or [B][nrows] when gathering)
  int B;
  const int32_t* rows;   // optional gathered row ids (mx_rank16_dot_ptrs)
  int nrows;
  int32_t* block_dots;   // optional debug output [B][N][K/32]
  // Optional MX output of y (co-resident batch-1 GEMV, N a multiple of 32):
  // u8 q+128 [N], E8M0 [N/32], and N/32 zeroed counters the kernel leaves zero.
  uint8_t* yq;
  uint8_t* ys;
  uint32_t* ycnt;
};

cudaError_t launch_gemv(const GemvArgs& a, cudaStream_t st, bool pdl);
int gemv_max_batch();

struct GemmArgs {
  WeightView w;
  const __nv_bfloat16* opnd; // tiled operand (from launch_quantize)
  float* y;                  // [B][N]
  int B, Bpad, BN;
  uint32_t* status;          // device status word (bounded waits)
  int splits;                // K splits over a cluster; 0 = chosen by occupancy
  uint64_t wait_ns;          // limit of every bounded wait; 0 = kWaitLimitNs
  // Test hook (mxq_debug_gemm_stall): the activation producer withholds its
  // first copy, so the waits on it run out and the error path is exercised.
  int withhold_x0;
};

cudaError_t launch_gemm(const GemmArgs& a, cudaStream_t st, bool pdl);
int gemm_pick_bn(int B);

// Batches up to this size take the GEMV in MXQ_PATH_AUTO (larger ones up to
// kBgemvMaxBatch too, where the small-batch MMA GEMV supports the shape).
constexpr int kGemvAutoBatch = 4;

// Small-batch decode GEMV on the int8 MMA (mxq_bgemv.cu), kBgemvMinBatch <=
// batch <= kBgemvMaxBatch, MX input only (GemvArgs.xq/xs); no
// gather/dots/prefetch.  Batch 2 stays on the cp.async-ring kernel, which
// measured faster there (10.2 vs 11.6 us for the 7B up projection).
constexpr int kBgemvMinBatch = 3;
constexpr int kBgemvMaxBatch = 16;
bool bgemv_supported(const WeightView& w, int B);
cudaError_t launch_bgemv(const GemvArgs& a, cudaStream_t st, bool pdl);

// Persistent decode GEMV (mxq_rgemv.cu), batch <= kRgemvMaxBatch: MX or fp32
// input (GemvArgs.xq/xs or .xf), optional L2 prefetch; no gather/dots.
constexpr int kRgemvMaxBatch = 4;
bool rgemv_supported(const WeightView& w, int B);
cudaError_t launch_rgemv(const GemvArgs& a, cudaStream_t st, bool pdl);
// kernels one launch_rgemv call launches (batch-1 row slices: several)
int rgemv_launches(const GemvArgs& a);

// Peer mailboxes of a column-sharded batch-1 pair (mxq_cogemv.cu): where a
// launch writes into every rank's mailbox, the flags it waits on and sets,
// and the device epoch whose parity selects the mailbox half in use.
constexpr int kMaxPeers = 8;
struct PeerArgs {
  int world, rank;
  uint32_t* epoch;                 // local: calls completed (advanced at the end of role 2)
  uint32_t* grid_cnt;              // local: CTAs of this launch that have finished
  const uint32_t* wait_flags;      // local flags this launch waits on, [world]
  uint32_t* flag_out[kMaxPeers];   // per rank: the flag slot this launch sets
  uint8_t* q_out[kMaxPeers];       // per rank: MX bytes [2][q_stride] (role 1)
  uint8_t* s_out[kMaxPeers];       // per rank: MX scales [2][s_stride] (role 1)
  float* f_out[kMaxPeers];         // per rank: fp32 rows [2][f_stride] (role 2)
  size_t q_stride, s_stride, f_stride;
  int row_off;                     // this rank's first row in the full vector
  const uint8_t* xq_base;          // local MX input [2][xq_stride] (role 2)
  const uint8_t* xs_base;
  size_t xq_stride, xs_stride;
  const uint32_t* done_flags;      // local flags of the second linear's rows, [world] (role 2)
  const float* f_in;               // local fp32 rows [2][f_in_stride] (role 2's copy out)
  size_t f_in_stride;
  int n_out;                       // full output length (role 2)
  uint32_t* status;
  uint64_t wait_ns;
};
// role 1 / 2: the first / second linear of the pair (see the kernel)
cudaError_t launch_cogemv_peer(const GemvArgs& a, const PeerArgs& p, int role, cudaStream_t st, bool pdl);

// Peer exchange over mailboxes (mxq_tp.cu).  This rank's `rows` rows of
// row_bytes (a multiple of 16) at src, contiguous, go to every rank's
// mailbox (but skip_rank's, -1 for none): row r at
// dst_off + r * row_stride + rank * rank_stride.  The launch then sets this
// rank's flag word in every mailbox to the slot's next sequence number, and
// its last CTA waits (bounded) until every rank's flag in the local mailbox
// has reached it.  rows may be 0 (only the flags).
struct TpGatherArgs {
  int world, rank, rows, skip_rank;
  const uint8_t* src;              // 16-byte aligned
  size_t row_bytes, dst_off, row_stride, rank_stride;
  uint8_t* base[kMaxPeers];        // every rank's mailbox as mapped here
  uint32_t* flag_out[kMaxPeers];   // per rank: this rank's flag word of the slot
  const uint32_t* wait_flags;      // local mailbox: the slot's flags, [world]
  uint32_t* seq;                   // local: the slot's completed exchanges
  uint32_t* grid_cnt;              // local: CTAs of this launch that have finished
  uint32_t* status;
  uint64_t wait_ns;
};
cudaError_t launch_tp_gather(const TpGatherArgs& a, cudaStream_t st);

// The tensor-parallel decoder's exchange fused into its residual + RMSNorm
// (mxq_decoder_kernels.cu), for at most kExchNormMaxRows rows (one CTA a
// row, all resident at once): each CTA stores this rank's partial row into
// every other rank's mailbox at [row][rank][d] of the slot, the last CTA
// releases this rank's flag there, and every CTA waits (bounded) for every
// other rank's flag, then adds the partials in rank order (its own from
// y_own), the residual, and normalises.
constexpr int kExchNormMaxRows = 148;
struct ExchNormArgs {
  float* h;                        // [R][d] residual stream (updated)
  const float* y_own;              // [R][d] this rank's partial sums
  const float* g;                  // RMSNorm weights [d]
  float* out;                      // [R][d]
  int R, d, world, rank;
  float eps;
  uint8_t* base[kMaxPeers];        // every rank's mailbox as mapped here
  size_t slot_off;                 // the slot's [R][world][d] fp32 in every mailbox
  uint32_t* flag_out[kMaxPeers];   // per rank: this rank's flag word of the slot
  const uint32_t* wait_flags;      // local mailbox: the slot's flags, [world]
  uint32_t* seq;                   // local: the slot's completed exchanges
  uint32_t* grid_cnt;              // local
  uint32_t* status;
  uint64_t wait_ns;
};
cudaError_t dk_exchange_add_rmsnorm(const ExchNormArgs& a, cudaStream_t s);

// Batch-1 GEMV with two launches resident per SM (mxq_cogemv.cu): MX or fp32
// input, fp32 output, optionally also MX bytes of the output (GemvArgs.yq).
bool cogemv_supported(const WeightView& w, int B, bool inf32, bool qout);
cudaError_t launch_cogemv(const GemvArgs& a, cudaStream_t st, bool pdl);
// Batch 1, a weight too tall for one co-resident launch: the number of
// 128-row-tile slices (2-8) that each fit, 0 if none; and the launches (one
// per slice, in row order, each writing its rows of y).
int cogemv_row_parts(const WeightView& w, int B, bool inf32);
cudaError_t launch_cogemv_rows(const GemvArgs& a, int parts, cudaStream_t st, bool pdl);

// Context internals for the other host translation units (mxq_api.cu).
cudaStream_t ctx_stream(mxq_context* c);
void ctx_set_stream_raw(mxq_context* c, cudaStream_t s);
int ctx_fail(mxq_context* c, int code, const char* msg);
int ctx_cuda_fail(mxq_context* c, cudaError_t e, const char* what);
uint32_t* ctx_status_word(mxq_context* c);
int ctx_device(mxq_context* c);
void ctx_add_launches(mxq_context* c, uint64_t n);
uint64_t ctx_ws_gen(mxq_context* c);
uint64_t ctx_launches(mxq_context* c);
void ctx_set_launches(mxq_context* c, uint64_t n);
const WeightView* weight_view(mxq_weight w);

// Dense decoder steps (mxq_decoder_kernels.cu).
cudaError_t dk_embed(const int32_t* tok, const float* table, int R, int d, int vocab, float* h, cudaStream_t s);
cudaError_t dk_rmsnorm(const float* x, const float* g, int R, int d, float eps, float* y, cudaStream_t s);
cudaError_t dk_add(float* h, const float* y, size_t n, cudaStream_t s);
cudaError_t dk_add_rmsnorm(float* h, const float* y, const float* g, int R, int d, float eps, float* out,
                           cudaStream_t s);
// h += y[0] + ... + y[nparts - 1] (row r of y: nparts rows of d side by side), then RMSNorm
cudaError_t dk_add_parts_rmsnorm(float* h, const float* y, int nparts, const float* g, int R, int d, float eps,
                                 float* out, cudaStream_t s);
cudaError_t dk_swiglu(const float* gu, int R, int F, float* act, cudaStream_t s);
cudaError_t dk_rope_kv(float* qkv, int R, int T, int d, int H, int pos0, const int32_t* pos_dev, const float* cs,
                       int max_ctx, __nv_bfloat16* kc, __nv_bfloat16* vc, cudaStream_t s);
size_t dk_attn_prompt_smem();
cudaError_t dk_attn_prompt(const float* qkv, int B, int T, int d, int H, int pos0, const __nv_bfloat16* kc,
                           const __nv_bfloat16* vc, int max_ctx, float* att, cudaStream_t s);
int dk_decode_chunks(int max_ctx);
// `done` [B][H] counters, zero before the first call (each call leaves them zero).
cudaError_t dk_attn_decode(const float* qkv, int B, int d, int H, const int32_t* pos_dev, const __nv_bfloat16* kc,
                           const __nv_bfloat16* vc, int max_ctx, float* part, uint32_t* done, float* att,
                           cudaStream_t s);
cudaError_t dk_pos_advance(int32_t* pos, int by, cudaStream_t s);
cudaError_t dk_logprob(const float* logits, int R, int ld, int V, const int32_t* target, float* logp, cudaStream_t s);
cudaError_t dk_column(const float* x, int R, int ld, int col, float* out, cudaStream_t s);
cudaError_t dk_last_rows(const float* x, int B, int T, int n, float* y, cudaStream_t s);
cudaError_t dk_synth_weight(uint8_t* data, size_t data_bytes, uint8_t* scales, size_t nscales, int fmt, int emin,
                            int emax, uint64_t seed, cudaStream_t s);
cudaError_t dk_synth_normal(float* out, size_t n, uint64_t seed, float sd, cudaStream_t s);
cudaError_t dk_fill(float* out, size_t n, float v, cudaStream_t s);

// MoE bookkeeping (mxq_moe.cu): per-expert route counts, slot offsets, the
// token row gathered into each slot, the slot of each route; the weighted
// combine of the k expert outputs per token.
cudaError_t launch_moe_assign(const int32_t* idx, int T, int k, int E, int32_t* counts,
                              int32_t* offsets, int32_t* slot_token, int32_t* route_pos,
                              cudaStream_t st);
cudaError_t launch_moe_combine(const float* yr, const float* gate, const int32_t* route_pos, int T,
                               int D, int k, float* y, cudaStream_t st);

cudaError_t launch_scale_range(const uint8_t* scales, size_t count, uint32_t* out2,
                               cudaStream_t st);

// Small operators around the linear layer (mxq_ops.cu).
// mx_quantize_w: fp32 [N][K] -> int8 [N][K] / packed int4 [N][K/2] + E8M0
// [N][K/32] + optional w_sums int32 [N][K/32].
cudaError_t launch_quantize_w(int fmt, const float* w, int N, int K, uint8_t* data, uint8_t* scales,
                              int32_t* wsums, cudaStream_t st);
// Online weight update (mx_update_gaussian_moment): w += step * g x^T in
// the weight's own E8M0 grid, re-clamped to the int8 / int4 range; `data` is
// the weight's tiled bytes (w.data, written in place).
cudaError_t launch_moment_update(const WeightView& w, const float* g, const float* x, float step, uint8_t* data,
                                 cudaStream_t st);
// L2 norm of MX activation rows (mx_compute_activation_norm).
cudaError_t launch_act_norm(const uint8_t* xq, const uint8_t* xs, int B, int K, float* out, cudaStream_t st);
// Micro-expert layer (16-row experts, top-k routed + shared), one CTA per token.
size_t micro_moe_smem(int D, int nsel);
cudaError_t launch_micro_moe(const WeightView& wg, const WeightView& wu, const WeightView& wd, int n_routed,
                             int n_shared, const float* x, const int32_t* idx, const float* gate, int T, int k,
                             float* y, cudaStream_t st);
// ACT halting step on a 1-row weight, one state per token.
constexpr float kHaltEps = 0.01f;
cudaError_t launch_halting(const WeightView& w, const uint8_t* xq, const uint8_t* xs, int B, float bias,
                           float eps, mxq_halting_state* st, float* p, uint8_t* halt, cudaStream_t s);
// Dots against row 0 of up to kRowPtrsMax separate weights (same fmt and K).
constexpr int kRowPtrsMax = 64;
cudaError_t launch_row_ptrs(const WeightView* const* ws, int nrows, const uint8_t* xq, const uint8_t* xs, int B,
                            float* y, cudaStream_t s);
// LSH top-K router over fp32 rows [T][D] with H <= 32 hyperplanes.
cudaError_t launch_hashed_route(const float* x, int T, int D, int E, int K, int H, uint64_t seed, int32_t* idx,
                                int32_t* score, cudaStream_t s);

cudaError_t launch_repack(const uint8_t* data, const uint8_t* scales, int fmt,
                          int N, int K, int Npad, int Kpad, uint8_t* out_data,
                          uint8_t* out_scales, cudaStream_t st);

}  // namespace mxq
