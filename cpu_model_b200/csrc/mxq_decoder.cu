// mxq_decoder.cu -- a dense decoder built on the MX linears: the execution
// graph the qlinear hot path drops into (north_star's 7B decoder shape and the
// 1B rollout policy).  Per layer: RMSNorm -> QKV linear (one [3d][d] MX
// weight) -> rotary embedding, K/V to a bf16 cache -> causal attention ->
// O linear -> residual -> RMSNorm -> gate|up linear (one [2F][d] MX weight)
// -> SwiGLU -> down linear -> residual; then RMSNorm and the vocabulary head
// (plus, optionally, one value row).  Every linear is mxq_linear (GEMV by
// batch <= 16, tcgen05 GEMM above), so the decoder runs exactly the kernels
// the single-linear entry points run.
//
// Prompts go through in chunks of at most max_rows token rows (chunked
// prefill: a chunk's queries attend to the cached keys of earlier chunks);
// one-token steps read the position from device memory and advance it on
// the device, so a decode step is recorded once per batch size as a CUDA
// graph and replayed.  Weights are synthetic (seeded, generated on the
// device), as no checkpoint is available; mxq_decoder_weight exposes the
// handles, so real weights can be uploaded into the same shapes.
//
// Tensor parallel (mxq_decoder_create_sharded): rank r of p holds heads
// [r H/p, (r+1) H/p) -- their q, k, v rows, K/V cache and attention -- and
// FFN units [r F/p, (r+1) F/p) -- their gate and up rows; the O and down
// weights are split along K the same way (the columns of its heads and of
// its units), so each rank's O and down outputs are partial sums of every
// row.  Two peer all-gathers a layer (mxq_tp.cu) bring every rank's partial
// sums into every rank's mailbox, and the residual kernel adds them in rank
// order, so all ranks hold the same hidden state.  Embedding, RMSNorm and
// the vocabulary head are replicated.  The MX block dots are the unsharded
// decoder's (shards end on 32-blocks); only the fp32 order of the block sums
// of O and down differs.
#include <cmath>
#include <cstring>
#include <initializer_list>
#include <new>
#include <vector>

#include "../../include/mxq.h"
#include "mxq_internal.h"

using namespace mxq;

struct mxq_decoder_s {
  mxq_context* c = nullptr;
  mxq_decoder_config cfg{};
  int d = 0, H = 0, hd = 0, F = 0, V = 0, Vo = 0, L = 0, Bmax = 0, Cmax = 0, Rmax = 0, nch = 0;
  // tensor parallel: this rank of `world`; its width, heads and FFN columns
  // (dl = d, Hl = H, Fl = F unsharded)
  bool tp = false;
  int rank = 0, world = 1, dl = 0, Hl = 0, Fl = 0;
  uint8_t* mbox = nullptr;            // flags [2 slots][8 ranks] u32, then slot 0 (O), slot 1 (down)
  size_t slot_bytes = 0, mbox_bytes = 0;
  uint8_t* peer[kMaxPeers] = {};      // every rank's mailbox as mapped here
  bool opened[kMaxPeers] = {};
  uint32_t* tpw = nullptr;            // local: slot sequence numbers [2], grid counters [2]
  uint64_t wait_ns = kWaitLimitNs;
  std::vector<mxq_weight> qkv, o, gu, down;
  mxq_weight lm = nullptr;
  float* embed = nullptr;      // [V][d]
  float* gains = nullptr;      // [2L + 1][d]: per layer the attention then the MLP RMSNorm weights, then the final
  float* cs = nullptr;         // [Cmax][hd/2][2] rotary cos, sin
  __nv_bfloat16* kc = nullptr; // [L][Bmax][Hl][Cmax][hd]
  __nv_bfloat16* vc = nullptr;
  int32_t* pos_dev = nullptr;  // position of the next token (all sequences)
  int len = 0;                 // host mirror of *pos_dev
  float *h = nullptr, *hn = nullptr, *qkvb = nullptr, *att = nullptr, *tmp = nullptr, *gub = nullptr,
        *act = nullptr, *logits = nullptr, *part = nullptr, *hl = nullptr;
  int32_t* tok = nullptr;      // [Rmax + 1]
  uint32_t* done = nullptr;    // [Bmax][Hl] one-token attention chunk counters (zero between calls)
  int trace_layer = -1;
  float* trace[MXQ_TRACE_COUNT] = {};
  size_t trace_elems[MXQ_TRACE_COUNT] = {};
  struct StepGraph {
    int B;
    uint64_t gen;
    cudaGraphExec_t exec;
  };
  std::vector<StepGraph> graphs;
  // decode steps run on a private stream (capturable even when the caller's
  // is the legacy default stream), ordered after and before the caller's
  cudaStream_t dstream = nullptr;
  cudaEvent_t ev_in = nullptr, ev_out = nullptr;
};

namespace {

size_t kv_layer_elems(const mxq_decoder_s* D) { return (size_t)D->Bmax * D->Hl * D->Cmax * D->hd; }

int dfail(mxq_decoder_s* D, int code, const char* msg) { return ctx_fail(D->c, code, msg); }

int dcheck(mxq_decoder_s* D, cudaError_t e, const char* what) {
  if (e != cudaSuccess) return ctx_cuda_fail(D->c, e, what);
  ctx_add_launches(D->c, 1);
  return MXQ_OK;
}

template <typename T>
cudaError_t dalloc(T*& p, size_t count) {
  void* q = nullptr;
  const cudaError_t e = cudaMalloc(&q, count * sizeof(T) + 16);
  p = static_cast<T*>(q);
  return e;
}

struct RowRange {
  int row0, rows;
};

// Synthetic MX weight [n][k] on the device (seeded), uploaded as a handle;
// with row ranges, only those rows of it, in range order; with cols > 0,
// only columns [col0, col0 + cols) of every row (whole 32-blocks).  A
// rank's shard: the same bytes the unsharded weight has there.
int synth_weight(mxq_decoder_s* D, int n, int k, uint64_t seed, mxq_weight* out,
                 std::initializer_list<RowRange> ranges = {}, int col0 = 0, int cols = 0) {
  const int fmt = D->cfg.fmt;
  const size_t rb = fmt == 4 ? (size_t)k / 2 : (size_t)k, rs = (size_t)k / 32;   // data, scale bytes a row
  const size_t db = rb * n, sb = rs * n;
  size_t ns = 0;
  for (const RowRange& r : ranges) ns += (size_t)r.rows;
  uint8_t* tmp = nullptr;
  cudaError_t e = cudaMalloc(&tmp, db + sb + (ns ? (rb + rs) * ns : 0) + (cols ? db + sb : 0) + 16);
  if (e != cudaSuccess) return ctx_cuda_fail(D->c, e, "decoder weight scratch");
  cudaStream_t st = ctx_stream(D->c);
  const int emin = fmt == 4 ? -8 : -10, emax = fmt == 4 ? -3 : -4;
  e = dk_synth_weight(tmp, db, tmp + db, sb, fmt, emin, emax, seed, st);
  const uint8_t *wd = tmp, *ws = tmp + db;
  size_t rows = (size_t)n;
  if (ns && e == cudaSuccess) {
    uint8_t *sd = tmp + db + sb, *ss = sd + rb * ns;
    size_t at = 0;
    for (const RowRange& r : ranges) {
      if (e == cudaSuccess)
        e = cudaMemcpyAsync(sd + rb * at, wd + rb * r.row0, rb * r.rows, cudaMemcpyDeviceToDevice, st);
      if (e == cudaSuccess)
        e = cudaMemcpyAsync(ss + rs * at, ws + rs * r.row0, rs * r.rows, cudaMemcpyDeviceToDevice, st);
      at += (size_t)r.rows;
    }
    wd = sd;
    ws = ss;
    rows = ns;
  }
  size_t kk = (size_t)k;
  if (cols && e == cudaSuccess) {
    const size_t cb = fmt == 4 ? (size_t)cols / 2 : (size_t)cols, c0 = fmt == 4 ? (size_t)col0 / 2 : (size_t)col0;
    uint8_t *cd = tmp + db + sb + (ns ? (rb + rs) * ns : 0), *cs = cd + cb * rows;
    e = cudaMemcpy2DAsync(cd, cb, wd + c0, rb, cb, rows, cudaMemcpyDeviceToDevice, st);
    if (e == cudaSuccess)
      e = cudaMemcpy2DAsync(cs, (size_t)cols / 32, ws + col0 / 32, rs, (size_t)cols / 32, rows,
                            cudaMemcpyDeviceToDevice, st);
    wd = cd;
    ws = cs;
    kk = (size_t)cols;
  }
  int rc = e == cudaSuccess ? mxq_weight_create(D->c, fmt, rows, kk, wd, ws, 1, out)
                            : ctx_cuda_fail(D->c, e, "decoder weight synth");
  cudaStreamSynchronize(st);
  cudaFree(tmp);
  return rc;
}

int trace_copy(mxq_decoder_s* D, int layer, int id, const float* src, size_t n) {
  if (D->trace_layer != layer || id < 0 || id >= MXQ_TRACE_COUNT) return MXQ_OK;
  if (D->trace_elems[id] < n) {
    if (D->trace[id]) cudaFree(D->trace[id]);
    D->trace[id] = nullptr;
    D->trace_elems[id] = 0;
    if (cudaError_t e = dalloc(D->trace[id], n)) return ctx_cuda_fail(D->c, e, "trace buffer");
    D->trace_elems[id] = n;
  }
  if (cudaError_t e = cudaMemcpyAsync(D->trace[id], src, n * sizeof(float), cudaMemcpyDeviceToDevice,
                                      ctx_stream(D->c)))
    return ctx_cuda_fail(D->c, e, "trace copy");
  return MXQ_OK;
}

// --- tensor parallel: the peer all-gathers --------------------------------
constexpr size_t kTpFlagBytes = 256;

uint32_t* tp_flags(const mxq_decoder_s* D, int r, int slot) {
  return reinterpret_cast<uint32_t*>(D->peer[r]) + slot * kMaxPeers;
}
size_t tp_slot_off(const mxq_decoder_s* D, int slot) { return kTpFlagBytes + (size_t)slot * D->slot_bytes; }

int tp_gather(mxq_decoder_s* D, int slot, int rows, const uint8_t* src, size_t row_bytes) {
  TpGatherArgs a{};
  a.world = D->world;
  a.rank = D->rank;
  a.rows = rows;
  a.skip_rank = -1;
  a.src = src;
  a.row_bytes = row_bytes;
  a.dst_off = tp_slot_off(D, slot);
  a.row_stride = row_bytes * D->world;       // [row][rank][values]
  a.rank_stride = row_bytes;
  if (a.dst_off + (size_t)rows * row_bytes * D->world > tp_slot_off(D, slot + 1))
    return dfail(D, MXQ_ERR_INVALID_ARGUMENT, "tensor-parallel exchange larger than its mailbox slot");
  for (int r = 0; r < D->world; ++r) {
    a.base[r] = D->peer[r];
    a.flag_out[r] = tp_flags(D, r, slot) + D->rank;
  }
  a.wait_flags = tp_flags(D, D->rank, slot);
  a.seq = D->tpw + slot;
  a.grid_cnt = D->tpw + 2 + slot;
  a.status = ctx_status_word(D->c);
  a.wait_ns = D->wait_ns;
  return dcheck(D, launch_tp_gather(a, ctx_stream(D->c)), "tensor-parallel all-gather");
}

// this rank's [R][n] fp32 -> every rank's [R][world][n] in slot `slot`
int tp_gather_f32(mxq_decoder_s* D, int slot, const float* src, int R, int n, const float** full) {
  if (int rc = tp_gather(D, slot, R, reinterpret_cast<const uint8_t*>(src), (size_t)n * 4)) return rc;
  *full = reinterpret_cast<const float*>(D->mbox + tp_slot_off(D, slot));
  return MXQ_OK;
}

// Every rank's partial sums [R][d] of this exchange (this rank's in
// D->tmp), added in rank order, then the residual and the RMSNorm with
// gains g into D->hn.  Up to kExchNormMaxRows rows in one kernel (the
// exchange fused into the residual); more rows through the mailbox slot.
int tp_exchange_norm(mxq_decoder_s* D, int slot, int R, const float* g) {
  const int d = D->d;
  const float eps = D->cfg.norm_eps;
  if (R <= kExchNormMaxRows) {
    ExchNormArgs a{};
    a.h = D->h;
    a.y_own = D->tmp;
    a.g = g;
    a.out = D->hn;
    a.R = R;
    a.d = d;
    a.world = D->world;
    a.rank = D->rank;
    a.eps = eps;
    a.slot_off = tp_slot_off(D, slot);
    for (int r = 0; r < D->world; ++r) {
      a.base[r] = D->peer[r];
      a.flag_out[r] = tp_flags(D, r, slot) + D->rank;
    }
    a.wait_flags = tp_flags(D, D->rank, slot);
    a.seq = D->tpw + slot;
    a.grid_cnt = D->tpw + 2 + slot;
    a.status = ctx_status_word(D->c);
    a.wait_ns = D->wait_ns;
    return dcheck(D, dk_exchange_add_rmsnorm(a, ctx_stream(D->c)), "exchange + residual + rmsnorm");
  }
  const float* full = nullptr;
  if (int rc = tp_gather_f32(D, slot, D->tmp, R, d, &full)) return rc;
  return dcheck(D, dk_add_parts_rmsnorm(D->h, full, D->world, g, R, d, eps, D->hn, ctx_stream(D->c)),
                "residual + rmsnorm");
}

// The layers of a tensor-parallel decoder (see the file comment): as layers()
// below, over this rank's heads and FFN units, with the two exchanges.
int layers_tp(mxq_decoder_s* D, int B, int T, int pos0, bool decode) {
  mxq_context* c = D->c;
  cudaStream_t st = ctx_stream(c);
  const int R = B * T, d = D->d, dl = D->dl, Fl = D->Fl;
  const float eps = D->cfg.norm_eps;
  int rc;
  for (int l = 0; l < D->L; ++l) {
    __nv_bfloat16* kc = D->kc + (size_t)l * kv_layer_elems(D);
    __nv_bfloat16* vc = D->vc + (size_t)l * kv_layer_elems(D);
    if ((rc = trace_copy(D, l, MXQ_TRACE_IN, D->h, (size_t)R * d))) return rc;
    if (l == 0 && (rc = dcheck(D, dk_rmsnorm(D->h, D->gains, R, d, eps, D->hn, st), "rmsnorm"))) return rc;
    if ((rc = trace_copy(D, l, MXQ_TRACE_NORM1, D->hn, (size_t)R * d))) return rc;
    // this rank's heads: q, k, v rows [R][3 dl]
    if ((rc = mxq_linear(c, D->qkv[l], D->hn, (size_t)R, D->qkvb))) return rc;
    if ((rc = trace_copy(D, l, MXQ_TRACE_QKV, D->qkvb, (size_t)R * 3 * dl))) return rc;
    if ((rc = dcheck(D, dk_rope_kv(D->qkvb, R, T, dl, D->Hl, pos0, decode ? D->pos_dev : nullptr, D->cs, D->Cmax,
                                   kc, vc, st), "rope")))
      return rc;
    if ((rc = trace_copy(D, l, MXQ_TRACE_ROPE, D->qkvb, (size_t)R * 3 * dl))) return rc;
    if (decode) {
      if ((rc = dcheck(D, dk_attn_decode(D->qkvb, B, dl, D->Hl, D->pos_dev, kc, vc, D->Cmax, D->part, D->done,
                                         D->att, st),
                       "attention")))
        return rc;
    } else {
      if ((rc = dcheck(D, dk_attn_prompt(D->qkvb, B, T, dl, D->Hl, pos0, kc, vc, D->Cmax, D->att, st),
                       "attention")))
        return rc;
    }
    if ((rc = trace_copy(D, l, MXQ_TRACE_ATT, D->att, (size_t)R * dl))) return rc;
    // O over this rank's heads (its K columns): a partial sum of every
    // output row; every rank's partials, added in rank order, then the
    // residual and the RMSNorm
    if ((rc = mxq_linear(c, D->o[l], D->att, (size_t)R, D->tmp))) return rc;
    if ((rc = tp_exchange_norm(D, 0, R, D->gains + (size_t)(2 * l + 1) * d))) return rc;
    if ((rc = trace_copy(D, l, MXQ_TRACE_H1, D->h, (size_t)R * d))) return rc;
    if ((rc = trace_copy(D, l, MXQ_TRACE_NORM2, D->hn, (size_t)R * d))) return rc;
    // this rank's gate rows, then its up rows: [R][2 Fl]
    if ((rc = mxq_linear(c, D->gu[l], D->hn, (size_t)R, D->gub))) return rc;
    if ((rc = trace_copy(D, l, MXQ_TRACE_GU, D->gub, (size_t)R * 2 * Fl))) return rc;
    // down over this rank's FFN units (its K columns): partial sums again
    if (R == 1) {
      uint8_t* hq = reinterpret_cast<uint8_t*>(D->act);
      QuantArgs qa{};
      qa.x = D->gub;
      qa.up = D->gub + Fl;
      qa.B = 1;
      qa.K = Fl;
      qa.out_q = hq;
      qa.out_s = hq + (Fl + 15) / 16 * 16;
      if ((rc = dcheck(D, launch_quantize(qa, 2, st, true), "swiglu quantize"))) return rc;
      if ((rc = mxq_gemv(c, D->down[l], qa.out_q, qa.out_s, 1, D->tmp))) return rc;
    } else {
      if ((rc = dcheck(D, dk_swiglu(D->gub, R, Fl, D->act, st), "swiglu"))) return rc;
      if ((rc = mxq_linear(c, D->down[l], D->act, (size_t)R, D->tmp))) return rc;
    }
    if ((rc = tp_exchange_norm(D, 1, R, D->gains + (size_t)(2 * l + 2) * d))) return rc;
    if ((rc = trace_copy(D, l, MXQ_TRACE_OUT, D->h, (size_t)R * d))) return rc;
  }
  return trace_copy(D, D->L, MXQ_TRACE_IN, D->h, (size_t)R * d);
}

// All layers over R = B * T rows already embedded in D->h.  decode: one token
// per sequence at the device position (T == 1); otherwise a prompt chunk at
// positions pos0 .. pos0 + T - 1.  Leaves the final RMSNorm output in D->hn.
int layers(mxq_decoder_s* D, int B, int T, int pos0, bool decode) {
  if (D->tp) return layers_tp(D, B, T, pos0, decode);
  mxq_context* c = D->c;
  cudaStream_t st = ctx_stream(c);
  const int R = B * T, d = D->d;
  const float eps = D->cfg.norm_eps;
  int rc;
  for (int l = 0; l < D->L; ++l) {
    __nv_bfloat16* kc = D->kc + (size_t)l * kv_layer_elems(D);
    __nv_bfloat16* vc = D->vc + (size_t)l * kv_layer_elems(D);
    if ((rc = trace_copy(D, l, MXQ_TRACE_IN, D->h, (size_t)R * d))) return rc;
    // layer 0 normalises the embeddings; later layers received D->hn from the
    // previous layer's fused residual + RMSNorm
    if (l == 0 && (rc = dcheck(D, dk_rmsnorm(D->h, D->gains, R, d, eps, D->hn, st), "rmsnorm"))) return rc;
    if ((rc = trace_copy(D, l, MXQ_TRACE_NORM1, D->hn, (size_t)R * d))) return rc;
    if ((rc = mxq_linear(c, D->qkv[l], D->hn, (size_t)R, D->qkvb))) return rc;
    if ((rc = trace_copy(D, l, MXQ_TRACE_QKV, D->qkvb, (size_t)R * 3 * d))) return rc;
    if ((rc = dcheck(D, dk_rope_kv(D->qkvb, R, T, d, D->H, pos0, decode ? D->pos_dev : nullptr, D->cs, D->Cmax,
                                   kc, vc, st), "rope")))
      return rc;
    if ((rc = trace_copy(D, l, MXQ_TRACE_ROPE, D->qkvb, (size_t)R * 3 * d))) return rc;
    if (decode) {
      if ((rc = dcheck(D, dk_attn_decode(D->qkvb, B, d, D->H, D->pos_dev, kc, vc, D->Cmax, D->part, D->done,
                                         D->att, st),
                       "attention")))
        return rc;
    } else {
      if ((rc = dcheck(D, dk_attn_prompt(D->qkvb, B, T, d, D->H, pos0, kc, vc, D->Cmax, D->att, st), "attention")))
        return rc;
    }
    if ((rc = trace_copy(D, l, MXQ_TRACE_ATT, D->att, (size_t)R * d))) return rc;
    if ((rc = mxq_linear(c, D->o[l], D->att, (size_t)R, D->tmp))) return rc;
    if ((rc = dcheck(D, dk_add_rmsnorm(D->h, D->tmp, D->gains + (size_t)(2 * l + 1) * d, R, d, eps, D->hn, st),
                     "residual + rmsnorm")))
      return rc;
    if ((rc = trace_copy(D, l, MXQ_TRACE_H1, D->h, (size_t)R * d))) return rc;
    if ((rc = trace_copy(D, l, MXQ_TRACE_NORM2, D->hn, (size_t)R * d))) return rc;
    if ((rc = mxq_linear(c, D->gu[l], D->hn, (size_t)R, D->gub))) return rc;
    if ((rc = trace_copy(D, l, MXQ_TRACE_GU, D->gub, (size_t)R * 2 * D->F))) return rc;
    if (R == 1) {
      // one token: silu(gate) * up straight to MX bytes (one kernel, the
      // fused SwiGLU quantiser), which the down GEMV reads as its activation
      uint8_t* hq = reinterpret_cast<uint8_t*>(D->act);
      QuantArgs qa{};
      qa.x = D->gub;
      qa.up = D->gub + D->F;
      qa.B = 1;
      qa.K = D->F;
      qa.out_q = hq;
      qa.out_s = hq + D->F;
      if ((rc = dcheck(D, launch_quantize(qa, 2, st, true), "swiglu quantize"))) return rc;
      if ((rc = mxq_gemv(c, D->down[l], hq, hq + D->F, 1, D->tmp))) return rc;
    } else {
      if ((rc = dcheck(D, dk_swiglu(D->gub, R, D->F, D->act, st), "swiglu"))) return rc;
      if ((rc = mxq_linear(c, D->down[l], D->act, (size_t)R, D->tmp))) return rc;
    }
    // residual, then the next layer's (or the final) RMSNorm, in one kernel
    if ((rc = dcheck(D, dk_add_rmsnorm(D->h, D->tmp, D->gains + (size_t)(2 * l + 2) * d, R, d, eps, D->hn, st),
                     "residual + rmsnorm")))
      return rc;
    if ((rc = trace_copy(D, l, MXQ_TRACE_OUT, D->h, (size_t)R * d))) return rc;
  }
  return trace_copy(D, D->L, MXQ_TRACE_IN, D->h, (size_t)R * d);
}

// logits of rows `hrows` [B][d] -> user [B][V] (the value row, if any, dropped)
int head(mxq_decoder_s* D, const float* hrows, int B, float* logits_out) {
  int rc;
  if ((rc = mxq_linear(D->c, D->lm, hrows, (size_t)B, D->logits))) return rc;
  if (!logits_out) return MXQ_OK;
  cudaError_t e = cudaMemcpy2DAsync(logits_out, (size_t)D->V * 4, D->logits, (size_t)D->Vo * 4, (size_t)D->V * 4,
                                    (size_t)B, cudaMemcpyDeviceToDevice, ctx_stream(D->c));
  return e == cudaSuccess ? MXQ_OK : ctx_cuda_fail(D->c, e, "logits copy");
}

int decode_body(mxq_decoder_s* D, int B) {
  int rc;
  cudaStream_t st = ctx_stream(D->c);
  if ((rc = dcheck(D, dk_embed(D->tok, D->embed, B, D->d, D->V, D->h, st), "embed"))) return rc;
  if ((rc = layers(D, B, 1, 0, true))) return rc;
  if ((rc = head(D, D->hn, B, nullptr))) return rc;
  return dcheck(D, dk_pos_advance(D->pos_dev, 1, st), "position");
}

}  // namespace

#define DEC_TRY(...)                                                       \
  try {                                                                    \
    __VA_ARGS__                                                            \
  } catch (const std::bad_alloc&) {                                        \
    return MXQ_ERR_OUT_OF_MEMORY;                                          \
  } catch (...) {                                                          \
    return MXQ_ERR_CUDA;                                                   \
  }

extern "C" {

int mxq_decoder_destroy(mxq_decoder D) {
  if (!D) return MXQ_ERR_INVALID_ARGUMENT;
  cudaStreamSynchronize(ctx_stream(D->c));
  for (auto* v : {&D->qkv, &D->o, &D->gu, &D->down})
    for (mxq_weight w : *v)
      if (w) mxq_weight_destroy(w);
  if (D->lm) mxq_weight_destroy(D->lm);
  for (void* p : {(void*)D->embed, (void*)D->gains, (void*)D->cs, (void*)D->kc, (void*)D->vc, (void*)D->pos_dev,
                  (void*)D->h, (void*)D->hn, (void*)D->qkvb, (void*)D->att, (void*)D->tmp, (void*)D->gub,
                  (void*)D->act, (void*)D->logits, (void*)D->part, (void*)D->hl, (void*)D->tok, (void*)D->done})
    if (p) cudaFree(p);
  for (float* t : D->trace)
    if (t) cudaFree(t);
  for (auto& g : D->graphs)
    if (g.exec) cudaGraphExecDestroy(g.exec);
  if (D->tp) {
    cudaDeviceSynchronize();
    for (int r = 0; r < D->world; ++r)
      if (D->opened[r]) cudaIpcCloseMemHandle(D->peer[r]);
    if (D->mbox) cudaFree(D->mbox);
    if (D->tpw) cudaFree(D->tpw);
  }
  if (D->dstream) cudaStreamSynchronize(D->dstream), cudaStreamDestroy(D->dstream);
  if (D->ev_in) cudaEventDestroy(D->ev_in);
  if (D->ev_out) cudaEventDestroy(D->ev_out);
  delete D;
  return MXQ_OK;
}

}  // extern "C"

namespace {

// world == 0: the unsharded decoder; otherwise rank `rank` of a
// tensor-parallel group of `world` (one rank: the sharded code path on one
// GPU, its exchanges through its own mailbox)
int create_decoder(mxq_ctx c, const mxq_decoder_config* cfg, uint64_t seed, int rank, int world, mxq_decoder* out,
                   void* handle_out) {
  DEC_TRY({
    if (!c || !cfg || !out || (world && !handle_out)) return MXQ_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    const mxq_decoder_config& g = *cfg;
    if (g.n_layers < 1 || g.d_model < 128 || g.n_heads < 1 || g.d_model % g.n_heads || g.d_model / g.n_heads != 128 ||
        g.d_model % 64 || g.ffn < 64 || g.ffn % 64 || g.vocab < 2 || (g.fmt != MXQ_FMT_INT4 && g.fmt != MXQ_FMT_INT8) ||
        g.max_batch < 1 || g.max_ctx < 1 || g.max_rows < g.max_batch || !(g.norm_eps > 0.0f) || !(g.rope_theta > 1.0f))
      return ctx_fail(c, MXQ_ERR_INVALID_ARGUMENT,
                      "decoder config: head dim 128, d and ffn multiples of 64, vocab >= 2, fmt 4/8, "
                      "max_rows >= max_batch >= 1, max_ctx >= 1");
    if (world && (world > kMaxPeers || rank < 0 || rank >= world || g.n_heads % world || g.ffn % (32 * world)))
      return ctx_fail(c, MXQ_ERR_INVALID_ARGUMENT,
                      "sharded decoder: rank in [0, world), world in [1, 8] dividing the heads, ffn a multiple of "
                      "32 * world");
    auto* D = new mxq_decoder_s();
    D->c = c;
    D->cfg = g;
    D->d = g.d_model;
    D->H = g.n_heads;
    D->hd = 128;
    D->F = g.ffn;
    D->V = g.vocab;
    D->Vo = g.vocab + (g.value_head ? 1 : 0);
    D->L = g.n_layers;
    D->Bmax = g.max_batch;
    D->Cmax = g.max_ctx;
    D->Rmax = g.max_rows;
    D->nch = dk_decode_chunks(g.max_ctx);
    D->tp = world > 0;
    D->rank = D->tp ? rank : 0;
    D->world = D->tp ? world : 1;
    D->dl = D->d / D->world;
    D->Hl = D->H / D->world;
    D->Fl = D->F / D->world;
    cudaStream_t st = ctx_stream(c);
    int rc = MXQ_OK;
    auto bail = [&](int code) {
      mxq_decoder_destroy(D);
      return code;
    };
    const int d = D->d, F = D->F, dl = D->dl, Fl = D->Fl, r0 = D->rank;
    for (int l = 0; l < D->L && rc == MXQ_OK; ++l) {
      mxq_weight w;
      const uint64_t s = seed * 1000003ull + (uint64_t)l * 16;
      if (!D->tp) {
        if ((rc = synth_weight(D, 3 * d, d, s + 1, &w)) == MXQ_OK) D->qkv.push_back(w);
        if (rc == MXQ_OK && (rc = synth_weight(D, d, d, s + 2, &w)) == MXQ_OK) D->o.push_back(w);
        if (rc == MXQ_OK && (rc = synth_weight(D, 2 * F, d, s + 3, &w)) == MXQ_OK) D->gu.push_back(w);
        if (rc == MXQ_OK && (rc = synth_weight(D, d, F, s + 4, &w)) == MXQ_OK) D->down.push_back(w);
        continue;
      }
      // this rank's parts of the same weights: its heads' q, k, v rows; the
      // O columns of its heads; its gate rows then its up rows; the down
      // columns of its FFN units
      if ((rc = synth_weight(D, 3 * d, d, s + 1, &w, {{r0 * dl, dl}, {d + r0 * dl, dl}, {2 * d + r0 * dl, dl}})) ==
          MXQ_OK)
        D->qkv.push_back(w);
      if (rc == MXQ_OK && (rc = synth_weight(D, d, d, s + 2, &w, {}, r0 * dl, dl)) == MXQ_OK) D->o.push_back(w);
      if (rc == MXQ_OK && (rc = synth_weight(D, 2 * F, d, s + 3, &w, {{r0 * Fl, Fl}, {F + r0 * Fl, Fl}})) == MXQ_OK)
        D->gu.push_back(w);
      if (rc == MXQ_OK && (rc = synth_weight(D, d, F, s + 4, &w, {}, r0 * Fl, Fl)) == MXQ_OK) D->down.push_back(w);
    }
    if (rc == MXQ_OK) rc = synth_weight(D, D->Vo, d, seed * 1000003ull + 999983ull, &D->lm);
    if (rc) return bail(rc);
    cudaError_t e = dalloc(D->embed, (size_t)D->V * d);
    if (e == cudaSuccess) e = dk_synth_normal(D->embed, (size_t)D->V * d, seed ^ 0xE3BEDull, 1.0f, st);
    if (e == cudaSuccess) e = dalloc(D->gains, (size_t)(2 * D->L + 1) * d);
    if (e == cudaSuccess) e = dk_fill(D->gains, (size_t)(2 * D->L + 1) * d, 1.0f, st);
    // rotary table in double precision, rounded once
    if (e == cudaSuccess) {
      std::vector<float> tab((size_t)D->Cmax * 64 * 2);
      for (int p = 0; p < D->Cmax; ++p)
        for (int j = 0; j < 64; ++j) {
          const double ang = (double)p * std::pow((double)g.rope_theta, -2.0 * j / 128.0);
          tab[((size_t)p * 64 + j) * 2] = (float)std::cos(ang);
          tab[((size_t)p * 64 + j) * 2 + 1] = (float)std::sin(ang);
        }
      e = dalloc(D->cs, tab.size());
      if (e == cudaSuccess) e = cudaMemcpy(D->cs, tab.data(), tab.size() * 4, cudaMemcpyHostToDevice);
    }
    const size_t kv = (size_t)D->L * kv_layer_elems(D);
    if (e == cudaSuccess) e = dalloc(D->kc, kv);
    if (e == cudaSuccess) e = dalloc(D->vc, kv);
    if (e == cudaSuccess) e = cudaMemsetAsync(D->kc, 0, kv * 2, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(D->vc, 0, kv * 2, st);
    if (e == cudaSuccess) e = dalloc(D->pos_dev, 1);
    if (e == cudaSuccess) e = cudaMemsetAsync(D->pos_dev, 0, 4, st);
    const size_t R = (size_t)D->Rmax;
    if (e == cudaSuccess) e = dalloc(D->h, R * d);
    if (e == cudaSuccess) e = dalloc(D->hn, R * d);
    if (e == cudaSuccess) e = dalloc(D->qkvb, R * 3 * d);
    if (e == cudaSuccess) e = dalloc(D->att, R * d);
    if (e == cudaSuccess) e = dalloc(D->tmp, R * d);
    if (e == cudaSuccess) e = dalloc(D->gub, R * 2 * F);
    if (e == cudaSuccess) e = dalloc(D->act, R * F);
    if (e == cudaSuccess) e = dalloc(D->logits, R * D->Vo);
    if (e == cudaSuccess) e = dalloc(D->hl, (size_t)D->Bmax * d);
    if (e == cudaSuccess) e = dalloc(D->part, (size_t)D->Bmax * D->Hl * D->nch * (128 + 2));
    if (e == cudaSuccess) e = dalloc(D->tok, R + 1);
    if (e == cudaSuccess) e = dalloc(D->done, (size_t)D->Bmax * D->Hl);
    if (e == cudaSuccess) e = cudaMemsetAsync(D->done, 0, (size_t)D->Bmax * D->Hl * 4 + 16, st);
    if (D->tp) {
      // mailbox: flags, then two slots of [max_rows][world][d] fp32 each
      D->slot_bytes = (R * (size_t)D->world * d * 4 + 255) / 256 * 256;
      D->mbox_bytes = kTpFlagBytes + 2 * D->slot_bytes;
      if (e == cudaSuccess) e = cudaMalloc(&D->mbox, D->mbox_bytes);
      if (e == cudaSuccess) e = cudaMemsetAsync(D->mbox, 0, D->mbox_bytes, st);
      if (e == cudaSuccess) e = dalloc(D->tpw, 4);
      if (e == cudaSuccess) e = cudaMemsetAsync(D->tpw, 0, 4 * sizeof(uint32_t), st);
      cudaIpcMemHandle_t ih{};
      if (e == cudaSuccess) e = cudaIpcGetMemHandle(&ih, D->mbox);
      if (e == cudaSuccess) {
        static_assert(sizeof(cudaIpcMemHandle_t) == MXQ_PEER_HANDLE_BYTES, "IPC handle size");
        std::memcpy(handle_out, &ih, sizeof(ih));
        D->peer[D->rank] = D->mbox;
      }
    }
    if (e == cudaSuccess) e = cudaMemsetAsync(D->tok, 0, (R + 1) * 4, st);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&D->dstream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&D->ev_in, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&D->ev_out, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return bail(ctx_cuda_fail(c, e, "decoder buffers"));
    *out = D;
    return MXQ_OK;
  })
}

bool tp_ready(mxq_decoder_s* D) {
  for (int r = 0; r < D->world; ++r)
    if (!D->peer[r]) return false;
  return true;
}

}  // namespace

extern "C" {

int mxq_decoder_create(mxq_ctx c, const mxq_decoder_config* cfg, uint64_t seed, mxq_decoder* out) {
  return create_decoder(c, cfg, seed, 0, 0, out, nullptr);
}

int mxq_decoder_create_sharded(mxq_ctx c, const mxq_decoder_config* cfg, uint64_t seed, int rank, int world,
                               mxq_decoder* out, void* handle_out) {
  if (!c) return MXQ_ERR_INVALID_ARGUMENT;
  if (world < 1) return ctx_fail(c, MXQ_ERR_INVALID_ARGUMENT, "sharded decoder: world >= 1");
  return create_decoder(c, cfg, seed, rank, world, out, handle_out);
}

int mxq_decoder_connect(mxq_decoder D, const void* handles) {
  DEC_TRY({
    if (!D || !handles) return MXQ_ERR_INVALID_ARGUMENT;
    if (!D->tp) return dfail(D, MXQ_ERR_INVALID_ARGUMENT, "connect: the decoder is not sharded");
    for (int r = 0; r < D->world; ++r) {
      if (r == D->rank || D->peer[r]) continue;
      cudaIpcMemHandle_t h;
      std::memcpy(&h, static_cast<const uint8_t*>(handles) + (size_t)r * sizeof(h), sizeof(h));
      void* p = nullptr;
      const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
      if (e != cudaSuccess) return ctx_cuda_fail(D->c, e, "open a peer's decoder mailbox");
      D->peer[r] = static_cast<uint8_t*>(p);
      D->opened[r] = true;
    }
    return MXQ_OK;
  })
}

int mxq_decoder_set_wait_limit(mxq_decoder D, uint32_t wait_us) {
  if (!D) return MXQ_ERR_INVALID_ARGUMENT;
  if (wait_us == 0 || wait_us > 10000000u)
    return dfail(D, MXQ_ERR_INVALID_ARGUMENT, "decoder wait limit must be in [1, 1e7] microseconds");
  D->wait_ns = (uint64_t)wait_us * 1000ull;
  return MXQ_OK;
}

int mxq_decoder_reset(mxq_decoder D) {
  if (!D) return MXQ_ERR_INVALID_ARGUMENT;
  D->len = 0;
  cudaError_t e = cudaMemsetAsync(D->pos_dev, 0, 4, ctx_stream(D->c));
  if (e == cudaSuccess) e = cudaMemsetAsync(D->done, 0, (size_t)D->Bmax * D->Hl * 4, ctx_stream(D->c));
  return e == cudaSuccess ? MXQ_OK : ctx_cuda_fail(D->c, e, "decoder reset");
}

int mxq_decoder_length(mxq_decoder D, int* len) {
  if (!D || !len) return MXQ_ERR_INVALID_ARGUMENT;
  *len = D->len;
  return MXQ_OK;
}

int mxq_decoder_prefill(mxq_decoder D, const int32_t* tokens, size_t b, size_t t, float* logits) {
  DEC_TRY({
    if (!D || !tokens) return MXQ_ERR_INVALID_ARGUMENT;
    if (D->tp && !tp_ready(D))
      return dfail(D, MXQ_ERR_INVALID_ARGUMENT, "sharded decoder not connected (mxq_decoder_connect)");
    if (b == 0 || t == 0 || (int)b > D->Bmax || t > (size_t)D->Cmax)
      return dfail(D, MXQ_ERR_INVALID_ARGUMENT, "prefill: batch in [1, max_batch], prompt in [1, max_ctx]");
    cudaStream_t st = ctx_stream(D->c);
    const int B = (int)b, T = (int)t;
    int Tc = D->Rmax / B;                        // tokens per chunk
    if (Tc > T) Tc = T;
    int rc;
    for (int t0 = 0; t0 < T; t0 += Tc) {
      const int tc = T - t0 < Tc ? T - t0 : Tc;
      // this chunk's tokens, row b * tc + i
      cudaError_t e = cudaMemcpy2DAsync(D->tok, (size_t)tc * 4, tokens + t0, (size_t)T * 4, (size_t)tc * 4, (size_t)B,
                                        cudaMemcpyDefault, st);
      if (e != cudaSuccess) return ctx_cuda_fail(D->c, e, "prefill tokens");
      if ((rc = dcheck(D, dk_embed(D->tok, D->embed, B * tc, D->d, D->V, D->h, st), "embed"))) return rc;
      if ((rc = layers(D, B, tc, t0, false))) return rc;
      if (t0 + tc == T) {
        if ((rc = dcheck(D, dk_last_rows(D->hn, B, tc, D->d, D->hl, st), "last rows"))) return rc;
        if ((rc = head(D, D->hl, B, logits))) return rc;
      }
    }
    D->len = T;
    cudaError_t e = cudaMemsetAsync(D->pos_dev, 0, 4, st);
    if (e == cudaSuccess) e = dk_pos_advance(D->pos_dev, T, st);
    return e == cudaSuccess ? MXQ_OK : ctx_cuda_fail(D->c, e, "prefill position");
  })
}

int mxq_decoder_decode(mxq_decoder D, const int32_t* tokens, size_t b, float* logits) {
  DEC_TRY({
    if (!D || !tokens || !logits) return MXQ_ERR_INVALID_ARGUMENT;
    if (D->tp && !tp_ready(D))
      return dfail(D, MXQ_ERR_INVALID_ARGUMENT, "sharded decoder not connected (mxq_decoder_connect)");
    if (b == 0 || (int)b > D->Bmax) return dfail(D, MXQ_ERR_INVALID_ARGUMENT, "decode: batch in [1, max_batch]");
    if (D->len >= D->Cmax) return dfail(D, MXQ_ERR_INVALID_ARGUMENT, "decode: the context is full (max_ctx)");
    mxq_context* c = D->c;
    const cudaStream_t user = ctx_stream(c);
    // the step runs on the decoder's stream, after the caller's queued work
    cudaError_t e = cudaEventRecord(D->ev_in, user);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(D->dstream, D->ev_in, 0);
    if (e != cudaSuccess) return ctx_cuda_fail(c, e, "decode ordering");
    // on every exit: the caller's stream waits for the step, and gets its
    // stream back
    struct Swap {
      mxq_decoder_s* D;
      cudaStream_t user;
      ~Swap() {
        if (cudaEventRecord(D->ev_out, D->dstream) == cudaSuccess) cudaStreamWaitEvent(user, D->ev_out, 0);
        ctx_set_stream_raw(D->c, user);
      }
    } swap{D, user};
    ctx_set_stream_raw(c, D->dstream);
    cudaStream_t st = D->dstream;
    const int B = (int)b;
    e = cudaMemcpyAsync(D->tok, tokens, (size_t)B * 4, cudaMemcpyDefault, st);
    if (e != cudaSuccess) return ctx_cuda_fail(c, e, "decode tokens");
    int rc;
    mxq_decoder_s::StepGraph* g = nullptr;
    for (auto& x : D->graphs)
      if (x.B == B) g = &x;
    if (g && g->exec && g->gen == ctx_ws_gen(c) && D->trace_layer < 0) {
      e = cudaGraphLaunch(g->exec, st);
      if (e != cudaSuccess) return ctx_cuda_fail(c, e, "decode graph");
      ctx_add_launches(c, 1);
    } else {
      // plain launches (sizing every workspace), then record the step
      const uint64_t gen0 = ctx_ws_gen(c);
      if ((rc = decode_body(D, B))) return rc;
      if (D->trace_layer < 0 && ctx_ws_gen(c) == gen0) {
        if (!g) {
          D->graphs.push_back({B, 0, nullptr});
          g = &D->graphs.back();
        }
        if (g->exec) cudaGraphExecDestroy(g->exec);
        g->exec = nullptr;
        cudaGraph_t graph = nullptr;
        const uint64_t l0 = ctx_launches(c);
        bool good = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) == cudaSuccess;
        if (good) {
          const bool inner = decode_body(D, B) == MXQ_OK;
          good = cudaStreamEndCapture(st, &graph) == cudaSuccess && inner && graph && ctx_ws_gen(c) == gen0;
        }
        ctx_set_launches(c, l0);
        cudaGraphExec_t exec = nullptr;
        if (good) good = cudaGraphInstantiate(&exec, graph, 0) == cudaSuccess;
        if (graph) cudaGraphDestroy(graph);
        (void)cudaGetLastError();
        g->exec = good ? exec : nullptr;
        g->gen = ctx_ws_gen(c);
      }
    }
    D->len += 1;
    e = cudaMemcpy2DAsync(logits, (size_t)D->V * 4, D->logits, (size_t)D->Vo * 4, (size_t)D->V * 4, (size_t)B,
                          cudaMemcpyDefault, st);
    return e == cudaSuccess ? MXQ_OK : ctx_cuda_fail(c, e, "logits copy");
  })
}

int mxq_decoder_score(mxq_decoder D, const int32_t* tokens, size_t b, size_t t, float* logp, float* values) {
  DEC_TRY({
    if (!D || !tokens || !logp) return MXQ_ERR_INVALID_ARGUMENT;
    if (D->tp && !tp_ready(D))
      return dfail(D, MXQ_ERR_INVALID_ARGUMENT, "sharded decoder not connected (mxq_decoder_connect)");
    if (b == 0 || t < 2 || t > (size_t)D->Cmax || t > (size_t)D->Rmax)
      return dfail(D, MXQ_ERR_INVALID_ARGUMENT, "score: batch >= 1, sequence length in [2, min(max_ctx, max_rows)]");
    if (values && !D->cfg.value_head) return dfail(D, MXQ_ERR_INVALID_ARGUMENT, "score: the decoder has no value head");
    cudaStream_t st = ctx_stream(D->c);
    const int T = (int)t;
    int G = D->Rmax / T;                        // sequences per pass
    if (G > D->Bmax) G = D->Bmax;
    int rc;
    for (size_t b0 = 0; b0 < b; b0 += (size_t)G) {
      const int Bg = (int)(b - b0 < (size_t)G ? b - b0 : (size_t)G);
      const int R = Bg * T;
      cudaError_t e = cudaMemcpyAsync(D->tok, tokens + b0 * T, (size_t)R * 4, cudaMemcpyDefault, st);
      if (e != cudaSuccess) return ctx_cuda_fail(D->c, e, "score tokens");
      if ((rc = dcheck(D, dk_embed(D->tok, D->embed, R, D->d, D->V, D->h, st), "embed"))) return rc;
      if ((rc = layers(D, Bg, T, 0, false))) return rc;
      if ((rc = mxq_linear(D->c, D->lm, D->hn, (size_t)R, D->logits))) return rc;
      // target of row b*T + i is token i + 1 of the same sequence (D->tok + 1)
      if ((rc = dcheck(D, dk_logprob(D->logits, R, D->Vo, D->V, D->tok + 1, D->tmp, st), "logprob"))) return rc;
      e = cudaMemcpy2DAsync(logp + b0 * (T - 1), (size_t)(T - 1) * 4, D->tmp, (size_t)T * 4, (size_t)(T - 1) * 4,
                            (size_t)Bg, cudaMemcpyDefault, st);
      if (e != cudaSuccess) return ctx_cuda_fail(D->c, e, "logp copy");
      if (values) {
        if ((rc = dcheck(D, dk_column(D->logits, R, D->Vo, D->V, values + b0 * T, st), "values"))) return rc;
      }
    }
    return mxq_decoder_reset(D);
  })
}

int mxq_decoder_weight(mxq_decoder D, int layer, int which, mxq_weight* out) {
  if (!D || !out) return MXQ_ERR_INVALID_ARGUMENT;
  if (which == MXQ_DEC_LM_HEAD) {
    *out = D->lm;
    return MXQ_OK;
  }
  if (layer < 0 || layer >= D->L) return dfail(D, MXQ_ERR_INVALID_ARGUMENT, "decoder weight: layer out of range");
  switch (which) {
    case MXQ_DEC_QKV: *out = D->qkv[layer]; return MXQ_OK;
    case MXQ_DEC_O: *out = D->o[layer]; return MXQ_OK;
    case MXQ_DEC_GATE_UP: *out = D->gu[layer]; return MXQ_OK;
    case MXQ_DEC_DOWN: *out = D->down[layer]; return MXQ_OK;
  }
  return dfail(D, MXQ_ERR_INVALID_ARGUMENT, "decoder weight: unknown kind");
}

int mxq_decoder_embedding(mxq_decoder D, size_t row0, size_t nrows, float* out) {
  if (!D || !out) return MXQ_ERR_INVALID_ARGUMENT;
  if (row0 + nrows > (size_t)D->V) return dfail(D, MXQ_ERR_INVALID_ARGUMENT, "embedding: rows out of range");
  cudaStream_t st = ctx_stream(D->c);
  cudaError_t e = cudaMemcpyAsync(out, D->embed + row0 * D->d, nrows * D->d * 4, cudaMemcpyDefault, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  return e == cudaSuccess ? MXQ_OK : ctx_cuda_fail(D->c, e, "embedding read");
}

int mxq_decoder_set_trace(mxq_decoder D, int layer) {
  if (!D) return MXQ_ERR_INVALID_ARGUMENT;
  if (layer > D->L) return dfail(D, MXQ_ERR_INVALID_ARGUMENT, "trace: layer out of range");
  D->trace_layer = layer;
  return MXQ_OK;
}

int mxq_decoder_get_trace(mxq_decoder D, int id, float* out, size_t count) {
  if (!D || !out || id < 0 || id >= MXQ_TRACE_COUNT) return MXQ_ERR_INVALID_ARGUMENT;
  if (!D->trace[id] || count > D->trace_elems[id]) return dfail(D, MXQ_ERR_INVALID_ARGUMENT, "trace: nothing recorded");
  cudaStream_t st = ctx_stream(D->c);
  cudaError_t e = cudaMemcpyAsync(out, D->trace[id], count * 4, cudaMemcpyDefault, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  return e == cudaSuccess ? MXQ_OK : ctx_cuda_fail(D->c, e, "trace read");
}

}  // extern "C"
