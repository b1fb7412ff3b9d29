// nca_mx_linear.hpp -- C++ restoration of the reference's nca::linalg MX
// operator interface (the removed core/linalg/mx_linear.hpp; names in
// nn/tests/test_auto_generated.cpp:46-56, containers in
// nn/tests/autotest.hpp:93-136) on top of the C-ABI in mxq.h.
//
// Header-only.  Containers hold DEVICE memory; weights are owned by an
// MXINT8Tensor (upload once, reuse).  Like the reference operators, shape
// errors throw std::invalid_argument; CUDA or device-timeout failures throw
// std::runtime_error.  The C-ABI below never throws.
//
// Every operator comes in two forms: with an explicit Context first, and in
// the reference's own call shape (mx_gemv(x, w, y), mx_rank16_dot_ptrs(x,
// const MXINT8Tensor** rows, y), halting_step(x_q, w_halt, b, state, halt),
// HashedRouter{cfg}.route(x, idx), ...) on the calling thread's default
// context (default_context(): device set_default_device(), 0 unless set; the
// legacy default stream).
#pragma once
#include <cstddef>
#include <cstdint>
#include <memory>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "mxq.h"

namespace nca::linalg {

inline void mxq_check(int rc, mxq_ctx ctx) {
  if (rc == MXQ_OK) return;
  std::string msg = mxq_last_error(ctx);
  if (rc == MXQ_ERR_INVALID_ARGUMENT) throw std::invalid_argument(msg);
  throw std::runtime_error(msg + " (status " + std::to_string(rc) + ")");
}

// One library context per thread/stream (the reference's Dispatcher bound a
// kernel per process; here the binding is the device + stream).
class Context {
 public:
  explicit Context(int device = 0, void* stream = nullptr) {
    mxq_check(mxq_create(device, &ctx_), nullptr);
    if (stream) mxq_check(mxq_set_stream(ctx_, stream), ctx_);
  }
  ~Context() {
    if (ctx_) mxq_destroy(ctx_);
  }
  Context(const Context&) = delete;
  Context& operator=(const Context&) = delete;
  mxq_ctx get() const { return ctx_; }
  void synchronize() const { mxq_check(mxq_synchronize(ctx_), ctx_); }
  // counterpart of nca::simd::set_override_backend: force GEMV or GEMM
  void set_override_path(int path) const { mxq_check(mxq_set_path(ctx_, path), ctx_); }

 private:
  mxq_ctx ctx_ = nullptr;
};

// The calling thread's default context (created on first use).
inline int& default_device_slot() {
  thread_local int dev = 0;
  return dev;
}
inline std::unique_ptr<Context>& default_context_slot() {
  thread_local std::unique_ptr<Context> ctx;
  return ctx;
}
// Selects the device of this thread's default context (before its first use,
// or it is recreated on the new device).
inline void set_default_device(int device) {
  if (default_device_slot() != device) default_context_slot().reset();
  default_device_slot() = device;
}
inline const Context& default_context() {
  auto& c = default_context_slot();
  if (!c) c = std::make_unique<Context>(default_device_slot());
  return *c;
}

// MXUINT8Tensor: activation view, data = q + 128 (u8), scales = E8M0, one per
// 32 elements.  `batch` rows of `num_blocks` blocks each; device pointers.
struct MXUINT8Tensor {
  uint8_t* data = nullptr;
  uint8_t* scales = nullptr;
  size_t num_blocks = 0;  // per row
  size_t batch = 1;
  size_t k() const { return num_blocks * 32; }
};

// MXINT8Tensor: an uploaded MX weight (int8 or packed int4) [rows][K].
class MXINT8Tensor {
 public:
  MXINT8Tensor() = default;
  MXINT8Tensor(const Context& ctx, int fmt, size_t rows, size_t k, const void* data,
               const uint8_t* scales, bool on_device) {
    mxq_check(mxq_weight_create(ctx.get(), fmt, rows, k, data, scales, on_device ? 1 : 0, &w_),
              ctx.get());
    rows_ = rows;
    k_ = k;
    fmt_ = fmt;
  }
  // A shaped, empty weight that mx_quantize_w fills.
  MXINT8Tensor(int fmt, size_t rows, size_t k) : rows_(rows), k_(k), fmt_(fmt) {}
  ~MXINT8Tensor() {
    if (w_) mxq_weight_destroy(w_);
  }
  MXINT8Tensor(MXINT8Tensor&& o) noexcept
      : w_(std::exchange(o.w_, nullptr)), rows_(o.rows_), k_(o.k_), fmt_(o.fmt_) {}
  MXINT8Tensor& operator=(MXINT8Tensor&& o) noexcept {
    if (this != &o) {
      if (w_) mxq_weight_destroy(w_);
      w_ = std::exchange(o.w_, nullptr);
      rows_ = o.rows_;
      k_ = o.k_;
      fmt_ = o.fmt_;
    }
    return *this;
  }
  // Replaces the held weight (mx_quantize_w's output).
  void reset(mxq_weight w) {
    if (w_) mxq_weight_destroy(w_);
    w_ = w;
  }
  // Block-sparse form (64x64 blocks; block_mask host bytes [ceil(rows/64)][k/64]).
  MXINT8Tensor(const Context& ctx, int fmt, size_t rows, size_t k, const void* data,
               const uint8_t* scales, const uint8_t* block_mask, bool on_device) {
    mxq_check(mxq_weight_create_bsr(ctx.get(), fmt, rows, k, data, scales, block_mask, on_device ? 1 : 0,
                                    &w_),
              ctx.get());
    rows_ = rows;
    k_ = k;
    fmt_ = fmt;
  }
  MXINT8Tensor(const MXINT8Tensor&) = delete;
  MXINT8Tensor& operator=(const MXINT8Tensor&) = delete;
  mxq_weight handle() const { return w_; }
  size_t rows() const { return rows_; }
  size_t k() const { return k_; }
  size_t num_blocks() const { return rows_ * k_ / 32; }
  int fmt() const { return fmt_; }

 private:
  mxq_weight w_ = nullptr;
  size_t rows_ = 0, k_ = 0;
  int fmt_ = MXQ_FMT_INT8;
};

inline void require(bool ok, const char* what) {
  if (!ok) throw std::invalid_argument(what);
}

// mx_quantize_x: fp32 [batch][k] (device) -> MXUINT8Tensor
inline void mx_quantize_x(const Context& c, const float* x, MXUINT8Tensor& out) {
  mxq_check(mxq_quantize_x(c.get(), x, out.batch, out.k(), MXQ_ACT_NONE, out.data, out.scales),
            c.get());
}

// mx_fused_silu_quantize_x: silu(x) -> MXUINT8Tensor
inline void mx_fused_silu_quantize_x(const Context& c, const float* x, MXUINT8Tensor& out) {
  mxq_check(mxq_quantize_x(c.get(), x, out.batch, out.k(), MXQ_ACT_SILU, out.data, out.scales),
            c.get());
}

// fused_gated_silu_quantize: silu(gate) * up -> MXUINT8Tensor
inline void fused_gated_silu_quantize(const Context& c, const float* gate, const float* up,
                                      MXUINT8Tensor& out) {
  mxq_check(mxq_swiglu_quantize(c.get(), gate, up, out.batch, out.k(), out.data, out.scales),
            c.get());
}

// mx_gemv: y[batch][rows] = W x (fp32, device)
inline void mx_gemv(const Context& c, const MXUINT8Tensor& x, const MXINT8Tensor& w, float* y) {
  require(x.k() == w.k(), "mx_gemv: activation and weight K differ");
  mxq_check(mxq_gemv(c.get(), w.handle(), x.data, x.scales, x.batch, y), c.get());
}

// mx_dot / mx_dual_dot / mx_quad_dot / mx_rank16_dot: 1/2/4/16-row weights
inline void mx_dot(const Context& c, const MXUINT8Tensor& x, const MXINT8Tensor& w, float* y) {
  require(w.rows() == 1, "mx_dot: weight must have 1 row");
  mx_gemv(c, x, w, y);
}
inline void mx_dual_dot(const Context& c, const MXUINT8Tensor& x, const MXINT8Tensor& w, float* y) {
  require(w.rows() == 2, "mx_dual_dot: weight must have 2 rows");
  mx_gemv(c, x, w, y);
}
inline void mx_quad_dot(const Context& c, const MXUINT8Tensor& x, const MXINT8Tensor& w, float* y) {
  require(w.rows() == 4, "mx_quad_dot: weight must have 4 rows");
  mx_gemv(c, x, w, y);
}
inline void mx_rank16_dot(const Context& c, const MXUINT8Tensor& x, const MXINT8Tensor& w, float* y) {
  require(w.rows() == 16, "mx_rank16_dot: weight must have 16 rows");
  mx_gemv(c, x, w, y);
}

// mx_rank16_dot_ptrs: rows gathered by id from an expert-pool weight
// (device int32 ids; the reference passed 16 MXINT8Tensor pointers).
inline void mx_rank16_dot_ptrs(const Context& c, const MXUINT8Tensor& x, const MXINT8Tensor& pool,
                               const int32_t* row_ids, size_t nrows, float* y) {
  require(x.k() == pool.k(), "mx_rank16_dot_ptrs: activation and weight K differ");
  mxq_check(mxq_gather_dot(c.get(), pool.handle(), x.data, x.scales, x.batch, row_ids, nrows, y),
            c.get());
}

// fp32 in -> fp32 out (drop-in for a dense projection)
inline void mx_linear(const Context& c, const float* x, size_t batch, const MXINT8Tensor& w, float* y) {
  mxq_check(mxq_linear(c.get(), w.handle(), x, batch, y), c.get());
}

// mx_rank16_dot_ptrs in the reference's pointer-array form
// (nn/tests/autotest.hpp:126-136): 16 one-row weights, y[batch][16].
inline void mx_rank16_dot_ptrs(const Context& c, const MXUINT8Tensor& x, const MXINT8Tensor* const* rows,
                               float* y, size_t nrows = 16) {
  require(nrows > 0 && nrows <= 64, "mx_rank16_dot_ptrs: 1..64 row pointers");
  mxq_weight h[64];
  for (size_t j = 0; j < nrows; ++j) {
    require(rows[j] != nullptr, "mx_rank16_dot_ptrs: null row pointer");
    require(rows[j]->rows() == 1 && rows[j]->k() == x.k(), "mx_rank16_dot_ptrs: each row a 1 x K weight");
    h[j] = rows[j]->handle();
  }
  mxq_check(mxq_rank16_dot_ptrs(c.get(), h, nrows, x.data, x.scales, x.batch, y), c.get());
}

// mx_quantize_w (training/fidelity_test.cpp:60-61): fp32 rows (device) into
// `out` (a weight of out.fmt(), out.rows() x out.k()), quantised on the
// device straight into the weight's own layout.
inline void mx_quantize_w(const Context& c, const float* w, MXINT8Tensor& out) {
  require(out.rows() > 0 && out.k() > 0 && out.k() % 32 == 0,
          "mx_quantize_w: weight shape must be rows x K, K a multiple of 32");
  mxq_weight h = nullptr;
  mxq_check(mxq_weight_quantize(c.get(), out.fmt(), out.rows(), out.k(), w, 1, &h), c.get());
  out.reset(h);
}

// ---------------------------------------------------------------------------
// The reference's call shapes, on the calling thread's default context.
inline void mx_quantize_x(const float* x, MXUINT8Tensor& out) { mx_quantize_x(default_context(), x, out); }
inline void mx_fused_silu_quantize_x(const float* x, MXUINT8Tensor& out) {
  mx_fused_silu_quantize_x(default_context(), x, out);
}
inline void mx_quantize_w(const float* w, MXINT8Tensor& out) { mx_quantize_w(default_context(), w, out); }
inline void mx_gemv(const MXUINT8Tensor& x, const MXINT8Tensor& w, float* y) { mx_gemv(default_context(), x, w, y); }
inline void mx_dot(const MXUINT8Tensor& x, const MXINT8Tensor& w, float* y) { mx_dot(default_context(), x, w, y); }
inline void mx_dual_dot(const MXUINT8Tensor& x, const MXINT8Tensor& w, float* y) {
  mx_dual_dot(default_context(), x, w, y);
}
inline void mx_quad_dot(const MXUINT8Tensor& x, const MXINT8Tensor& w, float* y) {
  mx_quad_dot(default_context(), x, w, y);
}
inline void mx_rank16_dot(const MXUINT8Tensor& x, const MXINT8Tensor& w, float* y) {
  mx_rank16_dot(default_context(), x, w, y);
}
inline void mx_rank16_dot_ptrs(const MXUINT8Tensor& x, const MXINT8Tensor** rows, float* y) {
  mx_rank16_dot_ptrs(default_context(), x, rows, y, 16);
}

// linalg::HashedRouter (nn/tests/test_robustness.cpp:13-35): Config{d,
// n_experts, top_k, n_hashes}; top_k > n_experts throws invalid_argument at
// construction; route(x, indices) takes host memory like the reference and
// fills `indices` with top_k expert ids (the library's LSH, mxq_hashed_route).
class HashedRouter {
 public:
  struct Config {
    size_t d;
    size_t n_experts;
    size_t top_k;
    size_t n_hashes;
  };
  explicit HashedRouter(const Config& cfg, uint64_t seed = 0) : cfg_(cfg), seed_(seed) {
    if (cfg.top_k == 0 || cfg.top_k > cfg.n_experts)
      throw std::invalid_argument("HashedRouter: top_k must be in [1, n_experts]");
    if (cfg.n_hashes == 0 || cfg.n_hashes > 32 || cfg.d == 0 || cfg.d % 32)
      throw std::invalid_argument("HashedRouter: n_hashes in [1, 32], d a multiple of 32");
  }
  void route(const float* x, std::vector<size_t>& indices, const Context& c = default_context()) const {
    std::vector<int32_t> idx(cfg_.top_k), score(cfg_.top_k);
    mxq_check(mxq_hashed_route_host(c.get(), x, 1, cfg_.d, cfg_.n_experts, cfg_.top_k, cfg_.n_hashes, seed_,
                                    idx.data(), score.data()),
              c.get());
    indices.assign(idx.begin(), idx.end());
  }
  const Config& config() const { return cfg_; }

 private:
  Config cfg_;
  uint64_t seed_;
};

}  // namespace nca::linalg

namespace nca::layers {

// nca::layers::HaltingState (nn/core/layers/halting.hpp:16-20); the same
// layout as mxq_halting_state.
struct HaltingState {
  float p_sum = 0.0f;
  float remainder = 0.0f;
  size_t steps = 0;
};
static_assert(sizeof(HaltingState) == sizeof(mxq_halting_state), "HaltingState layout");

// halting_step (nn/core/layers/halting.hpp:24-30): one token, host state and
// flag as in the reference; returns the halting probability p_t.
inline float halting_step(const nca::linalg::Context& c, const nca::linalg::MXUINT8Tensor& x_q,
                          const nca::linalg::MXINT8Tensor& w_halt, float b_halt, HaltingState& state,
                          bool& should_halt) {
  nca::linalg::require(w_halt.rows() == 1 && x_q.k() == w_halt.k() && x_q.batch == 1,
                       "halting_step: one token and a 1 x K halting weight");
  float p = 0.0f;
  uint8_t h = 0;
  mxq_halting_state st{state.p_sum, state.remainder, (uint64_t)state.steps};
  nca::linalg::mxq_check(mxq_halting_step_host(c.get(), w_halt.handle(), x_q.data, x_q.scales, b_halt, &st, &p, &h),
                         c.get());
  state.p_sum = st.p_sum;
  state.remainder = st.remainder;
  state.steps = (size_t)st.steps;
  should_halt = h != 0;
  return p;
}
inline float halting_step(const nca::linalg::MXUINT8Tensor& x_q, const nca::linalg::MXINT8Tensor& w_halt,
                          float b_halt, HaltingState& state, bool& should_halt) {
  return halting_step(nca::linalg::default_context(), x_q, w_halt, b_halt, state, should_halt);
}

// gated_mlp_step: down(quant(silu(gate x) * up x))
inline void gated_mlp_step(const nca::linalg::Context& c, const float* x, size_t batch,
                           const nca::linalg::MXINT8Tensor& gate,
                           const nca::linalg::MXINT8Tensor& up,
                           const nca::linalg::MXINT8Tensor& down, float* y) {
  nca::linalg::mxq_check(mxq_mlp_swiglu(c.get(), gate.handle(), up.handle(), down.handle(), x, batch, y),
                         c.get());
}

inline void gated_mlp_step(const float* x, size_t batch, const nca::linalg::MXINT8Tensor& gate,
                           const nca::linalg::MXINT8Tensor& up, const nca::linalg::MXINT8Tensor& down, float* y) {
  gated_mlp_step(nca::linalg::default_context(), x, batch, gate, up, down, y);
}

inline void fused_gated_silu_quantize(const float* gate, const float* up, nca::linalg::MXUINT8Tensor& out) {
  nca::linalg::fused_gated_silu_quantize(nca::linalg::default_context(), gate, up, out);
}

// Top-k SwiGLU mixture-of-experts layer over E experts (gate/up [F][D],
// down [D][F]); x [T][D], logits [T][E], y [T][D] on the device.  k > E
// throws std::invalid_argument like HashedRouter.
inline void moe_swiglu(const nca::linalg::Context& c, const std::vector<const nca::linalg::MXINT8Tensor*>& gate,
                       const std::vector<const nca::linalg::MXINT8Tensor*>& up,
                       const std::vector<const nca::linalg::MXINT8Tensor*>& down, const float* x,
                       const float* logits, size_t tokens, size_t k, float* y) {
  nca::linalg::require(gate.size() == up.size() && gate.size() == down.size() && !gate.empty(),
                       "moe_swiglu: gate/up/down expert lists differ in length");
  std::vector<mxq_weight> g, u, d;
  for (size_t e = 0; e < gate.size(); ++e) {
    g.push_back(gate[e]->handle());
    u.push_back(up[e]->handle());
    d.push_back(down[e]->handle());
  }
  nca::linalg::mxq_check(mxq_moe_swiglu(c.get(), g.data(), u.data(), d.data(), gate.size(), x, logits,
                                        tokens, k, y),
                         c.get());
}

inline void moe_swiglu(const std::vector<const nca::linalg::MXINT8Tensor*>& gate,
                       const std::vector<const nca::linalg::MXINT8Tensor*>& up,
                       const std::vector<const nca::linalg::MXINT8Tensor*>& down, const float* x,
                       const float* logits, size_t tokens, size_t k, float* y) {
  moe_swiglu(nca::linalg::default_context(), gate, up, down, x, logits, tokens, k, y);
}

// PPOTrainer::update_step's rollout head (training/ppo_trainer.cpp:64-66,
// :77) after its MX linears: log_softmax, action log-probability, entropy.
inline void policy_head(const nca::linalg::Context& c, const float* logits, const float* actions,
                        size_t rows, size_t cols, float* log_probs, float* action_logp, float* entropy) {
  nca::linalg::mxq_check(
      mxq_policy_head(c.get(), logits, actions, rows, cols, log_probs, action_logp, entropy), c.get());
}

}  // namespace nca::layers
