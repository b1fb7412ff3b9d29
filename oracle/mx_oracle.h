/*
 * mx_oracle.h -- CPU restatement of the MX (E8M0 block-scaled) int8/int4
 * linear-layer path of saoxdxd2/cpu_model.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker: only tests, the
 * smoke entry and the CPU-baseline leg of the benchmark may load it.  The
 * product path (cpu_model_b200/libmxq.so) never links or calls it.
 *
 * The reference's own MX kernels (core/linalg/mx_linear.hpp,
 * core/simd/avx512_vnni.hpp) are absent from the reference snapshot, so this
 * is a restatement built from the surviving residues:
 *   - activation quantiser: nn/core/layers/ssm.cpp:164-177 (scalar) and
 *     nn/core/layers/ssm.cpp:234-260 (AVX-512),
 *   - container layouts: nn/tests/autotest.hpp:93-136,
 *   - VNNI dot contract (u8 = q+128 times s8, w_sums correction):
 *     nn/user.md:17, research_paper/HARDWARE_SATURATION.md:7-13,
 *   - operator inventory: nn/tests/test_auto_generated.cpp:46-56,
 *   - GAE: agentic_env/replay_memory.cpp:204-253.
 * MX results are "parity unpinned": no reference test holds MX golden
 * vectors.  The GAE restatement is pinned by agentic_env/test_memory.cpp:47-83.
 *
 * Numeric conventions fixed here (the reference leaves them open):
 *   E8M0 byte s encodes 2^(s-127); s = 0xFF is NaN.
 *   Activation/weight block exponent e = smallest integer with
 *     max|v| <= QMAX * 2^e (QMAX = 127 for int8, 7 for int4), clamped to
 *     e >= -127; an all-zero block has byte 0; a non-finite block has 0xFF.
 *   q = round-half-to-even(v * 2^-e), stored as u8 = q + 128 for activations.
 *   int4: two's complement nibbles, element 2i in the low nibble of byte i.
 *   Per-block dot = sum_{i<32} q_x[i] * q_w[i] (exact in int32).
 *   y = sum_b dot_b * 2^(e_x,b + e_w,b) accumulated in double, rounded to
 *     float once.
 */
#ifndef MX_ORACLE_H
#define MX_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MXO_BLOCK 32
#define MXO_FMT_INT8 8
#define MXO_FMT_INT4 4

/* extract_e8m0 / decode_e8m0_scale (nn/core/layers/ssm.cpp:170-172). */
uint8_t mxo_e8m0_from_absmax(float max_abs, int qmax);
double  mxo_e8m0_decode(uint8_t s);

/* Deterministic exp / SiLU used by every fused-SiLU quantiser (CPU and GPU
 * evaluate the same float operations in the same order, so results are
 * bit-identical). Cody-Waite reduction + degree-7 Taylor polynomial. */
float mxo_expf(float x);
float mxo_silu(float x);

/* mx_quantize_x / mx_fused_silu_quantize_x
 * (nn/tests/test_auto_generated.cpp:47-48; nn/core/layers/ssm.cpp:164-177).  x fp32 [B][K] ->
 * q u8 [B][K] (= q+128), s E8M0 [B][K/32].  act: 0 = none, 1 = SiLU. */
void mxo_quantize_x(const float* x, size_t B, size_t K, int act,
                    uint8_t* q, uint8_t* s);

/* fused_gated_silu_quantize (nn/tests/test_auto_generated.cpp:41):
 * y = silu(g) * u, then quantise. */
void mxo_swiglu_quantize(const float* gate, const float* up, size_t B, size_t K,
                         uint8_t* q, uint8_t* s);

/* mx_quantize_w (nn/tests/test_auto_generated.cpp:46; training/fidelity_test.cpp:60).  w fp32 [N][K] -> data (int8 [N][K] or packed int4
 * [N][K/2]), scales [N][K/32], w_sums int32 [N][K/32] (may be NULL). */
void mxo_quantize_w(int fmt, const float* w, size_t N, size_t K,
                    void* data, uint8_t* scales, int32_t* w_sums);

/* Signed weight value (row n, column k) of an int8 or int4 matrix. */
int mxo_weight_at(int fmt, const void* data, size_t K, size_t n, size_t k);

/* The mx_dot contract (nn/tests/test_auto_generated.cpp:51-54): per-block
 * int32 dots, out [B][N][K/32]. */
void mxo_block_dots(int fmt, const uint8_t* xq, const void* w, size_t B,
                    size_t N, size_t K, int32_t* out);

/* mx_gemv, batched (nn/tests/test_auto_generated.cpp:56). y fp32 [B][N]. */
void mxo_gemv(int fmt, const uint8_t* xq, const uint8_t* xs, const void* w,
              const uint8_t* ws, size_t B, size_t N, size_t K, float* y);

/* mx_rank16_dot_ptrs (nn/tests/test_auto_generated.cpp:55; nn/tests/autotest.hpp:126-136):
 * rows gathered through a row-index list:
 * y[b][j] = row rows[j] of w dotted with activation b, j < nrows. */
void mxo_gather_dot(int fmt, const uint8_t* xq, const uint8_t* xs,
                    const void* w, const uint8_t* ws, size_t K,
                    const int32_t* rows, size_t nrows, size_t B, float* y);

/* mx_rank16_dot_ptrs in the pointer-array form (nn/tests/autotest.hpp:126-136):
 * y[b][j] = row 0 of rows[j] (scales row_scales[j]) dotted with activation b,
 * summed in the GPU's fixed order: lane l of a warp adds the fp32 terms
 * (d * 2^e_x) * 2^e_w of blocks l, l+32, ... in order, then a xor-butterfly
 * over the 32 lanes (so the result is bit-identical to the GPU's). */
void mxo_rank16_dot_ptrs(int fmt, const uint8_t* xq, const uint8_t* xs,
                         const void* const* rows, const uint8_t* const* row_scales,
                         size_t nrows, size_t B, size_t K, float* y);

/* layers::halting_step (nn/core/layers/halting.hpp:24-30), ACT: p = sigmoid(
 * w . x + bias) (the dot in the order above, exp by mxo_expf), steps += 1;
 * halt when p_sum + p >= 1 - eps: remainder = 1 - p_sum, p_sum = 1; else
 * p_sum += p.  State arrays [B] are updated in place. */
void mxo_halting_step(int fmt, const uint8_t* xq, const uint8_t* xs, const void* w,
                      const uint8_t* ws, size_t B, size_t K, float bias, float eps,
                      float* p_sum, float* remainder, uint64_t* steps, float* p, uint8_t* halt);

/* The micro-expert pool (nn/config/model_config.hpp:23-25) as the library
 * states it (mxq_micro_moe), in the GPU's operation order. */
void mxo_micro_moe(int fmt, const void* wg, const uint8_t* sg, const void* wu, const uint8_t* su,
                   const void* wd, const uint8_t* sd, size_t n_routed, size_t n_shared, size_t D,
                   const float* x, const int32_t* idx, const float* gate, size_t T, size_t k, float* y);

/* mx_update_gaussian_moment (nn/tests/test_auto_generated.cpp:49;
 * research_paper/MATH_FOUNDATIONS.md:33-40) as the library states it:
 * w = clamp(rint(w + ((step * g[n]) * x[k]) * 2^-e), lo, hi), scales kept. */
void mxo_update_gaussian_moment(int fmt, void* data, const uint8_t* scales, size_t N, size_t K,
                                const float* g, const float* x, float step);
/* mx_compute_activation_norm (nn/tests/test_auto_generated.cpp:50): the L2
 * norm of each MX activation row, in the GPU's summation order. */
void mxo_activation_norm(const uint8_t* xq, const uint8_t* xs, size_t B, size_t K, float* out);

/* linalg::HashedRouter::route (nn/tests/test_robustness.cpp:13-35) as the
 * library defines it (the reference's algorithm is absent): sign-of-
 * projection LSH over the MX-quantised input with H seeded +-1 hyperplanes,
 * Hamming similarity to seeded expert codes, top-K (ties to the lower id).
 * Returns -1 when K > E, K == 0, H not in [1, 32] or D % 32 != 0. */
int mxo_hashed_route(const float* x, size_t T, size_t D, size_t E, size_t K, size_t H,
                     uint64_t seed, int32_t* idx, int32_t* score);

/* gated_mlp_step (nn/tests/test_auto_generated.cpp:42).  x fp32 [B][D] -> quantise -> gate,up [F] ->
 * swiglu-quantise -> down [D].  If mid_q/mid_s are non-NULL the intermediate
 * MX activation is written there ([B][F], [B][F/32]). */
void mxo_mlp_swiglu(int fmt, const float* x, size_t B, size_t D, size_t F,
                    const void* wg, const uint8_t* sg, const void* wu,
                    const uint8_t* su, const void* wd, const uint8_t* sd,
                    float* y, uint8_t* mid_q, uint8_t* mid_s);

/* Top-k routing with the HashedRouter error contract (nn/tests/test_robustness.cpp:13-35).  logits [T][E] -> idx [T][k] (descending logit, ties
 * to the lower expert id), gate [T][k] = softmax over the k chosen logits.
 * Returns -1 (invalid argument) when k > E or k == 0, else 0. */
int mxo_route_topk(const float* logits, size_t T, size_t E, size_t k,
                   int32_t* idx, float* gate);

/* ReplayMemory::fused_compute_gae (agentic_env/replay_memory.cpp:204-253)
 * over an interleaved [T][E] trajectory. */
void mxo_gae(const float* rewards, const float* values, const uint8_t* dones,
             const float* next_values, size_t T, size_t E, float gamma,
             float lambda, float* adv, float* ret);

/* The same on the ReplayMemory ring (agentic_env/replay_memory.cpp:204-253):
 * rewards/values/dones/adv/ret hold `cap` items, `size` of them valid, the
 * next write at `cursor`; the latest T*E items are swept (T cut to size/E),
 * environments beyond the reference's MAX_ENVS = 1024 are left untouched. */
void mxo_gae_ring(const float* rewards, const float* values, const uint8_t* dones,
                  const float* next_values, size_t cap, size_t size, size_t cursor,
                  size_t T, size_t E, float gamma, float lambda, float* adv, float* ret);

/* PPO rollout head of PPOTrainer::update_step (training/ppo_trainer.cpp:64-66
 * and :77): per row, log_probs = log_softmax(logits) (max, then the sum of
 * exp(x - max) in column order, lse = max + log(sum)), action_logp =
 * sum_j log_probs * actions, entropy = -sum_j exp(log_probs) * log_probs. */
void mxo_policy_head(const float* logits, const float* actions, size_t rows,
                     size_t cols, float* log_probs, float* action_logp,
                     float* entropy);

/* Block-sparse MoE layer on dense-with-zero-blocks expert matrices:
 * route top-k over logits [T][E]; per token, x is quantised once; each chosen
 * expert e runs gated_mlp on it; y[t] = sum_j gate_j * expert_j(x_t)
 * (double accumulation, rounded to float).  wg/wu are [E] pointers to
 * [F][D] matrices, wd to [D][F]. */
int mxo_moe(int fmt, const float* x, const float* logits, size_t T, size_t D,
            size_t F, size_t E, size_t k, const void* const* wg,
            const uint8_t* const* sg, const void* const* wu,
            const uint8_t* const* su, const void* const* wd,
            const uint8_t* const* sd, float* y);

#ifdef __cplusplus
}
#endif
#endif
