/*
 * mxq.h -- C-ABI of the B200 MX (E8M0 block-scaled) int8/int4 linear-layer
 * library, libmxq.so.
 *
 * Drop-in boundary for the nca::linalg MX operators of saoxdxd2/cpu_model
 * (core/linalg/mx_linear.hpp and core/simd/avx512_vnni.hpp, removed from the
 * snapshot; their names are registered in nn/tests/test_auto_generated.cpp:
 * 46-56 and their containers shown in nn/tests/autotest.hpp:93-136).  The
 * opaque-handle / plain-pointer style follows the reference's own C-ABI,
 * deployment/nca_deploy.h:25-46.
 *
 * Conventions
 *   - Every function returns an int status: MXQ_OK (0) or a negative
 *     MXQ_ERR_* code; nothing throws across this boundary.  Unlike
 *     deployment/nca_deploy.cpp:28-61, which silently returns on a null
 *     handle, a null handle or pointer is MXQ_ERR_INVALID_ARGUMENT.
 *     mxq_last_error() describes the last failure on a context.
 *   - Data pointers are DEVICE pointers owned by the caller (16-byte
 *     aligned; MX activations and fp32 inputs off a 16-byte boundary are
 *     refused with MXQ_ERR_INVALID_ARGUMENT before any launch), except in
 *     the *_host entry points, which take host memory.
 *     Weight handles own their device copy of the weights.
 *   - Work is enqueued on the context's stream (mxq_set_stream; default the
 *     legacy stream) and is asynchronous; mxq_synchronize() waits and
 *     reports a device-side timeout (MXQ_ERR_TIMEOUT) if any bounded wait in a
 *     kernel gave up.
 *   - One context per host thread/stream.  The context grows its device
 *     workspace on demand (cudaMalloc) the first time a larger batch or K is
 *     seen; mxq_reserve() sizes it ahead of time so the hot path allocates
 *     nothing.
 *
 * Layouts (the reference's containers, nn/tests/autotest.hpp:93-136)
 *   MX activation (MXUINT8Tensor): q u8 [B][K] holding q+128, scales E8M0
 *     [B][K/32].
 *   MX weight (MXINT8Tensor): int8 [N][K] row-major (or int4 packed
 *     [N][K/2], element 2i in the low nibble of byte i, two's complement),
 *     scales E8M0 [N][K/32].  K must be a multiple of 32.  The reference's
 *     w_sums are a CPU dpbusd artefact and are not needed.
 *   E8M0 byte s = 2^(s-127), 0xFF = NaN.
 */
#ifndef MXQ_H
#define MXQ_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(_WIN32)
#define MXQ_API __declspec(dllexport)
#else
#define MXQ_API __attribute__((visibility("default")))
#endif

#define MXQ_OK 0
#define MXQ_ERR_INVALID_ARGUMENT (-1)
#define MXQ_ERR_CUDA (-2)
#define MXQ_ERR_TIMEOUT (-3)
#define MXQ_ERR_OUT_OF_MEMORY (-4)
#define MXQ_ERR_UNSUPPORTED (-5)

#define MXQ_FMT_INT4 4
#define MXQ_FMT_INT8 8

#define MXQ_ACT_NONE 0
#define MXQ_ACT_SILU 1

#define MXQ_PATH_AUTO 0 /* GEMV kernels for batch <= 4, and up to 16 where the int8-MMA GEMV fits the
                          shape; tensor-core GEMM above */
#define MXQ_PATH_GEMV 1
#define MXQ_PATH_GEMM 2

typedef struct mxq_context* mxq_ctx;
typedef struct mxq_weight_s* mxq_weight;
typedef struct mxq_peers_s* mxq_peers;

/* nca::layers::HaltingState (nn/core/layers/halting.hpp:16-20): the same
 * members and, with size_t of 8 bytes, the same layout. */
typedef struct mxq_halting_state {
  float p_sum;
  float remainder;
  uint64_t steps;
} mxq_halting_state;

/* Halting threshold: a token halts once p_sum + p >= 1 - MXQ_HALT_EPS. */
#define MXQ_HALT_EPS 0.01f

/* ---------------------------------------------------------- lifecycle --- */
/* deployment/nca_deploy.h:28-30 (create/destroy) pattern. */
MXQ_API int mxq_abi_version(void);
MXQ_API int mxq_create(int device, mxq_ctx* out);
MXQ_API int mxq_destroy(mxq_ctx ctx);
MXQ_API int mxq_set_stream(mxq_ctx ctx, void* cuda_stream);
/* Regime override, the counterpart of nca::simd::set_override_backend
 * (nn/core/simd/dispatch.cpp:83-87): MXQ_PATH_*.  MXQ_PATH_GEMV accepts
 * batch <= 8 on every shape (batch 1 weight-resident kernel, 2 cp.async-ring
 * kernel, 3-8 int8-MMA kernel where it fits, register-blocked otherwise) and
 * batch <= 16 where the int8-MMA kernel fits the shape. */
MXQ_API int mxq_set_path(mxq_ctx ctx, int path);
MXQ_API int mxq_reserve(mxq_ctx ctx, size_t max_batch, size_t max_k);
MXQ_API int mxq_synchronize(mxq_ctx ctx);
MXQ_API const char* mxq_last_error(mxq_ctx ctx);
/* Number of kernels this context has launched (for launch accounting). */
MXQ_API int mxq_launch_count(mxq_ctx ctx, uint64_t* out);

/* ------------------------------------------------------------ weights --- */
/* Uploads an MX weight (MXINT8Tensor layout; int8 or packed int4) from host
 * (on_device = 0) or device (on_device = 1) memory; replaces the
 * mx_quantize_w output container (training/fidelity_test.cpp:60-61). */
MXQ_API int mxq_weight_create(mxq_ctx ctx, int fmt, size_t n, size_t k,
                              const void* data, const uint8_t* scales,
                              int on_device, mxq_weight* out);
/* Block-sparse MX weight for the MoE expert matrices (the gathered-row
 * expert pool of nn/tests/autotest.hpp:126-136 as 64x64-block sparse
 * matrices): the same dense data/scales as mxq_weight_create plus a host
 * byte mask [ceil(n/64)][k/64] (nonzero = block present).  Only tiles with a
 * present block are stored; masked-out blocks read as zero.  K must be a
 * multiple of 64.  Linears on such a weight always take the tensor-core
 * path; mxq_gather_dot and mxq_block_dots return MXQ_ERR_UNSUPPORTED. */
MXQ_API int mxq_weight_create_bsr(mxq_ctx ctx, int fmt, size_t n, size_t k,
                                  const void* data, const uint8_t* scales,
                                  const uint8_t* block_mask, int on_device,
                                  mxq_weight* out);
MXQ_API int mxq_weight_destroy(mxq_weight w);
MXQ_API int mxq_weight_shape(mxq_weight w, int* fmt, size_t* n, size_t* k);

/* nca::linalg::mx_quantize_w (nn/tests/test_auto_generated.cpp:46;
 * training/fidelity_test.cpp:60-61) on the device: fp32 rows w [N][K] ->
 * data int8 [N][K] (fmt 8) or packed int4 [N][K/2] (fmt 4), E8M0 scales
 * [N][K/32] (block exponent: the smallest e with max|w| <= QMAX * 2^e, QMAX
 * 127 / 7), and, when w_sums is not null, the per-block sums of the
 * quantised values [N][K/32] (the reference's dpbusd correction term).  A
 * block holding a NaN or inf gets scale 0xFF and zero values. */
MXQ_API int mxq_quantize_w(mxq_ctx ctx, int fmt, const float* w, size_t n,
                           size_t k, void* data, uint8_t* scales,
                           int32_t* w_sums);

/* mx_quantize_w and upload in one call: fp32 rows w [N][K] (host when
 * on_device = 0, device when 1) are quantised on the device
 * (mxq_quantize_w's rules) into a new weight handle. */
MXQ_API int mxq_weight_quantize(mxq_ctx ctx, int fmt, size_t n, size_t k,
                                const float* w, int on_device, mxq_weight* out);

/* --------------------------------------------------------- quantisers --- */
/* nca::linalg::mx_quantize_x / mx_fused_silu_quantize_x
 * (nn/tests/test_auto_generated.cpp:47-48; semantics
 * nn/core/layers/ssm.cpp:164-177): x fp32 [B][K] -> q [B][K], s [B][K/32].
 * act = MXQ_ACT_NONE or MXQ_ACT_SILU. */
MXQ_API int mxq_quantize_x(mxq_ctx ctx, const float* x, size_t b, size_t k,
                           int act, uint8_t* q, uint8_t* s);
/* nca::layers::fused_gated_silu_quantize
 * (nn/tests/test_auto_generated.cpp:41): silu(gate) * up -> MX. */
MXQ_API int mxq_swiglu_quantize(mxq_ctx ctx, const float* gate,
                                const float* up, size_t b, size_t k,
                                uint8_t* q, uint8_t* s);

/* ------------------------------------------------------------- linear --- */
/* nca::linalg::mx_gemv (nn/tests/test_auto_generated.cpp:56), batched;
 * mx_dot / mx_dual_dot / mx_quad_dot / mx_rank16_dot (:51-54) are this call
 * on a 1/2/4/16-row weight.  MX activations in, y fp32 [B][N]. */
MXQ_API int mxq_gemv(mxq_ctx ctx, mxq_weight w, const uint8_t* xq,
                     const uint8_t* xs, size_t b, float* y);
/* nca::linalg::mx_rank16_dot_ptrs (nn/tests/test_auto_generated.cpp:55;
 * pointer-array form nn/tests/autotest.hpp:126-136): rows gathered through
 * a device int32 row-id list; y [B][nrows]. */
MXQ_API int mxq_gather_dot(mxq_ctx ctx, mxq_weight w, const uint8_t* xq,
                           const uint8_t* xs, size_t b, const int32_t* rows,
                           size_t nrows, float* y);
/* nca::linalg::mx_rank16_dot_ptrs in the reference's pointer-array form
 * (const MXINT8Tensor** of 16 one-row tensors, nn/tests/autotest.hpp:126-136):
 * y[b][j] = row 0 of weight rows[j] dotted with activation b, for nrows <= 64
 * weights of one format and K (host array of handles; device activations and
 * y [B][nrows]).  The fp32 sum runs in a fixed order (lane l of a warp takes
 * blocks l, l+32, ...; a xor-butterfly combines the lanes). */
MXQ_API int mxq_rank16_dot_ptrs(mxq_ctx ctx, const mxq_weight* rows, size_t nrows,
                                const uint8_t* xq, const uint8_t* xs, size_t b,
                                float* y);
/* Per-block int32 dots sum_{i<32} q_x * q_w, out [B][N][K/32]; the
 * dpbusd - 128 * w_sum quantity of the reference's VNNI kernel. */
MXQ_API int mxq_block_dots(mxq_ctx ctx, mxq_weight w, const uint8_t* xq,
                           size_t b, int32_t* dots);
/* fp32 in -> quantise -> MX linear -> fp32 out (the drop-in for the
 * training/ppo_trainer.cpp:57-61 projections). */
MXQ_API int mxq_linear(mxq_ctx ctx, mxq_weight w, const float* x, size_t b,
                       float* y);
/* Same with HOST buffers; copies in and out on the context stream and
 * returns when y_host is written. */
MXQ_API int mxq_linear_host(mxq_ctx ctx, mxq_weight w, const float* x_host,
                            size_t b, float* y_host);
/* Two chained linears (w1: K -> M, w2: M -> N) with MX requantisation of the
 * intermediate, as in a 7B MLP's up/down pair. */
MXQ_API int mxq_linear_pair(mxq_ctx ctx, mxq_weight w1, mxq_weight w2,
                            const float* x, size_t b, float* y);
MXQ_API int mxq_linear_pair_host(mxq_ctx ctx, mxq_weight w1, mxq_weight w2,
                                 const float* x_host, size_t b, float* y_host);

/* ------------------------------------------- column-sharded pair (GPUs) ---
 * The batch-1 pair above column-sharded over `world` GPUs of one node, one
 * process (context) per GPU: output-feature sharding of mx_gemv
 * (nn/tests/test_auto_generated.cpp:56; each rank owns whole rows, full K,
 * so a row's block sums are untouched).  No NCCL on the data path: the
 * first linear writes its rows of the MX intermediate straight into every
 * rank's mailbox (peer stores over NVLink into CUDA IPC memory) and sets its
 * flag there; the second waits (bounded) for every rank's flag, reads the
 * whole intermediate locally and writes its fp32 rows the same way, and its
 * last CTA waits for every rank's rows and copies the full output.  Two
 * kernels a call.  Usage:
 *   mxq_peers_create(ctx, rank, world, n1, n2, &p, handle)   -- n1: the
 *     intermediate's length (a multiple of 32 * world), n2: the output's
 *     (a multiple of world); handle: MXQ_PEER_HANDLE_BYTES to exchange;
 *   (the caller gathers every rank's handle, in rank order)
 *   mxq_peers_connect(p, handles)       -- handles: world * 64 bytes
 *   mxq_linear_pair_sharded(ctx, p, w1, w2, x, y) -- w1: this rank's
 *     n1/world x K rows, w2: its n2/world x n1 rows, x: [K] fp32 (device),
 *     y: [n2] fp32 (device), the full output on every rank.
 * Every rank must make the same calls in the same order.  A wait that runs
 * out (a rank that never calls; limit mxq_peers_set_wait_limit, default 2 s)
 * sets the context's status word: mxq_synchronize then returns
 * MXQ_ERR_TIMEOUT, and the group must be destroyed and created again (its
 * ranks' epochs no longer agree).  CUDA-graph capture of the call is
 * supported (the mailbox half is chosen on the device). */
#define MXQ_PEER_HANDLE_BYTES 64
MXQ_API int mxq_peers_create(mxq_ctx ctx, int rank, int world, size_t n1, size_t n2,
                             mxq_peers* out, void* handle_out);
MXQ_API int mxq_peers_connect(mxq_peers peers, const void* handles);
MXQ_API int mxq_peers_set_wait_limit(mxq_peers peers, uint32_t wait_us);
MXQ_API int mxq_peers_destroy(mxq_peers peers);
MXQ_API int mxq_linear_pair_sharded(mxq_ctx ctx, mxq_peers peers, mxq_weight w1, mxq_weight w2,
                                    const float* x, float* y);
/* Test hook, no counterpart in the reference: on a one-rank group, the
 * second linear of the sharded pair (w2: n2 x n1) waiting on a flag that
 * nothing sets, with its wait limited to wait_us (1 .. 1e6) microseconds:
 * the wait runs out, the timeout lands in the status word, and the call
 * returns mxq_synchronize's MXQ_ERR_TIMEOUT.  The group and the context
 * stay usable. */
MXQ_API int mxq_debug_peer_stall(mxq_ctx ctx, mxq_peers peers, mxq_weight w2, uint32_t wait_us);
/* nca::layers::gated_mlp_step (nn/tests/test_auto_generated.cpp:42):
 * y = down(quant(silu(gate(x)) * up(x))). */
MXQ_API int mxq_mlp_swiglu(mxq_ctx ctx, mxq_weight gate, mxq_weight up,
                           mxq_weight down, const float* x, size_t b,
                           float* y);

/* Same result as mxq_linear on the tensor-core path (quantise -> GEMM), but
 * the call allocates nothing: the quantised-activation operand lives in a
 * fixed 4 MiB device array inside this library, not in the context
 * workspace.  No counterpart in the reference.  It is for callers that may
 * not allocate device memory -- an engine whose device memory is owned by its
 * own pool allocator, or a serving loop held to a no-allocation rule -- and
 * who cannot rely on mxq_reserve having sized the workspace.
 * Limit: 2 * Bpad * Kpad bytes <= 4 MiB (Bpad = batch rounded up to the
 * GEMM's token tile, Kpad = K rounded up to 64), e.g. batch 512 at K 4096;
 * larger shapes return MXQ_ERR_INVALID_ARGUMENT.  The first call on a device
 * looks up the array's device address (once per device, with that device
 * current); make that first call before any stream capture.  All calls, on
 * every context and stream of a device, share the one array: calls that
 * overlap on the GPU race and must be serialised by the caller. */
MXQ_API int mxq_linear_noalloc(mxq_ctx ctx, mxq_weight w, const float* x,
                               size_t b, float* y);

/* Test hook for the failure path; no counterpart in the reference.  Runs
 * the tensor-core linear (one K split) with the first activation copy
 * withheld and every device-side wait limited to wait_us microseconds
 * (1 .. 1e6), so the kernel's bounded waits run out: the kernel drains the
 * copies and tensor-core work it started, frees its tensor memory, records
 * the timeout in the status word and returns.  The call then synchronises and
 * returns mxq_synchronize's status, MXQ_ERR_TIMEOUT; y is left undefined and
 * the context stays usable. */
MXQ_API int mxq_debug_gemm_stall(mxq_ctx ctx, mxq_weight w, const float* x,
                                 size_t b, float* y, uint32_t wait_us);

/* ---------------------------------------------------- online update --- */
/* nca::linalg::mx_update_gaussian_moment (nn/tests/test_auto_generated.cpp:49;
 * described in research_paper/MATH_FOUNDATIONS.md:33-40 as "dW = eta * A_t *
 * grad_W log pi, then re-clamp to the MX boundary"; its code is absent, so
 * this is the library's statement of it): in place, every element of w
 * becomes clamp(rint(w + ((step * g[n]) * x[k]) * 2^-e), lo, hi) with e its
 * block's E8M0 exponent (unchanged) and [lo, hi] = [-127, 127] (int8) or
 * [-8, 7] (int4); step = eta * advantage, g [N] and x [K] (device) the
 * output gradient and the input of the linear (grad_W = g x^T).  Blocks with
 * scale 0xFF are left as they are; dense weights only. */
MXQ_API int mxq_update_gaussian_moment(mxq_ctx ctx, mxq_weight w, const float* g,
                                       const float* x, float step);
/* nca::linalg::mx_compute_activation_norm (nn/tests/test_auto_generated.cpp:50):
 * norms[b] = ||dequant(x_b)||_2 of MX activations xq [B][K], xs [B][K/32]
 * (per block the exact int sum of q^2 times 2^(2e), fp32 sum in a fixed
 * order). */
MXQ_API int mxq_activation_norm(mxq_ctx ctx, const uint8_t* xq, const uint8_t* xs,
                                size_t b, size_t k, float* norms);

/* ------------------------------------------------------------ halting --- */
/* nca::layers::halting_step (nn/core/layers/halting.hpp:24-30), batched: per
 * token b, p = sigmoid(w_halt . x_b + bias) with the 1-row MX dot of
 * mxq_rank16_dot_ptrs's fixed order and the library's deterministic exp;
 * state[b].steps += 1; if state[b].p_sum + p >= 1 - MXQ_HALT_EPS the token
 * halts (should_halt[b] = 1, remainder = 1 - p_sum, p_sum = 1), else p_sum
 * += p (should_halt[b] = 0).  p[b] = the halting probability.  Device
 * pointers: xq [B][K], xs [B][K/32], state [B], p [B], should_halt [B]. */
MXQ_API int mxq_halting_step(mxq_ctx ctx, mxq_weight w_halt, const uint8_t* xq,
                             const uint8_t* xs, size_t b, float bias,
                             mxq_halting_state* state, float* p,
                             uint8_t* should_halt);

/* One token with the state and outputs in HOST memory, the reference's
 * halting_step(x_q, w_halt, b_halt, state, should_halt) call shape
 * (device activation xq [K], xs [K/32]); synchronous. */
MXQ_API int mxq_halting_step_host(mxq_ctx ctx, mxq_weight w_halt,
                                  const uint8_t* xq, const uint8_t* xs,
                                  float bias, mxq_halting_state* state_host,
                                  float* p_host, uint8_t* should_halt_host);

/* ------------------------------------------------------------ routing --- */
/* Top-k expert selection with the HashedRouter contract
 * (nn/tests/test_robustness.cpp:13-35: k > n_experts is an invalid
 * argument): descending logit, ties to the lower id, gate = softmax over
 * the chosen logits.  idx int32 [T][k], gate fp32 [T][k]. */
MXQ_API int mxq_route_topk(mxq_ctx ctx, const float* logits, size_t t,
                           size_t n_experts, size_t k, int32_t* idx,
                           float* gate);

/* linalg::HashedRouter{Config{d, n_experts, top_k, n_hashes}}::route(x, idx)
 * (nn/tests/test_robustness.cpp:13-35; "rank-16 VNNI LSH router",
 * nn/docs/job.md:11).  The reference's algorithm is absent from its
 * snapshot; this one is a sign-of-projection LSH over the MX-quantised input:
 * x fp32 [T][d] is quantised per 32-block as mxq_quantize_x does; hyperplane
 * h < n_hashes (<= 32) has +-1 entries generated from `seed` (no stored
 * weights); bit h of the token's code is 1 when its projection (per-block
 * exact int dot, scaled by 2^e_x, summed in block order in fp32) is > 0;
 * expert e has a seeded n_hashes-bit code, its score is n_hashes minus the
 * Hamming distance of the two codes; idx [T][top_k] = the top_k scores,
 * descending, ties to the lower expert id; score [T][top_k] those scores.
 * top_k > n_experts (or 0) is MXQ_ERR_INVALID_ARGUMENT, the reference's
 * invalid_argument.  d must be a multiple of 32.  Device pointers. */
MXQ_API int mxq_hashed_route(mxq_ctx ctx, const float* x, size_t t, size_t d,
                             size_t n_experts, size_t top_k, size_t n_hashes,
                             uint64_t seed, int32_t* idx, int32_t* score);
/* Same with host buffers (the reference's call passes host memory). */
MXQ_API int mxq_hashed_route_host(mxq_ctx ctx, const float* x_host, size_t t,
                                  size_t d, size_t n_experts, size_t top_k,
                                  size_t n_hashes, uint64_t seed,
                                  int32_t* idx_host, int32_t* score_host);

/* Top-k SwiGLU mixture-of-experts layer (the expert execution behind
 * mx_rank16_dot_ptrs, nn/tests/test_auto_generated.cpp:55, with the 1024 x
 * 16-row micro-experts of nn/config/model_config.hpp:23-25 generalised to
 * block-sparse expert matrices): routes with mxq_route_topk's contract over
 * logits [T][E], then per expert e: y_e = down_e(quant(silu(gate_e(x)) *
 * up_e(x))) on the tokens routed to it, and y[t] = sum_j gate_j * y_{e_j}[t]
 * in routing order.  w_gate/w_up: E weights [F][D]; w_down: E weights
 * [D][F] (dense or block-sparse).  x [T][D], logits [T][E], y [T][D], all
 * device pointers.  Reads back the per-expert token counts once (a stream
 * synchronisation) to size the expert launches. */
MXQ_API int mxq_moe_swiglu(mxq_ctx ctx, const mxq_weight* w_gate,
                           const mxq_weight* w_up, const mxq_weight* w_down,
                           size_t n_experts, const float* x,
                           const float* logits, size_t t, size_t k,
                           float* y);

/* The same layer expert-parallel over `world` GPUs of one node (one process
 * and context per GPU): rank r owns experts [r E/world, (r+1) E/world)
 * (E a multiple of world) and passes only their weights.  Every rank passes
 * the same x and logits (all T tokens) and gets the full y.  Each rank routes
 * every token the same way, runs its own experts' GEMMs on the tokens
 * routed to them, writing the expert outputs into its mailbox, then one
 * kernel copies those rows into every other rank's mailbox over NVLink
 * (peer stores into CUDA IPC memory), sets its flag there and waits
 * (bounded) for every rank's flag; the combine then runs as on one GPU.
 * No NCCL on the data path.  y is bit-identical to mxq_moe_swiglu over all
 * E experts on one GPU.  Usage:
 *   mxq_moe_group_create(ctx, rank, world, max_tokens, top_k, d_model, &g,
 *                        handle)  -- handle: MXQ_PEER_HANDLE_BYTES to
 *     exchange; the mailbox holds 2 x max_tokens x top_k x d_model fp32;
 *   (the caller gathers every rank's handle, in rank order)
 *   mxq_moe_group_connect(g, handles)      -- world * 64 bytes
 *   mxq_moe_swiglu_sharded(ctx, g, w_gate, w_up, w_down, E, x, logits, T,
 *                          k, y)           -- w_*: this rank's E/world
 * Every rank must make the same calls in the same order.  A wait that runs
 * out (mxq_moe_group_set_wait_limit, default 2 s) sets the context's status
 * word (mxq_synchronize returns MXQ_ERR_TIMEOUT) and the group must be
 * created again. */
typedef struct mxq_moe_group_s* mxq_moe_group;
MXQ_API int mxq_moe_group_create(mxq_ctx ctx, int rank, int world,
                                 size_t max_tokens, size_t top_k,
                                 size_t d_model, mxq_moe_group* out,
                                 void* handle_out);
MXQ_API int mxq_moe_group_connect(mxq_moe_group g, const void* handles);
MXQ_API int mxq_moe_group_set_wait_limit(mxq_moe_group g, uint32_t wait_us);
MXQ_API int mxq_moe_group_destroy(mxq_moe_group g);
MXQ_API int mxq_moe_swiglu_sharded(mxq_ctx ctx, mxq_moe_group g,
                                   const mxq_weight* w_gate,
                                   const mxq_weight* w_up,
                                   const mxq_weight* w_down,
                                   size_t n_experts, const float* x,
                                   const float* logits, size_t t, size_t k,
                                   float* y);

/* The reference's micro-expert pool (nn/config/model_config.hpp:23-25:
 * 1024 experts, top-16 routed, 2 shared always active; 16-row expert slices
 * of the gate/up matrices, training/fidelity_test.cpp:57-59; executed by
 * mx_rank16_dot_ptrs over the 16 gathered rows, nn/tests/autotest.hpp:
 * 126-136).  The pool's code is absent; this is the library's statement:
 * E = n_routed + n_shared experts (E even), expert e owning rows 16e..16e+15
 * of wg and wu [E*16][D] and columns 16e..16e+15 of wd [D][E*16], shared
 * experts e = n_routed .. E-1.  Per token: h_e = silu(gate rows . x) * (up
 * rows . x) * w_e (w_e = gate[t][j] for routed expert idx[t][j], 1 for
 * shared; gate may be null = 1), MX-quantised per 32-block of wd's K,
 * y[t] = wd . h over the chosen blocks.  Every sum runs in a fixed order, so
 * results are bit-reproducible.  idx/gate [T][k] come from mxq_route_topk or
 * mxq_hashed_route; k > n_routed is MXQ_ERR_INVALID_ARGUMENT.  x [T][D],
 * y [T][D] device pointers; dense weights. */
MXQ_API int mxq_micro_moe(mxq_ctx ctx, mxq_weight wg, mxq_weight wu, mxq_weight wd,
                          size_t n_routed, size_t n_shared, const float* x,
                          const int32_t* idx, const float* gate, size_t t,
                          size_t k, float* y);

/* --------------------------------------------------------- PPO head --- */
/* The rollout head of PPOTrainer::update_step (training/ppo_trainer.cpp:64-66
 * and :77) after its three MX linears (states -> latent -> logits, latent ->
 * value): per row log_probs = log_softmax(logits), action_logp = sum_j
 * log_probs * actions, entropy = -sum_j exp(log_probs) * log_probs.
 * logits/actions/log_probs [rows][cols], action_logp/entropy [rows]. */
MXQ_API int mxq_policy_head(mxq_ctx ctx, const float* logits,
                            const float* actions, size_t rows, size_t cols,
                            float* log_probs, float* action_logp,
                            float* entropy);

/* ---------------------------------------------------------------- GAE --- */
/* nca::env::ReplayMemory::fused_compute_gae
 * (agentic_env/replay_memory.cpp:204-253) over an interleaved [T][E]
 * trajectory (dones as bytes); writes advantages and returns.  Every
 * environment is computed; the reference stops at its MAX_ENVS = 1024 and
 * leaves the others untouched (mxq_gae_ring keeps that cap). */
MXQ_API int mxq_gae(mxq_ctx ctx, const float* rewards, const float* values,
                    const uint8_t* dones, const float* next_values, size_t t,
                    size_t e, float gamma, float lambda, float* adv,
                    float* ret);

/* The same sweep on ReplayMemory's own ring buffer
 * (agentic_env/replay_memory.cpp:204-253, fused_compute_gae(rollout_steps,
 * num_envs, gamma, lambda, final_next_values)): rewards/values/dones/adv/ret
 * are device ring arrays of `capacity` items, `size` of them stored, the
 * next write at `cursor` (a ring that is not full has cursor == size).  The
 * latest t*e items ending at the cursor are swept, t cut to size/e when
 * fewer are stored; indices wrap at the capacity; like the reference, only
 * the first 1024 environments (its MAX_ENVS) are computed and the rest of the
 * ring is left as it was. */
MXQ_API int mxq_gae_ring(mxq_ctx ctx, const float* rewards, const float* values,
                         const uint8_t* dones, const float* next_values,
                         size_t capacity, size_t size, size_t cursor, size_t t,
                         size_t e, float gamma, float lambda, float* adv,
                         float* ret);

/* ------------------------------------------------------------ decoder --- */
/* A dense decoder assembled from the MX linears -- the execution graph the
 * hot path drops into (the caller of nca::linalg::mx_gemv in a model's
 * forward; the 16-row expert slicing of training/fidelity_test.cpp:57-62
 * and the rollout forward of training/ppo_trainer.cpp:57-63 are its
 * reference-side counterparts).  No reference counterpart exists for the
 * decoder itself: the reference's model code is not a transformer.  Per
 * layer: RMSNorm (nn/core/normalization.cpp:16-47) -> QKV linear -> rotary
 * embedding, K/V into a bf16 cache -> causal softmax attention -> O linear ->
 * residual -> RMSNorm -> gate|up linear -> SwiGLU -> down linear -> residual;
 * then RMSNorm and the vocabulary head.  Head dim is 128.  Weights are MX
 * (int4 exponents uniform in [-8, -3], int8 in [-10, -4]) generated from
 * `seed` on the device; the embedding table fp32 ~ N(0, 1); RMSNorm weights
 * 1.  All sequences of a batch share one position. */
typedef struct mxq_decoder_config {
  int n_layers, d_model, n_heads, ffn, vocab;
  int fmt;          /* MXQ_FMT_INT4 or MXQ_FMT_INT8 */
  int max_batch;    /* sequences (K/V cache slots) */
  int max_ctx;      /* positions per sequence */
  int max_rows;     /* token rows per pass (prompt chunking), >= max_batch */
  int value_head;   /* 1: one more head row after the vocabulary (a value) */
  float rope_theta; /* e.g. 10000 */
  float norm_eps;   /* e.g. 1e-5 */
} mxq_decoder_config;
typedef struct mxq_decoder_s* mxq_decoder;

#define MXQ_DEC_QKV 0     /* [3d][d]: q rows, then k, then v */
#define MXQ_DEC_O 1       /* [d][d] */
#define MXQ_DEC_GATE_UP 2 /* [2F][d]: gate rows, then up */
#define MXQ_DEC_DOWN 3    /* [d][F] */
#define MXQ_DEC_LM_HEAD 4 /* [vocab (+1)][d] */

/* Trace points of one layer (mxq_decoder_set_trace): the layer input, the
 * first RMSNorm, QKV before and after the rotary embedding, the attention
 * output, the residual after attention, the second RMSNorm, gate|up, the
 * layer output.  Layer n_layers records its input (the last layer's output)
 * as MXQ_TRACE_IN. */
#define MXQ_TRACE_IN 0
#define MXQ_TRACE_NORM1 1
#define MXQ_TRACE_QKV 2
#define MXQ_TRACE_ROPE 3
#define MXQ_TRACE_ATT 4
#define MXQ_TRACE_H1 5
#define MXQ_TRACE_NORM2 6
#define MXQ_TRACE_GU 7
#define MXQ_TRACE_OUT 8
#define MXQ_TRACE_COUNT 9

MXQ_API int mxq_decoder_create(mxq_ctx ctx, const mxq_decoder_config* cfg,
                               uint64_t seed, mxq_decoder* out);
/* The same decoder tensor-parallel over `world` GPUs of one node (one process
 * and context per GPU; world 1..8 dividing n_heads, ffn a multiple of
 * 32 * world).  Rank `rank` holds the q, k, v rows, K/V cache and attention
 * of heads [rank * n_heads / world, (rank + 1) * n_heads / world), the gate
 * and up rows of FFN units [rank * ffn / world, (rank + 1) * ffn / world),
 * and the O and down columns (K) of those heads and units, whole 32-blocks
 * (the MX block dots of mx_gemv, nn/tests/test_auto_generated.cpp:56, are
 * the unsharded weight's); every weight byte is the unsharded decoder's for
 * the same seed.  The embedding, RMSNorm weights and vocabulary head are
 * replicated.  After the O and after the down linear of every layer, one
 * kernel stores this rank's partial sums into every rank's mailbox (peer
 * stores over NVLink into CUDA IPC memory), sets its flag there and waits
 * (bounded) for every rank's flag; the residual kernel adds the partials in
 * rank order, so every rank holds the same hidden state.  No NCCL on the
 * data path.  Usage:
 *   mxq_decoder_create_sharded(ctx, cfg, seed, rank, world, &dec, handle)
 *     -- handle: MXQ_PEER_HANDLE_BYTES to exchange;
 *   (the caller gathers every rank's handle, in rank order)
 *   mxq_decoder_connect(dec, handles)   -- world * 64 bytes
 * then prefill / decode / score as on one GPU, with the same tokens in the
 * same order on every rank; every rank returns the same full logits.  They
 * equal the unsharded decoder's within fp32 rounding (the block sums of O
 * and down are added in another order); with world 1 (the sharded code path
 * on one GPU, exchanging through its own mailbox) bit for bit.  A wait that
 * runs out (mxq_decoder_set_wait_limit, default 2 s) sets the context's
 * status word (mxq_synchronize returns MXQ_ERR_TIMEOUT) and the group must
 * be created again.  Trace points QKV, ROPE, ATT and GU hold this rank's
 * columns ([rows][3 d / world], [rows][d / world], [rows][2 ffn / world]);
 * the others the full rows. */
MXQ_API int mxq_decoder_create_sharded(mxq_ctx ctx, const mxq_decoder_config* cfg,
                                       uint64_t seed, int rank, int world,
                                       mxq_decoder* out, void* handle_out);
MXQ_API int mxq_decoder_connect(mxq_decoder dec, const void* handles);
MXQ_API int mxq_decoder_set_wait_limit(mxq_decoder dec, uint32_t wait_us);
MXQ_API int mxq_decoder_destroy(mxq_decoder dec);
/* Forget every cached position. */
MXQ_API int mxq_decoder_reset(mxq_decoder dec);
MXQ_API int mxq_decoder_length(mxq_decoder dec, int* len);
/* Prompt tokens int32 [b][t] (host or device) from position 0; fills the
 * cache and writes the last position's logits fp32 [b][vocab] (device or
 * host; may be null). */
MXQ_API int mxq_decoder_prefill(mxq_decoder dec, const int32_t* tokens,
                                size_t b, size_t t, float* logits);
/* One new token per sequence at the current position; logits [b][vocab].
 * The first call for a batch size runs plain launches and records the step
 * as a CUDA graph; later calls replay it. */
MXQ_API int mxq_decoder_decode(mxq_decoder dec, const int32_t* tokens,
                               size_t b, float* logits);
/* Teacher-forced scoring (the PPO rollout forward): tokens [b][t] ->
 * logp [b][t-1] = log p(token i+1 | tokens 0..i) and, with a value head,
 * values [b][t] (may be null).  Sequences go through max_rows / t at a time;
 * the cache is reset afterwards. */
MXQ_API int mxq_decoder_score(mxq_decoder dec, const int32_t* tokens, size_t b,
                              size_t t, float* logp, float* values);
/* The decoder's weight handles (MXQ_DEC_*; layer ignored for the head). */
MXQ_API int mxq_decoder_weight(mxq_decoder dec, int layer, int which,
                               mxq_weight* out);
/* Rows [row0, row0 + nrows) of the embedding table fp32 [vocab][d] into
 * `out` (device or host memory). */
MXQ_API int mxq_decoder_embedding(mxq_decoder dec, size_t row0, size_t nrows,
                                  float* out);
/* Record the trace points of `layer` (-1: off) on the following passes;
 * mxq_decoder_get_trace copies `count` floats of trace `id` (the last pass's
 * rows) to device or host memory. */
MXQ_API int mxq_decoder_set_trace(mxq_decoder dec, int layer);
MXQ_API int mxq_decoder_get_trace(mxq_decoder dec, int id, float* out,
                                  size_t count);

/* The MX bytes of a dense weight back in the MXINT8Tensor layout: data int8
 * [N][K] or packed int4 [N][K/2], scales [N][K/32] (host memory).  The
 * inverse of mxq_weight_create (for serialisation and checking). */
MXQ_API int mxq_weight_download(mxq_weight w, void* data_host,
                                uint8_t* scales_host);

/* On-disk MX weight (no counterpart in the reference, whose MX containers
 * lived only in memory; its checkpoints were LibTorch archives,
 * training/offline_trainer.cpp:105-128).  Little-endian file: magic "MXQW",
 * u32 version 1, u32 fmt (4 or 8), u32 flags (0), u64 N, u64 K, then
 * the MXINT8Tensor bytes (data [N][K] int8 or [N][K/2] packed int4), then the
 * E8M0 scales [N][K/32].  Dense weights only (block-sparse:
 * MXQ_ERR_UNSUPPORTED). */
MXQ_API int mxq_weight_save(mxq_weight w, const char* path);
MXQ_API int mxq_weight_load(mxq_ctx ctx, const char* path, mxq_weight* out);

#ifdef __cplusplus
}
#endif
#endif /* MXQ_H */
