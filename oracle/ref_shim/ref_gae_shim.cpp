// ref_gae_shim.cpp -- C entry point around the reference's own
// nca::env::ReplayMemory::fused_compute_gae (agentic_env/replay_memory.cpp),
// compiled from the reference sources by oracle/Makefile into
// oracle/_ref/libref_gae.so.  Test infrastructure: used only to pin the GAE
// restatement in mx_oracle.c against the reference's compiled code.
#include "agentic_env/replay_memory.hpp"
#include "agentic_env/env.hpp"
#include <cstdlib>
#include <cstring>
#include <vector>

namespace nca::env {
// The reference declares these in agentic_env/env.hpp and defines them with
// Windows _aligned_malloc; this is the POSIX equivalent.
void* alloc_aligned(size_t size, size_t alignment) {
    size_t s = (size + alignment - 1) / alignment * alignment;
    return std::aligned_alloc(alignment, s ? s : alignment);
}
void free_aligned(void* p) { std::free(p); }
}

extern "C" int ref_gae(const float* rewards, const float* values,
                       const unsigned char* dones, const float* next_values,
                       size_t T, size_t E, float gamma, float lambda,
                       float* adv, float* ret) {
    size_t n = T * E;
    nca::env::ReplayMemory rm(n, 1, 1);
    float s = 0.f, a = 0.f;
    for (size_t i = 0; i < n; ++i) rm.push(&s, &a, rewards[i], dones[i] != 0);
    rm.write_values(n, values);
    rm.fused_compute_gae(T, E, gamma, lambda, next_values);
    std::memcpy(adv, rm.get_advantages(), n * sizeof(float));
    std::memcpy(ret, rm.get_returns(), n * sizeof(float));
    return 0;
}

// The ring form: push n_push items one by one into a ReplayMemory of `cap`
// items (it wraps when n_push > cap), write the latest n_val values, run
// fused_compute_gae(T, E), and copy out the whole ring plus (size, cursor).
extern "C" int ref_gae_ring(const float* rewards, const unsigned char* dones, size_t n_push,
                            const float* values, size_t n_val, size_t cap, size_t T, size_t E,
                            const float* next_values, float gamma, float lambda,
                            float* r_out, float* v_out, unsigned char* d_out, float* adv_out,
                            float* ret_out, unsigned long long* meta) {
    nca::env::ReplayMemory rm(cap, 1, 1);
    float s = 0.f, a = 0.f;
    for (size_t i = 0; i < n_push; ++i) rm.push(&s, &a, rewards[i], dones[i] != 0);
    rm.write_values(n_val, values);
    rm.fused_compute_gae(T, E, gamma, lambda, next_values);
    // the ring's own arrays: the latest span views expose rewards/dones, the
    // accessors values/advantages/returns (all `cap` long)
    nca::env::BatchSpan spans[2];
    size_t ns = rm.get_latest_spans(rm.size(), spans);
    std::memset(r_out, 0, cap * sizeof(float));
    std::memset(d_out, 0, cap);
    const float* base_r = nullptr;
    const bool* base_d = nullptr;
    for (size_t j = 0; j < ns; ++j) {
        // the span starting lowest in memory starts at ring index 0 when the
        // ring has wrapped; otherwise the single span starts at index 0 too
        if (!base_r || spans[j].rewards < base_r) {
            base_r = spans[j].rewards;
            base_d = spans[j].dones;
        }
    }
    for (size_t j = 0; j < ns; ++j) {
        size_t off = (size_t)(spans[j].rewards - base_r);
        for (size_t i = 0; i < spans[j].count; ++i) {
            r_out[off + i] = spans[j].rewards[i];
            d_out[off + i] = spans[j].dones[i] ? 1 : 0;
        }
    }
    (void)base_d;
    std::memcpy(v_out, rm.get_values(), cap * sizeof(float));
    std::memcpy(adv_out, rm.get_advantages(), cap * sizeof(float));
    std::memcpy(ret_out, rm.get_returns(), cap * sizeof(float));
    meta[0] = rm.size();
    meta[1] = n_push % cap;
    return 0;
}
