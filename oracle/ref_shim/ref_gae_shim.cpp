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
