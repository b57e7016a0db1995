// rcu_kernels.h -- host launchers of librie_cuda's kernels (internal).
#pragma once
#include "rcu_internal.cuh"

namespace rcu {

int launch_quantize(rcu_ctx *ctx, const ActsView &a, const float *x, uint32_t n_tok, uint32_t k, uint32_t formats);

struct HostJob {
    const rcu_weight *w;
    float *out;
    uint64_t ld;
};
// Decode GEMV over up to kGemvMaxJobs jobs sharing one activation batch (n_tok <= 8).
constexpr int kGemvMaxJobs = 96;
int launch_gemv(rcu_ctx *ctx, const ActsView &a, const HostJob *jobs, int n_jobs, uint32_t tok0, uint32_t n_tok);
// Int8 tensor-core GEMM (n_tok > 8). Returns RCU_ERR_UNSUPPORTED for types it lacks.
int launch_gemm(rcu_ctx *ctx, const ActsView &a, const HostJob *jobs, int n_jobs);
// Exact per-block integer sums of one (row, token) pair.
int launch_block_sums(rcu_ctx *ctx, const ActsView &a, const rcu_weight *w, uint64_t row, uint64_t tok,
                      int32_t *out);

// KV append / attention with the position either by value (pos_ptr == nullptr) or read
// from device memory (graph replay). n_split == 0 sizes the split grid from pos0; scratch
// == nullptr uses the context's growable scratch (may allocate).
int launch_kv_store(rcu_ctx *ctx, rcu_kv *kv, const float *k, const float *v, uint64_t n_tok, uint64_t pos0,
                    const uint64_t *pos_ptr);
int launch_attention(rcu_ctx *ctx, const rcu_kv *kv, const float *q, uint64_t n_tok, uint64_t n_head, uint64_t pos0,
                     const uint64_t *pos_ptr, uint64_t window, float softcap, float *out, uint32_t n_split,
                     float *scratch);
uint32_t attention_max_splits(const rcu_kv *kv, uint64_t window);
uint64_t attention_scratch_bytes(const rcu_kv *kv, uint64_t n_tok, uint64_t n_head, uint32_t n_split);

}  // namespace rcu
