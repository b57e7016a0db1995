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

}  // namespace rcu
