// rcu_static.cu -- a matmul entry point that allocates no device memory.
//
// Some callers cannot call cudaMalloc at the point where they need a matmul: an engine
// that hands all of HBM to its own pool at start-up (weights + KV cache), or a process whose
// memory belongs to PyTorch's caching allocator, would either fail the allocation or break
// the pool's accounting, and cudaMalloc/cudaFree can also synchronise the device in the
// middle of a latency-critical decode step. rcu_matmul_f32_static serves them: it takes f32
// activations and a weight, quantizes the activations into a fixed scratch area that lives
// in this file as a static __device__ array, and runs the same GEMV as rcu_matmul_multi.
//
// The scratch holds at most kStaticMaxTok tokens of kStaticMaxK values in both activation
// formats (about 322 KB); every GPU that loads this library keeps it until process exit.
// All calls share it, so calls whose work overlaps on the GPU (different streams, or
// different contexts on the same device) race on it and must be ordered by the caller.
#include "rcu_kernels.h"

namespace rcu {

constexpr uint64_t kStaticMaxTok = 8;
constexpr uint64_t kStaticMaxK = 16384;
constexpr uint64_t al256(uint64_t x) { return (x + 255) & ~255ull; }
// Q8_0: codes, d, s, code sums; Q8_K: codes, d, bsums
constexpr uint64_t kOffQ0 = 0;
constexpr uint64_t kOffD0 = kOffQ0 + al256(kStaticMaxTok * kStaticMaxK);
constexpr uint64_t kOffS0 = kOffD0 + al256(kStaticMaxTok * (kStaticMaxK / QK) * 4);
constexpr uint64_t kOffSum0 = kOffS0 + al256(kStaticMaxTok * (kStaticMaxK / QK) * 4);
constexpr uint64_t kOffQK = kOffSum0 + al256(kStaticMaxTok * (kStaticMaxK / QK) * 4);
constexpr uint64_t kOffDK = kOffQK + al256(kStaticMaxTok * kStaticMaxK);
constexpr uint64_t kOffBsK = kOffDK + al256(kStaticMaxTok * (kStaticMaxK / QK_K) * 4);
constexpr uint64_t kStaticBytes = kOffBsK + al256(kStaticMaxTok * (kStaticMaxK / 16) * 2);

// Host code must never use this name as an address: on the host it is only a stand-in.
// The device address comes from cudaGetSymbolAddress (static_base below).
static __device__ __align__(256) uint8_t g_static_acts[kStaticBytes];

// Device address of g_static_acts on the context's device, looked up by the context's first
// call and kept in the context. A context belongs to one device, and one created after a
// device reset looks the address up again.
static int static_base(rcu_ctx *ctx, uint8_t **out) {
    if (!ctx->static_scratch) {
        int cur = -1;
        RCU_CUDA_TRY(ctx, cudaGetDevice(&cur));
        if (cur != ctx->device) RCU_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_static_acts);
        if (cur != ctx->device && cur >= 0) cudaSetDevice(cur);
        if (e != cudaSuccess) return cuda_err(ctx, e, "cudaGetSymbolAddress(g_static_acts)");
        ctx->static_scratch = (uint8_t *)p;
    }
    *out = ctx->static_scratch;
    return RCU_OK;
}

}  // namespace rcu

using namespace rcu;

extern "C" {

int32_t rcu_matmul_f32_static(rcu_ctx *ctx, const rcu_weight *w, const float *x_dev, uint64_t n_tok, float *out_dev,
                              uint64_t ld) {
    if (!ctx || !w || !x_dev || !out_dev) return set_err(ctx, RCU_ERR_INVALID, "null argument");
    if (n_tok == 0) return set_err(ctx, RCU_ERR_RUNTIME, "empty batch");
    if (n_tok > kStaticMaxTok)
        return set_err(ctx, RCU_ERR_INVALID, "static matmul: at most " + std::to_string(kStaticMaxTok) + " tokens");
    if (w->cols > kStaticMaxK)
        return set_err(ctx, RCU_ERR_INVALID, "static matmul: rows longer than " + std::to_string(kStaticMaxK) + " values");
    if (!gemv_supported(w->type))
        return set_err(ctx, RCU_ERR_UNSUPPORTED, "no GPU kernel for ggml type " + std::to_string(w->type));
    if (ld < w->rows) return set_err(ctx, RCU_ERR_INVALID, "ld smaller than rows");
    uint8_t *base = nullptr;
    if (int st = static_base(ctx, &base)) return st;
    ActsView a{};
    a.q0 = (int8_t *)(base + kOffQ0);
    a.d0 = (float *)(base + kOffD0);
    a.s0 = (float *)(base + kOffS0);
    a.sum0 = (int32_t *)(base + kOffSum0);
    a.qk = (int8_t *)(base + kOffQK);
    a.dk = (float *)(base + kOffDK);
    a.bsk = (int16_t *)(base + kOffBsK);
    a.n_tok = (uint32_t)n_tok;
    a.k = (uint32_t)w->cols;
    const uint32_t fmt = act_format(w->type);
    if (int st = launch_quantize(ctx, a, x_dev, (uint32_t)n_tok, (uint32_t)w->cols, fmt)) return st;
    a.have = fmt;
    const HostJob job{w, out_dev, ld};
    return launch_gemv(ctx, a, &job, 1, 0, (uint32_t)n_tok);
}

}  // extern "C"
