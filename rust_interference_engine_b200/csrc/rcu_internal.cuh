// rcu_internal.cuh -- shared device/host helpers of librie_cuda (sm_100a only).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/rie_cuda.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "librie_cuda is built for sm_100a (B200) only"
#endif

namespace rcu {

// ggml type ids (reference: crates/rie-core/src/quant/mod.rs:34-51)
enum : int { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q4_1 = 3, T_Q5_0 = 6, T_Q5_1 = 7, T_Q8_0 = 8,
             T_Q2_K = 10, T_Q3_K = 11, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14, T_BF16 = 30 };
constexpr int QK = 32, QK_K = 256;

__host__ __device__ inline int block_size(int t) {
    switch (t) {
        case T_Q4_0: case T_Q4_1: case T_Q5_0: case T_Q5_1: case T_Q8_0: return QK;
        case T_Q2_K: case T_Q3_K: case T_Q4_K: case T_Q5_K: case T_Q6_K: return QK_K;
        case T_F32: case T_F16: case T_BF16: return 1;
        default: return 0;
    }
}
__host__ __device__ inline int block_bytes(int t) {
    switch (t) {
        case T_F32: return 4;
        case T_F16: case T_BF16: return 2;
        case T_Q4_0: return 18;
        case T_Q4_1: return 20;
        case T_Q5_0: return 22;
        case T_Q5_1: return 24;
        case T_Q8_0: return 34;
        case T_Q2_K: return 84;
        case T_Q3_K: return 110;
        case T_Q4_K: return 144;
        case T_Q5_K: return 176;
        case T_Q6_K: return 210;
        default: return 0;
    }
}
// Activation format consumed by each weight type (quant/mod.rs:118-124).
__host__ __device__ inline uint32_t act_format(int t) {
    switch (t) {
        case T_Q4_0: case T_Q4_1: case T_Q5_0: case T_Q5_1: case T_Q8_0: return RCU_ACT_Q8_0;
        case T_Q4_K: case T_Q5_K: case T_Q6_K: return RCU_ACT_Q8K;
        default: return 0;
    }
}
inline bool gemv_supported(int t) {
    return t == T_Q4_0 || t == T_Q4_1 || t == T_Q5_0 || t == T_Q5_1 || t == T_Q8_0 || t == T_Q4_K ||
           t == T_Q5_K || t == T_Q6_K;
}

// Device-side error bits (written with atomicOr into rcu_ctx::dev_err).
enum : uint32_t {
    ERR_TIMEOUT_FULL = 1u,
    ERR_TIMEOUT_EMPTY = 2u,
    ERR_TIMEOUT_DRAIN = 4u,
    ERR_BAD_ARG = 8u,
    ERR_TIMEOUT_PEER = 16u  // a tensor-parallel peer's partial rows did not arrive in time
};

// Quantized activations in HBM, structure-of-arrays (the reference's BlockQ8_0 /
// BlockQ8K hold the same fields per block; rcu_acts_export writes that layout).
struct ActsView {
    // Q8_0 (32-value blocks)
    int8_t *q0;       // [n_tok][k]
    float *d0;        // [n_tok][k/32]
    float *s0;        // [n_tok][k/32]  s = d * sum(q) as the selected tier defines it
    int32_t *sum0;    // [n_tok][k/32]  exact sum of the stored (clamped) codes
    // Q8_K (256-value blocks)
    int8_t *qk;       // [n_tok][k]
    float *dk;        // [n_tok][k/256]
    int16_t *bsk;     // [n_tok][k/16]
    uint32_t n_tok, k;
    uint32_t have;    // RCU_ACT_* bits
};

// ---- small device helpers -----------------------------------------------------------
__device__ __forceinline__ float f16_bits_to_f32(uint32_t bits) {
    return __half2float(__ushort_as_half((unsigned short)(bits & 0xffffu)));
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

// Every wait in this library is bounded by wall time; on expiry the waiting thread
// records an error bit and gives up, so a bug surfaces as a status, never as a hang.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, uint32_t *err, uint32_t code) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
            atomicOr(err, code);
            return false;
        }
    }
}
// As mbar_wait_bounded, but each try_wait may suspend the thread for up to `hint_ns` until the
// phase completes (fewer spin instructions taken from the warps doing the work).
__device__ __forceinline__ bool mbar_try_wait_hint(uint64_t *bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t *bar, uint32_t parity, uint32_t *err, uint32_t code) {
    constexpr uint32_t kHintNs = 100000;  // 0.1 ms; the phase completing wakes the thread earlier
    if (mbar_try_wait_hint(bar, parity, kHintNs)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        if (mbar_try_wait_hint(bar, parity, kHintNs)) return true;
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
            atomicOr(err, code);
            return false;
        }
    }
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// 1-D bulk copy global -> shared (TMA engine), completion counted on an mbarrier.
// Both addresses 16-byte aligned, bytes a multiple of 16. No multicast.
__device__ __forceinline__ void bulk_g2s(void *dst_smem, const void *src_gmem, uint32_t bytes, uint64_t *bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// 4 bytes starting at an even (2-aligned) shared-memory byte offset.
__device__ __forceinline__ uint32_t lds_u32_at(const uint8_t *base, uint32_t off) {
    const uint32_t *w = reinterpret_cast<const uint32_t *>(base + (off & ~3u));
    const uint32_t sh = (off & 3u) * 8u;
    return __funnelshift_r(w[0], w[1], sh);
}
__device__ __forceinline__ int dp4a(uint32_t a, uint32_t b, int c) { return __dp4a((int)a, (int)b, c); }

}  // namespace rcu

// ---- host-side context ---------------------------------------------------------------
struct rcu_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    int rounding = RCU_ROUND_NEAREST_EVEN;
    int num_sms = 148;
    size_t max_smem_optin = 0;
    uint32_t *dev_err = nullptr;  // device error bits
    bool pdl = true;              // programmatic dependent launch for the kernels of this library
    // limit of the waits on other ranks (fused all-reduce): RIE_WAIT_LIMIT_MS, rcu_set_wait_limit_ms
    uint64_t wait_limit_ns = 2000000000ull;
    // GEMV weights may be streamed before the previous kernel has finished (set while the
    // forward scheduler runs: its weights are written once, at load time)
    bool early_weights = false;
    bool static_weights = false;  // caller promise (rcu_set_static_weights): early_weights outside the forward too
    bool gemm_i8 = false;          // prefill: int8 GEMM with exact block sums for Q4_0 weights
    bool gemv_kq = true;           // batch-1 K-quant GEMV on the tensor cores (RIE_GEMV_KQ=0: lane GEMV)
    uint64_t gemv_kq_min_bytes = 8ull << 20;  // ... for launches of at least this many weight bytes (RIE_GEMV_KQ_MIN_MB)
    uint32_t gemv_kq_q4_0_min_k = 4096;       // ... and Q4_0 rows of at least this many values (RIE_GEMV_KQ_Q4_0_MIN_K)
    void *h_act = nullptr;         // f16 activations of the prefill GEMM (grown on demand)
    size_t h_act_cap = 0;
    void *k_part = nullptr;        // split-K partial tiles of the prefill GEMM (grown on demand)
    size_t k_part_cap = 0;
    uint32_t *k_cnt = nullptr;     // split-K tile counters (zero between launches)
    size_t k_cnt_cap = 0;
    // device address of the allocation-free matmul's static scratch (rcu_static.cu), looked
    // up by this context's first such call
    uint8_t *static_scratch = nullptr;
    bool fuse_post = true;  // decode attention does the q/k post-processing and KV append (RIE_FUSE_POST=0: own kernel)
    // block-sum capture (rcu_matmul_block_sums): set only for the duration of that call
    int32_t *dbg_sums = nullptr;
    uint32_t dbg_nbs = 0;
    int dbg_kernel = -1;  // 0: lane GEMV, 1: tensor-core GEMV
    std::string last_error;
};

struct rcu_weight {
    rcu_ctx *ctx = nullptr;
    int type = 0;
    uint64_t rows = 0, cols = 0, row_bytes = 0;
    uint8_t *data = nullptr;  // device, GGUF block layout, row-major
    bool owned = false;
    bool padded = false;  // >= 16 readable bytes past the end (bulk copies may round up)
};

struct rcu_acts {
    rcu_ctx *ctx = nullptr;
    uint64_t max_tok = 0, max_k = 0;
    void *buf = nullptr;
    rcu::ActsView v{};
};

namespace rcu {
int set_err(rcu_ctx *c, int code, const std::string &msg);
int cuda_err(rcu_ctx *c, cudaError_t e, const char *what);
}  // namespace rcu

namespace rcu {
// Programmatic dependent launch. Kernels started with launch_k may begin while the kernel
// before them in the stream is still running. Each of them calls pdl_wait() before its first
// access to memory that an earlier kernel writes or reads (everything but the weights), and
// pdl_trigger() to let the kernel after it launch early. pdl_wait() returns once the previous
// kernel has completed and its writes are visible; on a plain launch both are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
// Orders this thread's generic-proxy global writes before later async-proxy accesses (bulk
// copies) that another thread issues after synchronizing with it.
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// Every kernel of the library runs with the largest shared-memory carveout, so that an SM
// never has to drain and re-split L1 / shared memory between consecutive kernels (the GEMV
// needs the maximum) and a dependent kernel can become resident next to the running one.
cudaError_t prefer_max_shared(const void *kern);

template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(const rcu_ctx *ctx, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                            Args... args) {
    if (cudaError_t e = prefer_max_shared(reinterpret_cast<const void *>(kern))) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = ctx->pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}
}  // namespace rcu

#define RCU_CUDA_TRY(ctx, expr)                                           \
    do {                                                                  \
        cudaError_t _e = (expr);                                          \
        if (_e != cudaSuccess) return rcu::cuda_err((ctx), _e, #expr);    \
    } while (0)
