// rcu_forward.cu -- device forward scheduler: the transformer layer loop of the reference's
// CPU backend (crates/rie-core/src/model/cpu.rs:210-409, dense_ffn :431-467) over the
// quantized matmul, KV-cache and attention kernels of this library.
//
// Per layer and batch: [residual +] RMSNorm + Q8 activations -> one matmul_multi for Q,K,V
// -> bias / per-head q,k RMSNorm / RoPE / attn_scale + KV append -> attention (merge +
// Q8 activations) -> Wo -> post-norm + residual + RMSNorm + Q8 activations -> gate+up in
// one launch -> SwiGLU/GELU + Q8 activations -> down; the down residual is added by the
// next norm. Ten launches per layer, all queued on the backend stream; the host only
// validates arguments and launches.
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include <nccl.h>

#include "rcu_actq.cuh"
#include "rcu_blocks.cuh"
#include "rcu_kernels.h"

namespace rcu {

struct LayerW {
    const rcu_weight *wq = nullptr, *wk = nullptr, *wv = nullptr, *wo = nullptr;
    const rcu_weight *gate = nullptr, *up = nullptr, *down = nullptr;
    const float *attn_norm = nullptr, *ffn_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
    const float *bq = nullptr, *bk = nullptr, *bv = nullptr, *post_attn = nullptr, *post_ffn = nullptr;
    bool swa = false;
    // mixture of experts (model/mod.rs:147-180): F32 router [n_expert][n_embd], experts
    // stacked [expert][rows][cols], optional shared expert with an F32 gate vector
    const rcu_weight *router = nullptr, *gate_exps = nullptr, *up_exps = nullptr, *down_exps = nullptr;
    const rcu_weight *gate_sh = nullptr, *up_sh = nullptr, *down_sh = nullptr;
    const float *sh_gate = nullptr;
};

}  // namespace rcu

struct rcu_model {
    rcu_ctx *ctx = nullptr;
    rcu_model_config cfg{};
    int tp_rank = 0, tp_world = 1;  // tensor-parallel shard held by this model
    std::map<std::string, rcu_weight *> w;
    std::map<std::string, float *> vec;  // 1-D float tensors as device f32
    std::vector<rcu_weight *> slices;
};

struct rcu_backend {
    rcu_model *m = nullptr;
    rcu_ctx *ctx = nullptr;
    rcu_model_config cfg{};  // this rank's dimensions (heads, FFN rows, vocab rows) under TP
    ncclComm_t comm = nullptr;  // tensor-parallel communicator (world > 1)
    float *logits_local = nullptr, *logits_gather = nullptr;
    // fused all-reduce over NVLink (tensor parallel, batches of <= 8 tokens): receive buffer
    // [2 slots][P ranks][max_batch][n_embd], arrival counters [2 per layer][P], the forward
    // count, and the peers' buffers / counters mapped into this process (CUDA IPC)
    // mixture-of-experts scratch: router logits, shared-expert gates, chosen experts and
    // their weights per token, expert hidden rows and outputs, second activation batch
    float *moe_logits = nullptr, *moe_sgate = nullptr, *moe_w = nullptr, *moe_g = nullptr, *moe_u = nullptr;
    float *moe_y = nullptr, *moe_ys = nullptr;
    uint32_t *moe_sel = nullptr;
    // grouped expert GEMMs (batches of kMoeGroupedMinTok tokens or more): slot of every
    // (token, choice) pair in the expert-sorted order, source token of every slot, expert
    // offsets on the device and their host copy (pinned)
    uint32_t *moe_slot = nullptr, *moe_row = nullptr, *moe_off = nullptr, *moe_off_host = nullptr;
    // pinned staging of rcu_backend_forward's host tokens (max_batch) and one row of logits, so
    // that both copies run as DMA instead of through the driver's pageable staging
    uint32_t *tok_pin = nullptr;
    float *logits_pin = nullptr;
    uint32_t ep_e0 = 0, ep_n = 0xffffffffu;  // experts of this rank: [ep_e0, ep_e0 + ep_n)
    rcu_acts *acts2 = nullptr;
    bool ar_ok = false;
    float *ar_buf = nullptr;
    uint32_t *ar_flags = nullptr;
    uint64_t *ar_epoch = nullptr;
    float *ar_peer_buf[8] = {};
    uint32_t *ar_peer_flags[8] = {};
    uint64_t n_ctx = 0, max_batch = 0;
    int kv_type = 0;
    std::vector<rcu::LayerW> layers;
    const rcu_weight *embd = nullptr, *out = nullptr;
    const float *out_norm = nullptr;
    std::vector<rcu_kv *> kv;
    rcu_acts *acts = nullptr;
    float *x = nullptr, *xn = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *att = nullptr, *o = nullptr;
    float *g = nullptr, *u = nullptr, *logits = nullptr, *inv_freq = nullptr, *inv_freq_swa = nullptr;
    uint32_t *tokens = nullptr;
    uint64_t *pos_dev = nullptr;  // position of the batch, read by the kernels (graph replay)
    float *attn_scratch = nullptr;
    bool fused_merge = true;  // attention merge quantizes for Wo in the same kernel
    uint32_t ff_max = 0;
    uint64_t hidden_rows = 0;
    std::vector<void *> allocs;
    // The backend runs on its own stream (stream capture needs a non-default stream) and
    // joins the context stream with events on entry and exit.
    cudaStream_t stream = nullptr;
    cudaEvent_t ev_in = nullptr, ev_out = nullptr, ev_plan = nullptr;
    bool use_graphs = true;
    int decode_calls = 0;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t graph_exec = nullptr;
};

namespace rcu {

// ---- kernels ---------------------------------------------------------------------------

// Dequantize one GGUF block (reference.rs:53-215) into y (block_size values).
__device__ void dequant_block(int t, const uint8_t *b, float *y, int lane, int nl) {
    auto f16 = [&](int off) { return __half2float(__ushort_as_half((unsigned short)(b[off] | (b[off + 1] << 8)))); };
    switch (t) {
        case T_Q4_0: {
            const float d = f16(0);
            for (int j = lane; j < 16; j += nl) {
                y[j] = (float)((b[2 + j] & 0xF) - 8) * d;
                y[j + 16] = (float)((b[2 + j] >> 4) - 8) * d;
            }
            break;
        }
        case T_Q4_1: {
            const float d = f16(0), m = f16(2);
            for (int j = lane; j < 16; j += nl) {
                y[j] = (float)(b[4 + j] & 0xF) * d + m;
                y[j + 16] = (float)(b[4 + j] >> 4) * d + m;
            }
            break;
        }
        case T_Q5_0: case T_Q5_1: {
            const bool one = t == T_Q5_1;
            const float d = f16(0), m = one ? f16(2) : 0.0f;
            const int o = one ? 4 : 2;
            const uint32_t qh = b[o] | (b[o + 1] << 8) | (b[o + 2] << 16) | ((uint32_t)b[o + 3] << 24);
            for (int j = lane; j < 16; j += nl) {
                const uint32_t xh0 = ((qh >> j) << 4) & 0x10, xh1 = (qh >> (j + 12)) & 0x10;
                const uint32_t a = (b[o + 4 + j] & 0xFu) | xh0, c = (b[o + 4 + j] >> 4) | xh1;
                y[j] = one ? (float)a * d + m : (float)((int)a - 16) * d;
                y[j + 16] = one ? (float)c * d + m : (float)((int)c - 16) * d;
            }
            break;
        }
        case T_Q8_0: {
            const float d = f16(0);
            for (int j = lane; j < 32; j += nl) y[j] = (float)(int8_t)b[2 + j] * d;
            break;
        }
        case T_Q4_K: case T_Q5_K: {
            const float d = f16(0), mn = f16(2);
            const uint32_t s[3] = {(uint32_t)b[4] | (b[5] << 8) | (b[6] << 16) | ((uint32_t)b[7] << 24),
                                   (uint32_t)b[8] | (b[9] << 8) | (b[10] << 16) | ((uint32_t)b[11] << 24),
                                   (uint32_t)b[12] | (b[13] << 8) | (b[14] << 16) | ((uint32_t)b[15] << 24)};
            for (int i = lane; i < 256; i += nl) {
                const int j = i / 64, l = i % 32, hi = (i / 32) & 1;
                uint32_t sc, m;
                scale_min_k4(2 * j + hi, s, sc, m);
                uint32_t q;
                if (t == T_Q4_K) {
                    q = hi ? (b[16 + 32 * j + l] >> 4) : (b[16 + 32 * j + l] & 0xF);
                } else {
                    q = (hi ? (b[48 + 32 * j + l] >> 4) : (b[48 + 32 * j + l] & 0xF)) +
                        ((b[16 + l] & ((hi ? 2u : 1u) << (2 * j))) ? 16u : 0u);
                }
                y[i] = d * (float)sc * (float)q - mn * (float)m;
            }
            break;
        }
        case T_Q6_K: {
            const float d = f16(208);
            for (int i = lane; i < 256; i += nl) {
                const int n = i / 128, r = i % 128, k = r / 32, l = r % 32, is = l / 16;
                const uint8_t *ql = b + 64 * n, *qh = b + 128 + 32 * n;
                const int8_t *sc = (const int8_t *)(b + 192 + 8 * n);
                const int lo = (k & 1) ? ql[l + 32] : ql[l];
                const int q = (((k < 2) ? (lo & 0xF) : (lo >> 4)) | (((qh[l] >> (2 * k)) & 3) << 4)) - 32;
                y[i] = d * (float)sc[is + 2 * k] * (float)q;
            }
            break;
        }
        default: break;
    }
}

__global__ void k_embed(const uint32_t *__restrict__ tokens, int type, const uint8_t *__restrict__ w, uint64_t row_bytes,
                        uint32_t e, float scale, float *__restrict__ x) {
    pdl_wait();
    pdl_trigger();
    const uint32_t t = blockIdx.x;
    const uint8_t *row = w + (uint64_t)tokens[t] * row_bytes;
    float *y = x + (uint64_t)t * e;
    if (type == T_F32) {
        for (uint32_t i = threadIdx.x; i < e; i += blockDim.x) y[i] = reinterpret_cast<const float *>(row)[i] * scale;
        return;
    }
    if (type == T_F16) {
        for (uint32_t i = threadIdx.x; i < e; i += blockDim.x)
            y[i] = __half2float(reinterpret_cast<const __half *>(row)[i]) * scale;
        return;
    }
    const int bs = block_size(type), bb = block_bytes(type);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (uint32_t blk = warp; blk < e / bs; blk += nw) {
        dequant_block(type, row + (uint64_t)blk * bb, y + (uint64_t)blk * bs, lane, 32);
        __syncwarp();
        if (scale != 1.0f)
            for (int i = lane; i < bs; i += 32) y[blk * bs + i] *= scale;
    }
}

__device__ __forceinline__ float block_sum(float v, float *red) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float s = 0.0f;
    for (int i = 0; i < nw; i++) s += red[i];
    return s;
}

// Residual + RMSNorm + activation quantization in one pass over a token row (one CTA of
// 1024 threads per token, value i of the row in thread i % 1024, slot i / 1024):
//   x += post_norm(o) * rs        when o is given (ops.rs:17-24, cpu.rs:330-345)
//   xn = (x * (1 / rms(x))) * w   (ops.rs:7-14)
// then xn is quantized into the matmul activations (ActOut formats) and, when xn_f32 is
// given, stored as f32. Each thread writes back only the x values it read, so x may be
// updated in place. The norm weights, and x when `x_ready` (x was last written by a kernel
// that has completed before this one starts: three or more launches earlier), are loaded
// before waiting for the previous kernel, which produced o.
constexpr int kNormThreads = 1024;

// Tensor parallel with the fused all-reduce: instead of o, the norm sums the P ranks' partial
// rows that the row-parallel GEMVs pushed into this GPU's receive buffer (in rank order, so
// every rank computes the same values), after every rank's arrival counter has reached
// epoch * expect (each producer launch adds `expect` per forward).
struct ArSum {
    const float *src;       // [P][stride] receive buffer slot
    const uint32_t *flag;   // [P] arrival counters of this all-reduce
    const uint64_t *epoch;  // forwards run with the fused all-reduce, this one included
    uint32_t expect, P, stride;
    uint32_t *err;
    uint64_t limit_ns;  // the context's wait limit
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Waits (thread 0, bounded) until every rank's partial rows have arrived.
__device__ __forceinline__ void ar_wait(const ArSum &ar) {
    __shared__ int s_ok;
    if (threadIdx.x == 0) {
        const uint32_t target = (uint32_t)(*ar.epoch * ar.expect);
        const uint64_t t0 = globaltimer_ns();
        bool ok = true;
        for (uint32_t q = 0; q < ar.P && ok; q++) {
            while ((int32_t)(ld_acquire_sys(ar.flag + q) - target) < 0) {
                if (globaltimer_ns() - t0 > ar.limit_ns) {
                    atomicOr(ar.err, (uint32_t)ERR_TIMEOUT_PEER);
                    ok = false;
                    break;
                }
            }
        }
        s_ok = ok;
    }
    __syncthreads();
}

template <int NIT>
__global__ void __launch_bounds__(kNormThreads) k_norm_q(float *__restrict__ x, const float *__restrict__ o,
                                                         const float *__restrict__ post_w, float rs,
                                                         const float *__restrict__ w, uint32_t e, float eps,
                                                         float *__restrict__ xn_f32, const ActOut ao, int x_ready,
                                                         const ArSum ar) {
    __shared__ float red[32];
    __shared__ Q8kShared sh;
    const uint32_t t = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    float *xr = x + (uint64_t)t * e;
    float v[NIT], wv[NIT], pw[NIT];
#pragma unroll
    for (int j = 0; j < NIT; j++) {
        const uint32_t i = tid + kNormThreads * j;
        wv[j] = i < e ? w[i] : 0.0f;
        pw[j] = (post_w && i < e) ? post_w[i] : 0.0f;
        if (x_ready) v[j] = i < e ? xr[i] : 0.0f;
    }
    pdl_wait();
    pdl_trigger();
    if (!x_ready) {
#pragma unroll
        for (int j = 0; j < NIT; j++) {
            const uint32_t i = tid + kNormThreads * j;
            v[j] = i < e ? xr[i] : 0.0f;
        }
    }
    if (o || ar.P) {
        float ov[NIT];
        if (ar.P) {
            ar_wait(ar);
#pragma unroll
            for (int j = 0; j < NIT; j++) ov[j] = 0.0f;
            for (uint32_t q = 0; q < ar.P; q++) {
                const float *src = ar.src + (uint64_t)q * ar.stride + (uint64_t)t * e;
#pragma unroll
                for (int j = 0; j < NIT; j++) {
                    const uint32_t i = tid + kNormThreads * j;
                    if (i < e) ov[j] += __ldcg(src + i);
                }
            }
        } else {
            const float *orow = o + (uint64_t)t * e;
#pragma unroll
            for (int j = 0; j < NIT; j++) {
                const uint32_t i = tid + kNormThreads * j;
                ov[j] = i < e ? orow[i] : 0.0f;
            }
        }
        if (post_w) {
            float ss = 0.0f;
#pragma unroll
            for (int j = 0; j < NIT; j++) ss += ov[j] * ov[j];
            ss = block_sum(ss, red);
            const float scale = 1.0f / sqrtf(ss / (float)e + eps);
#pragma unroll
            for (int j = 0; j < NIT; j++) ov[j] *= scale * pw[j];
        }
#pragma unroll
        for (int j = 0; j < NIT; j++) {
            const uint32_t i = tid + kNormThreads * j;
            v[j] += rs == 1.0f ? ov[j] : ov[j] * rs;
            if (i < e) xr[i] = v[j];
        }
    }
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < NIT; j++) ss += v[j] * v[j];
    ss = block_sum(ss, red);
    const float scale = 1.0f / sqrtf(ss / (float)e + eps);
#pragma unroll
    for (int j = 0; j < NIT; j++) {
        const uint32_t i = tid + kNormThreads * j;
        const float xn = i < e ? v[j] * scale * wv[j] : 0.0f;
        if (xn_f32 && i < e) xn_f32[(uint64_t)t * e + i] = xn;
        const uint32_t i0 = kNormThreads * j + 32 * warp;  // first value of this warp's block
        if ((ao.fmt & RCU_ACT_Q8_0) && i0 < e) q8_0_block(xn, (uint64_t)t * (e / QK) + i0 / QK, lane, ao);
        if (ao.fmt & RCU_ACT_Q8K) {
            const uint32_t g0 = kNormThreads * j + QK_K * (warp / 8);
            q8_k_block(xn, tid % QK_K, warp & ~7u, (uint64_t)t * (e / QK_K) + g0 / QK_K, g0 < e, ao, sh, j & 1);
        }
    }
}

// k_norm_q with 8 consecutive values per thread (e / 8 threads, whole warps): a warp spans one
// Q8_K block (or eight Q8_0 blocks), so only the two RMS sums need CTA barriers. Same
// arithmetic as k_norm_q; rows of whole 256-value blocks, at most 8192 values.
__device__ __forceinline__ void ld8(const float *p, float (&v)[8]) {
    const float4 a = reinterpret_cast<const float4 *>(p)[0], b = reinterpret_cast<const float4 *>(p)[1];
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
}
__device__ __forceinline__ void st8(float *p, const float (&v)[8]) {
    reinterpret_cast<float4 *>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4 *>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}
__global__ void __launch_bounds__(1024) k_norm_q8(float *__restrict__ x, const float *__restrict__ o,
                                                  const float *__restrict__ post_w, float rs,
                                                  const float *__restrict__ w, uint32_t e, float eps,
                                                  float *__restrict__ xn_f32, const ActOut ao, int x_ready,
                                                  const ArSum ar) {
    __shared__ float red[32];
    const uint32_t t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, i0 = 8 * tid;
    float *xr = x + (uint64_t)t * e + i0;
    float v[8], wv[8], pw[8];
    ld8(w + i0, wv);
    if (post_w) ld8(post_w + i0, pw);
    if (x_ready) ld8(xr, v);
    pdl_wait();
    pdl_trigger();
    if (!x_ready) ld8(xr, v);
    if (o || ar.P) {
        float ov[8];
        if (ar.P) {
            ar_wait(ar);
#pragma unroll
            for (int j = 0; j < 8; j++) ov[j] = 0.0f;
            for (uint32_t q = 0; q < ar.P; q++) {
                const float4 *src = reinterpret_cast<const float4 *>(ar.src + (uint64_t)q * ar.stride + (uint64_t)t * e + i0);
                const float4 a = __ldcg(src), b = __ldcg(src + 1);
                ov[0] += a.x, ov[1] += a.y, ov[2] += a.z, ov[3] += a.w;
                ov[4] += b.x, ov[5] += b.y, ov[6] += b.z, ov[7] += b.w;
            }
        } else {
            ld8(o + (uint64_t)t * e + i0, ov);
        }
        if (post_w) {
            float ss = 0.0f;
#pragma unroll
            for (int j = 0; j < 8; j++) ss += ov[j] * ov[j];
            ss = block_sum(ss, red);
            const float scale = 1.0f / sqrtf(ss / (float)e + eps);
#pragma unroll
            for (int j = 0; j < 8; j++) ov[j] *= scale * pw[j];
        }
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] += rs == 1.0f ? ov[j] : ov[j] * rs;
        st8(xr, v);
    }
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; j++) ss += v[j] * v[j];
    ss = block_sum(ss, red);
    const float scale = 1.0f / sqrtf(ss / (float)e + eps);
    float xn[8];
#pragma unroll
    for (int j = 0; j < 8; j++) xn[j] = v[j] * scale * wv[j];
    if (xn_f32) st8(xn_f32 + (uint64_t)t * e + i0, xn);
    if (ao.fmt & RCU_ACT_Q8_0) q8_0_block8(xn, (uint64_t)t * (e / QK) + i0 / QK, lane, true, ao);
    if (ao.fmt & RCU_ACT_Q8K) q8_k_block8(xn, (uint64_t)t * (e / QK_K) + i0 / QK_K, lane, ao);
}

// g = act(g) * u (SwiGLU / GELU-tanh, ops.rs:41-58) quantized for the down matmul; one
// value per thread, grid (ceil(ff / 1024), tokens).
__global__ void __launch_bounds__(1024) k_glu_q(const float *__restrict__ g, const float *__restrict__ u, uint32_t ff,
                                                int act, const ActOut ao) {
    pdl_wait();
    pdl_trigger();
    __shared__ Q8kShared sh;
    const uint32_t t = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t i = blockIdx.x * 1024 + tid;
    float f = 0.0f;
    if (i < ff) {
        const float a = g[(uint64_t)t * ff + i];
        if (act == 1) {
            f = 0.5f * a * (1.0f + tanhf(0.7978846f * a * (1.0f + 0.044715f * a * a)));
        } else {
            f = a / (1.0f + expf(-a));
        }
        f *= u[(uint64_t)t * ff + i];
    }
    const uint32_t i0 = blockIdx.x * 1024 + 32 * warp;
    if ((ao.fmt & RCU_ACT_Q8_0) && i0 < ff) q8_0_block(f, (uint64_t)t * (ff / QK) + i0 / QK, lane, ao);
    if (ao.fmt & RCU_ACT_Q8K) {
        const uint32_t g0 = blockIdx.x * 1024 + QK_K * (warp / 8);
        q8_k_block(f, tid % QK_K, warp & ~7u, (uint64_t)t * (ff / QK_K) + g0 / QK_K, g0 < ff, ao, sh, 0);
    }
}

// The same with 8 consecutive values per thread (two float4 loads of g and u): a warp spans one
// Q8_K block (or eight Q8_0 blocks), so the quantization needs no CTA barrier. 256 threads cover
// 2048 values; grid (ceil(ff / 2048), tokens). Rows of whole 256-value blocks (Q8_K) or 32-value
// blocks (Q8_0 only).
constexpr int kGlu8Threads = 256;
__global__ void __launch_bounds__(kGlu8Threads) k_glu_q8(const float *__restrict__ g, const float *__restrict__ u,
                                                         uint32_t ff, int act, const ActOut ao) {
    pdl_wait();
    pdl_trigger();
    const uint32_t t = blockIdx.y, lane = threadIdx.x & 31;
    const uint32_t i0 = (blockIdx.x * kGlu8Threads + threadIdx.x) * 8;  // first value of this thread
    const bool in = i0 < ff;
    float f[8];
    if (in) {
        const float4 *gp = reinterpret_cast<const float4 *>(g + (uint64_t)t * ff + i0);
        const float4 *up = reinterpret_cast<const float4 *>(u + (uint64_t)t * ff + i0);
        const float4 g0 = gp[0], g1 = gp[1], u0 = up[0], u1 = up[1];
        const float gv[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
        const float uv[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const float a = gv[i];
            const float y = act == 1 ? 0.5f * a * (1.0f + tanhf(0.7978846f * a * (1.0f + 0.044715f * a * a)))
                                     : a / (1.0f + expf(-a));
            f[i] = y * uv[i];
        }
    } else {
#pragma unroll
        for (int i = 0; i < 8; i++) f[i] = 0.0f;
    }
    if (ao.fmt & RCU_ACT_Q8_0) q8_0_block8(f, (uint64_t)t * (ff / QK) + i0 / QK, lane, in, ao);
    if ((ao.fmt & RCU_ACT_Q8K) && (i0 & ~(QK_K - 1)) < ff) q8_k_block8(f, (uint64_t)t * (ff / QK_K) + i0 / QK_K, lane, ao);
}

// GLU + quantization of `rows` rows of ff values (k_glu_q8 when the row holds whole blocks).
static int launch_glu(rcu_ctx *ctx, const float *g, const float *u, uint32_t ff, uint32_t rows, int act,
                      const ActOut &ao) {
    if (rows == 0) return RCU_OK;
    const bool whole = (ao.fmt & RCU_ACT_Q8K) ? ff % QK_K == 0 : ff % QK == 0;
    if (whole)
        RCU_CUDA_TRY(ctx, launch_k(ctx, (k_glu_q8), dim3((ff + 8 * kGlu8Threads - 1) / (8 * kGlu8Threads), rows),
                                   dim3(kGlu8Threads), 0, g, u, ff, act, ao));
    else
        RCU_CUDA_TRY(ctx, launch_k(ctx, (k_glu_q), dim3((ff + 1023) / 1024, rows), dim3(1024), 0, g, u, ff, act, ao));
    return RCU_OK;
}

// ---- mixture of experts (model/cpu.rs:469-524) ---------------------------------------------
// Router logits l[t][x] = R[x] . xn[t] over the f32 normed rows (F32 router, dot in f32), and
// the shared expert's gate sigmoid(g . xn[t]) as an extra row. One warp per (token, row).
__global__ void k_router(const float *__restrict__ R, const float *__restrict__ gs, const float *__restrict__ xn,
                         uint32_t n, uint32_t ne, uint32_t e, float *__restrict__ logits, float *__restrict__ sgate) {
    pdl_wait();
    pdl_trigger();
    const uint32_t per = ne + (gs ? 1 : 0), lane = threadIdx.x & 31;
    const uint64_t item = (uint64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    if (item >= (uint64_t)n * per) return;
    const uint32_t t = (uint32_t)(item / per), x = (uint32_t)(item % per);
    const float *row = x < ne ? R + (uint64_t)x * e : gs, *v = xn + (uint64_t)t * e;
    float acc = 0.0f;
    for (uint32_t i = lane; i < e; i += 32) acc = fmaf(row[i], v[i], acc);
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) {
        if (x < ne)
            logits[(uint64_t)t * ne + x] = acc;
        else
            sgate[t] = 1.0f / (1.0f + expf(-acc));
    }
}

// Softmax over the router logits, top-k by (probability desc, index asc), weights
// p / sum(top-k p) (norm_topk), p, or 1 (unit weights). The k choices are written in
// increasing expert id, the order in which the reference adds the experts' outputs.
// One warp per token; ne <= 256.
__global__ void k_moe_route(const float *__restrict__ logits, uint32_t n, uint32_t ne, uint32_t k, int norm_topk,
                            int unit, uint32_t e0, uint32_t n_local, uint32_t *__restrict__ sel,
                            float *__restrict__ wsel) {
    pdl_wait();
    pdl_trigger();
    const uint32_t lane = threadIdx.x & 31;
    const uint64_t t = (uint64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    if (t >= n) return;
    const float *l = logits + t * ne;
    float p[8];
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const uint32_t i = lane + 32 * j;
        p[j] = i < ne ? l[i] : -INFINITY;
        mx = fmaxf(mx, p[j]);
    }
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        p[j] = p[j] == -INFINITY ? 0.0f : expf(p[j] - mx);
        sum += p[j];
    }
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float inv = 1.0f / sum;
#pragma unroll
    for (int j = 0; j < 8; j++) p[j] *= inv;
    uint32_t ids[16];
    float ps[16];
    float norm = 0.0f;
    for (uint32_t r = 0; r < k; r++) {
        unsigned long long key = 0;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const uint32_t i = lane + 32 * j;
            if (i < ne && p[j] >= 0.0f) {
                const unsigned long long kk = ((unsigned long long)__float_as_uint(p[j]) << 32) | (0xffffffffu - i);
                key = kk > key ? kk : key;
            }
        }
        for (int o = 16; o; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
            key = other > key ? other : key;
        }
        const uint32_t win = 0xffffffffu - (uint32_t)(key & 0xffffffffu);
        const float pw = __uint_as_float((uint32_t)(key >> 32));
#pragma unroll
        for (int j = 0; j < 8; j++)
            if (lane + 32 * j == win) p[j] = -1.0f;  // taken
        ids[r] = win;
        ps[r] = pw;
        norm += pw;  // in probability order, as the reference sums the sorted top-k
    }
    if (lane == 0) {
        if (!norm_topk) norm = 1.0f;
        // insertion order by expert id
        for (uint32_t r = 0; r < k; r++) {
            uint32_t best = r;
            for (uint32_t q = r + 1; q < k; q++)
                if (ids[q] < ids[best]) best = q;
            const uint32_t ti = ids[r];
            ids[r] = ids[best];
            ids[best] = ti;
            const float tp = ps[r];
            ps[r] = ps[best];
            ps[best] = tp;
            // expert parallelism: this rank holds experts [e0, e0 + n_local), as local ids
            sel[t * k + r] = ids[r] - e0 < n_local ? ids[r] - e0 : kNoExpert;
            wsel[t * k + r] = unit ? 1.0f : ps[r] / norm;
        }
    }
}

// out[t] = sum_j w[t][j] * y[t*k + j] (experts in id order, those of this rank) [+ sgate[t] * ys[t]].
// slot != nullptr: the output of pair t*k + j is row slot[t*k + j] of y (grouped GEMMs).
__global__ void k_moe_combine(const float *__restrict__ y, const float *__restrict__ wsel, const uint32_t *__restrict__ sel,
                              const uint32_t *__restrict__ slot, const float *__restrict__ ys,
                              const float *__restrict__ sgate, uint32_t n, uint32_t k, uint32_t e,
                              float *__restrict__ out) {
    pdl_wait();
    pdl_trigger();
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (uint64_t)n * e) return;
    const uint64_t t = i / e, c = i % e;
    float o = 0.0f;
    for (uint32_t j = 0; j < k; j++)
        if (sel[t * k + j] != kNoExpert) o += wsel[t * k + j] * y[(slot ? slot[t * k + j] : t * k + j) * (uint64_t)e + c];
    if (ys) o += (sgate ? sgate[t] : 1.0f) * ys[t * e + c];
    out[i] = o;
}

// Expert-sorted order of the (token, choice) pairs for the grouped GEMMs (one CTA): counts per
// local expert, their exclusive prefix off[0..n_exp], and for every pair its slot (kNoExpert
// for another rank's expert) and for every slot its token. Slots of one expert are in no fixed
// order; every slot is computed on its own, so the results do not depend on it.
constexpr int kMoePlanThreads = 1024;
constexpr uint64_t kMoeGroupedMinTok = 32;  // tokens per forward from which experts run as grouped GEMMs
__global__ void __launch_bounds__(kMoePlanThreads) k_moe_plan(const uint32_t *__restrict__ sel, uint32_t n_pairs,
                                                              uint32_t k, uint32_t n_exp, uint32_t *__restrict__ off,
                                                              uint32_t *__restrict__ slot, uint32_t *__restrict__ row) {
    pdl_wait();
    pdl_trigger();
    __shared__ uint32_t cnt[256], cur[256];
    const uint32_t tid = threadIdx.x;
    for (uint32_t e = tid; e < n_exp; e += kMoePlanThreads) cnt[e] = 0;
    __syncthreads();
    for (uint32_t q = tid; q < n_pairs; q += kMoePlanThreads)
        if (sel[q] != kNoExpert) atomicAdd(&cnt[sel[q]], 1u);
    __syncthreads();
    if (tid == 0) {
        uint32_t acc = 0;
        for (uint32_t e = 0; e < n_exp; e++) {
            off[e] = acc;
            cur[e] = acc;
            acc += cnt[e];
        }
        off[n_exp] = acc;
    }
    __syncthreads();
    for (uint32_t q = tid; q < n_pairs; q += kMoePlanThreads) {
        const uint32_t e = sel[q];
        if (e == kNoExpert) {
            slot[q] = kNoExpert;
        } else {
            const uint32_t s = atomicAdd(&cur[e], 1u);
            slot[q] = s;
            row[s] = q / k;
        }
    }
}

__global__ void k_set_pos(uint64_t *pos_dev, uint64_t pos, uint64_t *epoch) {
    pdl_wait();
    pdl_trigger();
    *pos_dev = pos;
    if (epoch) *epoch += 1;  // a forward with the fused all-reduce starts
}

__global__ void k_logit_post(float *__restrict__ l, uint64_t n, float scale, float cap) {
    pdl_wait();
    pdl_trigger();
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float v = l[i];
    if (scale != 1.0f) v /= scale;
    if (cap > 0.0f) v = cap * tanhf(v / cap);
    l[i] = v;
}

// ---- host helpers -------------------------------------------------------------------------
static int dalloc(rcu_backend *b, void **p, size_t bytes) {
    RCU_CUDA_TRY(b->ctx, cudaMalloc(p, bytes));
    b->allocs.push_back(*p);
    return RCU_OK;
}

// Activation formats the weights of one matmul_multi call consume.
static uint32_t formats(std::initializer_list<const rcu_weight *> ws) {
    uint32_t f = 0;
    for (auto *w : ws) f |= act_format(w->type);
    return f;
}

static ActOut acts_out(rcu_backend *b, uint32_t fmt) { return act_out(b->acts->v, fmt, b->ctx->rounding); }

// Matmuls over activations that a fused producer kernel already quantized into b->acts.
static int matmul(rcu_backend *b, uint32_t n, uint32_t k, uint32_t fmt, std::vector<rcu_job> jobs) {
    b->acts->v.n_tok = n;
    b->acts->v.k = k;
    b->acts->v.have = fmt;
    return rcu_matmul_multi(b->ctx, b->acts, jobs.data(), jobs.size());
}

// x (+)= post_norm(o) * rs; quantized RMSNorm(x) * w into b->acts (and f32 into xn_f32).
static int norm_q(rcu_backend *b, uint64_t n, float *x, const float *o, const float *post_w, const float *w,
                  float *xn_f32, uint32_t fmt, bool x_ready, const ArSum &ar) {
    const rcu_model_config &c = b->cfg;
    const uint32_t e = c.n_embd, nit = (e + kNormThreads - 1) / kNormThreads;
    const ActOut ao = acts_out(b, fmt);
    const float rs = c.residual_scale, eps = c.rms_eps;
    if (e % QK_K == 0 && e <= 8192) {
        RCU_CUDA_TRY(b->ctx, launch_k(b->ctx, k_norm_q8, dim3((uint32_t)n), dim3(e / 8), 0, x, o, post_w, rs, w, e, eps,
                                      xn_f32, ao, x_ready ? 1 : 0, ar));
        return RCU_OK;
    }
    auto kern = nit <= 1 ? k_norm_q<1> : nit <= 2 ? k_norm_q<2> : nit <= 4 ? k_norm_q<4> : nit <= 8 ? k_norm_q<8> : k_norm_q<16>;
    if (nit > 16) return set_err(b->ctx, RCU_ERR_UNSUPPORTED, "n_embd above 16384");
    RCU_CUDA_TRY(b->ctx, launch_k(b->ctx, kern, dim3((uint32_t)n), dim3(kNormThreads), 0, x, o, post_w, rs, w, e, eps,
                                  xn_f32, ao, x_ready ? 1 : 0, ar));
    return RCU_OK;
}

// One forward of n tokens at the position stored in b->pos_dev (pos0 is its host copy, used
// to size the attention grid unless `fixed_grid`, which sizes it for the whole cache so the
// launch sequence does not depend on the position and can be replayed as a graph).
// Per layer: norm+quantize, QKV matmul, q/k post-processing + KV append, attention with the
// merge quantizing for Wo, Wo, residual+norm+quantize, gate+up, GLU+quantize, down; the
// down residual is folded into the next layer's (or the output) norm.
static int nccl_err(rcu_ctx *ctx, ncclResult_t r, const char *what) {
    return set_err(ctx, RCU_ERR_RUNTIME, std::string(what) + ": " + ncclGetErrorString(r));
}

// [P][rows][cols] (rank-major, as all-gather leaves it) -> [rows][P * cols]
__global__ void k_unshard_cols(const float *__restrict__ src, float *__restrict__ dst, uint32_t P, uint32_t rows,
                               uint32_t cols) {
    pdl_wait();
    pdl_trigger();
    const uint64_t n = (uint64_t)P * rows * cols;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t c = i % cols, r = (i / cols) % rows, p = i / ((uint64_t)cols * rows);
        dst[r * (uint64_t)P * cols + p * cols + c] = src[i];
    }
}

// Mixture-of-experts FFN of one layer (model/cpu.rs:469-524) for n tokens: residual + norm
// (f32 rows for the router and quantized rows for the experts), router logits, softmax /
// top-k on the device, the shared expert, then the chosen experts as GEMVs whose weights
// and activation rows come from the routing (graph-capturable), 8 tokens at a time; the
// weighted sum lands in b->o.
static int moe_ffn(rcu_backend *b, const LayerW &L, uint64_t n, const float *o_attn, const ArSum &ar_o) {
    rcu_ctx *ctx = b->ctx;
    const rcu_model_config &c = b->cfg;
    // expert parallelism: this rank holds experts [e0, e0 + n_local); the shared expert (kept
    // whole on every rank) is added by rank 0 only, and the ranks' sums are all-reduced below
    const int P = b->m->tp_world, rank = b->m->tp_rank;
    const bool shared_here = L.gate_sh && rank == 0;
    const uint32_t e = c.n_embd, ne = (uint32_t)L.router->rows, fx = c.n_ff_exp;
    const uint32_t k = std::min<uint32_t>(std::max<uint32_t>(c.n_expert_used, 1), ne);
    const uint32_t fx_in = formats({L.gate_exps, L.up_exps}) | (L.gate_sh ? formats({L.gate_sh, L.up_sh}) : 0);
    if (int st = norm_q(b, n, b->x, o_attn, L.post_attn, L.ffn_norm, b->xn, fx_in, true, ar_o)) return st;
    const uint32_t per = ne + (L.sh_gate ? 1 : 0);
    RCU_CUDA_TRY(ctx, launch_k(ctx, (k_router), dim3((uint32_t)((n * per + 7) / 8)), dim3(256), 0,
                               (const float *)L.router->data, L.sh_gate, (const float *)b->xn, (uint32_t)n, ne, e,
                               b->moe_logits, b->moe_sgate));
    RCU_CUDA_TRY(ctx, launch_k(ctx, (k_moe_route), dim3((uint32_t)((n + 7) / 8)), dim3(256), 0,
                               (const float *)b->moe_logits, (uint32_t)n, ne, k, c.expert_norm_topk,
                               c.expert_unit_weights, b->ep_e0, b->ep_n, b->moe_sel, b->moe_w));
    auto view = [&](rcu_acts *a, uint32_t rows, uint32_t kk, uint32_t fmt) {
        ActsView v = a->v;
        v.n_tok = rows;
        v.k = kk;
        v.have = fmt;
        return v;
    };
    // Batches of kMoeGroupedMinTok tokens or more: the (token, choice) pairs sorted by expert
    // (k_moe_plan), then one grouped tensor-core GEMM per stacked expert tensor, which reads
    // every expert's weights once; the host needs the expert offsets to size those launches.
    const uint32_t n_loc = std::min<uint32_t>(ne, b->ep_n);
    const uint32_t fg = act_format(L.gate_exps->type), fdn = formats({L.down_exps});
    const bool grouped = n >= kMoeGroupedMinTok && b->moe_slot && L.gate_exps->type == L.up_exps->type &&
                         gemm_f16_grouped_ok(L.gate_exps, e, n_loc, fx) && gemm_f16_grouped_ok(L.up_exps, e, n_loc, fx) &&
                         gemm_f16_grouped_ok(L.down_exps, fx, n_loc, e);
    if (grouped) {
        RCU_CUDA_TRY(ctx, launch_k(ctx, (k_moe_plan), dim3(1), dim3(kMoePlanThreads), 0, (const uint32_t *)b->moe_sel,
                                   (uint32_t)(n * k), k, n_loc, b->moe_off, b->moe_slot, b->moe_row));
        RCU_CUDA_TRY(ctx, cudaMemcpyAsync(b->moe_off_host, b->moe_off, (n_loc + 1) * sizeof(uint32_t),
                                          cudaMemcpyDeviceToHost, ctx->stream));
        RCU_CUDA_TRY(ctx, cudaEventRecord(b->ev_plan, ctx->stream));
    }
    // shared expert first: it reads the norm's activations, its GLU goes to the second batch
    if (shared_here) {
        const uint32_t fs = (uint32_t)L.gate_sh->rows, fsd = formats({L.down_sh});
        if (int st = matmul(b, (uint32_t)n, e, fx_in, {{L.gate_sh, b->g, fs}, {L.up_sh, b->u, fs}})) return st;
        if (int st = launch_glu(ctx, b->g, b->u, fs, (uint32_t)n, c.act, act_out(b->acts2->v, fsd, ctx->rounding)))
            return st;
        b->acts2->v.n_tok = (uint32_t)n;
        b->acts2->v.k = fs;
        b->acts2->v.have = fsd;
        const rcu_job dj{L.down_sh, b->moe_ys, e};
        if (int st = rcu_matmul_multi(ctx, b->acts2, &dj, 1)) return st;
    }
    if (grouped) {
        RCU_CUDA_TRY(ctx, cudaEventSynchronize(b->ev_plan));
        const uint32_t n_slots = b->moe_off_host[n_loc];
        if (n_slots > 0) {
            const __half *act = nullptr;
            const float *sc = nullptr;
            if (int st = gemm_f16_gather(ctx, view(b->acts, (uint32_t)n, e, fg), fg, b->moe_row, n_slots, &act, &sc))
                return st;
            const HostJob gu[2] = {{L.gate_exps, b->moe_g, fx}, {L.up_exps, b->moe_u, fx}};
            if (int st = launch_gemm_f16_grouped(ctx, act, sc, n_slots, e, gu, 2, fx, b->moe_off_host, n_loc)) return st;
            if (int st = launch_glu(ctx, b->moe_g, b->moe_u, fx, n_slots, c.act, act_out(b->acts2->v, fdn, ctx->rounding)))
                return st;
            if (int st = gemm_f16_gather(ctx, view(b->acts2, n_slots, fx, fdn), fdn, nullptr, n_slots, &act, &sc))
                return st;
            const HostJob dj{L.down_exps, b->moe_y, e};
            if (int st = launch_gemm_f16_grouped(ctx, act, sc, n_slots, fx, &dj, 1, e, b->moe_off_host, n_loc)) return st;
        }
    } else {
        const uint64_t rb_g = L.gate_exps->row_bytes, rb_u = L.up_exps->row_bytes, rb_d = L.down_exps->row_bytes;
        for (uint32_t c0 = 0; c0 < n; c0 += 8) {
            const uint32_t nt = std::min<uint32_t>(8, (uint32_t)n - c0);
            std::vector<HostJob> gu, dn;
            for (uint32_t t = 0; t < nt; t++)
                for (uint32_t j = 0; j < k; j++) {
                    const uint32_t idx = (c0 + t) * k + j;
                    HostJob g{L.gate_exps, b->moe_g + (uint64_t)idx * fx, fx};
                    g.sel = b->moe_sel + idx, g.w_stride = (uint64_t)fx * rb_g, g.rows = fx, g.tok = t;
                    HostJob u{L.up_exps, b->moe_u + (uint64_t)idx * fx, fx};
                    u.sel = b->moe_sel + idx, u.w_stride = (uint64_t)fx * rb_u, u.rows = fx, u.tok = t;
                    gu.push_back(g);
                    gu.push_back(u);
                    HostJob d{L.down_exps, b->moe_y + (uint64_t)idx * e, e};
                    d.sel = b->moe_sel + idx, d.w_stride = (uint64_t)e * rb_d, d.rows = e, d.tok = t * k + j;
                    dn.push_back(d);
                }
            for (size_t j0 = 0; j0 < gu.size(); j0 += kGemvMaxJobs)
                if (int st = launch_gemv(ctx, view(b->acts, (uint32_t)n, e, fx_in), gu.data() + j0,
                                         (int)std::min<size_t>(kGemvMaxJobs, gu.size() - j0), c0, 1))
                    return st;
            const uint64_t r0 = (uint64_t)c0 * k;
            if (int st = launch_glu(ctx, b->moe_g + r0 * fx, b->moe_u + r0 * fx, fx, nt * k, c.act,
                                    act_out(b->acts2->v, fdn, ctx->rounding)))
                return st;
            for (size_t j0 = 0; j0 < dn.size(); j0 += kGemvMaxJobs)
                if (int st = launch_gemv(ctx, view(b->acts2, nt * k, fx, fdn), dn.data() + j0,
                                         (int)std::min<size_t>(kGemvMaxJobs, dn.size() - j0), 0, 1))
                    return st;
        }
    }
    const uint64_t tot = n * e;
    RCU_CUDA_TRY(ctx, launch_k(ctx, (k_moe_combine), dim3((uint32_t)((tot + 255) / 256)), dim3(256), 0,
                               (const float *)b->moe_y, (const float *)b->moe_w, (const uint32_t *)b->moe_sel,
                               grouped ? (const uint32_t *)b->moe_slot : (const uint32_t *)nullptr,
                               shared_here ? (const float *)b->moe_ys : (const float *)nullptr,
                               L.sh_gate ? (const float *)b->moe_sgate : (const float *)nullptr, (uint32_t)n, k, e, b->o));
    if (P > 1) {  // the experts of the other ranks
        const ncclResult_t r = ncclAllReduce(b->o, b->o, tot, ncclFloat32, ncclSum, b->comm, ctx->stream);
        if (r != ncclSuccess) return nccl_err(ctx, r, "ncclAllReduce (experts)");
    }
    return RCU_OK;
}

// Layers [l0, l1) of n tokens: from token embeddings (x_in == nullptr) or from hidden rows
// x_in (n x n_embd, device). x_out: the residual stream after layer l1 - 1 (the pending
// residual added first). logits: the head over the last row (or all rows), only with l1 ==
// n_layer.
static int forward_span(rcu_backend *b, uint64_t n, uint64_t pos0, bool all_logits, float *logits, bool fixed_grid,
                        const float *x_in, uint32_t l0, uint32_t l1, float *x_out) {
    rcu_ctx *ctx = b->ctx;
    const rcu_model_config &c = b->cfg;
    const int P = b->m->tp_world;
    // tensor parallel: the row-parallel outputs (Wo, down) are partial sums over this rank's
    // slice of K; all-reduce them before the residual add
    auto all_reduce = [&](float *buf, uint64_t count) -> int {
        if (P == 1) return RCU_OK;
        const ncclResult_t r = ncclAllReduce(buf, buf, count, ncclFloat32, ncclSum, b->comm, ctx->stream);
        return r == ncclSuccess ? RCU_OK : nccl_err(ctx, r, "ncclAllReduce");
    };
    const uint32_t e = c.n_embd, hd = c.head_dim, qd = c.n_head * hd, kvd = c.n_head_kv * hd;
    if (x_in) {
        RCU_CUDA_TRY(ctx, cudaMemcpyAsync(b->x, x_in, n * e * sizeof(float), cudaMemcpyDeviceToDevice, ctx->stream));
    } else {
        RCU_CUDA_TRY(ctx, launch_k(ctx, (k_embed), dim3((uint32_t)n), dim3(128), 0, b->tokens, b->embd->type,
                                   b->embd->data, b->embd->row_bytes, e, c.embd_scale, b->x));
    }
    // [residual +] RMSNorm + quantize (its own kernel), then the matmuls that consume it.
    // x_ready: x was written three or more launches back (the norm kernel may load it early).
    auto norm_matmul = [&](uint64_t rows, uint64_t row0, const float *o, const float *post, const float *w,
                           float *xn_f32, bool x_ready, const ArSum &ar, std::vector<rcu_job> jobs) -> int {
        uint32_t fmt = 0;
        for (auto &j : jobs) fmt |= act_format(j.w->type);
        ArSum a = ar;
        if (a.P) a.src += row0 * e;
        if (int st = norm_q(b, rows, b->x + row0 * e, o ? o + row0 * e : nullptr, post, w, xn_f32, fmt, x_ready, a))
            return st;
        return matmul(b, (uint32_t)rows, e, fmt, jobs);
    };
    // Row-parallel matmul (Wo, down) of all-reduce number j. Fused (NVLink): the GEMV pushes
    // this rank's partial rows into every rank's receive buffer and the next norm sums them;
    // otherwise into b->o followed by an NCCL all-reduce.
    const bool fused = P > 1 && b->ar_ok && n <= 8;
    const int rank = b->m->tp_rank;
    auto row_parallel = [&](const rcu_weight *w, uint32_t k, uint32_t j, ArSum *sum) -> int {
        const uint32_t fmt = formats({w});
        *sum = ArSum{};
        if (!fused) {
            if (int st = matmul(b, (uint32_t)n, k, fmt, {{w, b->o, e}})) return st;
            return all_reduce(b->o, n * e);
        }
        const uint64_t stride = b->max_batch * e, slot = (uint64_t)(j & 1) * P * stride;
        ArPush push{};
        for (int q = 0; q < P; q++) {
            if (q != rank) push.dst[push.n_dst++] = b->ar_peer_buf[q] + slot + rank * stride;
            push.flag[push.n_flag++] = (q == rank ? b->ar_flags : b->ar_peer_flags[q]) + (uint64_t)j * P + rank;
        }
        ActsView a = b->acts->v;
        a.n_tok = (uint32_t)n;
        a.k = k;
        a.have = fmt;
        const HostJob hj{w, b->ar_buf + slot + rank * stride, e};
        if (int st = launch_gemv(ctx, a, &hj, 1, 0, (uint32_t)n, &push)) return st;
        *sum = ArSum{b->ar_buf + slot, b->ar_flags + (uint64_t)j * P, b->ar_epoch, kArUnit, (uint32_t)P,
                     (uint32_t)stride, ctx->dev_err, ctx->wait_limit_ns};
        return RCU_OK;
    };
    const float *pend_o = nullptr, *pend_post = nullptr;  // residual not yet added to x
    ArSum pend_ar{};                                       // (or the ranks' partial rows)
    uint32_t ar_j = 0;
    int st;
    for (uint32_t il = l0; il < l1; il++) {
        const LayerW &L = b->layers[il];
        // x comes from k_embed (or the copy of x_in: the launch just before) in the first layer,
        // else from this layer's previous norm (four launches back)
        if ((st = norm_matmul(n, 0, pend_o, pend_post, L.attn_norm, nullptr, il > l0, pend_ar,
                              {{L.wq, b->q, qd}, {L.wk, b->k, kvd}, {L.wv, b->v, kvd}})))
            return st;
        const bool swa_rope = L.swa && c.rope_base_swa > 0.0f;
        QkvPostParams qp{b->q, b->k, b->v, L.bq, L.bk, L.bv, L.q_norm, L.k_norm,
                         swa_rope ? b->inv_freq_swa : b->inv_freq, b->pos_dev, (uint32_t)n, c.n_head, hd,
                         c.rope_dim, c.rope_neox, c.rms_eps, c.attn_scale};
        // decode steps over the head_dim-128 decode attention fold the post-processing and KV
        // append into it (one launch less per layer)
        const bool fuse_post = ctx->fuse_post && attention_fuses_post(b->kv[il], n, c.n_head);
        if (!fuse_post && (st = launch_qkv_post_store(ctx, b->kv[il], qp))) return st;
        const QkvPostParams *post = fuse_post ? &qp : nullptr;
        const uint64_t window = L.swa ? c.swa_window : 0;
        const uint32_t fo = formats({L.wo});
        const ActOut ao = acts_out(b, fo);
        const uint32_t nsp = fixed_grid ? attention_max_splits(b->kv[il], window) : 0;
        if (b->fused_merge) {
            st = launch_attention(ctx, b->kv[il], b->q, n, c.n_head, pos0, b->pos_dev, window, c.attn_softcap, nullptr,
                                  nsp, b->attn_scratch, &ao, post);
        } else {
            st = launch_attention(ctx, b->kv[il], b->q, n, c.n_head, pos0, b->pos_dev, window, c.attn_softcap, b->att,
                                  nsp, b->attn_scratch, nullptr, post);
            if (!st) st = launch_quantize(ctx, b->acts->v, b->att, (uint32_t)n, qd, fo);
        }
        if (st) return st;
        ArSum ar_o;
        if ((st = row_parallel(L.wo, qd, ar_j++, &ar_o))) return st;
        if (L.router) {
            if ((st = moe_ffn(b, L, n, fused ? nullptr : b->o, ar_o))) return st;
            pend_o = b->o;
            pend_ar = ArSum{};
            pend_post = L.post_ffn;
            continue;
        }
        const uint32_t ff = (uint32_t)L.gate->rows;
        if ((st = norm_matmul(n, 0, fused ? nullptr : b->o, L.post_attn, L.ffn_norm, nullptr, true, ar_o,
                              {{L.gate, b->g, ff}, {L.up, b->u, ff}})))
            return st;
        const uint32_t fd = formats({L.down});
        if ((st = launch_glu(ctx, b->g, b->u, ff, (uint32_t)n, c.act, acts_out(b, fd)))) return st;
        if ((st = row_parallel(L.down, ff, ar_j++, &pend_ar))) return st;
        pend_o = fused ? nullptr : b->o;
        pend_post = L.post_ffn;
    }
    if (x_out) {  // add the pending residual (no quantization), then copy the rows out
        if (pend_o || pend_ar.P)
            if ((st = norm_q(b, n, b->x, pend_o, pend_post, b->out_norm, nullptr, 0, l1 > l0, pend_ar))) return st;
        pend_o = nullptr;
        pend_post = nullptr;
        pend_ar = ArSum{};
        RCU_CUDA_TRY(ctx, cudaMemcpyAsync(x_out, b->x, n * e * sizeof(float), cudaMemcpyDeviceToDevice, ctx->stream));
    }
    if (!logits) return RCU_OK;
    const uint64_t first = all_logits ? 0 : n - 1, m = n - first;
    b->hidden_rows = m;
    // vocab-parallel head: each rank computes its rows of the vocabulary, then all-gather
    float *lg = P == 1 ? logits : b->logits_local;
    if ((st = norm_matmul(m, first, pend_o, pend_post, b->out_norm, b->xn, true, pend_ar, {{b->out, lg, c.n_vocab}})))
        return st;
    const uint64_t vocab = (uint64_t)c.n_vocab * P;
    if (P > 1) {
        float *dst = m == 1 ? logits : b->logits_gather;
        const ncclResult_t r = ncclAllGather(lg, dst, m * c.n_vocab, ncclFloat32, b->comm, ctx->stream);
        if (r != ncclSuccess) return nccl_err(ctx, r, "ncclAllGather");
        if (m > 1)
            RCU_CUDA_TRY(ctx, launch_k(ctx, (k_unshard_cols), dim3(ctx->num_sms * 4), dim3(256), 0, b->logits_gather,
                                       logits, (uint32_t)P, (uint32_t)m, (uint32_t)c.n_vocab));
    }
    if (c.logit_scale != 1.0f || c.final_softcap > 0.0f) {
        const uint64_t nl = m * vocab;
        RCU_CUDA_TRY(ctx, launch_k(ctx, (k_logit_post), dim3((uint32_t)((nl + 255) / 256)), dim3(256), 0, logits, nl,
                                   c.logit_scale, c.final_softcap));
    }
    RCU_CUDA_TRY(ctx, cudaGetLastError());
    return RCU_OK;
}

static int forward_dev(rcu_backend *b, uint64_t n, uint64_t pos0, bool all_logits, float *logits, bool fixed_grid) {
    return forward_span(b, n, pos0, all_logits, logits, fixed_grid, nullptr, 0, b->cfg.n_layer, nullptr);
}

static bool ends_with(const std::string &s, const char *suf) {
    const size_t n = std::strlen(suf);
    return s.size() >= n && s.compare(s.size() - n, n, suf) == 0;
}

// ---- tensor-parallel sharding (host side) ---------------------------------------------------
// Column-parallel (rows split): q/k/v (by head), gate/up, the vocabulary rows of the output
// head, q/k/v biases. Row-parallel (columns split, whole blocks): attn_output, ffn_down.
// Everything else (embeddings, norms) is replicated. With fewer KV heads than ranks each KV
// head is replicated on world / n_head_kv consecutive ranks, whose query heads are all in its
// group (Qwen3-30B-A3B: 4 KV heads at 8 GPUs).
enum TpKind { TP_REPL = 0, TP_ROWS = 1, TP_COLS = 2, TP_QKV = 3, TP_UPGATE = 4, TP_EXPERTS = 5, TP_KV = 6 };

// The KV heads [kv0, kv0 + nkv) that `rank` holds; false when the split is not even.
static bool kv_slice(const rcu_model_config &c, int rank, int world, uint64_t *kv0, uint64_t *nkv) {
    const uint64_t nk = c.n_head_kv, P = (uint64_t)world;
    if (nk == 0 || c.n_head % P) return false;
    if (nk % P == 0) {
        *nkv = nk / P, *kv0 = (uint64_t)rank * (nk / P);
        return true;
    }
    if (P % nk) return false;
    *nkv = 1, *kv0 = (uint64_t)rank / (P / nk);
    return true;
}

static int tp_kind(const std::string &n, const rcu_model_config &c, uint64_t rows) {
    if (n == "output.weight") return TP_ROWS;  // (not "blk.N.attn_output.weight")
    if (ends_with(n, ".attn_output.weight") || ends_with(n, ".ffn_down.weight")) return TP_COLS;
    if (ends_with(n, ".attn_qkv.weight")) return TP_QKV;
    // expert parallelism: stacked expert tensors keep this rank's experts (router and shared
    // expert stay whole)
    if (ends_with(n, ".ffn_gate_exps.weight") || ends_with(n, ".ffn_up_exps.weight") ||
        ends_with(n, ".ffn_down_exps.weight"))
        return TP_EXPERTS;
    if (ends_with(n, ".ffn_up.weight") && rows == 2ull * c.n_ff) return TP_UPGATE;
    for (const char *suf : {".attn_k.weight", ".attn_v.weight", ".attn_k.bias", ".attn_v.bias"})
        if (ends_with(n, suf)) return TP_KV;
    for (const char *suf : {".attn_q.weight", ".ffn_gate.weight", ".ffn_up.weight", ".attn_q.bias"})
        if (ends_with(n, suf)) return TP_ROWS;
    return TP_REPL;
}

// Shard of one tensor for `rank` of `world`. 1-D tensors (rows == 1) split their elements.
// out == nullptr only reports the shape; otherwise out holds out_cap bytes.
static int tp_shard(rcu_ctx *ctx, const rcu_model_config &c, const std::string &name, uint32_t type, uint64_t rows,
                    uint64_t cols, const uint8_t *host, int rank, int world, std::vector<uint8_t> *out, uint64_t *out_rows,
                    uint64_t *out_cols) {
    const int kind = world > 1 ? tp_kind(name, c, rows) : TP_REPL;
    const bool vec1d = rows == 1 && (type == T_F32 || type == T_F16 || type == T_BF16) && (kind == TP_ROWS || kind == TP_KV);
    const uint64_t rb = vec1d ? (type == T_F32 ? 4 : 2) * cols : rcu_row_bytes(type, cols);
    if (!vec1d && rb == 0) return set_err(ctx, RCU_ERR_INVALID, "tensor " + name + ": bad row length");
    auto bad = [&](const char *why) { return set_err(ctx, RCU_ERR_INVALID, "tensor parallel: " + name + " " + why); };
    auto copy_rows = [&](uint64_t r0, uint64_t nr, uint64_t at) {
        if (out) std::memcpy(out->data() + at * rb, host + r0 * rb, nr * rb);
    };
    switch (kind) {
        case TP_REPL:
            *out_rows = rows, *out_cols = cols;
            if (out) out->assign(host, host + rows * rb);
            return RCU_OK;
        case TP_ROWS: {
            if (vec1d) {  // bias vector: split elements
                if (cols % world) return bad("length not divisible by the tensor-parallel degree");
                const uint64_t es = rb / cols, n = cols / world;
                *out_rows = 1, *out_cols = n;
                if (out) out->assign(host + rank * n * es, host + (rank + 1) * n * es);
                return RCU_OK;
            }
            uint64_t total = rows;
            if (name == "output.weight") total = c.n_vocab;  // padded vocab rows are dropped
            if (total % world) return bad("rows not divisible by the tensor-parallel degree");
            const uint64_t n = total / world;
            *out_rows = n, *out_cols = cols;
            if (out) out->resize(n * rb);
            copy_rows(rank * n, n, 0);
            return RCU_OK;
        }
        case TP_KV: {  // k / v rows (or bias elements) of this rank's KV heads
            uint64_t kv0 = 0, nkv = 0;
            const uint64_t kvd = (uint64_t)c.n_head_kv * c.head_dim, len = vec1d ? cols : rows;
            if (!kv_slice(c, rank, world, &kv0, &nkv) || len != kvd) return bad("KV heads do not split over the ranks");
            const uint64_t r0 = kv0 * c.head_dim, n = nkv * c.head_dim;
            if (vec1d) {
                const uint64_t es = rb / cols;
                *out_rows = 1, *out_cols = n;
                if (out) out->assign(host + r0 * es, host + (r0 + n) * es);
                return RCU_OK;
            }
            *out_rows = n, *out_cols = cols;
            if (out) out->resize(n * rb);
            copy_rows(r0, n, 0);
            return RCU_OK;
        }
        case TP_EXPERTS: {
            const uint64_t ne = c.n_expert;
            if (ne == 0 || rows % ne || ne % world) return bad("experts do not split evenly");
            const uint64_t per = rows / ne, n = ne / world * per;
            *out_rows = n, *out_cols = cols;
            if (out) out->resize(n * rb);
            copy_rows(rank * n, n, 0);
            return RCU_OK;
        }
        case TP_QKV: {
            const uint64_t qd = (uint64_t)c.n_head * c.head_dim, kvd = (uint64_t)c.n_head_kv * c.head_dim;
            uint64_t kv0 = 0, nkv = 0;
            if (rows != qd + 2 * kvd || qd % world || !kv_slice(c, rank, world, &kv0, &nkv))
                return bad("q/k/v rows do not split evenly");
            const uint64_t nq = qd / world, nk = nkv * c.head_dim, k0 = kv0 * c.head_dim;
            *out_rows = nq + 2 * nk, *out_cols = cols;
            if (out) out->resize((nq + 2 * nk) * rb);
            copy_rows(rank * nq, nq, 0);
            copy_rows(qd + k0, nk, nq);
            copy_rows(qd + kvd + k0, nk, nq + nk);
            return RCU_OK;
        }
        case TP_UPGATE: {
            if (c.n_ff % world) return bad("FFN rows not divisible by the tensor-parallel degree");
            const uint64_t nf = c.n_ff / world;
            *out_rows = 2 * nf, *out_cols = cols;
            if (out) out->resize(2 * nf * rb);
            copy_rows(rank * nf, nf, 0);
            copy_rows(c.n_ff + rank * nf, nf, nf);
            return RCU_OK;
        }
        default: {  // TP_COLS: each row keeps its rank's run of whole blocks
            const uint64_t bs = block_size(type);
            if (cols % world || (cols / world) % bs) return bad("columns do not split into whole blocks");
            const uint64_t nc = cols / world, srb = rcu_row_bytes(type, nc);
            *out_rows = rows, *out_cols = nc;
            if (out) {
                out->resize(rows * srb);
                for (uint64_t r = 0; r < rows; r++) std::memcpy(out->data() + r * srb, host + r * rb + rank * srb, srb);
            }
            return RCU_OK;
        }
    }
}


// Receive buffer, arrival counters and forward count for the fused all-reduce, exported to
// the other ranks with CUDA IPC (handles exchanged through the communicator). If peer
// mappings are not available the backend keeps using NCCL (ar_ok stays false).
static int setup_fused_all_reduce(rcu_backend *b) {
    rcu_ctx *ctx = b->ctx;
    const int P = b->m->tp_world, rank = b->m->tp_rank;
    // Opt-in (RIE_TP_FUSED=1): at 2 GPUs on the 8B shape it measured no faster than NCCL,
    // because its one-float remote stores are scattered (see the GEMV push).
    const char *v = std::getenv("RIE_TP_FUSED");
    if (P > 8 || !v || std::strcmp(v, "1") != 0) return RCU_OK;
    const uint64_t stride = b->max_batch * b->cfg.n_embd;
    const uint64_t nflag = std::max<uint64_t>(2ull * b->cfg.n_layer * P, 64);
    RCU_CUDA_TRY(ctx, cudaMalloc(&b->ar_buf, 2 * P * stride * sizeof(float)));
    RCU_CUDA_TRY(ctx, cudaMemset(b->ar_buf, 0, 2 * P * stride * sizeof(float)));
    RCU_CUDA_TRY(ctx, cudaMalloc(&b->ar_flags, nflag * sizeof(uint32_t)));
    RCU_CUDA_TRY(ctx, cudaMemset(b->ar_flags, 0, nflag * sizeof(uint32_t)));
    if (int st = dalloc(b, (void **)&b->ar_epoch, sizeof(uint64_t))) return st;
    RCU_CUDA_TRY(ctx, cudaMemset(b->ar_epoch, 0, sizeof(uint64_t)));
    cudaIpcMemHandle_t mine[2];
    RCU_CUDA_TRY(ctx, cudaIpcGetMemHandle(&mine[0], b->ar_buf));
    RCU_CUDA_TRY(ctx, cudaIpcGetMemHandle(&mine[1], b->ar_flags));
    uint8_t *dh = nullptr;
    const size_t hb = sizeof(mine);
    if (int st = dalloc(b, (void **)&dh, P * hb)) return st;
    RCU_CUDA_TRY(ctx, cudaMemcpy(dh + rank * hb, mine, hb, cudaMemcpyHostToDevice));
    const ncclResult_t r = ncclAllGather(dh + rank * hb, dh, hb, ncclUint8, b->comm, b->stream);
    if (r != ncclSuccess) return nccl_err(ctx, r, "ncclAllGather(ipc handles)");
    RCU_CUDA_TRY(ctx, cudaStreamSynchronize(b->stream));
    std::vector<cudaIpcMemHandle_t> all(2 * P);
    RCU_CUDA_TRY(ctx, cudaMemcpy(all.data(), dh, P * hb, cudaMemcpyDeviceToHost));
    bool mapped = true;
    for (int q = 0; q < P && mapped; q++) {
        if (q == rank) {
            b->ar_peer_buf[q] = b->ar_buf;
            b->ar_peer_flags[q] = b->ar_flags;
            continue;
        }
        void *pb = nullptr, *pf = nullptr;
        cudaError_t e1 = cudaIpcOpenMemHandle(&pb, all[2 * q], cudaIpcMemLazyEnablePeerAccess);
        cudaError_t e2 = e1 == cudaSuccess ? cudaIpcOpenMemHandle(&pf, all[2 * q + 1], cudaIpcMemLazyEnablePeerAccess) : e1;
        if (e1 != cudaSuccess || e2 != cudaSuccess) {
            cudaGetLastError();
            if (pb) cudaIpcCloseMemHandle(pb);
            mapped = false;
            break;
        }
        b->ar_peer_buf[q] = (float *)pb;
        b->ar_peer_flags[q] = (uint32_t *)pf;
    }
    if (!mapped) {  // no peer mapping here: this backend keeps NCCL (and so do the others)
        for (int q = 0; q < P; q++)
            if (q != rank && b->ar_peer_buf[q]) {
                cudaIpcCloseMemHandle(b->ar_peer_buf[q]);
                cudaIpcCloseMemHandle(b->ar_peer_flags[q]);
            }
        std::fill(b->ar_peer_buf, b->ar_peer_buf + 8, nullptr);
        std::fill(b->ar_peer_flags, b->ar_peer_flags + 8, nullptr);
    }
    // every rank must agree: a rank without mappings would skip the pushes the others wait for
    int ok_here = mapped ? 1 : 0, *dok = nullptr;
    if (int st = dalloc(b, (void **)&dok, sizeof(int))) return st;
    RCU_CUDA_TRY(ctx, cudaMemcpy(dok, &ok_here, sizeof(int), cudaMemcpyHostToDevice));
    const ncclResult_t r2 = ncclAllReduce(dok, dok, 1, ncclInt32, ncclMin, b->comm, b->stream);
    if (r2 != ncclSuccess) return nccl_err(ctx, r2, "ncclAllReduce(fused all-reduce agreement)");
    RCU_CUDA_TRY(ctx, cudaStreamSynchronize(b->stream));
    int ok_all = 0;
    RCU_CUDA_TRY(ctx, cudaMemcpy(&ok_all, dok, sizeof(int), cudaMemcpyDeviceToHost));
    b->ar_ok = ok_all == 1;
    return RCU_OK;
}

}  // namespace rcu

using namespace rcu;

extern "C" {

int32_t rcu_model_create(rcu_ctx *ctx, const rcu_model_config *cfg, rcu_model **out) {
    return rcu_model_create_tp(ctx, cfg, 0, 1, out);
}

int32_t rcu_model_create_tp(rcu_ctx *ctx, const rcu_model_config *cfg, int32_t rank, int32_t world, rcu_model **out) {
    if (world < 1 || rank < 0 || rank >= world) return set_err(ctx, RCU_ERR_INVALID, "bad tensor-parallel rank/world");
    if (!ctx || !cfg || !out) return set_err(ctx, RCU_ERR_INVALID, "null argument");
    *out = nullptr;
    const rcu_model_config &c = *cfg;
    if (!c.n_vocab || !c.n_embd || !c.n_layer || !c.n_head || !c.n_head_kv || !c.head_dim)
        return set_err(ctx, RCU_ERR_INVALID, "model config: zero dimension");
    if (c.n_head % c.n_head_kv) return set_err(ctx, RCU_ERR_INVALID, "n_head not divisible by n_head_kv");
    if (c.rope_dim > c.head_dim || c.rope_dim % 2) return set_err(ctx, RCU_ERR_INVALID, "invalid rope dimension");
    if (c.head_dim > 256 || c.head_dim % 32) return set_err(ctx, RCU_ERR_UNSUPPORTED, "head_dim must be a multiple of 32, <= 256");
    rcu_model *m = new (std::nothrow) rcu_model();
    if (!m) return RCU_ERR_OOM;
    m->ctx = ctx;
    m->cfg = c;
    m->tp_rank = rank;
    m->tp_world = world;
    *out = m;
    return RCU_OK;
}

int32_t rcu_tp_shard(const rcu_model_config *cfg, const char *name, uint32_t ggml_type, uint64_t rows, uint64_t cols,
                     const void *host_bytes, int32_t rank, int32_t world, void *out, uint64_t out_cap,
                     uint64_t *out_rows, uint64_t *out_cols) {
    if (!cfg || !name || !out_rows || !out_cols || (out && !host_bytes)) return RCU_ERR_INVALID;
    if (world < 1 || rank < 0 || rank >= world) return RCU_ERR_INVALID;
    rcu_ctx scratch_ctx;  // error text only
    std::vector<uint8_t> buf;
    const int st = tp_shard(&scratch_ctx, *cfg, name, ggml_type, rows, cols, (const uint8_t *)host_bytes, rank, world,
                            out ? &buf : nullptr, out_rows, out_cols);
    if (st || !out) return st;
    if (buf.size() > out_cap) return RCU_ERR_INVALID;
    std::memcpy(out, buf.data(), buf.size());
    return RCU_OK;
}

void rcu_model_free(rcu_model *m) {
    if (!m) return;
    for (auto &kv : m->w) rcu_weight_free(kv.second);
    for (auto *s : m->slices) rcu_weight_free(s);
    cudaSetDevice(m->ctx->device);
    for (auto &kv : m->vec) cudaFree(kv.second);
    delete m;
}

// rcu_model_set_tensor from device bytes: this rank's shard is cut with device-to-device copies
// (whole row ranges, or each row's run of blocks for the row-parallel matrices); 1-D vectors
// and float matrices take the host path.
int32_t rcu_model_set_tensor_device(rcu_model *m, const char *name, uint32_t ggml_type, uint64_t rows, uint64_t cols,
                                    const void *dev_bytes) {
    if (!m || !name || !dev_bytes) return RCU_ERR_INVALID;
    rcu_ctx *ctx = m->ctx;
    const std::string n(name);
    if (rows == 1 || ggml_type == T_F32 || ggml_type == T_F16 || ggml_type == T_BF16) {
        const uint64_t bytes = ggml_type == T_F32 ? 4 * rows * cols
                               : (ggml_type == T_F16 || ggml_type == T_BF16) ? 2 * rows * cols
                                                                             : rows * rcu_row_bytes(ggml_type, cols);
        std::vector<uint8_t> h(bytes);
        RCU_CUDA_TRY(ctx, cudaMemcpy(h.data(), dev_bytes, bytes, cudaMemcpyDeviceToHost));
        return rcu_model_set_tensor(m, name, ggml_type, rows, cols, h.data());
    }
    const uint64_t rb = rcu_row_bytes(ggml_type, cols);
    if (rb == 0) return set_err(ctx, RCU_ERR_INVALID, "tensor " + n + ": bad row length");
    uint64_t r2 = rows, c2 = cols;
    const int kind = m->tp_world > 1 ? tp_kind(n, m->cfg, rows) : TP_REPL;
    if (kind != TP_REPL)
        if (int st = tp_shard(ctx, m->cfg, n, ggml_type, rows, cols, nullptr, m->tp_rank, m->tp_world, nullptr, &r2, &c2))
            return st;
    const uint64_t srb = rcu_row_bytes(ggml_type, c2);
    uint8_t *d = nullptr;
    RCU_CUDA_TRY(ctx, cudaMalloc(&d, r2 * srb + 256));
    RCU_CUDA_TRY(ctx, cudaMemset(d + r2 * srb, 0, 256));
    const uint8_t *src = (const uint8_t *)dev_bytes;
    auto rows_at = [&](uint64_t r0, uint64_t nr, uint64_t at) -> cudaError_t {
        return cudaMemcpy(d + at * srb, src + r0 * rb, nr * rb, cudaMemcpyDeviceToDevice);
    };
    cudaError_t e = cudaSuccess;
    const int P = m->tp_world, rank = m->tp_rank;
    const rcu_model_config &c = m->cfg;
    switch (kind) {
        case TP_REPL: e = rows_at(0, rows, 0); break;
        case TP_ROWS:
        case TP_EXPERTS: e = rows_at((uint64_t)rank * r2, r2, 0); break;
        case TP_KV: {  // r2 rows of this rank's KV heads (tp_shard checked the split)
            uint64_t kv0 = 0, nkv = 0;
            kv_slice(c, rank, P, &kv0, &nkv);
            e = rows_at(kv0 * c.head_dim, r2, 0);
            break;
        }
        case TP_QKV: {
            const uint64_t qd = (uint64_t)c.n_head * c.head_dim, kvd = (uint64_t)c.n_head_kv * c.head_dim;
            uint64_t kv0 = 0, nkv = 0;
            kv_slice(c, rank, P, &kv0, &nkv);
            const uint64_t nq = qd / P, nk = nkv * c.head_dim, k0 = kv0 * c.head_dim;
            e = rows_at(rank * nq, nq, 0);
            if (e == cudaSuccess) e = rows_at(qd + k0, nk, nq);
            if (e == cudaSuccess) e = rows_at(qd + kvd + k0, nk, nq + nk);
            break;
        }
        case TP_UPGATE: {
            const uint64_t nf = c.n_ff / P;
            e = rows_at(rank * nf, nf, 0);
            if (e == cudaSuccess) e = rows_at(c.n_ff + rank * nf, nf, nf);
            break;
        }
        default:  // TP_COLS: each row keeps its rank's run of blocks
            e = cudaMemcpy2D(d, srb, src + rank * srb, rb, srb, rows, cudaMemcpyDeviceToDevice);
            break;
    }
    if (e != cudaSuccess) {
        cudaFree(d);
        return cuda_err(ctx, e, "set_tensor_device copy");
    }
    rcu_weight *w = new rcu_weight();
    w->ctx = ctx, w->type = (int)ggml_type, w->rows = r2, w->cols = c2, w->row_bytes = srb, w->data = d;
    w->owned = true, w->padded = true;
    auto it = m->w.find(n);
    if (it != m->w.end()) rcu_weight_free(it->second);
    m->w[n] = w;
    return RCU_OK;
}

int32_t rcu_model_set_tensor(rcu_model *m, const char *name, uint32_t ggml_type, uint64_t rows, uint64_t cols,
                             const void *host_bytes) {
    if (!m || !name || !host_bytes) return RCU_ERR_INVALID;
    rcu_ctx *ctx = m->ctx;
    const std::string n(name);
    std::vector<uint8_t> shard;  // this rank's part of a tensor-parallel tensor
    if (m->tp_world > 1 && tp_kind(n, m->cfg, rows) != TP_REPL) {
        uint64_t r2 = 0, c2 = 0;
        if (int st = tp_shard(ctx, m->cfg, n, ggml_type, rows, cols, (const uint8_t *)host_bytes, m->tp_rank,
                              m->tp_world, &shard, &r2, &c2))
            return st;
        rows = r2, cols = c2, host_bytes = shard.data();
    }
    if (rows == 1 && (ggml_type == T_F32 || ggml_type == T_F16 || ggml_type == T_BF16)) {
        std::vector<float> v(cols);
        for (uint64_t i = 0; i < cols; i++) {
            if (ggml_type == T_F32) {
                std::memcpy(&v[i], (const uint8_t *)host_bytes + 4 * i, 4);
            } else {
                uint16_t h;
                std::memcpy(&h, (const uint8_t *)host_bytes + 2 * i, 2);
                if (ggml_type == T_BF16) {
                    uint32_t u = (uint32_t)h << 16;
                    std::memcpy(&v[i], &u, 4);
                } else {
                    v[i] = __half2float(__ushort_as_half(h));
                }
            }
        }
        float *d = nullptr;
        RCU_CUDA_TRY(ctx, cudaMalloc(&d, cols * 4));
        RCU_CUDA_TRY(ctx, cudaMemcpy(d, v.data(), cols * 4, cudaMemcpyHostToDevice));
        auto it = m->vec.find(n);
        if (it != m->vec.end()) cudaFree(it->second);
        m->vec[n] = d;
        return RCU_OK;
    }
    rcu_weight *w = nullptr;
    if (ggml_type == T_F32 || ggml_type == T_F16) {  // float matrices (embeddings only on this path)
        const uint64_t rb = cols * (ggml_type == T_F32 ? 4 : 2);
        uint8_t *d = nullptr;
        RCU_CUDA_TRY(ctx, cudaMalloc(&d, rows * rb + 256));
        RCU_CUDA_TRY(ctx, cudaMemcpy(d, host_bytes, rows * rb, cudaMemcpyHostToDevice));
        w = new rcu_weight();
        w->ctx = ctx, w->type = (int)ggml_type, w->rows = rows, w->cols = cols, w->row_bytes = rb, w->data = d;
        w->owned = true, w->padded = true;
    } else {
        const int32_t st = rcu_weight_upload(ctx, ggml_type, rows, cols, host_bytes, &w);
        if (st) return st;
    }
    auto it = m->w.find(n);
    if (it != m->w.end()) rcu_weight_free(it->second);
    m->w[n] = w;
    return RCU_OK;
}

int32_t rcu_backend_create(rcu_model *m, uint64_t n_ctx, uint64_t max_batch, int32_t kv_type, rcu_backend **out) {
    return rcu_backend_create_tp(m, n_ctx, max_batch, kv_type, nullptr, out);
}

int32_t rcu_tp_unique_id(uint8_t *out, uint64_t cap) {
    if (!out || cap < sizeof(ncclUniqueId)) return RCU_ERR_INVALID;
    ncclUniqueId id;
    if (ncclGetUniqueId(&id) != ncclSuccess) return RCU_ERR_RUNTIME;
    std::memcpy(out, &id, sizeof(id));
    return RCU_OK;
}

int32_t rcu_backend_create_tp(rcu_model *m, uint64_t n_ctx, uint64_t max_batch, int32_t kv_type, const uint8_t *uid,
                              rcu_backend **out) {
    if (!m || !out) return RCU_ERR_INVALID;
    *out = nullptr;
    rcu_ctx *ctx = m->ctx;
    const int P = m->tp_world;
    if (P > 1 && !uid) return set_err(ctx, RCU_ERR_INVALID, "tensor-parallel backend needs the communicator id");
    if (n_ctx == 0) return set_err(ctx, RCU_ERR_INVALID, "n_ctx must be positive");
    if (kv_type < RCU_KV_F16 || kv_type > RCU_KV_TURBO4) return set_err(ctx, RCU_ERR_INVALID, "unknown kv type");
    uint64_t kv0 = 0, n_kv_loc = 0;
    if (!kv_slice(m->cfg, m->tp_rank, P, &kv0, &n_kv_loc) || m->cfg.n_ff % P || m->cfg.n_vocab % P ||
        m->cfg.n_expert % P)
        return set_err(ctx, RCU_ERR_INVALID,
                       "heads, FFN rows, vocabulary and experts must divide by the tensor-parallel degree, and KV "
                       "heads must divide by it or divide it");
    rcu_backend *b = new (std::nothrow) rcu_backend();
    if (!b) return RCU_ERR_OOM;
    b->cfg = m->cfg;
    b->cfg.n_head /= P;
    b->cfg.n_head_kv = (uint32_t)n_kv_loc;
    b->cfg.n_ff /= P;
    b->cfg.n_vocab /= P;
    if (m->cfg.n_expert > 0) {  // expert parallelism
        b->ep_n = m->cfg.n_expert / P;
        b->ep_e0 = (uint32_t)m->tp_rank * b->ep_n;
    }
    const rcu_model_config &c = b->cfg;
    b->m = m;
    b->ctx = ctx;
    b->n_ctx = n_ctx;
    b->max_batch = std::max<uint64_t>(1, std::min<uint64_t>(max_batch, n_ctx));  // cpu.rs:102
    b->kv_type = kv_type;
    auto fail = [&](int st) {
        rcu_backend_free(b);
        return st;
    };
    auto W = [&](const std::string &n) -> const rcu_weight * {
        auto it = m->w.find(n);
        return it == m->w.end() ? nullptr : it->second;
    };
    auto V = [&](const std::string &n) -> const float * {
        auto it = m->vec.find(n);
        return it == m->vec.end() ? nullptr : it->second;
    };
    auto need = [&](bool ok, const std::string &what) { return ok ? RCU_OK : set_err(ctx, RCU_ERR_INVALID, "missing or bad tensor " + what); };
    const uint32_t e = c.n_embd, qd = c.n_head * c.head_dim, kvd = c.n_head_kv * c.head_dim;
    b->embd = W("token_embd.weight");
    if (int st = need(b->embd && b->embd->cols == e, "token_embd.weight")) return fail(st);
    b->out = W("output.weight");
    if (!b->out) {  // tied head: this rank's vocabulary rows of the embedding
        if (P > 1) {
            rcu_weight *s = nullptr;
            if (int st = rcu_weight_slice_rows(b->embd, (uint64_t)m->tp_rank * c.n_vocab, c.n_vocab, &s)) return fail(st);
            m->slices.push_back(s);
            b->out = s;
        } else {
            b->out = b->embd;
        }
    }
    if (int st = need(b->out->cols == e && b->out->rows >= c.n_vocab && gemv_supported(b->out->type), "output.weight"))
        return fail(st);
    if (b->out->rows > c.n_vocab) {
        rcu_weight *s = nullptr;
        if (int st = rcu_weight_slice_rows(b->out, 0, c.n_vocab, &s)) return fail(st);
        m->slices.push_back(s);
        b->out = s;
    }
    b->out_norm = V("output_norm.weight");
    if (int st = need(b->out_norm != nullptr, "output_norm.weight")) return fail(st);
    for (uint32_t il = 0; il < c.n_layer; il++) {
        const std::string p = "blk." + std::to_string(il) + ".";
        LayerW L;
        if (const rcu_weight *qkv = W(p + "attn_qkv.weight")) {
            if (int st = need(qkv->rows == (uint64_t)qd + 2 * kvd, p + "attn_qkv.weight")) return fail(st);
            rcu_weight *a = nullptr, *bb = nullptr, *cc = nullptr;
            if (int st = rcu_weight_slice_rows(qkv, 0, qd, &a)) return fail(st);
            m->slices.push_back(a);
            if (int st = rcu_weight_slice_rows(qkv, qd, kvd, &bb)) return fail(st);
            m->slices.push_back(bb);
            if (int st = rcu_weight_slice_rows(qkv, qd + kvd, kvd, &cc)) return fail(st);
            m->slices.push_back(cc);
            L.wq = a, L.wk = bb, L.wv = cc;
        } else {
            L.wq = W(p + "attn_q.weight"), L.wk = W(p + "attn_k.weight"), L.wv = W(p + "attn_v.weight");
        }
        L.wo = W(p + "attn_output.weight");
        L.router = W(p + "ffn_gate_inp.weight");
        L.gate = W(p + "ffn_gate.weight");
        L.up = W(p + "ffn_up.weight");
        L.down = W(p + "ffn_down.weight");
        if (!L.router && !L.gate && L.up && L.up->rows == 2ull * c.n_ff) {
            rcu_weight *g = nullptr, *u = nullptr;
            if (int st = rcu_weight_slice_rows(L.up, 0, c.n_ff, &g)) return fail(st);
            m->slices.push_back(g);
            if (int st = rcu_weight_slice_rows(L.up, c.n_ff, c.n_ff, &u)) return fail(st);
            m->slices.push_back(u);
            L.gate = g, L.up = u;
        }
        if (L.router) {  // mixture of experts (model/mod.rs:147-180)
            const uint64_t ne = c.n_expert, fx = c.n_ff_exp, ne_loc = std::min<uint64_t>(ne, b->ep_n);
            if (int st = need(L.router->type == T_F32 && L.router->rows == ne && L.router->cols == e && ne <= 256 &&
                                  c.n_expert_used <= 16 && fx > 0,
                              p + "ffn_gate_inp.weight"))
                return fail(st);
            L.gate_exps = W(p + "ffn_gate_exps.weight"), L.up_exps = W(p + "ffn_up_exps.weight");
            L.down_exps = W(p + "ffn_down_exps.weight");
            const rcu_weight *ex[3] = {L.gate_exps, L.up_exps, L.down_exps};
            const uint64_t exs[3][2] = {{ne_loc * fx, e}, {ne_loc * fx, e}, {ne_loc * e, fx}};
            for (int i = 0; i < 3; i++)
                if (int st = need(ex[i] && ex[i]->rows == exs[i][0] && ex[i]->cols == exs[i][1] && gemv_supported(ex[i]->type),
                                  p + "ffn_*_exps.weight"))
                    return fail(st);
            L.gate_sh = W(p + "ffn_gate_shexp.weight");
            if (L.gate_sh) {
                L.up_sh = W(p + "ffn_up_shexp.weight"), L.down_sh = W(p + "ffn_down_shexp.weight");
                if (int st = need(L.up_sh && L.down_sh && L.gate_sh->cols == e && L.up_sh->rows == L.gate_sh->rows &&
                                      L.down_sh->rows == e && L.down_sh->cols == L.gate_sh->rows,
                                  p + "ffn_*_shexp.weight"))
                    return fail(st);
                L.sh_gate = V(p + "ffn_gate_inp_shexp.weight");
                b->ff_max = std::max<uint32_t>(b->ff_max, (uint32_t)L.gate_sh->rows);
            }
            L.gate = L.up = L.down = nullptr;
        }
        const rcu_weight *mats[7] = {L.wq, L.wk, L.wv, L.wo, L.gate, L.up, L.down};
        const uint64_t shp[7][2] = {{qd, e}, {kvd, e}, {kvd, e}, {e, qd}, {c.n_ff, e}, {c.n_ff, e}, {e, c.n_ff}};
        const char *names[7] = {"attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"};
        for (int i = 0; i < (L.router ? 4 : 7); i++)
            if (int st = need(mats[i] && mats[i]->rows == shp[i][0] && mats[i]->cols == shp[i][1] && gemv_supported(mats[i]->type),
                              p + names[i]))
                return fail(st);
        L.attn_norm = V(p + "attn_norm.weight");
        L.ffn_norm = V(p + "ffn_norm.weight");
        if (int st = need(L.attn_norm && L.ffn_norm, p + "attn_norm/ffn_norm")) return fail(st);
        L.q_norm = V(p + "attn_q_norm.weight"), L.k_norm = V(p + "attn_k_norm.weight");
        L.bq = V(p + "attn_q.bias"), L.bk = V(p + "attn_k.bias"), L.bv = V(p + "attn_v.bias");
        L.post_attn = V(p + "post_attention_norm.weight"), L.post_ffn = V(p + "post_ffw_norm.weight");
        L.swa = c.swa_window > 0 && c.swa_pattern > 0 && (il % c.swa_pattern) < c.swa_pattern - 1;
        if (L.gate) b->ff_max = std::max<uint32_t>(b->ff_max, (uint32_t)L.gate->rows);
        b->layers.push_back(L);
        const uint64_t slots = L.swa ? std::min<uint64_t>(c.swa_window + b->max_batch, n_ctx) : n_ctx;
        rcu_kv *kv = nullptr;
        if (int st = rcu_kv_create(ctx, kv_type, c.n_head_kv, c.head_dim, slots, &kv)) return fail(st);
        b->kv.push_back(kv);
    }
    const uint64_t T = b->max_batch;
    const uint64_t kmax = std::max<uint64_t>(std::max<uint64_t>(e, qd), b->ff_max);
    if (int st = rcu_acts_create(ctx, T, kmax, &b->acts)) return fail(st);
    if (T >= 32)  // prefill batches take the tensor-core GEMM: size its f16 activations now
        if (int st = gemm_f16_reserve(ctx, T, kmax)) return fail(st);
    bool moe = false;
    for (auto &L : b->layers) moe = moe || L.router;
    if (moe) {  // mixture-of-experts scratch (sizes for the largest batch)
        const uint64_t ne = c.n_expert, kk = std::min<uint64_t>(std::max<uint32_t>(c.n_expert_used, 1), ne);
        const uint64_t fx = c.n_ff_exp;
        struct {
            void **p;
            uint64_t bytes;
        } mb[] = {{(void **)&b->moe_logits, T * ne * 4}, {(void **)&b->moe_sgate, T * 4}, {(void **)&b->moe_w, T * kk * 4},
                  {(void **)&b->moe_sel, T * kk * 4},   {(void **)&b->moe_g, T * kk * fx * 4},
                  {(void **)&b->moe_u, T * kk * fx * 4}, {(void **)&b->moe_y, T * kk * e * 4},
                  {(void **)&b->moe_ys, T * e * 4}};
        for (auto &x : mb)
            if (int st = dalloc(b, x.p, x.bytes)) return fail(st);
        if (8 * kk > 64) return fail(set_err(ctx, RCU_ERR_UNSUPPORTED, "more than 8 experts per token"));
        // batches of kMoeGroupedMinTok tokens or more run grouped expert GEMMs over T * kk rows
        const bool grp = T >= kMoeGroupedMinTok && ne <= 256;
        const uint64_t rows2 = std::max<uint64_t>(grp ? T * kk : T, 8 * kk);
        if (int st = rcu_acts_create(ctx, rows2, std::max<uint64_t>(fx, b->ff_max), &b->acts2)) return fail(st);
        if (grp) {
            struct {
                void **p;
                uint64_t bytes;
            } gb[] = {{(void **)&b->moe_slot, T * kk * 4}, {(void **)&b->moe_row, T * kk * 4},
                      {(void **)&b->moe_off, (ne + 1) * 4}};
            for (auto &x : gb)
                if (int st = dalloc(b, x.p, x.bytes)) return fail(st);
            RCU_CUDA_TRY(ctx, cudaMallocHost((void **)&b->moe_off_host, (ne + 1) * 4));
            RCU_CUDA_TRY(ctx, cudaEventCreateWithFlags(&b->ev_plan, cudaEventDisableTiming));
            if (int st = gemm_f16_reserve(ctx, T * kk, std::max<uint64_t>(e, fx))) return fail(st);
        }
    }
    struct {
        float **p;
        uint64_t n;
    } bufs[] = {{&b->x, T * e}, {&b->xn, T * e}, {&b->q, T * qd}, {&b->k, T * kvd}, {&b->v, T * kvd}, {&b->att, T * qd},
                {&b->o, T * e}, {&b->g, T * b->ff_max}, {&b->u, T * b->ff_max},
                {&b->logits, T * (uint64_t)c.n_vocab * P}, {&b->logits_local, P > 1 ? T * (uint64_t)c.n_vocab : 1},
                {&b->logits_gather, P > 1 ? T * (uint64_t)c.n_vocab * P : 1}};
    for (auto &bf : bufs)
        if (int st = dalloc(b, (void **)bf.p, bf.n * sizeof(float))) return fail(st);
    if (int st = dalloc(b, (void **)&b->tokens, T * sizeof(uint32_t))) return fail(st);
    if (int st = dalloc(b, (void **)&b->pos_dev, sizeof(uint64_t))) return fail(st);
    uint64_t scratch = 0;  // split-context attention partials, sized for the longest layer
    for (uint32_t il = 0; il < c.n_layer; il++) {
        b->fused_merge = b->fused_merge &&
                         attention_fused_merge_ok(c.n_head, c.n_head_kv, c.head_dim, act_format(b->layers[il].wo->type));
        const uint64_t window = b->layers[il].swa ? c.swa_window : 0;
        scratch = std::max<uint64_t>(scratch, attention_scratch_bytes_upto(ctx, b->kv[il], T, c.n_head, window));
    }
    if (int st = dalloc(b, (void **)&b->attn_scratch, scratch)) return fail(st);
    RCU_CUDA_TRY(ctx, cudaMemset(b->attn_scratch, 0, scratch));  // attention completion counters
    RCU_CUDA_TRY(ctx, cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking));
    RCU_CUDA_TRY(ctx, cudaEventCreateWithFlags(&b->ev_in, cudaEventDisableTiming));
    RCU_CUDA_TRY(ctx, cudaEventCreateWithFlags(&b->ev_out, cudaEventDisableTiming));
    if (const char *g = std::getenv("RIE_CUDA_GRAPHS")) b->use_graphs = std::strcmp(g, "0") != 0;
    // RoPE inverse frequencies (ops.rs:65-79), computed like the reference in f32 on the host
    auto freqs = [&](float base, float fs, float **dst) -> int {
        const uint32_t half = c.rope_dim / 2;
        std::vector<float> f(std::max<uint32_t>(half, 1));
        for (uint32_t i = 0; i < half; i++) f[i] = std::pow(base, -2.0f * (float)i / (float)c.rope_dim) * fs;
        if (int st = dalloc(b, (void **)dst, f.size() * 4)) return st;
        RCU_CUDA_TRY(ctx, cudaMemcpy(*dst, f.data(), f.size() * 4, cudaMemcpyHostToDevice));
        return RCU_OK;
    };
    if (int st = freqs(c.rope_base, c.rope_freq_scale, &b->inv_freq)) return fail(st);
    if (int st = freqs(c.rope_base_swa > 0.0f ? c.rope_base_swa : c.rope_base, 1.0f, &b->inv_freq_swa)) return fail(st);
    if (P > 1) {  // every rank of the model calls this with the same id
        ncclUniqueId id;
        std::memcpy(&id, uid, sizeof(id));
        RCU_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
        const ncclResult_t r = ncclCommInitRank(&b->comm, P, id, m->tp_rank);
        if (r != ncclSuccess) return fail(nccl_err(ctx, r, "ncclCommInitRank"));
        if (int st = setup_fused_all_reduce(b)) return fail(st);
    }
    *out = b;
    return RCU_OK;
}

int32_t rcu_backend_kv(rcu_backend *b, uint64_t layer, rcu_kv **out) {
    if (!b || !out || layer >= b->kv.size()) return RCU_ERR_INVALID;
    *out = b->kv[layer];
    return RCU_OK;
}

void rcu_backend_free(rcu_backend *b) {
    if (!b) return;
    cudaSetDevice(b->ctx->device);
    if (b->stream) cudaStreamSynchronize(b->stream);
    if (b->graph_exec) cudaGraphExecDestroy(b->graph_exec);
    if (b->graph) cudaGraphDestroy(b->graph);
    for (int q = 0; q < 8; q++)
        if (b->ar_peer_buf[q] && b->ar_peer_buf[q] != b->ar_buf) {
            cudaIpcCloseMemHandle(b->ar_peer_buf[q]);
            cudaIpcCloseMemHandle(b->ar_peer_flags[q]);
        }
    // b->ar_buf / b->ar_flags stay allocated until the process exits: memory exported over
    // IPC may only be released after every importing rank has closed it, and free() cannot
    // synchronise with the other ranks.
    if (b->comm) ncclCommDestroy(b->comm);  // after the graph that holds its collectives
    if (b->ev_in) cudaEventDestroy(b->ev_in);
    if (b->ev_out) cudaEventDestroy(b->ev_out);
    if (b->ev_plan) cudaEventDestroy(b->ev_plan);
    if (b->moe_off_host) cudaFreeHost(b->moe_off_host);
    if (b->tok_pin) cudaFreeHost(b->tok_pin);
    if (b->logits_pin) cudaFreeHost(b->logits_pin);
    if (b->stream) cudaStreamDestroy(b->stream);
    for (auto *kv : b->kv) rcu_kv_free(kv);
    rcu_acts_free(b->acts);
    rcu_acts_free(b->acts2);
    cudaSetDevice(b->ctx->device);
    for (void *p : b->allocs) cudaFree(p);
    delete b;
}

uint64_t rcu_backend_max_batch(const rcu_backend *b) { return b ? b->max_batch : 0; }
uint64_t rcu_backend_n_ctx(const rcu_backend *b) { return b ? b->n_ctx : 0; }

static int32_t check_forward(rcu_backend *b, uint64_t n, uint64_t pos) {
    if (n == 0) return set_err(b->ctx, RCU_ERR_RUNTIME, "empty batch");  // cpu.rs:215-231
    if (n > b->max_batch)
        return set_err(b->ctx, RCU_ERR_RUNTIME,
                       "batch of " + std::to_string(n) + " tokens exceeds max batch " + std::to_string(b->max_batch));
    if (pos + n > b->n_ctx)
        return set_err(b->ctx, RCU_ERR_RUNTIME, "context window full (" + std::to_string(b->n_ctx) + " tokens)");
    return RCU_OK;
}

// Runs one forward on the backend stream, joined to the context stream by events. Single
// token, last-logits calls (decode) are captured once into a CUDA graph and replayed: every
// kernel reads the token and position from device memory and the attention grid covers the
// whole cache, so the launch sequence does not change between steps.
static int32_t run_forward(rcu_backend *b, const uint32_t *tokens, bool tokens_on_host, uint64_t n, uint64_t pos,
                           bool all_logits, float *logits) {
    rcu_ctx *ctx = b->ctx;
    cudaStream_t caller = ctx->stream;
    RCU_CUDA_TRY(ctx, cudaEventRecord(b->ev_in, caller));
    RCU_CUDA_TRY(ctx, cudaStreamWaitEvent(b->stream, b->ev_in, 0));
    ctx->stream = b->stream;
    ctx->early_weights = true;  // model weights are written only at load time
    struct Restore {
        rcu_ctx *c;
        cudaStream_t s;
        ~Restore() {
            c->stream = s;
            c->early_weights = c->static_weights;
        }
    } restore{ctx, caller};
    const cudaMemcpyKind kind = tokens_on_host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
    if (tokens != b->tokens) RCU_CUDA_TRY(ctx, cudaMemcpyAsync(b->tokens, tokens, n * 4, kind, b->stream));
    const bool fused_ar = b->m->tp_world > 1 && b->ar_ok && n <= 8;  // must match forward_dev's choice
    RCU_CUDA_TRY(ctx, launch_k(ctx, (k_set_pos), dim3(1), dim3(1), 0, b->pos_dev, pos,
                               fused_ar ? b->ar_epoch : (uint64_t *)nullptr));  // by value: no host buffer to keep alive
    const bool decode = n == 1 && !all_logits && logits == b->logits;
    if (decode && b->use_graphs && b->graph_exec) {
        RCU_CUDA_TRY(ctx, cudaGraphLaunch(b->graph_exec, b->stream));
    } else if (decode && b->use_graphs && b->decode_calls >= 1) {
        // the first decode ran eagerly (kernel attributes set, all lazily created state made);
        // capture the second one and replay it from then on
        RCU_CUDA_TRY(ctx, cudaStreamBeginCapture(b->stream, cudaStreamCaptureModeThreadLocal));
        const int st = forward_dev(b, 1, pos, false, b->logits, true);
        cudaGraph_t g = nullptr;
        const cudaError_t e = cudaStreamEndCapture(b->stream, &g);
        if (st) {
            if (g) cudaGraphDestroy(g);
            return st;
        }
        if (e != cudaSuccess) return cuda_err(ctx, e, "cudaStreamEndCapture");
        cudaGraphExec_t ge = nullptr;
        const cudaError_t e2 = cudaGraphInstantiate(&ge, g, 0);
        if (e2 != cudaSuccess) {
            cudaGraphDestroy(g);
            return cuda_err(ctx, e2, "cudaGraphInstantiate");
        }
        b->graph = g;
        b->graph_exec = ge;
        RCU_CUDA_TRY(ctx, cudaGraphLaunch(b->graph_exec, b->stream));
    } else {
        if (int32_t st = forward_dev(b, n, pos, all_logits, logits, decode && b->use_graphs)) return st;
    }
    if (decode) b->decode_calls++;
    RCU_CUDA_TRY(ctx, cudaEventRecord(b->ev_out, b->stream));
    RCU_CUDA_TRY(ctx, cudaStreamWaitEvent(caller, b->ev_out, 0));
    return RCU_OK;
}

int32_t rcu_backend_forward(rcu_backend *b, const uint32_t *tokens, uint64_t n, uint64_t pos, int32_t all_logits,
                            float *logits, uint64_t logits_len) {
    if (!b || !tokens || !logits) return b ? set_err(b->ctx, RCU_ERR_INVALID, "null argument") : RCU_ERR_INVALID;
    if (int32_t st = check_forward(b, n, pos)) return st;
    const uint64_t rows = all_logits ? n : 1;
    if (logits_len < rows * b->m->cfg.n_vocab) return set_err(b->ctx, RCU_ERR_RUNTIME, "logits buffer too small");  // full vocabulary
    for (uint64_t i = 0; i < n; i++)
        if (tokens[i] >= b->embd->rows) return set_err(b->ctx, RCU_ERR_RUNTIME, "token id " + std::to_string(tokens[i]) + " out of range");
    rcu_ctx *ctx = b->ctx;
    const uint64_t nv = b->m->cfg.n_vocab;
    if (!b->tok_pin) RCU_CUDA_TRY(ctx, cudaMallocHost(&b->tok_pin, b->max_batch * sizeof(uint32_t)));
    if (rows == 1 && !b->logits_pin) RCU_CUDA_TRY(ctx, cudaMallocHost(&b->logits_pin, nv * sizeof(float)));
    // the previous call synchronised before returning, so the staging buffers are free
    std::memcpy(b->tok_pin, tokens, n * sizeof(uint32_t));
    if (int32_t st = run_forward(b, b->tok_pin, true, n, pos, all_logits != 0, b->logits)) {
        cudaStreamSynchronize(b->stream);  // a token copy already queued must finish before the next call refills tok_pin
        return st;
    }
    if (rows > 1) {  // prompt logits of every token: straight into the caller's buffer
        RCU_CUDA_TRY(ctx, cudaMemcpyAsync(logits, b->logits, rows * nv * 4, cudaMemcpyDeviceToHost, ctx->stream));
        return rcu_sync(ctx);
    }
    RCU_CUDA_TRY(ctx, cudaMemcpyAsync(b->logits_pin, b->logits, nv * 4, cudaMemcpyDeviceToHost, ctx->stream));
    if (int32_t st = rcu_sync(ctx)) return st;
    std::memcpy(logits, b->logits_pin, nv * 4);
    return RCU_OK;
}

int32_t rcu_backend_forward_device(rcu_backend *b, const uint32_t *tokens_dev, uint64_t n, uint64_t pos,
                                   int32_t all_logits, float *logits_dev) {
    if (!b || !tokens_dev || !logits_dev) return b ? set_err(b->ctx, RCU_ERR_INVALID, "null argument") : RCU_ERR_INVALID;
    if (int32_t st = check_forward(b, n, pos)) return st;
    // decode steps run through the backend's own logits buffer (and graph), then copy out
    const bool decode = n == 1 && !all_logits;
    if (int32_t st = run_forward(b, tokens_dev, false, n, pos, all_logits != 0, decode ? b->logits : logits_dev)) return st;
    if (decode && logits_dev != b->logits)
        RCU_CUDA_TRY(b->ctx, cudaMemcpyAsync(logits_dev, b->logits, b->m->cfg.n_vocab * 4, cudaMemcpyDeviceToDevice,
                                             b->ctx->stream));
    return RCU_OK;
}

int32_t rcu_backend_forward_layers(rcu_backend *b, const float *x_dev, uint64_t n, uint64_t pos, uint64_t layer0,
                                   uint64_t layer1, float *x_out_dev, float *logits_dev) {
    if (!b || !x_dev) return b ? set_err(b->ctx, RCU_ERR_INVALID, "null argument") : RCU_ERR_INVALID;
    if (int32_t st = check_forward(b, n, pos)) return st;
    if (layer0 > layer1 || layer1 > b->cfg.n_layer) return set_err(b->ctx, RCU_ERR_INVALID, "layer range out of bounds");
    if (logits_dev && layer1 != b->cfg.n_layer) return set_err(b->ctx, RCU_ERR_INVALID, "logits need the last layer");
    if (!x_out_dev && !logits_dev) return set_err(b->ctx, RCU_ERR_INVALID, "nothing to write");
    rcu_ctx *ctx = b->ctx;
    cudaStream_t caller = ctx->stream;
    RCU_CUDA_TRY(ctx, cudaEventRecord(b->ev_in, caller));
    RCU_CUDA_TRY(ctx, cudaStreamWaitEvent(b->stream, b->ev_in, 0));
    ctx->stream = b->stream;
    ctx->early_weights = true;
    struct Restore {
        rcu_ctx *c;
        cudaStream_t s;
        ~Restore() {
            c->stream = s;
            c->early_weights = c->static_weights;
        }
    } restore{ctx, caller};
    const bool fused_ar = b->m->tp_world > 1 && b->ar_ok && n <= 8;  // must match forward_span's choice
    RCU_CUDA_TRY(ctx, launch_k(ctx, (k_set_pos), dim3(1), dim3(1), 0, b->pos_dev, pos,
                               fused_ar ? b->ar_epoch : (uint64_t *)nullptr));
    if (int32_t st = forward_span(b, n, pos, true, logits_dev, false, x_dev, (uint32_t)layer0, (uint32_t)layer1,
                                  x_out_dev))
        return st;
    RCU_CUDA_TRY(ctx, cudaEventRecord(b->ev_out, b->stream));
    RCU_CUDA_TRY(ctx, cudaStreamWaitEvent(caller, b->ev_out, 0));
    return RCU_OK;
}

int32_t rcu_diag_expire_peer_wait(rcu_ctx *ctx) {
    if (!ctx) return RCU_ERR_INVALID;
    // one 256-value row through the fused all-reduce norm, waiting for a second rank's partial
    // rows that never arrive: arrival counters at zero, one forward already counted
    constexpr uint32_t e = 256, P = 2;
    uint8_t *mem = nullptr;
    const size_t bytes = 2 * P * e * sizeof(float) + 64;
    RCU_CUDA_TRY(ctx, cudaMalloc(&mem, bytes));
    struct Free {
        uint8_t *p;
        ~Free() { cudaFree(p); }
    } free_mem{mem};
    RCU_CUDA_TRY(ctx, cudaMemsetAsync(mem, 0, bytes, ctx->stream));
    float *x = reinterpret_cast<float *>(mem), *src = x + e, *w = src + P * e;
    uint32_t *flag = reinterpret_cast<uint32_t *>(mem + 2 * P * e * sizeof(float));
    uint64_t *epoch = reinterpret_cast<uint64_t *>(flag + 8);
    const uint64_t one = 1;
    RCU_CUDA_TRY(ctx, cudaMemcpyAsync(epoch, &one, sizeof(one), cudaMemcpyHostToDevice, ctx->stream));
    const ArSum ar{src, flag, epoch, kArUnit, P, e, ctx->dev_err, ctx->wait_limit_ns};
    const ActOut ao{};
    RCU_CUDA_TRY(ctx, launch_k(ctx, k_norm_q8, dim3(1), dim3(e / 8), 0, x, (const float *)nullptr, (const float *)nullptr,
                               1.0f, (const float *)w, e, 1e-6f, (float *)nullptr, ao, 0, ar));
    RCU_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    return rcu_check_device(ctx, nullptr);
}

int32_t rcu_backend_hidden(const rcu_backend *b, float *host_out, uint64_t cap, uint64_t *rows_out) {
    if (!b || !host_out) return RCU_ERR_INVALID;
    const uint64_t n = b->hidden_rows * b->m->cfg.n_embd;
    if (rows_out) *rows_out = b->hidden_rows;
    if (cap < n) return set_err(b->ctx, RCU_ERR_INVALID, "hidden buffer too small");
    RCU_CUDA_TRY(b->ctx, cudaStreamSynchronize(b->stream));
    RCU_CUDA_TRY(b->ctx, cudaMemcpyAsync(host_out, b->xn, n * 4, cudaMemcpyDeviceToHost, b->ctx->stream));
    RCU_CUDA_TRY(b->ctx, cudaStreamSynchronize(b->ctx->stream));
    return RCU_OK;
}

}  // extern "C"
