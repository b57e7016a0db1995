// rcu_attn_prefill.cu -- causal (optionally sliding-window) grouped-query attention of a batch
// of prompt tokens over an f16 KV cache (crates/rie-core/src/model/cpu.rs:550-634, KvType::F16),
// flash-attention style on the tensor cores.
//
// The reference scores every (token, head) pair against its positions one at a time with
// dot_f16_f32 (kernels/mod.rs:387-400), softmaxes them with the row maximum, and sums the f16 V
// rows with axpy_f16 (kernels/mod.rs:402-417). Here a CTA takes 64 query rows (64 / G tokens x
// the G query heads of one KV head) and walks the keys in blocks of 64 staged in shared memory:
//   S = Q K^T with mma.sync m16n8k16 (f16 inputs, f32 accumulation); Q is split into an f16 high
//   part and an f16 remainder, so the scores carry the f32 query to about 2^-22,
//   online softmax in f32 (running row maximum and sum, the output rescaled when it grows),
//   O += P V with P split the same way, V exact in f16: the result differs from the reference's
//   f32 arithmetic by about as much as a different f32 summation order would.
// The rows of the ring-buffer cache (slot = position % slots) are copied with cp.async into
// padded rows (HD + 8 halves), so the ldmatrix reads of 8 consecutive keys hit 8 different
// 16-byte bank groups. Keys past the batch's last position are zero-filled and masked.
#include "rcu_kernels.h"

namespace rcu {

constexpr int kPfRows = 64;      // query rows (token, head) per CTA
constexpr int kPfKeys = 64;      // keys per block
constexpr int kPfThreads = 128;  // 4 warps x 16 query rows

struct PfParams {
    const __half *kc, *vc;  // [n_kv][slots][hd]
    const float *q;         // [n_tok][n_head * hd], attention scale applied
    float *out;             // [n_tok][n_head * hd]
    uint32_t n_tok, n_head, n_kv, slots, window, group;
    uint64_t pos0;
    const uint64_t *pos_ptr;
    float softcap;
};

__device__ __forceinline__ uint32_t pf_pack(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&h);
}
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void pf_cp16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

template <int HD>
__global__ void __launch_bounds__(kPfThreads) k_attn_prefill(const PfParams p) {
    extern __shared__ __align__(16) uint8_t pf_smem[];
    constexpr int LD = HD + 8;  // padded row, in halves
    constexpr int KS = HD / 16;  // k-steps of S = Q K^T
    constexpr int NO = HD / 8;   // n-tiles of O
    __half *sk = reinterpret_cast<__half *>(pf_smem);  // [2][kPfKeys][LD]
    __half *sv = sk + 2 * kPfKeys * LD;                 // [2][kPfKeys][LD]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
    const uint32_t kvh = blockIdx.x, G = p.group, qd = p.n_head * HD;
    const uint32_t row0 = blockIdx.y * kPfRows;
    pdl_wait();  // q and this batch's K/V rows come from the kernel before
    pdl_trigger();
    const uint64_t pos = p.pos_ptr ? *p.pos_ptr : p.pos0;

    // this thread's two query rows: g and g + 8 of the warp's 16
    uint32_t tok[2], head[2];
    bool live[2];
    uint64_t lo_pos[2], hi_pos[2];  // attended positions [lo, hi]
#pragma unroll
    for (int i = 0; i < 2; i++) {
        const uint32_t r = row0 + 16 * warp + g + 8 * i;
        tok[i] = r / G;
        head[i] = kvh * G + r % G;
        live[i] = tok[i] < p.n_tok;
        hi_pos[i] = pos + tok[i];
        lo_pos[i] = p.window > 0 && hi_pos[i] + 1 > p.window ? hi_pos[i] + 1 - p.window : 0;
    }
    // Q fragments: rows (g, g + 8), columns 16 ks + {2 t4, 2 t4 + 8} (+1), high and low f16 parts
    uint32_t qh[KS][4], ql[KS][4];
#pragma unroll
    for (int ks = 0; ks < KS; ks++) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int i = j & 1;
            const uint32_t col = 16 * ks + 2 * t4 + (j >= 2 ? 8 : 0);
            float2 x = make_float2(0.0f, 0.0f);
            if (live[i]) x = *reinterpret_cast<const float2 *>(p.q + (uint64_t)tok[i] * qd + head[i] * HD + col);
            const __half2 h = __floats2half2_rn(x.x, x.y);
            const float2 hf = __half22float2(h);
            qh[ks][j] = *reinterpret_cast<const uint32_t *>(&h);
            ql[ks][j] = pf_pack(x.x - hf.x, x.y - hf.y);
        }
    }
    // keys of the whole CTA: from its first row's window start to its last token's position
    const uint32_t t_first = row0 / G;
    const uint32_t t_last = (min(row0 + kPfRows, p.n_tok * G) - 1) / G;
    const uint64_t k_hi = pos + t_last;
    const uint64_t k_lo = p.window > 0 && pos + t_first + 1 > p.window ? pos + t_first + 1 - p.window : 0;
    const uint32_t n_blk = (uint32_t)((k_hi - k_lo) / kPfKeys + 1);

    auto stage = [&](uint32_t b, int buf) {
        constexpr int CH = HD / 8;  // 16-byte chunks per row
        for (uint32_t c = threadIdx.x; c < kPfKeys * CH; c += kPfThreads) {
            const uint32_t key = c / CH, ch = c % CH;
            const uint64_t kp = k_lo + (uint64_t)b * kPfKeys + key;
            __half *dk = sk + ((uint32_t)buf * kPfKeys + key) * LD + ch * 8;
            __half *dv = sv + ((uint32_t)buf * kPfKeys + key) * LD + ch * 8;
            if (kp <= k_hi) {
                const uint64_t off = ((uint64_t)kvh * p.slots + kp % p.slots) * HD + ch * 8;
                pf_cp16(dk, p.kc + off);
                pf_cp16(dv, p.vc + off);
            } else {  // past the batch: zeros (masked scores, and 0 * V must stay 0)
                *reinterpret_cast<uint4 *>(dk) = make_uint4(0, 0, 0, 0);
                *reinterpret_cast<uint4 *>(dv) = make_uint4(0, 0, 0, 0);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };

    float o[NO][4];
#pragma unroll
    for (int n = 0; n < NO; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.0f, 0.0f};

    stage(0, 0);
    for (uint32_t b = 0; b < n_blk; b++) {
        const int buf = b & 1;
        if (b + 1 < n_blk) {
            stage(b + 1, buf ^ 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
        const __half *kb = sk + (uint32_t)buf * kPfKeys * LD, *vb = sv + (uint32_t)buf * kPfKeys * LD;
        // ---- S = Q K^T (16 rows x 64 keys per warp) ----
        float s[8][4];
#pragma unroll
        for (int n = 0; n < 8; n++) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.0f;
#pragma unroll
        for (int ks = 0; ks < KS; ks++) {
#pragma unroll
            for (int np = 0; np < 4; np++) {  // n-tiles 2 np, 2 np + 1
                const int mi = lane >> 3;
                const uint32_t key = 8 * (2 * np + (mi >> 1)) + (lane & 7), col = 16 * ks + 8 * (mi & 1);
                uint32_t r[4];
                ldsm_x4(r, kb + key * LD + col);
                mma16816(s[2 * np], qh[ks], r[0], r[1]);
                mma16816(s[2 * np], ql[ks], r[0], r[1]);
                mma16816(s[2 * np + 1], qh[ks], r[2], r[3]);
                mma16816(s[2 * np + 1], ql[ks], r[2], r[3]);
            }
        }
        // ---- mask, softcap, online softmax ----
        const uint64_t kp0 = k_lo + (uint64_t)b * kPfKeys;
        float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int n = 0; n < 8; n++) {
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int i = j >> 1;
                const uint64_t kp = kp0 + 8 * n + 2 * t4 + (j & 1);
                float v = s[n][j];
                if (p.softcap > 0.0f) v = p.softcap * tanhf(v / p.softcap);
                if (!live[i] || kp > hi_pos[i] || kp < lo_pos[i]) v = -INFINITY;
                s[n][j] = v;
                mx[i] = fmaxf(mx[i], v);
            }
        }
        float alpha[2];
#pragma unroll
        for (int i = 0; i < 2; i++) {
            mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 1));
            mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 2));
            const float mn = fmaxf(m[i], mx[i]);
            alpha[i] = mn == -INFINITY ? 1.0f : __expf(m[i] - mn);
            m[i] = mn;
            l[i] *= alpha[i];
        }
#pragma unroll
        for (int n = 0; n < 8; n++) {
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int i = j >> 1;
                const float e = s[n][j] == -INFINITY ? 0.0f : __expf(s[n][j] - m[i]);
                s[n][j] = e;
                l[i] += e;
            }
        }
#pragma unroll
        for (int n = 0; n < NO; n++) {
            o[n][0] *= alpha[0], o[n][1] *= alpha[0];
            o[n][2] *= alpha[1], o[n][3] *= alpha[1];
        }
        // ---- O += P V ----
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {  // keys 16 kk .. 16 kk + 15
            // P as an f16 high part and an f16 remainder (A fragments of the two n-tiles' C values)
            const float *c0 = s[2 * kk], *c1 = s[2 * kk + 1];
            uint32_t ah[4], al[4];
            const float pv[4][2] = {{c0[0], c0[1]}, {c0[2], c0[3]}, {c1[0], c1[1]}, {c1[2], c1[3]}};
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const __half2 h = __floats2half2_rn(pv[j][0], pv[j][1]);
                const float2 hf = __half22float2(h);
                ah[j] = *reinterpret_cast<const uint32_t *>(&h);
                al[j] = pf_pack(pv[j][0] - hf.x, pv[j][1] - hf.y);
            }
#pragma unroll
            for (int nd = 0; nd < HD / 16; nd++) {  // hd n-tiles 2 nd, 2 nd + 1
                const int mi = lane >> 3;
                const uint32_t key = 16 * kk + 8 * (mi & 1) + (lane & 7), col = 16 * nd + 8 * (mi >> 1);
                uint32_t r[4];
                ldsm_x4_t(r, vb + key * LD + col);
                mma16816(o[2 * nd], ah, r[0], r[1]);
                mma16816(o[2 * nd], al, r[0], r[1]);
                mma16816(o[2 * nd + 1], ah, r[2], r[3]);
                mma16816(o[2 * nd + 1], al, r[2], r[3]);
            }
        }
        __syncthreads();  // the buffer is restaged two blocks later
    }
    // ---- normalise and store ----
#pragma unroll
    for (int i = 0; i < 2; i++) {
        l[i] += __shfl_xor_sync(0xffffffffu, l[i], 1);
        l[i] += __shfl_xor_sync(0xffffffffu, l[i], 2);
    }
#pragma unroll
    for (int i = 0; i < 2; i++) {
        if (!live[i]) continue;
        const float inv = l[i] > 0.0f ? 1.0f / l[i] : 0.0f;
        float *orow = p.out + (uint64_t)tok[i] * qd + head[i] * HD;
#pragma unroll
        for (int n = 0; n < NO; n++)
            *reinterpret_cast<float2 *>(orow + 8 * n + 2 * t4) = make_float2(o[n][2 * i] * inv, o[n][2 * i + 1] * inv);
    }
}

bool attention_prefill_ok(int kv_type, uint64_t hd, uint64_t group, uint64_t n_tok) {
    return kv_type == RCU_KV_F16 && (hd == 64 || hd == 128) && group >= 1 && kPfRows % group == 0 &&
           n_tok >= kPrefillAttnMinTok;
}

int launch_attention_prefill(rcu_ctx *ctx, const void *kc, const void *vc, uint64_t n_kv, uint64_t hd, uint64_t slots,
                             const float *q, uint64_t n_tok, uint64_t n_head, uint64_t pos0, const uint64_t *pos_ptr,
                             uint64_t window, float softcap, float *out) {
    PfParams p{};
    p.kc = reinterpret_cast<const __half *>(kc);
    p.vc = reinterpret_cast<const __half *>(vc);
    p.q = q;
    p.out = out;
    p.n_tok = (uint32_t)n_tok;
    p.n_head = (uint32_t)n_head;
    p.n_kv = (uint32_t)n_kv;
    p.slots = (uint32_t)slots;
    p.window = (uint32_t)window;
    p.group = (uint32_t)(n_head / n_kv);
    p.pos0 = pos0;
    p.pos_ptr = pos_ptr;
    p.softcap = softcap;
    const dim3 grid((uint32_t)n_kv, (uint32_t)((n_tok * p.group + kPfRows - 1) / kPfRows));
    const size_t smem = 4ull * kPfKeys * (hd + 8) * sizeof(__half);
    if (hd == 64) {
        RCU_CUDA_TRY(ctx, cudaFuncSetAttribute(k_attn_prefill<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        RCU_CUDA_TRY(ctx, launch_k(ctx, k_attn_prefill<64>, grid, dim3(kPfThreads), smem, p));
    } else {
        RCU_CUDA_TRY(ctx, cudaFuncSetAttribute(k_attn_prefill<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        RCU_CUDA_TRY(ctx, launch_k(ctx, k_attn_prefill<128>, grid, dim3(kPfThreads), smem, p));
    }
    return RCU_OK;
}

}  // namespace rcu
