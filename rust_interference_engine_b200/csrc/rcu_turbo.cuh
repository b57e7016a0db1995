// rcu_turbo.cuh -- turbo4 pieces shared by the KV-cache / attention translation units:
// the random-sign Hadamard rotation (turbo.rs:51-118) and the per-lane Q8_0 quantizer of
// the rotated queries (quant/mod.rs:175-189). Each translation unit that includes this
// header has its own copy of the sign table and fills it with ensure_signs() before its
// first launch.
#pragma once
#include "rcu_internal.cuh"

namespace rcu {

constexpr uint64_t KV_SEED = 0x75426F5175616E74ull;          // turbo.rs:122
constexpr int kMaxHd = 512;                                   // cpu.rs:106 (turbo needs hd <= 512)
static __constant__ int8_t c_levels[16] = {-126, -95, -74, -58, -43, -30, -18, -6, 6, 18, 30, 43, 58, 74, 95, 126};
static __constant__ float c_signs[kMaxHd];                            // sign(KV_SEED, i)
static __constant__ float c_levels46[16];  // the levels / 46 (kv_levels, turbo.rs:129-131), IEEE f32 division

static float host_sign(uint64_t seed, uint64_t i) {  // turbo.rs:80-89
    uint64_t z = seed + i * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return ((z ^ (z >> 31)) & 1) == 0 ? 1.0f : -1.0f;
}
static int ensure_signs(rcu_ctx *ctx) {
    static bool done[64] = {};
    if (done[ctx->device & 63]) return RCU_OK;
    float s[kMaxHd];
    for (int i = 0; i < kMaxHd; i++) s[i] = host_sign(KV_SEED, i);
    RCU_CUDA_TRY(ctx, cudaMemcpyToSymbol(c_signs, s, sizeof(s)));
    static const int8_t lv[16] = {-126, -95, -74, -58, -43, -30, -18, -6, 6, 18, 30, 43, 58, 74, 95, 126};
    float c[16];
    for (int i = 0; i < 16; i++) c[i] = (float)lv[i] / 46.0f;
    RCU_CUDA_TRY(ctx, cudaMemcpyToSymbol(c_levels46, c, sizeof(c)));
    done[ctx->device & 63] = true;
    return RCU_OK;
}
__host__ __device__ inline uint32_t turbo_block(uint32_t d) {  // turbo.rs:52-58
    uint32_t b = 1;
    while (d % (b * 2) == 0 && b < 256) b *= 2;
    return b;
}
__host__ __device__ inline uint32_t turbo_row_bytes(uint32_t d) { return 2 * (d / turbo_block(d)) + d / 2; }

// rotate_row for rows that are one rotation block of 32 V values: lane l holds values V l ..
// V l + V - 1 in registers; the butterflies of stride h < V stay in the lane, those of stride
// h >= V pair lanes l and l ^ (h / V) through a shuffle. The same pairs in the same order of
// strides as rotate_row below, with the same IEEE operations, so the results are identical.
template <int V>
static __device__ __forceinline__ void rotate_regs(float *x, bool inverse, int lane) {
    float v[V];
#pragma unroll
    for (int i = 0; i < V; i++) v[i] = x[V * lane + i];
    if (!inverse)
#pragma unroll
        for (int i = 0; i < V; i++) v[i] = __fmul_rn(v[i], c_signs[V * lane + i]);
#pragma unroll
    for (int h = 1; h < V; h <<= 1)
#pragma unroll
        for (int i = 0; i < V; i++)
            if ((i & h) == 0) {
                const float a = v[i], c = v[i + h];
                v[i] = __fadd_rn(a, c);
                v[i + h] = __fsub_rn(a, c);
            }
#pragma unroll
    for (int hl = 1; hl < 32; hl <<= 1) {
        const bool upper = (lane & hl) != 0;
#pragma unroll
        for (int i = 0; i < V; i++) {
            const float p = __shfl_xor_sync(0xffffffffu, v[i], hl);
            v[i] = upper ? __fsub_rn(p, v[i]) : __fadd_rn(v[i], p);
        }
    }
    const float s = 1.0f / sqrtf((float)(32 * V));
#pragma unroll
    for (int i = 0; i < V; i++) {
        float o = __fmul_rn(v[i], s);
        if (inverse) o = __fmul_rn(o, c_signs[V * lane + i]);
        x[V * lane + i] = o;
    }
    __syncwarp();
}

// x <- R x (signs then normalised block FWHT) or x <- R^T x, on a warp-owned shared row.
static __device__ void rotate_row(float *x, uint32_t d, bool inverse, int lane) {
    __syncwarp();
    if (d == 128) return rotate_regs<4>(x, inverse, lane);
    if (d == 64) return rotate_regs<2>(x, inverse, lane);
    if (d == 256) return rotate_regs<8>(x, inverse, lane);
    const uint32_t b = turbo_block(d);
    if (!inverse)
        for (uint32_t i = lane; i < d; i += 32) x[i] = __fmul_rn(x[i], c_signs[i]);
    __syncwarp();
    for (uint32_t h = 1; h < b; h *= 2) {
        for (uint32_t pr = lane; pr < d / 2; pr += 32) {
            const uint32_t blk = pr / (b / 2), q = pr % (b / 2);
            const uint32_t j = blk * b + (q / h) * 2 * h + (q % h);
            const float a = x[j], c = x[j + h];
            x[j] = __fadd_rn(a, c);
            x[j + h] = __fsub_rn(a, c);
        }
        __syncwarp();
    }
    const float s = 1.0f / sqrtf((float)b);
    for (uint32_t i = lane; i < d; i += 32) {
        float v = __fmul_rn(x[i], s);
        if (inverse) v = __fmul_rn(v, c_signs[i]);
        x[i] = v;
    }
    __syncwarp();
}

// One value of a 32-wide Q8_0 block per lane (quant/mod.rs:175-189 / avx2.rs:153-184).
__device__ __forceinline__ int quant32(float v, int rounding, float &d_out) {
    const float amax = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(v))));
    const float d = amax / 127.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    const float p = __fmul_rn(v, id);
    const int r = rounding == RCU_ROUND_HALF_AWAY ? __float2int_rz(roundf(p)) : __float2int_rn(p);
    d_out = d;
    return max(-127, min(127, r));
}

// ---- KV rows ----------------------------------------------------------------------------
// quantize_rotated_4 (turbo.rs:141-164) of a rotated shared row into a reference row.
static __device__ void encode_rotated_row(const float *y, uint32_t d, uint8_t *out, uint8_t *qtmp, int lane) {
    const uint32_t b = turbo_block(d), nb = d / b;
    float thr[15];
#pragma unroll
    for (int i = 0; i < 15; i++) thr[i] = __fmul_rn(0.5f, __fadd_rn(c_levels46[i], c_levels46[i + 1]));
    for (uint32_t bi = 0; bi < nb; bi++) {
        const float *yb = y + bi * b;
        float inv = 0.0f;
        if (lane == 0) {
            float ss = 0.0f;
            for (uint32_t j = 0; j < b; j++) ss = __fadd_rn(ss, __fmul_rn(yb[j], yb[j]));
            const float rms = sqrtf(ss / (float)b);
            inv = rms > 0.0f ? 1.0f / rms : 0.0f;
        }
        inv = __shfl_sync(0xffffffffu, inv, 0);
        for (uint32_t j = lane; j < b; j += 32) {
            const float v = __fmul_rn(yb[j], inv);
            uint32_t q = 0;
#pragma unroll
            for (int i = 0; i < 15; i++) q += v > thr[i] ? 1u : 0u;
            qtmp[bi * b + j] = (uint8_t)q;
        }
        __syncwarp();
        if (lane == 0) {
            float num = 0.0f, den = 0.0f;
            for (uint32_t j = 0; j < b; j++) {
                const float cq = c_levels46[qtmp[bi * b + j]];
                num = __fadd_rn(num, __fmul_rn(yb[j], cq));
                den = __fadd_rn(den, __fmul_rn(cq, cq));
            }
            const float s = den > 0.0f ? num / den : 0.0f;
            *reinterpret_cast<unsigned short *>(out + 2 * bi) = __half_as_ushort(__float2half_rn(s));
        }
    }
    __syncwarp();
    uint8_t *codes = out + 2 * nb;
    for (uint32_t m = lane; m < d / 2; m += 32) {
        const uint32_t g = (m / 16) * 32 + m % 16;
        codes[m] = (uint8_t)(qtmp[g] | (qtmp[g + 16] << 4));
    }
    __syncwarp();
}

// Encodes one warp-owned shared row x (hd values; turbo rotates it in place) into cache row dst.
static __device__ void store_row(int type, float *x, uint32_t hd, uint8_t *dst, uint8_t *qtmp, int lane) {
    if (type == RCU_KV_F16) {
        unsigned short *o = reinterpret_cast<unsigned short *>(dst);
        for (uint32_t i = lane; i < hd; i += 32) o[i] = __half_as_ushort(__float2half_rn(x[i]));
        return;
    }
    if (type == RCU_KV_Q8_0) {  // store_q8_0 (cpu.rs:637-647): scalar rounding, f16 scale
        for (uint32_t b = 0; b < hd / 32; b++) {
            float d;
            const int q = quant32(x[b * 32 + lane], RCU_ROUND_HALF_AWAY, d);
            uint8_t *ob = dst + b * 34;
            if (lane == 0) *reinterpret_cast<unsigned short *>(ob) = __half_as_ushort(__float2half_rn(d));
            ob[2 + lane] = (uint8_t)(int8_t)q;
        }
        return;
    }
    rotate_row(x, hd, false, lane);
    encode_rotated_row(x, hd, dst, qtmp, lane);
}


// Bias-added q or k head vector x (warp-owned shared row): RMSNorm with weights `norm` (when
// given) and RoPE at position pos (ops.rs:7-14, 65-99; cpu.rs:280-300), as the standalone q/k
// post-processing kernel and the decode attention's fused path both do it.
static __device__ void qk_post_vec(float *x, uint32_t hd, const float *norm, float eps, bool rope,
                                   const float *inv_freq, uint64_t pos, uint32_t rope_dim, int neox, int lane) {
    if (norm) {
        float ss = 0.0f;
        for (uint32_t i = lane; i < hd; i += 32) ss += x[i] * x[i];
        for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float scale = 1.0f / sqrtf(ss / (float)hd + eps);
        for (uint32_t i = lane; i < hd; i += 32) x[i] *= scale * norm[i];
        __syncwarp();
    }
    if (rope) {
        const uint32_t half = rope_dim / 2;
        const float fpos = (float)pos;
        for (uint32_t i = lane; i < half; i += 32) {
            float sn, cs;
            sincosf(fpos * inv_freq[i], &sn, &cs);
            const uint32_t i0 = neox ? i : 2 * i, i1 = neox ? i + half : 2 * i + 1;
            const float a = x[i0], b = x[i1];
            x[i0] = a * cs - b * sn;
            x[i1] = a * sn + b * cs;
        }
        __syncwarp();
    }
}

}  // namespace rcu
