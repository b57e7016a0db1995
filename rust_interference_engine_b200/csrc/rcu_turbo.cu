// rcu_turbo.cu -- KV cache (f16 / Q8_0 / turbo4) append and decode attention.
//
//   turbo4 rotation, encode       crates/rie-core/src/turbo.rs:51-171
//   turbo4 score / V accumulate   crates/rie-core/src/turbo.rs:178-250
//   KV append                     crates/rie-core/src/model/cpu.rs:300-328, 636-647
//   attention                     crates/rie-core/src/model/cpu.rs:552-634
//
// Encoding is bit-exact with the reference: the Walsh-Hadamard butterflies are the same
// IEEE additions in the same stage order, and the three order-sensitive sums of
// quantize_rotated_4 (sum of squares, num, den) run in the reference's sequential order.
// Attention is a split-context ("flash-decode") kernel: each CTA scores a chunk of cache
// rows for every query head of one KV head (GQA group), keeps an un-normalised partial
// output, and a second kernel merges the chunks and applies the inverse rotation.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "rcu_actq.cuh"
#include "rcu_blocks.cuh"
#include "rcu_kernels.h"

struct rcu_kv {
    rcu_ctx *ctx = nullptr;
    int type = 0;
    uint64_t n_kv = 0, hd = 0, slots = 0, row_bytes = 0;
    uint8_t *k = nullptr, *v = nullptr;  // device, [kv_head][slot][row_bytes]
};

namespace rcu {

constexpr uint64_t KV_SEED = 0x75426F5175616E74ull;          // turbo.rs:122
constexpr int kMaxHd = 512;                                   // cpu.rs:106 (turbo needs hd <= 512)
__constant__ int8_t c_levels[16] = {-126, -95, -74, -58, -43, -30, -18, -6, 6, 18, 30, 43, 58, 74, 95, 126};
__constant__ float c_signs[kMaxHd];                            // sign(KV_SEED, i)

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
    done[ctx->device & 63] = true;
    return RCU_OK;
}
__host__ __device__ inline uint32_t turbo_block(uint32_t d) {  // turbo.rs:52-58
    uint32_t b = 1;
    while (d % (b * 2) == 0 && b < 256) b *= 2;
    return b;
}
__host__ __device__ inline uint32_t turbo_row_bytes(uint32_t d) { return 2 * (d / turbo_block(d)) + d / 2; }

// x <- R x (signs then normalised block FWHT) or x <- R^T x, on a warp-owned shared row.
__device__ void rotate_row(float *x, uint32_t d, bool inverse, int lane) {
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

// quantize_rotated_4 (turbo.rs:141-164) of a rotated shared row into a reference row.
__device__ void encode_rotated_row(const float *y, uint32_t d, uint8_t *out, uint8_t *qtmp, int lane) {
    const uint32_t b = turbo_block(d), nb = d / b;
    float c[16], thr[15];
#pragma unroll
    for (int i = 0; i < 16; i++) c[i] = (float)c_levels[i] / 46.0f;
#pragma unroll
    for (int i = 0; i < 15; i++) thr[i] = __fmul_rn(0.5f, __fadd_rn(c[i], c[i + 1]));
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
                const float cq = c[qtmp[bi * b + j]];
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

// ---- KV append ----------------------------------------------------------------------------
// Encodes one warp-owned shared row x (hd values; turbo rotates it in place) into cache row dst.
__device__ void store_row(int type, float *x, uint32_t hd, uint8_t *dst, uint8_t *qtmp, int lane) {
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

// One warp per (token, kv head, k|v). Rows land at slot (pos0 + t) % slots.
__global__ void __launch_bounds__(128) k_kv_store(int type, const float *__restrict__ k, const float *__restrict__ v,
                                                  uint32_t n_tok, uint32_t n_kv, uint32_t hd, uint32_t slots,
                                                  uint64_t pos0, const uint64_t *__restrict__ pos_ptr, uint32_t row_bytes,
                                                  uint8_t *__restrict__ kc, uint8_t *__restrict__ vc) {
    pdl_wait();
    pdl_trigger();
    if (pos_ptr) pos0 = *pos_ptr;
    __shared__ float xs[4][kMaxHd];
    __shared__ uint8_t qs[4][kMaxHd];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint64_t item = (uint64_t)blockIdx.x * 4 + warp;
    if (item >= (uint64_t)n_tok * n_kv * 2) return;
    const uint32_t which = item & 1, h = (item >> 1) % n_kv, t = (uint32_t)((item >> 1) / n_kv);
    const float *src = (which ? v : k) + ((uint64_t)t * n_kv + h) * hd;
    const uint64_t slot = (pos0 + t) % slots;
    uint8_t *dst = (which ? vc : kc) + ((uint64_t)h * slots + slot) * row_bytes;
    float *x = xs[warp];
    for (uint32_t i = lane; i < hd; i += 32) x[i] = src[i];
    __syncwarp();
    store_row(type, x, hd, dst, qs[warp], lane);
}

// Per head vector of the fused QKV output, one warp each: bias, q/k RMSNorm (x *= scale*w),
// RoPE (ops.rs:65-99), then q heads are scaled by attn_scale and written back, while k and v
// heads go straight into the cache at slot (pos + t) % slots (cpu.rs:280-328).
// Vectors: [t][0..n_head) = q heads, [t][n_head..n_head+n_kv) = k heads, then v heads.
__global__ void __launch_bounds__(128) k_qkv_post_store(QkvPostParams p, int type, uint32_t n_kv, uint32_t slots,
                                                        uint32_t row_bytes, uint8_t *__restrict__ kc,
                                                        uint8_t *__restrict__ vc) {
    pdl_wait();
    pdl_trigger();
    __shared__ float buf[4][kMaxHd];
    __shared__ uint8_t qs[4][kMaxHd];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t hd = p.hd, per_tok = p.n_head + 2 * n_kv;
    const uint64_t item = (uint64_t)blockIdx.x * 4 + warp;
    if (item >= (uint64_t)p.n_tok * per_tok) return;
    const uint32_t t = (uint32_t)(item / per_tok), j = (uint32_t)(item % per_tok);
    const float *src, *bias, *norm;
    int kind;  // 0 q, 1 k, 2 v
    uint32_t h;
    if (j < p.n_head) {
        h = j, kind = 0, norm = p.qn;
        src = p.q + ((uint64_t)t * p.n_head + h) * hd, bias = p.bq ? p.bq + h * hd : nullptr;
    } else if (j < p.n_head + n_kv) {
        h = j - p.n_head, kind = 1, norm = p.kn;
        src = p.k + ((uint64_t)t * n_kv + h) * hd, bias = p.bk ? p.bk + h * hd : nullptr;
    } else {
        h = j - p.n_head - n_kv, kind = 2, norm = nullptr;
        src = p.v + ((uint64_t)t * n_kv + h) * hd, bias = p.bv ? p.bv + h * hd : nullptr;
    }
    float *x = buf[warp];
    for (uint32_t i = lane; i < hd; i += 32) x[i] = src[i] + (bias ? bias[i] : 0.0f);
    __syncwarp();
    if (norm) {
        float ss = 0.0f;
        for (uint32_t i = lane; i < hd; i += 32) ss += x[i] * x[i];
        for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float scale = 1.0f / sqrtf(ss / (float)hd + p.eps);
        for (uint32_t i = lane; i < hd; i += 32) x[i] *= scale * norm[i];
        __syncwarp();
    }
    const uint64_t pos = *p.pos_ptr + t;
    if (kind != 2) {
        const uint32_t half = p.rope_dim / 2;
        const float fpos = (float)pos;
        for (uint32_t i = lane; i < half; i += 32) {
            float sn, cs;
            sincosf(fpos * p.inv_freq[i], &sn, &cs);
            const uint32_t i0 = p.neox ? i : 2 * i, i1 = p.neox ? i + half : 2 * i + 1;
            const float a = x[i0], b = x[i1];
            x[i0] = a * cs - b * sn;
            x[i1] = a * sn + b * cs;
        }
        __syncwarp();
    }
    if (kind == 0) {
        float *dst = p.q + ((uint64_t)t * p.n_head + h) * hd;
        for (uint32_t i = lane; i < hd; i += 32) dst[i] = x[i] * p.attn_scale;
        return;
    }
    uint8_t *dst = (kind == 1 ? kc : vc) + ((uint64_t)h * slots + pos % slots) * row_bytes;
    store_row(type, x, hd, dst, qs[warp], lane);
}

// quantize_4 of arbitrary rows (turbo.rs:167-171), reference row layout out.
__global__ void __launch_bounds__(128) k_turbo_quantize(const float *__restrict__ x, uint32_t n_rows, uint32_t hd,
                                                        uint8_t *__restrict__ out) {
    __shared__ float xs[4][kMaxHd];
    __shared__ uint8_t qs[4][kMaxHd];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint64_t r = (uint64_t)blockIdx.x * 4 + warp;
    if (r >= n_rows) return;
    float *xr = xs[warp];
    for (uint32_t i = lane; i < hd; i += 32) xr[i] = x[r * hd + i];
    __syncwarp();
    rotate_row(xr, hd, false, lane);
    encode_rotated_row(xr, hd, out + r * turbo_row_bytes(hd), qs[warp], lane);
}

__global__ void __launch_bounds__(128) k_turbo_rotate(float *__restrict__ x, uint32_t n_rows, uint32_t hd, int inverse) {
    __shared__ float xs[4][kMaxHd];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint64_t r = (uint64_t)blockIdx.x * 4 + warp;
    if (r >= n_rows) return;
    float *xr = xs[warp];
    for (uint32_t i = lane; i < hd; i += 32) xr[i] = x[r * hd + i];
    __syncwarp();
    rotate_row(xr, hd, inverse != 0, lane);
    for (uint32_t i = lane; i < hd; i += 32) x[r * hd + i] = xr[i];
}

// ---- attention ----------------------------------------------------------------------------
constexpr int kAttnWarps = 4;
constexpr int kAttnThreads = kAttnWarps * 32;
constexpr int kMaxGroup = 16;
constexpr uint32_t kCombineMaxSplits = 256;  // split-plan cap (fused merge keeps weights in smem)
constexpr uint32_t kCombineMaxHeads = 8;
constexpr int kMaxAttnHd = 256;

struct AttnParams {
    const uint8_t *kc, *vc;
    const float *q;
    float *o_part, *m_part, *l_part;
    uint32_t n_tok, n_head, n_kv, hd, slots, window, n_split, rows_per_split, row_bytes;
    uint64_t pos0;
    const uint64_t *pos_ptr;  // when set, the position is read from device memory (graph replay)
    float softcap;
    int rounding;
};

// 4 nibble indices (one per byte, 0..15) -> 4 int8 levels, with byte permutes.
__device__ __forceinline__ uint32_t lut16(uint32_t idx, uint32_t t0, uint32_t t1, uint32_t t2, uint32_t t3) {
    const uint32_t sel = __byte_perm(idx | (idx >> 4), 0, 0x0020) & 0x7777u;
    const uint32_t lo = __byte_perm(t0, t1, sel), hi = __byte_perm(t2, t3, sel);
    const uint32_t m = ((idx & 0x08080808u) >> 3) * 0xffu;
    return (lo & ~m) | (hi & m);
}

// One CTA = (KV head g, query token t, split): scores rows [c0, c1) of the cache for the
// G query heads of the group in 64-row sub-chunks with an online softmax, and writes an
// un-normalised partial output with its running max / sum.
template <int KV, int G>
__global__ void __launch_bounds__(kAttnThreads) k_attn_partial(const __grid_constant__ AttnParams p) {
    pdl_wait();
    pdl_trigger();
    constexpr int SUB = 64, DPL = kMaxAttnHd / 32;
    const uint32_t g = blockIdx.x, t = blockIdx.y, split = blockIdx.z;
    const uint32_t hd = p.hd, dpl = hd / 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint64_t pt = (p.pos_ptr ? *p.pos_ptr : p.pos0) + t;
    const uint64_t start = p.window > 0 ? (pt + 1 > p.window ? pt + 1 - p.window : 0) : 0;
    const uint32_t len = (uint32_t)(pt + 1 - start);
    const uint32_t c0 = split * p.rows_per_split, c1 = min(len, c0 + p.rows_per_split);
    const uint64_t part_base = ((uint64_t)t * p.n_head + (uint64_t)g * G) * p.n_split + split;
    if (c0 >= len) {
        for (uint32_t hh = warp; hh < G; hh += kAttnWarps) {
            const uint64_t pb = part_base + (uint64_t)hh * p.n_split;
            if (lane == 0) {
                p.m_part[pb] = -INFINITY;
                p.l_part[pb] = 0.0f;
            }
            for (uint32_t d = lane; d < hd; d += 32) p.o_part[pb * hd + d] = 0.0f;
        }
        return;
    }
    __shared__ __align__(16) float qf[G][kMaxAttnHd];  // f32 query (f16 cache) / rotation scratch
    __shared__ __align__(16) int8_t qi[G][kMaxAttnHd];
    __shared__ float qd[G][kMaxAttnHd / 32];
    __shared__ float sc[G][SUB];
    __shared__ float red[kAttnWarps][kMaxAttnHd];
    __shared__ float mrun[G], lrun[G], alpha[G];

    // 1. queries of this group: rotate (turbo) and quantize to Q8_0 (turbo / Q8_0 caches)
    for (uint32_t hh = warp; hh < G; hh += kAttnWarps) {
        const float *qsrc = p.q + ((uint64_t)t * p.n_head + g * G + hh) * hd;
        for (uint32_t d = lane; d < hd; d += 32) qf[hh][d] = qsrc[d];
        __syncwarp();
        if (KV == RCU_KV_TURBO4) rotate_row(qf[hh], hd, false, lane);
        if (KV != RCU_KV_F16) {
            for (uint32_t b = 0; b < hd / 32; b++) {
                float d;
                const int q = quant32(qf[hh][b * 32 + lane], p.rounding, d);
                qi[hh][b * 32 + lane] = (int8_t)q;
                if (lane == 0) qd[hh][b] = d;
            }
        }
        if (lane == 0) {
            mrun[hh] = -INFINITY;
            lrun[hh] = 0.0f;
        }
        __syncwarp();
    }
    __syncthreads();

    const uint32_t tb[4] = {0xc6b6a182u, 0xfaeee2d5u, 0x2b1e1206u, 0x7e5f4a3au};  // c_levels as bytes
    const float inv46 = 1.0f / 46.0f;
    float acc[G][DPL];
#pragma unroll
    for (int hh = 0; hh < G; hh++)
#pragma unroll
        for (int e = 0; e < DPL; e++) acc[hh][e] = 0.0f;
    const uint32_t d0 = lane * dpl;

    for (uint32_t s0 = c0; s0 < c1; s0 += SUB) {
        const uint32_t s1 = min(c1, s0 + SUB);
        // 2. scores: two threads per row, each half of the head dimension
        {
            const uint32_t r = threadIdx.x >> 1, half = threadIdx.x & 1;
            const uint32_t i = s0 + r;
            float s[G];
#pragma unroll
            for (int hh = 0; hh < G; hh++) s[hh] = 0.0f;
            if (i < s1) {
                const uint64_t row = (uint64_t)g * p.slots + (start + i) % p.slots;
                const uint64_t kro = row * p.row_bytes;
                if (KV == RCU_KV_TURBO4) {
                    const uint32_t b = turbo_block(hd), nb = hd / b, nch = hd / 32;
                    for (uint32_t cc = half * (nch / 2); cc < (half + 1) * (nch / 2) + (half ? nch % 2 : 0); cc++) {
                        uint32_t sw[1];
                        ld_words<1>(p.kc, kro + 2 * ((cc * 32) / b), sw);
                        const float scale = f16_bits_to_f32(sw[0]);
                        uint32_t w[4];
                        ld_words<4>(p.kc, kro + 2 * nb + 16 * cc, w);
                        uint32_t lv[8];
#pragma unroll
                        for (int i2 = 0; i2 < 4; i2++) {
                            lv[i2] = lut16(w[i2] & 0x0F0F0F0Fu, tb[0], tb[1], tb[2], tb[3]);
                            lv[4 + i2] = lut16((w[i2] >> 4) & 0x0F0F0F0Fu, tb[0], tb[1], tb[2], tb[3]);
                        }
#pragma unroll
                        for (int hh = 0; hh < G; hh++) {
                            const uint4 *qv = reinterpret_cast<const uint4 *>(&qi[hh][cc * 32]);
                            const uint4 q0 = qv[0], q1 = qv[1];
                            int a0 = dp4a(lv[0], q0.x, 0), a1 = dp4a(lv[1], q0.y, 0);
                            a0 = dp4a(lv[2], q0.z, a0);
                            a1 = dp4a(lv[3], q0.w, a1);
                            a0 = dp4a(lv[4], q1.x, a0);
                            a1 = dp4a(lv[5], q1.y, a1);
                            a0 = dp4a(lv[6], q1.z, a0);
                            a1 = dp4a(lv[7], q1.w, a1);
                            s[hh] += scale * (qd[hh][cc] * (float)(a0 + a1));
                        }
                    }
                } else if (KV == RCU_KV_Q8_0) {
                    const uint32_t nbk = hd / 32;
                    for (uint32_t bi = half * (nbk / 2); bi < (half + 1) * (nbk / 2) + (half ? nbk % 2 : 0); bi++) {
                        BlkW w;
                        dec_q8_0(p.kc, kro + bi * 34, w);
#pragma unroll
                        for (int hh = 0; hh < G; hh++) {
                            const uint4 *qv = reinterpret_cast<const uint4 *>(&qi[hh][bi * 32]);
                            const uint4 q0 = qv[0], q1 = qv[1];
                            const uint32_t a[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
                            s[hh] += (w.d * qd[hh][bi]) * (float)blk_int<T_Q8_0>(w, a, 0);
                        }
                    }
                } else {
                    const uint4 *kh = reinterpret_cast<const uint4 *>(p.kc + kro) + half * (hd / 16);
                    for (uint32_t c = 0; c < hd / 16; c++) {  // 8 halves per 16-byte load
                        const uint4 raw = kh[c];
                        const __half2 *h2 = reinterpret_cast<const __half2 *>(&raw);
                        const uint32_t dbase = half * (hd / 2) + 8 * c;
#pragma unroll
                        for (int j = 0; j < 4; j++) {
                            const float2 kv = __half22float2(h2[j]);
#pragma unroll
                            for (int hh = 0; hh < G; hh++)
                                s[hh] += kv.x * qf[hh][dbase + 2 * j] + kv.y * qf[hh][dbase + 2 * j + 1];
                        }
                    }
                }
            }
#pragma unroll
            for (int hh = 0; hh < G; hh++) {
                float v = s[hh] + __shfl_xor_sync(0xffffffffu, s[hh], 1);
                if (KV == RCU_KV_TURBO4) v *= inv46;
                if (p.softcap > 0.0f) v = p.softcap * tanhf(v / p.softcap);
                if (half == 0 && r < SUB) sc[hh][r] = i < s1 ? v : -INFINITY;
            }
        }
        __syncthreads();
        // 3. online softmax per head
        for (uint32_t hh = warp; hh < G; hh += kAttnWarps) {
            const float v0 = sc[hh][lane], v1 = sc[hh][lane + 32];
            float m = fmaxf(v0, v1);
            for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            const float m_old = mrun[hh], m_new = fmaxf(m_old, m);
            const float e0 = v0 == -INFINITY ? 0.0f : expf(v0 - m_new), e1 = v1 == -INFINITY ? 0.0f : expf(v1 - m_new);
            sc[hh][lane] = e0;
            sc[hh][lane + 32] = e1;
            float l = e0 + e1;
            for (int o = 16; o; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
            if (lane == 0) {
                const float a = m_old == -INFINITY ? 0.0f : expf(m_old - m_new);
                alpha[hh] = a;
                lrun[hh] = lrun[hh] * a + l;
                mrun[hh] = m_new;
            }
        }
        __syncthreads();
        // 4. weighted V sum: warp w takes rows s0 + w (mod 4); lane owns dims lane*dpl..
#pragma unroll
        for (int hh = 0; hh < G; hh++) {
            const float a = alpha[hh];
#pragma unroll
            for (int e = 0; e < DPL; e++) acc[hh][e] *= a;
        }
        for (uint32_t i = s0 + warp; i < s1; i += kAttnWarps) {
            const uint64_t vro = ((uint64_t)g * p.slots + (start + i) % p.slots) * p.row_bytes;
            const uint8_t *vr = p.vc + vro;
            float val[DPL];
#pragma unroll
            for (int e = 0; e < DPL; e++) {
                if ((uint32_t)e >= dpl) break;
                const uint32_t dd = d0 + e;
                if (KV == RCU_KV_TURBO4) {
                    const uint32_t b = turbo_block(hd), nb = hd / b, c = dd / 32, m2 = dd % 32;
                    const uint32_t byte = vr[2 * nb + 16 * c + (m2 & 15)];
                    const uint32_t code = m2 < 16 ? (byte & 15) : (byte >> 4);
                    uint32_t sw[1];
                    ld_words<1>(p.vc, vro + 2 * (dd / b), sw);
                    val[e] = f16_bits_to_f32(sw[0]) * inv46 * (float)c_levels[code];
                } else if (KV == RCU_KV_Q8_0) {
                    const uint32_t bi = dd / 32;
                    uint32_t sw[1];
                    ld_words<1>(p.vc, vro + bi * 34, sw);
                    val[e] = f16_bits_to_f32(sw[0]) * (float)(int8_t)vr[bi * 34 + 2 + dd % 32];
                } else {
                    val[e] = __half2float(reinterpret_cast<const __half *>(vr)[dd]);
                }
            }
#pragma unroll
            for (int hh = 0; hh < G; hh++) {
                const float w = sc[hh][i - s0];
#pragma unroll
                for (int e = 0; e < DPL; e++)
                    if ((uint32_t)e < dpl) acc[hh][e] += w * val[e];
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int hh = 0; hh < G; hh++) {
#pragma unroll
        for (int e = 0; e < DPL; e++)
            if ((uint32_t)e < dpl) red[warp][d0 + e] = acc[hh][e];
        __syncthreads();
        for (uint32_t d = threadIdx.x; d < hd; d += kAttnThreads) {
            float o = 0.0f;
            for (int w = 0; w < kAttnWarps; w++) o += red[w][d];
            p.o_part[(part_base + (uint64_t)hh * p.n_split) * hd + d] = o;
        }
        __syncthreads();
    }
    if (threadIdx.x < G) {
        const uint64_t pb = part_base + (uint64_t)threadIdx.x * p.n_split;
        p.m_part[pb] = mrun[threadIdx.x];
        p.l_part[pb] = lrun[threadIdx.x];
    }
}

// Merge the chunks of one (token, head), normalise, rotate back (turbo).
template <int KV>
__global__ void __launch_bounds__(32) k_attn_combine(const __grid_constant__ AttnParams p, float *__restrict__ out) {
    pdl_wait();
    pdl_trigger();
    const uint32_t h = blockIdx.x, t = blockIdx.y, lane = threadIdx.x, hd = p.hd;
    const uint64_t base = ((uint64_t)t * p.n_head + h) * p.n_split;
    float M = -INFINITY;
    for (uint32_t s = 0; s < p.n_split; s++) M = fmaxf(M, p.m_part[base + s]);
    float L = 0.0f;
    for (uint32_t s = 0; s < p.n_split; s++) {
        const float m = p.m_part[base + s];
        if (m != -INFINITY) L += expf(m - M) * p.l_part[base + s];
    }
    const float invL = 1.0f / L;
    __shared__ float o[kMaxAttnHd];
    for (uint32_t d = lane; d < hd; d += 32) {
        float acc = 0.0f;
        for (uint32_t s = 0; s < p.n_split; s++) {
            const float m = p.m_part[base + s];
            if (m != -INFINITY) acc += expf(m - M) * p.o_part[(base + s) * hd + d];
        }
        o[d] = acc * invL;
    }
    __syncwarp();
    if (KV == RCU_KV_TURBO4) rotate_row(o, hd, true, lane);
    for (uint32_t d = lane; d < hd; d += 32) out[((uint64_t)t * p.n_head + h) * hd + d] = o[d];
}

static uint64_t kv_row_bytes(int type, uint64_t hd) {
    if (type == RCU_KV_F16) return 2 * hd;
    if (type == RCU_KV_Q8_0) return hd / 32 * 34;
    return turbo_row_bytes((uint32_t)hd);
}

struct Scratch {
    void *p = nullptr;
    size_t n = 0;
};
static int scratch_get(rcu_ctx *ctx, size_t bytes, void **out) {
    static Scratch s[64];
    Scratch &sc = s[ctx->device & 63];
    if (sc.n < bytes) {
        if (sc.p) {
            RCU_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
            cudaFree(sc.p);
            sc.p = nullptr;
            sc.n = 0;
        }
        RCU_CUDA_TRY(ctx, cudaMalloc(&sc.p, bytes));
        sc.n = bytes;
    }
    *out = sc.p;
    return RCU_OK;
}


int launch_qkv_post_store(rcu_ctx *ctx, rcu_kv *kv, const QkvPostParams &p) {
    if (p.hd != kv->hd) return set_err(ctx, RCU_ERR_INVALID, "qkv post: head_dim differs from the cache's");
    if (kv->type == RCU_KV_TURBO4) {
        if (int st = ensure_signs(ctx)) return st;
    }
    const uint64_t items = (uint64_t)p.n_tok * (p.n_head + 2 * kv->n_kv);
    RCU_CUDA_TRY(ctx, launch_k(ctx, (k_qkv_post_store), dim3((uint32_t)((items + 3) / 4)), dim3(128), 0, p, kv->type, (uint32_t)kv->n_kv, (uint32_t)kv->slots, (uint32_t)kv->row_bytes, kv->k, kv->v));
    RCU_CUDA_TRY(ctx, cudaGetLastError());
    return RCU_OK;
}

int launch_kv_store(rcu_ctx *ctx, rcu_kv *kv, const float *k, const float *v, uint64_t n_tok, uint64_t pos0,
                    const uint64_t *pos_ptr) {
    const uint64_t items = n_tok * kv->n_kv * 2;
    RCU_CUDA_TRY(ctx, launch_k(ctx, (k_kv_store), dim3((uint32_t)((items + 3) / 4)), dim3(128), 0, kv->type, k, v, (uint32_t)n_tok, (uint32_t)kv->n_kv, (uint32_t)kv->hd, (uint32_t)kv->slots, pos0, pos_ptr, (uint32_t)kv->row_bytes, kv->k, kv->v));
    RCU_CUDA_TRY(ctx, cudaGetLastError());
    return RCU_OK;
}

// Rows per CTA: a multiple of 64, chosen so that n_kv x n_tok x splits covers about two
// waves of SMs; both numbers depend only on (max_len, n_tok, n_kv), never on the position.
static void split_plan(uint64_t max_len, uint64_t n_tok, uint64_t n_kv, int num_sms, uint32_t *n_split,
                       uint32_t *rows_per_split) {
    const uint64_t n_sub = (max_len + 63) / 64;
    const uint64_t want = std::max<uint64_t>(1, (2 * (uint64_t)num_sms) / std::max<uint64_t>(1, n_kv * n_tok));
    const uint64_t splits = std::max<uint64_t>(1, std::min<uint64_t>(std::min(n_sub, want), kCombineMaxSplits));
    const uint64_t subs_per = (n_sub + splits - 1) / splits;
    *rows_per_split = (uint32_t)(subs_per * 64);
    *n_split = (uint32_t)((max_len + *rows_per_split - 1) / *rows_per_split);
}

uint32_t attention_max_splits(const rcu_kv *kv, uint64_t window) {
    const uint64_t max_len = window > 0 ? std::min<uint64_t>(window, kv->slots) : kv->slots;
    return (uint32_t)((max_len + 63) / 64);  // upper bound of any plan (64-row splits)
}

uint64_t attention_scratch_bytes(const rcu_kv *kv, uint64_t n_tok, uint64_t n_head, uint32_t n_split) {
    return n_tok * n_head * n_split * (kv->hd + 2) * sizeof(float);
}

// Merge of the splits fused with the activation quantization of the Wo matmul: one CTA per
// (token, run of hpc heads), one output value per thread (hpc * hd threads: whole Q8_0
// blocks, and whole Q8_K blocks when that format is asked for).
template <int KV>
__global__ void __launch_bounds__(1024) k_attn_combine_q(const __grid_constant__ AttnParams p, uint32_t hpc,
                                                         float *__restrict__ out, const ActOut ao) {
    pdl_wait();
    pdl_trigger();
    __shared__ float fac[kCombineMaxHeads][kCombineMaxSplits];
    __shared__ __align__(16) float ob[1024];
    __shared__ Q8kShared sh;
    const uint32_t t = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, hd = p.hd;
    const uint32_t h0 = blockIdx.x * hpc, nw = blockDim.x >> 5;
    // 1. per-head merge weights exp(m_s - M) / L
    for (uint32_t hh = warp; hh < hpc; hh += nw) {
        const uint64_t base = ((uint64_t)t * p.n_head + h0 + hh) * p.n_split;
        float M = -INFINITY;
        for (uint32_t s = lane; s < p.n_split; s += 32) M = fmaxf(M, p.m_part[base + s]);
        for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        float L = 0.0f;
        for (uint32_t s = lane; s < p.n_split; s += 32) {
            const float m = p.m_part[base + s];
            const float f = m == -INFINITY ? 0.0f : expf(m - M);
            fac[hh][s] = f;
            L += f * p.l_part[base + s];
        }
        for (int o = 16; o; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
        const float invL = 1.0f / L;
        for (uint32_t s = lane; s < p.n_split; s += 32) fac[hh][s] *= invL;
    }
    __syncthreads();
    // 2. one dimension per thread
    const uint32_t hh = tid / hd, d = tid % hd;
    const uint64_t base = ((uint64_t)t * p.n_head + h0 + hh) * p.n_split;
    float acc = 0.0f;
    for (uint32_t s = 0; s < p.n_split; s++) {
        const float f = fac[hh][s];
        if (f != 0.0f) acc += f * p.o_part[(base + s) * hd + d];
    }
    if (KV == RCU_KV_TURBO4) {
        ob[tid] = acc;
        __syncthreads();
        if (warp < hpc) rotate_row(ob + warp * hd, hd, true, lane);
        __syncthreads();
        acc = ob[tid];
    }
    const uint64_t row_k = (uint64_t)p.n_head * hd, col = (uint64_t)h0 * hd + tid;
    if (out) out[t * row_k + col] = acc;
    // 3. quantize (the CTA covers whole blocks)
    if (ao.fmt & RCU_ACT_Q8_0) q8_0_block(acc, (t * row_k + col) / QK, lane, ao);
    if (ao.fmt & RCU_ACT_Q8K) {
        const uint64_t g0 = (uint64_t)h0 * hd + QK_K * (warp / 8);
        q8_k_block(acc, tid % QK_K, warp & ~7u, (t * row_k + g0) / QK_K, true, ao, sh, 0);
    }
}

// Heads per CTA of the fused merge for this shape, or 0 when the fused kernel cannot cover it.
static uint32_t combine_heads(uint64_t n_head, uint64_t hd, uint32_t fmt) {
    uint32_t h = 1;
    if (fmt & RCU_ACT_Q8K) {
        while ((h * hd) % QK_K) h++;
    } else {
        while (2 * h * hd <= 256 && n_head % (2 * h) == 0) h *= 2;
    }
    if (h > kCombineMaxHeads || h * hd > 1024 || n_head % h) return 0;
    return h;
}

bool attention_fused_merge_ok(uint64_t n_head, uint64_t hd, uint32_t fmt) { return combine_heads(n_head, hd, fmt) != 0; }

template <int KV>
static int dispatch_group(rcu_ctx *ctx, const AttnParams &p, int group, dim3 grid, float *out, const ActOut *aq,
                          uint32_t hpc) {
    switch (group) {
        case 1: RCU_CUDA_TRY(ctx, launch_k(ctx, (k_attn_partial<KV, 1>), dim3(grid), dim3(kAttnThreads), 0, p)); break;
        case 2: RCU_CUDA_TRY(ctx, launch_k(ctx, (k_attn_partial<KV, 2>), dim3(grid), dim3(kAttnThreads), 0, p)); break;
        case 4: RCU_CUDA_TRY(ctx, launch_k(ctx, (k_attn_partial<KV, 4>), dim3(grid), dim3(kAttnThreads), 0, p)); break;
        case 8: RCU_CUDA_TRY(ctx, launch_k(ctx, (k_attn_partial<KV, 8>), dim3(grid), dim3(kAttnThreads), 0, p)); break;
        case 16: RCU_CUDA_TRY(ctx, launch_k(ctx, (k_attn_partial<KV, 16>), dim3(grid), dim3(kAttnThreads), 0, p)); break;
        default: return set_err(ctx, RCU_ERR_UNSUPPORTED, "attention: query heads per kv head must be 1, 2, 4, 8 or 16");
    }
    if (aq) {
        RCU_CUDA_TRY(ctx, launch_k(ctx, (k_attn_combine_q<KV>), dim3(dim3(p.n_head / hpc, p.n_tok)), dim3(hpc * p.hd), 0, p, hpc, out, *aq));
    } else {
        RCU_CUDA_TRY(ctx, launch_k(ctx, (k_attn_combine<KV>), dim3(dim3(p.n_head, p.n_tok)), dim3(32), 0, p, out));
    }
    return RCU_OK;
}

int launch_attention(rcu_ctx *ctx, const rcu_kv *kv, const float *q, uint64_t n_tok, uint64_t n_head, uint64_t pos0,
                     const uint64_t *pos_ptr, uint64_t window, float softcap, float *out, uint32_t n_split,
                     float *scratch, const ActOut *aq) {
    const uint64_t group = n_head / kv->n_kv;
    const uint32_t hpc = aq ? combine_heads(n_head, kv->hd, aq->fmt) : 0;
    if (aq && !hpc) return set_err(ctx, RCU_ERR_UNSUPPORTED, "attention: no fused merge for this head shape");
    if (group > kMaxGroup) return set_err(ctx, RCU_ERR_UNSUPPORTED, "attention: more than 16 query heads per kv head");
    AttnParams p{};
    p.kc = kv->k;
    p.vc = kv->v;
    p.q = q;
    p.n_tok = (uint32_t)n_tok;
    p.n_head = (uint32_t)n_head;
    p.n_kv = (uint32_t)kv->n_kv;
    p.hd = (uint32_t)kv->hd;
    p.slots = (uint32_t)kv->slots;
    p.window = (uint32_t)window;
    p.pos0 = pos0;
    p.pos_ptr = pos_ptr;
    p.softcap = softcap;
    p.rounding = ctx->rounding;
    p.row_bytes = (uint32_t)kv->row_bytes;
    // fixed plans (graph replay) cover the whole cache; otherwise the current length
    uint64_t max_len;
    if (n_split != 0) {
        max_len = window > 0 ? std::min<uint64_t>(window, kv->slots) : kv->slots;
    } else {
        const uint64_t last = pos0 + n_tok - 1;
        max_len = window > 0 ? std::min<uint64_t>(window, last + 1) : last + 1;
    }
    split_plan(max_len, n_tok, kv->n_kv, ctx->num_sms, &p.n_split, &p.rows_per_split);
    const uint64_t parts = n_tok * n_head * p.n_split;
    void *scr = scratch;
    if (!scr) {
        int st = scratch_get(ctx, parts * (kv->hd + 2) * sizeof(float), &scr);
        if (st) return st;
    }
    p.o_part = (float *)scr;
    p.m_part = p.o_part + parts * kv->hd;
    p.l_part = p.m_part + parts;
    dim3 grid((uint32_t)kv->n_kv, (uint32_t)n_tok, p.n_split);
    int st = RCU_OK;
    switch (kv->type) {
        case RCU_KV_F16: st = dispatch_group<RCU_KV_F16>(ctx, p, (int)group, grid, out, aq, hpc); break;
        case RCU_KV_Q8_0: st = dispatch_group<RCU_KV_Q8_0>(ctx, p, (int)group, grid, out, aq, hpc); break;
        default: st = dispatch_group<RCU_KV_TURBO4>(ctx, p, (int)group, grid, out, aq, hpc); break;
    }
    if (st) return st;
    RCU_CUDA_TRY(ctx, cudaGetLastError());
    return RCU_OK;
}

}  // namespace rcu

using namespace rcu;

extern "C" {

uint64_t rcu_turbo4_row_bytes(uint64_t hd) { return hd == 0 || hd % 32 ? 0 : turbo_row_bytes((uint32_t)hd); }

int32_t rcu_turbo4_quantize(rcu_ctx *ctx, const float *x_dev, uint64_t n_rows, uint64_t hd, uint8_t *rows_dev) {
    if (!ctx || !x_dev || !rows_dev) return set_err(ctx, RCU_ERR_INVALID, "null argument");
    if (hd == 0 || hd % 32 || hd > kMaxHd) return set_err(ctx, RCU_ERR_INVALID, "turbo4: hd must be a multiple of 32, <= 512");
    if (n_rows == 0) return RCU_OK;
    int st = ensure_signs(ctx);
    if (st) return st;
    k_turbo_quantize<<<(uint32_t)((n_rows + 3) / 4), 128, 0, ctx->stream>>>(x_dev, (uint32_t)n_rows, (uint32_t)hd, rows_dev);
    RCU_CUDA_TRY(ctx, cudaGetLastError());
    return RCU_OK;
}

int32_t rcu_turbo4_rotate(rcu_ctx *ctx, float *x_dev, uint64_t n_rows, uint64_t hd, int32_t inverse) {
    if (!ctx || !x_dev) return set_err(ctx, RCU_ERR_INVALID, "null argument");
    if (hd == 0 || hd > kMaxHd) return set_err(ctx, RCU_ERR_INVALID, "turbo4: hd <= 512");
    if (n_rows == 0) return RCU_OK;
    int st = ensure_signs(ctx);
    if (st) return st;
    k_turbo_rotate<<<(uint32_t)((n_rows + 3) / 4), 128, 0, ctx->stream>>>(x_dev, (uint32_t)n_rows, (uint32_t)hd, inverse);
    RCU_CUDA_TRY(ctx, cudaGetLastError());
    return RCU_OK;
}

int32_t rcu_kv_create(rcu_ctx *ctx, int32_t kv_type, uint64_t n_head_kv, uint64_t head_dim, uint64_t slots,
                      rcu_kv **out) {
    if (!ctx || !out) return set_err(ctx, RCU_ERR_INVALID, "null argument");
    *out = nullptr;
    if (kv_type < RCU_KV_F16 || kv_type > RCU_KV_TURBO4) return set_err(ctx, RCU_ERR_INVALID, "unknown kv type");
    if (n_head_kv == 0 || slots == 0 || head_dim == 0 || head_dim % 32 || head_dim > kMaxAttnHd)
        return set_err(ctx, RCU_ERR_INVALID, "kv: head_dim must be a multiple of 32 and <= 256");
    const uint64_t rb = kv_row_bytes(kv_type, head_dim), bytes = n_head_kv * slots * rb;
    rcu_kv *kv = new (std::nothrow) rcu_kv();
    if (!kv) return RCU_ERR_OOM;
    kv->ctx = ctx;
    kv->type = kv_type;
    kv->n_kv = n_head_kv;
    kv->hd = head_dim;
    kv->slots = slots;
    kv->row_bytes = rb;
    cudaError_t e = cudaMalloc(&kv->k, bytes + 256);
    if (e == cudaSuccess) e = cudaMalloc(&kv->v, bytes + 256);
    if (e == cudaSuccess) e = cudaMemsetAsync(kv->k, 0, bytes + 256, ctx->stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(kv->v, 0, bytes + 256, ctx->stream);
    if (e != cudaSuccess) {
        cudaFree(kv->k);
        cudaFree(kv->v);
        delete kv;
        return cuda_err(ctx, e, "kv alloc");
    }
    int st = ensure_signs(ctx);
    if (st) {
        rcu_kv_free(kv);
        return st;
    }
    *out = kv;
    return RCU_OK;
}

void rcu_kv_free(rcu_kv *kv) {
    if (!kv) return;
    cudaSetDevice(kv->ctx->device);
    cudaFree(kv->k);
    cudaFree(kv->v);
    delete kv;
}

int32_t rcu_kv_store(rcu_ctx *ctx, rcu_kv *kv, const float *k_dev, const float *v_dev, uint64_t n_tok, uint64_t pos0) {
    if (!ctx || !kv || !k_dev || !v_dev) return set_err(ctx, RCU_ERR_INVALID, "null argument");
    if (n_tok == 0) return RCU_OK;
    if (n_tok > kv->slots) return set_err(ctx, RCU_ERR_INVALID, "kv_store: more tokens than slots");
    return rcu::launch_kv_store(ctx, kv, k_dev, v_dev, n_tok, pos0, nullptr);
}

int32_t rcu_kv_export(rcu_ctx *ctx, const rcu_kv *kv, void *k_host, void *v_host) {
    if (!ctx || !kv) return set_err(ctx, RCU_ERR_INVALID, "null argument");
    const uint64_t bytes = kv->n_kv * kv->slots * kv->row_bytes;
    if (k_host) RCU_CUDA_TRY(ctx, cudaMemcpyAsync(k_host, kv->k, bytes, cudaMemcpyDeviceToHost, ctx->stream));
    if (v_host) RCU_CUDA_TRY(ctx, cudaMemcpyAsync(v_host, kv->v, bytes, cudaMemcpyDeviceToHost, ctx->stream));
    RCU_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    return RCU_OK;
}

int32_t rcu_kv_import(rcu_ctx *ctx, rcu_kv *kv, const void *k_host, const void *v_host) {
    if (!ctx || !kv) return set_err(ctx, RCU_ERR_INVALID, "null argument");
    const uint64_t bytes = kv->n_kv * kv->slots * kv->row_bytes;
    if (k_host) RCU_CUDA_TRY(ctx, cudaMemcpyAsync(kv->k, k_host, bytes, cudaMemcpyHostToDevice, ctx->stream));
    if (v_host) RCU_CUDA_TRY(ctx, cudaMemcpyAsync(kv->v, v_host, bytes, cudaMemcpyHostToDevice, ctx->stream));
    RCU_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    return RCU_OK;
}

int32_t rcu_attention(rcu_ctx *ctx, const rcu_kv *kv, const float *q_dev, uint64_t n_tok, uint64_t n_head,
                      uint64_t pos0, uint64_t window, float softcap, float *out_dev) {
    if (!ctx || !kv || !q_dev || !out_dev) return set_err(ctx, RCU_ERR_INVALID, "null argument");
    if (n_tok == 0) return set_err(ctx, RCU_ERR_RUNTIME, "empty batch");
    if (n_head % kv->n_kv) return set_err(ctx, RCU_ERR_INVALID, "n_head not divisible by n_head_kv");
    const uint64_t last = pos0 + n_tok - 1;
    const uint64_t max_len = window > 0 ? std::min<uint64_t>(window, last + 1) : last + 1;
    if (max_len > kv->slots) return set_err(ctx, RCU_ERR_RUNTIME, "context window full");
    return rcu::launch_attention(ctx, kv, q_dev, n_tok, n_head, pos0, nullptr, window, softcap, out_dev, 0, nullptr,
                                 nullptr);
}

}  // extern "C"
