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
#include "rcu_turbo.cuh"

struct rcu_kv {
    rcu_ctx *ctx = nullptr;
    int type = 0;
    uint64_t n_kv = 0, hd = 0, slots = 0, row_bytes = 0;
    uint8_t *k = nullptr, *v = nullptr;  // device, [kv_head][slot][row_bytes]
};

namespace rcu {

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
// Grid (tokens, ceil(vectors / 8)); the CTA computes its token's RoPE angles once (the same
// sincosf of pos * inv_freq[i] for every head) and its 8 warps take one vector each.
constexpr int kQkvWarps = 8;
__global__ void __launch_bounds__(kQkvWarps * 32) k_qkv_post_store(QkvPostParams p, int type, uint32_t n_kv,
                                                                   uint32_t slots, uint32_t row_bytes,
                                                                   uint8_t *__restrict__ kc, uint8_t *__restrict__ vc) {
    pdl_wait();
    pdl_trigger();
    __shared__ float buf[kQkvWarps][kMaxHd];
    __shared__ uint8_t qs[kQkvWarps][kMaxHd];
    __shared__ float rope_cs[2][kMaxHd / 2];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t hd = p.hd, per_tok = p.n_head + 2 * n_kv, t = blockIdx.x, half = p.rope_dim / 2;
    const uint64_t pos = *p.pos_ptr + t;
    {
        const float fpos = (float)pos;
        for (uint32_t i = threadIdx.x; i < half; i += kQkvWarps * 32) {
            float sn, cs;
            sincosf(fpos * p.inv_freq[i], &sn, &cs);
            rope_cs[0][i] = cs;
            rope_cs[1][i] = sn;
        }
    }
    __syncthreads();
    const uint32_t j = blockIdx.y * kQkvWarps + warp;
    if (j >= per_tok) return;
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
    if (kind != 2) {
        for (uint32_t i = lane; i < half; i += 32) {
            const float cs = rope_cs[0][i], sn = rope_cs[1][i];
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
constexpr int kAttnWarps = 8;
constexpr int kAttnThreads = kAttnWarps * 32;
constexpr int kMaxGroup = 16;
constexpr uint32_t kMaxSplits = 256;  // split-plan cap
constexpr int kMaxAttnHd = 256;
constexpr uint32_t kSub = 64;  // cache rows per sub-chunk staged in shared memory

struct AttnParams {
    const uint8_t *kc, *vc;
    const float *q;
    float *o_part, *m_part, *l_part;
    uint32_t *done;  // per (token, kv head): CTAs finished; the last one merges and resets it
    float *out;      // merged output [t][n_head * hd] (f32), may be null
    ActOut aq;       // quantization of the merged output for the Wo matmul (aq.fmt == 0: none)
    uint32_t n_tok, n_head, n_kv, hd, slots, window, n_split, rows_per_split, row_bytes, buf_bytes;
    uint64_t pos0;
    const uint64_t *pos_ptr;  // when set, the position is read from device memory (graph replay)
    float softcap;
    int rounding;
};

// Byte lookup of 16 entries (the turbo4 levels as int8) for 4 nibble indices at once.
__device__ __forceinline__ uint32_t lut16(uint32_t idx, uint32_t t0, uint32_t t1, uint32_t t2, uint32_t t3) {
    const uint32_t sel = __byte_perm(idx | (idx >> 4), 0, 0x0020) & 0x7777u;
    const uint32_t lo = __byte_perm(t0, t1, sel), hi = __byte_perm(t2, t3, sel);
    const uint32_t m = ((idx & 0x08080808u) >> 3) * 0xffu;
    return (lo & ~m) | (hi & m);
}

__device__ __forceinline__ void cp_async16(void *dst_smem, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst_smem)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Where the rows of one staged sub-chunk sit in its shared buffer: the ring of slots may wrap,
// so a sub-chunk is one or two contiguous byte ranges, each copied from its 16-byte aligned
// enclosure.
struct StagedRows {
    uint32_t n1, d1, d2;  // rows in the first range; byte offset of its first row; same for the second
    __device__ __forceinline__ uint32_t off(uint32_t r, uint32_t rb) const {
        return r < n1 ? d1 + r * rb : d2 + (r - n1) * rb;
    }
};
__device__ __forceinline__ StagedRows stage_rows(const uint8_t *cache, uint64_t head_base, uint32_t slots, uint32_t rb,
                                                 uint64_t first_slot, uint32_t n, uint8_t *buf) {
    StagedRows sr;
    const uint64_t room = slots - first_slot;
    sr.n1 = room < n ? (uint32_t)room : n;
    const uint64_t b1 = head_base + first_slot * rb, lo1 = b1 & ~15ull, hi1 = (b1 + (uint64_t)sr.n1 * rb + 15) & ~15ull;
    sr.d1 = (uint32_t)(b1 - lo1);
    for (uint32_t o = threadIdx.x * 16; o < hi1 - lo1; o += kAttnThreads * 16) cp_async16(buf + o, cache + lo1 + o);
    sr.d2 = (uint32_t)(hi1 - lo1);
    if (sr.n1 < n) {
        const uint64_t b2 = head_base, lo2 = b2 & ~15ull, hi2 = (b2 + (uint64_t)(n - sr.n1) * rb + 15) & ~15ull;
        uint8_t *buf2 = buf + sr.d2;
        sr.d2 += (uint32_t)(b2 - lo2);
        for (uint32_t o = threadIdx.x * 16; o < hi2 - lo2; o += kAttnThreads * 16) cp_async16(buf2 + o, cache + lo2 + o);
    }
    return sr;
}

// One CTA = (KV head g, query token t, split): the G query heads of the group against cache
// rows [c0, c1) in 64-row sub-chunks (K and V staged in shared memory by cp.async, the next
// sub-chunk in flight while the current one is scored), online softmax, un-normalised
// partial output. The last CTA of (t, g) to finish merges the splits (cpu.rs:590-634 softmax
// and weighted sum), applies the inverse rotation (turbo) and writes the f32 output and/or
// the quantized activations of the Wo matmul.
template <int KV, int G, int DPL>  // DPL: values per lane in the V sum (head_dim / 32, at most)
__global__ void __launch_bounds__(kAttnThreads) k_attn(const __grid_constant__ AttnParams p) {
    extern __shared__ __align__(16) uint8_t dsm[];
    __shared__ __align__(16) float qf[G][kMaxAttnHd];  // f32 query (f16 cache) / rotation scratch
    __shared__ __align__(16) int8_t qi[G][kMaxAttnHd];
    __shared__ float qd[G][kMaxAttnHd / 32];
    __shared__ float sc[G][kSub];
    __shared__ float red[kAttnWarps][kMaxAttnHd];
    __shared__ float mrun[G], lrun[G], alpha[G];
    __shared__ Q8kShared qsh;
    __shared__ uint32_t s_last;
    const uint32_t g = blockIdx.x, t = blockIdx.y, split = blockIdx.z;
    const uint32_t hd = p.hd, dpl = hd / 32, rb = p.row_bytes, tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const uint64_t pt = (p.pos_ptr ? *p.pos_ptr : p.pos0) + t;
    const uint64_t start = p.window > 0 ? (pt + 1 > p.window ? pt + 1 - p.window : 0) : 0;
    const uint32_t len = (uint32_t)(pt + 1 - start);
    const uint32_t c0 = split * p.rows_per_split, c1 = min(len, c0 + p.rows_per_split);
    const uint64_t part_base = ((uint64_t)t * p.n_head + (uint64_t)g * G) * p.n_split + split;
    const uint64_t head_base = (uint64_t)g * p.slots * rb;
    // buffers: K of even sub-chunks, K of odd ones, V even, V odd
    auto kbuf_of = [&](uint32_t b) { return dsm + b * p.buf_bytes; };
    auto vbuf_of = [&](uint32_t b) { return dsm + (2 + b) * p.buf_bytes; };

    // The first sub-chunk is staged before waiting for the previous kernel: its rows were
    // written by earlier steps, except the rows of this batch's own positions (written by the
    // kernel just before), which are copied again after the wait.
    const uint64_t pos_b = p.pos_ptr ? *p.pos_ptr : p.pos0;
    const uint32_t fresh0 = pos_b > start ? (uint32_t)(pos_b - start) : 0;  // first row of this batch
    StagedRows kr0{}, vr0{}, kr1{}, vr1{};
    if (c0 < len) {
        const uint32_t n = min(kSub, c1 - c0);
        kr0 = stage_rows(p.kc, head_base, p.slots, rb, (start + c0) % p.slots, n, kbuf_of(0));
        vr0 = stage_rows(p.vc, head_base, p.slots, rb, (start + c0) % p.slots, n, vbuf_of(0));
        cp_async_commit();
    }
    pdl_wait();
    pdl_trigger();
    if (c0 < len) {
        const uint32_t n0 = min(kSub, c1 - c0);
        if (c0 + n0 > fresh0) {  // re-copy this batch's rows (2-byte units: rows are 2-aligned)
            cp_async_wait<0>();
            __syncthreads();  // every thread's copies of the sub-chunk have landed
            const uint32_t r_first = fresh0 > c0 ? fresh0 - c0 : 0, hw = rb / 2;
            for (uint32_t u = tid; u < (n0 - r_first) * hw; u += kAttnThreads) {
                const uint32_t r = r_first + u / hw, h2 = u % hw;
                const uint64_t src = head_base + (uint64_t)((start + c0 + r) % p.slots) * rb + 2 * h2;
                *reinterpret_cast<uint16_t *>(kbuf_of(0) + kr0.off(r, rb) + 2 * h2) =
                    *reinterpret_cast<const uint16_t *>(p.kc + src);
                *reinterpret_cast<uint16_t *>(vbuf_of(0) + vr0.off(r, rb) + 2 * h2) =
                    *reinterpret_cast<const uint16_t *>(p.vc + src);
            }
        }
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
        const uint32_t tb[4] = {0xc6b6a182u, 0xfaeee2d5u, 0x2b1e1206u, 0x7e5f4a3au};  // c_levels as bytes
        const float inv46 = 1.0f / 46.0f;
        float acc[G][DPL];
#pragma unroll
        for (int hh = 0; hh < G; hh++)
#pragma unroll
            for (int e = 0; e < DPL; e++) acc[hh][e] = 0.0f;
        const uint32_t d0 = lane * dpl;
        // V-row byte offsets of this lane's codes and scale (turbo4: f16 scale per rotation
        // block, then Q4_0-ordered nibbles; Q8_0: 34-byte blocks)
        const uint32_t tbk = turbo_block(hd), tnb = hd / tbk;
        const bool v_hi = (d0 % 32) >= 16;
        const uint32_t v_code_off = KV == RCU_KV_TURBO4 ? 2 * tnb + 16 * (d0 / 32) + ((d0 % 32) & 15)
                                                         : 34 * (d0 / 32) + 2 + d0 % 32;
        const uint32_t v_scale_off = KV == RCU_KV_TURBO4 ? 2 * (d0 / tbk) : 34 * (d0 / 32);

        uint32_t sub = 0;
        for (uint32_t s0 = c0; s0 < c1; s0 += kSub, sub++) {
            const uint32_t s1 = min(c1, s0 + kSub), cur = sub & 1;
            if (s1 < c1) {  // prefetch the next sub-chunk into the other buffers
                const uint32_t n = min(kSub, c1 - s1);
                const StagedRows a = stage_rows(p.kc, head_base, p.slots, rb, (start + s1) % p.slots, n, kbuf_of(cur ^ 1));
                const StagedRows b = stage_rows(p.vc, head_base, p.slots, rb, (start + s1) % p.slots, n, vbuf_of(cur ^ 1));
                if (cur) {
                    kr0 = a;
                    vr0 = b;
                } else {
                    kr1 = a;
                    vr1 = b;
                }
                cp_async_commit();
                cp_async_wait<1>();
            } else {
                cp_async_wait<0>();
            }
            __syncthreads();
            const uint8_t *kbuf = kbuf_of(cur), *vbuf = vbuf_of(cur);
            const StagedRows krc = cur ? kr1 : kr0, vrc = cur ? vr1 : vr0;
            // 2. scores: four threads per row, each a quarter of the head dimension
            {
                const uint32_t r = tid >> 2, qq = tid & 3;
                float s[G];
#pragma unroll
                for (int hh = 0; hh < G; hh++) s[hh] = 0.0f;
                if (s0 + r < s1) {
                    const uint32_t ro = krc.off(r, rb);
                    if (KV == RCU_KV_TURBO4) {
                        for (uint32_t cc = qq; cc < hd / 32; cc += 4) {
                            const float scale =
                                f16_bits_to_f32(*reinterpret_cast<const uint16_t *>(kbuf + ro + 2 * ((cc * 32) / tbk)));
                            uint32_t w[4];
                            ld_words<4>(kbuf, ro + 2 * tnb + 16 * cc, w);
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
                        for (uint32_t bi = qq; bi < hd / 32; bi += 4) {
                            BlkW w;
                            dec_q8_0(kbuf, ro + bi * 34, w);
#pragma unroll
                            for (int hh = 0; hh < G; hh++) {
                                const uint4 *qv = reinterpret_cast<const uint4 *>(&qi[hh][bi * 32]);
                                const uint4 q0 = qv[0], q1 = qv[1];
                                const uint32_t av[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
                                s[hh] += (w.d * qd[hh][bi]) * (float)blk_int<T_Q8_0>(w, av, 0);
                            }
                        }
                    } else {
                        const uint4 *kh = reinterpret_cast<const uint4 *>(kbuf + ro);
                        const uint32_t per = hd / 32;  // 16-byte chunks (8 halves) per quarter
                        for (uint32_t c = 0; c < per; c++) {
                            const uint4 raw = kh[qq * per + c];
                            const __half2 *h2 = reinterpret_cast<const __half2 *>(&raw);
                            const uint32_t db = qq * (hd / 4) + 8 * c;
#pragma unroll
                            for (int j = 0; j < 4; j++) {
                                const float2 kv = __half22float2(h2[j]);
#pragma unroll
                                for (int hh = 0; hh < G; hh++)
                                    s[hh] += kv.x * qf[hh][db + 2 * j] + kv.y * qf[hh][db + 2 * j + 1];
                            }
                        }
                    }
                }
#pragma unroll
                for (int hh = 0; hh < G; hh++) {
                    float v = s[hh] + __shfl_xor_sync(0xffffffffu, s[hh], 1);
                    v += __shfl_xor_sync(0xffffffffu, v, 2);
                    if (KV == RCU_KV_TURBO4) v *= inv46;
                    if (p.softcap > 0.0f) v = p.softcap * tanhf(v / p.softcap);
                    if (qq == 0) sc[hh][r] = s0 + r < s1 ? v : -INFINITY;
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
            // 4. weighted V sum: warp w takes rows s0 + w (mod 8); lane owns dims lane*dpl..
#pragma unroll
            for (int hh = 0; hh < G; hh++) {
                const float a = alpha[hh];
#pragma unroll
                for (int e = 0; e < DPL; e++) acc[hh][e] *= a;
            }
#pragma unroll 2
            for (uint32_t i = s0 + warp; i < s1; i += kAttnWarps) {
                const uint32_t ro = vrc.off(i - s0, rb);
                float val[DPL];
                if (KV == RCU_KV_F16 && DPL >= 4) {
                    if (dpl == 4) {
                        const uint2 raw = *reinterpret_cast<const uint2 *>(vbuf + ro + 2 * d0);
                        const float2 a0 = __half22float2(*reinterpret_cast<const __half2 *>(&raw.x));
                        const float2 a1 = __half22float2(*reinterpret_cast<const __half2 *>(&raw.y));
                        val[0] = a0.x, val[1] = a0.y, val[2] = a1.x, val[3] = a1.y;
                    } else {
#pragma unroll
                        for (int e = 0; e < DPL; e++)
                            if ((uint32_t)e < dpl) val[e] = __half2float(reinterpret_cast<const __half *>(vbuf + ro)[d0 + e]);
                    }
                } else if (KV == RCU_KV_TURBO4 || KV == RCU_KV_Q8_0) {
                    // the lane's dpl values are consecutive codes of one 32-value chunk: one or
                    // two words, one f16 scale per row
                    uint32_t cw[2] = {0u, 0u};
                    if (dpl > 4)
                        ld_words<2>(vbuf, ro + v_code_off, cw);
                    else
                        ld_words<1>(vbuf, ro + v_code_off, *reinterpret_cast<uint32_t(*)[1]>(cw));
                    const float scale = f16_bits_to_f32(*reinterpret_cast<const uint16_t *>(vbuf + ro + v_scale_off)) *
                                        (KV == RCU_KV_TURBO4 ? inv46 : 1.0f);
                    if (KV == RCU_KV_TURBO4) {  // nibbles -> int8 levels (byte-shuffle lookup)
#pragma unroll
                        for (int w = 0; w < 2; w++)
                            cw[w] = lut16(v_hi ? (cw[w] >> 4) & 0x0F0F0F0Fu : cw[w] & 0x0F0F0F0Fu, tb[0], tb[1], tb[2], tb[3]);
                    }
#pragma unroll
                    for (int e = 0; e < DPL; e++)
                        if ((uint32_t)e < dpl) val[e] = scale * (float)sbyte(cw[e >> 2], e & 3);
                } else {
#pragma unroll
                    for (int e = 0; e < DPL; e++)
                        if ((uint32_t)e < dpl) val[e] = __half2float(reinterpret_cast<const __half *>(vbuf + ro)[d0 + e]);
                }
#pragma unroll
                for (int hh = 0; hh < G; hh++) {
                    const float w = sc[hh][i - s0];
#pragma unroll
                    for (int e = 0; e < DPL; e++)
                        if ((uint32_t)e < dpl) acc[hh][e] += w * val[e];
                }
            }
            __syncthreads();  // the buffers of this sub-chunk are refilled two iterations later
        }
#pragma unroll
        for (int hh = 0; hh < G; hh++) {
#pragma unroll
            for (int e = 0; e < DPL; e++)
                if ((uint32_t)e < dpl) red[warp][d0 + e] = acc[hh][e];
            __syncthreads();
            for (uint32_t d = tid; d < hd; d += kAttnThreads) {
                float o = 0.0f;
#pragma unroll
                for (int w = 0; w < kAttnWarps; w++) o += red[w][d];
                p.o_part[(part_base + (uint64_t)hh * p.n_split) * hd + d] = o;
            }
            __syncthreads();
        }
        if (tid < G) {
            const uint64_t pb = part_base + (uint64_t)tid * p.n_split;
            p.m_part[pb] = mrun[tid];
            p.l_part[pb] = lrun[tid];
        }
    } else {
        for (uint32_t hh = warp; hh < G; hh += kAttnWarps) {
            const uint64_t pb = part_base + (uint64_t)hh * p.n_split;
            if (lane == 0) {
                p.m_part[pb] = -INFINITY;
                p.l_part[pb] = 0.0f;
            }
            for (uint32_t d = lane; d < hd; d += 32) p.o_part[pb * hd + d] = 0.0f;
        }
    }

    // ---- merge: the last CTA of (t, g) ----------------------------------------------------
    __threadfence();
    __syncthreads();
    uint32_t *done = p.done + (uint64_t)t * p.n_kv + g;
    if (tid == 0) s_last = atomicAdd(done, 1u) == p.n_split - 1 ? 1u : 0u;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    float *fac = reinterpret_cast<float *>(dsm);  // [G][n_split]
    float *vals = fac + ((G * p.n_split + 3) & ~3u);  // [G][hd]
    const uint64_t base0 = ((uint64_t)t * p.n_head + (uint64_t)g * G) * p.n_split;
    for (uint32_t hh = warp; hh < G; hh += kAttnWarps) {
        const uint64_t base = base0 + (uint64_t)hh * p.n_split;
        float M = -INFINITY;
        for (uint32_t s = lane; s < p.n_split; s += 32) M = fmaxf(M, __ldcg(p.m_part + base + s));
        for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        float L = 0.0f;
        for (uint32_t s = lane; s < p.n_split; s += 32) {
            const float m = __ldcg(p.m_part + base + s);
            const float f = m == -INFINITY ? 0.0f : expf(m - M);
            fac[hh * p.n_split + s] = f;
            L += f * __ldcg(p.l_part + base + s);
        }
        for (int o = 16; o; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
        const float invL = 1.0f / L;
        __syncwarp();
        for (uint32_t s = lane; s < p.n_split; s += 32) fac[hh * p.n_split + s] *= invL;
    }
    __syncthreads();
    const uint32_t gv = G * hd;  // values of this group
    for (uint32_t v = tid; v < gv; v += kAttnThreads) {
        const uint32_t hh = v / hd, d = v % hd;
        const uint64_t base = base0 + (uint64_t)hh * p.n_split;
        const float *src = p.o_part + base * hd + d, *fh = fac + hh * p.n_split;
        float o = 0.0f;
        uint32_t s = 0;
        for (; s + 8 <= p.n_split; s += 8) {  // eight independent loads in flight
            float x[8];
#pragma unroll
            for (int j = 0; j < 8; j++) x[j] = __ldcg(src + (uint64_t)(s + j) * hd);
#pragma unroll
            for (int j = 0; j < 8; j++) o += fh[s + j] * x[j];
        }
        for (; s < p.n_split; s++) o += fh[s] * __ldcg(src + (uint64_t)s * hd);
        vals[v] = o;
    }
    __syncthreads();
    if (KV == RCU_KV_TURBO4) {
        for (uint32_t hh = warp; hh < G; hh += kAttnWarps) rotate_row(vals + hh * hd, hd, true, lane);
        __syncthreads();
    }
    const uint64_t row_k = (uint64_t)p.n_head * hd, col0 = (uint64_t)g * gv, row0 = (uint64_t)t * row_k + col0;
    if (p.out)
        for (uint32_t v = tid; v < gv; v += kAttnThreads) p.out[row0 + v] = vals[v];
    if (p.aq.fmt) {
        for (uint32_t v0 = 0; v0 < gv; v0 += kAttnThreads) {  // whole Q8_0 blocks; whole Q8_K blocks when asked
            const uint32_t v = v0 + tid;
            const float x = v < gv ? vals[v] : 0.0f;
            if ((p.aq.fmt & RCU_ACT_Q8_0) && v0 + 32 * warp < gv) q8_0_block(x, (row0 + v0 + 32 * warp) / QK, lane, p.aq);
            if (p.aq.fmt & RCU_ACT_Q8K) q8_k_block(x, tid, 0, (row0 + v0) / QK_K, v0 < gv, p.aq, qsh, (v0 / kAttnThreads) & 1);
        }
    }
    if (tid == 0) *done = 0u;
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
    if (p.rope_dim > p.hd || p.rope_dim % 2) return set_err(ctx, RCU_ERR_INVALID, "qkv post: rope_dim");
    const uint32_t per_tok = p.n_head + 2 * (uint32_t)kv->n_kv;
    RCU_CUDA_TRY(ctx, launch_k(ctx, (k_qkv_post_store), dim3(p.n_tok, (per_tok + kQkvWarps - 1) / kQkvWarps),
                               dim3(kQkvWarps * 32), 0, p, kv->type, (uint32_t)kv->n_kv, (uint32_t)kv->slots,
                               (uint32_t)kv->row_bytes, kv->k, kv->v));
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
    const uint64_t n_sub = (max_len + kSub - 1) / kSub;
    const uint64_t want = std::max<uint64_t>(1, (2 * (uint64_t)num_sms) / std::max<uint64_t>(1, n_kv * n_tok));
    const uint64_t splits = std::max<uint64_t>(1, std::min<uint64_t>(std::min(n_sub, want), kMaxSplits));
    const uint64_t subs_per = (n_sub + splits - 1) / splits;
    *rows_per_split = (uint32_t)(subs_per * kSub);
    *n_split = (uint32_t)((max_len + *rows_per_split - 1) / *rows_per_split);
}

uint32_t attention_max_splits(const rcu_kv *kv, uint64_t window) {
    const uint64_t max_len = window > 0 ? std::min<uint64_t>(window, kv->slots) : kv->slots;
    return (uint32_t)std::min<uint64_t>((max_len + kSub - 1) / kSub, kMaxSplits);  // bound of any plan
}

// Scratch: per (token, kv head) completion counters first (zeroed once, self-resetting),
// then the partial outputs, maxima and sums.
static uint64_t counters_bytes(uint64_t n_tok, uint64_t n_kv) { return (n_tok * n_kv * 4 + 255) & ~255ull; }
uint64_t attention_scratch_bytes(const rcu_kv *kv, uint64_t n_tok, uint64_t n_head, uint32_t n_split) {
    return counters_bytes(n_tok, kv->n_kv) + n_tok * n_head * n_split * (kv->hd + 2) * sizeof(float);
}

// Scratch for every batch of 1..max_batch tokens: a batch of n tokens splits the context into at
// most min(2 * SMs / (n_kv * n), 256) parts, so n * splits stays near max(max_batch, 2 * SMs / n_kv);
// single-token steps replayed as a graph use the fixed grid of attention_max_splits.
uint64_t attention_scratch_bytes_upto(const rcu_ctx *ctx, const rcu_kv *kv, uint64_t max_batch, uint64_t n_head,
                                      uint64_t window) {
    const uint64_t max_len = window > 0 ? std::min<uint64_t>(window, kv->slots) : kv->slots;
    uint64_t best = attention_scratch_bytes(kv, 1, n_head, attention_max_splits(kv, window));
    for (uint64_t n = 1; n <= max_batch; n++) {
        uint32_t ns = 0, rps = 0;
        split_plan(max_len, n, kv->n_kv, ctx->num_sms, &ns, &rps);
        best = std::max<uint64_t>(best, attention_scratch_bytes(kv, n, n_head, ns));
    }
    return best;
}

bool attention_fused_merge_ok(uint64_t n_head, uint64_t n_kv, uint64_t hd, uint32_t fmt) {
    const uint64_t gv = (n_head / n_kv) * hd;
    return (fmt & RCU_ACT_Q8K) ? gv % QK_K == 0 : gv % QK == 0;
}

template <int KV, int G, int DPL>
static int launch_group(rcu_ctx *ctx, const AttnParams &p, dim3 grid, uint32_t dyn) {
    static int max_dyn[64] = {};  // per device: opt-in limit minus the kernel's static shared memory
    int &md = max_dyn[ctx->device & 63];
    if (!md) {
        cudaFuncAttributes fa;
        RCU_CUDA_TRY(ctx, cudaFuncGetAttributes(&fa, k_attn<KV, G, DPL>));
        const int lim = (int)ctx->max_smem_optin - (int)fa.sharedSizeBytes;
        RCU_CUDA_TRY(ctx, cudaFuncSetAttribute(k_attn<KV, G, DPL>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim));
        md = lim;
    }
    if ((int)dyn > md) return set_err(ctx, RCU_ERR_UNSUPPORTED, "attention: cache rows too long for shared memory");
    RCU_CUDA_TRY(ctx, launch_k(ctx, (k_attn<KV, G, DPL>), grid, dim3(kAttnThreads), dyn, p));
    return RCU_OK;
}

template <int KV>
static int dispatch_group(rcu_ctx *ctx, const AttnParams &p, int group, dim3 grid, uint32_t dyn) {
    const bool wide = p.hd > 128;
    switch (group) {
        case 1: return wide ? launch_group<KV, 1, 8>(ctx, p, grid, dyn) : launch_group<KV, 1, 4>(ctx, p, grid, dyn);
        case 2: return wide ? launch_group<KV, 2, 8>(ctx, p, grid, dyn) : launch_group<KV, 2, 4>(ctx, p, grid, dyn);
        case 4: return wide ? launch_group<KV, 4, 8>(ctx, p, grid, dyn) : launch_group<KV, 4, 4>(ctx, p, grid, dyn);
        case 8: return wide ? launch_group<KV, 8, 8>(ctx, p, grid, dyn) : launch_group<KV, 8, 4>(ctx, p, grid, dyn);
        case 16: return wide ? launch_group<KV, 16, 8>(ctx, p, grid, dyn) : launch_group<KV, 16, 4>(ctx, p, grid, dyn);
        default: return set_err(ctx, RCU_ERR_UNSUPPORTED, "attention: query heads per kv head must be 1, 2, 4, 8 or 16");
    }
}

// Not for turbo4 caches: the new row's encode (sequential sums, as the reference) would sit on
// the path of the CTA holding the newest position (measured on the 70B shape: 59.7 vs 61.1
// tok/s), while the standalone kernel encodes all heads' rows in parallel.
// turbo4 caches fuse only with one or two KV heads: the CTA holding the newest position rotates
// and encodes its K / V rows on two of its warps before their tiles, which lengthens the launch by
// more than the standalone kernel costs when each CTA streams long splits (70B shape, 8 KV heads:
// 59.7 fused vs 61.2 tok/s) and by less when the splits are short (1 KV head: 179.7 vs 155.9).
bool attention_fuses_post(const rcu_kv *kv, uint64_t n_tok, uint64_t n_head) {
    if (kv->type == RCU_KV_TURBO4 && kv->n_kv > 2) return false;
    return n_tok == 1 && kv->n_kv > 0 && attention_dec_ok(kv->type, kv->hd, n_head / kv->n_kv);
}

int launch_attention(rcu_ctx *ctx, const rcu_kv *kv, const float *q, uint64_t n_tok, uint64_t n_head, uint64_t pos0,
                     const uint64_t *pos_ptr, uint64_t window, float softcap, float *out, uint32_t n_split,
                     float *scratch, const ActOut *aq, const QkvPostParams *post) {
    if (post && !attention_fuses_post(kv, n_tok, n_head))
        return set_err(ctx, RCU_ERR_INVALID, "attention: this shape does not fuse the q/k post-processing");
    const uint64_t group = n_head / kv->n_kv;
    if (group > kMaxGroup) return set_err(ctx, RCU_ERR_UNSUPPORTED, "attention: more than 16 query heads per kv head");
    if (aq && !attention_fused_merge_ok(n_head, kv->n_kv, kv->hd, aq->fmt))
        return set_err(ctx, RCU_ERR_UNSUPPORTED, "attention: group output does not hold whole activation blocks");
    if (n_split == 0 && attention_prefill_ok(kv->type, kv->hd, group, n_tok)) {
        // prompt batch: tensor-core kernel into f32 rows (out, else the scratch), then the
        // quantization for Wo when asked for
        float *o = out;
        if (!o) {
            if (scratch) {
                o = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(scratch) + counters_bytes(n_tok, kv->n_kv));
            } else {
                void *v = nullptr;
                if (int st = scratch_get(ctx, n_tok * n_head * kv->hd * sizeof(float), &v)) return st;
                o = reinterpret_cast<float *>(v);
            }
        }
        if (int st = launch_attention_prefill(ctx, kv->k, kv->v, kv->n_kv, kv->hd, kv->slots, q, n_tok, n_head, pos0,
                                              pos_ptr, window, softcap, o))
            return st;
        if (aq && aq->fmt) {
            ActsView v{};
            v.q0 = aq->q0, v.d0 = aq->d0, v.s0 = aq->s0, v.sum0 = aq->sum0;
            v.qk = aq->qk, v.dk = aq->dk, v.bsk = aq->bsk;
            v.n_tok = (uint32_t)n_tok, v.k = (uint32_t)(n_head * kv->hd), v.have = aq->fmt;
            return launch_quantize(ctx, v, o, (uint32_t)n_tok, (uint32_t)(n_head * kv->hd), aq->fmt);
        }
        return RCU_OK;
    }
    if (attention_dec_ok(kv->type, kv->hd, group)) {
        // head_dim 128, 4 or 8 query heads per KV head: warp-per-chunk kernel, splits merged in
        // a thread-block cluster (rcu_attn_dec.cu); fixed plans (graph replay) cover the whole cache
        const uint64_t cap = window > 0 ? std::min<uint64_t>(window, kv->slots) : kv->slots;
        const uint64_t last = pos0 + n_tok - 1;
        const uint64_t max_len = n_split != 0 ? cap : (window > 0 ? std::min<uint64_t>(window, last + 1) : last + 1);
        const uint64_t parts = n_tok * n_head * attention_dec_max_clusters(kv->type, max_len, n_tok, kv->n_kv, ctx->num_sms);
        uint8_t *scr = reinterpret_cast<uint8_t *>(scratch);
        if (!scr) {
            void *v = nullptr;
            if (int st = scratch_get(ctx, counters_bytes(n_tok, kv->n_kv) + parts * (kv->hd + 2) * sizeof(float), &v))
                return st;
            scr = reinterpret_cast<uint8_t *>(v);
            RCU_CUDA_TRY(ctx, cudaMemsetAsync(scr, 0, counters_bytes(n_tok, kv->n_kv), ctx->stream));
        }
        return launch_attention_dec(ctx, kv->k, kv->v, kv->type, kv->n_kv, kv->slots, kv->row_bytes, q, n_tok, n_head,
                                    pos0, pos_ptr, max_len, window, softcap, out, aq,
                                    reinterpret_cast<uint32_t *>(scr),
                                    reinterpret_cast<float *>(scr + counters_bytes(n_tok, kv->n_kv)), post);
    }
    AttnParams p{};
    p.kc = kv->k;
    p.vc = kv->v;
    p.q = q;
    p.out = out;
    if (aq) p.aq = *aq;
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
    p.buf_bytes = (uint32_t)((kSub * kv->row_bytes + 15) & ~15ull) + 64;
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
    uint8_t *scr = reinterpret_cast<uint8_t *>(scratch);
    if (!scr) {
        void *v = nullptr;
        int st = scratch_get(ctx, counters_bytes(n_tok, kv->n_kv) + parts * (kv->hd + 2) * sizeof(float), &v);
        if (st) return st;
        scr = reinterpret_cast<uint8_t *>(v);
        RCU_CUDA_TRY(ctx, cudaMemsetAsync(scr, 0, counters_bytes(n_tok, kv->n_kv), ctx->stream));
    }
    p.done = reinterpret_cast<uint32_t *>(scr);
    p.o_part = reinterpret_cast<float *>(scr + counters_bytes(n_tok, kv->n_kv));
    p.m_part = p.o_part + parts * kv->hd;
    p.l_part = p.m_part + parts;
    const uint64_t merge_bytes = 4 * (((group * p.n_split + 3) & ~3ull) + group * kv->hd);
    const uint32_t dyn = (uint32_t)std::max<uint64_t>(4ull * p.buf_bytes, merge_bytes);
    dim3 grid((uint32_t)kv->n_kv, (uint32_t)n_tok, p.n_split);
    switch (kv->type) {
        case RCU_KV_F16: return dispatch_group<RCU_KV_F16>(ctx, p, (int)group, grid, dyn);
        case RCU_KV_Q8_0: return dispatch_group<RCU_KV_Q8_0>(ctx, p, (int)group, grid, dyn);
        default: return dispatch_group<RCU_KV_TURBO4>(ctx, p, (int)group, grid, dyn);
    }
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
