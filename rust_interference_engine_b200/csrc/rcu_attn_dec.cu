// rcu_attn_dec.cu -- decode attention (one query row per token and head) over an f16, Q8_0 or
// turbo4 KV cache at head_dim 128, for GQA groups of 4 or 8 query heads per KV head.
// Replaces, for decode steps, the reference's attention (crates/rie-core/src/model/cpu.rs:552-634)
// with its turbo4 scoring and V accumulation in the rotated domain (turbo.rs:178-250).
//
// Why a second attention kernel: at decode the work per cache row is small (G x 128 MACs for
// the scores, as many for V) and the context of a decode step is short, so the general kernel's
// phases (scores, softmax and V sums separated by block-wide barriers, splits merged through
// global memory by the last CTA) leave it latency-bound (18 us per layer at 515 positions).
// Common to both kernels here:
//   * a producer warp bulk-copies the split's K and V rows into a ring of shared-memory stages;
//     the consumer warps take chunks of the stage with no block-wide barrier;
//   * online softmax per head in registers;
//   * the splits of a KV head (up to 8 CTAs) form a thread-block cluster and merge through
//     distributed shared memory; only contexts split over more than one cluster merge the
//     clusters through global memory (last cluster, counter per token and KV head);
//   * the merged rows are rotated back (turbo4) and written as f32 and / or quantized for the
//     Wo matmul in the same kernel.
// k_attn_dec (f16, Q8_0): a warp takes R = 32 / G rows; lane l holds dims 4l..4l+3 of each and
// the query of those dims for all G heads; the R x G partial scores are summed over the lanes by
// a transposing butterfly (31 shuffles for 32 sums), whose first three stages add the exact int32
// dp4a partials of a Q8_0 block's 8 lanes before its scales are applied.
// k_attn_dec_t4 (turbo4): the tensor-core kernel described above it.
// Every per-block integer sum is the reference's exactly; scores and sums are f32 as in the
// reference, in another order (and, for turbo4, with the V weights as an f16 pair, 22 bits).
#include <cooperative_groups.h>

#include "rcu_actq.cuh"
#include "rcu_blocks.cuh"
#include "rcu_kernels.h"
#include "rcu_turbo.cuh"

namespace cg = cooperative_groups;

namespace rcu {
namespace {

constexpr int kDW = 8;  // consumer warps per CTA (warp kDW copies the cache rows)
constexpr int kDThreads = (kDW + 1) * 32;
constexpr int kDMaxStages = 4;
constexpr int kDHd = 128;
constexpr int kDMaxCluster = 8;

struct DecParams {
    const uint8_t *kc, *vc;
    const float *q;
    float *o_part, *m_part, *l_part;  // per (token, query head, cluster) partials: more than one cluster
    uint32_t *done;                   // per (token, kv head): clusters finished (self-resetting)
    float *out;                       // [t][n_head * 128] f32, may be null
    ActOut aq;                        // quantization for the Wo matmul (aq.fmt == 0: none)
    uint32_t n_head, n_kv, slots, window, n_split, cs, rows_per_split, row_bytes;
    uint32_t stage_rows, n_stages, buf_bytes;  // rows per stage; stages; bytes of one K (or V) buffer
    uint32_t *err;
    uint64_t pos0;
    const uint64_t *pos_ptr;
    float softcap;
    int rounding;
    // decode with the q/k post-processing fused in (post != 0): q holds the raw query heads of
    // the QKV matmul, kraw / vraw its key / value heads; each CTA prepares its group's queries and
    // the CTA holding the newest position writes that position's K and V rows into the cache
    int post;
    const float *kraw, *vraw, *bq, *bk, *bv, *qn, *kn, *inv_freq;
    uint32_t rope_dim;
    int neox;
    float eps, attn_scale;
};

// Lane bit -> score index bit of the transposing butterfly (stages at lane offsets 4, 2, 1,
// 16, 8 decide score index bits 4, 3, 2, 1, 0): the (row, head) index k = row * G + head a
// lane holds at the end.
__device__ __forceinline__ uint32_t lane_k(uint32_t l) {
    return ((l >> 2) & 1u) << 4 | ((l >> 1) & 1u) << 3 | (l & 1u) << 2 | ((l >> 4) & 1u) << 1 | ((l >> 3) & 1u);
}

// One butterfly stage: N values -> N / 2, keeping the half selected by the lane's bit `o`.
template <int N, typename T>
__device__ __forceinline__ void bfly(T (&v)[32], uint32_t lane, int o) {
    const bool up = (lane & (uint32_t)o) != 0;
#pragma unroll
    for (int j = 0; j < N / 2; j++) {
        const T send = up ? v[j] : v[j + N / 2];
        const T keep = up ? v[j + N / 2] : v[j];
        v[j] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
}

// The 4 values of dims 4l..4l+3 of one cache row: K as exact codes (Q8_0) or f32, V as f32
// (the block's scale applied).
template <int KV>
struct Quad {
    uint32_t codes;  // Q8_0 int8 codes
    float f[4];      // f16 values / V values
    float scale;     // Q8_0: d of the lane's block
};

__device__ __forceinline__ uint32_t lds_u32_2a(const uint8_t *p) {  // 4 bytes at a 2-byte aligned shared address
    const uint16_t *h = reinterpret_cast<const uint16_t *>(p);
    return (uint32_t)h[0] | ((uint32_t)h[1] << 16);
}

template <int KV>
__device__ __forceinline__ void load_quad(const uint8_t *row, uint32_t lane, bool is_v, Quad<KV> &qd) {
    if (KV == RCU_KV_F16) {
        const uint2 raw = *reinterpret_cast<const uint2 *>(row + 8 * lane);
        const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&raw.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&raw.y));
        qd.f[0] = a.x, qd.f[1] = a.y, qd.f[2] = b.x, qd.f[3] = b.y;
    } else if (KV == RCU_KV_Q8_0) {  // 34-byte blocks: f16 d, 32 codes
        const uint32_t b = lane >> 3, o = 34 * b;
        qd.scale = f16_bits_to_f32(*reinterpret_cast<const uint16_t *>(row + o));
        qd.codes = lds_u32_2a(row + o + 2 + 4 * (lane & 7));
        if (is_v)
#pragma unroll
            for (int j = 0; j < 4; j++) qd.f[j] = qd.scale * (float)sbyte(qd.codes, j);
    }
}

// Rows [first_slot, first_slot + n) of one KV head's ring as a stage holds them: the ring may
// wrap, so one or two contiguous ranges, each copied from its 16-byte aligned enclosure.
struct Runs {
    uint64_t lo1, lo2;        // source byte offsets (from the cache base) of the copies
    uint32_t len1, len2;      // copy sizes (multiples of 16; len2 = 0: no second range)
    uint32_t n1, d1, d2;      // rows in the first range; stage offset of its first row; of the second's
};
// The ring slot SR rows after `slot` (no 64-bit modulo per stage).
__device__ __forceinline__ uint32_t next_slot(uint32_t slot, uint32_t SR, uint32_t slots) {
    slot += SR;
    while (slot >= slots) slot -= slots;
    return slot;
}
// What a consumer needs of a stage's Runs: where row r starts in the stage buffer.
struct RowMap {
    uint32_t n1, d1, d2;
    __device__ __forceinline__ uint32_t off(uint32_t r, uint32_t rb) const {
        return r < n1 ? d1 + r * rb : d2 + (r - n1) * rb;
    }
};
__device__ __forceinline__ Runs plan_runs(uint64_t head_base, uint32_t slots, uint32_t rb, uint64_t first_slot,
                                          uint32_t n) {
    Runs r;
    const uint64_t room = slots - first_slot;
    r.n1 = room < n ? (uint32_t)room : n;
    const uint64_t b1 = head_base + first_slot * rb, lo1 = b1 & ~15ull, hi1 = (b1 + (uint64_t)r.n1 * rb + 15) & ~15ull;
    r.lo1 = lo1;
    r.len1 = (uint32_t)(hi1 - lo1);
    r.d1 = (uint32_t)(b1 - lo1);
    r.lo2 = 0;
    r.len2 = 0;
    r.d2 = r.len1;
    if (r.n1 < n) {
        const uint64_t b2 = head_base, lo2 = b2 & ~15ull, hi2 = (b2 + (uint64_t)(n - r.n1) * rb + 15) & ~15ull;
        r.lo2 = lo2;
        r.len2 = (uint32_t)(hi2 - lo2);
        r.d2 += (uint32_t)(b2 - lo2);
    }
    return r;
}


// The producer warp's lane 0: bulk copies of the split's K and V rows, stage by stage, into the
// ring of n_stages buffers (full[s] completes with the bytes; empty[s] when every consumer warp
// has read the stage), and each stage's row map in maps[s]. Rows of earlier positions were
// written at least two launches back; this step's rows (logical index >= fresh) by the kernel
// just before (wait for it), or, with the fused post-processing, by this CTA (wait on newrow).
__device__ __forceinline__ void dec_produce(const DecParams &p, uint8_t *dsm, uint64_t *full, uint64_t *empty,
                                            RowMap *maps, uint64_t *newrow, uint32_t c0, uint32_t c1,
                                            uint32_t n_stage, uint64_t start, uint64_t pos_b, uint64_t head_base) {
    const uint32_t rb = p.row_bytes, SR = p.stage_rows, NS = p.n_stages, BB = p.buf_bytes;
    const uint32_t fresh = pos_b > start ? (uint32_t)(pos_b - start) : 0;
    bool waited = false;
    const uint64_t pol = policy_evict_first();
    uint32_t j = 0;
    uint32_t slot = (uint32_t)((start + c0) % p.slots);  // ring slot of the stage's first row
    for (; j < n_stage; j++) {
        const uint32_t s = j % NS;
        if (j >= NS && !mbar_wait_bounded(&empty[s], ((j / NS) - 1) & 1u, p.err, ERR_TIMEOUT_EMPTY)) break;
        const uint32_t ra = c0 + j * SR, n = min(SR, c1 - ra);
        if (!waited && ra + n > fresh) {
            if (p.post) {  // this CTA's consumers write the newest row (fused q/k post-processing)
                if (!mbar_wait_bounded(newrow, 0, p.err, ERR_TIMEOUT_FULL)) break;
                fence_proxy_async_global();
            } else {
                pdl_wait();
            }
            waited = true;
        }
        const Runs r = plan_runs(head_base, p.slots, rb, slot, n);
        slot = next_slot(slot, SR, p.slots);
        maps[s] = RowMap{r.n1, r.d1, r.d2};  // ordered before the stage's completion by the arrive below
        uint8_t *kb = dsm + (size_t)s * 2 * BB, *vb = kb + BB;
        mbar_arrive_expect_tx(&full[s], 2 * (r.len1 + r.len2));
        bulk_g2s(kb, p.kc + r.lo1, r.len1, &full[s], pol);
        bulk_g2s(vb, p.vc + r.lo1, r.len1, &full[s], pol);
        if (r.len2) {
            bulk_g2s(kb + r.len1, p.kc + r.lo2, r.len2, &full[s], pol);
            bulk_g2s(vb + r.len1, p.vc + r.lo2, r.len2, &full[s], pol);
        }
    }
    // never leave the CTA with copies in flight
    for (uint32_t st = 0; st < NS && st < j; st++) {
        const uint32_t last = ((j - 1 - st) / NS) * NS + st;
        mbar_wait_bounded(&full[st], (last / NS) & 1u, p.err, ERR_TIMEOUT_DRAIN);
    }
}

// The group's queries: f32 (f16 cache) or rotated (turbo4) and quantized to Q8_0 blocks.
template <int KV, int G>
__device__ __forceinline__ void dec_query(const DecParams &p, float (*qf)[kDHd], int8_t (*qi)[kDHd],
                                          float (*qds)[kDHd / 32], uint32_t t, uint32_t g, uint32_t warp,
                                          uint32_t lane) {
    for (uint32_t hh = warp; hh < (uint32_t)G; hh += kDW) {
        const uint64_t head = (uint64_t)g * G + hh;
        const float *qsrc = p.q + ((uint64_t)t * p.n_head + head) * kDHd;
        *reinterpret_cast<float4 *>(&qf[hh][4 * lane]) = *reinterpret_cast<const float4 *>(qsrc + 4 * lane);
        __syncwarp();
        if (p.post) {  // bias, q norm, RoPE and attn_scale (the standalone post-processing's arithmetic)
            const uint64_t pos = (p.pos_ptr ? *p.pos_ptr : p.pos0) + t;
            if (p.bq)
                for (uint32_t i = lane; i < kDHd; i += 32) qf[hh][i] = qf[hh][i] + p.bq[head * kDHd + i];
            __syncwarp();
            qk_post_vec(qf[hh], kDHd, p.qn, p.eps, true, p.inv_freq, pos, p.rope_dim, p.neox, (int)lane);
            for (uint32_t i = lane; i < kDHd; i += 32) qf[hh][i] = qf[hh][i] * p.attn_scale;
            __syncwarp();
        }
        if (KV == RCU_KV_TURBO4) rotate_row(qf[hh], kDHd, false, (int)lane);
        if (KV != RCU_KV_F16) {
#pragma unroll
            for (uint32_t b = 0; b < kDHd / 32; b++) {
                float d;
                const int qv = quant32(qf[hh][b * 32 + lane], p.rounding, d);
                qi[hh][b * 32 + lane] = (int8_t)qv;
                if (lane == 0) qds[hh][b] = d;
            }
        }
        __syncwarp();
    }
}

// The fused post-processing's K (which = 0) or V (1) row of the newest position for KV head g,
// one warp each: bias, and on the key k norm and RoPE, then encoded into the cache as the
// standalone kernel does; the writes are ordered before the producer's bulk copies (proxy
// fence, then an arrival on newrow, which completes with both rows).
template <int KV>
__device__ void dec_new_row(const DecParams &p, int which, uint32_t g, uint64_t pos, float *x, uint8_t *qtmp,
                            uint64_t *newrow, uint32_t lane) {
    const uint64_t slot = pos % p.slots;
    const float *src = (which ? p.vraw : p.kraw) + (uint64_t)g * kDHd;
    const float *bias = which ? p.bv : p.bk;
    for (uint32_t i = lane; i < kDHd; i += 32) x[i] = src[i] + (bias ? bias[(uint64_t)g * kDHd + i] : 0.0f);
    __syncwarp();
    if (!which) qk_post_vec(x, kDHd, p.kn, p.eps, true, p.inv_freq, pos, p.rope_dim, p.neox, (int)lane);
    uint8_t *dst = const_cast<uint8_t *>(which ? p.vc : p.kc) + ((uint64_t)g * p.slots + slot) * p.row_bytes;
    store_row(KV, x, kDHd, dst, qtmp, (int)lane);
    fence_proxy_async_global();
    __syncwarp();
    if (lane == 0) mbar_arrive(newrow);
}

// The split's partial rows (one per consumer warp: running max in natural-log units, sum of
// weights, weighted rows in wo = the stage buffers) merged into the CTA's, the cluster's (pushed
// into rank 0 through distributed shared memory) and, for contexts split over more than one
// cluster, the head's (through global memory, by the last cluster); then normalised, rotated back
// (turbo4) and written as f32 rows and / or the Wo matmul's quantized activations.
template <int KV, int G>
__device__ void dec_finish(const DecParams &p, uint8_t *dsm, float (*wm)[G], float (*wl)[G], uint32_t split,
                           uint32_t g, uint32_t t) {
    // partials of the cluster's CTAs, pushed into rank 0 with remote stores: [rank][G * 128 + 2G]
    __shared__ __align__(16) float cpart[kDMaxCluster][G * kDHd + 2 * G];
    __shared__ Q8kShared qsh;
    __shared__ uint32_t s_last;
    cg::cluster_group cluster = cg::this_cluster();
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t rank = cluster.block_rank();
    float(*wo)[G][kDHd] = reinterpret_cast<float(*)[G][kDHd]>(dsm);
    float *slot = cluster.map_shared_rank(&cpart[0][0], 0) + (size_t)rank * (G * kDHd + 2 * G);
    for (uint32_t e = tid; e < (uint32_t)G * kDHd; e += kDW * 32) {
        const uint32_t h = e / kDHd, d = e % kDHd;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kDW; w++) M = fmaxf(M, wm[w][h]);
        float o = 0.0f, L = 0.0f;
#pragma unroll
        for (int w = 0; w < kDW; w++) {
            const float f = wm[w][h] == -INFINITY ? 0.0f : __expf(wm[w][h] - M);
            o = fmaf(f, wo[w][h][d], o);
            L = fmaf(f, wl[w][h], L);
        }
        slot[e] = o;
        if (d == 0) {
            slot[G * kDHd + h] = M;
            slot[G * kDHd + G + h] = L;
        }
    }
    cluster.sync();  // every CTA's partial is in rank 0's shared memory
    const uint32_t cs = p.cs;
    float *vals = reinterpret_cast<float *>(dsm);  // [G][128] merged rows of the cluster (rank 0)
    __shared__ float fm[G], fl[G];
    if (rank != 0) return;
    for (uint32_t e = tid; e < (uint32_t)G * kDHd; e += kDW * 32) {
        const uint32_t h = e / kDHd;
        float mr[kDMaxCluster], M = -INFINITY;
#pragma unroll
        for (int r = 0; r < kDMaxCluster; r++) {
            mr[r] = (uint32_t)r < cs ? cpart[r][G * kDHd + h] : -INFINITY;
            M = fmaxf(M, mr[r]);
        }
        float o = 0.0f, L = 0.0f;
#pragma unroll
        for (int r = 0; r < kDMaxCluster; r++) {
            if ((uint32_t)r < cs) {
                const float f = mr[r] == -INFINITY ? 0.0f : __expf(mr[r] - M);
                o = fmaf(f, cpart[r][e], o);
                L = fmaf(f, cpart[r][G * kDHd + G + h], L);
            }
        }
        vals[e] = o;
        if ((e % kDHd) == 0) {
            fm[h] = M;
            fl[h] = L;
        }
    }
    named_bar_sync(1, kDW * 32);
    const uint32_t n_cl = p.n_split / cs, cl_id = split / cs;
    if (n_cl > 1) {  // more than one cluster: partials through global memory, the last cluster merges
        const uint64_t base = ((uint64_t)t * p.n_head + (uint64_t)g * G) * n_cl;
        for (uint32_t e = tid; e < (uint32_t)G * kDHd; e += kDW * 32) {
            const uint32_t h = e / kDHd, d = e % kDHd;
            p.o_part[(base + (uint64_t)h * n_cl + cl_id) * kDHd + d] = vals[e];
        }
        if (tid < (uint32_t)G) {
            p.m_part[base + (uint64_t)tid * n_cl + cl_id] = fm[tid];
            p.l_part[base + (uint64_t)tid * n_cl + cl_id] = fl[tid];
        }
        __threadfence();
        named_bar_sync(1, kDW * 32);
        uint32_t *done = p.done + (uint64_t)t * p.n_kv + g;
        if (tid == 0) s_last = atomicAdd(done, 1u) == n_cl - 1 ? 1u : 0u;
        named_bar_sync(1, kDW * 32);
        if (!s_last) return;
        __threadfence();
        // the clusters' weights per head, one warp per head: f[h][c] = exp(m_c - M), L = sum f l
        float *fw = vals + G * kDHd;  // [G][n_cl], after the merged rows in the stage buffers
        for (uint32_t h = warp; h < (uint32_t)G; h += kDW) {
            const uint64_t bh = base + (uint64_t)h * n_cl;
            float M = -INFINITY;
            for (uint32_t c = lane; c < n_cl; c += 32) M = fmaxf(M, __ldcg(p.m_part + bh + c));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
            float L = 0.0f;
            for (uint32_t c = lane; c < n_cl; c += 32) {
                const float m = __ldcg(p.m_part + bh + c);
                const float f = m == -INFINITY ? 0.0f : __expf(m - M);
                fw[h * n_cl + c] = f;
                L = fmaf(f, __ldcg(p.l_part + bh + c), L);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
            if (lane == 0) fl[h] = L;
        }
        named_bar_sync(1, kDW * 32);
        for (uint32_t e = tid; e < (uint32_t)G * kDHd; e += kDW * 32) {
            const uint32_t h = e / kDHd, d = e % kDHd;
            const float *op = p.o_part + (base + (uint64_t)h * n_cl) * kDHd + d;
            const float *f = fw + h * n_cl;
            float o0 = 0.0f, o1 = 0.0f, o2 = 0.0f, o3 = 0.0f;  // four chains: the loads overlap
            uint32_t c = 0;
            for (; c + 4 <= n_cl; c += 4) {
                o0 = fmaf(f[c], __ldcg(op + (uint64_t)c * kDHd), o0);
                o1 = fmaf(f[c + 1], __ldcg(op + (uint64_t)(c + 1) * kDHd), o1);
                o2 = fmaf(f[c + 2], __ldcg(op + (uint64_t)(c + 2) * kDHd), o2);
                o3 = fmaf(f[c + 3], __ldcg(op + (uint64_t)(c + 3) * kDHd), o3);
            }
            for (; c < n_cl; c++) o0 = fmaf(f[c], __ldcg(op + (uint64_t)c * kDHd), o0);
            vals[e] = (o0 + o1) + (o2 + o3);
        }
        named_bar_sync(1, kDW * 32);
        if (tid == 0) *done = 0u;
    }
    // 6. normalise, rotate back (turbo4), write f32 rows and / or the Wo activations
    for (uint32_t e = tid; e < (uint32_t)G * kDHd; e += kDW * 32) vals[e] /= fl[e / kDHd];
    named_bar_sync(1, kDW * 32);
    if (KV == RCU_KV_TURBO4) {
        for (uint32_t hh = warp; hh < (uint32_t)G; hh += kDW) rotate_row(vals + hh * kDHd, kDHd, true, (int)lane);
        named_bar_sync(1, kDW * 32);
    }
    constexpr uint32_t gv = G * kDHd;
    const uint64_t row_k = (uint64_t)p.n_head * kDHd, row0 = (uint64_t)t * row_k + (uint64_t)g * gv;
    if (p.out)
        for (uint32_t v = tid; v < gv; v += kDW * 32) p.out[row0 + v] = vals[v];
    if (p.aq.fmt) {
        for (uint32_t v0 = 0; v0 < gv; v0 += kDW * 32) {  // whole Q8_0 / Q8_K blocks
            const uint32_t v = v0 + tid;
            const float x = vals[v];
            if (p.aq.fmt & RCU_ACT_Q8_0) q8_0_block(x, (row0 + v0 + 32 * warp) / QK, (int)lane, p.aq);
            if (p.aq.fmt & RCU_ACT_Q8K) q8_k_block(x, tid, 0, (row0 + v0) / QK_K, true, p.aq, qsh, (v0 / (kDW * 32)) & 1);
        }
    }
}

template <int KV, int G>
__global__ void __launch_bounds__(kDThreads) k_attn_dec(const __grid_constant__ DecParams p) {
    static_assert(KV == RCU_KV_F16 || KV == RCU_KV_Q8_0, "turbo4 caches use k_attn_dec_t4");
    constexpr int R = 32 / G;  // cache rows per warp chunk
    extern __shared__ __align__(128) uint8_t dsm[];  // stages: [stage][K rows, V rows]
    __shared__ __align__(8) uint64_t full[kDMaxStages], empty[kDMaxStages];
    __shared__ RowMap maps[kDMaxStages];
    __shared__ __align__(8) uint64_t newrow;  // the fused post-processing's new K / V rows are in the cache
    __shared__ float nrx[2][kDHd];
    __shared__ uint8_t nrq[2][kDHd];
    __shared__ __align__(16) float qf[G][kDHd];
    __shared__ __align__(16) int8_t qi[G][kDHd];
    __shared__ float qds[G][kDHd / 32];
    __shared__ __align__(16) float pw[kDW][32];  // softmax weights of the warp's chunk, [row * G + head]
    __shared__ __align__(16) float aw[kDW][G];   // rescale factors of the warp's chunk
    __shared__ float wm[kDW][G], wl[kDW][G];
    const uint32_t split = blockIdx.x, g = blockIdx.y, t = blockIdx.z;
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint64_t pos_b = p.pos_ptr ? *p.pos_ptr : p.pos0;
    const uint64_t pt = pos_b + t;
    const uint64_t start = p.window > 0 ? (pt + 1 > p.window ? pt + 1 - p.window : 0) : 0;
    const uint32_t len = (uint32_t)(pt + 1 - start);
    const uint32_t c0 = split * p.rows_per_split, c1 = min(len, c0 + p.rows_per_split);
    const uint32_t rb = p.row_bytes, SR = p.stage_rows, NS = p.n_stages, BB = p.buf_bytes;
    const uint32_t n_stage = c1 > c0 ? (c1 - c0 + SR - 1) / SR : 0;
    const uint64_t head_base = (uint64_t)g * p.slots * rb;
    if (tid == 0) {
        for (uint32_t s = 0; s < NS; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kDW);
        }
        mbar_init(&newrow, 2);
        fence_mbar_init();
    }
    __syncthreads();
    pdl_trigger();

    if (warp == kDW) {  // ---- producer: bulk copies of the CTA's rows, stage by stage ----
        if (lane == 0) dec_produce(p, dsm, full, empty, maps, &newrow, c0, c1, n_stage, start, pos_b, head_base);
        return;
    }

    pdl_wait();  // q (and with the fused post-processing k / v) come from the kernel before
    {
        // fused post-processing: the CTA holding the newest position writes its K / V rows first
        // (its producer waits for them before the last stage), in the last two consumer warps
        const uint64_t fresh = pos_b - start;
        if (p.post && warp >= kDW - 2 && fresh >= c0 && fresh < c1)
            dec_new_row<KV>(p, (int)(kDW - 1 - warp), g, pos_b, nrx[kDW - 1 - warp], nrq[kDW - 1 - warp], &newrow, lane);
    }
    dec_query<KV, G>(p, qf, qi, qds, t, g, warp, lane);
    named_bar_sync(1, kDW * 32);
    // this lane's query dims 4l..4l+3 of every head
    float qv[G][4];
    uint32_t qc[G];
#pragma unroll
    for (int h = 0; h < G; h++) {
        const float4 f = *reinterpret_cast<const float4 *>(&qf[h][4 * lane]);
        qv[h][0] = f.x, qv[h][1] = f.y, qv[h][2] = f.z, qv[h][3] = f.w;
        qc[h] = *reinterpret_cast<const uint32_t *>(&qi[h][4 * lane]);
    }
    // after the first three butterfly stages the lane's 4 values share one row and are heads
    // h0 .. h0 + 3 of the lane's 32-dim block (lane >> 3): their query block scales
    const uint32_t kb = lane_k(lane) & ~3u;  // score index of value 0 after three stages
    const uint32_t h0 = kb % G, rowq = kb / G;
    float dq[4];
#pragma unroll
    for (int j = 0; j < 4; j++) dq[j] = qds[(h0 + j) % G][lane >> 3];
    const uint32_t kfin = lane_k(lane), hfin = kfin % G, rfin = kfin / G;

    float m_run = -INFINITY, l_run = 0.0f;  // of head hfin, the same in every lane of that head
    float acc[G][4];
#pragma unroll
    for (int h = 0; h < G; h++) acc[h][0] = acc[h][1] = acc[h][2] = acc[h][3] = 0.0f;

    bool ok = true;
    for (uint32_t j = 0; ok && j < n_stage; j++) {
        const uint32_t st = j % NS, ra = c0 + j * SR, n = min(SR, c1 - ra);
        const uint8_t *kbuf = dsm + (size_t)st * 2 * BB, *vbuf = kbuf + BB;
        if (!mbar_wait_bounded(&full[st], (j / NS) & 1u, p.err, ERR_TIMEOUT_FULL)) {
            ok = false;
            break;
        }
        const RowMap rr = maps[st];
        for (uint32_t r0 = R * warp; r0 < n; r0 += R * kDW) {
        Quad<KV> K[R], V[R];
#pragma unroll
        for (int i = 0; i < R; i++) {
            if (r0 + i < n) {
                const uint32_t ro = rr.off(r0 + i, rb);
                load_quad<KV>(kbuf + ro, lane, false, K[i]);
                load_quad<KV>(vbuf + ro, lane, true, V[i]);
            } else {
                K[i].codes = 0u, K[i].scale = 0.0f;
                V[i].f[0] = V[i].f[1] = V[i].f[2] = V[i].f[3] = 0.0f;
                K[i].f[0] = K[i].f[1] = K[i].f[2] = K[i].f[3] = 0.0f;
            }
        }
        // 2. scores of the chunk's R rows x G heads, summed over the warp by the butterfly
        float s;
        if (KV == RCU_KV_F16) {
            float v[32];
#pragma unroll
            for (int i = 0; i < R; i++)
#pragma unroll
                for (int h = 0; h < G; h++)
                    v[i * G + h] = fmaf(K[i].f[3], qv[h][3], fmaf(K[i].f[2], qv[h][2],
                                        fmaf(K[i].f[1], qv[h][1], K[i].f[0] * qv[h][0])));
            bfly<32>(v, lane, 4);
            bfly<16>(v, lane, 2);
            bfly<8>(v, lane, 1);
            bfly<4>(v, lane, 16);
            bfly<2>(v, lane, 8);
            s = v[0];
        } else {
            int v[32];
#pragma unroll
            for (int i = 0; i < R; i++)
#pragma unroll
                for (int h = 0; h < G; h++) v[i * G + h] = dp4a(K[i].codes, qc[h], 0);
            bfly<32>(v, lane, 4);  // exact sums over the 8 lanes of each 32-dim block
            bfly<16>(v, lane, 2);
            bfly<8>(v, lane, 1);
            // the block scales d_k(row, block) * d_q(head, block)
            float kscale = 0.0f;  // of row rowq, this lane's block
#pragma unroll
            for (int i = 0; i < R; i++)
                if ((uint32_t)i == rowq) kscale = K[i].scale;
            float f[32];
#pragma unroll
            for (int jj = 0; jj < 4; jj++) f[jj] = kscale * dq[jj] * (float)v[jj];
            bfly<4>(f, lane, 16);
            bfly<2>(f, lane, 8);
            s = f[0];
        }
        if (p.softcap > 0.0f) s = p.softcap * tanhf(s / p.softcap);
        if (r0 + rfin >= n) s = -INFINITY;
        // 3. online softmax per head over the lanes holding that head's rows
        float mx = s;
        if (G == 4) {
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        } else {
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        }
        const float m_new = fmaxf(m_run, mx);
        const float e = s == -INFINITY ? 0.0f : expf(s - m_new);
        float sum = e;
        if (G == 4) {
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            sum += __shfl_xor_sync(0xffffffffu, sum, 4);
        } else {
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            sum += __shfl_xor_sync(0xffffffffu, sum, 4);
        }
        const float alpha = m_run == -INFINITY ? 0.0f : expf(m_run - m_new);
        l_run = l_run * alpha + sum;
        m_run = m_new;
        pw[warp][kfin] = e;
        if (rfin == 0) aw[warp][hfin] = alpha;
        __syncwarp();
        // 4. V: the lane's 4 dims of every head
        if (__any_sync(0xffffffffu, alpha != 1.0f)) {  // a head's running maximum moved
#pragma unroll
            for (int h = 0; h < G; h++) {
                const float a = aw[warp][h];
#pragma unroll
                for (int jj = 0; jj < 4; jj++) acc[h][jj] *= a;
            }
        }
#pragma unroll
        for (int i = 0; i < R; i++) {
#pragma unroll
            for (int h4 = 0; h4 < G; h4 += 4) {
                const float4 pv = *reinterpret_cast<const float4 *>(&pw[warp][i * G + h4]);
                const float pa[4] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
                for (int hh = 0; hh < 4; hh++)
#pragma unroll
                    for (int jj = 0; jj < 4; jj++) acc[h4 + hh][jj] = fmaf(pa[hh], V[i].f[jj], acc[h4 + hh][jj]);
            }
        }
        __syncwarp();
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
    }
    (void)ok;

    // 5. merge the warps of the CTA, then the CTAs of the cluster (distributed shared memory);
    // the warps' rows go to the stage buffers, all consumed by now
    named_bar_sync(1, kDW * 32);
    float(*wo)[G][kDHd] = reinterpret_cast<float(*)[G][kDHd]>(dsm);
    if (rfin == 0) {
        wm[warp][hfin] = m_run;
        wl[warp][hfin] = l_run;
    }
#pragma unroll
    for (int h = 0; h < G; h++)
        *reinterpret_cast<float4 *>(&wo[warp][h][4 * lane]) = make_float4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
    named_bar_sync(1, kDW * 32);
    dec_finish<KV, G>(p, dsm, wm, wl, split, g, t);
}

// ---- turbo4 decode attention on the tensor cores ----
//
// A warp takes 16 cache rows at a time.
//   * Scores: mma.m16n8k32 (u8 x s8 -> s32) with the 16 rows as M, the group's heads as N and one
//     32-dim Q8_0 block of the rotated query as K, so every (row, head, block) int32 sum is the
//     reference's exactly. The 4-bit codes become level magnitudes with one byte permute per 4
//     codes and sign (kT4Pos for codes 8..15, kT4Neg for codes 0..7; a selector nibble with bit 3
//     set makes prmt replicate the sign bit of the byte it picks, 0 in these tables, so codes of
//     the other sign read 0), and the two halves go through two mma against the query codes and
//     their negation, accumulating into the same int32 block sums.
//   * Softmax: a running maximum M per head (log2 units) of t + log2(vscale), t = score * log2 e,
//     so the V weights 2^(t + log2 vscale - M) stay in (0, 1] whatever the rows' scales, and the
//     normaliser sums 2^(t - M) over the same M.
//   * V: mma.m16n8k16 (f16 -> f32) with 16 dims as M, the 16 rows as K and the heads as N. The
//     levels are exact f16 subnormals (magnitude * 2^-24: bytes [m, 0, m', 0] are a half2), again
//     as a positive and a negative half against the weights and their negation; the weights are
//     the f16 sum hi + lo of their f32 value (22 bits), moved from the scores' fragment layout
//     (rows x heads) to the B operand's (heads x rows) with movmatrix.
// Dim slot (g, t) of the V fragments (thread group g = lane / 4, tile t = 0..7) is the low
// nibble of code byte 8g + t, slot (g + 8, t) its high nibble, so a lane reads 8 consecutive code
// bytes of each of its rows.
constexpr uint32_t kT4Pos0 = 0x2b1e1206u, kT4Pos1 = 0x7e5f4a3au;  // codes 8..15: 6 18 30 43 58 74 95 126
constexpr uint32_t kT4Neg0 = 0x3a4a5f7eu, kT4Neg1 = 0x06121e2bu;  // codes 0..7: 126 95 74 58 43 30 18 6

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
// Magnitudes of the 4 codes in the low 16 bits of `sel` (codes 0..7) / of `sel ^ 0x8888` (8..15).
__device__ __forceinline__ uint32_t t4_neg(uint32_t sel) { return prmt(kT4Neg0, kT4Neg1, sel); }
__device__ __forceinline__ uint32_t t4_pos(uint32_t sel_x8) { return prmt(kT4Pos0, kT4Pos1, sel_x8); }
__device__ __forceinline__ void mma_k32(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_k16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t movm_t(uint32_t x) {
    uint32_t y;
    asm("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}
__device__ __forceinline__ uint32_t lds16(const uint8_t *p) { return *reinterpret_cast<const uint16_t *>(p); }
__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
// 2^x on the SFU (ex2.approx: 2^-22 relative; 2^-inf = +0, so masked rows need no test).
__device__ __forceinline__ float ex2a(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float lg2a(float x) {
    float y;
    asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ uint32_t pack_s8(int a, int b, int c, int d) {
    return (uint32_t)(uint8_t)a | (uint32_t)(uint8_t)b << 8 | (uint32_t)(uint8_t)c << 16 | (uint32_t)(uint8_t)d << 24;
}

// Both halves (positive, negative levels) of one V tile against the weights hi (+ lo): the f16
// subnormal half2 of rows A, B (C, D) from the lookup bytes [m(A lo), m(A hi), m(B lo), m(B hi)].
template <bool HILO>
__device__ __forceinline__ void t4_v_mma(float (&o)[4], uint32_t pab, uint32_t pcd, uint32_t nab, uint32_t ncd,
                                         const uint32_t (&bh)[2], const uint32_t (&bl)[2], const uint32_t (&nh)[2],
                                         const uint32_t (&nl)[2]) {
    const uint32_t p0 = prmt(pab, 0u, 0x4240u), p1 = prmt(pab, 0u, 0x4341u), p2 = prmt(pcd, 0u, 0x4240u),
                   p3 = prmt(pcd, 0u, 0x4341u);
    const uint32_t n0 = prmt(nab, 0u, 0x4240u), n1 = prmt(nab, 0u, 0x4341u), n2 = prmt(ncd, 0u, 0x4240u),
                   n3 = prmt(ncd, 0u, 0x4341u);
    mma_k16(o, p0, p1, p2, p3, bh[0], bh[1]);
    mma_k16(o, n0, n1, n2, n3, nh[0], nh[1]);
    if (HILO) {
        mma_k16(o, p0, p1, p2, p3, bl[0], bl[1]);
        mma_k16(o, n0, n1, n2, n3, nl[0], nl[1]);
    }
}

template <int G, bool HILO>
__global__ void __launch_bounds__(kDThreads, 2) k_attn_dec_t4(const __grid_constant__ DecParams p) {
    extern __shared__ __align__(128) uint8_t dsm[];  // stages: [stage][K rows, V rows]
    __shared__ __align__(8) uint64_t full[kDMaxStages], empty[kDMaxStages];
    __shared__ RowMap maps[kDMaxStages];
    __shared__ __align__(8) uint64_t newrow;  // the fused post-processing's new K / V rows are in the cache
    __shared__ __align__(16) float nrx[2][kDHd];
    __shared__ uint8_t nrq[2][kDHd];
    __shared__ __align__(16) float qf[G][kDHd];
    __shared__ __align__(16) int8_t qi[G][kDHd];
    __shared__ float qds[G][kDHd / 32];
    __shared__ float wm[kDW][G], wl[kDW][G];
    const uint32_t split = blockIdx.x, g = blockIdx.y, t = blockIdx.z;
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint64_t pos_b = p.pos_ptr ? *p.pos_ptr : p.pos0;
    const uint64_t pt = pos_b + t;
    const uint64_t start = p.window > 0 ? (pt + 1 > p.window ? pt + 1 - p.window : 0) : 0;
    const uint32_t len = (uint32_t)(pt + 1 - start);
    const uint32_t c0 = split * p.rows_per_split, c1 = min(len, c0 + p.rows_per_split);
    const uint32_t rb = p.row_bytes, SR = p.stage_rows, NS = p.n_stages, BB = p.buf_bytes;
    const uint32_t n_stage = c1 > c0 ? (c1 - c0 + SR - 1) / SR : 0;
    const uint64_t head_base = (uint64_t)g * p.slots * rb;
    if (tid == 0) {
        for (uint32_t s = 0; s < NS; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kDW);
        }
        mbar_init(&newrow, 2);
        fence_mbar_init();
    }
    __syncthreads();
    pdl_trigger();
    if (warp == kDW) {
        if (lane == 0) dec_produce(p, dsm, full, empty, maps, &newrow, c0, c1, n_stage, start, pos_b, head_base);
        return;
    }
    pdl_wait();  // q (and with the fused post-processing k / v) come from the kernel before
    {
        // fused post-processing: the CTA holding the newest position rotates and encodes its K / V
        // rows first (its producer waits for them before the last stage), in the last two warps
        const uint64_t fresh = pos_b - start;
        if (p.post && warp >= kDW - 2 && fresh >= c0 && fresh < c1)
            dec_new_row<RCU_KV_TURBO4>(p, (int)(kDW - 1 - warp), g, pos_b, nrx[kDW - 1 - warp], nrq[kDW - 1 - warp],
                                       &newrow, lane);
    }
    dec_query<RCU_KV_TURBO4, G>(p, qf, qi, qds, t, g, warp, lane);
    named_bar_sync(1, kDW * 32);

    const uint32_t gq = lane >> 2, tg = lane & 3;  // fragment row group, thread in group
    const bool hv0 = 2 * tg < (uint32_t)G, hv1 = 2 * tg + 1 < (uint32_t)G;  // the lane's score columns are heads
    // score B fragments: head gq's codes in the k order of the A fragments (k 4tg + 0..3 <- dims
    // j, j + 16, j + 1, j + 17 of the block, k 16 + 4tg + 0..3 <- j + 2, j + 18, j + 3, j + 19; j = 4tg)
    uint32_t bq[4][2], bn[4][2];
    float dqa[4], dqb[4];
#pragma unroll
    for (int ch = 0; ch < 4; ch++) {
        if (gq < (uint32_t)G) {
            const int8_t *qh = &qi[gq][32 * ch + 4 * tg];
            bq[ch][0] = pack_s8(qh[0], qh[16], qh[1], qh[17]);
            bq[ch][1] = pack_s8(qh[2], qh[18], qh[3], qh[19]);
            bn[ch][0] = pack_s8(-qh[0], -qh[16], -qh[1], -qh[17]);
            bn[ch][1] = pack_s8(-qh[2], -qh[18], -qh[3], -qh[19]);
        } else {
            bq[ch][0] = bq[ch][1] = bn[ch][0] = bn[ch][1] = 0u;
        }
        dqa[ch] = hv0 ? qds[2 * tg][ch] : 0.0f;
        dqb[ch] = hv1 ? qds[2 * tg + 1][ch] : 0.0f;
    }

    float M0 = -INFINITY, M1 = -INFINITY;  // heads 2tg, 2tg + 1: running max of t + log2(vscale)
    float l0 = 0.0f, l1 = 0.0f;            // the lane's rows' share of the sums of 2^(t - M)
    float O[8][4];                          // V tile k: (slot gq, 2tg), (gq, 2tg + 1), (gq + 8, 2tg), (gq + 8, 2tg + 1)
#pragma unroll
    for (int k = 0; k < 8; k++) O[k][0] = O[k][1] = O[k][2] = O[k][3] = 0.0f;
    constexpr float kInv46 = 1.0f / 46.0f, kLog2e = 1.4426950408889634f;

    for (uint32_t j = 0; j < n_stage; j++) {
        const uint32_t st = j % NS, n = min(SR, c1 - (c0 + j * SR));
        const uint8_t *kbuf = dsm + (size_t)st * 2 * BB, *vbuf = kbuf + BB;
        if (!mbar_wait_bounded(&full[st], (j / NS) & 1u, p.err, ERR_TIMEOUT_FULL)) break;
        const RowMap rr = maps[st];
        for (uint32_t r0 = 16 * warp; r0 < n; r0 += 16 * kDW) {
            const uint32_t nn = n - r0;  // rows of the tile in the stage (rows beyond read the last one, weight 0)
            const uint32_t og = rr.off(r0 + min(gq, nn - 1), rb), og8 = rr.off(r0 + min(gq + 8, nn - 1), rb);
            // 1. scores of rows gq, gq + 8 for heads 2tg, 2tg + 1: exact block sums, then the scales
            float sa[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
            for (int ch = 0; ch < 4; ch++) {
                const uint8_t *ka = kbuf + og + 2 + 16 * ch + 4 * tg, *kb = kbuf + og8 + 2 + 16 * ch + 4 * tg;
                const uint32_t wa = lds16(ka) | lds16(ka + 2) << 16, wb = lds16(kb) | lds16(kb + 2) << 16;
                const uint32_t xa = wa ^ 0x88888888u, xb = wb ^ 0x88888888u;
                int c[4] = {0, 0, 0, 0};
                mma_k32(c, t4_pos(xa), t4_pos(xb), t4_pos(xa >> 16), t4_pos(xb >> 16), bq[ch][0], bq[ch][1]);
                mma_k32(c, t4_neg(wa), t4_neg(wb), t4_neg(wa >> 16), t4_neg(wb >> 16), bn[ch][0], bn[ch][1]);
                sa[0] = fmaf(dqa[ch], (float)c[0], sa[0]);
                sa[1] = fmaf(dqb[ch], (float)c[1], sa[1]);
                sa[2] = fmaf(dqa[ch], (float)c[2], sa[2]);
                sa[3] = fmaf(dqb[ch], (float)c[3], sa[3]);
            }
            const float ks0 = f16_bits_to_f32(lds16(kbuf + og)), ks1 = f16_bits_to_f32(lds16(kbuf + og8));
            const float vs0 = f16_bits_to_f32(lds16(vbuf + og)), vs1 = f16_bits_to_f32(lds16(vbuf + og8));
            float sc[4] = {ks0 * sa[0] * kInv46, ks0 * sa[1] * kInv46, ks1 * sa[2] * kInv46, ks1 * sa[3] * kInv46};
            if (p.softcap > 0.0f) {
#pragma unroll
                for (int i = 0; i < 4; i++) sc[i] = p.softcap * tanhf(sc[i] / p.softcap);
            }
            const bool v0 = gq < nn, v1 = gq + 8 < nn;
            // zero rows (scale 0) get a tiny stand-in scale: their weight in the V sum is then
            // 2^-64 of a real row's, their share of the normaliser is exact
            const float lv0 = vs0 > 0.0f ? lg2a(vs0) : -64.0f, lv1 = vs1 > 0.0f ? lg2a(vs1) : -64.0f;
            const float tt0 = v0 && hv0 ? sc[0] * kLog2e : -INFINITY, tt1 = v0 && hv1 ? sc[1] * kLog2e : -INFINITY;
            const float tt2 = v1 && hv0 ? sc[2] * kLog2e : -INFINITY, tt3 = v1 && hv1 ? sc[3] * kLog2e : -INFINITY;
            const float u0 = tt0 + lv0, u1 = tt1 + lv0, u2 = tt2 + lv1, u3 = tt3 + lv1;
            // 2. online softmax per head over the 8 lanes holding it (lane bits 2..4 = row)
            float mx0 = fmaxf(u0, u2), mx1 = fmaxf(u1, u3);
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) {
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
            }
            const float Mn0 = fmaxf(M0, mx0), Mn1 = fmaxf(M1, mx1);
            // a head with no valid row yet keeps M = -inf: subtract 0 instead (every weight is 0)
            const float S0 = Mn0 == -INFINITY ? 0.0f : Mn0, S1 = Mn1 == -INFINITY ? 0.0f : Mn1;
            const float al0 = ex2a(M0 - S0), al1 = ex2a(M1 - S1);  // 1 when the max stays, 0 from -inf
            const float pw0 = ex2a(u0 - S0), pw1 = ex2a(u1 - S1), pw2 = ex2a(u2 - S0), pw3 = ex2a(u3 - S1);
            l0 = fmaf(l0, al0, ex2a(tt0 - S0) + ex2a(tt2 - S0));
            l1 = fmaf(l1, al1, ex2a(tt1 - S1) + ex2a(tt3 - S1));
            M0 = Mn0;
            M1 = Mn1;
            if (__any_sync(0xffffffffu, al0 != 1.0f || al1 != 1.0f)) {
#pragma unroll
                for (int k = 0; k < 8; k++) {
                    O[k][0] *= al0;
                    O[k][1] *= al1;
                    O[k][2] *= al0;
                    O[k][3] *= al1;
                }
            }
            // 3. the weights as V's B fragments (rows 2tg, 2tg + 1 | 2tg + 8, 2tg + 9 of head gq)
            const __half2 h0 = __floats2half2_rn(pw0, pw1), h1 = __floats2half2_rn(pw2, pw3);
            const uint32_t bh[2] = {movm_t(h2_bits(h0)), movm_t(h2_bits(h1))};
            uint32_t bl[2] = {0u, 0u};
            if (HILO) {
                const float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
                bl[0] = movm_t(h2_bits(__floats2half2_rn(pw0 - f0.x, pw1 - f0.y)));
                bl[1] = movm_t(h2_bits(__floats2half2_rn(pw2 - f1.x, pw3 - f1.y)));
            }
            const uint32_t nh[2] = {bh[0] ^ 0x80008000u, bh[1] ^ 0x80008000u};
            const uint32_t nl[2] = {bl[0] ^ 0x80008000u, bl[1] ^ 0x80008000u};
            // 4. V: code bytes 8gq .. 8gq + 7 of rows 2tg (A), 2tg + 1 (B), 2tg + 8 (C), 2tg + 9 (D)
            const uint8_t *va = vbuf + rr.off(r0 + min(2 * tg, nn - 1), rb) + 2 + 8 * gq;
            const uint8_t *vb = vbuf + rr.off(r0 + min(2 * tg + 1, nn - 1), rb) + 2 + 8 * gq;
            const uint8_t *vc = vbuf + rr.off(r0 + min(2 * tg + 8, nn - 1), rb) + 2 + 8 * gq;
            const uint8_t *vd = vbuf + rr.off(r0 + min(2 * tg + 9, nn - 1), rb) + 2 + 8 * gq;
#pragma unroll
            for (int k = 0; k < 4; k++) {  // code bytes 2k, 2k + 1: tiles 2k, 2k + 1
                const uint32_t xab = prmt(lds16(va + 2 * k), lds16(vb + 2 * k), 0x5140u);  // [A, B, A', B']
                const uint32_t xcd = prmt(lds16(vc + 2 * k), lds16(vd + 2 * k), 0x5140u);
                const uint32_t yab = xab ^ 0x88888888u, ycd = xcd ^ 0x88888888u;
                t4_v_mma<HILO>(O[2 * k], t4_pos(yab), t4_pos(ycd), t4_neg(xab), t4_neg(xcd), bh, bl, nh, nl);
                t4_v_mma<HILO>(O[2 * k + 1], t4_pos(yab >> 16), t4_pos(ycd >> 16), t4_neg(xab >> 16),
                               t4_neg(xcd >> 16), bh, bl, nh, nl);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
    }

    // 5. the warp's partial: sums over the lanes of each head, rows to dims, into the stage buffers
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
        l0 += __shfl_xor_sync(0xffffffffu, l0, o);
        l1 += __shfl_xor_sync(0xffffffffu, l1, o);
    }
    named_bar_sync(1, kDW * 32);  // every warp is done with the stages
    float(*wo)[G][kDHd] = reinterpret_cast<float(*)[G][kDHd]>(dsm);
    constexpr float kLn2 = 0.6931471805599453f;
    if (gq == 0) {
        if (hv0) wm[warp][2 * tg] = M0 * kLn2, wl[warp][2 * tg] = l0;
        if (hv1) wm[warp][2 * tg + 1] = M1 * kLn2, wl[warp][2 * tg + 1] = l1;
    }
    constexpr float kOut = 16777216.0f / 46.0f;  // the subnormal unit 2^-24 and the level scale 1/46
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const uint32_t d = 32 * (gq >> 1) + 8 * (gq & 1) + k;
        if (hv0) wo[warp][2 * tg][d] = O[k][0] * kOut, wo[warp][2 * tg][d + 16] = O[k][2] * kOut;
        if (hv1) wo[warp][2 * tg + 1][d] = O[k][1] * kOut, wo[warp][2 * tg + 1][d + 16] = O[k][3] * kOut;
    }
    named_bar_sync(1, kDW * 32);
    dec_finish<RCU_KV_TURBO4, G>(p, dsm, wm, wl, split, g, t);
}

}  // namespace

bool attention_dec_ok(int kv_type, uint64_t hd, uint64_t group) {
    (void)kv_type;
    return hd == kDHd && (group == 4 || group == 8);
}

// Splits of the context per (token, KV head): at least 64 rows each, about `per_sm` CTAs per SM
// in all (the turbo4 kernel fits two), a multiple of the cluster size cs (<= 8), and no more
// clusters than fit on the device at once (cap(cs), measured): a cluster that does not fit runs
// as a second wave and doubles the launch. Short contexts take one cluster per KV head; longer
// ones the cluster size (8, 4 or 2) that gives the most CTAs for the fewest clusters per head,
// merged through global memory when a head has more than one cluster.
template <typename Cap>
static void dec_plan(uint64_t per_sm, uint64_t max_len, uint64_t n_tok, uint64_t n_kv, int num_sms, Cap cap,
                     uint64_t min_rows, uint32_t *n_split, uint32_t *cs, uint32_t *rows) {
    const uint64_t heads = std::max<uint64_t>(1, n_kv * n_tok);
    const uint64_t want = std::max<uint64_t>(1, per_sm * (uint64_t)num_sms / heads);
    const uint64_t ns_max = std::max<uint64_t>(1, std::min<uint64_t>((max_len + min_rows - 1) / min_rows, want));
    uint64_t best_ns = 1, best_c = 1;
    if (ns_max <= kDMaxCluster) {
        best_ns = best_c = ns_max;
    } else {
        // each further cluster of a head costs about two splits: its partials wait for the last
        // cluster, whose merge through global memory is the launch's tail (measured, config 5:
        // 8 x 32 splits 39.1 us, 4 x 32 41.1, 2 x 36 47.7, 1 x 36 56.3 per layer)
        int64_t best = -1;
        for (const uint64_t c : {8ull, 4ull, 2ull}) {
            uint64_t ns = ns_max / c * c;
            const uint64_t fit = (uint64_t)std::max(cap((uint32_t)c), 1);
            while (ns > c && (ns / c) * heads > fit) ns -= c;
            if ((ns / c) * heads > fit) continue;  // not even one cluster per head fits at once
            const int64_t score = (int64_t)ns - 2 * (int64_t)(ns / c - 1);
            if (score > best) best = score, best_ns = ns, best_c = c;
        }
        if (best < 0) best_ns = best_c = 1;
    }
    *n_split = (uint32_t)best_ns;
    *cs = (uint32_t)best_c;
    *rows = (uint32_t)((max_len + best_ns - 1) / best_ns);
}

// Shortest split of the context (rows). The turbo4 kernel's fixed cost per CTA (query rotation
// and quantization, cluster merge, output rotation) is large next to a 64-row split: with one KV
// head at context 32768 (the 70B shape at 8 GPUs) 256-row splits measured 5.56 ms per token
// against 6.61 ms for 64-row splits and 6.47 ms for 1024-row ones. The f16 / Q8_0 kernel keeps
// 64 (config 3, context ~540, is fastest with eight 68-row splits per KV head).
// RIE_ATTN_MIN_ROWS overrides both.
static uint64_t dec_min_rows(bool turbo) {
    static const long env = [] {
        const char *e = getenv("RIE_ATTN_MIN_ROWS");
        return e ? atol(e) : 0L;
    }();
    if (env >= 16) return (uint64_t)env;
    return turbo ? 256 : 64;
}

// An upper bound of the clusters a decode launch merges through global memory (its splits).
uint32_t attention_dec_max_clusters(int kv_type, uint64_t max_len, uint64_t n_tok, uint64_t n_kv, int num_sms) {
    const uint64_t per_sm = kv_type == RCU_KV_TURBO4 ? 2 : 1;
    const uint64_t want = std::max<uint64_t>(1, per_sm * (uint64_t)num_sms / std::max<uint64_t>(1, n_kv * n_tok));
    return (uint32_t)std::max<uint64_t>(1, std::min<uint64_t>((max_len + 63) / 64, want));
}

// Launch one of the decode kernels: plan the splits, then stages of up to `max_sr` rows (at
// least two stages in the shared memory a CTA may use when `per_sm` of them share an SM), 2 to 4
// of them. `parts` holds the partials of contexts split over more than one cluster.
struct DecKern {
    void (*kern)(DecParams);
    int budget;          // per device: the CTA's share of shared memory minus the static part
    int cap[kDMaxCluster + 1];  // clusters of each size that fit at once (0: not measured)
};
template <int G>
static int launch_dec(rcu_ctx *ctx, DecParams &p, DecKern &K, int per_sm, uint32_t max_sr, uint64_t max_len,
                      uint64_t n_tok, float *parts) {
    auto kern = K.kern;
    if (!K.budget) {
        cudaFuncAttributes fa;
        RCU_CUDA_TRY(ctx, cudaFuncGetAttributes(&fa, kern));
        int per_cta = (int)ctx->max_smem_optin;
        if (per_sm > 1) {
            int sm_total = 0;
            RCU_CUDA_TRY(ctx, cudaDeviceGetAttribute(&sm_total, cudaDevAttrMaxSharedMemoryPerMultiprocessor, ctx->device));
            per_cta = std::min(per_cta, sm_total / per_sm - 1024);  // 1 KB per CTA is reserved
        }
        const int lim = per_cta - (int)fa.sharedSizeBytes;
        RCU_CUDA_TRY(ctx, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, lim));
        if (cudaError_t e = prefer_max_shared(reinterpret_cast<const void *>(kern))) return cuda_err(ctx, e, "attention");
        K.budget = lim;
    }
    const int budget = K.budget;
    const uint32_t rb = p.row_bytes;
    auto stage_plan = [&](uint32_t rows_per_split, uint32_t &sr, uint32_t &buf, uint32_t &ns) {
        const uint32_t sr_fit = (uint32_t)(((uint64_t)budget / 4 > 64 ? ((uint64_t)budget / 4 - 64) / rb : 0) / 16 * 16);
        const uint32_t want = (rows_per_split + 15) / 16 * 16;
        sr = std::max<uint32_t>(16, std::min<uint32_t>(std::min<uint32_t>(sr_fit, max_sr), want));
        buf = (sr * rb + 64 + 15) / 16 * 16;  // + the two ranges' 16-byte enclosures
        const uint32_t n_stage = (rows_per_split + sr - 1) / sr;
        ns = std::max<uint32_t>(1, std::min<uint32_t>(std::min<uint32_t>(kDMaxStages, n_stage), (uint32_t)budget / (2 * buf)));
        return std::max<uint32_t>(ns * 2 * buf, kDW * G * kDHd * 4);  // dynamic shared memory
    };
    // clusters of size c that fit, measured once per device with the largest stages this kernel uses
    auto cap = [&](uint32_t c) -> int {
        if (!K.cap[c]) {
            uint32_t sr, buf, nst;
            const uint32_t dyn = stage_plan(0xffff, sr, buf, nst);
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(c * 64);
            cfg.blockDim = dim3(kDThreads);
            cfg.dynamicSmemBytes = dyn;
            cudaLaunchAttribute at;
            at.id = cudaLaunchAttributeClusterDimension;
            at.val.clusterDim.x = c;
            at.val.clusterDim.y = 1;
            at.val.clusterDim.z = 1;
            cfg.attrs = &at;
            cfg.numAttrs = 1;
            int n = 0;
            if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
                (void)cudaGetLastError();
                n = 1;
            }
            K.cap[c] = std::max(n, 1);
        }
        return K.cap[c];
    };
    dec_plan((uint64_t)per_sm, max_len, n_tok, p.n_kv, ctx->num_sms, cap, dec_min_rows(per_sm > 1), &p.n_split,
             &p.cs, &p.rows_per_split);
    const uint64_t n_cl = p.n_split / p.cs, parts_n = n_tok * p.n_head * n_cl;
    p.o_part = parts;
    p.m_part = parts + parts_n * kDHd;
    p.l_part = p.m_part + parts_n;
    const uint32_t dyn = stage_plan(p.rows_per_split, p.stage_rows, p.buf_bytes, p.n_stages);
    if ((int)dyn > budget) return set_err(ctx, RCU_ERR_UNSUPPORTED, "attention: stage buffers exceed shared memory");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.n_split, p.n_kv, (uint32_t)n_tok);
    cfg.blockDim = dim3(kDThreads);
    cfg.dynamicSmemBytes = dyn;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = p.cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = ctx->pdl ? 2 : 1;
    RCU_CUDA_TRY(ctx, cudaLaunchKernelEx(&cfg, kern, p));
    return RCU_OK;
}

template <int KV, int G>
static int launch_dec_kv(rcu_ctx *ctx, DecParams &p, uint64_t max_len, uint64_t n_tok, float *parts) {
    static DecKern kerns[64] = {};  // per device
    if constexpr (KV == RCU_KV_TURBO4) {
        // RIE_ATTN_T4_HILO=0: the V weights as one f16 each (11 bits) instead of hi + lo
        static const bool hilo = !(getenv("RIE_ATTN_T4_HILO") && getenv("RIE_ATTN_T4_HILO")[0] == '0');
        static DecKern kerns1[64] = {};
        DecKern &K = (hilo ? kerns : kerns1)[ctx->device & 63];
        if (!K.kern) K.kern = hilo ? k_attn_dec_t4<G, true> : k_attn_dec_t4<G, false>;
        return launch_dec<G>(ctx, p, K, 2, 16 * kDW, max_len, n_tok, parts);
    } else {
        DecKern &K = kerns[ctx->device & 63];
        if (!K.kern) K.kern = k_attn_dec<KV, G>;
        return launch_dec<G>(ctx, p, K, 1, 256, max_len, n_tok, parts);
    }
}

int launch_attention_dec(rcu_ctx *ctx, const uint8_t *kc, const uint8_t *vc, int kv_type, uint64_t n_kv,
                         uint64_t slots, uint64_t row_bytes, const float *q, uint64_t n_tok, uint64_t n_head,
                         uint64_t pos0, const uint64_t *pos_ptr, uint64_t max_len, uint64_t window, float softcap,
                         float *out, const ActOut *aq, uint32_t *done, float *parts,
                         const QkvPostParams *post) {
    if (kv_type == RCU_KV_TURBO4)
        if (int st = ensure_signs(ctx)) return st;
    DecParams p{};
    if (post) {
        if (n_tok != 1) return set_err(ctx, RCU_ERR_INVALID, "attention: fused post-processing takes one token");
        p.post = 1;
        p.kraw = post->k, p.vraw = post->v, p.bq = post->bq, p.bk = post->bk, p.bv = post->bv;
        p.qn = post->qn, p.kn = post->kn, p.inv_freq = post->inv_freq, p.rope_dim = post->rope_dim;
        p.neox = post->neox, p.eps = post->eps, p.attn_scale = post->attn_scale;
    }
    p.kc = kc;
    p.vc = vc;
    p.q = q;
    p.out = out;
    if (aq) p.aq = *aq;
    p.n_head = (uint32_t)n_head;
    p.n_kv = (uint32_t)n_kv;
    p.slots = (uint32_t)slots;
    p.window = (uint32_t)window;
    p.pos0 = pos0;
    p.pos_ptr = pos_ptr;
    p.softcap = softcap;
    p.rounding = ctx->rounding;
    p.row_bytes = (uint32_t)row_bytes;
    p.err = ctx->dev_err;
    p.done = done;
    const uint64_t group = n_head / n_kv;
    switch (kv_type) {
        case RCU_KV_F16:
            return group == 4 ? launch_dec_kv<RCU_KV_F16, 4>(ctx, p, max_len, n_tok, parts)
                              : launch_dec_kv<RCU_KV_F16, 8>(ctx, p, max_len, n_tok, parts);
        case RCU_KV_Q8_0:
            return group == 4 ? launch_dec_kv<RCU_KV_Q8_0, 4>(ctx, p, max_len, n_tok, parts)
                              : launch_dec_kv<RCU_KV_Q8_0, 8>(ctx, p, max_len, n_tok, parts);
        default:
            return group == 4 ? launch_dec_kv<RCU_KV_TURBO4, 4>(ctx, p, max_len, n_tok, parts)
                              : launch_dec_kv<RCU_KV_TURBO4, 8>(ctx, p, max_len, n_tok, parts);
    }
}

}  // namespace rcu
