// rcu_attn_dec.cu -- decode attention (one query row per token and head) over an f16, Q8_0 or
// turbo4 KV cache at head_dim 128, for GQA groups of 4 or 8 query heads per KV head.
// Replaces, for decode steps, the reference's attention (crates/rie-core/src/model/cpu.rs:552-634)
// with its turbo4 scoring and V accumulation in the rotated domain (turbo.rs:178-250).
//
// Why a second attention kernel: at decode the work per cache row is small (G x 128 MACs for
// the scores, as many for V) and the context of a decode step is short, so the general kernel's
// phases (rows staged in shared memory, scores, softmax and V sums separated by block-wide
// barriers, splits merged through global memory by the last CTA) leave it latency-bound
// (18 us per layer at 515 positions). Here:
//   * every warp walks its own chunks of R = 32 / G cache rows with no block-wide barrier:
//     lane l loads dims 4l..4l+3 of each K and V row straight from global memory (one
//     coalesced row per load instruction) and keeps the query of those dims for all G heads
//     in registers;
//   * the R x G partial scores of a lane are summed over the 32 lanes by a transposing
//     butterfly (31 shuffles for 32 sums, each lane ending with one (row, head) score); with
//     quantized caches the first three stages add the exact int32 dp4a partials of the 8
//     lanes of a 32-dim block and the block scales are applied once per value after them, so
//     every per-block integer sum is the reference's exactly;
//   * online softmax per head in registers; the V sum keeps the lane's 4 dims of every head;
//   * the splits of a KV head (up to 8 CTAs) form a thread-block cluster and merge through
//     distributed shared memory; only contexts split over more than one cluster merge the
//     clusters through global memory (last cluster, counter per token and KV head);
//   * the merged rows are rotated back (turbo4) and written as f32 and / or quantized for the
//     Wo matmul in the same kernel.
// Scores and sums are f32 as in the reference; only the order of the f32 additions differs.
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

__device__ __forceinline__ uint32_t ld_u32_2a(const uint8_t *p) {  // 4 bytes at a 2-byte aligned address
    const uint16_t *h = reinterpret_cast<const uint16_t *>(p);
    return (uint32_t)__ldg(h) | ((uint32_t)__ldg(h + 1) << 16);
}

// Byte lookup of 16 entries (the turbo4 levels as int8) for 4 nibble indices at once.
__device__ __forceinline__ uint32_t lut16d(uint32_t idx) {
    const uint32_t t0 = 0xc6b6a182u, t1 = 0xfaeee2d5u, t2 = 0x2b1e1206u, t3 = 0x7e5f4a3au;  // levels as bytes
    const uint32_t sel = __byte_perm(idx | (idx >> 4), 0, 0x0020) & 0x7777u;
    const uint32_t lo = __byte_perm(t0, t1, sel), hi = __byte_perm(t2, t3, sel);
    const uint32_t m = ((idx & 0x08080808u) >> 3) * 0xffu;
    return (lo & ~m) | (hi & m);
}

// The 4 values of dims 4l..4l+3 of one cache row: K as exact codes (quantized caches) or f32,
// V as f32 (the row's scale applied).
template <int KV>
struct Quad {
    uint32_t codes;  // Q8_0 int8 codes / turbo4 int8 levels
    float f[4];      // f16 values / V values
    float scale;     // Q8_0: d of the lane's block; turbo4: row scale (f16)
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
    } else {  // turbo4 at hd 128: f16 scale, then 4 chunks of 16 bytes in Q4_0 nibble order
        const uint32_t ch = lane >> 3, j0 = 4 * (lane & 7);
        qd.scale = f16_bits_to_f32(*reinterpret_cast<const uint16_t *>(row));
        const uint32_t w = lds_u32_2a(row + 2 + 16 * ch + (j0 & 15));
        qd.codes = lut16d(j0 < 16 ? (w & 0x0F0F0F0Fu) : ((w >> 4) & 0x0F0F0F0Fu));
        if (is_v) {
            const float s = qd.scale * (1.0f / 46.0f);
#pragma unroll
            for (int j = 0; j < 4; j++) qd.f[j] = s * (float)sbyte(qd.codes, j);
        }
    }
}

// Rows [first_slot, first_slot + n) of one KV head's ring as a stage holds them: the ring may
// wrap, so one or two contiguous ranges, each copied from its 16-byte aligned enclosure.
struct Runs {
    uint64_t lo1, lo2;        // source byte offsets (from the cache base) of the copies
    uint32_t len1, len2;      // copy sizes (multiples of 16; len2 = 0: no second range)
    uint32_t n1, d1, d2;      // rows in the first range; stage offset of its first row; of the second's
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

template <int KV, int G>
__global__ void __launch_bounds__(kDThreads) k_attn_dec(const __grid_constant__ DecParams p) {
    constexpr int R = 32 / G;  // cache rows per warp chunk
    extern __shared__ __align__(128) uint8_t dsm[];  // stages: [stage][K rows, V rows]
    __shared__ __align__(8) uint64_t full[kDMaxStages], empty[kDMaxStages];
    __shared__ __align__(16) float qf[G][kDHd];
    __shared__ __align__(16) int8_t qi[G][kDHd];
    __shared__ float qds[G][kDHd / 32];
    __shared__ __align__(16) float pw[kDW][32];  // softmax weights of the warp's chunk, [row * G + head]
    __shared__ __align__(16) float aw[kDW][G];   // rescale factors of the warp's chunk
    __shared__ float wm[kDW][G], wl[kDW][G];
    // partials of the cluster's CTAs, pushed into rank 0 with remote stores: [rank][G * 128 + 2G]
    __shared__ __align__(16) float cpart[kDMaxCluster][G * kDHd + 2 * G];
    __shared__ Q8kShared qsh;
    __shared__ uint32_t s_last;
    cg::cluster_group cluster = cg::this_cluster();
    const uint32_t split = blockIdx.x, g = blockIdx.y, t = blockIdx.z;
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t rank = cluster.block_rank();
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
        fence_mbar_init();
    }
    __syncthreads();
    pdl_trigger();

    if (warp == kDW) {  // ---- producer: bulk copies of the CTA's rows, stage by stage ----
        if (lane == 0) {
            // rows of earlier positions were written at least two launches back; this step's rows
            // (logical index >= fresh) by the kernel just before: wait for it before copying them
            const uint32_t fresh = pos_b > start ? (uint32_t)(pos_b - start) : 0;
            bool waited = false;
            const uint64_t pol = policy_evict_first();
            uint32_t j = 0;
            for (; j < n_stage; j++) {
                const uint32_t s = j % NS;
                if (j >= NS && !mbar_wait_bounded(&empty[s], ((j / NS) - 1) & 1u, p.err, ERR_TIMEOUT_EMPTY)) break;
                const uint32_t ra = c0 + j * SR, n = min(SR, c1 - ra);
                if (!waited && ra + n > fresh) {
                    pdl_wait();
                    waited = true;
                }
                const Runs r = plan_runs(head_base, p.slots, rb, (start + ra) % p.slots, n);
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
        return;
    }

    pdl_wait();  // q comes from the kernel before
    // 1. the group's queries: f32 (f16 cache) or rotated (turbo4) and quantized to Q8_0 blocks
    for (uint32_t hh = warp; hh < (uint32_t)G; hh += kDW) {
        const float *qsrc = p.q + ((uint64_t)t * p.n_head + (uint64_t)g * G + hh) * kDHd;
        *reinterpret_cast<float4 *>(&qf[hh][4 * lane]) = *reinterpret_cast<const float4 *>(qsrc + 4 * lane);
        __syncwarp();
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
        const Runs rr = plan_runs(head_base, p.slots, rb, (start + ra) % p.slots, n);
        const uint8_t *kbuf = dsm + (size_t)st * 2 * BB, *vbuf = kbuf + BB;
        if (!mbar_wait_bounded(&full[st], (j / NS) & 1u, p.err, ERR_TIMEOUT_FULL)) {
            ok = false;
            break;
        }
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
            // the block scales: Q8_0 d_k(row, block) * d_q(head, block); turbo4 d_q only
            float kscale = 0.0f;  // of row rowq, this lane's block
#pragma unroll
            for (int i = 0; i < R; i++)
                if ((uint32_t)i == rowq) kscale = K[i].scale;
            float f[32];
#pragma unroll
            for (int jj = 0; jj < 4; jj++) f[jj] = (KV == RCU_KV_Q8_0 ? kscale * dq[jj] : dq[jj]) * (float)v[jj];
            bfly<4>(f, lane, 16);
            bfly<2>(f, lane, 8);
            s = f[0];
            if (KV == RCU_KV_TURBO4) s *= kscale * (1.0f / 46.0f);  // one f16 scale per 128-dim row
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
    float *slot = cluster.map_shared_rank(&cpart[0][0], 0) + (size_t)rank * (G * kDHd + 2 * G);
    for (uint32_t e = tid; e < (uint32_t)G * kDHd; e += kDW * 32) {
        const uint32_t h = e / kDHd, d = e % kDHd;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kDW; w++) M = fmaxf(M, wm[w][h]);
        float o = 0.0f, L = 0.0f;
#pragma unroll
        for (int w = 0; w < kDW; w++) {
            const float f = wm[w][h] == -INFINITY ? 0.0f : expf(wm[w][h] - M);
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
                const float f = mr[r] == -INFINITY ? 0.0f : expf(mr[r] - M);
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
        for (uint32_t e = tid; e < (uint32_t)G * kDHd; e += kDW * 32) {
            const uint32_t h = e / kDHd, d = e % kDHd;
            const uint64_t bh = base + (uint64_t)h * n_cl;
            float M = -INFINITY;
            for (uint32_t c = 0; c < n_cl; c++) M = fmaxf(M, __ldcg(p.m_part + bh + c));
            float o = 0.0f, L = 0.0f;
            for (uint32_t c = 0; c < n_cl; c++) {
                const float m = __ldcg(p.m_part + bh + c);
                const float f = m == -INFINITY ? 0.0f : expf(m - M);
                o = fmaf(f, __ldcg(p.o_part + (bh + c) * kDHd + d), o);
                L = fmaf(f, __ldcg(p.l_part + bh + c), L);
            }
            vals[e] = o;
            if (d == 0) fl[h] = L;
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

}  // namespace

bool attention_dec_ok(int kv_type, uint64_t hd, uint64_t group) {
    (void)kv_type;
    return hd == kDHd && (group == 4 || group == 8);
}

// Splits of the context per (token, KV head): at least 64 rows each, about one CTA per SM in
// all, a multiple of the cluster size (<= 8).
static void dec_plan(uint64_t max_len, uint64_t n_tok, uint64_t n_kv, int num_sms, uint32_t *n_split, uint32_t *cs,
                     uint32_t *rows) {
    const uint64_t want = std::max<uint64_t>(1, (uint64_t)num_sms / std::max<uint64_t>(1, n_kv * n_tok));
    uint64_t ns = std::max<uint64_t>(1, std::min<uint64_t>((max_len + 63) / 64, want));
    // one cluster up to 8 splits; beyond, clusters of 4 (clusters of 8 CTAs that each fill an SM
    // do not all fit in one wave on B200: 15 of them at a time)
    const uint64_t c = ns <= kDMaxCluster ? ns : 4;
    ns = std::max<uint64_t>(c, ns / c * c);
    *n_split = (uint32_t)ns;
    *cs = (uint32_t)c;
    *rows = (uint32_t)((max_len + ns - 1) / ns);
}

uint32_t attention_dec_max_clusters(uint64_t max_len, uint64_t n_tok, uint64_t n_kv, int num_sms) {
    uint32_t ns, cs, rows;
    dec_plan(max_len, n_tok, n_kv, num_sms, &ns, &cs, &rows);
    return ns / cs;
}

template <int KV, int G>
static int launch_dec(rcu_ctx *ctx, DecParams &p, dim3 grid) {
    auto kern = k_attn_dec<KV, G>;
    static int budget_of[64] = {};  // per device: opt-in limit minus the kernel's static shared memory
    int &budget = budget_of[ctx->device & 63];
    if (!budget) {
        cudaFuncAttributes fa;
        RCU_CUDA_TRY(ctx, cudaFuncGetAttributes(&fa, kern));
        const int lim = (int)ctx->max_smem_optin - (int)fa.sharedSizeBytes;
        RCU_CUDA_TRY(ctx, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, lim));
        budget = lim;
    }
    // stages: up to 256 rows (and at least two stages in the budget), 2 to 4 of them
    const uint32_t rb = p.row_bytes;
    const uint32_t sr_fit = (uint32_t)(((uint64_t)budget / 4 > 64 ? ((uint64_t)budget / 4 - 64) / rb : 0) / 16 * 16);
    const uint32_t want = (p.rows_per_split + 15) / 16 * 16;
    p.stage_rows = std::max<uint32_t>(16, std::min<uint32_t>(std::min<uint32_t>(sr_fit, 256), want));
    p.buf_bytes = (p.stage_rows * rb + 64 + 15) / 16 * 16;  // + the two ranges' 16-byte enclosures
    const uint32_t n_stage = (p.rows_per_split + p.stage_rows - 1) / p.stage_rows;
    p.n_stages = std::max<uint32_t>(1, std::min<uint32_t>(std::min<uint32_t>(kDMaxStages, n_stage),
                                                          (uint32_t)budget / (2 * p.buf_bytes)));
    const uint32_t wo_bytes = kDW * G * kDHd * 4;
    const uint32_t dyn = std::max<uint32_t>(p.n_stages * 2 * p.buf_bytes, wo_bytes);
    if ((int)dyn > budget) return set_err(ctx, RCU_ERR_UNSUPPORTED, "attention: stage buffers exceed shared memory");
    if (cudaError_t e = prefer_max_shared(reinterpret_cast<const void *>(kern))) return cuda_err(ctx, e, "attention");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
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

int launch_attention_dec(rcu_ctx *ctx, const uint8_t *kc, const uint8_t *vc, int kv_type, uint64_t n_kv,
                         uint64_t slots, uint64_t row_bytes, const float *q, uint64_t n_tok, uint64_t n_head,
                         uint64_t pos0, const uint64_t *pos_ptr, uint64_t max_len, uint64_t window, float softcap,
                         float *out, const ActOut *aq, uint32_t *done, float *parts) {
    if (kv_type == RCU_KV_TURBO4)
        if (int st = ensure_signs(ctx)) return st;
    DecParams p{};
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
    dec_plan(max_len, n_tok, n_kv, ctx->num_sms, &p.n_split, &p.cs, &p.rows_per_split);
    const uint64_t n_cl = p.n_split / p.cs, parts_n = n_tok * n_head * n_cl;
    p.done = done;
    p.o_part = parts;
    p.m_part = parts + parts_n * kDHd;
    p.l_part = p.m_part + parts_n;
    const dim3 grid(p.n_split, (uint32_t)n_kv, (uint32_t)n_tok);
    const uint64_t group = n_head / n_kv;
    switch (kv_type) {
        case RCU_KV_F16: return group == 4 ? launch_dec<RCU_KV_F16, 4>(ctx, p, grid) : launch_dec<RCU_KV_F16, 8>(ctx, p, grid);
        case RCU_KV_Q8_0: return group == 4 ? launch_dec<RCU_KV_Q8_0, 4>(ctx, p, grid) : launch_dec<RCU_KV_Q8_0, 8>(ctx, p, grid);
        default: return group == 4 ? launch_dec<RCU_KV_TURBO4, 4>(ctx, p, grid) : launch_dec<RCU_KV_TURBO4, 8>(ctx, p, grid);
    }
}

}  // namespace rcu
