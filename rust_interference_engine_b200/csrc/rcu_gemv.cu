// rcu_gemv.cu -- decode GEMV: y[t][r] = W[r] . X[t] for up to 8 activation rows, over
// weights kept in their GGUF block layout (Q4_0/Q4_1/Q5_0/Q5_1/Q8_0 x Q8_0 activations,
// Q4_K/Q5_K/Q6_K x Q8_K activations). Replaces kernels/matmul.rs:136-241 (matmul_multi,
// compute_rows) and the vec_dot family of kernels/mod.rs:134-232 for the decode case.
//
// Design (HBM-bound; every weight byte is read exactly once per call):
//   * persistent CTAs, one per SM; each walks a static list of row tiles covering all jobs
//     of the call (several weights share one launch, like matmul_multi's single region);
//   * warp 8 is a TMA producer: 1-D bulk copies (cp.async.bulk) stream whole row tiles
//     (contiguous GGUF bytes) into a ring of shared-memory stages, completion counted on
//     mbarriers, L2 evict-first;
//   * warps 0..7 consume: the quantized activations of the call sit in shared memory;
//     each lane unpacks GGUF blocks from the stage with word loads + funnel shifts and
//     forms the exact per-block int32 sums with dp4a, then combines in f32 like the
//     reference (d_w * d_a * s [+ m_w * s_a]); warp shuffles reduce each row.
//   * large rows are split over 2/4/8 warps; the last warp to finish combines the
//     partials in a fixed order (deterministic, no block-wide barrier inside the loop).
//   * every wait is bounded (2 s) and reports through the context's device error word.
#include <algorithm>
#include <atomic>

#include "rcu_blocks.cuh"
#include "rcu_kernels.h"

namespace rcu {

constexpr int kConsumerWarps = 16;  // upper bound; 1-2 token launches use 16, more tokens 8

constexpr int kMaxJobs = 96;
constexpr int kMaxTok = 8;
constexpr int kMaxStages = 8;
constexpr int kMaxRw = 2;  // weight rows per warp per tile
constexpr uint32_t kHdrBytes = 6144;  // barriers + reduction scratch
constexpr int kMaxPeers = 8;
constexpr uint32_t kMaxStageRows = 64;

struct GemvJobDev {
    const uint8_t *w;
    float *out;
    uint64_t ld;
    uint32_t rows, row_bytes;
    int32_t type;
    uint32_t rows_per_tile, tile_begin, wpr, rw;
    // indirect (mixture-of-experts) jobs: the weight is w + (*sel) * w_stride, chosen on
    // the device by the router; the job's activations start at staged row `tok`
    const uint32_t *sel;
    uint64_t w_stride;
    uint32_t tok;
};

struct GemvParams {
    GemvJobDev jobs[kMaxJobs];
    int32_t n_jobs;
    uint32_t total_tiles, stages, stage_bytes, stage_off;
    uint32_t k, n_tok, tok0, formats;
    uint32_t n_stage;  // activation rows staged in shared memory (>= n_tok + every job's tok)
    uint32_t early_weights;  // producer may load weights before the previous kernel ends
    // shared-memory offsets of the staged activations
    uint32_t o_q0, o_d0, o_s0, o_sum0, o_qk, o_dk, o_bsk;
    ActsView acts;
    uint32_t *err;
    // Fused all-reduce push (tensor parallel, one job): every output value is also stored
    // to ar_dst[q][t * ld + row] (peer GPUs' receive buffers, NVLink), and each CTA adds to
    // ar_flag[q] (every rank, itself included) once its rows are written, kArUnit per launch.
    float *ar_dst[kMaxPeers];
    uint32_t *ar_flag[kMaxPeers];
    uint32_t ar_ndst, ar_nflag;
    // block-sum capture (the k_gemv<1, 16, true> instantiation only): every exact per-block
    // integer sum of a row of token 0, in the layout of rcu_block_sums, added into
    // dbg[row * dbg_nbs + i]
    int32_t *dbg;
    uint32_t dbg_nbs;
};

struct SmemHdr {
    uint64_t full[kMaxStages];
    uint64_t empty[kMaxStages];
    int cnt[kMaxStages][kConsumerWarps];
    float red[kMaxStages][kConsumerWarps][kMaxTok];  // [stage][row in tile * wpr + part][token]
};
static_assert(sizeof(SmemHdr) <= kHdrBytes, "header too large");

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Output store of token t, row `row`: the job's own buffer, plus the peers' receive
// buffers when the launch pushes an all-reduce.
__device__ __forceinline__ void store_out(const GemvParams &p, const GemvJobDev &jb, uint32_t t, uint32_t row,
                                          float v) {
    const uint64_t at = (uint64_t)t * jb.ld + row;
    jb.out[at] = v;
    for (uint32_t q = 0; q < p.ar_ndst; q++) p.ar_dst[q][at] = v;
}

// Publish one warp's finished row sums v[t] (valid in every lane). With wpr > 1 the last
// of the row's warps to arrive adds the parts in order 0..wpr-1 and stores the row.
template <int T>
__device__ __forceinline__ void emit_row(const GemvParams &p, SmemHdr *h, int s, const GemvJobDev &jb, uint32_t row,
                                         int row_in_tile, int part, const float (&v)[T], int lane) {
    if (jb.wpr == 1) {
        if (lane < T) {
            float x = v[0];
#pragma unroll
            for (int t = 1; t < T; t++)
                if (lane == t) x = v[t];
            store_out(p, jb, lane, row, x);
        }
        return;
    }
    if (lane < T) {
        float x = v[0];
#pragma unroll
        for (int t = 1; t < T; t++)
            if (lane == t) x = v[t];
        h->red[s][row_in_tile * jb.wpr + part][lane] = x;
    }
    __syncwarp();
    __threadfence_block();
    int old = 0;
    if (lane == 0) old = atomicAdd(&h->cnt[s][row_in_tile], 1);
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old == (int)jb.wpr - 1) {
        __threadfence_block();
        if (lane < T) {
            float acc = 0.0f;
            for (uint32_t q = 0; q < jb.wpr; q++) acc += *((volatile float *)&h->red[s][row_in_tile * jb.wpr + q][lane]);
            store_out(p, jb, lane, row, acc);
        }
        __syncwarp();
        if (lane == 0) h->cnt[s][row_in_tile] = 0;
    }
}

// Reduce each row's per-lane partials over the warp and store the rows. Two rows share the
// first butterfly stage (lanes 0-15 end with row 0, lanes 16-31 with row 1).
template <int T>
__device__ __forceinline__ void finish_rows(const GemvParams &p, SmemHdr *h, int s, const GemvJobDev &jb, uint32_t r0,
                                            uint32_t row_first, uint32_t nr, int part, float (&acc)[kMaxRw][T],
                                            int lane) {
    if (kMaxRw == 2 && nr == 2 && jb.wpr == 1) {
        const bool up = lane & 16;
        float v[T];
#pragma unroll
        for (int t = 0; t < T; t++) {
            const float give = up ? acc[0][t] : acc[1][t];
            float keep = up ? acc[1][t] : acc[0][t];
            keep += __shfl_xor_sync(0xffffffffu, give, 16);
#pragma unroll
            for (int o = 8; o; o >>= 1) keep += __shfl_xor_sync(0xffffffffu, keep, o);
            v[t] = keep;
        }
        const int tl = lane & 15;
        if (tl < T) {
            float x = v[0];
#pragma unroll
            for (int t = 1; t < T; t++)
                if (tl == t) x = v[t];
            store_out(p, jb, tl, r0 + row_first + (up ? 1 : 0), x);
        }
        return;
    }
#pragma unroll
    for (int r = 0; r < kMaxRw; r++) {
        if ((uint32_t)r < nr) {
            float v[T];
#pragma unroll
            for (int t = 0; t < T; t++) v[t] = warp_sum(acc[r][t]);
            emit_row<T>(p, h, s, jb, r0 + row_first + r, row_first + r, part, v, lane);
        }
    }
}

// ---- 32-value block types: one block per lane per step ----------------------------------
template <int TYPE, int T, bool DBG>
__device__ __forceinline__ void tile_q(const GemvParams &p, SmemHdr *h, int s, const uint8_t *wsm, const GemvJobDev &jb,
                                       uint32_t r0, uint32_t nrows, const uint8_t *sm, int warp, int lane) {
    constexpr uint32_t BB = blk_bytes_c<TYPE>();
    const uint32_t nb = p.k / QK;
    uint32_t row_first, nr, b_begin, b_end;
    int part = 0;
    if (jb.wpr == 1) {
        row_first = warp * jb.rw;
        nr = jb.rw;
        b_begin = 0;
        b_end = nb;
    } else {
        row_first = warp / jb.wpr;
        part = warp % jb.wpr;
        nr = 1;
        b_begin = part * nb / jb.wpr;
        b_end = (part + 1) * nb / jb.wpr;
    }
    if (row_first >= nrows) return;
    if (row_first + nr > nrows) nr = nrows - row_first;
    const int8_t *aq = reinterpret_cast<const int8_t *>(sm + p.o_q0) + (size_t)jb.tok * p.k;
    const float *ad = reinterpret_cast<const float *>(sm + p.o_d0) + (size_t)jb.tok * nb;
    const float *as = reinterpret_cast<const float *>(sm + p.o_s0) + (size_t)jb.tok * nb;
    const int32_t *asm_ = reinterpret_cast<const int32_t *>(sm + p.o_sum0) + (size_t)jb.tok * nb;
    const uint32_t rb = jb.row_bytes, wrow0 = row_first * rb;
    float acc[kMaxRw][T];
#pragma unroll
    for (int r = 0; r < kMaxRw; r++)
#pragma unroll
        for (int t = 0; t < T; t++) acc[r][t] = 0.0f;
    for (uint32_t b = b_begin + lane; b < b_end; b += 32) {
        uint32_t a[T][8];
        int asum[T];
        float da[T], sa[T];
#pragma unroll
        for (int t = 0; t < T; t++) {
            const uint4 *src = reinterpret_cast<const uint4 *>(aq + (size_t)t * p.k + (size_t)b * QK);
            const uint4 x0 = src[0], x1 = src[1];
            a[t][0] = x0.x, a[t][1] = x0.y, a[t][2] = x0.z, a[t][3] = x0.w;
            a[t][4] = x1.x, a[t][5] = x1.y, a[t][6] = x1.z, a[t][7] = x1.w;
            asum[t] = (TYPE == T_Q4_0 || TYPE == T_Q5_0) ? asm_[t * nb + b] : 0;
            da[t] = ad[t * nb + b];
            sa[t] = (TYPE == T_Q4_1 || TYPE == T_Q5_1) ? as[t * nb + b] : 0.0f;
        }
#pragma unroll
        for (int r = 0; r < kMaxRw; r++) {
            if ((uint32_t)r < nr) {
                BlkW w;
                dec_blk<TYPE>(wsm, wrow0 + r * rb + b * BB, w);
#pragma unroll
                for (int t = 0; t < T; t++) {
                    const int si = blk_int<TYPE>(w, a[t], asum[t]);
                    if constexpr (DBG) {
                        if (t == 0) p.dbg[(uint64_t)(r0 + row_first + r) * p.dbg_nbs + b] = si;
                    }
                    float c = (w.d * da[t]) * (float)si;  // f16(d) * ab.d * s
                    if (TYPE == T_Q4_1 || TYPE == T_Q5_1) c += w.m * sa[t];
                    acc[r][t] += c;
                }
            }
        }
    }
    finish_rows<T>(p, h, s, jb, r0, row_first, nr, part, acc, lane);
}

// ---- 256-value superblock types: 4 groups of 8 lanes per warp, a superblock per group -----
// Each lane keeps its own f32 partial of every row; one warp reduction per row at the end
// (the sum of per-lane partials differs from the reference's per-superblock order only by
// f32 rounding).
template <int TYPE, int T, bool DBG>
__device__ __forceinline__ void tile_k(const GemvParams &p, SmemHdr *h, int s, const uint8_t *wsm, const GemvJobDev &jb,
                                       uint32_t r0, uint32_t nrows, const uint8_t *sm, int warp, int lane) {
    constexpr uint32_t BB = TYPE == T_Q4_K ? 144 : TYPE == T_Q5_K ? 176 : 210;
    const uint32_t nsb = p.k / QK_K;
    uint32_t row_first, nr, b_begin, b_end;
    int part = 0;
    if (jb.wpr == 1) {
        row_first = warp * jb.rw;
        nr = jb.rw;
        b_begin = 0;
        b_end = nsb;
    } else {
        row_first = warp / jb.wpr;
        part = warp % jb.wpr;
        nr = 1;
        b_begin = part * nsb / jb.wpr;
        b_end = (part + 1) * nsb / jb.wpr;
    }
    if (row_first >= nrows) return;
    if (row_first + nr > nrows) nr = nrows - row_first;
    const uint32_t g = lane >> 3, sub = lane & 7;
    const int8_t *aq = reinterpret_cast<const int8_t *>(sm + p.o_qk) + (size_t)jb.tok * p.k;
    const float *adk = reinterpret_cast<const float *>(sm + p.o_dk) + (size_t)jb.tok * nsb;
    const uint32_t *abs2 = reinterpret_cast<const uint32_t *>(sm + p.o_bsk) + (size_t)jb.tok * (p.k / 32);  // bsums pairs
    const uint32_t rb = jb.row_bytes, wrow0 = row_first * rb;
    float acc[kMaxRw][T];
#pragma unroll
    for (int r = 0; r < kMaxRw; r++)
#pragma unroll
        for (int t = 0; t < T; t++) acc[r][t] = 0.0f;
    if (TYPE == T_Q6_K) {
        const Q6Lane l = q6_lane(sub);
        const uint32_t aoff = 128 * l.n + 8 * l.lq;
        for (uint32_t sb = b_begin + g; sb < b_end; sb += 4) {
            uint2 a[T][4];
            uint32_t bs2[T];
            float ad[T];
#pragma unroll
            for (int t = 0; t < T; t++) {
                const int8_t *base = aq + (size_t)t * p.k + (size_t)sb * QK_K + aoff;
#pragma unroll
                for (int k = 0; k < 4; k++) a[t][k] = *reinterpret_cast<const uint2 *>(base + 32 * k);
                bs2[t] = abs2[(size_t)t * (p.k / 32) + 8 * sb + sub];
                ad[t] = adk[t * nsb + sb];
            }
#pragma unroll
            for (int r = 0; r < kMaxRw; r++) {
                if ((uint32_t)r < nr) {
#pragma unroll
                    for (int t = 0; t < T; t++) {
                        int I;
                        const uint32_t db = q6_lane_dot(l, wsm, wrow0 + r * rb + sb * BB, a[t], bs2[t], I);
                        acc[r][t] += (f16_bits_to_f32(db) * ad[t]) * (float)I;
                        if constexpr (DBG) {
                            if (t == 0) atomicAdd(p.dbg + (uint64_t)(r0 + row_first + r) * p.dbg_nbs + sb, I);
                        }
                    }
                }
            }
        }
    } else {
        const KLane l = k_lane(sub);
        const uint32_t alo_off = 64 * l.j + 16 * l.h;
        for (uint32_t sb = b_begin + g; sb < b_end; sb += 4) {
            uint4 alo[T], ahi[T];
            uint32_t bs2[T];
            float ad[T];
#pragma unroll
            for (int t = 0; t < T; t++) {
                const int8_t *base = aq + (size_t)t * p.k + (size_t)sb * QK_K + alo_off;
                alo[t] = *reinterpret_cast<const uint4 *>(base);
                ahi[t] = *reinterpret_cast<const uint4 *>(base + 32);
                bs2[t] = abs2[(size_t)t * (p.k / 32) + 8 * sb + sub];
                ad[t] = adk[t * nsb + sb];
            }
#pragma unroll
            for (int r = 0; r < kMaxRw; r++) {
                if ((uint32_t)r < nr) {
                    const uint8_t *sbp = wsm + wrow0 + r * rb + sb * BB;
#pragma unroll
                    for (int t = 0; t < T; t++) {
                        int I, M;
                        const uint32_t dm = k_lane_dot<TYPE>(l, sbp, alo[t], ahi[t], bs2[t], I, M);
                        if constexpr (DBG) {
                            if (t == 0) {
                                int32_t *d = p.dbg + (uint64_t)(r0 + row_first + r) * p.dbg_nbs + 2 * sb;
                                atomicAdd(d, I);
                                atomicAdd(d + 1, M);
                            }
                        }
                        // d * sumi - dmin * summ with d = f16(d)*ab.d, dmin = f16(dmin)*ab.d
                        const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&dm));
                        acc[r][t] = fmaf(ad[t], fmaf(-f.y, (float)M, f.x * (float)I), acc[r][t]);
                    }
                }
            }
        }
    }
    finish_rows<T>(p, h, s, jb, r0, row_first, nr, part, acc, lane);
}

template <int T, int NW, bool DBG = false>
__global__ void __launch_bounds__((NW + 1) * 32, 1) k_gemv(const __grid_constant__ GemvParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    SmemHdr *h = reinterpret_cast<SmemHdr *>(smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t S = p.stages;
    pdl_trigger();
    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < S; s++) {
            mbar_init(&h->full[s], 1);
            mbar_init(&h->empty[s], NW);
        }
        fence_mbar_init();
    }
    for (uint32_t i = threadIdx.x; i < kMaxStages * kConsumerWarps; i += blockDim.x) (&h->cnt[0][0])[i] = 0;
    __syncthreads();

    if (warp == NW) {  // ---- producer ----
        if (!p.early_weights) pdl_wait();
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            uint32_t li = 0, s = 0, ph = 0;  // tile count, stage, pass parity (li / S) & 1
            int ji = 0;  // tiles are visited in increasing order: the job index only advances
            for (uint32_t tile = blockIdx.x; tile < p.total_tiles; tile += gridDim.x, ++li) {
                if (li >= S && !mbar_wait_bounded(&h->empty[s], ph ^ 1u, p.err, ERR_TIMEOUT_EMPTY)) break;
                while (ji + 1 < p.n_jobs && p.jobs[ji + 1].tile_begin <= tile) ji++;
                const GemvJobDev &jb = p.jobs[ji];
                const uint32_t r0 = (tile - jb.tile_begin) * jb.rows_per_tile;
                const uint32_t nrows = min(jb.rows_per_tile, jb.rows - r0);
                const uint32_t bytes = (nrows * jb.row_bytes + 15u) & ~15u;
                uint8_t *dst = smem + p.stage_off + s * p.stage_bytes;
                const uint32_t ex = jb.sel ? *jb.sel : 0;
                if (ex == kNoExpert) {  // routed to an expert of another rank: nothing to load
                    mbar_arrive(&h->full[s]);
                } else {
                    mbar_arrive_expect_tx(&h->full[s], bytes);
                    bulk_g2s(dst, jb.w + (uint64_t)ex * jb.w_stride + (uint64_t)r0 * jb.row_bytes, bytes, &h->full[s],
                             pol);
                }
                if (++s == S) {
                    s = 0;
                    ph ^= 1u;
                }
            }
            // never leave the CTA with copies in flight: wait for the last phase of each stage
            const uint32_t issued = li;
            for (uint32_t s = 0; s < S && s < issued; s++) {
                const uint32_t last = ((issued - 1 - s) / S) * S + s;  // last li with li % S == s
                mbar_wait_bounded(&h->full[s], (last / S) & 1, p.err, ERR_TIMEOUT_DRAIN);
            }
        }
        return;
    }

    // ---- consumers: stage this call's quantized activations -------------------------------
    // (with early_weights the producer streams weights before the previous kernel ends;
    // everything else waits for it)
    pdl_wait();
    {
        const uint32_t nt = p.n_stage, k = p.k, tid = threadIdx.x, nthr = NW * 32;
        const ActsView &A = p.acts;
        if (p.formats & RCU_ACT_Q8_0) {
            const uint32_t nb = k / QK;
            const uint4 *src = reinterpret_cast<const uint4 *>(A.q0 + (size_t)p.tok0 * k);
            uint4 *dst = reinterpret_cast<uint4 *>(smem + p.o_q0);
            for (uint32_t i = tid; i < nt * k / 16; i += nthr) dst[i] = src[i];
            for (uint32_t i = tid; i < nt * nb; i += nthr) {
                reinterpret_cast<float *>(smem + p.o_d0)[i] = A.d0[(size_t)p.tok0 * nb + i];
                reinterpret_cast<float *>(smem + p.o_s0)[i] = A.s0[(size_t)p.tok0 * nb + i];
                reinterpret_cast<int32_t *>(smem + p.o_sum0)[i] = A.sum0[(size_t)p.tok0 * nb + i];
            }
        }
        if (p.formats & RCU_ACT_Q8K) {
            const uint32_t nsb = k / QK_K;
            const uint4 *src = reinterpret_cast<const uint4 *>(A.qk + (size_t)p.tok0 * k);
            uint4 *dst = reinterpret_cast<uint4 *>(smem + p.o_qk);
            for (uint32_t i = tid; i < nt * k / 16; i += nthr) dst[i] = src[i];
            for (uint32_t i = tid; i < nt * nsb; i += nthr)
                reinterpret_cast<float *>(smem + p.o_dk)[i] = A.dk[(size_t)p.tok0 * nsb + i];
            const uint32_t *bsrc = reinterpret_cast<const uint32_t *>(A.bsk + (size_t)p.tok0 * (k / 16));
            for (uint32_t i = tid; i < nt * k / 32; i += nthr) reinterpret_cast<uint32_t *>(smem + p.o_bsk)[i] = bsrc[i];
        }
        named_bar_sync(1, NW * 32);
    }

    uint32_t s = 0, ph = 0;
    int ji = 0;
    for (uint32_t tile = blockIdx.x; tile < p.total_tiles; tile += gridDim.x) {
        if (!mbar_wait_bounded(&h->full[s], ph, p.err, ERR_TIMEOUT_FULL)) break;
        while (ji + 1 < p.n_jobs && p.jobs[ji + 1].tile_begin <= tile) ji++;
        const GemvJobDev &jb = p.jobs[ji];
        const uint32_t r0 = (tile - jb.tile_begin) * jb.rows_per_tile;
        const uint32_t nrows = min(jb.rows_per_tile, jb.rows - r0);
        const uint8_t *wsm = smem + p.stage_off + s * p.stage_bytes;
        switch (jb.sel && *jb.sel == kNoExpert ? -1 : jb.type) {
            case T_Q4_0: tile_q<T_Q4_0, T, DBG>(p, h, s, wsm, jb, r0, nrows, smem, warp, lane); break;
            case T_Q4_1: tile_q<T_Q4_1, T, DBG>(p, h, s, wsm, jb, r0, nrows, smem, warp, lane); break;
            case T_Q5_0: tile_q<T_Q5_0, T, DBG>(p, h, s, wsm, jb, r0, nrows, smem, warp, lane); break;
            case T_Q5_1: tile_q<T_Q5_1, T, DBG>(p, h, s, wsm, jb, r0, nrows, smem, warp, lane); break;
            case T_Q8_0: tile_q<T_Q8_0, T, DBG>(p, h, s, wsm, jb, r0, nrows, smem, warp, lane); break;
            case T_Q4_K: tile_k<T_Q4_K, T, DBG>(p, h, s, wsm, jb, r0, nrows, smem, warp, lane); break;
            case T_Q5_K: tile_k<T_Q5_K, T, DBG>(p, h, s, wsm, jb, r0, nrows, smem, warp, lane); break;
            case T_Q6_K: tile_k<T_Q6_K, T, DBG>(p, h, s, wsm, jb, r0, nrows, smem, warp, lane); break;
            default: break;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&h->empty[s]);
        if (++s == S) {
            s = 0;
            ph ^= 1u;
        }
    }
    if (p.ar_nflag) {  // this CTA's rows are in every receive buffer: count it in
        __threadfence_system();
        named_bar_sync(1, NW * 32);
        // every launch adds exactly kArUnit to each counter, whatever its grid: CTA 0 adds
        // kArUnit - (grid - 1), the others 1
        const uint32_t add = blockIdx.x == 0 ? kArUnit - (gridDim.x - 1) : 1u;
        if (threadIdx.x == 0)
            for (uint32_t q = 0; q < p.ar_nflag; q++) atomicAdd_system(p.ar_flag[q], add);
    }
}

// ---- exact per-block integer sums of one (row, token) pair (validation path) ----------
// The same lane decoders as the GEMV; K-quant lane shares are reduced over the 8 lanes.
__global__ void __launch_bounds__(32) k_block_sums(const uint8_t *__restrict__ wrow, uint32_t row_bytes, int type,
                                                  ActsView A, uint32_t tok, int32_t *__restrict__ out) {
    extern __shared__ __align__(16) uint8_t srow[];
    const int lane = threadIdx.x;
    for (uint32_t i = lane; i < row_bytes; i += 32) srow[i] = wrow[i];
    if (lane < 16) srow[row_bytes + lane] = 0;
    __syncwarp();
    const uint32_t k = A.k;
    if (block_size(type) == QK) {
        const uint32_t nb = k / QK;
        const int8_t *aq = A.q0 + (size_t)tok * k;
        for (uint32_t b = lane; b < nb; b += 32) {
            uint32_t a[8];
            const uint4 x0 = reinterpret_cast<const uint4 *>(aq + b * QK)[0];
            const uint4 x1 = reinterpret_cast<const uint4 *>(aq + b * QK)[1];
            a[0] = x0.x, a[1] = x0.y, a[2] = x0.z, a[3] = x0.w, a[4] = x1.x, a[5] = x1.y, a[6] = x1.z, a[7] = x1.w;
            const int asum = A.sum0[(size_t)tok * nb + b];
            BlkW w;
            int s = 0;
            switch (type) {
                case T_Q4_0: dec_blk<T_Q4_0>(srow, b * 18, w); s = blk_int<T_Q4_0>(w, a, asum); break;
                case T_Q4_1: dec_blk<T_Q4_1>(srow, b * 20, w); s = blk_int<T_Q4_1>(w, a, asum); break;
                case T_Q5_0: dec_blk<T_Q5_0>(srow, b * 22, w); s = blk_int<T_Q5_0>(w, a, asum); break;
                case T_Q5_1: dec_blk<T_Q5_1>(srow, b * 24, w); s = blk_int<T_Q5_1>(w, a, asum); break;
                case T_Q8_0: dec_blk<T_Q8_0>(srow, b * 34, w); s = blk_int<T_Q8_0>(w, a, asum); break;
            }
            out[b] = s;
        }
        return;
    }
    const uint32_t nsb = k / QK_K;
    const uint32_t g = lane >> 3, sub = lane & 7;
    const int8_t *aq = A.qk + (size_t)tok * k;
    const uint32_t *bs = reinterpret_cast<const uint32_t *>(A.bsk + (size_t)tok * (k / 16));
    for (uint32_t sb0 = 0; sb0 < nsb; sb0 += 4) {
        const uint32_t sb = sb0 + g;
        const bool act = sb < nsb;  // uniform trip count: shuffles below need every lane
        int sumi = 0, summ = 0;
        if (act && type == T_Q6_K) {
            const Q6Lane l = q6_lane(sub);
            uint2 a[4];
            for (int kk = 0; kk < 4; kk++)
                a[kk] = *reinterpret_cast<const uint2 *>(aq + (size_t)sb * QK_K + 128 * l.n + 8 * l.lq + 32 * kk);
            q6_lane_dot(l, srow, sb * 210, a, bs[8 * sb + sub], sumi);
        } else if (act) {
            const KLane l = k_lane(sub);
            const int8_t *base = aq + (size_t)sb * QK_K + 64 * l.j + 16 * l.h;
            const uint4 alo = *reinterpret_cast<const uint4 *>(base), ahi = *reinterpret_cast<const uint4 *>(base + 32);
            if (type == T_Q4_K) {
                k_lane_dot<T_Q4_K>(l, srow + sb * 144, alo, ahi, bs[8 * sb + sub], sumi, summ);
            } else {
                k_lane_dot<T_Q5_K>(l, srow + sb * 176, alo, ahi, bs[8 * sb + sub], sumi, summ);
            }
        }
        for (int o = 4; o; o >>= 1) {
            sumi += __shfl_xor_sync(0xffffffffu, sumi, o);
            summ += __shfl_xor_sync(0xffffffffu, summ, o);
        }
        if (sub == 0 && act) {
            if (type == T_Q6_K) {
                out[sb] = sumi;
            } else {
                out[2 * sb] = sumi;
                out[2 * sb + 1] = summ;
            }
        }
    }
}

int launch_block_sums(rcu_ctx *ctx, const ActsView &a, const rcu_weight *w, uint64_t row, uint64_t tok,
                      int32_t *out) {
    const uint32_t rb = (uint32_t)w->row_bytes;
    const uint32_t smem = (rb + 16 + 15) & ~15u;
    if (smem > 48 * 1024) return set_err(ctx, RCU_ERR_UNSUPPORTED, "block_sums: row too long");
    k_block_sums<<<1, 32, smem, ctx->stream>>>(w->data + row * w->row_bytes, rb, w->type, a, (uint32_t)tok, out);
    RCU_CUDA_TRY(ctx, cudaGetLastError());
    return RCU_OK;
}

// ---- host side -------------------------------------------------------------------------
static uint32_t round_up(uint32_t x, uint32_t a) { return (x + a - 1) / a * a; }

template <int T, int NW, bool DBG = false>
static int launch_t(rcu_ctx *ctx, GemvParams &p, uint32_t smem_bytes, uint32_t grid) {
    static std::atomic<bool> attr_set[64] = {};  // per device; contexts may live on several threads
    if (!attr_set[ctx->device & 63].load(std::memory_order_acquire)) {
        RCU_CUDA_TRY(ctx, cudaFuncSetAttribute(k_gemv<T, NW, DBG>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)ctx->max_smem_optin));
        attr_set[ctx->device & 63].store(true, std::memory_order_release);
    }
    RCU_CUDA_TRY(ctx, launch_k(ctx, (k_gemv<T, NW, DBG>), dim3(grid), dim3((NW + 1) * 32), smem_bytes, p));
    RCU_CUDA_TRY(ctx, cudaGetLastError());
    return RCU_OK;
}

int launch_gemv(rcu_ctx *ctx, const ActsView &a, const HostJob *jobs, int n_jobs, uint32_t tok0, uint32_t n_tok,
                const ArPush *push) {
    if (n_jobs < 1 || n_jobs > kMaxJobs) return set_err(ctx, RCU_ERR_INVALID, "gemv: 1..96 jobs per launch");
    if (n_tok < 1 || n_tok > kMaxTok) return set_err(ctx, RCU_ERR_INVALID, "gemv: 1..8 tokens per launch");
    // one activation row over K-quant weights: the tensor-core GEMV (rcu_gemv_kq.cu), also for
    // launches that push a tensor-parallel all-reduce
    if (ctx->dbg_sums) {  // block-sum capture: the kernel the caller named, one job, token 0
        if (n_jobs != 1 || push || n_tok != 1) return set_err(ctx, RCU_ERR_INVALID, "block-sum capture: one job, one token");
        if (ctx->dbg_kernel == 1) return launch_gemv_kq(ctx, a, jobs, n_jobs, tok0, push);
    } else if (n_tok == 1 && gemv_kq_ok(ctx, a, jobs, n_jobs)) {
        return launch_gemv_kq(ctx, a, jobs, n_jobs, tok0, push);
    }
    GemvParams p{};
    if (push) {
        if (n_jobs != 1 || tok0 != 0 || push->n_dst > kMaxPeers || push->n_flag > kMaxPeers)
            return set_err(ctx, RCU_ERR_INVALID, "gemv: all-reduce push needs one job, one launch, <= 8 ranks");
        p.ar_ndst = push->n_dst;
        p.ar_nflag = push->n_flag;
        for (uint32_t q = 0; q < push->n_dst; q++) p.ar_dst[q] = push->dst[q];
        for (uint32_t q = 0; q < push->n_flag; q++) p.ar_flag[q] = push->flag[q];
    }
    p.n_jobs = n_jobs;
    p.k = a.k;
    p.n_tok = n_tok;
    p.tok0 = tok0;
    p.acts = a;
    p.err = ctx->dev_err;
    p.early_weights = ctx->early_weights ? 1u : 0u;
    uint32_t tiles = 0, stage_bytes = 0;
    for (int i = 0; i < n_jobs; i++) {
        const rcu_weight *w = jobs[i].w;
        GemvJobDev &jd = p.jobs[i];
        jd.w = w->data;
        jd.out = jobs[i].out + (jobs[i].sel ? 0 : (uint64_t)tok0 * jobs[i].ld);  // indirect jobs: own rows
        jd.ld = jobs[i].ld;
        jd.rows = jobs[i].rows ? jobs[i].rows : (uint32_t)w->rows;
        jd.sel = jobs[i].sel;
        jd.w_stride = jobs[i].w_stride;
        jd.tok = jobs[i].tok;
        if (jd.sel) p.early_weights = 0;  // the producer reads the router's choice: wait first
        p.n_stage = std::max(p.n_stage, jd.tok + n_tok);
        jd.row_bytes = (uint32_t)w->row_bytes;
        jd.type = w->type;
        p.formats |= act_format(w->type);
        // Tile = kConsumerWarps * rw rows (or kConsumerWarps / wpr rows when a row is split
        // over wpr warps), about 24-48 KB of contiguous GGUF bytes per bulk copy.
        const uint32_t rb = jd.row_bytes, target = 48u * 1024u, nw = n_tok <= 2 ? 16u : 8u;
        if (nw * rb <= target) {
            jd.wpr = 1;
            jd.rw = std::max(1u, std::min<uint32_t>(kMaxRw, target / (nw * rb)));
            jd.rows_per_tile = nw * jd.rw;
        } else {
            jd.wpr = 2;
            while (jd.wpr < nw && (nw / jd.wpr) * rb > target) jd.wpr *= 2;
            jd.rw = 1;
            jd.rows_per_tile = nw / jd.wpr;
            const uint32_t units = w->cols / block_size(w->type);
            if ((jd.rows_per_tile * rb) % 16 != 0 || units < jd.wpr) {
                jd.wpr = 1;
                jd.rows_per_tile = nw;
            }
        }
        jd.tile_begin = tiles;
        tiles += (jd.rows + jd.rows_per_tile - 1) / jd.rows_per_tile;
        stage_bytes = std::max(stage_bytes, round_up(jd.rows_per_tile * rb, 16) + 16);
    }
    p.total_tiles = tiles;
    p.stage_bytes = stage_bytes;
    // activations staged in shared memory (n_stage rows from tok0)
    if (p.n_stage > kMaxStageRows) return set_err(ctx, RCU_ERR_INVALID, "gemv: more than 64 activation rows");
    const uint32_t n_rows = p.n_stage;
    uint32_t off = kHdrBytes;
    const uint32_t k = a.k;
    if (p.formats & RCU_ACT_Q8_0) {
        const uint32_t nb = k / QK;
        p.o_q0 = off; off = round_up(off + n_rows * k, 16);
        p.o_d0 = off; off = round_up(off + n_rows * nb * 4, 16);
        p.o_s0 = off; off = round_up(off + n_rows * nb * 4, 16);
        p.o_sum0 = off; off = round_up(off + n_rows * nb * 4, 16);
    }
    if (p.formats & RCU_ACT_Q8K) {
        p.o_qk = off; off = round_up(off + n_rows * k, 16);
        p.o_dk = off; off = round_up(off + n_rows * (k / QK_K) * 4, 16);
        p.o_bsk = off; off = round_up(off + n_rows * (k / 16) * 2, 16);
    }
    p.stage_off = round_up(off, 128);
    const uint32_t budget = (uint32_t)ctx->max_smem_optin;
    if (p.stage_off + 2 * stage_bytes > budget) {
        // Long rows at 7-8 tokens (Q8_0 activations of 16384 values: 22.5 KB per staged row)
        // leave no room for two weight stages: run the tokens as two launches of half the
        // batch. Each launch offsets the outputs by its first token; indirect (expert) jobs
        // address their own rows and are never split.
        bool indirect = false;
        for (int i = 0; i < n_jobs; i++) indirect |= jobs[i].sel != nullptr;
        if (n_tok > 1 && !push && !indirect) {
            const uint32_t h = n_tok / 2;
            if (int st = launch_gemv(ctx, a, jobs, n_jobs, tok0, h)) return st;
            return launch_gemv(ctx, a, jobs, n_jobs, tok0 + h, n_tok - h);
        }
        return set_err(ctx, RCU_ERR_UNSUPPORTED, "gemv: activation batch + two weight stages exceed shared memory");
    }
    p.stages = std::min<uint32_t>(kMaxStages, (budget - p.stage_off) / stage_bytes);
    const uint32_t smem_bytes = p.stage_off + p.stages * stage_bytes;
    const uint32_t grid = std::min<uint32_t>(tiles, (uint32_t)ctx->num_sms);
    if (push && grid > kArUnit) return set_err(ctx, RCU_ERR_INVALID, "gemv: grid above the all-reduce counter unit");
    if (ctx->dbg_sums) {
        p.dbg = ctx->dbg_sums;
        p.dbg_nbs = ctx->dbg_nbs;
        return launch_t<1, 16, true>(ctx, p, smem_bytes, grid);
    }
    switch (n_tok) {
        case 1: return launch_t<1, 16>(ctx, p, smem_bytes, grid);
        case 2: return launch_t<2, 16>(ctx, p, smem_bytes, grid);
        case 3: return launch_t<3, 8>(ctx, p, smem_bytes, grid);
        case 4: return launch_t<4, 8>(ctx, p, smem_bytes, grid);
        case 5: return launch_t<5, 8>(ctx, p, smem_bytes, grid);
        case 6: return launch_t<6, 8>(ctx, p, smem_bytes, grid);
        case 7: return launch_t<7, 8>(ctx, p, smem_bytes, grid);
        default: return launch_t<8, 8>(ctx, p, smem_bytes, grid);
    }
}

}  // namespace rcu
