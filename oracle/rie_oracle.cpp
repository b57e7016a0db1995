// rie_oracle.cpp -- TEST INFRASTRUCTURE ONLY: the parity checker and CPU baseline.
//
// A C++ restatement of the Rust Inference Engine's CPU path for quantized matmul and the
// turbo4 KV cache. Paths below are relative to the reference project root.
//
//   block formats, activation quantizers   crates/rie-core/src/quant/mod.rs:12-218
//   weight quantizers q8_0 / q4_0          crates/rie-core/src/quant/mod.rs:265-298
//   dequantize_block, scalar dots          crates/rie-core/src/quant/reference.rs:8-401
//   AVX2 kernels                           crates/rie-core/src/kernels/avx2.rs:38-337
//   x86 dispatch (which type is SIMD)      crates/rie-core/src/kernels/mod.rs:134-296
//   matmul driver / chunking               crates/rie-core/src/kernels/matmul.rs:130-241
//   thread pool for_each                   crates/rie-core/src/threadpool.rs:136-160
//   turbo4                                 crates/rie-core/src/turbo.rs:23-311
//   attention + KV store                   crates/rie-core/src/model/cpu.rs:300-328, 550-658
//   rmsnorm / rope / silu                  crates/rie-core/src/ops.rs:6-109
//   Rng, random_weight                     crates/rie-core/src/testing.rs:9-91
//
// Arithmetic is kept in the reference's order (Rust never contracts a*b+c into an FMA, so
// this file is compiled with -ffp-contract=off; the AVX2 tier uses the same intrinsics and
// therefore the same rounding). The f16 conversion restates crate `half` 2.7.1
// (Cargo.lock), i.e. IEEE round-to-nearest-even, which the reference pins against F16C in
// crates/rie-core/tests/kernels.rs:128-132.
#include "rie_oracle.h"

#include <immintrin.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <condition_variable>
#include <cstring>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

namespace {

constexpr int T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q4_1 = 3, T_Q5_0 = 6, T_Q5_1 = 7, T_Q8_0 = 8,
              T_Q2_K = 10, T_Q3_K = 11, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14, T_BF16 = 30;
constexpr size_t QK = 32, QK_K = 256;

// quant/mod.rs:139-147 and :155-162 (repr(C, align(16)))
struct alignas(16) BlockQ8_0 {
    int8_t qs[QK];
    float d;
    float s;
};
struct alignas(16) BlockQ8K {
    int8_t qs[QK_K];
    int16_t bsums[QK_K / 16];
    float d;
};
static_assert(sizeof(BlockQ8_0) == 48, "BlockQ8_0 layout");
static_assert(sizeof(BlockQ8K) == 304, "BlockQ8K layout");

bool have_avx2() {
    static const bool v = __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma") &&
                          __builtin_cpu_supports("f16c");
    return v;
}
bool simd(int path) { return path == ORC_PATH_AVX2 && have_avx2(); }

// ---- half precision -------------------------------------------------------------------
uint16_t f32_to_f16(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t exp = (x >> 23) & 0xffu;
    const uint32_t man = x & 0x7fffffu;
    if (exp == 0xff) {  // inf / nan (quiet the nan, keep its top payload bits)
        if (man == 0) return (uint16_t)(sign | 0x7c00u);
        return (uint16_t)(sign | 0x7e00u | (man >> 13));
    }
    const int e = (int)exp - 127 + 15;
    if (e >= 0x1f) return (uint16_t)(sign | 0x7c00u);  // overflow -> inf
    if (e <= 0) {                                         // subnormal or zero in f16
        if (e < -10) return (uint16_t)sign;
        const uint32_t m = man | 0x800000u;  // implicit bit
        const int shift = 14 - e;            // bits dropped
        uint32_t h = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1);
        const uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (h & 1u))) h++;
        return (uint16_t)(sign | h);
    }
    uint32_t h = ((uint32_t)e << 10) | (man >> 13);
    const uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;  // may carry into the exponent
    return (uint16_t)(sign | h);
}

float f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t x;
    if (exp == 0) {
        if (man == 0) {
            x = sign;
        } else {  // normalise the subnormal
            int e = -1;
            do {
                man <<= 1;
                e++;
            } while (!(man & 0x400u));
            x = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3ffu) << 13);
        }
    } else if (exp == 0x1f) {
        x = sign | 0x7f800000u | (man << 13);
    } else {
        x = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &x, 4);
    return f;
}

inline float f16_at(const uint8_t *b) { return f16_to_f32((uint16_t)(b[0] | (b[1] << 8))); }
inline float bf16_to_f32(uint16_t h) {
    uint32_t x = (uint32_t)h << 16;
    float f;
    std::memcpy(&f, &x, 4);
    return f;
}
inline void put_f16(uint8_t *p, float v) {
    uint16_t h = f32_to_f16(v);
    p[0] = (uint8_t)h;
    p[1] = (uint8_t)(h >> 8);
}
inline uint32_t rd_u32(const uint8_t *p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

// Rust `f32 as i32`: saturating, NaN -> 0.
inline int32_t sat_i32(float v) {
    if (std::isnan(v)) return 0;
    if (v >= 2147483647.0f) return INT32_MAX;
    if (v <= -2147483648.0f) return INT32_MIN;
    return (int32_t)v;
}
inline int32_t clampi(int32_t v, int32_t lo, int32_t hi) { return v < lo ? lo : (v > hi ? hi : v); }
// Rust f32::round: half away from zero.
inline float rust_round(float v) { return std::round(v); }

size_t block_size(int t) {
    switch (t) {
        case T_F32: case T_F16: case T_BF16: return 1;
        case T_Q4_0: case T_Q4_1: case T_Q5_0: case T_Q5_1: case T_Q8_0: return QK;
        case T_Q2_K: case T_Q3_K: case T_Q4_K: case T_Q5_K: case T_Q6_K: return QK_K;
        default: return 0;
    }
}
size_t block_bytes(int t) {
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
enum ActFmt { ACT_F32 = 0, ACT_Q8_0 = 1, ACT_Q8K = 2 };
int act_format(int t) {
    switch (t) {
        case T_Q4_0: case T_Q4_1: case T_Q5_0: case T_Q5_1: case T_Q8_0: return ACT_Q8_0;
        case T_Q4_K: case T_Q5_K: case T_Q6_K: case T_Q2_K: case T_Q3_K: return ACT_Q8K;
        default: return ACT_F32;
    }
}

// ---- activation quantizers ---------------------------------------------------------
// quant/mod.rs:175-189 (scalar, half-away rounding)
void quantize_q8_0_scalar(const float *x, size_t nb, BlockQ8_0 *out) {
    for (size_t b = 0; b < nb; b++) {
        const float *xb = x + b * QK;
        float amax = 0.0f;
        for (size_t j = 0; j < QK; j++) amax = std::fmax(amax, std::fabs(xb[j]));
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        int32_t sum = 0;
        for (size_t j = 0; j < QK; j++) {
            const int32_t r = sat_i32(rust_round(xb[j] * id));
            out[b].qs[j] = (int8_t)clampi(r, -127, 127);
            sum += out[b].qs[j];
        }
        out[b].d = d;
        out[b].s = d * (float)sum;
    }
}

__attribute__((target("avx2,fma,f16c"))) int32_t hsum_i32x8(__m256i v) {
    __m128i s = _mm_add_epi32(_mm256_castsi256_si128(v), _mm256_extracti128_si256(v, 1));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0x4e));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0xb1));
    return _mm_cvtsi128_si32(s);
}
__attribute__((target("avx2,fma,f16c"))) float hsum_f32x8(__m256 v) {
    __m128 s = _mm_add_ps(_mm256_castps256_ps128(v), _mm256_extractf128_ps(v, 1));
    s = _mm_add_ps(s, _mm_movehl_ps(s, s));
    s = _mm_add_ss(s, _mm_movehdup_ps(s));
    return _mm_cvtss_f32(s);
}

// kernels/avx2.rs:153-184 (round-to-nearest-even conversion; s from the unclamped ints)
__attribute__((target("avx2,fma,f16c"))) void quantize_q8_0_avx2(const float *x, size_t nb, BlockQ8_0 *out) {
    const __m256 sign = _mm256_set1_ps(-0.0f);
    for (size_t b = 0; b < nb; b++) {
        const float *p = x + b * QK;
        __m256 m = _mm256_setzero_ps();
        for (int k = 0; k < 4; k++) m = _mm256_max_ps(m, _mm256_andnot_ps(sign, _mm256_loadu_ps(p + 8 * k)));
        __m128 s = _mm_max_ps(_mm256_castps256_ps128(m), _mm256_extractf128_ps(m, 1));
        s = _mm_max_ps(s, _mm_movehl_ps(s, s));
        s = _mm_max_ss(s, _mm_movehdup_ps(s));
        const float amax = _mm_cvtss_f32(s);
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        const __m256 vid = _mm256_set1_ps(id);
        __m256i isum = _mm256_setzero_si256();
        for (int k = 0; k < 4; k++) {
            const __m256i q = _mm256_cvtps_epi32(_mm256_mul_ps(_mm256_loadu_ps(p + 8 * k), vid));
            isum = _mm256_add_epi32(isum, q);
            alignas(32) int32_t tmp[8];
            _mm256_store_si256((__m256i *)tmp, q);
            for (int l = 0; l < 8; l++) out[b].qs[8 * k + l] = (int8_t)clampi(tmp[l], -127, 127);
        }
        out[b].d = d;
        out[b].s = d * (float)hsum_i32x8(isum);
    }
}

// quant/mod.rs:191-218 (scalar on every ISA; d = 1/iscale may be negative)
void quantize_q8_k(const float *x, size_t nb, BlockQ8K *out) {
    for (size_t b = 0; b < nb; b++) {
        const float *xb = x + b * QK_K;
        BlockQ8K &o = out[b];
        float amax = 0.0f, mx = 0.0f;
        for (size_t j = 0; j < QK_K; j++) {
            if (std::fabs(xb[j]) > amax) {
                amax = std::fabs(xb[j]);
                mx = xb[j];
            }
        }
        if (amax == 0.0f) {
            std::memset(&o, 0, sizeof(o));
            continue;
        }
        const float iscale = -127.0f / mx;
        for (size_t j = 0; j < QK_K; j++) o.qs[j] = (int8_t)clampi(sat_i32(rust_round(iscale * xb[j])), -127, 127);
        for (size_t g = 0; g < 16; g++) {
            int16_t s = 0;
            for (size_t j = 0; j < 16; j++) s = (int16_t)(s + o.qs[g * 16 + j]);
            o.bsums[g] = s;
        }
        o.d = 1.0f / iscale;
    }
}

// ---- dequantization (quant/reference.rs:8-215) -------------------------------------
void scale_min_k4(int j, const uint8_t *q, uint8_t *sc, uint8_t *m) {
    if (j < 4) {
        *sc = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *sc = (uint8_t)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
        *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}
void unpack_k4(const uint8_t *q, uint8_t sc[8], uint8_t mn[8]) {
    for (int j = 0; j < 8; j++) scale_min_k4(j, q, &sc[j], &mn[j]);
}
void unpack_q3k_scales(const uint8_t *s, int8_t out[16]) {
    const uint32_t km1 = 0x03030303u, km2 = 0x0f0f0f0fu;
    uint32_t a[4] = {rd_u32(s), rd_u32(s + 4), rd_u32(s + 8), 0};
    const uint32_t tmp = a[2];
    a[2] = ((a[0] >> 4) & km2) | (((tmp >> 4) & km1) << 4);
    a[3] = ((a[1] >> 4) & km2) | (((tmp >> 6) & km1) << 4);
    a[0] = (a[0] & km2) | ((tmp & km1) << 4);
    a[1] = (a[1] & km2) | (((tmp >> 2) & km1) << 4);
    for (int i = 0; i < 4; i++)
        for (int k = 0; k < 4; k++) out[4 * i + k] = (int8_t)((uint8_t)(a[i] >> (8 * k)) - 32);
}

void dequantize_block(int t, const uint8_t *b, float *y) {
    switch (t) {
        case T_Q4_0: {
            const float d = f16_at(b);
            for (int j = 0; j < 16; j++) {
                y[j] = (float)((b[2 + j] & 0xF) - 8) * d;
                y[j + 16] = (float)((b[2 + j] >> 4) - 8) * d;
            }
            break;
        }
        case T_Q4_1: {
            const float d = f16_at(b), m = f16_at(b + 2);
            for (int j = 0; j < 16; j++) {
                y[j] = (float)(b[4 + j] & 0xF) * d + m;
                y[j + 16] = (float)(b[4 + j] >> 4) * d + m;
            }
            break;
        }
        case T_Q5_0: {
            const float d = f16_at(b);
            const uint32_t qh = rd_u32(b + 2);
            for (int j = 0; j < 16; j++) {
                const uint32_t xh0 = ((qh >> j) << 4) & 0x10, xh1 = (qh >> (j + 12)) & 0x10;
                y[j] = (float)((int32_t)((b[6 + j] & 0xFu) | xh0) - 16) * d;
                y[j + 16] = (float)((int32_t)((b[6 + j] >> 4) | xh1) - 16) * d;
            }
            break;
        }
        case T_Q5_1: {
            const float d = f16_at(b), m = f16_at(b + 2);
            const uint32_t qh = rd_u32(b + 4);
            for (int j = 0; j < 16; j++) {
                const uint32_t xh0 = ((qh >> j) << 4) & 0x10, xh1 = (qh >> (j + 12)) & 0x10;
                y[j] = (float)((b[8 + j] & 0xFu) | xh0) * d + m;
                y[j + 16] = (float)((b[8 + j] >> 4) | xh1) * d + m;
            }
            break;
        }
        case T_Q8_0: {
            const float d = f16_at(b);
            for (size_t j = 0; j < QK; j++) y[j] = (float)(int8_t)b[2 + j] * d;
            break;
        }
        case T_Q2_K: {
            const uint8_t *scales = b, *q0 = b + 16;
            const float d = f16_at(b + 80), mn = f16_at(b + 82);
            int yi = 0, is = 0;
            for (int n = 0; n < 2; n++) {
                const uint8_t *q = q0 + n * 32;
                for (int shift = 0; shift < 8; shift += 2)
                    for (int h = 0; h < 2; h++) {
                        const uint8_t sc = scales[is++];
                        const float dl = d * (float)(sc & 0xF), ml = mn * (float)(sc >> 4);
                        for (int l = 0; l < 16; l++) y[yi++] = dl * (float)((q[l + 16 * h] >> shift) & 3) - ml;
                    }
            }
            break;
        }
        case T_Q3_K: {
            const uint8_t *hm = b, *q0 = b + 32;
            int8_t sc[16];
            unpack_q3k_scales(b + 96, sc);
            const float d_all = f16_at(b + 108);
            uint8_t m = 1;
            int is = 0, yi = 0;
            for (int n = 0; n < 2; n++) {
                const uint8_t *q = q0 + n * 32;
                for (int shift = 0; shift < 8; shift += 2) {
                    for (int h = 0; h < 2; h++) {
                        const float dl = d_all * (float)sc[is++];
                        for (int l = 0; l < 16; l++) {
                            const int idx = l + 16 * h;
                            const int v = ((q[idx] >> shift) & 3) - ((hm[idx] & m) ? 0 : 4);
                            y[yi++] = dl * (float)v;
                        }
                    }
                    m = (uint8_t)(m << 1);
                }
            }
            break;
        }
        case T_Q4_K: {
            const float d = f16_at(b), mn = f16_at(b + 2);
            uint8_t sc[8], m[8];
            unpack_k4(b + 4, sc, m);
            const uint8_t *q = b + 16;
            for (int j = 0; j < 4; j++) {
                const float d1 = d * sc[2 * j], m1 = mn * m[2 * j], d2 = d * sc[2 * j + 1], m2 = mn * m[2 * j + 1];
                for (int l = 0; l < 32; l++) {
                    y[64 * j + l] = d1 * (float)(q[32 * j + l] & 0xF) - m1;
                    y[64 * j + 32 + l] = d2 * (float)(q[32 * j + l] >> 4) - m2;
                }
            }
            break;
        }
        case T_Q5_K: {
            const float d = f16_at(b), mn = f16_at(b + 2);
            uint8_t sc[8], m[8];
            unpack_k4(b + 4, sc, m);
            const uint8_t *qh = b + 16, *ql = b + 48;
            for (int j = 0; j < 4; j++) {
                const float d1 = d * sc[2 * j], m1 = mn * m[2 * j], d2 = d * sc[2 * j + 1], m2 = mn * m[2 * j + 1];
                const uint8_t u1 = (uint8_t)(1u << (2 * j)), u2 = (uint8_t)(2u << (2 * j));
                for (int l = 0; l < 32; l++) {
                    const int h1 = (qh[l] & u1) ? 16 : 0, h2 = (qh[l] & u2) ? 16 : 0;
                    y[64 * j + l] = d1 * (float)((ql[32 * j + l] & 0xF) + h1) - m1;
                    y[64 * j + 32 + l] = d2 * (float)((ql[32 * j + l] >> 4) + h2) - m2;
                }
            }
            break;
        }
        case T_Q6_K: {
            const float d = f16_at(b + 208);
            for (int n = 0; n < 2; n++) {
                const uint8_t *ql = b + 64 * n, *qh = b + 128 + 32 * n;
                const int8_t *sc = (const int8_t *)(b + 192 + 8 * n);
                float *yy = y + 128 * n;
                for (int l = 0; l < 32; l++) {
                    const int is = l / 16;
                    const int q1 = ((ql[l] & 0xF) | ((qh[l] & 3) << 4)) - 32;
                    const int q2 = ((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                    const int q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                    const int q4 = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                    yy[l] = d * (float)sc[is] * (float)q1;
                    yy[l + 32] = d * (float)sc[is + 2] * (float)q2;
                    yy[l + 64] = d * (float)sc[is + 4] * (float)q3;
                    yy[l + 96] = d * (float)sc[is + 6] * (float)q4;
                }
            }
            break;
        }
        default: break;
    }
}

// ---- scalar int8 dots with per-block integer sums (quant/reference.rs:221-386) -------
// Each returns the f32 dot and, if bs != nullptr, the exact per-block integer sums.
float dot_q4_0_s(const uint8_t *w, const BlockQ8_0 *a, size_t nb, int32_t *bs) {
    float sum = 0.0f;
    for (size_t i = 0; i < nb; i++) {
        const uint8_t *b = w + i * 18, *qs = b + 2;
        int32_t s = 0;
        for (int j = 0; j < 16; j++) {
            s += ((qs[j] & 0xF) - 8) * a[i].qs[j];
            s += ((qs[j] >> 4) - 8) * a[i].qs[j + 16];
        }
        if (bs) bs[i] = s;
        sum += f16_at(b) * a[i].d * (float)s;
    }
    return sum;
}
float dot_q4_1_s(const uint8_t *w, const BlockQ8_0 *a, size_t nb, int32_t *bs) {
    float sum = 0.0f;
    for (size_t i = 0; i < nb; i++) {
        const uint8_t *b = w + i * 20, *qs = b + 4;
        int32_t s = 0;
        for (int j = 0; j < 16; j++) {
            s += (qs[j] & 0xF) * a[i].qs[j];
            s += (qs[j] >> 4) * a[i].qs[j + 16];
        }
        if (bs) bs[i] = s;
        sum += f16_at(b) * a[i].d * (float)s + f16_at(b + 2) * a[i].s;
    }
    return sum;
}
float dot_q5_0_s(const uint8_t *w, const BlockQ8_0 *a, size_t nb, int32_t *bs) {
    float sum = 0.0f;
    for (size_t i = 0; i < nb; i++) {
        const uint8_t *b = w + i * 22, *qs = b + 6;
        const uint32_t qh = rd_u32(b + 2);
        int32_t s = 0;
        for (int j = 0; j < 16; j++) {
            const uint32_t xh0 = ((qh >> j) << 4) & 0x10, xh1 = (qh >> (j + 12)) & 0x10;
            s += ((int32_t)((qs[j] & 0xFu) | xh0) - 16) * a[i].qs[j];
            s += ((int32_t)((qs[j] >> 4) | xh1) - 16) * a[i].qs[j + 16];
        }
        if (bs) bs[i] = s;
        sum += f16_at(b) * a[i].d * (float)s;
    }
    return sum;
}
float dot_q5_1_s(const uint8_t *w, const BlockQ8_0 *a, size_t nb, int32_t *bs) {
    float sum = 0.0f;
    for (size_t i = 0; i < nb; i++) {
        const uint8_t *b = w + i * 24, *qs = b + 8;
        const uint32_t qh = rd_u32(b + 4);
        int32_t s = 0;
        for (int j = 0; j < 16; j++) {
            const uint32_t xh0 = ((qh >> j) << 4) & 0x10, xh1 = (qh >> (j + 12)) & 0x10;
            s += (int32_t)((qs[j] & 0xFu) | xh0) * a[i].qs[j];
            s += (int32_t)((qs[j] >> 4) | xh1) * a[i].qs[j + 16];
        }
        if (bs) bs[i] = s;
        sum += f16_at(b) * a[i].d * (float)s + f16_at(b + 2) * a[i].s;
    }
    return sum;
}
float dot_q8_0_s(const uint8_t *w, const BlockQ8_0 *a, size_t nb, int32_t *bs) {
    float sum = 0.0f;
    for (size_t i = 0; i < nb; i++) {
        const uint8_t *b = w + i * 34;
        int32_t s = 0;
        for (size_t j = 0; j < QK; j++) s += (int8_t)b[2 + j] * a[i].qs[j];
        if (bs) bs[i] = s;
        sum += f16_at(b) * a[i].d * (float)s;
    }
    return sum;
}
float dot_q4_k_s(const uint8_t *w, const BlockQ8K *a, size_t nb, int32_t *bs) {
    float sum = 0.0f;
    for (size_t i = 0; i < nb; i++) {
        const uint8_t *b = w + i * 144, *q = b + 16;
        const float d = f16_at(b) * a[i].d, dmin = f16_at(b + 2) * a[i].d;
        uint8_t sc[8], mn[8];
        unpack_k4(b + 4, sc, mn);
        int32_t sumi = 0, summ = 0;
        for (int j = 0; j < 4; j++) {
            int32_t s1 = 0, s2 = 0;
            for (int l = 0; l < 32; l++) {
                s1 += (q[32 * j + l] & 0xF) * a[i].qs[64 * j + l];
                s2 += (q[32 * j + l] >> 4) * a[i].qs[64 * j + 32 + l];
            }
            sumi += s1 * sc[2 * j] + s2 * sc[2 * j + 1];
        }
        for (int j = 0; j < 8; j++) summ += (a[i].bsums[2 * j] + a[i].bsums[2 * j + 1]) * mn[j];
        if (bs) {
            bs[2 * i] = sumi;
            bs[2 * i + 1] = summ;
        }
        sum += d * (float)sumi - dmin * (float)summ;
    }
    return sum;
}
float dot_q5_k_s(const uint8_t *w, const BlockQ8K *a, size_t nb, int32_t *bs) {
    float sum = 0.0f;
    for (size_t i = 0; i < nb; i++) {
        const uint8_t *b = w + i * 176, *qh = b + 16, *ql = b + 48;
        const float d = f16_at(b) * a[i].d, dmin = f16_at(b + 2) * a[i].d;
        uint8_t sc[8], mn[8];
        unpack_k4(b + 4, sc, mn);
        int32_t sumi = 0, summ = 0;
        for (int j = 0; j < 4; j++) {
            const uint8_t u1 = (uint8_t)(1u << (2 * j)), u2 = (uint8_t)(2u << (2 * j));
            int32_t s1 = 0, s2 = 0;
            for (int l = 0; l < 32; l++) {
                const int h1 = (qh[l] & u1) ? 16 : 0, h2 = (qh[l] & u2) ? 16 : 0;
                s1 += ((ql[32 * j + l] & 0xF) + h1) * a[i].qs[64 * j + l];
                s2 += ((ql[32 * j + l] >> 4) + h2) * a[i].qs[64 * j + 32 + l];
            }
            sumi += s1 * sc[2 * j] + s2 * sc[2 * j + 1];
        }
        for (int j = 0; j < 8; j++) summ += (a[i].bsums[2 * j] + a[i].bsums[2 * j + 1]) * mn[j];
        if (bs) {
            bs[2 * i] = sumi;
            bs[2 * i + 1] = summ;
        }
        sum += d * (float)sumi - dmin * (float)summ;
    }
    return sum;
}
float dot_q6_k_s(const uint8_t *w, const BlockQ8K *a, size_t nb, int32_t *bs) {
    float sum = 0.0f;
    for (size_t i = 0; i < nb; i++) {
        const uint8_t *b = w + i * 210;
        const float d = f16_at(b + 208) * a[i].d;
        int32_t sumi = 0;
        for (int n = 0; n < 2; n++) {
            const uint8_t *ql = b + 64 * n, *qh = b + 128 + 32 * n;
            const int8_t *sc = (const int8_t *)(b + 192 + 8 * n);
            const int8_t *aq = a[i].qs + 128 * n;
            int32_t g[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            for (int l = 0; l < 32; l++) {
                const int is = l / 16;
                const int q1 = ((ql[l] & 0xF) | ((qh[l] & 3) << 4)) - 32;
                const int q2 = ((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                const int q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                const int q4 = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                g[is] += q1 * aq[l];
                g[is + 2] += q2 * aq[l + 32];
                g[is + 4] += q3 * aq[l + 64];
                g[is + 6] += q4 * aq[l + 96];
            }
            for (int k = 0; k < 8; k++) sumi += g[k] * sc[k];
        }
        if (bs) bs[i] = sumi;
        sum += d * (float)sumi;
    }
    return sum;
}
// quant/reference.rs:388-401
float dot_k_generic(int t, const uint8_t *w, const BlockQ8K *a, size_t nb) {
    const size_t bb = block_bytes(t);
    float tmp[QK_K];
    float sum = 0.0f;
    for (size_t i = 0; i < nb; i++) {
        dequantize_block(t, w + i * bb, tmp);
        float s = 0.0f;
        for (size_t j = 0; j < QK_K; j++) s += tmp[j] * (float)a[i].qs[j];
        sum += s * a[i].d;
    }
    return sum;
}

// ---- AVX2 dots (kernels/avx2.rs:38-151, 262-337) -----------------------------------
__attribute__((target("avx2,fma,f16c"))) inline __m256 mul_sum_i8(__m256i x, __m256i y) {
    const __m256i ax = _mm256_sign_epi8(x, x);
    const __m256i sy = _mm256_sign_epi8(y, x);
    return _mm256_cvtepi32_ps(_mm256_madd_epi16(_mm256_maddubs_epi16(ax, sy), _mm256_set1_epi16(1)));
}
__attribute__((target("avx2,fma,f16c"))) inline float ld_f16_hw(const uint8_t *p) {
    return _mm_cvtss_f32(_mm_cvtph_ps(_mm_cvtsi32_si128(p[0] | (p[1] << 8))));
}
__attribute__((target("avx2,fma,f16c"))) float dot_q8_0_avx2(const uint8_t *w, const BlockQ8_0 *a, size_t nb) {
    __m256 acc = _mm256_setzero_ps();
    for (size_t i = 0; i < nb; i++) {
        const uint8_t *b = w + i * 34;
        const __m256i x = _mm256_loadu_si256((const __m256i *)(b + 2));
        const __m256i y = _mm256_loadu_si256((const __m256i *)a[i].qs);
        acc = _mm256_fmadd_ps(_mm256_set1_ps(ld_f16_hw(b) * a[i].d), mul_sum_i8(x, y), acc);
    }
    return hsum_f32x8(acc);
}
__attribute__((target("avx2,fma,f16c"))) inline __m256i unpack_q4_0(const uint8_t *qs) {
    const __m128i q = _mm_loadu_si128((const __m128i *)qs);
    const __m256i both = _mm256_set_m128i(_mm_srli_epi16(q, 4), q);
    return _mm256_sub_epi8(_mm256_and_si256(both, _mm256_set1_epi8(0x0F)), _mm256_set1_epi8(8));
}
__attribute__((target("avx2,fma,f16c"))) float dot_q4_0_avx2(const uint8_t *w, const BlockQ8_0 *a, size_t nb) {
    __m256 acc = _mm256_setzero_ps();
    for (size_t i = 0; i < nb; i++) {
        const uint8_t *b = w + i * 18;
        const __m256i x = unpack_q4_0(b + 2);
        const __m256i y = _mm256_loadu_si256((const __m256i *)a[i].qs);
        acc = _mm256_fmadd_ps(_mm256_set1_ps(ld_f16_hw(b) * a[i].d), mul_sum_i8(x, y), acc);
    }
    return hsum_f32x8(acc);
}
__attribute__((target("avx2,fma,f16c"))) float dot_q4_k_avx2(const uint8_t *w, const BlockQ8K *a, size_t nb) {
    const __m256i m4 = _mm256_set1_epi8(0x0F);
    float sum = 0.0f;
    for (size_t i = 0; i < nb; i++) {
        const uint8_t *b = w + i * 144;
        const float d = ld_f16_hw(b) * a[i].d, dmin = ld_f16_hw(b + 2) * a[i].d;
        uint8_t sc[8], mn[8];
        unpack_k4(b + 4, sc, mn);
        int32_t summ = 0;
        for (int j = 0; j < 8; j++) summ += (a[i].bsums[2 * j] + a[i].bsums[2 * j + 1]) * mn[j];
        __m256i acc = _mm256_setzero_si256();
        for (int j = 0; j < 4; j++) {
            const __m256i v = _mm256_loadu_si256((const __m256i *)(b + 16 + 32 * j));
            const __m256i lo = _mm256_and_si256(v, m4), hi = _mm256_and_si256(_mm256_srli_epi16(v, 4), m4);
            const __m256i alo = _mm256_loadu_si256((const __m256i *)(a[i].qs + 64 * j));
            const __m256i ahi = _mm256_loadu_si256((const __m256i *)(a[i].qs + 64 * j + 32));
            const __m256i plo = _mm256_madd_epi16(_mm256_maddubs_epi16(lo, alo), _mm256_set1_epi16(sc[2 * j]));
            const __m256i phi = _mm256_madd_epi16(_mm256_maddubs_epi16(hi, ahi), _mm256_set1_epi16(sc[2 * j + 1]));
            acc = _mm256_add_epi32(acc, _mm256_add_epi32(plo, phi));
        }
        sum += d * (float)hsum_i32x8(acc) - dmin * (float)summ;
    }
    return sum;
}
__attribute__((target("avx2,fma,f16c"))) float dot_q6_k_avx2(const uint8_t *w, const BlockQ8K *a, size_t nb) {
    const __m256i m4 = _mm256_set1_epi8(0x0F), m3 = _mm256_set1_epi8(3);
    float sum = 0.0f;
    for (size_t i = 0; i < nb; i++) {
        const uint8_t *b = w + i * 210;
        const float d = ld_f16_hw(b + 208) * a[i].d;
        const int8_t *scp = (const int8_t *)(b + 192);
        __m256i acc = _mm256_setzero_si256();
        int32_t corr = 0;
        for (int n = 0; n < 2; n++) {
            const uint8_t *ql = b + 64 * n;
            const __m256i qh = _mm256_loadu_si256((const __m256i *)(b + 128 + 32 * n));
            const __m256i ql0 = _mm256_loadu_si256((const __m256i *)ql);
            const __m256i ql1 = _mm256_loadu_si256((const __m256i *)(ql + 32));
            __m256i v[4];
            v[0] = _mm256_or_si256(_mm256_and_si256(ql0, m4), _mm256_slli_epi16(_mm256_and_si256(qh, m3), 4));
            v[1] = _mm256_or_si256(_mm256_and_si256(ql1, m4),
                                   _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(qh, 2), m3), 4));
            v[2] = _mm256_or_si256(_mm256_and_si256(_mm256_srli_epi16(ql0, 4), m4),
                                   _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(qh, 4), m3), 4));
            v[3] = _mm256_or_si256(_mm256_and_si256(_mm256_srli_epi16(ql1, 4), m4),
                                   _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(qh, 6), m3), 4));
            const int8_t *aq = a[i].qs + 128 * n;
            for (int k = 0; k < 4; k++) {
                const int16_t s0 = scp[8 * n + 2 * k], s1 = scp[8 * n + 2 * k + 1];
                const __m256i y = _mm256_loadu_si256((const __m256i *)(aq + 32 * k));
                const __m256i p = _mm256_maddubs_epi16(v[k], y);
                const __m256i scales = _mm256_set_m128i(_mm_set1_epi16(s1), _mm_set1_epi16(s0));
                acc = _mm256_add_epi32(acc, _mm256_madd_epi16(p, scales));
                corr += s0 * a[i].bsums[8 * n + 2 * k] + s1 * a[i].bsums[8 * n + 2 * k + 1];
            }
        }
        sum += d * (float)(hsum_i32x8(acc) - 32 * corr);
    }
    return sum;
}
// 4-token tiles (kernels/avx2.rs:262-337)
__attribute__((target("avx2,fma,f16c"))) void dot4_q8_0_avx2(const uint8_t *w, const BlockQ8_0 *const a[4], size_t nb, float out[4]) {
    __m256 acc[4] = {_mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps()};
    for (size_t i = 0; i < nb; i++) {
        const uint8_t *b = w + i * 34;
        const __m256i x = _mm256_loadu_si256((const __m256i *)(b + 2));
        const __m256i ax = _mm256_sign_epi8(x, x);
        const float d = ld_f16_hw(b);
        for (int t = 0; t < 4; t++) {
            const __m256i y = _mm256_loadu_si256((const __m256i *)a[t][i].qs);
            const __m256i dot = _mm256_maddubs_epi16(ax, _mm256_sign_epi8(y, x));
            const __m256 s = _mm256_cvtepi32_ps(_mm256_madd_epi16(dot, _mm256_set1_epi16(1)));
            acc[t] = _mm256_fmadd_ps(_mm256_set1_ps(d * a[t][i].d), s, acc[t]);
        }
    }
    for (int t = 0; t < 4; t++) out[t] = hsum_f32x8(acc[t]);
}
__attribute__((target("avx2,fma,f16c"))) void dot4_q4_0_avx2(const uint8_t *w, const BlockQ8_0 *const a[4], size_t nb, float out[4]) {
    __m256 acc[4] = {_mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps()};
    for (size_t i = 0; i < nb; i++) {
        const uint8_t *b = w + i * 18;
        const __m256i x = unpack_q4_0(b + 2);
        const __m256i ax = _mm256_sign_epi8(x, x);
        const float d = ld_f16_hw(b);
        for (int t = 0; t < 4; t++) {
            const __m256i y = _mm256_loadu_si256((const __m256i *)a[t][i].qs);
            const __m256i dot = _mm256_maddubs_epi16(ax, _mm256_sign_epi8(y, x));
            const __m256 s = _mm256_cvtepi32_ps(_mm256_madd_epi16(dot, _mm256_set1_epi16(1)));
            acc[t] = _mm256_fmadd_ps(_mm256_set1_ps(d * a[t][i].d), s, acc[t]);
        }
    }
    for (int t = 0; t < 4; t++) out[t] = hsum_f32x8(acc[t]);
}
__attribute__((target("avx2,fma,f16c"))) void dot4_q4_k_avx2(const uint8_t *w, const BlockQ8K *const a[4], size_t nb, float out[4]) {
    const __m256i m4 = _mm256_set1_epi8(0x0F);
    for (int t = 0; t < 4; t++) out[t] = 0.0f;
    for (size_t i = 0; i < nb; i++) {
        const uint8_t *b = w + i * 144;
        const float d = ld_f16_hw(b), dmin = ld_f16_hw(b + 2);
        uint8_t sc[8], mn[8];
        unpack_k4(b + 4, sc, mn);
        __m256i acc[4] = {_mm256_setzero_si256(), _mm256_setzero_si256(), _mm256_setzero_si256(), _mm256_setzero_si256()};
        for (int j = 0; j < 4; j++) {
            const __m256i v = _mm256_loadu_si256((const __m256i *)(b + 16 + 32 * j));
            const __m256i lo = _mm256_and_si256(v, m4), hi = _mm256_and_si256(_mm256_srli_epi16(v, 4), m4);
            const __m256i slo = _mm256_set1_epi16(sc[2 * j]), shi = _mm256_set1_epi16(sc[2 * j + 1]);
            for (int t = 0; t < 4; t++) {
                const int8_t *aq = a[t][i].qs + 64 * j;
                const __m256i plo = _mm256_madd_epi16(_mm256_maddubs_epi16(lo, _mm256_loadu_si256((const __m256i *)aq)), slo);
                const __m256i phi = _mm256_madd_epi16(_mm256_maddubs_epi16(hi, _mm256_loadu_si256((const __m256i *)(aq + 32))), shi);
                acc[t] = _mm256_add_epi32(acc[t], _mm256_add_epi32(plo, phi));
            }
        }
        for (int t = 0; t < 4; t++) {
            int32_t summ = 0;
            for (int j = 0; j < 8; j++) summ += (a[t][i].bsums[2 * j] + a[t][i].bsums[2 * j + 1]) * mn[j];
            out[t] += d * a[t][i].d * (float)hsum_i32x8(acc[t]) - dmin * a[t][i].d * (float)summ;
        }
    }
}

// ---- float kernels (kernels/mod.rs:357-417, avx2.rs:186-256) ------------------------
__attribute__((target("avx2,fma,f16c"))) float dot_f32_avx2(const float *a, const float *b, size_t n) {
    __m256 acc0 = _mm256_setzero_ps(), acc1 = _mm256_setzero_ps();
    size_t i = 0;
    for (; i + 16 <= n; i += 16) {
        acc0 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(b + i), acc0);
        acc1 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i + 8), _mm256_loadu_ps(b + i + 8), acc1);
    }
    float s = hsum_f32x8(_mm256_add_ps(acc0, acc1));
    for (; i < n; i++) s += a[i] * b[i];
    return s;
}
float dot_f32_scalar(const float *a, const float *b, size_t n) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    const size_t chunks = n / 8;
    for (size_t i = 0; i < chunks; i++)
        for (int k = 0; k < 8; k++) acc[k] += a[i * 8 + k] * b[i * 8 + k];
    float s = 0.0f;
    for (int k = 0; k < 8; k++) s += acc[k];
    for (size_t i = chunks * 8; i < n; i++) s += a[i] * b[i];
    return s;
}
float dot_f32(const float *a, const float *b, size_t n, int path) {
    return simd(path) ? dot_f32_avx2(a, b, n) : dot_f32_scalar(a, b, n);
}
__attribute__((target("avx2,fma,f16c"))) float dot_f16_f32_avx2(const uint16_t *a, const float *b, size_t n) {
    __m256 acc0 = _mm256_setzero_ps(), acc1 = _mm256_setzero_ps();
    size_t i = 0;
    for (; i + 16 <= n; i += 16) {
        const __m256 h0 = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i *)(a + i)));
        const __m256 h1 = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i *)(a + i + 8)));
        acc0 = _mm256_fmadd_ps(h0, _mm256_loadu_ps(b + i), acc0);
        acc1 = _mm256_fmadd_ps(h1, _mm256_loadu_ps(b + i + 8), acc1);
    }
    float s = hsum_f32x8(_mm256_add_ps(acc0, acc1));
    for (; i < n; i++) s += f16_to_f32(a[i]) * b[i];
    return s;
}
float dot_f16_f32(const uint16_t *a, const float *b, size_t n, int path) {
    if (simd(path)) return dot_f16_f32_avx2(a, b, n);
    float s = 0.0f;
    for (size_t i = 0; i < n; i++) s += f16_to_f32(a[i]) * b[i];
    return s;
}
__attribute__((target("avx2,fma,f16c"))) void axpy_f16_avx2(float *y, float alpha, const uint16_t *x, size_t n) {
    const __m256 va = _mm256_set1_ps(alpha);
    size_t i = 0;
    for (; i + 8 <= n; i += 8) {
        const __m256 h = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i *)(x + i)));
        _mm256_storeu_ps(y + i, _mm256_fmadd_ps(h, va, _mm256_loadu_ps(y + i)));
    }
    for (; i < n; i++) y[i] += alpha * f16_to_f32(x[i]);
}
void axpy_f16(float *y, float alpha, const uint16_t *x, size_t n, int path) {
    if (simd(path)) return axpy_f16_avx2(y, alpha, x, n);
    for (size_t i = 0; i < n; i++) y[i] += alpha * f16_to_f32(x[i]);
}
__attribute__((target("avx2,fma,f16c"))) void f32_to_f16_avx2(const float *src, uint16_t *dst, size_t n) {
    size_t i = 0;
    for (; i + 8 <= n; i += 8) {
        const __m128i h = _mm256_cvtps_ph(_mm256_loadu_ps(src + i), _MM_FROUND_TO_NEAREST_INT);
        _mm_storeu_si128((__m128i *)(dst + i), h);
    }
    for (; i < n; i++) dst[i] = f32_to_f16(src[i]);
}

// ---- vec_dot dispatch (kernels/mod.rs:134-232, x86 tiers) ---------------------------
float vec_dot(int t, const uint8_t *w, const void *act, size_t n, int path) {
    const bool v = simd(path);
    switch (t) {
        case T_F32: return dot_f32((const float *)w, (const float *)act, n, path);
        case T_F16: return dot_f16_f32((const uint16_t *)w, (const float *)act, n, path);
        case T_BF16: {
            const uint16_t *h = (const uint16_t *)w;
            const float *x = (const float *)act;
            float s = 0.0f;
            for (size_t i = 0; i < n; i++) s += bf16_to_f32(h[i]) * x[i];
            return s;
        }
        case T_Q8_0: return v ? dot_q8_0_avx2(w, (const BlockQ8_0 *)act, n / QK) : dot_q8_0_s(w, (const BlockQ8_0 *)act, n / QK, nullptr);
        case T_Q4_0: return v ? dot_q4_0_avx2(w, (const BlockQ8_0 *)act, n / QK) : dot_q4_0_s(w, (const BlockQ8_0 *)act, n / QK, nullptr);
        case T_Q4_1: return dot_q4_1_s(w, (const BlockQ8_0 *)act, n / QK, nullptr);
        case T_Q5_0: return dot_q5_0_s(w, (const BlockQ8_0 *)act, n / QK, nullptr);
        case T_Q5_1: return dot_q5_1_s(w, (const BlockQ8_0 *)act, n / QK, nullptr);
        case T_Q4_K: return v ? dot_q4_k_avx2(w, (const BlockQ8K *)act, n / QK_K) : dot_q4_k_s(w, (const BlockQ8K *)act, n / QK_K, nullptr);
        case T_Q5_K: return dot_q5_k_s(w, (const BlockQ8K *)act, n / QK_K, nullptr);
        case T_Q6_K: return v ? dot_q6_k_avx2(w, (const BlockQ8K *)act, n / QK_K) : dot_q6_k_s(w, (const BlockQ8K *)act, n / QK_K, nullptr);
        case T_Q2_K: case T_Q3_K: return dot_k_generic(t, w, (const BlockQ8K *)act, n / QK_K);
        default: return 0.0f;
    }
}
bool has_x4(int t, int path) { return simd(path) && (t == T_Q8_0 || t == T_Q4_0 || t == T_Q4_K); }

// ---- fork/join pool (threadpool.rs:97-160: caller is worker 0, dynamic chunks) --------
class Pool {
  public:
    explicit Pool(int n) : n_(n < 1 ? 1 : n) {
        for (int i = 1; i < n_; i++) workers_.emplace_back([this, i] { loop(i); });
    }
    ~Pool() {
        {
            std::lock_guard<std::mutex> g(m_);
            stop_ = true;
            gen_.fetch_add(1);
        }
        cv_.notify_all();
        for (auto &t : workers_) t.join();
    }
    int size() const { return n_; }
    void for_each(size_t n, size_t grain, const std::function<void(size_t)> &f) {
        if (n == 0) return;
        if (n_ == 1 || n <= grain) {
            for (size_t i = 0; i < n; i++) f(i);
            return;
        }
        job_ = &f;
        n_items_ = n;
        grain_ = grain;
        next_.store(0);
        pending_.store(n_ - 1);
        {
            std::lock_guard<std::mutex> g(m_);
            gen_.fetch_add(1);
        }
        cv_.notify_all();
        work();
        while (pending_.load(std::memory_order_acquire) != 0) std::this_thread::yield();
        job_ = nullptr;
    }

  private:
    void work() {
        for (;;) {
            const size_t s = next_.fetch_add(grain_);
            if (s >= n_items_) break;
            const size_t e = std::min(n_items_, s + grain_);
            for (size_t i = s; i < e; i++) (*job_)(i);
        }
    }
    void loop(int) {
        uint64_t seen = 0;
        for (;;) {
            uint64_t g = gen_.load(std::memory_order_acquire);
            int spins = 0;
            while (g == seen && spins < 20000) {
                std::this_thread::yield();
                g = gen_.load(std::memory_order_acquire);
                spins++;
            }
            if (g == seen) {
                std::unique_lock<std::mutex> lk(m_);
                cv_.wait(lk, [&] { return gen_.load() != seen; });
                g = gen_.load();
            }
            seen = g;
            if (stop_) return;
            work();
            pending_.fetch_sub(1, std::memory_order_acq_rel);
        }
    }
    int n_;
    std::vector<std::thread> workers_;
    std::mutex m_;
    std::condition_variable cv_;
    std::atomic<uint64_t> gen_{0};
    std::atomic<size_t> next_{0};
    std::atomic<int> pending_{0};
    const std::function<void(size_t)> *job_ = nullptr;
    size_t n_items_ = 0, grain_ = 1;
    bool stop_ = false;
};

Pool &pool_for(int n_threads) {
    static std::mutex m;
    static std::vector<std::unique_ptr<Pool>> pools;
    std::lock_guard<std::mutex> g(m);
    for (auto &p : pools)
        if (p->size() == n_threads) return *p;
    pools.emplace_back(new Pool(n_threads));
    return *pools.back();
}

// ---- turbo4 (turbo.rs) --------------------------------------------------------------
constexpr uint64_t KV_SEED = 0x75426F5175616E74ull;
constexpr int8_t KV_LEVELS_I8[16] = {-126, -95, -74, -58, -43, -30, -18, -6, 6, 18, 30, 43, 58, 74, 95, 126};
constexpr float KV_I8_SCALE = 46.0f;
const float LM2[2] = {0.4528f, 1.5104f};
const float LM4[8] = {0.1284f, 0.3881f, 0.6568f, 0.9424f, 1.2562f, 1.6180f, 2.0690f, 2.7326f};

size_t turbo_block(size_t d) {  // turbo.rs:51-58
    size_t b = 1;
    while (d % (b * 2) == 0 && b < 256) b *= 2;
    return b;
}
void fwht(float *x, size_t n) {  // turbo.rs:60-76
    for (size_t h = 1; h < n; h *= 2)
        for (size_t i = 0; i < n; i += 2 * h)
            for (size_t j = i; j < i + h; j++) {
                const float a = x[j], b = x[j + h];
                x[j] = a + b;
                x[j + h] = a - b;
            }
    const float s = 1.0f / std::sqrt((float)n);
    for (size_t i = 0; i < n; i++) x[i] *= s;
}
float turbo_sign(uint64_t seed, size_t i) {  // turbo.rs:78-89 (splitmix64 finaliser)
    uint64_t z = seed + (uint64_t)i * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return ((z ^ (z >> 31)) & 1) == 0 ? 1.0f : -1.0f;
}
void rotate(uint64_t seed, float *x, size_t d, bool inverse) {  // turbo.rs:108-117
    const size_t b = turbo_block(d);
    if (!inverse)
        for (size_t i = 0; i < d; i++) x[i] *= turbo_sign(seed, i);
    for (size_t o = 0; o < d; o += b) fwht(x + o, b);
    if (inverse)
        for (size_t i = 0; i < d; i++) x[i] *= turbo_sign(seed, i);
}
void kv_levels(float c[16]) {  // turbo.rs:129-131
    for (int i = 0; i < 16; i++) c[i] = (float)KV_LEVELS_I8[i] / KV_I8_SCALE;
}
uint8_t nearest(const float *c, int n, float v) {  // turbo.rs:40-49
    uint8_t i = 0;
    for (int k = 0; k + 1 < n; k++) i += (uint8_t)(v > 0.5f * (c[k] + c[k + 1]));
    return i;
}
size_t row_bytes_4(size_t d) { return 2 * (d / turbo_block(d)) + d / 2; }  // turbo.rs:136-138

void quantize_rotated_4(const float *y, size_t d, uint8_t *out) {  // turbo.rs:141-164
    const size_t b = turbo_block(d), nb = d / b;
    float c[16];
    kv_levels(c);
    uint8_t *scales = out, *codes = out + 2 * nb;
    std::memset(codes, 0, d / 2);
    for (size_t bi = 0; bi < nb; bi++) {
        const float *yb = y + bi * b;
        float ss = 0.0f;
        for (size_t j = 0; j < b; j++) ss += yb[j] * yb[j];
        const float rms = std::sqrt(ss / (float)b);
        const float inv = rms > 0.0f ? 1.0f / rms : 0.0f;
        float num = 0.0f, den = 0.0f;
        for (size_t j = 0; j < b; j++) {
            const uint8_t q = nearest(c, 16, yb[j] * inv);
            const size_t g = bi * b + j;
            codes[(g / 32) * 16 + g % 16] |= (uint8_t)(q << (((g % 32) / 16) * 4));
            num += yb[j] * c[q];
            den += c[q] * c[q];
        }
        const float s = den > 0.0f ? num / den : 0.0f;
        put_f16(scales + 2 * bi, s);
    }
}

float dot_chunks_scalar(const BlockQ8_0 *q, const uint8_t *codes, size_t nchunks) {  // turbo.rs:209-220
    float s = 0.0f;
    for (size_t c = 0; c < nchunks; c++) {
        const uint8_t *cb = codes + 16 * c;
        int32_t acc = 0;
        for (int i = 0; i < 16; i++) {
            acc += KV_LEVELS_I8[cb[i] & 15] * q[c].qs[i];
            acc += KV_LEVELS_I8[cb[i] >> 4] * q[c].qs[i + 16];
        }
        s += q[c].d * (float)acc;
    }
    return s;
}
__attribute__((target("avx2,fma,f16c"))) inline __m256i turbo_decode(const uint8_t *p, __m256i tbl) {
    const __m128i q = _mm_loadu_si128((const __m128i *)p);
    const __m256i both = _mm256_set_m128i(_mm_srli_epi16(q, 4), q);
    return _mm256_shuffle_epi8(tbl, _mm256_and_si256(both, _mm256_set1_epi8(0x0F)));
}
__attribute__((target("avx2,fma,f16c"))) inline __m256i turbo_table() {
    const __m128i t = _mm_loadu_si128((const __m128i *)KV_LEVELS_I8);
    return _mm256_set_m128i(t, t);
}
__attribute__((target("avx2,fma,f16c"))) float dot_chunks_avx2(const BlockQ8_0 *q, const uint8_t *codes, size_t nchunks) {  // turbo.rs:279-294
    const __m256i tbl = turbo_table();
    __m256 acc = _mm256_setzero_ps();
    for (size_t i = 0; i < nchunks; i++) {
        const __m256i x = turbo_decode(codes + 16 * i, tbl);
        const __m256i y = _mm256_loadu_si256((const __m256i *)q[i].qs);
        const __m256i ax = _mm256_sign_epi8(x, x), sy = _mm256_sign_epi8(y, x);
        const __m256i p = _mm256_madd_epi16(_mm256_maddubs_epi16(ax, sy), _mm256_set1_epi16(1));
        acc = _mm256_fmadd_ps(_mm256_set1_ps(q[i].d), _mm256_cvtepi32_ps(p), acc);
    }
    __m128 h = _mm_add_ps(_mm256_castps256_ps128(acc), _mm256_extractf128_ps(acc, 1));
    h = _mm_add_ps(h, _mm_movehl_ps(h, h));
    return _mm_cvtss_f32(_mm_add_ss(h, _mm_shuffle_ps(h, h, 1)));
}
float dot_rotated_4(const BlockQ8_0 *q, const uint8_t *row, size_t d, int path) {  // turbo.rs:180-193
    const size_t b = turbo_block(d), nb = d / b, cpb = b / 32;
    const uint8_t *codes = row + 2 * nb;
    float total = 0.0f;
    for (size_t bi = 0; bi < nb; bi++) {
        const float dc = simd(path) ? dot_chunks_avx2(q + bi * cpb, codes + bi * cpb * 16, cpb)
                                    : dot_chunks_scalar(q + bi * cpb, codes + bi * cpb * 16, cpb);
        total += f16_at(row + 2 * bi) * dc;
    }
    return total * (1.0f / KV_I8_SCALE);
}
__attribute__((target("avx2,fma,f16c"))) void axpy_chunks_avx2(float *y, float a, const uint8_t *codes, size_t n) {  // turbo.rs:297-311
    const __m256i tbl = turbo_table();
    const __m256 va = _mm256_set1_ps(a);
    for (size_t c = 0; c < n / 32; c++) {
        const __m256i x = turbo_decode(codes + c * 16, tbl);
        const __m128i lo = _mm256_castsi256_si128(x), hi = _mm256_extracti128_si256(x, 1);
        const __m128i parts[4] = {lo, _mm_srli_si128(lo, 8), hi, _mm_srli_si128(hi, 8)};
        for (int k = 0; k < 4; k++) {
            const __m256 v = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(parts[k]));
            float *yp = y + c * 32 + k * 8;
            _mm256_storeu_ps(yp, _mm256_fmadd_ps(va, v, _mm256_loadu_ps(yp)));
        }
    }
}
void axpy_rotated_4(float *y, float a, const uint8_t *row, size_t d, int path) {  // turbo.rs:224-250
    const size_t b = turbo_block(d), nb = d / b;
    const uint8_t *codes = row + 2 * nb;
    for (size_t bi = 0; bi < nb; bi++) {
        const float s = a * f16_at(row + 2 * bi) * (1.0f / KV_I8_SCALE);
        float *yb = y + bi * b;
        const uint8_t *cb = codes + bi * b / 2;
        if (simd(path)) {
            axpy_chunks_avx2(yb, s, cb, b);
            continue;
        }
        for (size_t c = 0; c < b / 32; c++)
            for (int i = 0; i < 16; i++) {
                yb[32 * c + i] += s * (float)KV_LEVELS_I8[cb[16 * c + i] & 15];
                yb[32 * c + i + 16] += s * (float)KV_LEVELS_I8[cb[16 * c + i] >> 4];
            }
    }
}

// model/cpu.rs:636-658
void store_q8_0(const float *x, size_t hd, uint8_t *dst) {
    for (size_t b = 0; b < hd / QK; b++) {
        const float *xb = x + b * QK;
        uint8_t *ob = dst + b * 34;
        float amax = 0.0f;
        for (size_t j = 0; j < QK; j++) amax = std::fmax(amax, std::fabs(xb[j]));
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        put_f16(ob, d);
        for (size_t j = 0; j < QK; j++) ob[2 + j] = (uint8_t)(int8_t)clampi(sat_i32(rust_round(xb[j] * id)), -127, 127);
    }
}
void axpy_q8_0(float *y, float a, const uint8_t *row, size_t hd) {
    for (size_t b = 0; b < hd / QK; b++) {
        const uint8_t *rb = row + b * 34;
        const float s = a * f16_at(rb);
        for (size_t j = 0; j < QK; j++) y[b * QK + j] += s * (float)(int8_t)rb[2 + j];
    }
}

void quantize_acts_q8_0(const float *x, size_t n, BlockQ8_0 *out, int path) {
    if (simd(path))
        quantize_q8_0_avx2(x, n / QK, out);
    else
        quantize_q8_0_scalar(x, n / QK, out);
}

// ---- own weight quantizers for the block types the reference cannot produce ----------
// Valid blocks only; not tuned. Layouts follow quant/reference.rs dequantize_block.
void q_k4_pack(const uint8_t sc[8], const uint8_t mn[8], uint8_t *q) {  // inverse of scale_min_k4
    std::memset(q, 0, 12);
    for (int j = 0; j < 8; j++) {
        if (j < 4) {
            q[j] |= sc[j] & 63;
            q[j + 4] |= mn[j] & 63;
        } else {
            q[j + 4] |= (uint8_t)((sc[j] & 0xF) | ((mn[j] & 0xF) << 4));
            q[j - 4] |= (uint8_t)((sc[j] >> 4) << 6);
            q[j] |= (uint8_t)((mn[j] >> 4) << 6);
        }
    }
}
void quantize_block_own(int t, const float *x, uint8_t *o) {
    switch (t) {
        case T_Q4_1: case T_Q5_1: {
            const int nq = t == T_Q4_1 ? 15 : 31;
            float mn = x[0], mx = x[0];
            for (int j = 1; j < 32; j++) mn = std::fmin(mn, x[j]), mx = std::fmax(mx, x[j]);
            const float d = (mx - mn) / (float)nq, id = d != 0.0f ? 1.0f / d : 0.0f;
            put_f16(o, d);
            put_f16(o + 2, mn);
            uint8_t q[32];
            for (int j = 0; j < 32; j++) q[j] = (uint8_t)clampi((int)((x[j] - mn) * id + 0.5f), 0, nq);
            if (t == T_Q4_1) {
                for (int j = 0; j < 16; j++) o[4 + j] = (uint8_t)(q[j] | (q[j + 16] << 4));
            } else {
                uint32_t qh = 0;
                for (int j = 0; j < 16; j++) {
                    o[8 + j] = (uint8_t)((q[j] & 0xF) | ((q[j + 16] & 0xF) << 4));
                    qh |= (uint32_t)((q[j] >> 4) & 1) << j;
                    qh |= (uint32_t)((q[j + 16] >> 4) & 1) << (j + 16);
                }
                std::memcpy(o + 4, &qh, 4);
            }
            break;
        }
        case T_Q5_0: {
            float mx = 0.0f;
            for (int j = 0; j < 32; j++)
                if (std::fabs(x[j]) > std::fabs(mx)) mx = x[j];
            const float d = mx / -16.0f, id = d != 0.0f ? 1.0f / d : 0.0f;
            put_f16(o, d);
            uint32_t qh = 0;
            for (int j = 0; j < 16; j++) {
                const uint8_t q0 = (uint8_t)clampi(sat_i32(x[j] * id + 16.5f), 0, 31);
                const uint8_t q1 = (uint8_t)clampi(sat_i32(x[j + 16] * id + 16.5f), 0, 31);
                o[6 + j] = (uint8_t)((q0 & 0xF) | ((q1 & 0xF) << 4));
                qh |= (uint32_t)(q0 >> 4) << j;
                qh |= (uint32_t)(q1 >> 4) << (j + 16);
            }
            std::memcpy(o + 2, &qh, 4);
            break;
        }
        case T_Q4_K: case T_Q5_K: {
            const int nq = t == T_Q4_K ? 15 : 31;
            float scale[8], mins[8];
            for (int j = 0; j < 8; j++) {
                float mn = x[32 * j], mx = x[32 * j];
                for (int l = 1; l < 32; l++) mn = std::fmin(mn, x[32 * j + l]), mx = std::fmax(mx, x[32 * j + l]);
                if (mn > 0.0f) mn = 0.0f;
                scale[j] = (mx - mn) / (float)nq;
                mins[j] = -mn;
            }
            float ms = 0.0f, mm = 0.0f;
            for (int j = 0; j < 8; j++) ms = std::fmax(ms, scale[j]), mm = std::fmax(mm, mins[j]);
            const float d = ms / 63.0f, dmin = mm / 63.0f;
            put_f16(o, d);
            put_f16(o + 2, dmin);
            const float dh = f16_to_f32(f32_to_f16(d)), dmh = f16_to_f32(f32_to_f16(dmin));
            uint8_t sc[8], mq[8];
            for (int j = 0; j < 8; j++) {
                sc[j] = (uint8_t)clampi(dh > 0.0f ? (int)std::lround(scale[j] / dh) : 0, 0, 63);
                mq[j] = (uint8_t)clampi(dmh > 0.0f ? (int)std::lround(mins[j] / dmh) : 0, 0, 63);
            }
            q_k4_pack(sc, mq, o + 4);
            uint8_t q[256];
            for (int j = 0; j < 8; j++) {
                const float dd = dh * sc[j], m = dmh * mq[j];
                for (int l = 0; l < 32; l++)
                    q[32 * j + l] = (uint8_t)clampi(dd > 0.0f ? (int)std::lround((x[32 * j + l] + m) / dd) : 0, 0, nq);
            }
            if (t == T_Q4_K) {
                for (int j = 0; j < 4; j++)
                    for (int l = 0; l < 32; l++) o[16 + 32 * j + l] = (uint8_t)(q[64 * j + l] | (q[64 * j + 32 + l] << 4));
            } else {
                uint8_t *qh = o + 16, *ql = o + 48;
                std::memset(qh, 0, 32);
                for (int j = 0; j < 4; j++)
                    for (int l = 0; l < 32; l++) {
                        const uint8_t a = q[64 * j + l], b = q[64 * j + 32 + l];
                        ql[32 * j + l] = (uint8_t)((a & 0xF) | ((b & 0xF) << 4));
                        qh[l] |= (uint8_t)(((a >> 4) & 1) << (2 * j));
                        qh[l] |= (uint8_t)(((b >> 4) & 1) << (2 * j + 1));
                    }
            }
            break;
        }
        case T_Q6_K: {
            float sc_f[16];
            float amax_all = 0.0f;
            for (int g = 0; g < 16; g++) {
                float m = 0.0f;
                for (int l = 0; l < 16; l++) m = std::fmax(m, std::fabs(x[16 * g + l]));
                sc_f[g] = m / 31.0f;
                amax_all = std::fmax(amax_all, sc_f[g]);
            }
            const float d = amax_all / 127.0f;
            put_f16(o + 208, d);
            const float dh = f16_to_f32(f32_to_f16(d));
            int8_t sc[16];
            for (int g = 0; g < 16; g++) sc[g] = (int8_t)clampi(dh > 0.0f ? (int)std::lround(sc_f[g] / dh) : 0, -128, 127);
            std::memcpy(o + 192, sc, 16);
            uint8_t q[256];
            for (int g = 0; g < 16; g++) {
                const float dd = dh * sc[g];
                for (int l = 0; l < 16; l++)
                    q[16 * g + l] = (uint8_t)clampi((dd != 0.0f ? (int)std::lround(x[16 * g + l] / dd) : 0) + 32, 0, 63);
            }
            uint8_t *ql = o, *qh = o + 128;
            for (int n = 0; n < 2; n++)
                for (int l = 0; l < 32; l++) {
                    const uint8_t q1 = q[128 * n + l], q2 = q[128 * n + l + 32], q3 = q[128 * n + l + 64], q4 = q[128 * n + l + 96];
                    ql[64 * n + l] = (uint8_t)((q1 & 0xF) | ((q3 & 0xF) << 4));
                    ql[64 * n + l + 32] = (uint8_t)((q2 & 0xF) | ((q4 & 0xF) << 4));
                    qh[32 * n + l] = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
                }
            break;
        }
        default: break;
    }
}

}  // namespace

// ======================================================================================
extern "C" {

int orc_have_avx2(void) { return have_avx2() ? 1 : 0; }
size_t orc_block_size(int t) { return block_size(t); }
size_t orc_block_bytes(int t) { return block_bytes(t); }
size_t orc_row_bytes(int t, size_t n) { return block_size(t) ? n / block_size(t) * block_bytes(t) : 0; }
size_t orc_sizeof_block_q8_0(void) { return sizeof(BlockQ8_0); }
size_t orc_sizeof_block_q8_k(void) { return sizeof(BlockQ8K); }

uint16_t orc_f32_to_f16(float x) { return f32_to_f16(x); }
float orc_f16_to_f32(uint16_t h) { return f16_to_f32(h); }
void orc_f32_to_f16_n(const float *src, uint16_t *dst, size_t n, int path) {
    if (simd(path)) return f32_to_f16_avx2(src, dst, n);
    for (size_t i = 0; i < n; i++) dst[i] = f32_to_f16(src[i]);
}

// testing.rs:10-30
uint64_t orc_rng_new(uint64_t seed) { return (seed * 0x9E3779B97F4A7C15ull) | 1ull; }
uint64_t orc_rng_next(uint64_t *s) {
    *s ^= *s << 13;
    *s ^= *s >> 7;
    *s ^= *s << 17;
    return *s;
}
static float rng_f32(uint64_t *s) { return (float)(orc_rng_next(s) >> 40) / (float)(1ull << 24); }
static float rng_sym(uint64_t *s) { return rng_f32(s) * 2.0f - 1.0f; }
void orc_rng_vec(uint64_t *s, float *out, size_t n, float scale) {
    for (size_t i = 0; i < n; i++) out[i] = rng_sym(s) * scale;
}
// testing.rs:33-91
int orc_random_weight(uint64_t *s, int t, size_t rows, size_t cols, float gain, uint8_t *out) {
    const size_t n = rows * cols;
    if (t == T_F32 || t == T_F16 || t == T_BF16) {
        for (size_t i = 0; i < n; i++) {
            const float v = rng_sym(s) * (0.1f * gain);
            if (t == T_F32) {
                std::memcpy(out + 4 * i, &v, 4);
            } else if (t == T_F16) {
                const uint16_t h = f32_to_f16(v);
                std::memcpy(out + 2 * i, &h, 2);
            } else {  // half::bf16::from_f32: round to nearest even on the top 16 bits
                uint32_t x;
                std::memcpy(&x, &v, 4);
                uint16_t h;
                if ((x & 0x7fffffffu) > 0x7f800000u)
                    h = (uint16_t)((x >> 16) | 0x40);
                else
                    h = (uint16_t)((x + 0x7fffu + ((x >> 16) & 1u)) >> 16);
                std::memcpy(out + 2 * i, &h, 2);
            }
        }
        return 0;
    }
    const size_t bs = block_size(t), bb = block_bytes(t);
    if (!bs) return -1;
    const size_t nblocks = n / bs, total = nblocks * bb;
    for (size_t o = 0; o < total; o += 8) {
        const uint64_t r = orc_rng_next(s);
        std::memcpy(out + o, &r, std::min<size_t>(8, total - o));
    }
    float scale;
    switch (t) {
        case T_Q4_0: case T_Q4_1: scale = 0.01f; break;
        case T_Q5_0: case T_Q5_1: scale = 0.005f; break;
        case T_Q8_0: scale = 0.001f; break;
        case T_Q2_K: scale = 0.004f; break;
        case T_Q3_K: scale = 0.003f; break;
        case T_Q4_K: scale = 0.001f; break;
        case T_Q5_K: scale = 0.0007f; break;
        case T_Q6_K: scale = 0.0001f; break;
        default: scale = 0.01f;
    }
    scale *= gain;
    size_t offs[2];
    size_t n_offs;
    switch (t) {
        case T_Q4_0: case T_Q5_0: case T_Q8_0: offs[0] = 0; n_offs = 1; break;
        case T_Q4_1: case T_Q5_1: case T_Q4_K: case T_Q5_K: offs[0] = 0; offs[1] = 2; n_offs = 2; break;
        case T_Q2_K: offs[0] = 80; offs[1] = 82; n_offs = 2; break;
        case T_Q3_K: offs[0] = 108; n_offs = 1; break;
        case T_Q6_K: offs[0] = 208; n_offs = 1; break;
        default: n_offs = 0;
    }
    const bool neg_ok = t == T_Q4_0 || t == T_Q5_0 || t == T_Q8_0 || t == T_Q3_K || t == T_Q6_K;
    for (size_t b = 0; b < nblocks; b++)
        for (size_t i = 0; i < n_offs; i++) {
            float v = (rng_f32(s) * 0.5f + 0.5f) * scale;
            if (i == 0 && neg_ok && rng_f32(s) < 0.3f) v = -v;
            if (i == 1 && (t == T_Q4_1 || t == T_Q5_1)) v = -v * 8.0f;
            put_f16(out + b * bb + offs[i], v);
        }
    return 0;
}

void orc_quantize_row_q8_0(const float *x, size_t n, void *blocks, int path) {
    quantize_acts_q8_0(x, n, (BlockQ8_0 *)blocks, path);
}
void orc_quantize_row_q8_k(const float *x, size_t n, void *blocks) { quantize_q8_k(x, n / QK_K, (BlockQ8K *)blocks); }

size_t orc_quantize_weight(int t, const float *x, size_t n, uint8_t *out) {
    switch (t) {
        case T_F32: std::memcpy(out, x, 4 * n); return 4 * n;
        case T_F16:
            for (size_t i = 0; i < n; i++) put_f16(out + 2 * i, x[i]);
            return 2 * n;
        case T_Q8_0:  // quant/mod.rs:265-277
            for (size_t b = 0; b < n / QK; b++) {
                const float *xb = x + b * QK;
                float amax = 0.0f;
                for (size_t j = 0; j < QK; j++) amax = std::fmax(amax, std::fabs(xb[j]));
                const float d = amax / 127.0f, id = d != 0.0f ? 1.0f / d : 0.0f;
                put_f16(out + 34 * b, d);
                for (size_t j = 0; j < QK; j++)
                    out[34 * b + 2 + j] = (uint8_t)(int8_t)clampi(sat_i32(rust_round(xb[j] * id)), -127, 127);
            }
            return n / QK * 34;
        case T_Q4_0:  // quant/mod.rs:279-298
            for (size_t b = 0; b < n / QK; b++) {
                const float *xb = x + b * QK;
                float mx = 0.0f;
                for (size_t j = 0; j < QK; j++)
                    if (std::fabs(xb[j]) > std::fabs(mx)) mx = xb[j];
                const float d = mx / -8.0f, id = d != 0.0f ? 1.0f / d : 0.0f;
                put_f16(out + 18 * b, d);
                for (size_t j = 0; j < QK / 2; j++) {
                    const uint8_t q0 = (uint8_t)clampi(sat_i32(xb[j] * id + 8.5f), 0, 15);
                    const uint8_t q1 = (uint8_t)clampi(sat_i32(xb[j + 16] * id + 8.5f), 0, 15);
                    out[18 * b + 2 + j] = (uint8_t)(q0 | (q1 << 4));
                }
            }
            return n / QK * 18;
        case T_Q4_1: case T_Q5_0: case T_Q5_1: case T_Q4_K: case T_Q5_K: case T_Q6_K: {
            const size_t bs = block_size(t), bb = block_bytes(t);
            for (size_t b = 0; b < n / bs; b++) quantize_block_own(t, x + b * bs, out + b * bb);
            return n / bs * bb;
        }
        default: return 0;
    }
}

int orc_dequantize_row(int t, const uint8_t *src, float *dst, size_t n) {
    if (t == T_F32) {
        std::memcpy(dst, src, 4 * n);
        return 0;
    }
    if (t == T_F16 || t == T_BF16) {
        for (size_t i = 0; i < n; i++) {
            const uint16_t h = (uint16_t)(src[2 * i] | (src[2 * i + 1] << 8));
            dst[i] = t == T_F16 ? f16_to_f32(h) : bf16_to_f32(h);
        }
        return 0;
    }
    const size_t bs = block_size(t), bb = block_bytes(t);
    if (!bs) return -1;
    for (size_t b = 0; b < n / bs; b++) dequantize_block(t, src + b * bb, dst + b * bs);
    return 0;
}

float orc_vec_dot(int t, const uint8_t *w, const void *act, size_t n, int path) { return vec_dot(t, w, act, n, path); }

size_t orc_block_sums(int t, const uint8_t *w, const void *act, size_t n, int32_t *out) {
    const BlockQ8_0 *a0 = (const BlockQ8_0 *)act;
    const BlockQ8K *ak = (const BlockQ8K *)act;
    switch (t) {
        case T_Q4_0: dot_q4_0_s(w, a0, n / QK, out); return n / QK;
        case T_Q4_1: dot_q4_1_s(w, a0, n / QK, out); return n / QK;
        case T_Q5_0: dot_q5_0_s(w, a0, n / QK, out); return n / QK;
        case T_Q5_1: dot_q5_1_s(w, a0, n / QK, out); return n / QK;
        case T_Q8_0: dot_q8_0_s(w, a0, n / QK, out); return n / QK;
        case T_Q4_K: dot_q4_k_s(w, ak, n / QK_K, out); return 2 * (n / QK_K);
        case T_Q5_K: dot_q5_k_s(w, ak, n / QK_K, out); return 2 * (n / QK_K);
        case T_Q6_K: dot_q6_k_s(w, ak, n / QK_K, out); return n / QK_K;
        default: return 0;
    }
}

// kernels/matmul.rs:136-241 on pre-quantized activations
void orc_matmul_multi_q(int n_threads, const void *q8_0, const void *q8k, const float *xf32, size_t n_tok, size_t k,
                        const orc_job *jobs, size_t n_jobs, int path) {
    Pool &pool = pool_for(n_threads);
    struct Plan {
        const orc_job *j;
        size_t chunk, n_chunks;
    };
    std::vector<Plan> plans;
    size_t total = 0;
    for (size_t i = 0; i < n_jobs; i++) {
        const size_t rows = jobs[i].rows;
        const size_t target = std::max<size_t>(rows / ((size_t)pool.size() * 8), 16);
        const size_t chunk = (target + 3) / 4 * 4;
        const size_t nc = (rows + chunk - 1) / chunk;
        plans.push_back({&jobs[i], chunk, nc});
        total += nc;
    }
    const BlockQ8_0 *A0 = (const BlockQ8_0 *)q8_0;
    const BlockQ8K *AK = (const BlockQ8K *)q8k;
    auto act_row = [&](int fmt, size_t t) -> const void * {
        if (fmt == ACT_Q8_0) return A0 + t * (k / QK);
        if (fmt == ACT_Q8K) return AK + t * (k / QK_K);
        return xf32 + t * k;
    };
    pool.for_each(total, 1, [&](size_t c) {
        size_t pi = 0;
        while (c >= plans[pi].n_chunks) c -= plans[pi].n_chunks, pi++;
        const Plan &p = plans[pi];
        const orc_job &j = *p.j;
        const int t = j.ggml_type, fmt = act_format(t);
        const size_t rb = orc_row_bytes(t, j.cols);
        const size_t r0 = c * p.chunk, r1 = std::min<size_t>(r0 + p.chunk, j.rows);
        if (n_tok >= 4 && has_x4(t, path)) {
            for (size_t r = r0; r < r1; r++) {
                const uint8_t *wr = j.w + r * rb;
                size_t tt = 0;
                for (; tt + 4 <= n_tok; tt += 4) {
                    float res[4];
                    if (t == T_Q4_K) {
                        const BlockQ8K *a[4] = {AK + tt * (k / QK_K), AK + (tt + 1) * (k / QK_K), AK + (tt + 2) * (k / QK_K), AK + (tt + 3) * (k / QK_K)};
                        dot4_q4_k_avx2(wr, a, k / QK_K, res);
                    } else {
                        const BlockQ8_0 *a[4] = {A0 + tt * (k / QK), A0 + (tt + 1) * (k / QK), A0 + (tt + 2) * (k / QK), A0 + (tt + 3) * (k / QK)};
                        if (t == T_Q8_0)
                            dot4_q8_0_avx2(wr, a, k / QK, res);
                        else
                            dot4_q4_0_avx2(wr, a, k / QK, res);
                    }
                    for (int q = 0; q < 4; q++) j.out[(tt + q) * j.ld + r] = res[q];
                }
                for (; tt < n_tok; tt++) j.out[tt * j.ld + r] = vec_dot(t, wr, act_row(fmt, tt), k, path);
            }
            return;
        }
        for (size_t r = r0; r < r1; r++) {
            const uint8_t *wr = j.w + r * rb;
            for (size_t tt = 0; tt < n_tok; tt++) j.out[tt * j.ld + r] = vec_dot(t, wr, act_row(fmt, tt), k, path);
        }
    });
}

// QuantActs::prepare (kernels/matmul.rs:34-71) followed by matmul_multi.
void orc_matmul_multi(int n_threads, const float *x, size_t n_tok, size_t k, const orc_job *jobs, size_t n_jobs, int path) {
    Pool &pool = pool_for(n_threads);
    bool need0 = false, needk = false;
    for (size_t i = 0; i < n_jobs; i++) {
        const int f = act_format(jobs[i].ggml_type);
        need0 |= f == ACT_Q8_0;
        needk |= f == ACT_Q8K;
    }
    std::vector<BlockQ8_0> a0(need0 ? n_tok * (k / QK) : 0);
    std::vector<BlockQ8K> ak(needk ? n_tok * (k / QK_K) : 0);
    if (need0) pool.for_each(n_tok, 1, [&](size_t t) { quantize_acts_q8_0(x + t * k, k, a0.data() + t * (k / QK), path); });
    if (needk) pool.for_each(n_tok, 1, [&](size_t t) { quantize_q8_k(x + t * k, k / QK_K, ak.data() + t * (k / QK_K)); });
    orc_matmul_multi_q(n_threads, a0.data(), ak.data(), x, n_tok, k, jobs, n_jobs, path);
}

uint64_t orc_kv_seed(void) { return KV_SEED; }
float orc_turbo_sign(uint64_t seed, size_t i) { return turbo_sign(seed, i); }
size_t orc_turbo_block_size(size_t d) { return turbo_block(d); }
size_t orc_turbo_row_bytes_4(size_t d) { return row_bytes_4(d); }
void orc_turbo_rotate(uint64_t seed, float *x, size_t d, int inverse) { rotate(seed, x, d, inverse != 0); }
void orc_turbo_fwht(float *x, size_t n) { fwht(x, n); }
void orc_turbo_quantize_rotated_4(const float *y, size_t d, uint8_t *row) { quantize_rotated_4(y, d, row); }
void orc_turbo_quantize_4(uint64_t seed, const float *x, size_t d, uint8_t *row) {  // turbo.rs:167-171
    std::vector<float> s(x, x + d);
    rotate(seed, s.data(), d, false);
    quantize_rotated_4(s.data(), d, row);
}
float orc_turbo_dot_rotated_4(const void *q, const uint8_t *row, size_t d, int path) {
    return dot_rotated_4((const BlockQ8_0 *)q, row, d, path);
}
void orc_turbo_axpy_rotated_4(float *y, float a, const uint8_t *row, size_t d, int path) { axpy_rotated_4(y, a, row, d, path); }
void orc_turbo_dequantize_4(uint64_t seed, const uint8_t *row, float *out, size_t d) {  // turbo.rs:253-257
    std::fill(out, out + d, 0.0f);
    axpy_rotated_4(out, 1.0f, row, d, ORC_PATH_SCALAR);
    rotate(seed, out, d, true);
}
void orc_turbo_codebook(int bits, float *out) {  // turbo.rs:28-38
    const float *h = bits == 2 ? LM2 : LM4;
    const int n = bits == 2 ? 2 : 8;
    for (int i = 0; i < n; i++) out[i] = -h[n - 1 - i];
    for (int i = 0; i < n; i++) out[n + i] = h[i];
}
void orc_turbo_kv_levels(float *out16) { kv_levels(out16); }

void orc_kv_store(int kv_type, const float *x, size_t hd, void *dst, int path) {  // model/cpu.rs:300-328
    switch (kv_type) {
        case ORC_KV_F16: orc_f32_to_f16_n(x, (uint16_t *)dst, hd, path); break;
        case ORC_KV_Q8_0: store_q8_0(x, hd, (uint8_t *)dst); break;
        case ORC_KV_TURBO4: orc_turbo_quantize_4(KV_SEED, x, hd, (uint8_t *)dst); break;
        default: break;
    }
}

// model/cpu.rs:552-634
void orc_attention(int n_threads, size_t n_head, size_t n_head_kv, size_t hd, size_t n_tok, size_t pos0, size_t window,
                   float softcap, const float *q, int kv_type, const void *kcache, const void *vcache, size_t slots,
                   float *out, int path) {
    Pool &pool = pool_for(n_threads);
    const size_t qd = n_head * hd, group = n_head / n_head_kv;
    const size_t rb = kv_type == ORC_KV_TURBO4 ? row_bytes_4(hd) : hd / QK * 34;
    pool.for_each(n_tok * n_head, 1, [&](size_t task) {
        const size_t t = task / n_head, h = task % n_head, g = h / group;
        const size_t p = pos0 + t;
        const size_t start = window > 0 ? (p + 1 > window ? p + 1 - window : 0) : 0;
        const size_t len = p + 1 - start;
        const float *qh = q + t * qd + h * hd;
        std::vector<float> sc(len);
        std::vector<float> qrot(hd);
        std::vector<BlockQ8_0> qq(hd / QK);
        if (kv_type == ORC_KV_TURBO4) {
            std::copy(qh, qh + hd, qrot.begin());
            rotate(KV_SEED, qrot.data(), hd, false);
            quantize_acts_q8_0(qrot.data(), hd, qq.data(), path);
        } else if (kv_type == ORC_KV_Q8_0) {
            quantize_acts_q8_0(qh, hd, qq.data(), path);
        }
        float mx = -INFINITY;
        for (size_t i = 0; i < len; i++) {
            const size_t row = g * slots + (start + i) % slots;
            float v;
            if (kv_type == ORC_KV_F16)
                v = dot_f16_f32((const uint16_t *)kcache + row * hd, qh, hd, path);
            else if (kv_type == ORC_KV_Q8_0)
                v = vec_dot(T_Q8_0, (const uint8_t *)kcache + row * rb, qq.data(), hd, path);
            else
                v = dot_rotated_4(qq.data(), (const uint8_t *)kcache + row * rb, hd, path);
            if (softcap > 0.0f) v = softcap * std::tanh(v / softcap);
            sc[i] = v;
            mx = std::fmax(mx, v);
        }
        float sum = 0.0f;
        for (size_t i = 0; i < len; i++) {
            sc[i] = std::exp(sc[i] - mx);
            sum += sc[i];
        }
        const float inv = 1.0f / sum;
        float *o = out + t * qd + h * hd;
        std::fill(o, o + hd, 0.0f);
        for (size_t i = 0; i < len; i++) {
            const size_t row = g * slots + (start + i) % slots;
            if (kv_type == ORC_KV_F16)
                axpy_f16(o, sc[i] * inv, (const uint16_t *)vcache + row * hd, hd, path);
            else if (kv_type == ORC_KV_Q8_0)
                axpy_q8_0(o, sc[i] * inv, (const uint8_t *)vcache + row * rb, hd);
            else
                axpy_rotated_4(o, sc[i] * inv, (const uint8_t *)vcache + row * rb, hd, path);
        }
        if (kv_type == ORC_KV_TURBO4) rotate(KV_SEED, o, hd, true);
    });
}

// ops.rs:6-109
void orc_rmsnorm(float *out, const float *x, const float *w, size_t n, float eps, int path) {
    const float ss = dot_f32(x, x, n, path) / (float)n;
    const float scale = 1.0f / std::sqrt(ss + eps);
    for (size_t i = 0; i < n; i++) out[i] = x[i] * scale * w[i];
}
void orc_rope_table(size_t dim, float base, float freq_scale, size_t pos, float *cos_out, float *sin_out) {
    for (size_t i = 0; i < dim / 2; i++) {
        const float f = std::pow(base, -2.0f * (float)i / (float)dim) * freq_scale;
        const float theta = (float)pos * f;
        cos_out[i] = std::cos(theta);
        sin_out[i] = std::sin(theta);
    }
}
void orc_rope_apply(float *x, size_t dim, int neox, const float *c, const float *s) {
    const size_t half = dim / 2;
    for (size_t i = 0; i < half; i++) {
        const size_t i0 = neox ? i : 2 * i, i1 = neox ? i + half : 2 * i + 1;
        const float a = x[i0], b = x[i1];
        x[i0] = a * c[i] - b * s[i];
        x[i1] = a * s[i] + b * c[i];
    }
}
float orc_silu(float x) { return x / (1.0f + std::exp(-x)); }
float orc_dot_f32(const float *a, const float *b, size_t n, int path) { return dot_f32(a, b, n, path); }

}  // extern "C"
