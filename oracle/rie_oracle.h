/*
 * rie_oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * A CPU restatement of the Rust Inference Engine's (RIE) quantized matmul and turbo4
 * KV-cache path, used as the parity checker for the CUDA library and as the timed CPU
 * baseline. Nothing in the product (librie_cuda.so, the Python package) links or calls
 * this code; only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg do.
 *
 * Parity status: the reference is Rust-only and cannot be compiled in this image (no
 * cargo/rustc), so it is restated here. The restatement is pinned by the reference's own
 * known-answer and property tests (ported in tests/test_oracle.py); see the header of
 * rie_oracle.cpp for the file:line each function follows.
 *
 * "path" arguments select which of the reference's kernel tiers is mirrored:
 *   ORC_PATH_SCALAR = quant/reference.rs + quantize_row_q8_0_scalar (RIE_DISABLE=simd)
 *   ORC_PATH_AVX2   = the x86_64 dispatch of kernels/mod.rs (AVX2 kernels for
 *                     Q8_0/Q4_0/Q4_K/Q6_K and the Q8_0 quantizer, scalar for the rest)
 */
#ifndef RIE_ORACLE_H
#define RIE_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORC_PATH_SCALAR = 0, ORC_PATH_AVX2 = 1 };
enum { ORC_KV_F16 = 0, ORC_KV_Q8_0 = 1, ORC_KV_TURBO4 = 2 };

/* --- formats --------------------------------------------------------------------- */
int orc_have_avx2(void);
size_t orc_block_size(int ggml_type);
size_t orc_block_bytes(int ggml_type);
size_t orc_row_bytes(int ggml_type, size_t n);
size_t orc_sizeof_block_q8_0(void);   /* 48 */
size_t orc_sizeof_block_q8_k(void);   /* 304 */

/* --- half precision (crate `half` 2.7.1 semantics: RNE) ---------------------------- */
uint16_t orc_f32_to_f16(float x);
float orc_f16_to_f32(uint16_t h);
void orc_f32_to_f16_n(const float *src, uint16_t *dst, size_t n, int path);

/* --- RNG of crates/rie-core/src/testing.rs ----------------------------------------- */
uint64_t orc_rng_new(uint64_t seed);
uint64_t orc_rng_next(uint64_t *state);
void orc_rng_vec(uint64_t *state, float *out, size_t n, float scale);
int orc_random_weight(uint64_t *state, int ggml_type, size_t rows, size_t cols, float gain, uint8_t *out);

/* --- activation quantizers ---------------------------------------------------------- */
void orc_quantize_row_q8_0(const float *x, size_t n, void *blocks, int path);
void orc_quantize_row_q8_k(const float *x, size_t n, void *blocks);

/* --- weight quantizers / dequantizer ----------------------------------------------- */
/* Returns bytes written, 0 when the type has no quantizer. Q8_0/Q4_0/F16/F32 follow the
 * reference; the other block types use this oracle's own simple quantizers (the
 * reference has none), which only need to produce valid blocks. */
size_t orc_quantize_weight(int ggml_type, const float *x, size_t n, uint8_t *out);
int orc_dequantize_row(int ggml_type, const uint8_t *src, float *dst, size_t n);

/* --- dots ------------------------------------------------------------------------ */
/* act: BlockQ8_0[] or BlockQ8K[] (per weight type), or float[] for F32/F16/BF16. */
float orc_vec_dot(int ggml_type, const uint8_t *w, const void *act, size_t n, int path);
/* Exact per-block integer sums: one int32 per 32-block for Q4_0/Q4_1/Q5_0/Q5_1/Q8_0;
 * two per superblock (sumi, summ) for Q4_K/Q5_K; one (sumi) for Q6_K. Returns count. */
size_t orc_block_sums(int ggml_type, const uint8_t *w, const void *act, size_t n, int32_t *out);

/* --- matmul driver (kernels/matmul.rs) ---------------------------------------------- */
typedef struct orc_job {
    int32_t ggml_type;
    int32_t pad;
    uint64_t rows, cols;
    const uint8_t *w;
    float *out;
    uint64_t ld;
} orc_job;
/* Quantize x (n_tok x k) once per needed format, then run every job in one parallel
 * region, exactly like QuantActs::prepare + matmul_multi. */
void orc_matmul_multi(int n_threads, const float *x, size_t n_tok, size_t k, const orc_job *jobs,
                      size_t n_jobs, int path);
/* Same, on pre-quantized activations (q8_0 / q8k may be NULL if unused). */
void orc_matmul_multi_q(int n_threads, const void *q8_0, const void *q8k, const float *xf32,
                        size_t n_tok, size_t k, const orc_job *jobs, size_t n_jobs, int path);

/* --- turbo4 (turbo.rs) --------------------------------------------------------------- */
uint64_t orc_kv_seed(void);
float orc_turbo_sign(uint64_t seed, size_t i);
size_t orc_turbo_block_size(size_t d);
size_t orc_turbo_row_bytes_4(size_t d);
void orc_turbo_rotate(uint64_t seed, float *x, size_t d, int inverse);
void orc_turbo_fwht(float *x, size_t n);
void orc_turbo_quantize_4(uint64_t seed, const float *x, size_t d, uint8_t *row);
void orc_turbo_quantize_rotated_4(const float *y, size_t d, uint8_t *row);
float orc_turbo_dot_rotated_4(const void *q_blocks, const uint8_t *row, size_t d, int path);
void orc_turbo_axpy_rotated_4(float *y, float a, const uint8_t *row, size_t d, int path);
void orc_turbo_dequantize_4(uint64_t seed, const uint8_t *row, float *out, size_t d);
void orc_turbo_codebook(int bits, float *out);
void orc_turbo_kv_levels(float *out16);

/* --- attention (model/cpu.rs) -------------------------------------------------------- */
/* Cache layout [kv_head][slot][row]: f16 bits for ORC_KV_F16 (row = hd u16), Q8_0 rows of
 * hd/32*34 bytes for ORC_KV_Q8_0, turbo4 rows of row_bytes_4(hd) for ORC_KV_TURBO4. */
void orc_attention(int n_threads, size_t n_head, size_t n_head_kv, size_t hd, size_t n_tok,
                   size_t pos0, size_t window, float softcap, const float *q, int kv_type,
                   const void *kcache, const void *vcache, size_t slots, float *out, int path);
/* KV append of one head vector in the cache format (f16 / Q8_0 / turbo4 rows). */
void orc_kv_store(int kv_type, const float *x, size_t hd, void *dst_row, int path);

/* --- ops.rs ---------------------------------------------------------------------- */
void orc_rmsnorm(float *out, const float *x, const float *w, size_t n, float eps, int path);
void orc_rope_table(size_t dim, float base, float freq_scale, size_t pos, float *cos_out, float *sin_out);
void orc_rope_apply(float *x, size_t dim, int neox, const float *cos_t, const float *sin_t);
float orc_silu(float x);
float orc_dot_f32(const float *a, const float *b, size_t n, int path);

#ifdef __cplusplus
}
#endif
#endif
