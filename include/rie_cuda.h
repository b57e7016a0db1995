/*
 * rie_cuda.h -- C ABI of librie_cuda.so: the B200 (sm_100a) implementation of the Rust
 * Inference Engine's quantized-matmul + turbo4 KV-cache hot path.
 *
 * Conventions follow the reference's C ABI (crates/rie-ffi/include/rie.h:1-78 and
 * crates/rie-ffi/src/lib.rs:84-157): opaque handles, int32_t status (0 = ok), a
 * human-readable reason retrievable per context (rcu_last_error) or written into a
 * caller buffer, no exception or abort ever crosses the boundary, and one context must
 * not be used from two host threads at once. Device memory handed to the library
 * (x_dev, out, ...) is plain device pointers; the library never frees caller memory.
 * All operations are asynchronous on the context's stream; rcu_sync waits for them.
 *
 * Each entry point cites the reference interface it replaces (path:line within the
 * reference project).
 */
#ifndef RIE_CUDA_H
#define RIE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define RCU_API __attribute__((visibility("default")))
#else
#define RCU_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct rcu_ctx rcu_ctx;
typedef struct rcu_weight rcu_weight;
typedef struct rcu_acts rcu_acts;
typedef struct rcu_kv rcu_kv;

enum rcu_status {
    RCU_OK = 0,
    RCU_ERR_INVALID = 1,     /* bad argument, shape or handle */
    RCU_ERR_CUDA = 2,        /* CUDA runtime error (message holds cudaGetErrorString) */
    RCU_ERR_UNSUPPORTED = 3, /* type/format not implemented on this path */
    RCU_ERR_OOM = 4,         /* device allocation failed */
    RCU_ERR_TIMEOUT = 5,     /* a bounded device-side wait expired (see rcu_check_device) */
    RCU_ERR_RUNTIME = 6      /* reference Error::Runtime (empty batch, context full, ...) */
};

/* Rounding of the Q8_0 activation quantizer. The reference's SIMD tiers (AVX2
 * _mm256_cvtps_epi32, NEON vcvtnq_s32_f32: kernels/avx2.rs:173, kernels/neon.rs:478-505)
 * round half to even; its scalar tier (quant/mod.rs:182, f32::round) rounds half away from
 * zero. Q8_K quantization is scalar on every tier and always rounds half away. */
enum rcu_rounding { RCU_ROUND_NEAREST_EVEN = 0, RCU_ROUND_HALF_AWAY = 1 };

/* Activation formats (reference ActFormat, quant/mod.rs:127-132), as bit flags. */
enum rcu_act_format { RCU_ACT_Q8_0 = 2, RCU_ACT_Q8K = 4 };

/* KV cache formats (reference KvType, model/cpu.rs:12-36). */
enum rcu_kv_type { RCU_KV_F16 = 0, RCU_KV_Q8_0 = 1, RCU_KV_TURBO4 = 2 };

/* ---- context ------------------------------------------------------------------------ */
/* Creates a context on `device` issuing work on `stream` (cudaStream_t, NULL = the
 * legacy default stream). Replaces the CPU backend's thread pool / scratch ownership
 * (model/cpu.rs:93-177). On failure *out is NULL and err (if non-NULL) holds the reason. */
RCU_API int32_t rcu_ctx_create(int32_t device, void *stream, rcu_ctx **out, char *err, size_t err_len);
RCU_API void rcu_ctx_destroy(rcu_ctx *ctx);
RCU_API int32_t rcu_set_stream(rcu_ctx *ctx, void *stream);
RCU_API int32_t rcu_set_rounding(rcu_ctx *ctx, int32_t mode);
/* Prefill matmul kernel (batches above 8 tokens; replaces the 4-token / SMMLA tiles of
 * kernels/mod.rs:234-320 and matmul.rs:178-241). RCU_GEMM_F16 (default): every weight type,
 * weights dequantized as reference.rs:53-207 defines and activations as d * q of their Q8_0 /
 * Q8_K blocks, both rounded once to f16, f32 accumulation on the tensor cores. RCU_GEMM_I8:
 * Q4_0 weights through int8 MMA with the exact per-block int32 sums of reference.rs:221-233
 * (other types keep the f16 kernel). Both stay within the matmul tolerance of the reference. */
enum rcu_gemm_kind { RCU_GEMM_F16 = 0, RCU_GEMM_I8 = 1 };
RCU_API int32_t rcu_set_prefill_gemm(rcu_ctx *ctx, int32_t kind);
/* Caller promise (no counterpart in the reference): the weights of this context are never
 * written by a kernel after their upload. A matmul may then stream its weights before the
 * kernel ahead of it in the stream has finished (programmatic dependent launch), as the
 * forward always does. Off by default. */
RCU_API int32_t rcu_set_static_weights(rcu_ctx *ctx, int32_t on);
/* Last error message of this context ("" if none). Valid until the next call. */
RCU_API const char *rcu_last_error(const rcu_ctx *ctx);
/* Waits for all work on the context stream; returns RCU_ERR_TIMEOUT if any bounded
 * device wait expired since the last check (the bits are then cleared). */
RCU_API int32_t rcu_sync(rcu_ctx *ctx);
RCU_API int32_t rcu_check_device(rcu_ctx *ctx, uint32_t *bits_out);
/* Limit of the device-side waits on other ranks (the fused all-reduce), 1..600000 ms; default
 * 2000 ms or RIE_WAIT_LIMIT_MS at context creation. A wait that runs out sets a device error
 * bit (RCU_ERR_TIMEOUT from rcu_sync / rcu_check_device) and the kernel finishes. No counterpart
 * in the reference (no device waits there). */
RCU_API int32_t rcu_set_wait_limit_ms(rcu_ctx *ctx, uint64_t ms);
/* Diagnostics (no counterpart in the reference): launches the fused all-reduce norm of one row
 * against arrival counters that no rank will raise, so its bounded wait runs out after the
 * context's wait limit; returns what rcu_sync then reports (RCU_ERR_TIMEOUT, error bits 0x10).
 * The context stays usable. */
RCU_API int32_t rcu_diag_expire_peer_wait(rcu_ctx *ctx);
RCU_API int32_t rcu_version(void);

/* ---- weights (tensor.rs:6-98 Weight) -------------------------------------------------- */
/* Block layout helpers (quant/mod.rs:69-96). */
RCU_API uint64_t rcu_row_bytes(uint32_t ggml_type, uint64_t cols);
/* Copies `rows` rows of raw GGUF block bytes (ggml type id as in gguf: 2 = Q4_0, 12 =
 * Q4_K, ...) from host memory to the device. No repacking: rows keep the GGUF layout. */
RCU_API int32_t rcu_weight_upload(rcu_ctx *ctx, uint32_t ggml_type, uint64_t rows, uint64_t cols, const void *host_bytes,
                          rcu_weight **out);
/* Zero-copy view of GGUF block bytes already on the device (Weight::from_raw,
 * tensor.rs:31-35). The base must be 16-byte aligned and rows*row_bytes readable up to
 * the next multiple of 16. */
RCU_API int32_t rcu_weight_view(rcu_ctx *ctx, uint32_t ggml_type, uint64_t rows, uint64_t cols, const void *dev_bytes,
                        rcu_weight **out);
/* Quantizes f32 weights (rows x cols, row stride ld floats, device) into GGUF blocks of
 * ggml_type (rows x rcu_row_bytes(type, cols) bytes, device), asynchronously on the context
 * stream. Q8_0 and Q4_0 follow the reference's weight quantizers (quant/mod.rs:262-307); the
 * reference has none for Q4_1, Q5_0, Q5_1, Q4_K, Q5_K, Q6_K, which use this library's own rules
 * (valid blocks of the reference layouts, quant/reference.rs:53-207). */
RCU_API int32_t rcu_quantize_weight(rcu_ctx *ctx, uint32_t ggml_type, uint64_t rows, uint64_t cols, const float *x_dev,
                                    uint64_t ld, void *out_dev);
/* Rows [start, start+n) of w (Weight::slice_rows, tensor.rs:64-69); shares storage. */
RCU_API int32_t rcu_weight_slice_rows(const rcu_weight *w, uint64_t start, uint64_t n, rcu_weight **out);
RCU_API void rcu_weight_free(rcu_weight *w);
RCU_API const void *rcu_weight_device_ptr(const rcu_weight *w);

/* ---- activations (kernels/matmul.rs:19-97 QuantActs) ---------------------------------- */
RCU_API int32_t rcu_acts_create(rcu_ctx *ctx, uint64_t max_tok, uint64_t max_k, rcu_acts **out);
RCU_API void rcu_acts_free(rcu_acts *acts);
/* QuantActs::prepare (matmul.rs:34-71): quantize x_dev (n_tok x k f32, row-major, device)
 * once into every format in `formats` (RCU_ACT_* bits). Q8_0 follows the context's
 * rounding mode; Q8_K follows quant/mod.rs:191-218. */
RCU_API int32_t rcu_acts_prepare(rcu_ctx *ctx, rcu_acts *acts, const float *x_dev, uint64_t n_tok, uint64_t k,
                         uint32_t formats);
/* Writes the prepared blocks to host memory in the reference's own block layout
 * (BlockQ8_0 = 48 bytes: qs[32], f32 d, f32 s; BlockQ8K = 304 bytes: qs[256],
 * i16 bsums[16], f32 d; quant/mod.rs:139-168). Synchronous. */
RCU_API int32_t rcu_acts_export(rcu_ctx *ctx, const rcu_acts *acts, uint32_t format, void *host_out);

/* ---- matmul (kernels/matmul.rs:110-176) ----------------------------------------------- */
typedef struct rcu_job {
    const rcu_weight *w; /* rows x k weight */
    float *out;          /* device: out[t * ld + r] = W[r] . X[t] */
    uint64_t ld;         /* leading dimension (usually w->rows) */
} rcu_job;
/* matmul_multi: every job shares the prepared activations and runs in one launch.
 * Tokens <= 8 use the HBM-streaming GEMV; more tokens use the int8 tensor-core GEMM. */
RCU_API int32_t rcu_matmul_multi(rcu_ctx *ctx, const rcu_acts *acts, const rcu_job *jobs, uint64_t n_jobs);
RCU_API int32_t rcu_matmul(rcu_ctx *ctx, const rcu_acts *acts, const rcu_weight *w, float *out);
/* Exact per-block integer sums of weight row `row` with activation row `tok`
 * (the int32 `s`/`sumi`/`summ` of quant/reference.rs:221-386): one int32 per 32-block
 * for Q4_0/Q4_1/Q5_0/Q5_1/Q8_0, (sumi, summ) per superblock for Q4_K/Q5_K, sumi per
 * superblock for Q6_K. out_dev must hold that many int32. */
RCU_API int32_t rcu_block_sums(rcu_ctx *ctx, const rcu_acts *acts, const rcu_weight *w, uint64_t row, uint64_t tok,
                       int32_t *out_dev);

/* The batch-1 matmul of activation row 0 with every row of w, as rcu_matmul runs it, on the
 * kernel named by `kernel` (0: the lane GEMV, any block type; 1: the tensor-core GEMV, Q4_K /
 * Q5_K / Q6_K / Q4_0), with the exact per-block integer sums that kernel forms captured on the
 * way: sums_dev[row * n + i] in the layout of rcu_block_sums (n of them per row). A validation
 * variant of the same kernels (quant/reference.rs:221-386 block sums; kernels/matmul.rs:136-241
 * for the f32 outputs in `out`). sums_dev is cleared first. */
RCU_API int32_t rcu_matmul_block_sums(rcu_ctx *ctx, const rcu_acts *acts, const rcu_weight *w, float *out,
                                      int32_t *sums_dev, int32_t kernel);

/* ---- turbo4 (turbo.rs) --------------------------------------------------------------- */
/* row_bytes_4 (turbo.rs:136-138): f16 scale per rotation block + hd/2 code bytes. */
RCU_API uint64_t rcu_turbo4_row_bytes(uint64_t hd);
/* quantize_4 (turbo.rs:167-171) of n_rows rows of hd f32 (device) with the KV_SEED
 * rotation, written as reference-format rows (scales then Q4_0-order nibbles). */
RCU_API int32_t rcu_turbo4_quantize(rcu_ctx *ctx, const float *x_dev, uint64_t n_rows, uint64_t hd, uint8_t *rows_dev);
/* Rotation::apply / apply_inverse (turbo.rs:108-117) of n_rows rows, in place. */
RCU_API int32_t rcu_turbo4_rotate(rcu_ctx *ctx, float *x_dev, uint64_t n_rows, uint64_t hd, int32_t inverse);

/* ---- KV cache + attention (model/cpu.rs:38-50, 300-328, 550-658) ------------------- */
/* One layer's cache: n_head_kv heads x `slots` positions of head_dim values, in the given
 * format. Sliding-window layers pass slots = window + max_batch (cpu.rs:111). */
RCU_API int32_t rcu_kv_create(rcu_ctx *ctx, int32_t kv_type, uint64_t n_head_kv, uint64_t head_dim, uint64_t slots,
                      rcu_kv **out);
RCU_API void rcu_kv_free(rcu_kv *kv);
/* KV append of n_tok tokens at positions pos0.. (slot = pos % slots): k_dev, v_dev are
 * n_tok x (n_head_kv*head_dim) f32 on the device (post-RoPE keys). */
RCU_API int32_t rcu_kv_store(rcu_ctx *ctx, rcu_kv *kv, const float *k_dev, const float *v_dev, uint64_t n_tok, uint64_t pos0);
/* Reads/writes the cache as reference-layout rows [kv_head][slot][row] (f16 bits, Q8_0
 * blocks, or row_bytes_4 turbo rows) for parity checks. Synchronous, host buffers. */
RCU_API int32_t rcu_kv_export(rcu_ctx *ctx, const rcu_kv *kv, void *k_host, void *v_host);
RCU_API int32_t rcu_kv_import(rcu_ctx *ctx, rcu_kv *kv, const void *k_host, const void *v_host);
/* attention() (model/cpu.rs:552-634): causal GQA attention of n_tok queries at positions
 * pos0.. over the cache; q_dev is n_tok x (n_head*head_dim) f32 (already scaled by
 * attn_scale), out_dev the same shape. window = 0 means full attention; softcap <= 0
 * means none. */
RCU_API int32_t rcu_attention(rcu_ctx *ctx, const rcu_kv *kv, const float *q_dev, uint64_t n_tok, uint64_t n_head,
                      uint64_t pos0, uint64_t window, float softcap, float *out_dev);

/* ---- transformer forward (model/mod.rs Model + Backend trait, model/cpu.rs) --------- */
typedef struct rcu_model rcu_model;
typedef struct rcu_backend rcu_backend;
/* Hyper-parameters (reference ModelConfig, model/config.rs:54-104), flattened. Optional
 * features use 0 / <= 0 for "absent". */
typedef struct rcu_model_config {
    uint32_t n_vocab, n_embd, n_layer, n_head, n_head_kv, head_dim, n_ff;
    uint32_t rope_dim;
    int32_t rope_neox;                /* 1: rotate (x[i], x[i+dim/2]); 0: (x[2i], x[2i+1]) */
    float rope_base, rope_freq_scale;
    float rms_eps, attn_scale, embd_scale, residual_scale, logit_scale;
    float attn_softcap, final_softcap;
    uint32_t swa_window, swa_pattern;
    float rope_base_swa;
    int32_t act;                      /* 0 SiLU, 1 GELU (tanh) */
    uint32_t n_expert, n_expert_used, n_ff_exp;
    int32_t expert_norm_topk, expert_unit_weights;
} rcu_model_config;
/* Model::load (model/mod.rs:112-247) without the file: the caller hands over every GGUF
 * tensor by its GGUF name ("token_embd.weight", "blk.0.attn_q.weight", ...). */
RCU_API int32_t rcu_model_create(rcu_ctx *ctx, const rcu_model_config *cfg, rcu_model **out);
RCU_API void rcu_model_free(rcu_model *m);
RCU_API int32_t rcu_model_set_tensor(rcu_model *m, const char *name, uint32_t ggml_type, uint64_t rows, uint64_t cols,
                                     const void *host_bytes);
/* rcu_model_set_tensor from the tensor's GGUF bytes in device memory (no counterpart in the
 * reference: its weights come from a memory-mapped file). The model keeps its own copy (this
 * rank's shard under tensor parallelism); dev_bytes may be freed after the call. */
RCU_API int32_t rcu_model_set_tensor_device(rcu_model *m, const char *name, uint32_t ggml_type, uint64_t rows,
                                            uint64_t cols, const void *dev_bytes);
/* CpuBackend::with_kv_type (model/cpu.rs:100-177): KV caches and scratch for n_ctx
 * positions and batches of up to max_batch tokens. Validates the model's tensors. */
RCU_API int32_t rcu_backend_create(rcu_model *m, uint64_t n_ctx, uint64_t max_batch, int32_t kv_type,
                                   rcu_backend **out);
RCU_API void rcu_backend_free(rcu_backend *b);
RCU_API uint64_t rcu_backend_max_batch(const rcu_backend *b);
RCU_API uint64_t rcu_backend_n_ctx(const rcu_backend *b);
/* Backend::forward (model/mod.rs:313): evaluate tokens at positions pos..pos+n; writes the
 * last token's logits (n_vocab floats) or all n rows when all_logits. Host buffers;
 * synchronous. Errors as the reference: empty batch, batch > max, context full, token id
 * out of range (RCU_ERR_RUNTIME). */
RCU_API int32_t rcu_backend_forward(rcu_backend *b, const uint32_t *tokens, uint64_t n, uint64_t pos,
                                    int32_t all_logits, float *logits, uint64_t logits_len);
/* Same on device buffers, asynchronous on the context stream (tokens_dev: n uint32). */
RCU_API int32_t rcu_backend_forward_device(rcu_backend *b, const uint32_t *tokens_dev, uint64_t n, uint64_t pos,
                                           int32_t all_logits, float *logits_dev);
/* Partial forward (no counterpart in the reference): layers [layer0, layer1) for n tokens at
 * positions pos..pos+n-1, starting from hidden rows x_dev (n x n_embd f32, device) instead of
 * the token embeddings; those layers' KV caches are appended as by rcu_backend_forward. Writes
 * the residual stream after layer layer1 - 1 to x_out_dev (n x n_embd, may be NULL) and, when
 * logits_dev is not NULL (layer1 must be n_layer), every row's logits (n x n_vocab).
 * Asynchronous on the context stream. For pipeline stages and layer-by-layer parity checks. */
RCU_API int32_t rcu_backend_forward_layers(rcu_backend *b, const float *x_dev, uint64_t n, uint64_t pos,
                                           uint64_t layer0, uint64_t layer1, float *x_out_dev, float *logits_dev);
/* Backend::hidden (model/mod.rs:318): final normed rows of the last forward (rows x n_embd). */
RCU_API int32_t rcu_backend_hidden(const rcu_backend *b, float *host_out, uint64_t cap, uint64_t *rows_out);
/* The KV cache of one layer (owned by the backend), e.g. to fill it with rcu_kv_import. */
RCU_API int32_t rcu_backend_kv(rcu_backend *b, uint64_t layer, rcu_kv **out);

/* ---- tensor parallelism over NCCL (no counterpart in the reference: it has no multi-device
 * code). One process (or thread) per GPU, each with its own context. -------------------- */
/* A model holding rank `rank` of `world` shards: rcu_model_set_tensor takes the full GGUF
 * tensors and keeps this rank's part (q/k/v and gate/up rows by head / FFN row, the output
 * head's vocabulary rows, attn_output and ffn_down column blocks; the rest replicated). */
RCU_API int32_t rcu_model_create_tp(rcu_ctx *ctx, const rcu_model_config *cfg, int32_t rank, int32_t world,
                                    rcu_model **out);
/* Host-only: the shard rcu_model_set_tensor keeps for (rank, world); out == NULL reports the
 * shape only. With fewer KV heads than ranks, k / v rows and biases are those of KV head
 * rank / (world / n_head_kv): each KV head is replicated on world / n_head_kv ranks. */
RCU_API int32_t rcu_tp_shard(const rcu_model_config *cfg, const char *name, uint32_t ggml_type, uint64_t rows,
                             uint64_t cols, const void *host_bytes, int32_t rank, int32_t world, void *out,
                             uint64_t out_cap, uint64_t *out_rows, uint64_t *out_cols);
/* Communicator id (128 bytes) made on one rank and handed to every rank. */
RCU_API int32_t rcu_tp_unique_id(uint8_t *out, uint64_t cap);
/* rcu_backend_create for a tensor-parallel model: all ranks call it with the same id; Wo and
 * ffn_down outputs are all-reduced, the vocabulary-parallel logits all-gathered, so every
 * rank's forward returns the full logits. */
RCU_API int32_t rcu_backend_create_tp(rcu_model *m, uint64_t n_ctx, uint64_t max_batch, int32_t kv_type,
                                      const uint8_t *comm_id, rcu_backend **out);

/* ---- allocation-free matmul (no counterpart in the reference) ------------------------ */
/* W . X for f32 activations x_dev (n_tok x w->cols, device), out_dev[t * ld + r], without
 * allocating any device memory: the activations are quantized into a fixed scratch area
 * compiled into this library (about 322 KB, kept on every GPU that loads it until exit).
 * For callers that cannot cudaMalloc at matmul time, e.g. because all device memory is
 * owned by their own pool or by PyTorch's caching allocator. Limits: n_tok <= 8 and
 * w->cols <= 16384 (larger calls return RCU_ERR_INVALID); every call within them runs
 * (batches whose rows do not fit the GEMV's shared memory at once run as two launches).
 * All calls share the scratch, so calls that overlap on the GPU race; order them (one
 * stream per device). The first call through a context looks the scratch address up
 * (cudaGetSymbolAddress) and keeps it in the context: make that first call before any
 * stream capture. */
RCU_API int32_t rcu_matmul_f32_static(rcu_ctx *ctx, const rcu_weight *w, const float *x_dev, uint64_t n_tok,
                                      float *out_dev, uint64_t ld);

#ifdef __cplusplus
}
#endif
#endif /* RIE_CUDA_H */
