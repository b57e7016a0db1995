// rcu_kernels.h -- host launchers of librie_cuda's kernels (internal).
#pragma once
#include "rcu_internal.cuh"

namespace rcu {

int launch_quantize(rcu_ctx *ctx, const ActsView &a, const float *x, uint32_t n_tok, uint32_t k, uint32_t formats);

// Expert id an indirect job reads when the routed expert lives on another rank (expert
// parallelism): the GEMV skips the job and the combine leaves its output out.
constexpr uint32_t kNoExpert = 0xffffffffu;
struct HostJob {
    const rcu_weight *w;
    float *out;
    uint64_t ld;
    // indirect job (mixture of experts): weight = w + (*sel) * w_stride bytes with `rows`
    // rows (0: all of w), the expert id written on the device; activations from row `tok`
    const uint32_t *sel = nullptr;
    uint64_t w_stride = 0;
    uint32_t rows = 0;
    uint32_t tok = 0;
};
// Decode GEMV over up to kGemvMaxJobs jobs sharing one activation batch (n_tok <= 8).
constexpr int kGemvMaxJobs = 96;
// Fused all-reduce push of a one-job GEMV (tensor parallel): outputs also go to dst[q] (the
// peers' receive buffers, same [t][ld] layout) and, once all its CTAs have written their
// rows, the launch has added exactly kArUnit to each flag[q].
constexpr uint32_t kArUnit = 4096;
struct ArPush {
    float *dst[8];
    uint32_t *flag[8];
    uint32_t n_dst, n_flag;
};
int launch_gemv(rcu_ctx *ctx, const ActsView &a, const HostJob *jobs, int n_jobs, uint32_t tok0, uint32_t n_tok,
                const ArPush *push = nullptr);
// Batch-1 GEMV over Q4_K / Q5_K / Q6_K weights with the block dot products on the integer
// tensor-core path (launch_gemv uses it when gemv_kq_ok holds; same job semantics).
bool gemv_kq_ok(const rcu_ctx *ctx, const ActsView &a, const HostJob *jobs, int n_jobs);
int launch_gemv_kq(rcu_ctx *ctx, const ActsView &a, const HostJob *jobs, int n_jobs, uint32_t tok0,
                   const ArPush *push = nullptr);
// Prefill GEMM on the tensor cores (n_tok > 8). Returns RCU_ERR_UNSUPPORTED for shapes it
// lacks (the caller then runs GEMV slices). launch_gemm_f16: every weight type, operands
// dequantized to f16; the int8 kernel (exact per-block sums, Q4_0) when ctx->gemm_i8.
int launch_gemm(rcu_ctx *ctx, const ActsView &a, const HostJob *jobs, int n_jobs);
int launch_gemm_f16(rcu_ctx *ctx, const ActsView &a, const HostJob *jobs, int n_jobs);
bool gemm_f16_ok(const ActsView &a, const HostJob &j);
// Sizes the f16 activation scratch for n_tok x k (so a forward never allocates mid-stream).
int gemm_f16_reserve(rcu_ctx *ctx, uint64_t n_tok, uint64_t k);
// Grouped GEMM for mixture-of-experts batches: each weight is a stacked expert tensor
// (n_exp x grp_rows rows); the activation rows [off[e], off[e + 1]) (host copy of the device
// routing plan) go through expert e. gemm_f16_gather first writes those f16 rows (row i =
// activation row src_rows[i] of a) into the context scratch.
bool gemm_f16_grouped_ok(const rcu_weight *w, uint32_t k, uint32_t n_exp, uint32_t grp_rows);
int gemm_f16_gather(rcu_ctx *ctx, const ActsView &a, uint32_t fmt, const uint32_t *src_rows, uint32_t n_rows,
                    const __half **act, const float **scale);
int launch_gemm_f16_grouped(rcu_ctx *ctx, const __half *act, const float *scale, uint32_t n_rows, uint32_t k,
                            const HostJob *jobs, int n_jobs, uint32_t grp_rows, const uint32_t *off, uint32_t n_exp);
// Exact per-block integer sums of one (row, token) pair.
int launch_block_sums(rcu_ctx *ctx, const ActsView &a, const rcu_weight *w, uint64_t row, uint64_t tok,
                      int32_t *out);

// KV append / attention with the position either by value (pos_ptr == nullptr) or read
// from device memory (graph replay). n_split == 0 sizes the split grid from pos0; scratch
// == nullptr uses the context's growable scratch (may allocate). A caller-provided scratch
// (attention_scratch_bytes) must start zeroed: its leading completion counters reset
// themselves after every call.
int launch_kv_store(rcu_ctx *ctx, rcu_kv *kv, const float *k, const float *v, uint64_t n_tok, uint64_t pos0,
                    const uint64_t *pos_ptr);
// aq != nullptr fuses the activation quantization (for the Wo matmul) into the merge; out
// may then be nullptr.
struct ActOut;
struct QkvPostParams;
int launch_attention(rcu_ctx *ctx, const rcu_kv *kv, const float *q, uint64_t n_tok, uint64_t n_head, uint64_t pos0,
                     const uint64_t *pos_ptr, uint64_t window, float softcap, float *out, uint32_t n_split,
                     float *scratch, const ActOut *aq, const QkvPostParams *post = nullptr);
// Decode steps (one token) whose attention runs the head_dim-128 decode kernels can leave the
// q/k post-processing and KV append to them (launch_attention with `post`, q then raw).
bool attention_fuses_post(const rcu_kv *kv, uint64_t n_tok, uint64_t n_head);

// Bias, q/k norm, RoPE and attn_scale on the fused QKV output, with k and v appended to the
// cache at slot (*pos_ptr + t) % slots (q is updated in place).
struct QkvPostParams {
    float *q;
    const float *k, *v;
    const float *bq, *bk, *bv, *qn, *kn, *inv_freq;
    const uint64_t *pos_ptr;
    uint32_t n_tok, n_head, hd, rope_dim;
    int neox;
    float eps, attn_scale;
};
int launch_qkv_post_store(rcu_ctx *ctx, rcu_kv *kv, const QkvPostParams &p);
// Prompt batches of at least kPrefillAttnMinTok tokens over an f16 cache take the tensor-core
// attention (64 query rows per CTA, key blocks of 64); out is [n_tok][n_head * hd] f32.
constexpr uint64_t kPrefillAttnMinTok = 16;
bool attention_prefill_ok(int kv_type, uint64_t hd, uint64_t group, uint64_t n_tok);
int launch_attention_prefill(rcu_ctx *ctx, const void *kc, const void *vc, uint64_t n_kv, uint64_t hd, uint64_t slots,
                             const float *q, uint64_t n_tok, uint64_t n_head, uint64_t pos0, const uint64_t *pos_ptr,
                             uint64_t window, float softcap, float *out);
// Decode attention at head_dim 128 with 4 or 8 query heads per KV head (rcu_attn_dec.cu): the
// context of each (token, KV head) split over a cluster of CTAs (up to 8; more clusters merge
// through `parts`, per-(token, query head, cluster) rows of hd + 2 floats, with the counters
// `done`, zero between launches). max_len: the longest context the plan covers.
bool attention_dec_ok(int kv_type, uint64_t hd, uint64_t group);
uint32_t attention_dec_max_clusters(int kv_type, uint64_t max_len, uint64_t n_tok, uint64_t n_kv, int num_sms);
struct ActOut;
int launch_attention_dec(rcu_ctx *ctx, const uint8_t *kc, const uint8_t *vc, int kv_type, uint64_t n_kv,
                         uint64_t slots, uint64_t row_bytes, const float *q, uint64_t n_tok, uint64_t n_head,
                         uint64_t pos0, const uint64_t *pos_ptr, uint64_t max_len, uint64_t window, float softcap,
                         float *out, const ActOut *aq, uint32_t *done, float *parts,
                         const QkvPostParams *post = nullptr);
// Whether the merge can quantize in the same kernel for this head shape and act format
// (a GQA group's output must hold whole activation blocks).
bool attention_fused_merge_ok(uint64_t n_head, uint64_t n_kv, uint64_t hd, uint32_t fmt);
uint32_t attention_max_splits(const rcu_kv *kv, uint64_t window);
uint64_t attention_scratch_bytes(const rcu_kv *kv, uint64_t n_tok, uint64_t n_head, uint32_t n_split);
uint64_t attention_scratch_bytes_upto(const rcu_ctx *ctx, const rcu_kv *kv, uint64_t max_batch, uint64_t n_head,
                                      uint64_t window);

}  // namespace rcu
