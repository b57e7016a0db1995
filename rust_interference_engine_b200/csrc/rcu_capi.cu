// rcu_capi.cu -- the extern "C" boundary of librie_cuda: contexts, weights, quantized
// activations and the matmul dispatcher. Status codes and error strings follow the
// reference's C ABI conventions (crates/rie-ffi/src/lib.rs:84-157): nothing throws or
// aborts across the boundary; every failure returns a status and records a message.
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>
#include <vector>

#include "rcu_kernels.h"

namespace rcu {
int set_err(rcu_ctx *c, int code, const std::string &msg) {
    if (c) c->last_error = msg;
    return code;
}
int cuda_err(rcu_ctx *c, cudaError_t e, const char *what) {
    std::string m = std::string(what) + ": " + cudaGetErrorString(e);
    if (e == cudaErrorMemoryAllocation) return set_err(c, RCU_ERR_OOM, m);
    return set_err(c, RCU_ERR_CUDA, m);
}
static void write_err(char *err, size_t err_len, const std::string &m) {
    if (!err || err_len == 0) return;
    const size_t n = std::min(err_len - 1, m.size());
    std::memcpy(err, m.data(), n);
    err[n] = 0;
}
static uint64_t row_bytes(int t, uint64_t cols) {
    const int bs = block_size(t);
    return bs ? cols / bs * block_bytes(t) : 0;
}
}  // namespace rcu

using namespace rcu;

#define RCU_GUARD_BEGIN try {
#define RCU_GUARD_END(ctx)                                              \
    }                                                                   \
    catch (const std::bad_alloc &) {                                    \
        return set_err((ctx), RCU_ERR_OOM, "host allocation failed");   \
    }                                                                   \
    catch (...) {                                                       \
        return set_err((ctx), RCU_ERR_RUNTIME, "internal exception");   \
    }

namespace rcu {
cudaError_t prefer_max_shared(const void *kern) {
    // kernels already configured on the current device; a handful of entries
    static std::mutex mu;
    static std::vector<std::pair<int, const void *>> done;
    int dev = 0;
    if (cudaError_t e = cudaGetDevice(&dev)) return e;
    std::lock_guard<std::mutex> g(mu);
    for (auto &d : done)
        if (d.first == dev && d.second == kern) return cudaSuccess;
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                               (int)cudaSharedmemCarveoutMaxShared);
    if (e == cudaSuccess) done.emplace_back(dev, kern);
    return e;
}
}  // namespace rcu

extern "C" {

int32_t rcu_version(void) { return 1; }

int32_t rcu_ctx_create(int32_t device, void *stream, rcu_ctx **out, char *err, size_t err_len) {
    if (!out) return RCU_ERR_INVALID;
    *out = nullptr;
    rcu_ctx *c = new (std::nothrow) rcu_ctx();
    if (!c) {
        write_err(err, err_len, "host allocation failed");
        return RCU_ERR_OOM;
    }
    auto fail = [&](int code) {
        write_err(err, err_len, c->last_error);
        delete c;
        return code;
    };
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return fail(cuda_err(c, e, "cudaSetDevice"));
    cudaDeviceProp prop;
    e = cudaGetDeviceProperties(&prop, device);
    if (e != cudaSuccess) return fail(cuda_err(c, e, "cudaGetDeviceProperties"));
    if (prop.major < 10) {
        set_err(c, RCU_ERR_UNSUPPORTED, "librie_cuda needs an sm_100 (Blackwell B200) device");
        return fail(RCU_ERR_UNSUPPORTED);
    }
    c->device = device;
    c->stream = (cudaStream_t)stream;
    c->num_sms = prop.multiProcessorCount;
    c->max_smem_optin = prop.sharedMemPerBlockOptin;
    if (const char *v = std::getenv("RIE_CUDA_PDL")) c->pdl = std::strcmp(v, "0") != 0;
    if (const char *v = std::getenv("RIE_WAIT_LIMIT_MS")) {
        const uint64_t ms = std::strtoull(v, nullptr, 10);
        if (ms > 0) c->wait_limit_ns = ms * 1000000ull;
    }
    if (const char *v = std::getenv("RIE_GEMV_KQ")) c->gemv_kq = std::strcmp(v, "0") != 0;
    if (const char *v = std::getenv("RIE_GEMV_KQ_MIN_MB")) c->gemv_kq_min_bytes = std::strtoull(v, nullptr, 10) << 20;
    if (const char *v = std::getenv("RIE_GEMV_KQ_Q4_0_MIN_K")) c->gemv_kq_q4_0_min_k = (uint32_t)std::strtoul(v, nullptr, 10);
    if (const char *v = std::getenv("RIE_FUSE_POST")) c->fuse_post = std::strcmp(v, "0") != 0;
    e = cudaMalloc(&c->dev_err, sizeof(uint32_t));
    if (e != cudaSuccess) return fail(cuda_err(c, e, "cudaMalloc(err)"));
    e = cudaMemset(c->dev_err, 0, sizeof(uint32_t));
    if (e != cudaSuccess) return fail(cuda_err(c, e, "cudaMemset(err)"));
    *out = c;
    return RCU_OK;
}

void rcu_ctx_destroy(rcu_ctx *ctx) {
    if (!ctx) return;
    cudaSetDevice(ctx->device);
    if (ctx->dev_err) cudaFree(ctx->dev_err);
    if (ctx->h_act) cudaFree(ctx->h_act);
    if (ctx->k_part) cudaFree(ctx->k_part);
    if (ctx->k_cnt) cudaFree(ctx->k_cnt);
    delete ctx;
}

int32_t rcu_set_stream(rcu_ctx *ctx, void *stream) {
    if (!ctx) return RCU_ERR_INVALID;
    ctx->stream = (cudaStream_t)stream;
    return RCU_OK;
}

int32_t rcu_set_rounding(rcu_ctx *ctx, int32_t mode) {
    if (!ctx) return RCU_ERR_INVALID;
    if (mode != RCU_ROUND_NEAREST_EVEN && mode != RCU_ROUND_HALF_AWAY)
        return set_err(ctx, RCU_ERR_INVALID, "unknown rounding mode");
    ctx->rounding = mode;
    return RCU_OK;
}

int32_t rcu_set_static_weights(rcu_ctx *ctx, int32_t on) {
    if (!ctx) return RCU_ERR_INVALID;
    ctx->static_weights = on != 0;
    ctx->early_weights = ctx->static_weights;
    return RCU_OK;
}

int32_t rcu_set_prefill_gemm(rcu_ctx *ctx, int32_t kind) {
    if (!ctx) return RCU_ERR_INVALID;
    if (kind != RCU_GEMM_F16 && kind != RCU_GEMM_I8) return set_err(ctx, RCU_ERR_INVALID, "unknown prefill GEMM kind");
    ctx->gemm_i8 = kind == RCU_GEMM_I8;
    return RCU_OK;
}

const char *rcu_last_error(const rcu_ctx *ctx) { return ctx ? ctx->last_error.c_str() : "null context"; }

int32_t rcu_check_device(rcu_ctx *ctx, uint32_t *bits_out) {
    if (!ctx) return RCU_ERR_INVALID;
    uint32_t bits = 0;
    RCU_CUDA_TRY(ctx, cudaMemcpyAsync(&bits, ctx->dev_err, sizeof(bits), cudaMemcpyDeviceToHost, ctx->stream));
    RCU_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    if (bits_out) *bits_out = bits;
    if (bits) {
        RCU_CUDA_TRY(ctx, cudaMemsetAsync(ctx->dev_err, 0, sizeof(uint32_t), ctx->stream));
        char m[96];
        std::snprintf(m, sizeof m, "bounded device wait expired (error bits 0x%x)", bits);
        return set_err(ctx, RCU_ERR_TIMEOUT, m);
    }
    return RCU_OK;
}

int32_t rcu_set_wait_limit_ms(rcu_ctx *ctx, uint64_t ms) {
    if (!ctx || ms == 0 || ms > 600000) return set_err(ctx, RCU_ERR_INVALID, "wait limit must be 1..600000 ms");
    ctx->wait_limit_ns = ms * 1000000ull;
    return RCU_OK;
}

int32_t rcu_sync(rcu_ctx *ctx) {
    if (!ctx) return RCU_ERR_INVALID;
    RCU_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    return rcu_check_device(ctx, nullptr);
}

uint64_t rcu_row_bytes(uint32_t ggml_type, uint64_t cols) { return row_bytes((int)ggml_type, cols); }

static int32_t check_weight_shape(rcu_ctx *ctx, uint32_t t, uint64_t rows, uint64_t cols) {
    const int bs = block_size((int)t);
    if (bs == 0) return set_err(ctx, RCU_ERR_UNSUPPORTED, "unknown ggml type " + std::to_string(t));
    if (rows == 0 || cols == 0 || cols % bs != 0)
        return set_err(ctx, RCU_ERR_INVALID, "weight shape: cols must be a positive multiple of the block size");
    if (rows > 0xffffffffull || row_bytes((int)t, cols) > 0x7fffffffull)
        return set_err(ctx, RCU_ERR_INVALID, "weight too large");
    return RCU_OK;
}

int32_t rcu_weight_upload(rcu_ctx *ctx, uint32_t ggml_type, uint64_t rows, uint64_t cols, const void *host_bytes,
                          rcu_weight **out) {
    if (!ctx || !out || !host_bytes) return set_err(ctx, RCU_ERR_INVALID, "null argument");
    *out = nullptr;
    RCU_GUARD_BEGIN
    int32_t st = check_weight_shape(ctx, ggml_type, rows, cols);
    if (st) return st;
    const uint64_t rb = row_bytes((int)ggml_type, cols), bytes = rb * rows;
    uint8_t *d = nullptr;
    RCU_CUDA_TRY(ctx, cudaMalloc(&d, bytes + 256));  // padding: bulk copies round sizes up to 16
    cudaError_t e = cudaMemcpyAsync(d, host_bytes, bytes, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(d + bytes, 0, 256, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) {
        cudaFree(d);
        return cuda_err(ctx, e, "weight upload");
    }
    rcu_weight *w = new rcu_weight();
    w->ctx = ctx;
    w->type = (int)ggml_type;
    w->rows = rows;
    w->cols = cols;
    w->row_bytes = rb;
    w->data = d;
    w->owned = true;
    w->padded = true;
    *out = w;
    return RCU_OK;
    RCU_GUARD_END(ctx)
}

int32_t rcu_weight_view(rcu_ctx *ctx, uint32_t ggml_type, uint64_t rows, uint64_t cols, const void *dev_bytes,
                        rcu_weight **out) {
    if (!ctx || !out || !dev_bytes) return set_err(ctx, RCU_ERR_INVALID, "null argument");
    *out = nullptr;
    RCU_GUARD_BEGIN
    int32_t st = check_weight_shape(ctx, ggml_type, rows, cols);
    if (st) return st;
    if (((uintptr_t)dev_bytes & 15) != 0) return set_err(ctx, RCU_ERR_INVALID, "weight view must be 16-byte aligned");
    rcu_weight *w = new rcu_weight();
    w->ctx = ctx;
    w->type = (int)ggml_type;
    w->rows = rows;
    w->cols = cols;
    w->row_bytes = row_bytes((int)ggml_type, cols);
    w->data = (uint8_t *)dev_bytes;
    w->owned = false;
    w->padded = true;  // documented precondition of the view
    *out = w;
    return RCU_OK;
    RCU_GUARD_END(ctx)
}

int32_t rcu_weight_slice_rows(const rcu_weight *w, uint64_t start, uint64_t n, rcu_weight **out) {
    if (!w || !out) return RCU_ERR_INVALID;
    *out = nullptr;
    if (n == 0 || start + n > w->rows) return set_err(w->ctx, RCU_ERR_INVALID, "slice_rows out of range");
    if (((start * w->row_bytes) & 15) != 0)
        return set_err(w->ctx, RCU_ERR_INVALID, "slice_rows: start row must begin on a 16-byte boundary");
    rcu_weight *s = new (std::nothrow) rcu_weight(*w);
    if (!s) return RCU_ERR_OOM;
    s->rows = n;
    s->data = w->data + start * w->row_bytes;
    s->owned = false;
    *out = s;
    return RCU_OK;
}

void rcu_weight_free(rcu_weight *w) {
    if (!w) return;
    if (w->owned && w->data) {
        cudaSetDevice(w->ctx->device);
        cudaFree(w->data);
    }
    delete w;
}

const void *rcu_weight_device_ptr(const rcu_weight *w) { return w ? w->data : nullptr; }

int32_t rcu_acts_create(rcu_ctx *ctx, uint64_t max_tok, uint64_t max_k, rcu_acts **out) {
    if (!ctx || !out) return set_err(ctx, RCU_ERR_INVALID, "null argument");
    *out = nullptr;
    if (max_tok == 0 || max_k == 0 || max_k % QK_K != 0 && max_k % QK != 0)
        return set_err(ctx, RCU_ERR_INVALID, "acts: max_k must be a multiple of 32");
    RCU_GUARD_BEGIN
    const uint64_t T = max_tok, K = max_k;
    auto al = [](uint64_t x) { return (x + 255) & ~255ull; };
    const uint64_t sz_q = al(T * K), sz_b0 = al(T * (K / QK) * 4), sz_bk = al(T * (K / QK_K + 1) * 4),
                   sz_bs = al(T * (K / 16) * 2);
    const uint64_t total = 2 * sz_q + 3 * sz_b0 + sz_bk + sz_bs;
    void *buf = nullptr;
    RCU_CUDA_TRY(ctx, cudaMalloc(&buf, total));
    rcu_acts *a = new rcu_acts();
    a->ctx = ctx;
    a->max_tok = T;
    a->max_k = K;
    a->buf = buf;
    uint8_t *p = (uint8_t *)buf;
    a->v.q0 = (int8_t *)p; p += sz_q;
    a->v.d0 = (float *)p; p += sz_b0;
    a->v.s0 = (float *)p; p += sz_b0;
    a->v.sum0 = (int32_t *)p; p += sz_b0;
    a->v.qk = (int8_t *)p; p += sz_q;
    a->v.dk = (float *)p; p += sz_bk;
    a->v.bsk = (int16_t *)p;
    *out = a;
    return RCU_OK;
    RCU_GUARD_END(ctx)
}

void rcu_acts_free(rcu_acts *a) {
    if (!a) return;
    cudaSetDevice(a->ctx->device);
    cudaFree(a->buf);
    delete a;
}

int32_t rcu_acts_prepare(rcu_ctx *ctx, rcu_acts *acts, const float *x_dev, uint64_t n_tok, uint64_t k,
                         uint32_t formats) {
    if (!ctx || !acts || !x_dev) return set_err(ctx, RCU_ERR_INVALID, "null argument");
    if (n_tok == 0) return set_err(ctx, RCU_ERR_RUNTIME, "empty batch");
    if (n_tok > acts->max_tok || k > acts->max_k) return set_err(ctx, RCU_ERR_INVALID, "acts: batch exceeds capacity");
    if ((formats & RCU_ACT_Q8_0) && k % QK != 0)
        return set_err(ctx, RCU_ERR_INVALID, "row length " + std::to_string(k) + " not a multiple of 32");
    if ((formats & RCU_ACT_Q8K) && k % QK_K != 0)
        return set_err(ctx, RCU_ERR_INVALID, "row length " + std::to_string(k) + " not a multiple of 256");
    if (formats & ~(uint32_t)(RCU_ACT_Q8_0 | RCU_ACT_Q8K)) return set_err(ctx, RCU_ERR_UNSUPPORTED, "unknown act format");
    acts->v.n_tok = (uint32_t)n_tok;
    acts->v.k = (uint32_t)k;
    acts->v.have = 0;
    int st = launch_quantize(ctx, acts->v, x_dev, (uint32_t)n_tok, (uint32_t)k, formats);
    if (st) return st;
    acts->v.have = formats;
    return RCU_OK;
}

int32_t rcu_acts_export(rcu_ctx *ctx, const rcu_acts *acts, uint32_t format, void *host_out) {
    if (!ctx || !acts || !host_out) return set_err(ctx, RCU_ERR_INVALID, "null argument");
    if (!(acts->v.have & format)) return set_err(ctx, RCU_ERR_INVALID, "format not prepared");
    RCU_GUARD_BEGIN
    const ActsView &v = acts->v;
    const uint64_t T = v.n_tok, K = v.k;
    std::vector<int8_t> q(T * K);
    if (format == RCU_ACT_Q8_0) {
        const uint64_t nb = T * (K / QK);
        std::vector<float> d(nb), s(nb);
        RCU_CUDA_TRY(ctx, cudaMemcpyAsync(q.data(), v.q0, T * K, cudaMemcpyDeviceToHost, ctx->stream));
        RCU_CUDA_TRY(ctx, cudaMemcpyAsync(d.data(), v.d0, nb * 4, cudaMemcpyDeviceToHost, ctx->stream));
        RCU_CUDA_TRY(ctx, cudaMemcpyAsync(s.data(), v.s0, nb * 4, cudaMemcpyDeviceToHost, ctx->stream));
        RCU_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
        uint8_t *o = (uint8_t *)host_out;
        for (uint64_t b = 0; b < nb; b++, o += 48) {  // BlockQ8_0: qs[32], d, s, 8 pad bytes
            std::memset(o, 0, 48);
            std::memcpy(o, q.data() + b * QK, QK);
            std::memcpy(o + 32, &d[b], 4);
            std::memcpy(o + 36, &s[b], 4);
        }
        return RCU_OK;
    }
    if (format == RCU_ACT_Q8K) {
        const uint64_t nb = T * (K / QK_K);
        std::vector<float> d(nb);
        std::vector<int16_t> bs(nb * 16);
        RCU_CUDA_TRY(ctx, cudaMemcpyAsync(q.data(), v.qk, T * K, cudaMemcpyDeviceToHost, ctx->stream));
        RCU_CUDA_TRY(ctx, cudaMemcpyAsync(d.data(), v.dk, nb * 4, cudaMemcpyDeviceToHost, ctx->stream));
        RCU_CUDA_TRY(ctx, cudaMemcpyAsync(bs.data(), v.bsk, nb * 32, cudaMemcpyDeviceToHost, ctx->stream));
        RCU_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
        uint8_t *o = (uint8_t *)host_out;
        for (uint64_t b = 0; b < nb; b++, o += 304) {  // BlockQ8K: qs[256], bsums[16], d, pad
            std::memset(o, 0, 304);
            std::memcpy(o, q.data() + b * QK_K, QK_K);
            std::memcpy(o + 256, bs.data() + b * 16, 32);
            std::memcpy(o + 288, &d[b], 4);
        }
        return RCU_OK;
    }
    return set_err(ctx, RCU_ERR_INVALID, "export one format at a time");
    RCU_GUARD_END(ctx)
}

int32_t rcu_matmul_multi(rcu_ctx *ctx, const rcu_acts *acts, const rcu_job *jobs, uint64_t n_jobs) {
    if (!ctx || !acts || (!jobs && n_jobs)) return set_err(ctx, RCU_ERR_INVALID, "null argument");
    if (n_jobs == 0) return RCU_OK;
    RCU_GUARD_BEGIN
    const ActsView &a = acts->v;
    if (a.n_tok == 0) return set_err(ctx, RCU_ERR_RUNTIME, "empty batch");
    std::vector<HostJob> hj;
    for (uint64_t i = 0; i < n_jobs; i++) {
        const rcu_weight *w = jobs[i].w;
        if (!w || !jobs[i].out) return set_err(ctx, RCU_ERR_INVALID, "job with null weight or output");
        if (w->cols != a.k) return set_err(ctx, RCU_ERR_INVALID, "matmul inner dimension mismatch");
        if (!gemv_supported(w->type))
            return set_err(ctx, RCU_ERR_UNSUPPORTED, "no GPU kernel for ggml type " + std::to_string(w->type));
        if (!(a.have & act_format(w->type)))
            return set_err(ctx, RCU_ERR_INVALID, "activations not prepared in the format this weight needs");
        if (jobs[i].ld < w->rows) return set_err(ctx, RCU_ERR_INVALID, "ld smaller than rows");
        hj.push_back({w, jobs[i].out, jobs[i].ld});
    }
    const uint32_t n_tok = a.n_tok;
    if (n_tok > 8) {
        const int st = launch_gemm(ctx, a, hj.data(), (int)hj.size());
        if (st != RCU_ERR_UNSUPPORTED) return st;
        ctx->last_error.clear();
    }
    for (size_t j0 = 0; j0 < hj.size(); j0 += kGemvMaxJobs) {
        const int nj = (int)std::min<size_t>(kGemvMaxJobs, hj.size() - j0);
        for (uint32_t t0 = 0; t0 < n_tok; t0 += 8) {
            const int st = launch_gemv(ctx, a, hj.data() + j0, nj, t0, std::min<uint32_t>(8, n_tok - t0));
            if (st) return st;
        }
    }
    return RCU_OK;
    RCU_GUARD_END(ctx)
}

int32_t rcu_matmul(rcu_ctx *ctx, const rcu_acts *acts, const rcu_weight *w, float *out) {
    if (!w) return set_err(ctx, RCU_ERR_INVALID, "null weight");
    rcu_job j{w, out, w->rows};
    return rcu_matmul_multi(ctx, acts, &j, 1);
}

int32_t rcu_matmul_block_sums(rcu_ctx *ctx, const rcu_acts *acts, const rcu_weight *w, float *out,
                              int32_t *sums_dev, int32_t kernel) {
    if (!ctx || !acts || !w || !out || !sums_dev) return set_err(ctx, RCU_ERR_INVALID, "null argument");
    if (kernel != 0 && kernel != 1) return set_err(ctx, RCU_ERR_INVALID, "kernel: 0 (lane GEMV) or 1 (tensor-core GEMV)");
    const int t = w->type;
    if (!gemv_supported(t)) return set_err(ctx, RCU_ERR_UNSUPPORTED, "type");
    if (kernel == 1 && t != T_Q4_K && t != T_Q5_K && t != T_Q6_K && t != T_Q4_0)
        return set_err(ctx, RCU_ERR_UNSUPPORTED, "the tensor-core GEMV takes Q4_K, Q5_K, Q6_K and Q4_0 weights");
    if (w->cols != acts->v.k || !(acts->v.have & act_format(t)))
        return set_err(ctx, RCU_ERR_INVALID, "activations do not match the weight");
    RCU_GUARD_BEGIN
    const uint64_t k = w->cols;
    const uint32_t nbs = (uint32_t)(block_size(t) == QK ? k / QK : (t == T_Q6_K ? k / QK_K : 2 * (k / QK_K)));
    RCU_CUDA_TRY(ctx, cudaMemsetAsync(sums_dev, 0, w->rows * nbs * sizeof(int32_t), ctx->stream));
    ctx->dbg_sums = sums_dev;
    ctx->dbg_nbs = nbs;
    ctx->dbg_kernel = kernel;
    const HostJob hj{w, out, w->rows};
    const int st = launch_gemv(ctx, acts->v, &hj, 1, 0, 1);
    ctx->dbg_sums = nullptr;
    ctx->dbg_nbs = 0;
    ctx->dbg_kernel = -1;
    return st;
    RCU_GUARD_END(ctx)
}

int32_t rcu_block_sums(rcu_ctx *ctx, const rcu_acts *acts, const rcu_weight *w, uint64_t row, uint64_t tok,
                       int32_t *out_dev) {
    if (!ctx || !acts || !w || !out_dev) return set_err(ctx, RCU_ERR_INVALID, "null argument");
    if (row >= w->rows || tok >= acts->v.n_tok) return set_err(ctx, RCU_ERR_INVALID, "row/token out of range");
    if (!gemv_supported(w->type)) return set_err(ctx, RCU_ERR_UNSUPPORTED, "type");
    if (w->cols != acts->v.k || !(acts->v.have & act_format(w->type)))
        return set_err(ctx, RCU_ERR_INVALID, "activations do not match the weight");
    return launch_block_sums(ctx, acts->v, w, row, tok, out_dev);
}

}  // extern "C"
