// rie_oracle_model.cpp -- TEST INFRASTRUCTURE ONLY: the reference's CPU transformer forward
// restated on top of the oracle kernels (rie_oracle.cpp), as the parity checker and the
// tok/s CPU baseline of the device forward scheduler.
//
//   tensor names / model assembly   crates/rie-core/src/model/mod.rs:112-247
//   forward_impl                    crates/rie-core/src/model/cpu.rs:210-409
//   dense_ffn                       crates/rie-core/src/model/cpu.rs:431-467
//   moe_ffn                         crates/rie-core/src/model/cpu.rs:469-524
//   rmsnorm / rmsnorm_inplace       crates/rie-core/src/ops.rs:6-24
//   Rope                            crates/rie-core/src/ops.rs:51-109
#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <memory>
#include <numeric>
#include <string>
#include <vector>

#include "rie_oracle.h"

extern "C" {
typedef struct orc_model_config {
    uint32_t n_vocab, n_embd, n_layer, n_head, n_head_kv, head_dim, n_ff;
    uint32_t rope_dim;
    int32_t rope_neox;
    float rope_base, rope_freq_scale;
    float rms_eps, attn_scale, embd_scale, residual_scale, logit_scale;
    float attn_softcap, final_softcap;  // <= 0: none
    uint32_t swa_window, swa_pattern;
    float rope_base_swa;                // <= 0: none
    int32_t act;                        // 0 silu, 1 gelu_tanh
    uint32_t n_expert, n_expert_used, n_ff_exp;
    int32_t expert_norm_topk, expert_unit_weights;
} orc_model_config;
}

namespace {

struct Tensor {
    int type = 0;
    uint64_t rows = 0, cols = 0;
    std::vector<uint8_t> data;
    const uint8_t *row(uint64_t r) const { return data.data() + r * orc_row_bytes(type, cols); }
};

struct Model {
    orc_model_config cfg{};
    std::map<std::string, Tensor> t;
    const Tensor *get(const std::string &n) const {
        auto it = t.find(n);
        return it == t.end() ? nullptr : &it->second;
    }
    std::vector<float> vec(const std::string &n) const {
        const Tensor *x = get(n);
        if (!x) return {};
        std::vector<float> v(x->rows * x->cols);
        orc_dequantize_row(x->type, x->data.data(), v.data(), v.size());
        return v;
    }
};

struct Backend {
    Model *m;
    size_t n_ctx, max_batch;
    int kv_type, n_threads, path;
    std::vector<std::vector<uint8_t>> kc, vc;
    std::vector<size_t> slots;
    std::vector<float> hidden;
    // when capture is set: the residual stream at the entry of layer 0 and after every layer
    // ([n_layer + 1][n][n_embd] of the latest forward), for layer-by-layer parity checks
    bool capture = false;
    std::vector<float> layer_x;
    // teacher forcing: when set ([n_layer + 1][n][n_embd]), the residual stream is replaced by
    // these rows at the entry of every layer and before the head
    std::vector<float> teacher;
    std::string err;
};

bool is_swa(const orc_model_config &c, size_t il) {  // model/config.rs:110-112
    return c.swa_window > 0 && c.swa_pattern > 0 && (il % c.swa_pattern) < c.swa_pattern - 1;
}

void rmsnorm_inplace(float *x, const float *w, size_t n, float eps, int path) {  // ops.rs:17-24
    const float ss = orc_dot_f32(x, x, n, path) / (float)n;
    const float scale = 1.0f / std::sqrt(ss + eps);
    for (size_t i = 0; i < n; i++) x[i] *= scale * w[i];
}

float gelu_tanh(float x) {  // ops.rs:32-35
    const float k = 0.7978846f;
    return 0.5f * x * (1.0f + std::tanh(k * x * (1.0f + 0.044715f * x * x)));
}

void matmul(Backend &b, const float *x, size_t n, size_t k, std::vector<std::pair<const Tensor *, float *>> jobs,
            std::vector<size_t> lds = {}) {
    std::vector<orc_job> js;
    for (size_t i = 0; i < jobs.size(); i++) {
        const Tensor *w = jobs[i].first;
        orc_job j{};
        j.ggml_type = w->type;
        j.rows = w->rows;
        j.cols = w->cols;
        j.w = w->data.data();
        j.out = jobs[i].second;
        j.ld = lds.empty() ? w->rows : lds[i];
        js.push_back(j);
    }
    orc_matmul_multi(b.n_threads, x, n, k, js.data(), js.size(), b.path);
}

// Tensor row view for fused / stacked weights (Weight::slice_rows, tensor.rs:64-69).
Tensor slice(const Tensor &w, uint64_t start, uint64_t n) {
    Tensor s;
    s.type = w.type;
    s.rows = n;
    s.cols = w.cols;
    const size_t rb = orc_row_bytes(w.type, w.cols);
    s.data.assign(w.data.begin() + start * rb, w.data.begin() + (start + n) * rb);
    return s;
}

void dense_ffn(Backend &b, const Tensor &gate, const Tensor &up, const Tensor &down, const float *x, size_t n,
               float *out) {  // model/cpu.rs:433-467
    const size_t e = gate.cols, ff = gate.rows;
    std::vector<float> g(n * ff), u(n * ff);
    matmul(b, x, n, e, {{&gate, g.data()}, {&up, u.data()}});
    for (size_t i = 0; i < n * ff; i++) {
        const float a = g[i];
        g[i] = (b.m->cfg.act == 1 ? gelu_tanh(a) : orc_silu(a)) * u[i];
    }
    matmul(b, g.data(), n, ff, {{&down, out}}, {e});
}

int forward(Backend &b, const uint32_t *tokens, size_t n, size_t pos0, bool all_logits, float *logits) {
    const Model &m = *b.m;
    const orc_model_config &c = m.cfg;
    if (n == 0) return b.err = "empty batch", 6;
    if (n > b.max_batch) return b.err = "batch exceeds max batch", 6;
    if (pos0 + n > b.n_ctx) return b.err = "context window full", 6;
    const size_t e = c.n_embd, hd = c.head_dim, qd = c.n_head * hd, kvd = c.n_head_kv * hd, half = c.rope_dim / 2;
    const Tensor *embd = m.get("token_embd.weight");
    std::vector<float> x(n * e), xn(n * e);
    for (size_t t = 0; t < n; t++) {
        if (tokens[t] >= embd->rows) return b.err = "token id out of range", 6;
        orc_dequantize_row(embd->type, embd->row(tokens[t]), x.data() + t * e, e);
        if (c.embd_scale != 1.0f)
            for (size_t i = 0; i < e; i++) x[t * e + i] *= c.embd_scale;
    }
    std::vector<float> cosg(n * half), sing(n * half), coss(n * half), sins(n * half);
    for (size_t t = 0; t < n; t++) {
        orc_rope_table(c.rope_dim, c.rope_base, c.rope_freq_scale, pos0 + t, cosg.data() + t * half, sing.data() + t * half);
        if (c.rope_base_swa > 0.0f)
            orc_rope_table(c.rope_dim, c.rope_base_swa, 1.0f, pos0 + t, coss.data() + t * half, sins.data() + t * half);
    }
    std::vector<float> q(n * qd), k(n * kvd), v(n * kvd), att(n * qd), o(n * e);
    if (b.capture) b.layer_x.clear();
    const bool teach = b.teacher.size() == (c.n_layer + 1) * n * e;
    for (size_t il = 0; il < c.n_layer; il++) {
        if (teach) std::copy(b.teacher.begin() + il * n * e, b.teacher.begin() + (il + 1) * n * e, x.begin());
        if (b.capture && il == 0) b.layer_x.insert(b.layer_x.end(), x.begin(), x.end());
        const std::string p = "blk." + std::to_string(il) + ".";
        const bool swa = is_swa(c, il);
        const std::vector<float> attn_norm = m.vec(p + "attn_norm.weight");
        for (size_t t = 0; t < n; t++) orc_rmsnorm(xn.data() + t * e, x.data() + t * e, attn_norm.data(), e, c.rms_eps, b.path);
        Tensor wq, wk, wv;
        const Tensor *pq, *pk, *pv;
        if (const Tensor *qkv = m.get(p + "attn_qkv.weight")) {
            wq = slice(*qkv, 0, qd);
            wk = slice(*qkv, qd, kvd);
            wv = slice(*qkv, qd + kvd, kvd);
            pq = &wq, pk = &wk, pv = &wv;
        } else {
            pq = m.get(p + "attn_q.weight"), pk = m.get(p + "attn_k.weight"), pv = m.get(p + "attn_v.weight");
        }
        matmul(b, xn.data(), n, e, {{pq, q.data()}, {pk, k.data()}, {pv, v.data()}});
        const std::vector<float> bq = m.vec(p + "attn_q.bias"), bk = m.vec(p + "attn_k.bias"), bv = m.vec(p + "attn_v.bias");
        for (size_t t = 0; t < n; t++) {
            for (size_t i = 0; i < bq.size(); i++) q[t * qd + i] += bq[i];
            for (size_t i = 0; i < bk.size(); i++) k[t * kvd + i] += bk[i];
            for (size_t i = 0; i < bv.size(); i++) v[t * kvd + i] += bv[i];
        }
        const std::vector<float> qn = m.vec(p + "attn_q_norm.weight"), kn = m.vec(p + "attn_k_norm.weight");
        const bool use_swa_rope = swa && c.rope_base_swa > 0.0f;
        for (size_t t = 0; t < n; t++) {
            const float *ct = (use_swa_rope ? coss.data() : cosg.data()) + t * half;
            const float *st = (use_swa_rope ? sins.data() : sing.data()) + t * half;
            for (size_t h = 0; h < c.n_head; h++) {
                float *qh = q.data() + t * qd + h * hd;
                if (!qn.empty()) rmsnorm_inplace(qh, qn.data(), hd, c.rms_eps, b.path);
                orc_rope_apply(qh, c.rope_dim, c.rope_neox, ct, st);
                for (size_t i = 0; i < hd; i++) qh[i] *= c.attn_scale;
            }
            for (size_t h = 0; h < c.n_head_kv; h++) {
                float *kh = k.data() + t * kvd + h * hd;
                if (!kn.empty()) rmsnorm_inplace(kh, kn.data(), hd, c.rms_eps, b.path);
                orc_rope_apply(kh, c.rope_dim, c.rope_neox, ct, st);
            }
        }
        const size_t slots = b.slots[il];
        const size_t rb = b.kv_type == ORC_KV_F16 ? 2 * hd : b.kv_type == ORC_KV_Q8_0 ? hd / 32 * 34 : orc_turbo_row_bytes_4(hd);
        for (size_t t = 0; t < n; t++) {
            const size_t slot = (pos0 + t) % slots;
            for (size_t h = 0; h < c.n_head_kv; h++) {
                const size_t row = h * slots + slot;
                orc_kv_store(b.kv_type, k.data() + t * kvd + h * hd, hd, b.kc[il].data() + row * rb, b.path);
                orc_kv_store(b.kv_type, v.data() + t * kvd + h * hd, hd, b.vc[il].data() + row * rb, b.path);
            }
        }
        orc_attention(b.n_threads, c.n_head, c.n_head_kv, hd, n, pos0, swa ? c.swa_window : 0,
                      c.attn_softcap, q.data(), b.kv_type, b.kc[il].data(), b.vc[il].data(), slots, att.data(), b.path);
        matmul(b, att.data(), n, qd, {{m.get(p + "attn_output.weight"), o.data()}});
        const std::vector<float> pan = m.vec(p + "post_attention_norm.weight");
        if (!pan.empty())
            for (size_t t = 0; t < n; t++) rmsnorm_inplace(o.data() + t * e, pan.data(), e, c.rms_eps, b.path);
        for (size_t i = 0; i < n * e; i++) x[i] += c.residual_scale == 1.0f ? o[i] : o[i] * c.residual_scale;
        const std::vector<float> fn = m.vec(p + "ffn_norm.weight");
        for (size_t t = 0; t < n; t++) orc_rmsnorm(xn.data() + t * e, x.data() + t * e, fn.data(), e, c.rms_eps, b.path);
        if (const Tensor *router = m.get(p + "ffn_gate_inp.weight")) {  // moe_ffn (cpu.rs:473-524)
            const size_t ne = router->rows, ff = c.n_ff_exp;
            std::vector<float> lg(n * ne);
            matmul(b, xn.data(), n, e, {{router, lg.data()}});
            std::vector<std::vector<std::pair<size_t, float>>> assign(ne);
            std::vector<size_t> idx(ne);
            for (size_t t = 0; t < n; t++) {
                float *l = lg.data() + t * ne;
                float mx = -INFINITY;
                for (size_t i = 0; i < ne; i++) mx = std::fmax(mx, l[i]);
                float sum = 0.0f;
                for (size_t i = 0; i < ne; i++) {
                    l[i] = std::exp(l[i] - mx);
                    sum += l[i];
                }
                const float inv = 1.0f / sum;
                for (size_t i = 0; i < ne; i++) l[i] *= inv;
                std::iota(idx.begin(), idx.end(), 0);
                std::sort(idx.begin(), idx.end(), [&](size_t a, size_t bb) { return l[a] > l[bb] || (l[a] == l[bb] && a < bb); });
                const size_t used = std::min<size_t>(std::max<size_t>(c.n_expert_used, 1), ne);
                float norm = 1.0f;
                if (c.expert_norm_topk) {
                    norm = 0.0f;
                    for (size_t j = 0; j < used; j++) norm += l[idx[j]];
                }
                for (size_t j = 0; j < used; j++)
                    assign[idx[j]].push_back({t, c.expert_unit_weights ? 1.0f : l[idx[j]] / norm});
            }
            std::fill(o.begin(), o.end(), 0.0f);
            const Tensor *ga = m.get(p + "ffn_gate_exps.weight"), *ua = m.get(p + "ffn_up_exps.weight"),
                         *da = m.get(p + "ffn_down_exps.weight");
            for (size_t ex = 0; ex < ne; ex++) {
                if (assign[ex].empty()) continue;
                const size_t kk = assign[ex].size();
                std::vector<float> xg(kk * e), yg(kk * e);
                for (size_t j = 0; j < kk; j++) std::copy(xn.begin() + assign[ex][j].first * e, xn.begin() + (assign[ex][j].first + 1) * e, xg.begin() + j * e);
                const Tensor g = slice(*ga, ex * ff, ff), u = slice(*ua, ex * ff, ff), d = slice(*da, ex * e, e);
                dense_ffn(b, g, u, d, xg.data(), kk, yg.data());
                for (size_t j = 0; j < kk; j++)
                    for (size_t i = 0; i < e; i++) o[assign[ex][j].first * e + i] += assign[ex][j].second * yg[j * e + i];
            }
            if (const Tensor *sg = m.get(p + "ffn_gate_shexp.weight")) {
                std::vector<float> ys(n * e);
                dense_ffn(b, *sg, *m.get(p + "ffn_up_shexp.weight"), *m.get(p + "ffn_down_shexp.weight"), xn.data(), n, ys.data());
                const std::vector<float> gate = m.vec(p + "ffn_gate_inp_shexp.weight");
                for (size_t t = 0; t < n; t++) {
                    const float scale = gate.empty() ? 1.0f : 1.0f / (1.0f + std::exp(-orc_dot_f32(gate.data(), xn.data() + t * e, e, b.path)));
                    for (size_t i = 0; i < e; i++) o[t * e + i] += scale * ys[t * e + i];
                }
            }
        } else {
            const Tensor *gate = m.get(p + "ffn_gate.weight"), *up = m.get(p + "ffn_up.weight");
            Tensor gs, us;
            if (!gate) {
                gs = slice(*up, 0, c.n_ff);
                us = slice(*up, c.n_ff, c.n_ff);
                gate = &gs, up = &us;
            }
            dense_ffn(b, *gate, *up, *m.get(p + "ffn_down.weight"), xn.data(), n, o.data());
        }
        const std::vector<float> pfn = m.vec(p + "post_ffw_norm.weight");
        if (!pfn.empty())
            for (size_t t = 0; t < n; t++) rmsnorm_inplace(o.data() + t * e, pfn.data(), e, c.rms_eps, b.path);
        for (size_t i = 0; i < n * e; i++) x[i] += c.residual_scale == 1.0f ? o[i] : o[i] * c.residual_scale;
        if (b.capture) b.layer_x.insert(b.layer_x.end(), x.begin(), x.end());
    }
    if (teach) std::copy(b.teacher.begin() + c.n_layer * n * e, b.teacher.end(), x.begin());
    const size_t first = all_logits ? 0 : n - 1, mrows = n - first, nv = c.n_vocab;
    const std::vector<float> on = m.vec("output_norm.weight");
    for (size_t t = 0; t < mrows; t++) orc_rmsnorm(xn.data() + t * e, x.data() + (first + t) * e, on.data(), e, c.rms_eps, b.path);
    b.hidden.assign(xn.begin(), xn.begin() + mrows * e);
    const Tensor *out = m.get("output.weight");
    if (!out) out = embd;
    Tensor outv;
    if (out->rows > nv) {
        outv = slice(*out, 0, nv);
        out = &outv;
    }
    matmul(b, xn.data(), mrows, e, {{out, logits}});
    for (size_t i = 0; i < mrows * nv; i++) {
        if (c.logit_scale != 1.0f) logits[i] /= c.logit_scale;
        if (c.final_softcap > 0.0f) logits[i] = c.final_softcap * std::tanh(logits[i] / c.final_softcap);
    }
    return 0;
}

}  // namespace

extern "C" {

void *orc_model_create(const orc_model_config *cfg) {
    Model *m = new Model();
    m->cfg = *cfg;
    return m;
}
void orc_model_free(void *m) { delete (Model *)m; }
int orc_model_set_tensor(void *mp, const char *name, int type, uint64_t rows, uint64_t cols, const void *data) {
    Model *m = (Model *)mp;
    Tensor t;
    t.type = type;
    t.rows = rows;
    t.cols = cols;
    const size_t bytes = rows * orc_row_bytes(type, cols);
    t.data.assign((const uint8_t *)data, (const uint8_t *)data + bytes);
    m->t[name] = std::move(t);
    return 0;
}
void *orc_backend_create(void *mp, uint64_t n_ctx, uint64_t max_batch, int kv_type, int n_threads, int path) {
    Model *m = (Model *)mp;
    const orc_model_config &c = m->cfg;
    Backend *b = new Backend();
    b->m = m;
    b->n_ctx = n_ctx;
    b->max_batch = std::max<uint64_t>(1, std::min<uint64_t>(max_batch, n_ctx));
    b->kv_type = kv_type;
    b->n_threads = n_threads;
    b->path = path;
    const size_t hd = c.head_dim;
    const size_t rb = kv_type == ORC_KV_F16 ? 2 * hd : kv_type == ORC_KV_Q8_0 ? hd / 32 * 34 : orc_turbo_row_bytes_4(hd);
    for (size_t il = 0; il < c.n_layer; il++) {
        const size_t slots = is_swa(c, il) ? std::min<size_t>(c.swa_window + b->max_batch, n_ctx) : n_ctx;
        b->slots.push_back(slots);
        b->kc.emplace_back(c.n_head_kv * slots * rb + 16, 0);
        b->vc.emplace_back(c.n_head_kv * slots * rb + 16, 0);
    }
    return b;
}
void orc_backend_free(void *b) { delete (Backend *)b; }
int orc_backend_forward(void *bp, const uint32_t *tokens, uint64_t n, uint64_t pos, int all_logits, float *logits) {
    return forward(*(Backend *)bp, tokens, n, pos, all_logits != 0, logits);
}
const char *orc_backend_error(void *bp) { return ((Backend *)bp)->err.c_str(); }
void orc_backend_set_capture(void *bp, int on) { ((Backend *)bp)->capture = on != 0; }
// Teacher rows for the next forwards ([n_layer + 1][n][n_embd]); count 0 turns it off.
void orc_backend_set_teacher(void *bp, const float *x, uint64_t count) {
    Backend *b = (Backend *)bp;
    if (!x || count == 0) b->teacher.clear();
    else b->teacher.assign(x, x + count);
}
// Residual rows captured by the latest forward: [n_layer + 1][n][n_embd]; returns the count.
int64_t orc_backend_layer_x(void *bp, float *out, uint64_t cap) {
    Backend *b = (Backend *)bp;
    if (!out) return (int64_t)b->layer_x.size();
    if (cap < b->layer_x.size()) return -1;
    std::copy(b->layer_x.begin(), b->layer_x.end(), out);
    return (int64_t)b->layer_x.size();
}
int orc_backend_hidden(void *bp, float *out, uint64_t cap) {
    Backend *b = (Backend *)bp;
    if (cap < b->hidden.size()) return -1;
    std::copy(b->hidden.begin(), b->hidden.end(), out);
    return (int)b->hidden.size();
}

}  // extern "C"
