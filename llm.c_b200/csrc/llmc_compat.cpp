// llmc_compat.cpp — llm.c's own entry points over the C-ABI:
//   moe_forward     (src/transformer.c:287-366)  block / prefill MoE
//   inference_step  (src/inference.c:231-358)    single-token decode step,
//                                                 with the MoE branch filled in
//   moe_b200_llmc_block_ffn (src/transformer.c:752-767)  block_forward's
//                                                 RMSNorm + FFN + residual
//   moe_backward    the MoE counterpart of ffn_backward (src/transformer.c:
//                   181-264), which llm.c's model_backward lacks
//
// Residency cache: one device expert set per MoEWeights pointer (and, for
// dense blocks run through moe_b200_llmc_block_ffn, one single-expert set
// per FFNWeights pointer), uploaded on first sight from the host matrices
// (include/transformer.h:53-58) and kept until moe_b200_invalidate or
// shutdown.
#include "../../include/llmc_moe.h"
#include "../../include/moe_b200.h"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <unordered_map>
#include <vector>

namespace {
// a resident expert set and the host matrices it was uploaded from
struct Resident {
    moe_b200_weights *w = nullptr;
    std::vector<const float *> src;      // W_router, then gate, up, down of each expert
};
std::mutex g_cache_mu;
std::unordered_map<const void *, Resident> g_cache;
std::unordered_map<const void *, Resident> g_dense;   // keyed by FFNWeights pointer
std::unordered_map<const void *, moe_b200_grads *> g_grads;   // moe_backward's, per MoEWeights

std::vector<const float *> host_sources(const llmc_MoEWeights *mw) {
    std::vector<const float *> v;
    v.reserve(1 + 3 * (size_t)mw->n_experts);
    v.push_back(mw->W_router.data);
    for (int e = 0; e < mw->n_experts; e++) {
        v.push_back(mw->experts[e].W_gate.data);
        v.push_back(mw->experts[e].W_up.data);
        v.push_back(mw->experts[e].W_down.data);
    }
    return v;
}

int env_path() {
    const char *p = std::getenv("MOE_B200_PATH");
    if (!p || !*p || !std::strcmp(p, "auto")) return MOE_B200_PATH_AUTO;
    if (!std::strcmp(p, "tf32")) return MOE_B200_PATH_TF32;
    if (!std::strcmp(p, "fp32")) return MOE_B200_PATH_FP32;
    if (!std::strcmp(p, "tf32x3")) return MOE_B200_PATH_TF32X3;
    return MOE_B200_PATH_AUTO;
}

[[noreturn]] void die(const char *where, const char *what, int rc) {
    std::fprintf(stderr, "[moe_b200] %s: %s: %s (%s)\n", where, what, moe_b200_strerror(rc),
                 moe_b200_last_error());
    std::abort();
}

// Device expert set of `mw`, uploaded on first sight.  An entry whose host
// matrices moved (a different model reusing the MoEWeights address) is
// uploaded again; same-address reuse needs moe_b200_invalidate.
moe_b200_weights *resident(const llmc_MoEWeights *mw, int d, int F, const char *where) {
    std::lock_guard<std::mutex> lk(g_cache_mu);
    auto it = g_cache.find(mw);
    if (it != g_cache.end()) {
        if (it->second.src == host_sources(mw)) return it->second.w;
        moe_b200_weights_free(it->second.w);
        g_cache.erase(it);
    }
    const int E = mw->n_experts, k = mw->top_k;
    if (mw->W_router.rows != d || mw->W_router.cols != E)
        die(where, "router shape mismatch", MOE_B200_E_INVALID);
    std::vector<const float *> g(E), u(E), dn(E);
    for (int e = 0; e < E; e++) {
        const llmc_FFNWeights &fw = mw->experts[e];
        if (fw.W_gate.rows != d || fw.W_gate.cols != F || fw.W_up.rows != d ||
            fw.W_up.cols != F || fw.W_down.rows != F || fw.W_down.cols != d)
            die(where, "expert shape mismatch", MOE_B200_E_INVALID);
        g[e] = fw.W_gate.data;
        u[e] = fw.W_up.data;
        dn[e] = fw.W_down.data;
    }
    moe_b200_weights *w = nullptr;
    int rc = moe_b200_weights_upload(mw->W_router.data, g.data(), u.data(), dn.data(), d, F, E,
                                     k, &w);
    if (rc) die(where, "weight upload", rc);
    g_cache[mw] = Resident{w, host_sources(mw)};
    return w;
}

// A dense FFN (FFNWeights) as a one-expert set with a zero router: softmax
// over one logit is 1, so the combine returns the expert's output exactly.
moe_b200_weights *resident_dense(const llmc_FFNWeights *fw, int d, int F, const char *where) {
    std::lock_guard<std::mutex> lk(g_cache_mu);
    const std::vector<const float *> src{fw->W_gate.data, fw->W_up.data, fw->W_down.data};
    auto it = g_dense.find(fw);
    if (it != g_dense.end()) {
        if (it->second.src == src) return it->second.w;
        moe_b200_weights_free(it->second.w);
        g_dense.erase(it);
    }
    if (fw->W_gate.rows != d || fw->W_gate.cols != F || fw->W_up.rows != d ||
        fw->W_up.cols != F || fw->W_down.rows != F || fw->W_down.cols != d)
        die(where, "dense FFN shape mismatch", MOE_B200_E_INVALID);
    const std::vector<float> zero_router((size_t)d, 0.0f);
    const float *g = fw->W_gate.data, *u = fw->W_up.data, *dn = fw->W_down.data;
    moe_b200_weights *w = nullptr;
    const int rc = moe_b200_weights_upload(zero_router.data(), &g, &u, &dn, d, F, 1, 1, &w);
    if (rc) die(where, "weight upload", rc);
    g_dense[fw] = Resident{w, src};
    return w;
}

// The forward shared by both entry points: host buffers in, host buffers out.
void run_moe(const llmc_MoEWeights *mw, int F, const float *x, int T, int d, float *out,
             float *probs, int *ids, const char *where) {
    moe_b200_weights *w = resident(mw, d, F, where);
    moe_b200_opts opts;
    std::memset(&opts, 0, sizeof opts);
    opts.path = env_path();
    const int rc = moe_b200_forward(w, nullptr, x, T, out, probs, ids, &opts);
    if (rc) die(where, "forward", rc);
}
}  // namespace

// block_forward's FFN half (src/transformer.c:752-767): x_norm =
// rms_norm(x, rms_ffn); FFN or MoE of x_norm; x += result — one device call.
extern "C" void moe_b200_llmc_block_ffn(llmc_Matrix *x, const llmc_BlockWeights *bw,
                                        llmc_ForwardCache *cache, const llmc_ModelConfig *cfg) {
    const char *where = "moe_b200_llmc_block_ffn";
    const int T = x->rows, d = x->cols;
    if (d != cfg->d_model) die(where, "x width is not d_model", MOE_B200_E_INVALID);
    moe_b200_opts opts;
    std::memset(&opts, 0, sizeof opts);
    opts.path = env_path();
    int rc;
    if (bw->use_moe) {
        moe_b200_weights *w = resident(&bw->moe, d, cfg->ffn_hidden, where);
        rc = moe_b200_block_ffn(w, bw->rms_ffn, cfg->rms_norm_eps, nullptr, x->data, T, nullptr,
                                cache ? cache->router_probs : nullptr,
                                cache ? cache->expert_ids : nullptr, &opts);
    } else {
        moe_b200_weights *w = resident_dense(&bw->ffn, d, cfg->ffn_hidden, where);
        rc = moe_b200_block_ffn(w, bw->rms_ffn, cfg->rms_norm_eps, nullptr, x->data, T, nullptr,
                                nullptr, nullptr, &opts);
    }
    if (rc) die(where, "block FFN", rc);
}

float env_aux_coef() {
    const char *p = std::getenv("MOE_B200_AUX_COEF");
    return p && *p ? std::strtof(p, nullptr) : 0.0f;
}

// The MoE block's backward with ffn_backward's conventions: the weight
// gradients are added into the host .grad matrices (those that exist),
// d_x is overwritten.  The device gradient buffers of each MoEWeights are
// kept between calls (zeroed per call).
extern "C" void moe_backward(const llmc_Matrix *x, const llmc_MoEWeights *mw,
                             const llmc_ModelConfig *cfg, const llmc_ForwardCache *cache,
                             const llmc_Matrix *d_out, llmc_Matrix *d_x) {
    (void)cache;
    const char *where = "moe_backward";
    const int T = x->rows, d = x->cols, E = mw->n_experts, F = cfg->ffn_hidden;
    if (d_out->rows != T || d_out->cols != d || d_x->rows != T || d_x->cols != d)
        die(where, "shape mismatch", MOE_B200_E_INVALID);
    moe_b200_weights *w = resident(mw, d, F, where);
    moe_b200_grads *g = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_cache_mu);
        auto it = g_grads.find(mw);
        if (it != g_grads.end()) {
            g = it->second;
        } else {
            const int rc = moe_b200_grads_create(w, &g);
            if (rc) die(where, "gradient buffers", rc);
            g_grads[mw] = g;
        }
    }
    int rc = moe_b200_grads_zero(g);
    if (rc) die(where, "gradient buffers", rc);
    moe_b200_opts opts;
    std::memset(&opts, 0, sizeof opts);
    opts.path = env_path();
    rc = moe_b200_backward(w, nullptr, x->data, T, d_out->data, env_aux_coef(), d_x->data, g,
                           nullptr, &opts);
    if (rc) die(where, "backward", rc);
    const size_t dF = (size_t)d * F;
    std::vector<float> wr((size_t)d * E), buf(3 * dF * (size_t)E);
    std::vector<float *> gp(E), up(E), dp(E);
    for (int e = 0; e < E; e++) {
        gp[e] = buf.data() + (3 * (size_t)e + 0) * dF;
        up[e] = buf.data() + (3 * (size_t)e + 1) * dF;
        dp[e] = buf.data() + (3 * (size_t)e + 2) * dF;
    }
    rc = moe_b200_grads_download(g, wr.data(), nullptr, gp.data(), up.data(), dp.data());
    if (rc) die(where, "gradient download", rc);
    auto add = [](float *dst, const float *src, size_t n) {
        if (dst)
            for (size_t i = 0; i < n; i++) dst[i] += src[i];
    };
    add(mw->W_router.grad, wr.data(), wr.size());
    for (int e = 0; e < E; e++) {
        add(mw->experts[e].W_gate.grad, gp[e], dF);
        add(mw->experts[e].W_up.grad, up[e], dF);
        add(mw->experts[e].W_down.grad, dp[e], dF);
    }
}

extern "C" void moe_forward(const llmc_Matrix *x, const llmc_MoEWeights *mw,
                            const llmc_ModelConfig *cfg, llmc_ForwardCache *cache,
                            llmc_Matrix *out) {
    const int T = x->rows, d = x->cols;
    if (out->rows != T || out->cols != d) die("moe_forward", "shape mismatch", MOE_B200_E_INVALID);
    run_moe(mw, cfg->ffn_hidden, x->data, T, d, out->data, cache ? cache->router_probs : nullptr,
            cache ? cache->expert_ids : nullptr, "moe_forward");
}

// device decoders of inference_step's device mode, one per Model
std::mutex g_dec_mu;
std::unordered_map<const void *, moe_b200_decoder *> g_decoders;

extern "C" int moe_b200_invalidate(const void *ptr) {
    int rc = MOE_B200_OK;
    {
        std::lock_guard<std::mutex> lk(g_cache_mu);
        for (auto *map : {&g_cache, &g_dense}) {
            auto it = map->find(ptr);
            if (it != map->end()) {
                const int r = moe_b200_weights_free(it->second.w);
                if (!rc) rc = r;
                map->erase(it);
            }
        }
        auto gi = g_grads.find(ptr);
        if (gi != g_grads.end()) {
            moe_b200_grads_free(gi->second);
            g_grads.erase(gi);
        }
    }
    std::lock_guard<std::mutex> lk(g_dec_mu);
    auto it = g_decoders.find(ptr);
    if (it != g_decoders.end()) {
        const int r2 = moe_b200_decoder_destroy(it->second);
        g_decoders.erase(it);
        if (!rc) rc = r2;
    }
    return rc;
}

// ---------------------------------------------------------------------------
// inference_step: CPU restatement of the reference's single-token forward
// (src/inference.c:161-228 helpers, 231-358 body) with the MoE branch added.
// ---------------------------------------------------------------------------
namespace {

// out[N] = vec[M]ᵀ · mat[M×N], rows with vec[i] == 0 skipped
// (matvec, src/inference.c:174-182)
void matvec(const float *mat, const float *vec, float *out, int M, int N) {
    std::memset(out, 0, (size_t)N * sizeof(float));
    for (int i = 0; i < M; i++) {
        const float vi = vec[i];
        if (vi == 0.0f) continue;
        const float *row = mat + (size_t)i * N;
        for (int j = 0; j < N; j++) out[j] += vi * row[j];
    }
}

// RMSNorm of one vector (rmsnorm_vec, src/inference.c:209-215)
void rmsnorm_vec(const float *x, const float *w, float eps, float *out, int d) {
    float ss = 0.0f;
    for (int i = 0; i < d; i++) ss += x[i] * x[i];
    const float inv = 1.0f / std::sqrt(ss / (float)d + eps);
    for (int i = 0; i < d; i++) out[i] = x[i] * inv * w[i];
}

// RoPE at absolute position pos (rope_apply_pos, src/inference.c:189-203)
void rope_apply_pos(float *qk, const llmc_RoPEBuffer *rb, int n_heads, int head_dim, int pos) {
    const int half = head_dim / 2;
    const float *cr = rb->cos_table + (size_t)pos * half;
    const float *sr = rb->sin_table + (size_t)pos * half;
    for (int h = 0; h < n_heads; h++) {
        float *v = qk + (size_t)h * head_dim;
        for (int i = 0; i < half; i++) {
            const float v0 = v[2 * i] * cr[i] - v[2 * i + 1] * sr[i];
            const float v1 = v[2 * i] * sr[i] + v[2 * i + 1] * cr[i];
            v[2 * i] = v0;
            v[2 * i + 1] = v1;
        }
    }
}

// dot product with eight interleaved partial sums (a fixed order, so the
// result is deterministic; the reference's vec_dot, src/inference.c:133-155,
// likewise sums in vector lanes)
float dot8(const float *a, const float *b, int n) {
    float p[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int i = 0;
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; l++) p[l] += a[i + l] * b[i + l];
    float s = ((p[0] + p[4]) + (p[1] + p[5])) + ((p[2] + p[6]) + (p[3] + p[7]));
    for (; i < n; i++) s += a[i] * b[i];
    return s;
}

// softmax of one vector (softmax_vec, src/inference.c:218-225)
void softmax_vec(float *v, int n) {
    float mx = v[0];
    for (int i = 1; i < n; i++) if (v[i] > mx) mx = v[i];
    float sum = 0.0f;
    for (int i = 0; i < n; i++) { v[i] = std::exp(v[i] - mx); sum += v[i]; }
    const float inv = 1.0f / sum;
    for (int i = 0; i < n; i++) v[i] *= inv;
}

}  // namespace

// MOE_B200_DECODE=device: the whole step on the B200 (moe_b200_decoder),
// one decoder per Model, created on first use with the state's max_seq_len.
// The device keeps its own KV cache: s->kv_cache is not written; logits and
// seq_pos are.  A rewound seq_pos rewinds the device cache; a seq_pos ahead
// of it (steps taken on the host meanwhile) cannot be reconstructed.
// Per-layer trace of the host step's FFN half (moe_b200_llmc_trace_*): the
// pre-FFN x_norm and the FFN/MoE output of every layer of the last step.
std::mutex g_trace_mu;
bool g_trace_on = false;
std::vector<float> g_trace;      // [L][2][d]
int g_trace_d = 0, g_trace_L = 0;

static void trace_layer(int L, int l, int d, const float *x_norm, const float *ffn_out) {
    std::lock_guard<std::mutex> lk(g_trace_mu);
    if (!g_trace_on) return;
    if (g_trace_d != d || g_trace_L != L) {
        g_trace.assign((size_t)L * 2 * d, 0.0f);
        g_trace_d = d;
        g_trace_L = L;
    }
    std::memcpy(g_trace.data() + (size_t)l * 2 * d, x_norm, (size_t)d * sizeof(float));
    std::memcpy(g_trace.data() + ((size_t)l * 2 + 1) * d, ffn_out, (size_t)d * sizeof(float));
}

extern "C" int moe_b200_llmc_trace_enable(int enable) {
    std::lock_guard<std::mutex> lk(g_trace_mu);
    g_trace_on = enable != 0;
    g_trace.clear();
    g_trace_d = g_trace_L = 0;
    return MOE_B200_OK;
}

extern "C" int moe_b200_llmc_trace_read(int layer, float *x_norm, float *ffn_out) {
    std::lock_guard<std::mutex> lk(g_trace_mu);
    if (!g_trace_on || g_trace_L == 0) return MOE_B200_E_STATE;
    if (layer < 0 || layer >= g_trace_L) return MOE_B200_E_INVALID;
    const size_t d = (size_t)g_trace_d;
    if (x_norm) std::memcpy(x_norm, g_trace.data() + (size_t)layer * 2 * d, d * sizeof(float));
    if (ffn_out)
        std::memcpy(ffn_out, g_trace.data() + ((size_t)layer * 2 + 1) * d, d * sizeof(float));
    return MOE_B200_OK;
}

static bool device_mode() {
    const char *p = std::getenv("MOE_B200_DECODE");
    return p && !std::strcmp(p, "device");
}

static void device_step(const llmc_Model *m, llmc_InferenceState *s, int token) {
    moe_b200_decoder *dec = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_dec_mu);
        auto it = g_decoders.find(m);
        if (it == g_decoders.end()) {
            const int rc = moe_b200_decoder_create(m, s->max_seq_len, 0, &dec);
            if (rc) die("inference_step", "device decoder", rc);
            g_decoders[m] = dec;
        } else {
            dec = it->second;
        }
    }
    const int dpos = moe_b200_decoder_pos(dec);
    if (s->seq_pos != dpos) {
        if (s->seq_pos > dpos)
            die("inference_step", "state advanced past the device KV cache", MOE_B200_E_STATE);
        const int rc = moe_b200_decoder_set_pos(dec, s->seq_pos);
        if (rc) die("inference_step", "device decoder rewind", rc);
    }
    const int rc = moe_b200_decoder_step(dec, token, s->logits);
    if (rc) die("inference_step", "device decode step", rc);
    s->seq_pos++;
}

extern "C" void inference_step(const llmc_Model *m, llmc_InferenceState *s, int token) {
    if (device_mode()) {
        device_step(m, s, token);
        return;
    }
    const llmc_ModelConfig *cfg = &m->cfg;
    const int d = cfg->d_model, nh = cfg->n_heads, nkv = cfg->n_kv_heads, hd = cfg->head_dim;
    const int kv_dim = s->kv_dim, gqa = nh / nkv, pos = s->seq_pos;
    const float scale = 1.0f / std::sqrt((float)hd);
    if (pos >= s->max_seq_len) die("inference_step", "KV cache full", MOE_B200_E_INVALID);

    std::memcpy(s->x, m->weights.embed.data + (size_t)token * d, (size_t)d * sizeof(float));
    std::vector<float> ffn_scratch;
    for (int l = 0; l < cfg->n_layers; l++) {
        const llmc_BlockWeights *bw = &m->weights.blocks[l];
        llmc_LayerKVCache *kvc = &s->kv_cache[l];

        rmsnorm_vec(s->x, bw->rms_attn, cfg->rms_norm_eps, s->x_norm, d);
        matvec(bw->attn.W_Q.data, s->x_norm, s->q, d, nh * hd);
        matvec(bw->attn.W_K.data, s->x_norm, s->k, d, kv_dim);
        matvec(bw->attn.W_V.data, s->x_norm, s->v, d, kv_dim);
        rope_apply_pos(s->q, &m->rope, nh, hd, pos);
        rope_apply_pos(s->k, &m->rope, nkv, hd, pos);
        std::memcpy(kvc->K + (size_t)pos * kv_dim, s->k, (size_t)kv_dim * sizeof(float));
        std::memcpy(kvc->V + (size_t)pos * kv_dim, s->v, (size_t)kv_dim * sizeof(float));

        std::memset(s->head_out, 0, (size_t)nh * hd * sizeof(float));
        for (int qh = 0; qh < nh; qh++) {
            const int kvh = qh / gqa;
            const float *qv = s->q + (size_t)qh * hd;
            float *oh = s->head_out + (size_t)qh * hd;
            for (int j = 0; j <= pos; j++) {
                const float *kj = kvc->K + (size_t)j * kv_dim + (size_t)kvh * hd;
                s->attn_buf[j] = dot8(qv, kj, hd) * scale;
            }
            softmax_vec(s->attn_buf, pos + 1);
            for (int j = 0; j <= pos; j++) {
                const float *vj = kvc->V + (size_t)j * kv_dim + (size_t)kvh * hd;
                const float a = s->attn_buf[j];
                for (int i = 0; i < hd; i++) oh[i] += a * vj[i];
            }
        }
        float *attn_out = s->x_norm;      // scratch reuse, as the reference does
        matvec(bw->attn.W_O.data, s->head_out, attn_out, nh * hd, d);
        for (int i = 0; i < d; i++) s->x[i] += attn_out[i];

        rmsnorm_vec(s->x, bw->rms_ffn, cfg->rms_norm_eps, s->x_norm, d);
        const int F = cfg->ffn_hidden;
        if (!bw->use_moe) {
            ffn_scratch.resize((size_t)3 * F);
            float *gate = ffn_scratch.data(), *up = gate + F, *h = up + F;
            float *ffn_out = s->q;
            matvec(bw->ffn.W_gate.data, s->x_norm, gate, d, F);
            matvec(bw->ffn.W_up.data, s->x_norm, up, d, F);
            for (int i = 0; i < F; i++) h[i] = (gate[i] / (1.0f + std::exp(-gate[i]))) * up[i];
            matvec(bw->ffn.W_down.data, h, ffn_out, F, d);
            trace_layer(cfg->n_layers, l, d, s->x_norm, ffn_out);
            for (int i = 0; i < d; i++) s->x[i] += ffn_out[i];
        } else {
            // the MoE branch the reference leaves out (src/inference.c:342-343)
            ffn_scratch.resize((size_t)d);
            float *ffn_out = ffn_scratch.data();
            run_moe(&bw->moe, F, s->x_norm, 1, d, ffn_out, nullptr, nullptr, "inference_step");
            trace_layer(cfg->n_layers, l, d, s->x_norm, ffn_out);
            for (int i = 0; i < d; i++) s->x[i] += ffn_out[i];
        }
    }
    rmsnorm_vec(s->x, m->weights.rms_final, cfg->rms_norm_eps, s->x_norm, d);
    matvec(m->weights.lm_head.data, s->x_norm, s->logits, d, cfg->vocab_size);
    s->seq_pos++;
}
