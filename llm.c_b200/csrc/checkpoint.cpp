// checkpoint.cpp — llm.c checkpoints (model_save / model_load format,
// src/transformer.c:573-697) read straight to the device.
//
// The file is the magic 0x4C4C4D43 ("CLLM"), llm.c's ModelConfig as stored
// by fwrite (13 four-byte fields), then every tensor as raw little-endian
// fp32 in a fixed order: the embedding [vocab × d]; per block rms_attn [d],
// W_Q [d × nq], W_K [d × kvd], W_V [d × kvd], W_O [nq × d], rms_ffn [d],
// then either the dense FFN (W_gate, W_up [d × F], W_down [F × d]) or, when
// n_experts > 1 (every block, src/transformer.c:437), the router [d × E]
// and each expert's W_gate, W_up, W_down; then rms_final [d] and the LM
// head [d × vocab].
//
// Experts are streamed: two pinned host buffers and two device staging
// buffers of one expert each, so the disk read of expert e+1 overlaps the
// copy and the repack of expert e, and the host never holds more than two
// experts (c5's 45 GB of experts pass through 1.4 GB of pinned memory).
#include "weights.cuh"

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <memory>
#include <vector>

namespace {

constexpr uint32_t kMagic = 0x4C4C4D43u;
static_assert(sizeof(llmc_ModelConfig) == 52, "llm.c's ModelConfig is 13 four-byte fields");

int cfail(int code, const char *msg) { return moe::set_last_error(code, msg); }

struct FileCloser {
    void operator()(FILE *f) const { if (f) std::fclose(f); }
};
using File = std::unique_ptr<FILE, FileCloser>;

int open_checkpoint(const char *path, File &f, llmc_ModelConfig &cfg) {
    if (!path) return cfail(MOE_B200_E_INVALID, "null path");
    f.reset(std::fopen(path, "rb"));
    if (!f) return cfail(MOE_B200_E_INVALID, "cannot open the checkpoint");
    uint32_t magic = 0;
    if (std::fread(&magic, 4, 1, f.get()) != 1 || magic != kMagic)
        return cfail(MOE_B200_E_INVALID, "not an llm.c checkpoint (bad magic)");
    if (std::fread(&cfg, sizeof cfg, 1, f.get()) != 1)
        return cfail(MOE_B200_E_INVALID, "truncated checkpoint header");
    if (cfg.vocab_size <= 0 || cfg.d_model <= 0 || cfg.n_layers <= 0 || cfg.n_heads <= 0 ||
        cfg.n_kv_heads <= 0 || cfg.head_dim <= 0 || cfg.ffn_hidden <= 0 ||
        cfg.n_heads % cfg.n_kv_heads || cfg.n_experts > 4096 || cfg.top_k_experts < 0)
        return cfail(MOE_B200_E_INVALID, "checkpoint config out of range");
    return MOE_B200_OK;
}

int read_floats(FILE *f, float *dst, size_t n) {
    return std::fread(dst, sizeof(float), n, f) == n
               ? MOE_B200_OK
               : cfail(MOE_B200_E_INVALID, "truncated checkpoint");
}

int skip_floats(FILE *f, size_t n) {
    return fseeko(f, (off_t)(n * sizeof(float)), SEEK_CUR) == 0
               ? MOE_B200_OK
               : cfail(MOE_B200_E_INVALID, "truncated checkpoint");
}

struct Shape {
    size_t d, nq, kvd, F, E, vocab;
    bool moe;
    size_t attn_floats() const { return d + d * nq + 2 * d * kvd + nq * d + d; }
    size_t ffn_floats() const { return moe ? d * E + E * 3 * d * F : 3 * d * F; }
};

Shape shape_of(const llmc_ModelConfig &c) {
    Shape s;
    s.d = (size_t)c.d_model;
    s.nq = (size_t)c.n_heads * c.head_dim;
    s.kvd = (size_t)c.n_kv_heads * c.head_dim;
    s.F = (size_t)c.ffn_hidden;
    s.moe = c.n_experts > 1;
    s.E = s.moe ? (size_t)c.n_experts : 1;
    s.vocab = (size_t)c.vocab_size;
    return s;
}

// The FFN block at the file position into a new device expert set: the
// router and every expert (or the dense FFN as one expert with router 0).
int stream_ffn(FILE *f, const llmc_ModelConfig &cfg, moe_b200_weights **out) {
    const Shape S = shape_of(cfg);
    const int k = S.moe ? cfg.top_k_experts : 1;
    moe_b200_weights *w = nullptr;
    int rc = moe::weights_create((int)S.d, (int)S.F, (int)S.E, k, &w);
    if (rc) return rc;
    cudaStream_t s = moe::current_stream();
    const size_t per = 3 * S.d * S.F;           // W_gate, W_up, W_down back to back
    float *pin[2] = {nullptr, nullptr}, *dst[2] = {nullptr, nullptr};
    cudaEvent_t ev[2] = {nullptr, nullptr};
    auto cleanup = [&]() {
        if (s) cudaStreamSynchronize(s);
        for (int b = 0; b < 2; b++) {
            if (pin[b]) cudaFreeHost(pin[b]);
            if (dst[b]) cudaFree(dst[b]);
            if (ev[b]) cudaEventDestroy(ev[b]);
        }
    };
    do {
        if (!s) { rc = cfail(MOE_B200_E_CUDA, "no library stream"); break; }
        std::vector<float> router(S.d * S.E, 0.0f);
        if (S.moe && (rc = read_floats(f, router.data(), router.size()))) break;
        if (cudaMemcpy(w->router, router.data(), router.size() * 4, cudaMemcpyHostToDevice)) {
            rc = cfail(MOE_B200_E_CUDA, "router upload failed");
            break;
        }
        bool ok = true;
        for (int b = 0; b < 2 && ok; b++)
            ok = cudaMallocHost(&pin[b], per * 4) == cudaSuccess &&
                 cudaMalloc(&dst[b], per * 4) == cudaSuccess &&
                 cudaEventCreateWithFlags(&ev[b], cudaEventDisableTiming) == cudaSuccess;
        if (!ok) {
            cudaGetLastError();
            rc = cfail(MOE_B200_E_NOMEM, "checkpoint staging buffers");
            break;
        }
        for (size_t e = 0; e < S.E && !rc; e++) {
            const int b = (int)(e & 1);
            // pin[b] is free once its previous copy (expert e - 2) finished
            if (e >= 2 && cudaEventSynchronize(ev[b])) { rc = cfail(MOE_B200_E_CUDA, "copy"); break; }
            if ((rc = read_floats(f, pin[b], per))) break;
            if (cudaMemcpyAsync(dst[b], pin[b], per * 4, cudaMemcpyHostToDevice, s) ||
                cudaEventRecord(ev[b], s)) {
                rc = cfail(MOE_B200_E_CUDA, "expert copy failed");
                break;
            }
            // dst[b] is next written (expert e + 2) only after this repack, in stream order
            rc = moe::weights_put_expert(w, (int)e, dst[b], s);
        }
        if (!rc && cudaStreamSynchronize(s)) rc = cfail(MOE_B200_E_CUDA, "expert repack failed");
    } while (0);
    cleanup();
    if (rc) {
        moe_b200_weights_free(w);
        return rc;
    }
    *out = w;
    return MOE_B200_OK;
}

}  // namespace

extern "C" int moe_b200_checkpoint_config(const char *path, void *cfg) {
    if (!cfg) return cfail(MOE_B200_E_INVALID, "null config");
    File f;
    llmc_ModelConfig c;
    const int rc = open_checkpoint(path, f, c);
    if (rc) return rc;
    std::memcpy(cfg, &c, sizeof c);
    return MOE_B200_OK;
}

extern "C" int moe_b200_checkpoint_load_experts(const char *path, int layer, moe_b200_weights **out) {
    if (!out) return cfail(MOE_B200_E_INVALID, "null output");
    *out = nullptr;
    File f;
    llmc_ModelConfig c;
    int rc = open_checkpoint(path, f, c);
    if (rc) return rc;
    if (layer < 0 || layer >= c.n_layers) return cfail(MOE_B200_E_INVALID, "layer out of range");
    const Shape S = shape_of(c);
    // skip the embedding, the earlier blocks and this block's attention part
    const size_t skip = S.vocab * S.d + (size_t)layer * (S.attn_floats() + S.ffn_floats()) +
                        S.attn_floats();
    if ((rc = skip_floats(f.get(), skip))) return rc;
    return stream_ffn(f.get(), c, out);
}

extern "C" int moe_b200_decoder_load(const char *path, int max_seq, int flags,
                                     moe_b200_decoder **out) {
    if (!out) return cfail(MOE_B200_E_INVALID, "null output");
    *out = nullptr;
    File f;
    llmc_ModelConfig c;
    int rc = open_checkpoint(path, f, c);
    if (rc) return rc;
    if ((rc = moe_b200_init(-1))) return rc;
    const Shape S = shape_of(c);
    const int L = c.n_layers, hd = c.head_dim, half = hd / 2;
    // model_load builds its RoPE table for cfg.max_seq_len positions (src/transformer.c:505)
    if (max_seq <= 0 || max_seq > c.max_seq_len)
        return cfail(MOE_B200_E_INVALID, "max_seq exceeds the model's RoPE table");
    if (hd % 2) return cfail(MOE_B200_E_INVALID, "odd head_dim");
    moe::DecSrc src;
    src.cfg = c;
    std::vector<float> embed(S.vocab * S.d), rms_final(S.d), lm_head(S.d * S.vocab);
    struct HostBlock {
        std::vector<float> rms_attn, W_Q, W_K, W_V, W_O, rms_ffn;
    };
    std::vector<HostBlock> hb(L);
    src.blocks.resize(L);
    auto drop = [&](int n) {
        for (int q = 0; q < n; q++) moe_b200_weights_free(src.blocks[q].ffn);
    };
    if ((rc = read_floats(f.get(), embed.data(), embed.size()))) return rc;
    for (int l = 0; l < L; l++) {
        HostBlock &h = hb[l];
        h.rms_attn.resize(S.d); h.W_Q.resize(S.d * S.nq); h.W_K.resize(S.d * S.kvd);
        h.W_V.resize(S.d * S.kvd); h.W_O.resize(S.nq * S.d); h.rms_ffn.resize(S.d);
        if ((rc = read_floats(f.get(), h.rms_attn.data(), h.rms_attn.size())) ||
            (rc = read_floats(f.get(), h.W_Q.data(), h.W_Q.size())) ||
            (rc = read_floats(f.get(), h.W_K.data(), h.W_K.size())) ||
            (rc = read_floats(f.get(), h.W_V.data(), h.W_V.size())) ||
            (rc = read_floats(f.get(), h.W_O.data(), h.W_O.size())) ||
            (rc = read_floats(f.get(), h.rms_ffn.data(), h.rms_ffn.size())) ||
            (rc = stream_ffn(f.get(), c, &src.blocks[l].ffn))) {
            drop(l);
            return rc;
        }
        moe::DecBlockSrc &o = src.blocks[l];
        o.rms_attn = h.rms_attn.data(); o.rms_ffn = h.rms_ffn.data();
        o.W_Q = h.W_Q.data(); o.W_K = h.W_K.data(); o.W_V = h.W_V.data(); o.W_O = h.W_O.data();
    }
    if ((rc = read_floats(f.get(), rms_final.data(), rms_final.size())) ||
        (rc = read_floats(f.get(), lm_head.data(), lm_head.size()))) {
        drop(L);
        return rc;
    }
    // RoPE tables as llm.c builds them (rope_buffer_init, src/attention.c:151-167)
    std::vector<float> cos_t((size_t)max_seq * half), sin_t((size_t)max_seq * half);
    for (int pos = 0; pos < max_seq; pos++)
        for (int i = 0; i < half; i++) {
            const float angle = (float)pos / powf(c.rope_theta, 2.f * (float)i / (float)hd);
            cos_t[(size_t)pos * half + i] = cosf(angle);
            sin_t[(size_t)pos * half + i] = sinf(angle);
        }
    src.embed = embed.data();
    src.rms_final = rms_final.data();
    src.lm_head = lm_head.data();
    src.rope_cos = cos_t.data();
    src.rope_sin = sin_t.data();
    src.rope_len = max_seq;
    return moe::decoder_build(src, max_seq, flags, out);
}
