// llmc_compat.cpp — llm.c's moe_forward entry point over the C-ABI.
//
// Residency cache: one device expert set per MoEWeights pointer, uploaded
// on first sight from the host matrices (include/transformer.h:53-58) and
// kept until moe_b200_invalidate or shutdown.
#include "../../include/llmc_moe.h"
#include "../../include/moe_b200.h"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <unordered_map>
#include <vector>

namespace {
std::mutex g_cache_mu;
std::unordered_map<const void *, moe_b200_weights *> g_cache;

int env_path() {
    const char *p = std::getenv("MOE_B200_PATH");
    if (!p || !*p || !std::strcmp(p, "auto")) return MOE_B200_PATH_AUTO;
    if (!std::strcmp(p, "tf32")) return MOE_B200_PATH_TF32;
    if (!std::strcmp(p, "fp32")) return MOE_B200_PATH_FP32;
    return MOE_B200_PATH_AUTO;
}

[[noreturn]] void die(const char *what, int rc) {
    std::fprintf(stderr, "[moe_b200] moe_forward: %s: %s (%s)\n", what, moe_b200_strerror(rc),
                 moe_b200_last_error());
    std::abort();
}
}  // namespace

extern "C" void moe_forward(const llmc_Matrix *x, const llmc_MoEWeights *mw,
                            const llmc_ModelConfig *cfg, llmc_ForwardCache *cache,
                            llmc_Matrix *out) {
    const int T = x->rows, d = x->cols, E = mw->n_experts, k = mw->top_k, F = cfg->ffn_hidden;
    if (out->rows != T || out->cols != d || mw->W_router.rows != d || mw->W_router.cols != E)
        die("shape mismatch", MOE_B200_E_INVALID);
    moe_b200_weights *w = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_cache_mu);
        auto it = g_cache.find(mw);
        if (it != g_cache.end()) {
            w = it->second;
        } else {
            std::vector<const float *> g(E), u(E), dn(E);
            for (int e = 0; e < E; e++) {
                const llmc_FFNWeights &fw = mw->experts[e];
                if (fw.W_gate.rows != d || fw.W_gate.cols != F || fw.W_up.rows != d ||
                    fw.W_up.cols != F || fw.W_down.rows != F || fw.W_down.cols != d)
                    die("expert shape mismatch", MOE_B200_E_INVALID);
                g[e] = fw.W_gate.data;
                u[e] = fw.W_up.data;
                dn[e] = fw.W_down.data;
            }
            int rc = moe_b200_weights_upload(mw->W_router.data, g.data(), u.data(), dn.data(), d,
                                             F, E, k, &w);
            if (rc) die("weight upload", rc);
            g_cache[mw] = w;
        }
    }
    moe_b200_opts opts;
    std::memset(&opts, 0, sizeof opts);
    opts.path = env_path();
    int rc = moe_b200_forward(w, nullptr, x->data, T, out->data, cache ? cache->router_probs : nullptr,
                              cache ? cache->expert_ids : nullptr, &opts);
    if (rc) die("forward", rc);
}

extern "C" int moe_b200_invalidate(const void *moe_weights) {
    std::lock_guard<std::mutex> lk(g_cache_mu);
    auto it = g_cache.find(moe_weights);
    if (it == g_cache.end()) return MOE_B200_OK;
    int rc = moe_b200_weights_free(it->second);
    g_cache.erase(it);
    return rc;
}
