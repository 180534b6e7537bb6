// weights.cuh — the device-resident expert set behind the opaque
// moe_b200_weights handle (internal to the library).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <vector>

#include "../../include/llmc_moe.h"
#include "../../include/moe_b200.h"

struct moe_b200_weights {
    int device;
    int d, F, E, k, d_pad, F_pad;
    // Packed expert slots.  A full set has n_slots == E with slot e holding
    // expert e.  An expert-parallel shard (shard = 1) holds only some
    // experts: slot_expert[j] is the global id in slot j, or -1 for a spare
    // slot that a hot expert's replica may fill later.  The router always
    // covers all E experts.
    int n_slots = 0, shard = 0;
    std::vector<int> slot_expert;
    float *router;   // [d × E] row-major (host layout)
    float *ug;       // [n_slots][2F_pad × d_pad]
    float *dn;       // [n_slots][d_pad × F_pad]
    CUtensorMap tm_ug;        // box {32, 256}
    CUtensorMap tm_dn;        // box {32, 256 or 128}
    CUtensorMap tm_ug64;      // box {32, 64}: decode up/gate (64 gate + 64 up rows)
    CUtensorMap tm_dn128;     // box {32, 128}: decode down
    CUtensorMap tm_ug128;     // box {32, 128}: CTA-pair up/gate (one 128-row gate or up block per CTA)
    int down_bn;
};


namespace moe {
// Record a status and its detail text as this host thread's last error
// (read back through moe_b200_last_error); returns `code`.
__attribute__((visibility("hidden"))) int set_last_error(int code, const char *detail);
// Stage-timing events for one forward on `device` (nullptr when timing is
// off): MOE_B200_NUM_STAGES + 1 events recorded between the stages.
__attribute__((visibility("hidden"))) cudaEvent_t *profile_events(int device);
// Record the expert count and kernel launches of the last forward.
__attribute__((visibility("hidden"))) void note_forward(int device, int E, int launches, int path);
// Number of SMs of `device` (0 if the device is unusable).
__attribute__((visibility("hidden"))) int device_sms(int device);
// cudaMalloc through the fault-injection hook (moe_b200_debug_fail_alloc).
__attribute__((visibility("hidden"))) cudaError_t dev_alloc(void **p, size_t bytes);
// MOE_B200_OK for a full expert set; MOE_B200_E_INVALID (with a message)
// for an expert-parallel shard, which only the moe_b200_ep_* calls run.
__attribute__((visibility("hidden"))) int weights_full(const moe_b200_weights *w);

// ---- building blocks shared by the upload, the checkpoint loader and the
// device decoder ----
// A device expert set of the given shape, weights not yet filled.
__attribute__((visibility("hidden"))) int weights_create(int d, int F, int E, int k,
                                                         moe_b200_weights **out);
// Repack expert `ex` from a device staging buffer holding its W_gate, W_up
// [d × F] and W_down [F × d] (llm.c's host layouts, back to back) into the
// set's packed layout, on `s`.
__attribute__((visibility("hidden"))) int weights_put_expert(moe_b200_weights *w, int ex,
                                                             const float *d_stage, cudaStream_t s);
// The library stream of the current device.
__attribute__((visibility("hidden"))) cudaStream_t current_stream();

// A device decoder from host tensors (llm.c layouts) and the blocks' FFNs
// already on the device; owns every blocks[l].ffn afterwards.
struct DecBlockSrc {
    const float *rms_attn = nullptr, *rms_ffn = nullptr;
    const float *W_Q = nullptr, *W_K = nullptr, *W_V = nullptr, *W_O = nullptr;
    moe_b200_weights *ffn = nullptr;
};
struct DecSrc {
    llmc_ModelConfig cfg;
    const float *embed = nullptr, *rms_final = nullptr, *lm_head = nullptr;
    const float *rope_cos = nullptr, *rope_sin = nullptr;   // [rope_len × head_dim/2]
    int rope_len = 0;
    std::vector<DecBlockSrc> blocks;
};
__attribute__((visibility("hidden"))) int decoder_build(const DecSrc &src, int max_seq, int flags,
                                                        moe_b200_decoder **out);
}  // namespace moe
