// weights.cuh — the device-resident expert set behind the opaque
// moe_b200_weights handle (internal to the library).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

struct moe_b200_weights {
    int device;
    int d, F, E, k, d_pad, F_pad;
    float *router;   // [d × E] row-major (host layout)
    float *ug;       // [E][2F_pad × d_pad]
    float *dn;       // [E][d_pad × F_pad]
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
}  // namespace moe
