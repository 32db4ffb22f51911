// Host-side definitions shared by the C-ABI sources of g4attn (not part of
// the ABI): the context object and the error helpers that fill its message.
#pragma once

#include <cstdarg>
#include <cstdio>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/g4attn.h"
#include "internal.h"

struct g4a_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    g4a_hparams hp{};
    std::vector<float> rope_freqs;  // head_dim_global / 2 divisors
    int32_t max_positions = 0;
    float2 *d_rope_local = nullptr;
    float2 *d_rope_global = nullptr;
    int *d_err = nullptr;
    std::string last_error;
    float *d_part_o = nullptr;
    size_t part_o_cap = 0;  // floats
    float *d_part_ml = nullptr;
    size_t part_ml_cap = 0;
    unsigned *d_tickets = nullptr;
    size_t tickets_cap = 0;
    // Device errors reported so far, and the count when d_tickets was last
    // cleared: a step that aborted may leave split-task tickets counted.
    uint32_t err_epoch = 0;
    uint32_t tickets_epoch = 0;
    uint8_t *d_meta = nullptr;
    size_t meta_cap = 0;
    std::vector<uint8_t> h_meta;
    g4a::PrefillScratch *prefill = nullptr;
    int n_sm = 148;
    uint8_t *d_qblocks = nullptr;
    size_t qblocks_cap = 0;
    // per-kernel timing (g4a_profile_enable): events around each launch
    bool profiling = false;
    struct Rec {
        int kernel;
        cudaEvent_t a, b;
    };
    std::vector<Rec> recs;
    std::vector<cudaEvent_t> spare;
    double prof_ms[G4A_K_COUNT] = {};
    int64_t prof_n[G4A_K_COUNT] = {};
    // Pinned staging for the small per-call uploads (decode metadata, block
    // tables): a copy from pageable memory goes through the driver's own
    // staging and costs tens of microseconds per call. Slots are reused in
    // turn; an event per slot keeps a slot from being rewritten before the
    // GPU has read its previous contents.
    struct PinnedSlot {
        uint8_t *p = nullptr;
        size_t cap = 0;
        cudaEvent_t ev = nullptr;
        bool pending = false;
    };
    PinnedSlot pin[4];
    int pin_next = 0;
    // Q8_0 mat-vec: the quantized activations of the current call
    int8_t *d_q8x = nullptr;
    size_t q8x_cap = 0;
    float *d_q8s = nullptr;
    size_t q8s_cap = 0;
    // g4a_decode_host: device copies of the callers' host q/k/v/out, and a
    // pinned word receiving the error flag at the end of the call
    float *d_io = nullptr;
    size_t io_cap = 0;  // floats
    int *h_flag = nullptr;
    // g4a_decode_host's copy streams (host-to-device inputs, device-to-host
    // outputs) and its events: per layer, inputs copied and kernels done
    cudaStream_t copy_in = nullptr, copy_out = nullptr;
    std::vector<cudaEvent_t> io_events;
    // g4a_debug_stall: kernels (bit per g4a_kernel id) whose next launch runs
    // the bounded test wait instead of its work
    uint32_t stall_mask = 0;
    // context-parallel prefill state (cp_host.cpp), freed by cp_free
    void *cp = nullptr;
    void (*cp_free)(void *) = nullptr;
};

namespace g4a {

// Sets the context's message (g4a_last_error) and returns `code`.
inline int fail(g4a_ctx *ctx, int code, const char *fmt, ...) {
    if (ctx) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof buf, fmt, ap);
        va_end(ap);
        ctx->last_error = buf;
    }
    return code;
}

inline int cuda_fail(g4a_ctx *ctx, cudaError_t e, const char *what) {
    return fail(ctx, G4A_CUDA, "compute: %s: %s", what, cudaGetErrorString(e));
}

}  // namespace g4a

#define G4A_CUDA_TRY(ctx, call)                                  \
    do {                                                         \
        cudaError_t e_ = (call);                                 \
        if (e_ != cudaSuccess) return g4a::cuda_fail(ctx, e_, #call); \
    } while (0)
