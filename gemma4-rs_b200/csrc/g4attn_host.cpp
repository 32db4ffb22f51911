// Host side of g4attn: the C ABI declared in include/g4attn.h.
//
// Mirrors the reference's attention boundary: hyperparameters and layer
// policies (crates/llm-gemma4/src/idea/mod.rs, eng/mod.rs), the per-layer
// K/V memory (crates/llm-eng/src/context_memory.rs) as a paged device cache,
// and the attention block of TransformerSpec::layer
// (crates/llm-gemma4/src/impl_/model.rs:393-410) as one fused device call.
// Error statuses and messages follow crates/llm-eng/src/error.rs.
#include <algorithm>
#include <chrono>
#include <functional>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/g4attn.h"
#include "internal.h"
#include "host_internal.h"

using namespace g4a;

// --------------------------------------------------------------------------
// hyperparameters and policies
// --------------------------------------------------------------------------

extern "C" void g4a_hparams_e2b(g4a_hparams *hp) {  // idea/mod.rs:48-68
    hp->n_layers = 35;
    hp->n_heads = 8;
    hp->n_kv_heads = 1;
    hp->head_dim_local = 256;
    hp->head_dim_global = 512;
    hp->sliding_window = 512;
    hp->shared_kv_layers = 20;
    hp->local_rope_base = 10000.0f;
    hp->global_rope_base = 1000000.0f;
    hp->global_p = 0.25f;
    hp->rms_norm_eps = 1e-6f;
}

extern "C" int g4a_layer_is_global(const g4a_hparams *hp, int32_t layer) {  // idea/mod.rs:148-156
    return (layer + 1 == hp->n_layers) || (layer % 5 == 4);
}

extern "C" int32_t g4a_head_dim(const g4a_hparams *hp, int32_t layer) {  // idea/mod.rs:140-145
    return g4a_layer_is_global(hp, layer) ? hp->head_dim_global : hp->head_dim_local;
}

extern "C" int g4a_kv_source_layer(const g4a_hparams *hp, int32_t layer, int32_t *source, int32_t *detail) {
    // eng/mod.rs:71-90
    const int32_t n = hp->n_layers;
    if (layer < 0 || layer >= n) {
        if (detail) *detail = 1;
        return G4A_BAD_LAYER;
    }
    const int32_t first_shared = n - hp->shared_kv_layers;
    if (hp->shared_kv_layers > n || first_shared <= 0) {
        if (detail) *detail = 2;
        return G4A_BAD_LAYER;
    }
    if (layer < first_shared) {
        *source = layer;
        return G4A_OK;
    }
    const int kind = g4a_layer_is_global(hp, layer);
    for (int32_t e = first_shared - 1; e >= 0; e--) {
        if (g4a_layer_is_global(hp, e) == kind) {
            *source = e;
            return G4A_OK;
        }
    }
    if (detail) *detail = 3;
    return G4A_BAD_LAYER;
}

extern "C" void g4a_windowed_len(int64_t seq_len, int64_t window, int64_t *lo, int64_t *hi) {  // eng/mod.rs:10-12
    *lo = seq_len > window ? seq_len - window : 0;
    *hi = seq_len;
}

extern "C" void g4a_proportional_rope_freq_factors(int32_t head_dim, float p, float *out) {  // idea/mod.rs:162-165
    const int32_t rotated = (int32_t)((float)head_dim * p / 2.0f);
    for (int32_t pair = 0; pair < head_dim / 2; pair++) out[pair] = pair < rotated ? 1.0f : 1e30f;
}

// --------------------------------------------------------------------------
// context
// --------------------------------------------------------------------------


namespace {

// Host-to-device copy of `bytes` from `src` on the context's stream through
// a pinned staging slot (falls back to a pageable copy if pinning fails).
cudaError_t upload(g4a_ctx *ctx, void *dst, const void *src, size_t bytes) {
    if (!bytes) return cudaSuccess;
    g4a_ctx::PinnedSlot &sl = ctx->pin[ctx->pin_next];
    ctx->pin_next = (ctx->pin_next + 1) % 4;
    if (sl.pending) {
        cudaError_t e = cudaEventSynchronize(sl.ev);
        if (e != cudaSuccess) return e;
        sl.pending = false;
    }
    if (!sl.ev && cudaEventCreateWithFlags(&sl.ev, cudaEventDisableTiming) != cudaSuccess) sl.ev = nullptr;
    if (sl.cap < bytes) {
        if (sl.p) cudaFreeHost(sl.p);
        sl.p = nullptr;
        sl.cap = 0;
        const size_t want = std::max<size_t>(bytes, 1 << 16);
        if (cudaHostAlloc(reinterpret_cast<void **>(&sl.p), want, cudaHostAllocDefault) == cudaSuccess) sl.cap = want;
        else sl.p = nullptr;
    }
    if (!sl.p || !sl.ev) return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream);
    std::memcpy(sl.p, src, bytes);
    cudaError_t e = cudaMemcpyAsync(dst, sl.p, bytes, cudaMemcpyHostToDevice, ctx->stream);
    if (e != cudaSuccess) return e;
    e = cudaEventRecord(sl.ev, ctx->stream);
    sl.pending = e == cudaSuccess;
    return e;
}


// Builds (sin, cos) of every pair at positions [0, n_pos) exactly as
// ops.rs:150-159 does: theta_scale = base^(-2/n_rot) by powf, theta grows by
// repeated f32 multiplication, angle = theta / factor.
std::vector<float2> rope_table(int32_t n_pos, float base, int32_t n_rot, const float *factors) {
    const int32_t half = n_rot / 2;
    std::vector<float2> t((size_t)n_pos * half);
    const float theta_scale = powf(base, -2.0f / (float)n_rot);
    for (int32_t pos = 0; pos < n_pos; pos++) {
        float theta = (float)pos;
        float2 *row = t.data() + (size_t)pos * half;
        for (int32_t i = 0; i < half; i++) {
            const float factor = factors ? factors[i] : 1.0f;
            const float angle = theta / factor;
            row[i] = make_float2(sinf(angle), cosf(angle));
            theta *= theta_scale;
        }
    }
    return t;
}

int ensure_rope(g4a_ctx *ctx, int32_t n_pos) {
    if (n_pos <= ctx->max_positions && ctx->d_rope_local) return G4A_OK;
    cudaSetDevice(ctx->device);
    if (ctx->d_rope_local) {
        cudaStreamSynchronize(ctx->stream);
        cudaFree(ctx->d_rope_local);
        cudaFree(ctx->d_rope_global);
        ctx->d_rope_local = ctx->d_rope_global = nullptr;
    }
    const g4a_hparams &hp = ctx->hp;
    auto loc = rope_table(n_pos, hp.local_rope_base, hp.head_dim_local, nullptr);
    auto glo = rope_table(n_pos, hp.global_rope_base, hp.head_dim_global, ctx->rope_freqs.data());
    G4A_CUDA_TRY(ctx, cudaMalloc(&ctx->d_rope_local, loc.size() * sizeof(float2)));
    G4A_CUDA_TRY(ctx, cudaMalloc(&ctx->d_rope_global, glo.size() * sizeof(float2)));
    G4A_CUDA_TRY(ctx, cudaMemcpy(ctx->d_rope_local, loc.data(), loc.size() * sizeof(float2), cudaMemcpyHostToDevice));
    G4A_CUDA_TRY(ctx, cudaMemcpy(ctx->d_rope_global, glo.data(), glo.size() * sizeof(float2), cudaMemcpyHostToDevice));
    ctx->max_positions = n_pos;
    return G4A_OK;
}

template <typename T>
int grow(g4a_ctx *ctx, T **ptr, size_t *cap, size_t need, bool zero) {
    if (need <= *cap) return G4A_OK;
    size_t n = std::max(need, *cap * 2);
    if (*ptr) {
        cudaStreamSynchronize(ctx->stream);
        cudaFree(*ptr);
        *ptr = nullptr;
        *cap = 0;
    }
    G4A_CUDA_TRY(ctx, cudaMalloc(ptr, n * sizeof(T)));
    if (zero) G4A_CUDA_TRY(ctx, cudaMemsetAsync(*ptr, 0, n * sizeof(T), ctx->stream));
    *cap = n;
    return G4A_OK;
}

// Runs `launch` between two events on the context's stream when profiling.
template <typename F>
cudaError_t timed(g4a_ctx *ctx, int kernel, F launch) {
    if (!ctx->profiling) return launch();
    cudaEvent_t ev[2];
    for (auto &e : ev) {
        if (!ctx->spare.empty()) {
            e = ctx->spare.back();
            ctx->spare.pop_back();
        } else {
            cudaEventCreate(&e);
        }
    }
    cudaEventRecord(ev[0], ctx->stream);
    cudaError_t err = launch();
    cudaEventRecord(ev[1], ctx->stream);
    ctx->recs.push_back({kernel, ev[0], ev[1]});
    return err;
}

void collect_profile(g4a_ctx *ctx) {
    if (ctx->recs.empty()) return;
    cudaStreamSynchronize(ctx->stream);
    for (auto &r : ctx->recs) {
        float ms = 0.0f;
        if (cudaEventElapsedTime(&ms, r.a, r.b) == cudaSuccess) {
            ctx->prof_ms[r.kernel] += ms;
            ctx->prof_n[r.kernel] += 1;
        }
        ctx->spare.push_back(r.a);
        ctx->spare.push_back(r.b);
    }
    ctx->recs.clear();
}

}  // namespace

extern "C" int g4a_profile_enable(g4a_ctx *ctx, int enable) {
    if (!ctx) return G4A_COMPUTE;
    cudaSetDevice(ctx->device);
    collect_profile(ctx);
    for (int k = 0; k < G4A_K_COUNT; k++) ctx->prof_ms[k] = 0.0, ctx->prof_n[k] = 0;
    ctx->profiling = enable != 0;
    return G4A_OK;
}

extern "C" int g4a_profile_read(g4a_ctx *ctx, int32_t kernel, double *total_ms, int64_t *launches) {
    if (!ctx || kernel < 0 || kernel >= G4A_K_COUNT || !total_ms || !launches) return G4A_COMPUTE;
    cudaSetDevice(ctx->device);
    collect_profile(ctx);
    *total_ms = ctx->prof_ms[kernel];
    *launches = ctx->prof_n[kernel];
    return G4A_OK;
}

extern "C" int g4a_ctx_create(int device, const g4a_hparams *hp, const float *rope_freqs, int32_t max_positions,
                              g4a_ctx **out) {
    if (!hp || !out) return G4A_COMPUTE;
    *out = nullptr;
    if (hp->n_layers <= 0 || hp->n_heads <= 0 || hp->n_kv_heads <= 0 || hp->n_heads % hp->n_kv_heads != 0 ||
        hp->head_dim_local <= 0 || hp->head_dim_global <= 0 || hp->head_dim_local % 2 || hp->head_dim_global % 2 ||
        hp->rms_norm_eps < 0.0f || max_positions <= 0)
        return G4A_COMPUTE;  // idea/mod.rs:125-137 validate
    auto *ctx = new g4a_ctx();
    ctx->device = device;
    ctx->hp = *hp;
    ctx->rope_freqs.resize(hp->head_dim_global / 2);
    if (rope_freqs)
        std::copy(rope_freqs, rope_freqs + hp->head_dim_global / 2, ctx->rope_freqs.begin());
    else
        g4a_proportional_rope_freq_factors(hp->head_dim_global, hp->global_p, ctx->rope_freqs.data());
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) {
        delete ctx;
        return G4A_CUDA;
    }
    ctx->prefill = prefill_scratch_new();
    cudaDeviceGetAttribute(&ctx->n_sm, cudaDevAttrMultiProcessorCount, device);
    if (ctx->n_sm <= 0) ctx->n_sm = 148;
    int rc = ensure_rope(ctx, max_positions);
    if (rc == G4A_OK) {
        e = cudaMalloc(&ctx->d_err, sizeof(int));
        if (e == cudaSuccess) e = cudaMemset(ctx->d_err, 0, sizeof(int));
        if (e != cudaSuccess) rc = G4A_CUDA;
    }
    if (rc != G4A_OK) {
        g4a_ctx_destroy(ctx);
        return rc;
    }
    *out = ctx;
    return G4A_OK;
}

extern "C" void g4a_ctx_destroy(g4a_ctx *ctx) {
    if (!ctx) return;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    cudaFree(ctx->d_rope_local);
    cudaFree(ctx->d_rope_global);
    cudaFree(ctx->d_err);
    cudaFree(ctx->d_part_o);
    cudaFree(ctx->d_part_ml);
    cudaFree(ctx->d_tickets);
    cudaFree(ctx->d_meta);
    cudaFree(ctx->d_qblocks);
    for (auto &r : ctx->recs) cudaEventDestroy(r.a), cudaEventDestroy(r.b);
    for (auto e : ctx->spare) cudaEventDestroy(e);
    cudaFree(ctx->d_q8x);
    cudaFree(ctx->d_q8s);
    cudaFree(ctx->d_io);
    if (ctx->h_flag) cudaFreeHost(ctx->h_flag);
    if (ctx->copy_in) cudaStreamSynchronize(ctx->copy_in), cudaStreamDestroy(ctx->copy_in);
    if (ctx->copy_out) cudaStreamSynchronize(ctx->copy_out), cudaStreamDestroy(ctx->copy_out);
    for (auto e : ctx->io_events) cudaEventDestroy(e);
    for (auto &sl : ctx->pin) {
        if (sl.p) cudaFreeHost(sl.p);
        if (sl.ev) cudaEventDestroy(sl.ev);
    }
    prefill_scratch_free(ctx->prefill);
    if (ctx->cp_free) ctx->cp_free(ctx->cp);
    delete ctx;
}

extern "C" const char *g4a_last_error(const g4a_ctx *ctx) { return ctx ? ctx->last_error.c_str() : "no context"; }

extern "C" int g4a_ctx_set_stream(g4a_ctx *ctx, void *stream) {
    if (!ctx) return G4A_COMPUTE;
    ctx->stream = (cudaStream_t)stream;
    return G4A_OK;
}

extern "C" int g4a_debug_stall(g4a_ctx *ctx, int32_t kernel) {
    if (!ctx) return G4A_COMPUTE;
    if (kernel != G4A_K_DECODE_MAIN && kernel != G4A_K_PREFILL)
        return fail(ctx, G4A_COMPUTE, "compute: no stall test for kernel %d", kernel);
    ctx->stall_mask |= 1u << kernel;
    return G4A_OK;
}

extern "C" int g4a_sync(g4a_ctx *ctx) {
    if (!ctx) return G4A_COMPUTE;
    cudaSetDevice(ctx->device);
    G4A_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    int flag = 0;
    G4A_CUDA_TRY(ctx, cudaMemcpy(&flag, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (flag) {
        ctx->err_epoch++;
        G4A_CUDA_TRY(ctx, cudaMemset(ctx->d_err, 0, sizeof(int)));
        if (flag & 6)  // bit 1: a prefill wait ran out, bit 2: a decode wait ran out
            return fail(ctx, G4A_TIMEOUT, "compute: a device wait ran out (flag %d)", flag);
        return fail(ctx, G4A_NONFINITE, "compute: softmax input is not finite");
    }
    return G4A_OK;
}

// --------------------------------------------------------------------------
// paged KV cache
// --------------------------------------------------------------------------

struct g4a_kv {
    g4a_ctx *ctx = nullptr;
    int32_t n_seqs = 0, max_tokens = 0, page_tokens = 0, n_pages = 0, dtype = 0, max_pages = 0;
    size_t elem = 4;
    struct Layer {
        bool held = false;
        int32_t hd = 0;
        void *k = nullptr, *v = nullptr;
    };
    std::vector<Layer> layers;       // indexed by model layer
    std::vector<int32_t> h_bt;       // [n_seqs][max_pages], -1 = unassigned
    int32_t *d_bt = nullptr;
    bool bt_dirty = true;
    std::vector<int64_t> len;        // [n_seqs][n_layers] rows stored
    std::vector<int32_t> seq_pages;  // logical pages assigned per sequence
    std::vector<int32_t> free_pages;
    uint8_t *d_tmaps = nullptr;  // f16 caches: [n_layers][K, V] 128-byte TMA descriptors
};

namespace {

int64_t &kv_len(g4a_kv *kv, int32_t seq, int32_t layer) { return kv->len[(size_t)seq * kv->layers.size() + layer]; }

int ensure_rows(g4a_kv *kv, int32_t seq, int64_t rows) {
    const int32_t need = (int32_t)((rows + kv->page_tokens - 1) / kv->page_tokens);
    while (kv->seq_pages[seq] < need) {
        if (kv->free_pages.empty())
            return fail(kv->ctx, G4A_OUT_OF_PAGES, "compute: KV page pool exhausted (%d pages)", kv->n_pages);
        const int32_t page = kv->free_pages.back();
        kv->free_pages.pop_back();
        kv->h_bt[(size_t)seq * kv->max_pages + kv->seq_pages[seq]] = page;
        kv->seq_pages[seq]++;
        kv->bt_dirty = true;
    }
    return G4A_OK;
}

int upload_bt(g4a_kv *kv) {
    if (!kv->bt_dirty) return G4A_OK;
    G4A_CUDA_TRY(kv->ctx, upload(kv->ctx, kv->d_bt, kv->h_bt.data(), kv->h_bt.size() * sizeof(int32_t)));
    kv->bt_dirty = false;
    return G4A_OK;
}

// view (context_memory.rs:53-69) checks, for a layer this cache may hold.
int check_view(g4a_kv *kv, int32_t seq, int32_t layer, int64_t want) {
    g4a_ctx *ctx = kv->ctx;
    if (seq < 0 || seq >= kv->n_seqs) return fail(ctx, G4A_COMPUTE, "compute: sequence %d out of range", seq);
    if (layer < 0 || layer >= (int32_t)kv->layers.size() || !kv->layers[layer].held) {
        if (want == 0) return G4A_OK;
        return fail(ctx, G4A_MISSING_LAYER, "layer %d has no cached K/V", layer);
    }
    const int64_t have = kv_len(kv, seq, layer);
    if (want > have)
        return fail(ctx, G4A_CONTEXT_TOO_LONG, "context length %lld exceeds configured max %lld", (long long)want,
                    (long long)have);
    return G4A_OK;
}

}  // namespace

extern "C" int g4a_kv_create(g4a_ctx *ctx, int32_t n_seqs, int32_t max_tokens, int32_t page_tokens, int32_t n_pages,
                             int32_t dtype, const int32_t *layers, int32_t n_layers, g4a_kv **out) {
    if (!ctx || !out) return G4A_COMPUTE;
    *out = nullptr;
    if (n_seqs <= 0 || max_tokens <= 0 || page_tokens <= 0 || n_pages < 0 || (dtype != G4A_KV_F32 && dtype != G4A_KV_F16))
        return fail(ctx, G4A_COMPUTE, "compute: invalid KV cache shape");
    cudaSetDevice(ctx->device);
    const g4a_hparams &hp = ctx->hp;
    auto *kv = new g4a_kv();
    kv->ctx = ctx;
    kv->n_seqs = n_seqs;
    kv->max_tokens = max_tokens;
    kv->page_tokens = page_tokens;
    kv->max_pages = (max_tokens + page_tokens - 1) / page_tokens;
    kv->n_pages = n_pages ? n_pages : n_seqs * kv->max_pages;
    kv->dtype = dtype;
    kv->elem = dtype == G4A_KV_F16 ? 2 : 4;
    kv->layers.resize(hp.n_layers);
    std::vector<int32_t> want;
    if (layers) {
        want.assign(layers, layers + n_layers);
    } else {
        for (int32_t l = 0; l < hp.n_layers; l++) {
            int32_t src = -1;
            if (g4a_kv_source_layer(&hp, l, &src, nullptr) == G4A_OK && src == l) want.push_back(l);
        }
    }
    for (int32_t l : want) {
        int32_t src = -1;
        if (g4a_kv_source_layer(&hp, l, &src, nullptr) != G4A_OK || src != l) {
            delete kv;
            return fail(ctx, G4A_BAD_LAYER, "layer %d does not own a K/V cache", l);
        }
        auto &L = kv->layers[l];
        if (L.held) continue;
        L.held = true;
        L.hd = g4a_head_dim(&hp, l) * hp.n_kv_heads;
        const size_t bytes = (size_t)kv->n_pages * page_tokens * L.hd * kv->elem;
        if (cudaMalloc(&L.k, bytes) != cudaSuccess || cudaMalloc(&L.v, bytes) != cudaSuccess) {
            g4a_kv_destroy(kv);
            return fail(ctx, G4A_CUDA, "compute: out of device memory for the KV cache");
        }
        // rows never written stay finite (zero), so masked rows cannot turn into NaN
        cudaMemset(L.k, 0, bytes);
        cudaMemset(L.v, 0, bytes);
    }
    if (dtype == G4A_KV_F16) {
        // TMA descriptors of each held layer's pools: [n_pages * page_tokens][hd] f16,
        // boxes of 64 columns x one decode stage of rows.
        std::vector<uint8_t> maps((size_t)hp.n_layers * 2 * 128, 0);
        bool ok = page_tokens % 64 == 0;
        for (int32_t l = 0; l < hp.n_layers && ok; l++) {
            const auto &L = kv->layers[l];
            if (!L.held) continue;
            if (L.hd != 256 && L.hd != 512) continue;
            const uint64_t rows = (uint64_t)kv->n_pages * page_tokens;
            const uint32_t box = (uint32_t)f16_stage_rows(L.hd);
            ok = encode_tmap_2d(maps.data() + (size_t)l * 256, 1, L.k, L.hd, rows, box) &&
                 encode_tmap_2d(maps.data() + (size_t)l * 256 + 128, 1, L.v, L.hd, rows, box);
        }
        if (ok && cudaMalloc(&kv->d_tmaps, maps.size()) == cudaSuccess &&
            cudaMemcpy(kv->d_tmaps, maps.data(), maps.size(), cudaMemcpyHostToDevice) == cudaSuccess) {
        } else if (page_tokens % 64 == 0) {
            g4a_kv_destroy(kv);
            return fail(ctx, G4A_CUDA, "compute: TMA descriptors for the KV cache could not be created");
        }
    }
    kv->h_bt.assign((size_t)n_seqs * kv->max_pages, -1);
    kv->len.assign((size_t)n_seqs * hp.n_layers, 0);
    kv->seq_pages.assign(n_seqs, 0);
    kv->free_pages.resize(kv->n_pages);
    for (int32_t i = 0; i < kv->n_pages; i++) kv->free_pages[i] = kv->n_pages - 1 - i;  // pop gives 0, 1, ...
    if (cudaMalloc(&kv->d_bt, kv->h_bt.size() * sizeof(int32_t)) != cudaSuccess) {
        g4a_kv_destroy(kv);
        return fail(ctx, G4A_CUDA, "compute: out of device memory for the block table");
    }
    *out = kv;
    return G4A_OK;
}

extern "C" void g4a_kv_destroy(g4a_kv *kv) {
    if (!kv) return;
    cudaSetDevice(kv->ctx->device);
    cudaStreamSynchronize(kv->ctx->stream);
    for (auto &L : kv->layers) {
        cudaFree(L.k);
        cudaFree(L.v);
    }
    cudaFree(kv->d_bt);
    cudaFree(kv->d_tmaps);
    delete kv;
}

extern "C" int g4a_kv_clear(g4a_kv *kv, int32_t seq) {
    if (!kv) return G4A_COMPUTE;
    const int32_t lo = seq < 0 ? 0 : seq, hi = seq < 0 ? kv->n_seqs : seq + 1;
    if (seq >= kv->n_seqs) return fail(kv->ctx, G4A_COMPUTE, "compute: sequence %d out of range", seq);
    for (int32_t s = lo; s < hi; s++) {
        for (int32_t j = 0; j < kv->seq_pages[s]; j++) {
            int32_t &e = kv->h_bt[(size_t)s * kv->max_pages + j];
            kv->free_pages.push_back(e);
            e = -1;
        }
        kv->seq_pages[s] = 0;
        for (size_t l = 0; l < kv->layers.size(); l++) kv_len(kv, s, (int32_t)l) = 0;
    }
    kv->bt_dirty = true;
    return G4A_OK;
}

extern "C" int g4a_kv_len(const g4a_kv *kv, int32_t seq, int32_t layer, int64_t *len) {
    if (!kv || !len || seq < 0 || seq >= kv->n_seqs || layer < 0 || layer >= (int32_t)kv->layers.size())
        return G4A_COMPUTE;
    *len = kv->len[(size_t)seq * kv->layers.size() + layer];
    return G4A_OK;
}

namespace {

int append_impl(g4a_kv *kv, int32_t seq, int32_t layer, const float *k, const float *v, const float *k_w,
                int64_t n, bool raw) {
    g4a_ctx *ctx = kv->ctx;
    cudaSetDevice(ctx->device);
    if (seq < 0 || seq >= kv->n_seqs) return fail(ctx, G4A_COMPUTE, "compute: sequence %d out of range", seq);
    if (layer < 0 || layer >= (int32_t)kv->layers.size() || !kv->layers[layer].held)
        return fail(ctx, G4A_MISSING_LAYER, "layer %d has no cached K/V", layer);
    if (n < 0 || (n > 0 && (!k || !v))) return fail(ctx, G4A_COMPUTE, "compute: invalid append rows");
    if (raw && !k_w) return fail(ctx, G4A_MISSING_WEIGHT, "missing weight `blk.%d.attn_k_norm.weight`", layer);
    const auto &L = kv->layers[layer];
    if (raw && L.hd != 256 && L.hd != 512)
        return fail(ctx, G4A_COMPUTE, "compute: fused norm/RoPE append needs head width 256 or 512");
    int64_t &len = kv_len(kv, seq, layer);
    if (len + n > kv->max_tokens)
        return fail(ctx, G4A_CONTEXT_TOO_LONG, "context length %lld exceeds configured max %d", (long long)(len + n),
                    kv->max_tokens);
    if (raw && len + n > ctx->max_positions)
        return fail(ctx, G4A_CONTEXT_TOO_LONG, "context length %lld exceeds configured max %d", (long long)(len + n),
                    ctx->max_positions);
    int rc = ensure_rows(kv, seq, len + n);
    if (rc) return rc;
    if ((rc = upload_bt(kv))) return rc;
    AppendParams p{};
    p.k_pool = L.k;
    p.v_pool = L.v;
    p.block_table = kv->d_bt + (size_t)seq * kv->max_pages;
    p.k_src = k;
    p.v_src = v;
    p.k_w = k_w;
    const bool global = g4a_layer_is_global(&ctx->hp, layer);
    p.rope = global ? ctx->d_rope_global : ctx->d_rope_local;
    p.hd = L.hd;
    p.page_tokens = kv->page_tokens;
    p.first_row = (int32_t)len;
    p.first_pos = (int32_t)len;
    p.n_rows = (int32_t)n;
    p.raw = raw;
    p.eps = ctx->hp.rms_norm_eps;
    G4A_CUDA_TRY(ctx, launch_append(p, kv->dtype == G4A_KV_F16, ctx->stream));
    len += n;
    return G4A_OK;
}

}  // namespace

extern "C" int g4a_kv_append(g4a_kv *kv, int32_t seq, int32_t layer, const float *k, const float *v, int64_t n) {
    if (!kv) return G4A_COMPUTE;
    return append_impl(kv, seq, layer, k, v, nullptr, n, false);
}

extern "C" int g4a_kv_append_tokens(g4a_kv *kv, int32_t seq, int32_t layer, const float *k_raw, const float *v_raw,
                                    const float *k_w, int64_t n) {
    if (!kv) return G4A_COMPUTE;
    return append_impl(kv, seq, layer, k_raw, v_raw, k_w, n, true);
}

extern "C" int g4a_kv_view(const g4a_kv *kv_c, int32_t seq, int32_t layer, int64_t len, float *k_out, float *v_out) {
    if (!kv_c) return G4A_COMPUTE;
    auto *kv = const_cast<g4a_kv *>(kv_c);
    g4a_ctx *ctx = kv->ctx;
    cudaSetDevice(ctx->device);
    int rc = check_view(kv, seq, layer, len);
    if (rc || len == 0) return rc;
    if (!k_out || !v_out) return fail(ctx, G4A_COMPUTE, "compute: null view output");
    if ((rc = upload_bt(kv))) return rc;
    ViewParams p{};
    p.k_pool = kv->layers[layer].k;
    p.v_pool = kv->layers[layer].v;
    p.block_table = kv->d_bt + (size_t)seq * kv->max_pages;
    p.k_out = k_out;
    p.v_out = v_out;
    p.hd = kv->layers[layer].hd;
    p.page_tokens = kv->page_tokens;
    p.n_rows = (int32_t)len;
    G4A_CUDA_TRY(ctx, launch_view(p, kv->dtype == G4A_KV_F16, ctx->stream));
    return G4A_OK;
}

// --------------------------------------------------------------------------
// decode
// --------------------------------------------------------------------------

namespace {

struct Plan {
    std::vector<DecodeTask> tasks;
    std::vector<DecodeItem> items[2];  // by head width: [0] 256, [1] 512
    int32_t slots = 0;
    bool f16_fast = false;             // f16 paged cache: the TMA / tensor-core kernel
    std::vector<int32_t> cta_start;    // f16 kernel: per-CTA item ranges (items[0] holds all items)
    // assign_ctas scratch
    std::vector<DecodeItem> all;
    std::vector<uint64_t> keys, keys_tmp, heap;
    std::vector<int32_t> cta_of, fill;
    void clear() {
        tasks.clear();
        items[0].clear();
        items[1].clear();
        slots = 0;
        f16_fast = false;
        cta_start.clear();
    }
};

// A plan per thread, its vectors' capacity kept from call to call (a call
// plans about a hundred tasks and several hundred items; allocating them
// anew cost more than the planning).
Plan &scratch_plan() {
    static thread_local Plan plan;
    plan.clear();
    return plan;
}

// Rows per work item. Aims at about two items per SM over the whole call,
// weighting rows by head width, with at least 64 rows per item: the last CTA
// of a split task merges every partial alone, so a small call (one sequence of
// a few hundred rows) is faster with a few long items than with many short
// ones.
int32_t rows_per_item(int64_t weighted_total, int32_t weight) {
    const int64_t target_items = 2 * 148;
    int64_t w = (weighted_total + target_items - 1) / target_items;
    int64_t rows = (w + weight - 1) / weight;
    rows = std::max<int64_t>(64, (rows + 15) / 16 * 16);
    return (int32_t)std::min<int64_t>(rows, 1 << 20);
}

void add_items(Plan &plan, DecodeTask &t, int32_t task_index, int32_t rows_per, int which) {
    const int32_t n_rows = t.hi - t.lo;
    const int32_t n = std::max<int32_t>(1, (n_rows + rows_per - 1) / rows_per);
    t.n_splits = n;
    t.partial_base = n > 1 ? plan.slots : 0;
    if (n > 1) plan.slots += n;
    for (int32_t s = 0; s < n; s++) {
        DecodeItem it;
        it.task = task_index;
        it.split = s;
        it.row_lo = t.lo + (int32_t)((int64_t)n_rows * s / n);
        it.row_hi = t.lo + (int32_t)((int64_t)n_rows * (s + 1) / n);
        plan.items[which].push_back(it);
    }
}

// Device-side form of a plan: metadata, split-KV partials and tickets, and
// the kernel parameters of the two head-width launches.
struct Staged {
    uint8_t *meta = nullptr;
    float *part_o = nullptr;
    float *part_ml = nullptr;
    unsigned *tickets = nullptr;
    DecodeParams params{};
    int32_t n_items[2] = {0, 0};
    size_t items_offset = 0;
    int kv_f16 = 0;
    bool f16_fast = false;
    int32_t n_ctas = 0;
    int32_t n_tasks = 0;
    int32_t n_split_tasks = 0;
    uint8_t *q_blocks = nullptr;  // f16 kernel scratch
    bool own = false;             // buffers of this plan alone
    uint32_t ticket_epoch = 0;    // the context's error count when the tickets were last clear
};

// Copies a plan's metadata to the device. With own_buffers the buffers are
// allocated for this plan alone; otherwise the context's reusable ones are
// grown as needed.
int stage_plan(g4a_ctx *ctx, const Plan &plan, const int32_t *d_bt, int32_t max_pages, int32_t page_tokens,
               int kv_f16, bool own_buffers, Staged *st) {
    const size_t n_tasks = plan.tasks.size();
    const size_t n_items = plan.items[0].size() + plan.items[1].size();
    const size_t bytes_tasks = n_tasks * sizeof(DecodeTask);
    const size_t bytes_items = n_items * sizeof(DecodeItem);
    std::vector<int32_t> split_tasks;
    if (plan.f16_fast)
        for (size_t i = 0; i < n_tasks; i++)
            if (plan.tasks[i].n_splits > 1) split_tasks.push_back((int32_t)i);
    const size_t bytes_cta = plan.cta_start.size() * sizeof(int32_t);
    const size_t bytes = bytes_tasks + bytes_items + bytes_cta + split_tasks.size() * sizeof(int32_t);
    const size_t n_qb = plan.f16_fast ? std::max<size_t>(n_tasks, 1) * kQBlockBytes : 0;
    const size_t n_po = (size_t)std::max(plan.slots, 1) * kHeads * 512;
    const size_t n_ml = (size_t)std::max(plan.slots, 1) * 2 * kHeads;
    const size_t n_tk = std::max<size_t>(n_tasks, 1);
    int rc;
    if (own_buffers) {
        if (n_qb) G4A_CUDA_TRY(ctx, cudaMalloc(&st->q_blocks, n_qb));
        G4A_CUDA_TRY(ctx, cudaMalloc(&st->meta, std::max<size_t>(bytes, 16)));
        G4A_CUDA_TRY(ctx, cudaMalloc(&st->part_o, n_po * sizeof(float)));
        G4A_CUDA_TRY(ctx, cudaMalloc(&st->part_ml, n_ml * sizeof(float)));
        G4A_CUDA_TRY(ctx, cudaMalloc(&st->tickets, n_tk * sizeof(unsigned)));
        G4A_CUDA_TRY(ctx, cudaMemsetAsync(st->tickets, 0, n_tk * sizeof(unsigned), ctx->stream));
        st->own = true;
        st->ticket_epoch = ctx->err_epoch;
    } else {
        if ((rc = grow(ctx, &ctx->d_meta, &ctx->meta_cap, bytes, false))) return rc;
        if ((rc = grow(ctx, &ctx->d_part_o, &ctx->part_o_cap, n_po, false))) return rc;
        if ((rc = grow(ctx, &ctx->d_part_ml, &ctx->part_ml_cap, n_ml, false))) return rc;
        if ((rc = grow(ctx, &ctx->d_tickets, &ctx->tickets_cap, n_tk, true))) return rc;
        if (ctx->tickets_epoch != ctx->err_epoch) {  // an aborted step may have left counts
            G4A_CUDA_TRY(ctx, cudaMemsetAsync(ctx->d_tickets, 0, ctx->tickets_cap * sizeof(unsigned), ctx->stream));
            ctx->tickets_epoch = ctx->err_epoch;
        }
        if (n_qb && (rc = grow(ctx, &ctx->d_qblocks, &ctx->qblocks_cap, n_qb, false))) return rc;
        st->q_blocks = ctx->d_qblocks;
        st->meta = ctx->d_meta;
        st->part_o = ctx->d_part_o;
        st->part_ml = ctx->d_part_ml;
        st->tickets = ctx->d_tickets;
    }
    ctx->h_meta.resize(std::max<size_t>(bytes, 1));
    std::memcpy(ctx->h_meta.data(), plan.tasks.data(), bytes_tasks);
    std::memcpy(ctx->h_meta.data() + bytes_tasks, plan.items[0].data(), plan.items[0].size() * sizeof(DecodeItem));
    std::memcpy(ctx->h_meta.data() + bytes_tasks + plan.items[0].size() * sizeof(DecodeItem), plan.items[1].data(),
                plan.items[1].size() * sizeof(DecodeItem));
    if (!plan.cta_start.empty())
        std::memcpy(ctx->h_meta.data() + bytes_tasks + bytes_items, plan.cta_start.data(), bytes_cta);
    if (!split_tasks.empty())
        std::memcpy(ctx->h_meta.data() + bytes_tasks + bytes_items + bytes_cta, split_tasks.data(),
                    split_tasks.size() * sizeof(int32_t));
    G4A_CUDA_TRY(ctx, upload(ctx, st->meta, ctx->h_meta.data(), bytes));
    DecodeParams &p = st->params;
    p = DecodeParams{};
    p.tasks = reinterpret_cast<const DecodeTask *>(st->meta);
    p.block_table = d_bt;
    p.max_pages = max_pages;
    p.page_tokens = page_tokens;
    p.rope_local = ctx->d_rope_local;
    p.rope_global = ctx->d_rope_global;
    p.eps = ctx->hp.rms_norm_eps;
    p.part_o = st->part_o;
    p.part_ml = st->part_ml;
    p.tickets = st->tickets;
    p.err_flag = ctx->d_err;
    st->n_items[0] = (int32_t)plan.items[0].size();
    st->n_items[1] = (int32_t)plan.items[1].size();
    st->items_offset = bytes_tasks;
    st->kv_f16 = kv_f16;
    st->f16_fast = plan.f16_fast;
    p.cta_start = plan.cta_start.empty()
                      ? nullptr
                      : reinterpret_cast<const int32_t *>(st->meta + bytes_tasks + bytes_items);
    st->n_ctas = plan.cta_start.empty() ? 0 : (int32_t)plan.cta_start.size() - 1;
    p.q_blocks = st->q_blocks;
    p.split_tasks = reinterpret_cast<const int32_t *>(st->meta + bytes_tasks + bytes_items + bytes_cta);
    st->n_tasks = (int32_t)n_tasks;
    st->n_split_tasks = (int32_t)split_tasks.size();
    return G4A_OK;
}

int launch_staged(g4a_ctx *ctx, Staged &st) {
    if (st.own && st.ticket_epoch != ctx->err_epoch) {  // an aborted step may have left counts
        G4A_CUDA_TRY(ctx, cudaMemsetAsync(st.tickets, 0, std::max<size_t>(st.n_tasks, 1) * sizeof(unsigned), ctx->stream));
        st.ticket_epoch = ctx->err_epoch;
    }
    DecodeParams p = st.params;
    if (st.f16_fast && (ctx->stall_mask & (1u << G4A_K_DECODE_MAIN))) {
        p.stall = 1;
        ctx->stall_mask &= ~(1u << G4A_K_DECODE_MAIN);
    }
    const DecodeItem *items = reinterpret_cast<const DecodeItem *>(st.meta + st.items_offset);
    if (st.f16_fast) {  // both head widths in one launch
        p.items = items;
        p.n_items = st.n_items[0] + st.n_items[1];
        G4A_CUDA_TRY(ctx, timed(ctx, G4A_K_DECODE_PREP, [&] { return launch_decode_f16(p, 0, st.n_tasks, ctx->stream); }));
        G4A_CUDA_TRY(ctx, timed(ctx, G4A_K_DECODE_MAIN, [&] { return launch_decode_f16(p, 1, st.n_ctas, ctx->stream); }));
        G4A_CUDA_TRY(ctx,
                     timed(ctx, G4A_K_DECODE_COMBINE, [&] { return launch_decode_f16(p, 2, st.n_split_tasks, ctx->stream); }));
        return G4A_OK;
    }
    for (int which = 0; which < 2; which++) {
        p.items = items;
        p.n_items = st.n_items[which];
        G4A_CUDA_TRY(ctx, timed(ctx, G4A_K_DECODE_SPLITKV,
                                [&] { return launch_decode(p, which ? 512 : 256, st.kv_f16, true, ctx->stream); }));
        items += st.n_items[which];
    }
    return G4A_OK;
}

// Splits for the f16 kernel: boundaries at absolute multiples of rows_per (a
// multiple of 64, so items start on stage boundaries), at most
// kF16MaxSplits items per task.
void add_items_aligned(Plan &plan, DecodeTask &t, int32_t task_index, int32_t rows_per, int which) {
    const int32_t n_rows = t.hi - t.lo;
    int64_t rp = std::max<int64_t>(rows_per, 64);
    rp = std::max<int64_t>(rp, (n_rows + kF16MaxSplits - 2) / (kF16MaxSplits - 1));  // +1 for the unaligned start
    rp = (rp + 63) / 64 * 64;
    // cuts: lo, then every multiple of rp above lo and below hi, then hi
    const int64_t first = ((int64_t)t.lo / rp + 1) * rp;
    const int32_t n = 1 + (first < t.hi ? (int32_t)((t.hi - 1 - first) / rp + 1) : 0);
    t.n_splits = n;
    t.partial_base = n > 1 ? plan.slots : 0;
    if (n > 1) plan.slots += n;
    int32_t a = t.lo;
    for (int32_t s = 0; s < n; s++) {
        const int32_t b = s + 1 < n ? (int32_t)(first + (int64_t)s * rp) : t.hi;
        plan.items[which].push_back(DecodeItem{task_index, s, a, b});
        a = b;
    }
}

// Longest-processing-time assignment of the f16 kernel's items to persistent
// CTAs: cost = K/V bytes of the rows (in units of a 256-wide row) plus a fixed
// per-item charge for the q preparation and, for split tasks, the partial
// write. Items are taken longest first (ties in list order), each to the
// least loaded CTA (ties to the lower index), then stored CTA by CTA, in
// the order they were assigned, with a start table.
void assign_ctas(Plan &plan, int n_sm) {
    std::vector<DecodeItem> &all = plan.all;
    all.assign(plan.items[0].begin(), plan.items[0].end());
    all.insert(all.end(), plan.items[1].begin(), plan.items[1].end());
    plan.items[0].clear();
    plan.items[1].clear();
    const size_t n = all.size();
    // (~cost, position) packed: an ascending sort is longest first, stable
    std::vector<uint64_t> &keys = plan.keys;
    keys.resize(n);
    uint64_t max_cost = 0;
    for (size_t i = 0; i < n; i++) {
        const DecodeItem &it = all[i];
        const DecodeTask &t = plan.tasks[it.task];
        const uint64_t cost = (uint64_t)((int64_t)(it.row_hi - it.row_lo) * (t.hd / 256) + 64 + (t.n_splits > 1 ? 32 : 0));
        keys[i] = ((~cost & 0xFFFFFFFFFFull) << 24) | (uint64_t)i;
        max_cost = std::max(max_cost, cost);
    }
    if (max_cost < (1u << 16)) {
        // the same order by a stable radix sort of 65535 - cost (two 8-bit
        // passes), the keys being in position order to begin with
        std::vector<uint64_t> &tmp = plan.keys_tmp;
        tmp.resize(n);
        for (int pass = 0; pass < 2; pass++) {
            auto digit = [pass](uint64_t key) {
                const uint32_t cost = (uint32_t)(~(key >> 24) & 0xFFFFFFFFFFull);
                return ((65535u - cost) >> (8 * pass)) & 255u;
            };
            uint32_t start[257] = {};
            for (const uint64_t key : keys) start[digit(key) + 1]++;
            for (int d = 0; d < 256; d++) start[d + 1] += start[d];
            for (const uint64_t key : keys) tmp[start[digit(key)]++] = key;
            keys.swap(tmp);
        }
    } else {
        std::sort(keys.begin(), keys.end());
    }
    const int n_ctas = std::max(1, std::min<int>(n_sm, (int)n));
    // min-heap of (load, cta) packed. The first n_ctas items meet empty CTAs
    // (every cost is positive), so item j goes to CTA j; the heap starts after.
    std::vector<uint64_t> &heap = plan.heap;
    heap.resize(n_ctas);
    std::vector<int32_t> &cta_of = plan.cta_of;
    cta_of.resize(n);
    plan.cta_start.assign(n_ctas + 1, 0);
    const size_t head = std::min<size_t>(n, (size_t)n_ctas);
    for (size_t j = 0; j < head; j++) {
        const uint64_t cost = ~(keys[j] >> 24) & 0xFFFFFFFFFFull;
        heap[j] = (cost << 24) | (uint64_t)j;
        cta_of[j] = (int32_t)j;
        plan.cta_start[j + 1]++;
    }
    std::make_heap(heap.begin(), heap.end(), std::greater<uint64_t>());
    for (size_t j = head; j < n; j++) {
        const uint64_t cost = ~(keys[j] >> 24) & 0xFFFFFFFFFFull;
        std::pop_heap(heap.begin(), heap.end(), std::greater<uint64_t>());
        const int b = (int)(heap.back() & 0xFFFFFFull);
        heap.back() += cost << 24;
        std::push_heap(heap.begin(), heap.end(), std::greater<uint64_t>());
        cta_of[j] = b;
        plan.cta_start[b + 1]++;
    }
    for (int b = 0; b < n_ctas; b++) plan.cta_start[b + 1] += plan.cta_start[b];
    std::vector<int32_t> &fill = plan.fill;
    fill.assign(plan.cta_start.begin(), plan.cta_start.end() - 1);
    plan.items[0].resize(n);
    for (size_t j = 0; j < n; j++) plan.items[0][fill[cta_of[j]]++] = all[keys[j] & 0xFFFFFFull];
}

int run_plan(g4a_ctx *ctx, Plan &plan, const int32_t *d_bt, int32_t max_pages, int32_t page_tokens, int kv_f16) {
    Staged st;
    int rc = stage_plan(ctx, plan, d_bt, max_pages, page_tokens, kv_f16, false, &st);
    if (rc) return rc;
    return launch_staged(ctx, st);
}

}  // namespace

extern "C" int g4a_attend(g4a_ctx *ctx, const float *q, const float *keys, const float *values, int64_t len,
                          int32_t n_heads, int32_t n_kv, int32_t hd, float scale, float *out) {
    if (!ctx) return G4A_COMPUTE;
    cudaSetDevice(ctx->device);
    if (n_heads <= 0 || n_kv <= 0 || hd <= 0 || n_heads % n_kv != 0 || len < 0 || !q || !out)
        return fail(ctx, G4A_COMPUTE, "compute: invalid attention shape");
    if (len == 0) return fail(ctx, G4A_NONFINITE, "compute: softmax input is not finite");  // model.rs:337,362-364
    if (!keys || !values) return fail(ctx, G4A_COMPUTE, "compute: null keys or values");
    if (n_heads == kHeads && n_kv == 1 && (hd == 256 || hd == 512) && len < (1LL << 31)) {
        Plan &plan = scratch_plan();
        DecodeTask t{};
        t.k_base = keys;
        t.v_base = values;
        t.q_raw = q;
        t.out = out;
        t.lo = 0;
        t.hi = (int32_t)len;
        t.new_row = -1;
        t.q_ready = 1;
        t.scale = scale;
        const int which = hd == 512;
        add_items(plan, t, 0, rows_per_item(len * (hd / 256), hd / 256), which);
        plan.tasks.push_back(t);
        return run_plan(ctx, plan, nullptr, 0, 1, 0);
    }
    if (hd > 1024) return fail(ctx, G4A_COMPUTE, "compute: head width %d above 1024", hd);
    G4A_CUDA_TRY(ctx, launch_attend_generic(q, keys, values, len, n_heads, n_kv, hd, scale, out, ctx->d_err, ctx->stream));
    return G4A_OK;
}

namespace {

// Per-layer facts of a decode step, found by check_decode.
struct DecodeLayers {
    std::vector<int32_t> src, hd;
    std::vector<char> owner, global;
};

// Validates one decode step (model.rs:389-399, context_memory.rs:53-69) and
// allocates the pages its appends need; changes no cache length.
int check_decode(g4a_ctx *ctx, g4a_kv *kv, int32_t n_layers, const g4a_decode_layer *layers, int32_t n_seqs,
                 const int32_t *seq_ids, const int32_t *positions, DecodeLayers &info) {
    if (!ctx || !kv || kv->ctx != ctx) return fail(ctx, G4A_COMPUTE, "compute: cache belongs to another context");
    cudaSetDevice(ctx->device);
    const g4a_hparams &hp = ctx->hp;
    if (n_layers < 0 || n_seqs < 0 || (n_layers > 0 && !layers) || (n_seqs > 0 && (!seq_ids || !positions)))
        return fail(ctx, G4A_COMPUTE, "compute: invalid decode arguments");
    if (hp.n_heads != kHeads || hp.n_kv_heads != 1)
        return fail(ctx, G4A_COMPUTE, "compute: fused decode serves %d query heads over 1 KV head", kHeads);
    // ---- validate layers (model.rs:389-399) ----
    info.src.assign(n_layers, 0);
    info.hd.assign(n_layers, 0);
    info.owner.assign(n_layers, 0);
    info.global.assign(n_layers, 0);
    std::vector<int32_t> &src = info.src, &hd = info.hd;
    std::vector<char> &owner = info.owner, &global = info.global;
    for (int32_t i = 0; i < n_layers; i++) {
        const g4a_decode_layer &a = layers[i];
        int32_t detail = 0;
        if (g4a_kv_source_layer(&hp, a.layer, &src[i], &detail) != G4A_OK)
            return fail(ctx, G4A_BAD_LAYER, "compute: layer %d has no KV source (kind %d)", a.layer, detail);
        owner[i] = src[i] == a.layer;
        global[i] = (char)g4a_layer_is_global(&hp, a.layer);
        hd[i] = g4a_head_dim(&hp, a.layer);
        if (hd[i] != 256 && hd[i] != 512) return fail(ctx, G4A_COMPUTE, "compute: head width %d unsupported", hd[i]);
        if (!a.q_raw_dev || !a.out_dev) return fail(ctx, G4A_COMPUTE, "compute: null q or output");
        if (!a.q_norm_w_dev) return fail(ctx, G4A_MISSING_WEIGHT, "missing weight `blk.%d.attn_q_norm.weight`", a.layer);
        if (owner[i] && (!a.k_raw_dev || !a.v_raw_dev))
            return fail(ctx, G4A_COMPUTE, "compute: layer %d owns its cache and needs k and v", a.layer);
        if (owner[i] && !a.k_norm_w_dev)
            return fail(ctx, G4A_MISSING_WEIGHT, "missing weight `blk.%d.attn_k_norm.weight`", a.layer);
        if (src[i] >= (int32_t)kv->layers.size() || !kv->layers[src[i]].held)
            return fail(ctx, G4A_MISSING_LAYER, "layer %d has no cached K/V", src[i]);
        for (int32_t j = 0; j < n_layers; j++)
            if (j != i && (layers[j].layer == a.layer || (!owner[i] && layers[j].layer == src[i])))
                return fail(ctx, G4A_COMPUTE, "compute: layer %d listed with itself or its KV source", a.layer);
    }
    // ---- validate sequences and positions (context_memory.rs:53-69) ----
    std::vector<char> seen(kv->n_seqs, 0);
    for (int32_t j = 0; j < n_seqs; j++) {
        const int32_t s = seq_ids[j];
        if (s < 0 || s >= kv->n_seqs) return fail(ctx, G4A_COMPUTE, "compute: sequence %d out of range", s);
        if (seen[s]) return fail(ctx, G4A_COMPUTE, "compute: sequence %d listed twice", s);
        seen[s] = 1;
        const int64_t pos = positions[j];
        if (pos < 0) return fail(ctx, G4A_COMPUTE, "compute: negative position");
        if (pos >= ctx->max_positions)
            return fail(ctx, G4A_CONTEXT_TOO_LONG, "context length %lld exceeds configured max %d", (long long)pos + 1,
                        ctx->max_positions);
        for (int32_t i = 0; i < n_layers; i++) {
            if (owner[i]) {
                const int64_t new_row = kv_len(kv, s, layers[i].layer);
                if (new_row + 1 > kv->max_tokens)
                    return fail(ctx, G4A_CONTEXT_TOO_LONG, "context length %lld exceeds configured max %d",
                                (long long)new_row + 1, kv->max_tokens);
                if (pos + 1 > new_row + 1)
                    return fail(ctx, G4A_CONTEXT_TOO_LONG, "context length %lld exceeds configured max %lld",
                                (long long)pos + 1, (long long)new_row + 1);
            } else {
                int rc = check_view(kv, s, src[i], pos + 1);
                if (rc) return rc;
            }
        }
    }
    // ---- allocate rows for the appends, then plan ----
    for (int32_t j = 0; j < n_seqs; j++)
        for (int32_t i = 0; i < n_layers; i++)
            if (owner[i]) {
                int rc = ensure_rows(kv, seq_ids[j], kv_len(kv, seq_ids[j], layers[i].layer) + 1);
                if (rc) return rc;
            }
    return upload_bt(kv);
}

// Fills `plan` with the tasks of layers [first, first + count) of a checked
// step: one task per (sequence, layer), its rows cut into work items.
void plan_decode(g4a_ctx *ctx, g4a_kv *kv, const g4a_decode_layer *layers, int32_t n_seqs, const int32_t *seq_ids,
                 const int32_t *positions, const DecodeLayers &info, int32_t first, int32_t count, Plan &plan) {
    const g4a_hparams &hp = ctx->hp;
    const std::vector<int32_t> &src = info.src, &hd = info.hd;
    const std::vector<char> &owner = info.owner, &global = info.global;
    int64_t weighted = 0;
    for (int32_t i = first; i < first + count; i++)
        for (int32_t j = 0; j < n_seqs; j++) {
            int64_t lo, hi;
            if (global[i]) lo = 0, hi = (int64_t)positions[j] + 1;
            else g4a_windowed_len((int64_t)positions[j] + 1, hp.sliding_window, &lo, &hi);
            weighted += (hi - lo) * (hd[i] / 256);
        }
    plan.f16_fast = kv->dtype == G4A_KV_F16 && kv->d_tmaps != nullptr;
    // f16 kernel: about three items per SM over the whole call, by K/V bytes
    const int64_t weighted_all = weighted;
    // (measured on configuration 2: 2, 4, 6 and 8 items per SM were 1-15 % slower)
    const int64_t item_weight = std::max<int64_t>(64, (weighted_all + 3 * ctx->n_sm - 1) / (3 * ctx->n_sm));
    for (int32_t i = first; i < first + count; i++) {
        const g4a_decode_layer &a = layers[i];
        const auto &L = kv->layers[src[i]];
        const int which = hd[i] == 512;
        const int32_t rows_per = rows_per_item(weighted, hd[i] / 256);
        for (int32_t j = 0; j < n_seqs; j++) {
            const int32_t s = seq_ids[j];
            DecodeTask t{};
            t.k_base = L.k;
            t.v_base = L.v;
            const size_t qw = (size_t)kHeads * hd[i];
            t.q_raw = a.q_raw_dev + (size_t)j * qw;
            t.k_raw = owner[i] ? a.k_raw_dev + (size_t)j * hd[i] : nullptr;
            t.v_raw = owner[i] ? a.v_raw_dev + (size_t)j * hd[i] : nullptr;
            t.q_w = a.q_norm_w_dev;
            t.k_w = a.k_norm_w_dev;
            t.out = a.out_dev + (size_t)j * qw;
            t.seq = s;
            t.position = positions[j];
            int64_t lo, hi;
            if (global[i]) lo = 0, hi = (int64_t)positions[j] + 1;
            else g4a_windowed_len((int64_t)positions[j] + 1, hp.sliding_window, &lo, &hi);
            t.lo = (int32_t)lo;
            t.hi = (int32_t)hi;
            t.new_row = owner[i] ? (int32_t)kv_len(kv, s, a.layer) : -1;
            t.global = global[i];
            t.q_ready = 0;
            t.scale = 1.0f;
            t.hd = hd[i];
            if (plan.f16_fast) {
                t.tmap_k = kv->d_tmaps + (size_t)src[i] * 256;
                t.tmap_v = kv->d_tmaps + (size_t)src[i] * 256 + 128;
                add_items_aligned(plan, t, (int32_t)plan.tasks.size(), (int32_t)(item_weight / (hd[i] / 256)), which);
            } else {
                add_items(plan, t, (int32_t)plan.tasks.size(), rows_per, which);
            }
            plan.tasks.push_back(t);
        }
    }
    if (plan.f16_fast) assign_ctas(plan, ctx->n_sm);
}

// The appended rows of a planned step count as stored (context_memory.rs:44-51).
void commit_decode(g4a_kv *kv, int32_t n_layers, const g4a_decode_layer *layers, int32_t n_seqs,
                   const int32_t *seq_ids, const DecodeLayers &info) {
    for (int32_t i = 0; i < n_layers; i++)
        if (info.owner[i])
            for (int32_t j = 0; j < n_seqs; j++) kv_len(kv, seq_ids[j], layers[i].layer) += 1;
}

// Validates one decode step, allocates the pages its appends need, advances
// the cache lengths and fills `plan` (model.rs:393-410 per sequence and layer).
int build_decode(g4a_ctx *ctx, g4a_kv *kv, int32_t n_layers, const g4a_decode_layer *layers, int32_t n_seqs,
                 const int32_t *seq_ids, const int32_t *positions, Plan &plan) {
    DecodeLayers info;
    const int rc = check_decode(ctx, kv, n_layers, layers, n_seqs, seq_ids, positions, info);
    if (rc) return rc;
    plan_decode(ctx, kv, layers, n_seqs, seq_ids, positions, info, 0, n_layers, plan);
    commit_decode(kv, n_layers, layers, n_seqs, seq_ids, info);
    return G4A_OK;
}

}  // namespace

extern "C" int g4a_decode(g4a_ctx *ctx, g4a_kv *kv, int32_t n_layers, const g4a_decode_layer *layers, int32_t n_seqs,
                          const int32_t *seq_ids, const int32_t *positions) {
    Plan &plan = scratch_plan();
    int rc = build_decode(ctx, kv, n_layers, layers, n_seqs, seq_ids, positions, plan);
    if (rc) return rc;
    return run_plan(ctx, plan, kv->d_bt, kv->max_pages, kv->page_tokens, kv->dtype == G4A_KV_F16);
}

namespace {

// Event from the context's spare list (profiling records).
cudaEvent_t spare_event(g4a_ctx *ctx) {
    cudaEvent_t e = nullptr;
    if (!ctx->spare.empty()) {
        e = ctx->spare.back();
        ctx->spare.pop_back();
    } else {
        cudaEventCreate(&e);
    }
    return e;
}

}  // namespace

namespace {

constexpr size_t kInPlaceMaxBytes = 256 * 1024;  // host-buffer steps up to this size run in place

// The device-side address of page-locked host memory the device can reach
// (cudaHostAlloc'd or registered memory under unified addressing), or false
// for pageable memory.
bool mapped_host(const void *p, void **dev) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    if (a.type != cudaMemoryTypeHost || !a.devicePointer) return false;
    *dev = a.devicePointer;
    return true;
}

// The end of a host-buffer step: the step's device flags read back with the
// stream drained, mapped to the reference's errors. When profiling, the host
// time from the call's entry `t0` to here (validation, planning, launches and
// copies queued) and the time blocked in the final synchronisation are added
// to G4A_K_HOST_ISSUE / G4A_K_HOST_WAIT.
int finish_host_step(g4a_ctx *ctx, std::chrono::steady_clock::time_point t0, cudaStream_t also = nullptr) {
    const auto t1 = std::chrono::steady_clock::now();
    G4A_CUDA_TRY(ctx, cudaMemcpyAsync(ctx->h_flag, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream));
    if (also) G4A_CUDA_TRY(ctx, cudaStreamSynchronize(also));
    G4A_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    if (ctx->profiling) {
        const auto t2 = std::chrono::steady_clock::now();
        ctx->prof_ms[G4A_K_HOST_ISSUE] += std::chrono::duration<double, std::milli>(t1 - t0).count();
        ctx->prof_n[G4A_K_HOST_ISSUE] += 1;
        ctx->prof_ms[G4A_K_HOST_WAIT] += std::chrono::duration<double, std::milli>(t2 - t1).count();
        ctx->prof_n[G4A_K_HOST_WAIT] += 1;
    }
    const int flag = *ctx->h_flag;
    if (flag) {
        ctx->err_epoch++;
        G4A_CUDA_TRY(ctx, cudaMemset(ctx->d_err, 0, sizeof(int)));
        if (flag & 6) return fail(ctx, G4A_TIMEOUT, "compute: a device wait ran out (flag %d)", flag);
        return fail(ctx, G4A_NONFINITE, "compute: softmax input is not finite");
    }
    return G4A_OK;
}

}  // namespace

extern "C" int g4a_decode_host(g4a_ctx *ctx, g4a_kv *kv, int32_t n_layers, const g4a_decode_layer_host *layers,
                               int32_t n_seqs, const int32_t *seq_ids, const int32_t *positions) {
    if (!ctx || !kv) return G4A_COMPUTE;
    const auto t_entry = std::chrono::steady_clock::now();
    cudaSetDevice(ctx->device);
    if (n_layers < 0 || n_seqs < 0 || (n_layers > 0 && !layers))
        return fail(ctx, G4A_COMPUTE, "compute: invalid decode arguments");
    if (!ctx->h_flag) G4A_CUDA_TRY(ctx, cudaHostAlloc(reinterpret_cast<void **>(&ctx->h_flag), sizeof(int),
                                                      cudaHostAllocDefault));
    // Page-locked buffers the device can address: the step's kernels read
    // q/k/v and write the outputs in place over the bus (the prep kernel
    // reads each input once, the main and combine kernels write each output
    // once), one launch for all layers and no staging copies; the transfers
    // overlap the attention of other tasks. Other buffers go through the
    // context's device slots below.
    // Large steps are faster through the DMA pipeline below (measured: the
    // kernels' own reads over the bus reach about half its copy rate), small
    // ones in place (a copy's fixed cost dominates them).
    size_t step_bytes = 0;
    for (int32_t i = 0; i < n_layers; i++)
        step_bytes += (size_t)n_seqs * g4a_head_dim(&ctx->hp, layers[i].layer) * (2 * kHeads + 2) * sizeof(float);
    if (step_bytes <= kInPlaceMaxBytes) {
        bool mapped = n_layers > 0;
        std::vector<g4a_decode_layer> zc(n_layers);
        for (int32_t i = 0; i < n_layers && mapped; i++) {
            const g4a_decode_layer_host &h = layers[i];
            void *q = nullptr, *k = nullptr, *v = nullptr, *o = nullptr;
            mapped = (!h.q_raw_host || mapped_host(h.q_raw_host, &q)) &&
                     (!h.k_raw_host || mapped_host(h.k_raw_host, &k)) &&
                     (!h.v_raw_host || mapped_host(h.v_raw_host, &v)) && (!h.out_host || mapped_host(h.out_host, &o));
            zc[i] = g4a_decode_layer{h.layer, static_cast<const float *>(q), static_cast<const float *>(k),
                                     static_cast<const float *>(v), h.q_norm_w_dev, h.k_norm_w_dev,
                                     static_cast<float *>(o)};
        }
        if (mapped) {
            Plan &plan = scratch_plan();
            int rc = build_decode(ctx, kv, n_layers, zc.data(), n_seqs, seq_ids, positions, plan);
            if (rc) return rc;
            if ((rc = run_plan(ctx, plan, kv->d_bt, kv->max_pages, kv->page_tokens, kv->dtype == G4A_KV_F16)))
                return rc;
            return finish_host_step(ctx, t_entry);
        }
    }
    // device slots: per layer q [n][8 hd], k and v [n][hd], out [n][8 hd]
    std::vector<size_t> off(n_layers);
    std::vector<int32_t> width(n_layers);
    size_t total = 0;
    for (int32_t i = 0; i < n_layers; i++) {
        width[i] = g4a_head_dim(&ctx->hp, layers[i].layer);  // the layer itself is checked by check_decode
        off[i] = total;
        total += (size_t)n_seqs * width[i] * (2 * kHeads + 2);
    }
    int rc = grow(ctx, &ctx->d_io, &ctx->io_cap, std::max<size_t>(total, 1), false);
    if (rc) return rc;
    if (!ctx->copy_in) G4A_CUDA_TRY(ctx, cudaStreamCreateWithFlags(&ctx->copy_in, cudaStreamNonBlocking));
    if (!ctx->copy_out) G4A_CUDA_TRY(ctx, cudaStreamCreateWithFlags(&ctx->copy_out, cudaStreamNonBlocking));
    // events: [0] call start, [1] inputs in, [2] kernels done
    while (ctx->io_events.size() < 3) {
        cudaEvent_t e = nullptr;
        G4A_CUDA_TRY(ctx, cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        ctx->io_events.push_back(e);
    }
    cudaEvent_t *ev = ctx->io_events.data();
    std::vector<g4a_decode_layer> dev(n_layers);
    // Outputs in page-locked memory the device can address are written in
    // place by the kernels (posted writes over the bus while the step runs);
    // other outputs go through the device slots and a copy after the kernels.
    // The appended k and v rows (one row per sequence, a fifth of the input
    // bytes but two of every layer's three copies) are read in place by the
    // prep kernel when they sit in page-locked memory the device can address:
    // each prep block reads its two rows over the bus in parallel with the
    // others, which costs less than two more copies with their fixed cost.
    std::vector<char> out_in_place(n_layers, 0), kv_in_place(n_layers, 0);
    for (int32_t i = 0; i < n_layers; i++) {
        const size_t qn = (size_t)n_seqs * kHeads * width[i], kn = (size_t)n_seqs * width[i];
        float *base = ctx->d_io + off[i];
        const g4a_decode_layer_host &h = layers[i];
        void *o_mapped = nullptr, *k_mapped = nullptr, *v_mapped = nullptr;
        out_in_place[i] = h.out_host && mapped_host(h.out_host, &o_mapped);
        kv_in_place[i] = h.k_raw_host && h.v_raw_host && mapped_host(h.k_raw_host, &k_mapped) &&
                         mapped_host(h.v_raw_host, &v_mapped);
        float *out_dev = out_in_place[i] ? static_cast<float *>(o_mapped) : h.out_host ? base + qn + 2 * kn : nullptr;
        const float *k_dev = kv_in_place[i] ? static_cast<const float *>(k_mapped) : h.k_raw_host ? base + qn : nullptr;
        const float *v_dev =
            kv_in_place[i] ? static_cast<const float *>(v_mapped) : h.v_raw_host ? base + qn + kn : nullptr;
        dev[i] = g4a_decode_layer{h.layer, h.q_raw_host ? base : nullptr, k_dev, v_dev, h.q_norm_w_dev,
                                  h.k_norm_w_dev, out_dev};
    }
    // The inputs go first on the copy-in stream (after the work already
    // queued on the context's stream), into the context's own slots, so that
    // the copies overlap the host-side validation and planning (measured: a
    // second copy stream does not shorten them; the host link's rate bounds
    // them). On a rejected call the copy stream is drained before returning
    // (no copy still reads the caller's buffers) and neither the cache nor
    // out_host has been touched.
    G4A_CUDA_TRY(ctx, cudaEventRecord(ev[0], ctx->stream));
    G4A_CUDA_TRY(ctx, cudaStreamWaitEvent(ctx->copy_in, ev[0], 0));
    cudaEvent_t prof_a = ctx->profiling ? spare_event(ctx) : nullptr;
    if (prof_a) cudaEventRecord(prof_a, ctx->copy_in);
    for (int32_t i = 0; i < n_layers; i++) {
        const size_t qb = (size_t)n_seqs * kHeads * width[i] * sizeof(float), kb = (size_t)n_seqs * width[i] * sizeof(float);
        const g4a_decode_layer_host &h = layers[i];
        int32_t src = -1;
        const bool owner = g4a_kv_source_layer(&ctx->hp, h.layer, &src, nullptr) == G4A_OK && src == h.layer;
        if (h.q_raw_host && qb)
            G4A_CUDA_TRY(ctx, cudaMemcpyAsync(const_cast<float *>(dev[i].q_raw_dev), h.q_raw_host, qb,
                                              cudaMemcpyHostToDevice, ctx->copy_in));
        if (owner && h.k_raw_host && h.v_raw_host && kb && !kv_in_place[i]) {
            G4A_CUDA_TRY(ctx, cudaMemcpyAsync(const_cast<float *>(dev[i].k_raw_dev), h.k_raw_host, kb,
                                              cudaMemcpyHostToDevice, ctx->copy_in));
            G4A_CUDA_TRY(ctx, cudaMemcpyAsync(const_cast<float *>(dev[i].v_raw_dev), h.v_raw_host, kb,
                                              cudaMemcpyHostToDevice, ctx->copy_in));
        }
    }
    G4A_CUDA_TRY(ctx, cudaEventRecord(ev[1], ctx->copy_in));
    if (prof_a) {
        cudaEvent_t b = spare_event(ctx);
        cudaEventRecord(b, ctx->copy_in);
        ctx->recs.push_back({G4A_K_COPY_IN, prof_a, b});
    }
    DecodeLayers info;
    if ((rc = check_decode(ctx, kv, n_layers, dev.data(), n_seqs, seq_ids, positions, info))) {
        cudaStreamSynchronize(ctx->copy_in);
        return rc;
    }
    // One launch set for all layers once every input is in (per-layer
    // launches each pay a persistent kernel's ramp and tail, which cost more
    // than the copy overlap they buy), then every output copied out.
    G4A_CUDA_TRY(ctx, cudaStreamWaitEvent(ctx->stream, ev[1], 0));
    {
        Plan &plan = scratch_plan();
        plan_decode(ctx, kv, dev.data(), n_seqs, seq_ids, positions, info, 0, n_layers, plan);
        if ((rc = run_plan(ctx, plan, kv->d_bt, kv->max_pages, kv->page_tokens, kv->dtype == G4A_KV_F16))) return rc;
    }
    G4A_CUDA_TRY(ctx, cudaEventRecord(ev[2], ctx->stream));
    G4A_CUDA_TRY(ctx, cudaStreamWaitEvent(ctx->copy_out, ev[2], 0));
    {
        cudaEvent_t a = ctx->profiling ? spare_event(ctx) : nullptr;
        if (a) cudaEventRecord(a, ctx->copy_out);
        for (int32_t i = 0; i < n_layers; i++) {
            if (!layers[i].out_host || out_in_place[i]) continue;
            G4A_CUDA_TRY(ctx, cudaMemcpyAsync(layers[i].out_host, dev[i].out_dev,
                                              (size_t)n_seqs * kHeads * width[i] * sizeof(float),
                                              cudaMemcpyDeviceToHost, ctx->copy_out));
        }
        if (a) {
            cudaEvent_t b = spare_event(ctx);
            cudaEventRecord(b, ctx->copy_out);
            ctx->recs.push_back({G4A_K_COPY_OUT, a, b});
        }
    }
    commit_decode(kv, n_layers, dev.data(), n_seqs, seq_ids, info);
    return finish_host_step(ctx, t_entry, ctx->copy_out);
}

struct g4a_plan {
    g4a_ctx *ctx = nullptr;
    Staged st;
};

extern "C" int g4a_decode_plan(g4a_ctx *ctx, g4a_kv *kv, int32_t n_layers, const g4a_decode_layer *layers,
                               int32_t n_seqs, const int32_t *seq_ids, const int32_t *positions, g4a_plan **out) {
    if (!out) return fail(ctx, G4A_COMPUTE, "compute: null plan output");
    *out = nullptr;
    Plan &plan = scratch_plan();
    int rc = build_decode(ctx, kv, n_layers, layers, n_seqs, seq_ids, positions, plan);
    if (rc) return rc;
    auto *pl = new g4a_plan();
    pl->ctx = ctx;
    rc = stage_plan(ctx, plan, kv->d_bt, kv->max_pages, kv->page_tokens, kv->dtype == G4A_KV_F16, true, &pl->st);
    if (rc) {
        g4a_plan_destroy(pl);
        return rc;
    }
    *out = pl;
    return G4A_OK;
}

extern "C" int g4a_plan_run(g4a_plan *plan) {
    if (!plan) return G4A_COMPUTE;
    cudaSetDevice(plan->ctx->device);
    return launch_staged(plan->ctx, plan->st);
}

extern "C" void g4a_plan_destroy(g4a_plan *plan) {
    if (!plan) return;
    cudaSetDevice(plan->ctx->device);
    cudaStreamSynchronize(plan->ctx->stream);
    cudaFree(plan->st.meta);
    cudaFree(plan->st.part_o);
    cudaFree(plan->st.part_ml);
    cudaFree(plan->st.tickets);
    cudaFree(plan->st.q_blocks);
    delete plan;
}

extern "C" int g4a_lse_merge(g4a_ctx *ctx, int32_t n_parts, const float *const *parts_out, const float *const *parts_lse,
                             int64_t rows, int32_t n_heads, int32_t hd, float *out, float *lse) {
    if (!ctx) return G4A_COMPUTE;
    cudaSetDevice(ctx->device);
    if (n_parts < 1 || n_parts > 16 || rows < 0 || n_heads <= 0 || hd <= 0 || !parts_out || !parts_lse || !out)
        return fail(ctx, G4A_COMPUTE, "compute: invalid merge arguments");
    G4A_CUDA_TRY(ctx, launch_lse_merge(n_parts, parts_out, parts_lse, rows, n_heads, hd, out, lse, ctx->stream));
    return G4A_OK;
}

extern "C" int g4a_prefill(g4a_ctx *ctx, int32_t n, const g4a_prefill_problem *problems) {
    if (!ctx) return G4A_COMPUTE;
    cudaSetDevice(ctx->device);
    if (ctx->hp.n_heads != kHeads || ctx->hp.n_kv_heads != 1)
        return fail(ctx, G4A_COMPUTE, "compute: prefill serves %d query heads over 1 KV head", kHeads);
    const char *msg = "";
    int rc = G4A_OK;
    const bool stall = (ctx->stall_mask & (1u << G4A_K_PREFILL)) != 0;
    ctx->stall_mask &= ~(1u << G4A_K_PREFILL);
    const cudaError_t e = timed(ctx, G4A_K_PREFILL, [&] {
        rc = prefill_run(ctx->prefill, ctx->d_err, n, problems, ctx->stream, &msg, stall);
        return cudaSuccess;
    });
    (void)e;
    if (rc != G4A_OK) return fail(ctx, rc, "compute: %s", msg);
    return G4A_OK;
}

// ---- Q8_0 mat-vec family (matvec.rs) -------------------------------------

namespace {

int q8_entry(g4a_ctx *ctx, int kind, const uint8_t *w, const uint8_t *w2, int64_t rows, int64_t cols, const float *x,
             int32_t n_vec, float cap, float *out) {
    if (!ctx) return G4A_COMPUTE;
    cudaSetDevice(ctx->device);
    if (cols <= 0 || cols % 32 != 0)  // matvec.rs:37-42
        return fail(ctx, G4A_COMPUTE, "Q8_0 activation length %lld is not a multiple of 32", (long long)cols);
    if (rows < 0 || n_vec < 1 || n_vec > 65535 || cols > (1LL << 30) || !x || (rows > 0 && (!w || !out)) ||
        (kind == 1 && rows > 0 && !w2))
        return fail(ctx, G4A_COMPUTE, "compute: invalid Q8_0 mat-vec arguments");
    int rc;
    if ((rc = grow(ctx, &ctx->d_q8x, &ctx->q8x_cap, (size_t)n_vec * cols, false)) ||
        (rc = grow(ctx, &ctx->d_q8s, &ctx->q8s_cap, (size_t)n_vec * cols / 32, false)))
        return rc;
    const char *msg = "";
    int status = G4A_OK;
    const cudaError_t e = timed(ctx, G4A_K_MATVEC_Q8, [&] {
        status = q8_run(kind, w, w2, rows, cols, x, n_vec, cap, out, ctx->d_q8x, ctx->d_q8s, ctx->d_err, ctx->n_sm,
                        ctx->stream, &msg);
        return cudaSuccess;
    });
    (void)e;
    if (status != G4A_OK) return fail(ctx, status, "compute: %s", msg);
    return G4A_OK;
}

}  // namespace

extern "C" int g4a_matvec_q8_0(g4a_ctx *ctx, const uint8_t *w_dev, int64_t rows, int64_t cols, const float *x_dev,
                               int32_t n_vec, float *out_dev) {
    return q8_entry(ctx, 0, w_dev, nullptr, rows, cols, x_dev, n_vec, 0.0f, out_dev);
}

extern "C" int g4a_geglu_q8_0(g4a_ctx *ctx, const uint8_t *gate_dev, const uint8_t *up_dev, int64_t rows, int64_t cols,
                              const float *x_dev, int32_t n_vec, float *out_dev) {
    return q8_entry(ctx, 1, gate_dev, up_dev, rows, cols, x_dev, n_vec, 0.0f, out_dev);
}

extern "C" int g4a_matvec_q8_0_softcap(g4a_ctx *ctx, const uint8_t *w_dev, int64_t rows, int64_t cols,
                                       const float *x_dev, int32_t n_vec, float cap, float *out_dev) {
    if (!(cap != 0.0f)) return fail(ctx, G4A_COMPUTE, "compute: soft-cap of zero");
    return q8_entry(ctx, 2, w_dev, nullptr, rows, cols, x_dev, n_vec, cap, out_dev);
}

extern "C" int g4a_quantize_q8_0(g4a_ctx *ctx, const float *x_dev, int64_t n, float *scales_dev, int8_t *quants_dev) {
    if (!ctx) return G4A_COMPUTE;
    cudaSetDevice(ctx->device);
    if (n < 0 || n % 32 != 0)
        return fail(ctx, G4A_COMPUTE, "Q8_0 activation length %lld is not a multiple of 32", (long long)n);
    if (n == 0) return G4A_OK;
    if (!x_dev || !scales_dev || !quants_dev) return fail(ctx, G4A_COMPUTE, "compute: null Q8_0 buffers");
    const char *msg = "";
    // rows = 0: quantize only
    int status = q8_run(0, nullptr, nullptr, 0, n, x_dev, 1, 0.0f, nullptr, quants_dev, scales_dev, ctx->d_err,
                        ctx->n_sm, ctx->stream, &msg);
    if (status != G4A_OK) return fail(ctx, status, "compute: %s", msg);
    return G4A_OK;
}
