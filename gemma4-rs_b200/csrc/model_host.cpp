// Host side of the E2B decoder (include/g4attn.h, g4a_model_*): one token per
// sequence through embed, the 35 layers and the logits of
// crates/llm-gemma4/src/impl_/model.rs:252-449, and the prompt-then-greedy
// loop of generate.rs:15-64, for many sequences at once. A prompt goes
// through in chunks of many positions per step (rows), each row's arithmetic
// the same as in a one-token step, so the result does not depend on the
// chunking.
//
// A step is one fixed sequence of launches on the model's own stream (about
// 10 per layer at small batches): the attention plan, embedding, per-layer inputs, then per
// layer the fused residual/norm/quantize kernels, the Q8_0 mat-vecs and the
// fused decode attention, then the soft-capped head and the argmax. Every
// kernel rounds as the reference does (integer Q8_0 dots summed in block
// order, attention in the reference's order with glibc's expf, glibc's
// tanhf), so the logits are the reference's bit for bit. Nothing
// in it depends on the host values of the step (tokens and positions are read
// on the device), so after one eager run per batch size the step is captured
// into a CUDA graph with its input upload and result download, and every
// later step of that size is one graph launch.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/g4attn.h"
#include "host_internal.h"
#include "internal.h"

using namespace g4a;

struct g4a_model {
    g4a_ctx *ctx = nullptr;
    g4a_model_weights w{};
    int32_t S = 0, T = 0;  // max sequences, max positions per sequence
    int32_t R = 0;         // max rows (tokens) of one step: S, or more for prompt chunks
    int32_t L = 0, d = 0, d_ff = 0, ple = 0, vocab = 0, hd_max = 0, qd_max = 0, cmax = 0;
    int32_t rows_per_item = 64, ms_local = 1, ms_global = 1;
    bool exact = true;  // attention in the reference's order (one CTA per task); up to kExactMaxRows positions
    std::vector<int32_t> len, source, hd, global;
    cudaStream_t st = nullptr;
    cudaEvent_t ev = nullptr;
    std::vector<void *> allocs;
    // a step of n rows and n_out result rows: sequence ids [n], tokens [n],
    // positions [n], the rows whose logits are returned [n_out]
    int32_t *d_in = nullptr;  // [3R + S]
    int32_t *h_in = nullptr;              // pinned [3R + S]
    unsigned long long *h_out = nullptr;  // pinned [S]: the argmax slots (index in the low 32 bits)
    int32_t *h_err = nullptr;             // pinned: the device error flags after the step
    float *x = nullptr, *y = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *att = nullptr;
    float *gate = nullptr, *gated = nullptr, *P = nullptr, *pli = nullptr, *logits = nullptr;
    int8_t *xq = nullptr, *xq_out = nullptr;  // xq_out/xs_out: the head's input rows of a prompt chunk
    float *xs = nullptr, *xs_out = nullptr;
    E2bLayerDesc *d_layers = nullptr;
    DecodeTask *d_tasks = nullptr;
    DecodeItem *d_items_local = nullptr, *d_items_global = nullptr;
    float *part_o = nullptr, *part_ml = nullptr, *scores = nullptr;
    unsigned *tickets = nullptr;
    unsigned long long *d_best = nullptr;  // [S] packed (total-order key, index) of each row's argmax
    std::map<int32_t, cudaGraphExec_t> graphs;
    std::map<int32_t, int> eager_runs;
    bool use_graphs = true;  // G4A_NO_GRAPH=1 in the environment: every step eager
    bool pdl = true;         // programmatic dependent launch along the step (G4A_NO_PDL=1: off)
    std::vector<float *> k_cache, v_cache;  // per layer: its KV source's caches
    int32_t last_n = 0;
    std::vector<int32_t> eos;  // eos_token_ids (model.rs:88): a sequence ends after emitting one
};

namespace {

// Rows of a prompt chunk (all sequences' positions together): enough for the
// batched Q8_0 kernel to reach its weight-streaming rate, a few hundred MB
// of activations.
constexpr int64_t kChunkRows = 2048;

template <typename T>
T *dalloc(g4a_model *m, size_t n) {
    void *p = nullptr;
    if (cudaMalloc(&p, std::max<size_t>(n, 1) * sizeof(T)) != cudaSuccess) return nullptr;
    m->allocs.push_back(p);
    return static_cast<T *>(p);
}

// The weights a layer needs (model.rs:386-435); the name of the first one
// missing, or nullptr.
const char *missing_weight(const g4a_model_weights &w, int32_t layer, bool owner) {
    const g4a_layer_weights &l = w.layers[layer];
    if (!l.attn_norm) return "attn_norm";
    if (!l.attn_q) return "attn_q";
    if (!l.attn_q_norm) return "attn_q_norm";
    if (owner && !l.attn_k) return "attn_k";
    if (owner && !l.attn_v) return "attn_v";
    if (owner && !l.attn_k_norm) return "attn_k_norm";
    if (!l.attn_output) return "attn_output";
    if (!l.post_attention_norm) return "post_attention_norm";
    if (!l.ffn_norm) return "ffn_norm";
    if (!l.ffn_gate) return "ffn_gate";
    if (!l.ffn_up) return "ffn_up";
    if (!l.ffn_down) return "ffn_down";
    if (!l.post_ffw_norm) return "post_ffw_norm";
    if (w.ple_dim > 0 && !l.inp_gate) return "inp_gate";
    if (w.ple_dim > 0 && !l.proj) return "proj";
    if (w.ple_dim > 0 && !l.post_norm) return "post_norm";
    return nullptr;
}

int mv(g4a_model *m, int kind, const uint8_t *w, const uint8_t *w2, int64_t rows, int64_t cols, const float *x, int n,
       float cap, float *out, const float *pli = nullptr, int32_t pli_stride = 0, const Q8Seg *extra = nullptr,
       int n_extra = 0) {
    const char *msg = "";
    const int rc = q8_run(kind, w, w2, rows, cols, x, n, cap, out, m->xq, m->xs, m->ctx->d_err, m->ctx->n_sm, m->st,
                          &msg, m->pdl, pli, pli_stride, extra, n_extra);
    return rc == G4A_OK ? G4A_OK : fail(m->ctx, rc, "compute: %s", msg);
}

#define MODEL_TRY(call)                                                   \
    do {                                                                  \
        cudaError_t e_ = (call);                                          \
        if (e_ != cudaSuccess) return cuda_fail(m->ctx, e_, #call);       \
    } while (0)

// The kernels of one step over the n rows of d_in. A decode step (chunk
// false) has one row per sequence, and each attention task stores its own
// token's K/V row; its logits are every row's. A prompt chunk (chunk true)
// may hold several positions of a sequence: all K/V rows are stored first,
// and the logits are those of the n_out rows listed after the positions
// (none for a chunk that does not end a prompt). A chunk's rows are cl
// consecutive positions of each of its sequences, sequence-major.
int enqueue_step(g4a_model *m, int32_t n, int32_t n_out, bool chunk, int32_t cl) {
    g4a_ctx *ctx = m->ctx;
    const g4a_model_weights &w = m->w;
    const float eps = ctx->hp.rms_norm_eps;
    const int32_t *d_seq = m->d_in, *d_tok = m->d_in + n, *d_pos = m->d_in + 2 * n, *d_sel = m->d_in + 3 * n;
    const int d = m->d, L = m->L, ple = m->ple;

    E2bPlanArgs pa{};
    pa.layers = m->d_layers;
    pa.n_layers = L;
    pa.n = n;
    pa.task_stride = m->R;
    pa.seqs = d_seq;
    pa.pos = d_pos;
    pa.max_tokens = m->T;
    pa.window = ctx->hp.sliding_window;
    pa.rows_per_item = m->rows_per_item;
    pa.max_splits_local = m->ms_local;
    pa.max_splits_global = m->ms_global;
    pa.q = m->q;
    pa.k = m->k;
    pa.v = m->v;
    pa.att = m->att;
    pa.tasks = m->d_tasks;
    pa.items_local = m->d_items_local;
    pa.items_global = m->d_items_global;
    pa.best = m->d_best;
    pa.n_best = n_out;
    pa.fused_append = chunk ? 0 : 1;
    MODEL_TRY(e2b_plan(pa, m->st));

    // embed (model.rs:376-384) and per-layer inputs (:252-270)
    MODEL_TRY(e2b_embed(w.token_embd, d, d_tok, n, std::sqrt((float)d), m->x, m->st, m->pdl));
    int rc;
    if (ple > 0) {
        if ((rc = mv(m, 0, w.ple_model_proj, nullptr, (int64_t)L * ple, d, m->x, n, 0.0f, m->P))) return rc;
        MODEL_TRY(e2b_ple_inputs(m->P, w.ple_token_embd, d_tok, w.ple_proj_norm, L, ple, 1.0f / std::sqrt((float)d),
                                 std::sqrt((float)ple), 1.0f / std::sqrt(2.0f), eps, m->pli, n, m->st, m->pdl));
    }
    MODEL_TRY(e2b_resid(m->x, nullptr, nullptr, 1.0f, w.layers[0].attn_norm, d, eps, m->xq, m->xs, n, m->st, m->pdl));

    for (int l = 0; l < L; l++) {
        const g4a_layer_weights &lw = w.layers[l];
        const int hd = m->hd[l], qd = kHeads * hd;
        const bool owner = m->source[l] == l;
        // q, k, v of the normalized input (model.rs:392-401); small batches
        // stream the three matrices in one launch
        if (owner && n <= 8) {
            const Q8Seg kv[2] = {{lw.attn_k, hd, m->k}, {lw.attn_v, hd, m->v}};
            if ((rc = mv(m, 0, lw.attn_q, nullptr, qd, d, nullptr, n, 0.0f, m->q, nullptr, 0, kv, 2))) return rc;
        } else {
            if ((rc = mv(m, 0, lw.attn_q, nullptr, qd, d, nullptr, n, 0.0f, m->q))) return rc;
            if (owner) {
                if ((rc = mv(m, 0, lw.attn_k, nullptr, hd, d, nullptr, n, 0.0f, m->k))) return rc;
                if ((rc = mv(m, 0, lw.attn_v, nullptr, hd, d, nullptr, n, 0.0f, m->v))) return rc;
            }
        }
        // q/k/v norms, RoPE, append, window and attention (:394-410)
        DecodeParams p{};
        p.tasks = m->d_tasks + (size_t)l * m->R;
        p.items = m->global[l] ? m->d_items_global : m->d_items_local;
        p.block_table = nullptr;
        p.page_tokens = 1;
        p.rope_local = ctx->d_rope_local;
        p.rope_global = ctx->d_rope_global;
        p.eps = eps;
        p.part_o = m->part_o;
        p.part_ml = m->part_ml;
        p.tickets = m->tickets;
        p.err_flag = ctx->d_err;
        p.n_items = n * (m->global[l] ? m->ms_global : m->ms_local);
        if (chunk && owner) MODEL_TRY(launch_task_append(p, hd, n, m->st, m->pdl));
        if (m->exact) {
            p.max_rows = m->T;
            p.scores = m->scores;
            if (chunk && cl > 1)  // positions of one sequence share their key rows
                MODEL_TRY(launch_prompt_exact(p, hd, n, cl, m->st, m->pdl));
            else
                MODEL_TRY(launch_decode_exact(p, hd, n, m->st, m->pdl));
        } else {
            MODEL_TRY(launch_decode(p, hd, 0, true, m->st));
        }
        // output projection, post-attention norm, residual, FFN norm (:411-415)
        if ((rc = mv(m, 0, lw.attn_output, nullptr, d, qd, m->att, n, 0.0f, m->y))) return rc;
        MODEL_TRY(e2b_resid(m->x, m->y, lw.post_attention_norm, 1.0f, lw.ffn_norm, d, eps, m->xq, m->xs, n, m->st,
                            m->pdl));
        // GEGLU, down projection, post-FFN norm, residual (:416-420)
        if ((rc = mv(m, 1, lw.ffn_gate, lw.ffn_up, m->d_ff, d, nullptr, n, 0.0f, m->gated))) return rc;
        if ((rc = mv(m, 0, lw.ffn_down, nullptr, d, m->d_ff, m->gated, n, 0.0f, m->y))) return rc;
        const float *next_norm = l + 1 < L ? w.layers[l + 1].attn_norm : w.output_norm;
        if (ple > 0) {
            // per-layer embedding (:422-432), then layer_output_scale (:433-435)
            MODEL_TRY(e2b_resid(m->x, m->y, lw.post_ffw_norm, 1.0f, nullptr, d, eps, m->xq, m->xs, n, m->st, m->pdl));
            if ((rc = mv(m, 0, lw.inp_gate, nullptr, ple, d, nullptr, n, 0.0f, m->gate))) return rc;
            if (n <= 8) {  // the gate rides on the proj mat-vec's input quantization
                if ((rc = mv(m, 0, lw.proj, nullptr, d, ple, m->gate, n, 0.0f, m->y, m->pli + (size_t)l * ple,
                             L * ple)))
                    return rc;
            } else {
                MODEL_TRY(e2b_gelu_quant(m->gate, m->pli, l, L, ple, m->xq, m->xs, n, m->st, m->pdl));
                if ((rc = mv(m, 0, lw.proj, nullptr, d, ple, nullptr, n, 0.0f, m->y))) return rc;
            }
            MODEL_TRY(e2b_resid(m->x, m->y, lw.post_norm, lw.layer_output_scale, next_norm, d, eps, m->xq, m->xs, n,
                                m->st, m->pdl));
        } else {
            MODEL_TRY(e2b_resid(m->x, m->y, lw.post_ffw_norm, lw.layer_output_scale, next_norm, d, eps, m->xq, m->xs,
                                n, m->st, m->pdl));
        }
    }
    // logits (:438-449) and greedy sampling (sample.rs:27-36)
    if (!chunk) {
        if ((rc = mv(m, 2, w.token_embd, nullptr, m->vocab, d, nullptr, n, w.final_logit_softcap, m->logits)))
            return rc;
    } else if (n_out > 0) {
        MODEL_TRY(e2b_gather_rows(m->xq, m->xs, d, d_sel, n_out, m->xq_out, m->xs_out, m->st, m->pdl));
        const char *msg = "";
        rc = q8_run(2, w.token_embd, nullptr, m->vocab, d, nullptr, n_out, w.final_logit_softcap, m->logits,
                    m->xq_out, m->xs_out, ctx->d_err, ctx->n_sm, m->st, &msg, m->pdl);
        if (rc) return fail(ctx, rc, "compute: %s", msg);
    }
    if (n_out > 0) MODEL_TRY(e2b_argmax(m->logits, m->vocab, n_out, m->d_best, m->st, m->pdl));
    return G4A_OK;
}

// Upload of the step's inputs, the step, download of its tokens and flags.
int record_step(g4a_model *m, int32_t n, int32_t n_out, bool chunk, int32_t cl) {
    const size_t n_in = 3 * (size_t)n + (chunk ? n_out : 0);
    MODEL_TRY(cudaMemcpyAsync(m->d_in, m->h_in, n_in * sizeof(int32_t), cudaMemcpyHostToDevice, m->st));
    const int rc = enqueue_step(m, n, n_out, chunk, cl);
    if (rc) return rc;
    if (n_out > 0)
        MODEL_TRY(cudaMemcpyAsync(m->h_out, m->d_best, (size_t)n_out * sizeof(unsigned long long),
                                  cudaMemcpyDeviceToHost, m->st));
    MODEL_TRY(cudaMemcpyAsync(m->h_err, m->ctx->d_err, sizeof(int32_t), cudaMemcpyDeviceToHost, m->st));
    return G4A_OK;
}

// A decode step of n sequences: eager the first time a size is seen, then
// captured, then one graph launch per step of that size. Prompt chunks are
// eager (their row counts vary and each runs once per prompt).
int run_step(g4a_model *m, int32_t n, int32_t n_out = -1, bool chunk = false, int32_t cl = 1) {
    if (chunk) return record_step(m, n, n_out, true, cl);
    n_out = n;
    auto it = m->graphs.find(n);
    if (it != m->graphs.end()) {
        MODEL_TRY(cudaGraphLaunch(it->second, m->st));
        return G4A_OK;
    }
    if (!m->use_graphs || m->eager_runs[n]++ == 0) return record_step(m, n, n_out, false, 1);  // first of a size: eager
    cudaGraph_t g = nullptr;
    MODEL_TRY(cudaStreamBeginCapture(m->st, cudaStreamCaptureModeThreadLocal));
    const int rc = record_step(m, n, n_out, false, 1);
    const cudaError_t e = cudaStreamEndCapture(m->st, &g);
    if (rc || e != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        return rc ? rc : cuda_fail(m->ctx, e, "cudaStreamEndCapture");
    }
    cudaGraphExec_t exec = nullptr;
    const cudaError_t ei = cudaGraphInstantiate(&exec, g, 0);
    cudaGraphDestroy(g);
    if (ei != cudaSuccess) return cuda_fail(m->ctx, ei, "cudaGraphInstantiate");
    m->graphs[n] = exec;
    MODEL_TRY(cudaGraphLaunch(exec, m->st));
    return G4A_OK;
}

}  // namespace

extern "C" int g4a_synth_q8_0(g4a_ctx *ctx, uint8_t *dst_dev, int64_t n_values, uint64_t seed, uint64_t tensor,
                              float sigma) {
    if (!ctx) return G4A_COMPUTE;
    cudaSetDevice(ctx->device);
    if (n_values < 0 || n_values % 32 || (n_values && !dst_dev))
        return fail(ctx, G4A_COMPUTE, "compute: Q8_0 tensor of %lld values", (long long)n_values);
    G4A_CUDA_TRY(ctx, e2b_synth_q8(dst_dev, n_values / 32, seed, tensor, sigma, ctx->stream));
    return G4A_OK;
}

extern "C" int g4a_synth_norm(g4a_ctx *ctx, float *dst_dev, int64_t n, uint64_t seed, uint64_t tensor, float center,
                              float spread) {
    if (!ctx) return G4A_COMPUTE;
    cudaSetDevice(ctx->device);
    if (n < 0 || (n && !dst_dev)) return fail(ctx, G4A_COMPUTE, "compute: invalid norm tensor");
    G4A_CUDA_TRY(ctx, e2b_synth_norm(dst_dev, n, seed, tensor, center, spread, ctx->stream));
    return G4A_OK;
}

extern "C" void g4a_model_destroy(g4a_model *m) {
    if (!m) return;
    cudaSetDevice(m->ctx->device);
    if (m->st) cudaStreamSynchronize(m->st);
    for (auto &g : m->graphs) cudaGraphExecDestroy(g.second);
    for (void *p : m->allocs) cudaFree(p);
    if (m->h_in) cudaFreeHost(m->h_in);
    if (m->h_out) cudaFreeHost(m->h_out);
    if (m->h_err) cudaFreeHost(m->h_err);
    if (m->ev) cudaEventDestroy(m->ev);
    if (m->st) cudaStreamDestroy(m->st);
    delete m;
}

extern "C" int g4a_model_create(g4a_ctx *ctx, const g4a_model_weights *w, int32_t max_seqs, int32_t max_tokens,
                                g4a_model **out) {
    if (!ctx || !w || !out) return G4A_COMPUTE;
    *out = nullptr;
    cudaSetDevice(ctx->device);
    const g4a_hparams &hp = ctx->hp;
    if (hp.n_heads != kHeads || hp.n_kv_heads != 1)
        return fail(ctx, G4A_COMPUTE, "compute: the decoder serves %d query heads over 1 KV head", kHeads);
    if ((hp.head_dim_local != 256 && hp.head_dim_local != 512) ||
        (hp.head_dim_global != 256 && hp.head_dim_global != 512))
        return fail(ctx, G4A_COMPUTE, "compute: head widths must be 256 or 512");
    if (hp.n_layers > G4A_MAX_LAYERS) return fail(ctx, G4A_COMPUTE, "compute: more than %d layers", G4A_MAX_LAYERS);
    if (w->d_model <= 0 || w->d_model % 32 || w->d_model > 4096 || w->d_ff <= 0 || w->d_ff % 32 || w->ple_dim < 0 ||
        w->ple_dim % 32 || w->ple_dim > 1024 || w->vocab_size <= 0 || !(w->final_logit_softcap != 0.0f))
        return fail(ctx, G4A_COMPUTE, "compute: unsupported model dimensions");
    if (max_seqs <= 0 || max_tokens <= 0) return fail(ctx, G4A_COMPUTE, "compute: empty model capacity");
    if (max_tokens > ctx->max_positions)
        return fail(ctx, G4A_COMPUTE, "compute: max_tokens %d exceeds the context's %d RoPE positions", max_tokens,
                    ctx->max_positions);
    if (!w->token_embd) return fail(ctx, G4A_MISSING_WEIGHT, "missing weight `token_embd.weight`");
    if (!w->output_norm) return fail(ctx, G4A_MISSING_WEIGHT, "missing weight `output_norm.weight`");
    if (w->ple_dim > 0 && !w->ple_token_embd)
        return fail(ctx, G4A_MISSING_WEIGHT, "missing weight `per_layer_token_embd.weight`");
    if (w->ple_dim > 0 && !w->ple_model_proj)
        return fail(ctx, G4A_MISSING_WEIGHT, "missing weight `per_layer_model_proj.weight`");
    if (w->ple_dim > 0 && !w->ple_proj_norm)
        return fail(ctx, G4A_MISSING_WEIGHT, "missing weight `per_layer_proj_norm.weight`");

    auto *m = new g4a_model();
    m->ctx = ctx;
    m->w = *w;
    m->S = max_seqs;
    m->T = max_tokens;
    m->L = hp.n_layers;
    m->d = w->d_model;
    m->d_ff = w->d_ff;
    m->ple = w->ple_dim;
    m->vocab = w->vocab_size;
    m->len.assign(max_seqs, 0);
    m->source.resize(m->L);
    m->hd.resize(m->L);
    m->global.resize(m->L);
    for (int l = 0; l < m->L; l++) {
        int32_t src = -1, detail = 0;
        const int rc = g4a_kv_source_layer(&hp, l, &src, &detail);
        if (rc != G4A_OK) {
            g4a_model_destroy(m);
            return fail(ctx, rc, "layer %d has no KV source (kind %d)", l, detail);
        }
        m->source[l] = src;
        m->hd[l] = g4a_head_dim(&hp, l);
        m->global[l] = g4a_layer_is_global(&hp, l);
        if (const char *name = missing_weight(*w, l, src == l)) {
            g4a_model_destroy(m);
            return fail(ctx, G4A_MISSING_WEIGHT, "missing weight `blk.%d.%s.weight`", l, name);
        }
    }
    m->hd_max = std::max(hp.head_dim_local, hp.head_dim_global);
    m->qd_max = kHeads * m->hd_max;
    m->cmax = std::max(std::max(m->d, m->d_ff), std::max(m->qd_max, m->ple));
    // Up to kExactMaxRows positions every task is one CTA in the reference's
    // order of operations (bit-exact logits); longer caches split tasks
    // across CTAs (split-KV, within the decode tolerance).
    m->exact = max_tokens <= kExactMaxRows;
    if (m->exact) m->rows_per_item = kExactRowsPerItem;
    const int32_t per_item = m->rows_per_item;
    m->ms_local = (std::min(hp.sliding_window, max_tokens) + per_item - 1) / per_item;
    m->ms_global = (max_tokens + per_item - 1) / per_item;
    const int32_t ms = std::max(m->ms_local, m->ms_global);
    const size_t S = (size_t)max_seqs;
    // Rows of a step: a prompt chunk takes up to kChunkRows positions (all
    // sequences' together; G4A_CHUNK_ROWS=<n> in the environment sets
    // another bound) in exact mode; the split-KV path keeps one partial
    // buffer per sequence, so its steps hold S rows.
    int64_t chunk_rows = kChunkRows;
    if (const char *cr = std::getenv("G4A_CHUNK_ROWS")) chunk_rows = std::max(1L, std::strtol(cr, nullptr, 10));
    m->R = m->exact ? (int32_t)std::max<int64_t>(max_seqs, std::min<int64_t>(chunk_rows, (int64_t)max_seqs * max_tokens))
                    : max_seqs;
    const size_t R = (size_t)m->R;

    bool ok = cudaStreamCreateWithFlags(&m->st, cudaStreamNonBlocking) == cudaSuccess &&
              cudaEventCreateWithFlags(&m->ev, cudaEventDisableTiming) == cudaSuccess &&
              cudaHostAlloc(reinterpret_cast<void **>(&m->h_in), (3 * R + S) * sizeof(int32_t),
                            cudaHostAllocDefault) == cudaSuccess &&
              cudaHostAlloc(reinterpret_cast<void **>(&m->h_out), S * sizeof(unsigned long long),
                            cudaHostAllocDefault) == cudaSuccess &&
              cudaHostAlloc(reinterpret_cast<void **>(&m->h_err), sizeof(int32_t), cudaHostAllocDefault) == cudaSuccess;
    if (ok) {
        ok = (m->d_in = dalloc<int32_t>(m, 3 * R + S)) &&
             (m->x = dalloc<float>(m, R * m->d)) && (m->y = dalloc<float>(m, R * m->d)) &&
             (m->q = dalloc<float>(m, R * m->qd_max)) && (m->att = dalloc<float>(m, R * m->qd_max)) &&
             (m->k = dalloc<float>(m, R * m->hd_max)) && (m->v = dalloc<float>(m, R * m->hd_max)) &&
             (m->gated = dalloc<float>(m, R * m->d_ff)) && (m->gate = dalloc<float>(m, R * std::max(m->ple, 1))) &&
             (m->P = dalloc<float>(m, R * m->L * std::max(m->ple, 1))) &&
             (m->pli = dalloc<float>(m, R * m->L * std::max(m->ple, 1))) &&
             (m->logits = dalloc<float>(m, S * m->vocab)) && (m->xq = dalloc<int8_t>(m, R * m->cmax)) &&
             (m->xs = dalloc<float>(m, R * m->cmax / 32)) && (m->xq_out = dalloc<int8_t>(m, S * m->d)) &&
             (m->xs_out = dalloc<float>(m, S * m->d / 32)) && (m->d_layers = dalloc<E2bLayerDesc>(m, m->L)) &&
             (m->d_tasks = dalloc<DecodeTask>(m, (size_t)m->L * R)) &&
             (m->d_items_local = dalloc<DecodeItem>(m, R * m->ms_local)) &&
             (m->d_items_global = dalloc<DecodeItem>(m, R * m->ms_global)) &&
             (m->part_o = dalloc<float>(m, R * ms * kHeads * m->hd_max)) &&
             (m->part_ml = dalloc<float>(m, R * ms * 2 * kHeads)) && (m->tickets = dalloc<unsigned>(m, R)) &&
             (m->scores = dalloc<float>(m, m->exact ? R * kHeads * max_tokens : 1)) &&
             (m->d_best = dalloc<unsigned long long>(m, S));
    }
    // K/V caches of the owner layers: [max_seqs][max_tokens][hd] f32 each
    std::vector<E2bLayerDesc> desc(m->L);
    std::vector<float *> kc(m->L, nullptr), vc(m->L, nullptr);
    for (int l = 0; ok && l < m->L; l++) {
        if (m->source[l] != l) continue;
        const size_t n = S * max_tokens * m->hd[l];
        ok = (kc[l] = dalloc<float>(m, n)) && (vc[l] = dalloc<float>(m, n));
    }
    if (!ok) {
        g4a_model_destroy(m);
        return fail(ctx, G4A_CUDA, "compute: out of device memory for the decoder");
    }
    const char *no_graph = std::getenv("G4A_NO_GRAPH");
    m->use_graphs = !(no_graph && no_graph[0] == '1');
    const char *no_pdl = std::getenv("G4A_NO_PDL");
    m->pdl = !(no_pdl && no_pdl[0] == '1');
    m->k_cache.resize(m->L);
    m->v_cache.resize(m->L);
    for (int l = 0; l < m->L; l++) {
        m->k_cache[l] = kc[m->source[l]];
        m->v_cache[l] = vc[m->source[l]];
        desc[l].q_w = w->layers[l].attn_q_norm;
        desc[l].k_w = w->layers[m->source[l]].attn_k_norm;
        desc[l].k_cache = kc[m->source[l]];
        desc[l].v_cache = vc[m->source[l]];
        desc[l].hd = m->hd[l];
        desc[l].global = m->global[l];
        desc[l].owner = m->source[l] == l;
    }
    cudaError_t e = cudaMemcpy(m->d_layers, desc.data(), desc.size() * sizeof(E2bLayerDesc), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemset(m->tickets, 0, R * sizeof(unsigned));
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        g4a_model_destroy(m);
        return cuda_fail(ctx, e, "model setup");
    }
    *out = m;
    return G4A_OK;
}

extern "C" int g4a_model_clear(g4a_model *m, int32_t seq) {
    if (!m) return G4A_COMPUTE;
    if (seq < 0 || seq >= m->S) return fail(m->ctx, G4A_COMPUTE, "compute: sequence %d out of range", seq);
    m->len[seq] = 0;  // rows past the length are never read before they are rewritten
    return G4A_OK;
}

extern "C" int g4a_model_len(const g4a_model *m, int32_t seq, int32_t *len) {
    if (!m || !len || seq < 0 || seq >= m->S) return G4A_COMPUTE;
    *len = m->len[seq];
    return G4A_OK;
}

namespace {

// Runs a step whose inputs are in h_in, after the caller's work on the
// context's stream, and reads its flags.
int submit(g4a_model *m, int32_t n, int32_t n_out, bool chunk, int32_t cl = 1) {
    g4a_ctx *ctx = m->ctx;
    G4A_CUDA_TRY(ctx, cudaEventRecord(m->ev, ctx->stream));
    G4A_CUDA_TRY(ctx, cudaStreamWaitEvent(m->st, m->ev, 0));
    const int rc = run_step(m, n, n_out, chunk, cl);
    if (rc) {
        cudaStreamSynchronize(m->st);
        return rc;
    }
    G4A_CUDA_TRY(ctx, cudaStreamSynchronize(m->st));
    m->last_n = n_out;
    const int32_t flags = *m->h_err;
    if (flags) {
        cudaMemset(ctx->d_err, 0, sizeof(int));
        // an aborted step may leave split-task tickets counted
        cudaMemset(m->tickets, 0, (size_t)m->R * sizeof(unsigned));
        ctx->err_epoch++;
        if (flags & 1) return fail(ctx, G4A_NONFINITE, "compute: softmax input is not finite");
        return fail(ctx, G4A_TIMEOUT, "compute: a device wait timed out (flags %d)", flags);
    }
    return G4A_OK;
}

// Sequence ids distinct and in range; tokens in the vocabulary (model.rs:378);
// room for `adding` more positions in every sequence.
int check_batch(g4a_model *m, int32_t n, const int32_t *seq_ids, const int32_t *tokens, int64_t n_tokens,
                int32_t adding) {
    g4a_ctx *ctx = m->ctx;
    std::vector<char> used(m->S, 0);
    for (int i = 0; i < n; i++) {
        const int32_t s = seq_ids[i];
        if (s < 0 || s >= m->S || used[s]) return fail(ctx, G4A_COMPUTE, "compute: bad or repeated sequence id %d", s);
        used[s] = 1;
        if ((int64_t)m->len[s] + adding > m->T)  // ContextMemory::view past capacity
            return fail(ctx, G4A_CONTEXT_TOO_LONG, "context too long: got %lld, max %d",
                        (long long)m->len[s] + adding, m->T);
    }
    for (int64_t i = 0; i < n_tokens; i++)
        if (tokens[i] < 0 || tokens[i] >= m->vocab)
            return fail(ctx, G4A_COMPUTE, "compute: token %d exceeds vocabulary", tokens[i]);
    return G4A_OK;
}

}  // namespace

extern "C" int g4a_model_step(g4a_model *m, int32_t n, const int32_t *seq_ids, const int32_t *tokens, int32_t *next) {
    if (!m) return G4A_COMPUTE;
    g4a_ctx *ctx = m->ctx;
    cudaSetDevice(ctx->device);
    if (n < 1 || n > m->S || !seq_ids || !tokens)
        return fail(ctx, G4A_COMPUTE, "compute: step of %d sequences (capacity %d)", n, m->S);
    int rc = check_batch(m, n, seq_ids, tokens, n, 1);
    if (rc) return rc;
    for (int i = 0; i < n; i++) {
        m->h_in[i] = seq_ids[i];
        m->h_in[n + i] = tokens[i];
        m->h_in[2 * n + i] = m->len[seq_ids[i]];
    }
    if ((rc = submit(m, n, n, false))) return rc;
    for (int i = 0; i < n; i++) m->len[seq_ids[i]]++;
    if (next)
        for (int i = 0; i < n; i++) next[i] = (int32_t)(m->h_out[i] & 0xFFFFFFFFull);
    return G4A_OK;
}

extern "C" int g4a_model_prefill(g4a_model *m, int32_t n, const int32_t *seq_ids, const int32_t *tokens, int32_t len,
                                 int32_t *next) {
    if (!m) return G4A_COMPUTE;
    g4a_ctx *ctx = m->ctx;
    cudaSetDevice(ctx->device);
    if (n < 1 || n > m->S || len < 1 || !seq_ids || !tokens)
        return fail(ctx, G4A_COMPUTE, "compute: prompt of %d tokens for %d sequences (capacity %d)", len, n, m->S);
    int rc = check_batch(m, n, seq_ids, tokens, (int64_t)n * len, len);
    if (rc) return rc;
    // chunks of C positions of every sequence, rows sequence-major
    const int32_t C = std::max<int32_t>(1, m->R / n);
    for (int32_t c0 = 0; c0 < len; c0 += C) {
        const int32_t cl = std::min(C, len - c0), rows = n * cl;
        const bool last = c0 + cl == len;
        for (int i = 0; i < n; i++) {
            const int32_t s = seq_ids[i];
            for (int j = 0; j < cl; j++) {
                const int32_t r = i * cl + j;
                m->h_in[r] = s;
                m->h_in[rows + r] = tokens[(size_t)i * len + c0 + j];
                m->h_in[2 * rows + r] = m->len[s] + j;
            }
            m->h_in[3 * rows + i] = i * cl + cl - 1;  // the sequence's last row of the chunk
        }
        // one position per sequence: a decode step (its graph)
        rc = cl == 1 ? submit(m, n, n, false) : submit(m, rows, last ? n : 0, true, cl);
        if (rc) return rc;
        for (int i = 0; i < n; i++) m->len[seq_ids[i]] += cl;
    }
    if (next)
        for (int i = 0; i < n; i++) next[i] = (int32_t)(m->h_out[i] & 0xFFFFFFFFull);
    return G4A_OK;
}

extern "C" int g4a_model_logits(g4a_model *m, const float **logits_dev) {
    if (!m || !logits_dev) return G4A_COMPUTE;
    *logits_dev = m->logits;
    return G4A_OK;
}

extern "C" int g4a_model_set_eos(g4a_model *m, const int32_t *ids, int32_t n) {
    if (!m || n < 0 || (n && !ids)) return G4A_COMPUTE;
    m->eos.assign(ids, ids + n);
    return G4A_OK;
}

extern "C" int g4a_model_generate(g4a_model *m, int32_t n, const int32_t *prompts, int32_t prompt_len, int32_t max_new,
                                  int32_t max_context, int32_t *out) {
    if (!m) return G4A_COMPUTE;
    g4a_ctx *ctx = m->ctx;
    if (n < 1 || n > m->S || prompt_len < 0 || max_new < 0 || (prompt_len && !prompts) || (max_new && !out))
        return fail(ctx, G4A_COMPUTE, "compute: invalid generate arguments");
    if (prompt_len > max_context)  // generate.rs:23-28
        return fail(ctx, G4A_CONTEXT_TOO_LONG, "context too long: got %d, max %d", prompt_len, max_context);
    if (max_new == 0) return G4A_OK;
    if (prompt_len == 0) return fail(ctx, G4A_COMPUTE, "generation requires at least one prompt token");
    std::vector<int32_t> ids(n), next(n), act_ids, act_tok, act_next;
    for (int i = 0; i < n; i++) {
        ids[i] = i;
        m->len[i] = 0;  // clear_context
    }
    for (size_t e = 0; e < (size_t)n * max_new; e++) out[e] = -1;  // slots after an eos stay -1
    int rc;
    // the prompt (generate.rs:38-42, one position per forward pass there) in
    // chunks of many positions; the same logits
    if ((rc = g4a_model_prefill(m, n, ids.data(), prompts, prompt_len, next.data()))) return rc;
    std::vector<char> active(n, 1);
    for (int index = 0; index < max_new; index++) {  // generate.rs:45-70
        if (prompt_len + index >= max_context)
            return fail(ctx, G4A_CONTEXT_TOO_LONG, "context too long: got %d, max %d", prompt_len + index + 1,
                        max_context);
        act_ids.clear();
        act_tok.clear();
        for (int i = 0; i < n; i++) {
            if (!active[i]) continue;
            out[(size_t)i * max_new + index] = next[i];
            if (std::find(m->eos.begin(), m->eos.end(), next[i]) != m->eos.end()) {
                active[i] = 0;  // the eos token is kept, then the sequence stops
                continue;
            }
            act_ids.push_back(i);
            act_tok.push_back(next[i]);
        }
        if (index + 1 == max_new || act_ids.empty()) break;
        act_next.resize(act_ids.size());
        if ((rc = g4a_model_step(m, (int32_t)act_ids.size(), act_ids.data(), act_tok.data(), act_next.data())))
            return rc;
        for (size_t j = 0; j < act_ids.size(); j++) next[act_ids[j]] = act_next[j];
    }
    return G4A_OK;
}

extern "C" int g4a_model_kv_view(const g4a_model *m, int32_t seq, int32_t layer, int32_t len, float *keys_dev,
                                 float *values_dev) {
    if (!m) return G4A_COMPUTE;
    g4a_ctx *ctx = m->ctx;
    cudaSetDevice(ctx->device);
    if (seq < 0 || seq >= m->S || layer < 0 || layer >= m->L || len < 0 || (len && (!keys_dev || !values_dev)))
        return fail(ctx, G4A_COMPUTE, "compute: invalid view arguments");
    const int32_t src = m->source[layer];
    if (len > m->len[seq])  // context_memory.rs:53-69
        return fail(ctx, G4A_CONTEXT_TOO_LONG, "context too long: got %d, max %d", len, m->len[seq]);
    const size_t hd = (size_t)m->hd[src], off = (size_t)seq * m->T * hd, bytes = (size_t)len * hd * sizeof(float);
    G4A_CUDA_TRY(ctx, cudaMemcpyAsync(keys_dev, m->k_cache[layer] + off, bytes, cudaMemcpyDeviceToDevice, ctx->stream));
    G4A_CUDA_TRY(ctx, cudaMemcpyAsync(values_dev, m->v_cache[layer] + off, bytes, cudaMemcpyDeviceToDevice,
                                      ctx->stream));
    return G4A_OK;
}
