/*
 * g4attn — Gemma 4 E2B attention on B200 (sm_100a), C ABI.
 *
 * This is the drop-in boundary for gemma4-rs's attention path. Everything a
 * Rust `llm-backend-cuda` crate would bind is declared here: plain C types,
 * explicit lengths, an int status per call. No CUDA or torch type appears in
 * a signature (streams are passed as `void *`).
 *
 * Reference interfaces replaced (paths relative to the gemma4-rs workspace):
 *   crates/llm-gemma4/src/impl_/model.rs:348  attend(q, keys, values, n_heads, n_kv_heads, scale)
 *   crates/llm-gemma4/src/impl_/model.rs:393-410  the attention block of TransformerSpec::layer
 *   crates/llm-gemma4/src/impl_/model.rs:283-304  norm_heads / rope_heads (fused into decode)
 *   crates/llm-eng/src/context_memory.rs:11-18  ContextMemory::{append, view, clear}
 *   crates/llm-gemma4/src/eng/mod.rs:10-36,71-90  window policies, kv_source_layer
 *   crates/llm-gemma4/src/idea/mod.rs:48-68,140-165  E2B hyperparameters, layer kinds, p-RoPE factors
 *
 * Memory: pointers named `*_dev` are device pointers owned by the caller;
 * `*_host` pointers are host memory. The context owns the RoPE tables, the
 * split-KV scratch and the KV pages.
 *
 * Threading: one context drives one CUDA stream; calls on a context (and on
 * the caches made from it) are not thread-safe, as `&mut self` in the
 * reference's `layer`. Device work is asynchronous: a call returns once its
 * kernels are queued. Shape, position and capacity errors are returned
 * immediately; a non-finite softmax is detected on the device and returned
 * by the next g4a_sync (the reference returns it from `attend`).
 */
#ifndef G4ATTN_H
#define G4ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* Status codes. 1-5 map 1:1 onto crates/llm-eng/src/error.rs:3-15 EngError. */
typedef enum g4a_status {
    G4A_OK = 0,
    G4A_CONTEXT_TOO_LONG = 1, /* EngError::ContextTooLong { got, max } */
    G4A_MISSING_LAYER = 2,    /* EngError::MissingLayer(layer) */
    G4A_MISSING_WEIGHT = 3,   /* EngError::MissingWeight (a required norm weight is NULL) */
    G4A_COMPUTE = 4,          /* EngError::Compute: invalid shapes or inputs */
    G4A_NONFINITE = 5,        /* EngError::Compute("softmax input is not finite"), model.rs:363 */
    G4A_BAD_LAYER = 6,        /* KvShareError, crates/llm-gemma4/src/eng/mod.rs:38-43 */
    G4A_CUDA = 7,             /* a CUDA runtime call failed */
    G4A_NCCL = 8,             /* a collective failed */
    G4A_TIMEOUT = 9,          /* a bounded wait ran out */
    G4A_OUT_OF_PAGES = 10     /* the paged KV cache has no free page */
} g4a_status;

/* Storage type of the paged KV cache. */
typedef enum g4a_kv_dtype { G4A_KV_F32 = 0, G4A_KV_F16 = 1 } g4a_kv_dtype;

/* Attention-relevant fields of Gemma4HyperParams (idea/mod.rs:16-34). */
typedef struct g4a_hparams {
    int32_t n_layers, n_heads, n_kv_heads, head_dim_local, head_dim_global;
    int32_t sliding_window, shared_kv_layers;
    float local_rope_base, global_rope_base, global_p, rms_norm_eps;
} g4a_hparams;

typedef struct g4a_ctx g4a_ctx;
typedef struct g4a_kv g4a_kv;

/* ---- hyperparameters and policies (host only, no device work) ---------- */

/* idea/mod.rs:48-68 Gemma4HyperParams::e2b. */
void g4a_hparams_e2b(g4a_hparams *out);
/* idea/mod.rs:148-156 layer_attention_kind: 1 = global, 0 = sliding window. */
int g4a_layer_is_global(const g4a_hparams *hp, int32_t layer);
/* idea/mod.rs:140-145 head_dim. */
int32_t g4a_head_dim(const g4a_hparams *hp, int32_t layer);
/* eng/mod.rs:71-90 kv_source_layer. On G4A_BAD_LAYER, *detail (if non-NULL)
 * is 1 LayerOutOfRange, 2 TooManySharedLayers, 3 NoEarlierLayerOfSameKind. */
int g4a_kv_source_layer(const g4a_hparams *hp, int32_t layer, int32_t *source, int32_t *detail);
/* eng/mod.rs:10-12 windowed_len: [seq_len - window saturating, seq_len). */
void g4a_windowed_len(int64_t seq_len, int64_t window, int64_t *lo, int64_t *hi);
/* idea/mod.rs:162-165 proportional_rope_freq_factors: head_dim/2 values. */
void g4a_proportional_rope_freq_factors(int32_t head_dim, float p, float *out_host);

/* ---- context ---------------------------------------------------------- */

/* Creates a context on `device`. rope_freqs_host holds head_dim_global/2
 * per-pair divisors for global layers (the GGUF `rope_freqs.weight`,
 * model.rs:298); NULL derives them from hp->global_p. max_positions bounds
 * the positions decode and append accept (RoPE tables are built for
 * [0, max_positions)). */
int g4a_ctx_create(int device, const g4a_hparams *hp, const float *rope_freqs_host,
                   int32_t max_positions, g4a_ctx **out);
void g4a_ctx_destroy(g4a_ctx *ctx);
/* The message of the last failed call on this context (EngError's Display). */
const char *g4a_last_error(const g4a_ctx *ctx);
/* Sets the cudaStream_t all later calls queue on (NULL = legacy default). */
int g4a_ctx_set_stream(g4a_ctx *ctx, void *cuda_stream);
/* Waits for queued work and returns G4A_NONFINITE if a softmax since the
 * last g4a_sync saw a non-finite input (the flag is then cleared). */
int g4a_sync(g4a_ctx *ctx);

/* Per-kernel device timing (no counterpart in the reference, which logs one
 * wall-clock line per token, crates/llm-cli/src/main.rs:82-90): when enabled,
 * every kernel launch of the context is bracketed by CUDA events on its
 * stream. Enabling (or disabling) clears the totals; reading waits for the
 * stream and returns the summed device milliseconds and launch count. */
typedef enum g4a_kernel {
    G4A_K_DECODE_PREP = 0,     /* f16 decode: q blocks + appended rows */
    G4A_K_DECODE_MAIN = 1,     /* f16 decode: TMA / tensor-core attention */
    G4A_K_DECODE_COMBINE = 2,  /* f16 decode: merge of split tasks */
    G4A_K_DECODE_SPLITKV = 3,  /* f32 caches and g4a_attend */
    G4A_K_PREFILL = 4,         /* tcgen05 prefill (with its V conversion) */
    G4A_K_MATVEC_Q8 = 5,       /* Q8_0 mat-vec family (with its activation quantization) */
    G4A_K_CP_EXCHANGE = 6,     /* g4a_cp_prefill: NCCL collectives (gathers, all-reduce, reduce-scatter) */
    G4A_K_CP_ATTEND_LOCAL = 7, /* g4a_cp_prefill: attention over this rank's own data */
    G4A_K_CP_ATTEND_REMOTE = 8,/* g4a_cp_prefill: attention over exchanged data */
    G4A_K_CP_MERGE = 9,        /* g4a_cp_prefill: log-sum-exp merges, weights, packing */
    G4A_K_COPY_IN = 10,        /* g4a_decode_host: host-to-device copies of the inputs */
    G4A_K_COPY_OUT = 11,       /* g4a_decode_host: device-to-host copies of the outputs */
    G4A_K_HOST_ISSUE = 12,     /* g4a_decode_host: host time from entry until everything is queued */
    G4A_K_HOST_WAIT = 13,      /* g4a_decode_host: host time blocked in the final synchronisation */
    G4A_K_COUNT = 14
} g4a_kernel;
int g4a_profile_enable(g4a_ctx *ctx, int enable);
int g4a_profile_read(g4a_ctx *ctx, int32_t kernel, double *total_ms, int64_t *launches);

/* For tests of failure handling (no reference counterpart; the reference's
 * failures are EngError results, crates/llm-eng/src/error.rs:3-15): the next
 * launch of `kernel` (G4A_K_DECODE_MAIN: the f16 paged decode, or
 * G4A_K_PREFILL) on this context waits, before it loads anything, on a bit of
 * the context's device error word that nothing sets; the wait gives up after
 * about 2 ms as any bounded wait of the kernel gives up, records the
 * time-out and skips the kernel's work. The call's g4a_sync (or
 * g4a_decode_host itself) then returns G4A_TIMEOUT and the context stays
 * usable. Other kernels return G4A_COMPUTE. */
int g4a_debug_stall(g4a_ctx *ctx, int32_t kernel);

/* ---- attention primitive ---------------------------------------------- */

/* model.rs:348-366 attend: grouped-query attention for one query position.
 * q_dev [n_heads*head_dim] f32; keys_dev/values_dev [len][n_kv_heads*head_dim]
 * f32 rows (the reference's concatenated rows); out_dev [n_heads*head_dim].
 * len == 0 is reported as G4A_NONFINITE like the reference (empty softmax). */
int g4a_attend(g4a_ctx *ctx, const float *q_dev, const float *keys_dev, const float *values_dev,
               int64_t len, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, float scale,
               float *out_dev);

/* No counterpart in the reference. The same attention as g4a_attend for the
 * E2B shape (n_heads 8, n_kv_heads 1, head_dim 256 or 512), for callers that
 * cannot allocate device memory when they call it (e.g. a server that gave
 * its device memory to its own pools at start-up). It allocates nothing: its
 * scratch is a file-scope device array of about 1 MiB (64 row ranges x 8
 * heads x 512 columns of f32 plus their max/sum), held by every GPU that
 * loads the library until exit. Other shapes return G4A_COMPUTE. The work
 * runs on the device cuda_stream belongs to; the first call on a device looks
 * the array up there (making that device current for the call); make it
 * before any stream capture. Each call clears the array's arrival counter
 * with an async memset on cuda_stream before its kernel. Calls share the
 * array, so calls that overlap on the GPU race; queue them on one stream. No
 * context is used, and a non-finite softmax shows as NaN in out_dev. */
int g4a_attend_static(void *cuda_stream, const float *q_dev, const float *keys_dev,
                      const float *values_dev, int64_t len, int32_t n_heads, int32_t n_kv_heads,
                      int32_t head_dim, float scale, float *out_dev);

/* ---- paged KV cache: ContextMemory (context_memory.rs:11-18) ------------ */

/* A paged cache for n_seqs sequences of up to max_tokens rows per layer.
 * page_tokens rows per page (64 recommended); n_pages 0 = enough for every
 * sequence at max_tokens. layers_host lists the owner layers to hold
 * (kv_source_layer(l) == l); NULL holds every owner layer. Pages are shared
 * by index across layers: a sequence's logical page j is one physical page in
 * every held layer's pool. */
int g4a_kv_create(g4a_ctx *ctx, int32_t n_seqs, int32_t max_tokens, int32_t page_tokens,
                  int32_t n_pages, int32_t dtype, const int32_t *layers_host, int32_t n_layers,
                  g4a_kv **out);
void g4a_kv_destroy(g4a_kv *kv);
/* ContextMemory::clear (context_memory.rs:83-85) for one sequence, or all
 * when seq < 0; frees its pages. */
int g4a_kv_clear(g4a_kv *kv, int32_t seq);
/* Rows stored for (seq, layer). */
int g4a_kv_len(const g4a_kv *kv, int32_t seq, int32_t layer, int64_t *len);
/* ContextMemory::append (context_memory.rs:44-51) of n_rows already
 * normalised and rotated rows: k_dev/v_dev [n_rows][n_kv_heads*head_dim] f32,
 * stored in the cache's dtype. */
int g4a_kv_append(g4a_kv *kv, int32_t seq, int32_t layer, const float *k_dev, const float *v_dev,
                  int64_t n_rows);
/* ContextMemory::view (context_memory.rs:53-69): copies rows [0, len) of
 * (seq, layer) out as f32. MissingLayer / ContextTooLong as the reference. */
int g4a_kv_view(const g4a_kv *kv, int32_t seq, int32_t layer, int64_t len, float *keys_dev,
                float *values_dev);
/* The K/V half of model.rs:400-405 for n_tokens consecutive tokens of one
 * sequence: k = rope(rms_norm(k_raw, k_norm_w)), v = rms_norm(v_raw), appended
 * at positions len .. len+n_tokens-1. k_raw_dev/v_raw_dev [n_tokens][hd] f32. */
int g4a_kv_append_tokens(g4a_kv *kv, int32_t seq, int32_t layer, const float *k_raw_dev,
                         const float *v_raw_dev, const float *k_norm_w_dev, int64_t n_tokens);

/* ---- fused decode step: model.rs:393-410 without the projections ------- */

/* One layer's inputs for a decode batch. q_raw_dev [n][n_heads*hd] f32 are
 * the attn_q projections; k_raw_dev/v_raw_dev [n][hd] f32 the attn_k/attn_v
 * projections (ignored, may be NULL, for KV-shared layers); q_norm_w_dev /
 * k_norm_w_dev [hd] the attn_q_norm / attn_k_norm weights; out_dev
 * [n][n_heads*hd] f32 receives the attention output (attn_output's input). */
typedef struct g4a_decode_layer {
    int32_t layer;
    const float *q_raw_dev;
    const float *k_raw_dev;
    const float *v_raw_dev;
    const float *q_norm_w_dev;
    const float *k_norm_w_dev;
    float *out_dev;
} g4a_decode_layer;

/* Decode step for n_seqs sequences over n_layers layers in one launch. For
 * sequence i (cache row seq_ids_host[i]) at position positions_host[i] and
 * each listed layer: q-norm + RoPE, and on KV-owning layers k-norm, v-norm,
 * k RoPE and append; then attention over the window of the source layer's
 * cache (local: the last `sliding_window` rows up to the position; global:
 * all), scale 1. A call may not list a shared layer together with its
 * source layer (the shared layer would race the append). */
int g4a_decode(g4a_ctx *ctx, g4a_kv *kv, int32_t n_layers, const g4a_decode_layer *layers_host,
               int32_t n_seqs, const int32_t *seq_ids_host, const int32_t *positions_host);

/* g4a_decode for a caller whose vectors live in host memory, as the
 * reference's attend (model.rs:345-366) takes host slices: q_raw_host
 * [n][n_heads*hd], k_raw_host/v_raw_host [n][hd] (owner layers; may be NULL
 * on KV-shared layers) are copied in, the step runs on the context's stream,
 * out_host [n][n_heads*hd] is copied back, and the call returns when it is
 * there, with the device's softmax/timeout flags checked (G4A_NONFINITE,
 * G4A_TIMEOUT). For a small step (up to 256 KB of q/k/v/out, e.g. one
 * sequence) whose buffers are all page-locked memory the device can address
 * (cudaHostAlloc'd or registered, under unified addressing), the step's
 * kernels read the inputs and write the outputs in place over the bus, all
 * layers in one launch, with no staging copies. Otherwise q is copied into
 * device slots of the context (a copy stream of the context; pageable memory
 * is staged by the driver), as are k and v unless both are page-locked memory
 * the device can address, which the prep kernel then reads in place; all
 * layers run in one launch set once the copies are in; outputs in page-locked
 * memory the device can address are written in place by the kernels, other
 * outputs are copied back after them. The norm weights stay device
 * pointers (model weights are resident). A rejected call leaves the cache and
 * the outputs untouched. */
typedef struct g4a_decode_layer_host {
    int32_t layer;
    const float *q_raw_host;
    const float *k_raw_host;
    const float *v_raw_host;
    const float *q_norm_w_dev;
    const float *k_norm_w_dev;
    float *out_host;
} g4a_decode_layer_host;
int g4a_decode_host(g4a_ctx *ctx, g4a_kv *kv, int32_t n_layers, const g4a_decode_layer_host *layers_host,
                    int32_t n_seqs, const int32_t *seq_ids_host, const int32_t *positions_host);

/* A decode step staged for repeated launches: g4a_decode's validation, page
 * allocation and cache-length update happen here once; the plan owns device
 * copies of its work list and its split-KV scratch. */
typedef struct g4a_plan g4a_plan;
int g4a_decode_plan(g4a_ctx *ctx, g4a_kv *kv, int32_t n_layers, const g4a_decode_layer *layers_host,
                    int32_t n_seqs, const int32_t *seq_ids_host, const int32_t *positions_host,
                    g4a_plan **out);
/* Launches a staged step on the context's stream (kernel launches only, no
 * host-device copies, so it can be captured into a CUDA graph). Running a
 * plan again recomputes the same step and rewrites the same appended rows. */
int g4a_plan_run(g4a_plan *plan);
void g4a_plan_destroy(g4a_plan *plan);

/* ---- prefill attention (tcgen05 tensor cores) -------------------------- */

/* One causal attention problem over bf16 inputs that are already normalised
 * and rotated: q [n_q][n_heads][hd], k/v [n_kv][hd] (1 KV head). Query row i
 * has absolute position q_pos0 + i and sees key row j (position kv_pos0 + j)
 * when key_pos <= q_pos and, for window > 0, q_pos - key_pos < window
 * (eng/mod.rs:10-12 applied per position, as the reference's token-at-a-time
 * prefill does). out [n_q][n_heads][hd] f32 is normalised; lse (optional,
 * [n_q][n_heads] f32) receives the natural-log sum of exp(scores) for merging
 * partial results; rows that see no key get out 0 and lse -inf. */
typedef struct g4a_prefill_problem {
    int32_t head_dim;  /* 256 or 512 */
    int32_t window;    /* 0 = global (full causal) */
    int32_t n_q, q_pos0, n_kv, kv_pos0;
    const void *q_dev; /* bf16 */
    const void *k_dev; /* bf16 */
    const void *v_dev; /* bf16 */
    float *out_dev;
    float *lse_dev;
} g4a_prefill_problem;

/* Runs n problems (e.g. the 35 layers of a prompt) in one launch. */
int g4a_prefill(g4a_ctx *ctx, int32_t n, const g4a_prefill_problem *problems_host);

/* Merges partial attention results over disjoint key sets (log-sum-exp):
 * out = sum_i exp(lse_i - L) * out_i with L = log sum_i exp(lse_i).
 * parts_out_dev / parts_lse_dev hold n_parts arrays of rows*n_heads*hd and
 * rows*n_heads; results go to out_dev / lse_dev (lse_dev may be NULL). */
int g4a_lse_merge(g4a_ctx *ctx, int32_t n_parts, const float *const *parts_out_host,
                  const float *const *parts_lse_host, int64_t rows, int32_t n_heads,
                  int32_t head_dim, float *out_dev, float *lse_dev);

/* ---- context-parallel prefill of one long global layer over NCCL -------
 * Replaces the reference's prompt loop on a global layer
 * (crates/llm-gemma4/src/impl_/generate.rs:37-41, each position through
 * model.rs:326-366 over all earlier keys, eng/mod.rs:33-35) for a sequence
 * split over the W ranks of an NCCL communicator. The sequence of T tokens is
 * cut into 2W equal chunks of c = T / (2W) tokens; rank r holds chunks r and
 * 2W-1-r ("zigzag", equal causal work per rank) of the queries, keys and
 * values, already normalised and rotated, and receives the attention output
 * of those two chunks. Every rank calls with the same schedule, head_dim and
 * seq_len.
 *
 *  G4A_CP_KV_SHARDS: keys and values stay on their rank. The queries are
 *    gathered (all-gather and point-to-point), each rank attends every query
 *    row that sees its two key chunks (rows of its own queries first, while
 *    the gather runs), and the partial results are merged across ranks by
 *    log-sum-exp: an all-reduce (MAX) of the per-row maxima, then a
 *    reduce-scatter (SUM) of the weighted outputs and weights, which hands
 *    each rank the rows of its own chunks.
 *  G4A_CP_GATHER_KV: the key/value chunks are gathered (all-gather and
 *    point-to-point, on a second stream) while each rank attends its two
 *    diagonal blocks; then its query chunks against all earlier keys; the
 *    two partials of each chunk are merged by log-sum-exp on the device.
 *
 * nccl_comm is the caller's ncclComm_t (for example the communicator of a
 * torch ProcessGroupNCCL) of the libnccl.so.2 already loaded in the process
 * (loaded on first use if none is). The call queues everything on the
 * context's stream (and a stream of its own that it joins back) and returns;
 * g4a_cp_wait or g4a_sync waits. q_dev [2][c][n_heads][hd], k_dev / v_dev
 * [2][c][hd] bf16 (chunk r first); out_dev [2][c][n_heads][hd] f32. The
 * context keeps the exchange buffers between calls. */
typedef enum g4a_cp_schedule { G4A_CP_KV_SHARDS = 0, G4A_CP_GATHER_KV = 1 } g4a_cp_schedule;
typedef struct g4a_cp_problem {
    int32_t head_dim; /* 256 or 512 */
    int32_t seq_len;  /* T, a multiple of 2 x ranks */
    const void *q_dev;
    const void *k_dev;
    const void *v_dev;
    float *out_dev;
} g4a_cp_problem;
int g4a_cp_prefill(g4a_ctx *ctx, void *nccl_comm, int32_t schedule, const g4a_cp_problem *problem);

/* Waits for the context's stream from the host, polling the communicator's
 * asynchronous error state (ncclCommGetAsyncError) as it waits. A
 * communicator error, or timeout_ms passing first, aborts the communicator
 * (ncclCommAbort: its pending collectives end, it is unusable afterwards)
 * and returns G4A_NCCL or G4A_TIMEOUT; otherwise the device flags are
 * checked as g4a_sync does. The reference reports failures as EngError
 * results (crates/llm-eng/src/error.rs:3-15); there is no collective there. */
int g4a_cp_wait(g4a_ctx *ctx, void *nccl_comm, int32_t timeout_ms);

/* A communicator for callers that have none (no reference counterpart):
 * one rank calls g4a_nccl_unique_id and hands the 128 bytes to the others,
 * then every rank calls g4a_nccl_comm_init with its device. */
int g4a_nccl_unique_id(uint8_t *id_host_128);
int g4a_nccl_comm_init(int32_t n_ranks, int32_t rank, const uint8_t *id_host_128, int device, void **comm_out);
void g4a_nccl_comm_destroy(void *comm);

/* ---- Q8_0 mat-vec: the projections either side of attention ------------
 * crates/llm-backend-cpu/src/matvec.rs with the model's default numerics
 * (quantized activations, model.rs:46-63). Weights are GGUF Q8_0 rows as the
 * reference reads them: `rows` rows of cols/32 blocks of [f16 scale (little
 * endian), 32 x int8], in device memory. x_dev holds n_vec activation vectors
 * [n_vec][cols] f32; each is quantized like quantize_q8_0 (matvec.rs:36-54)
 * and out_dev receives [n_vec][rows] f32. cols must be a multiple of 32
 * (G4A_COMPUTE otherwise, as the reference's error). Results equal the
 * reference's bit for bit for the plain mat-vec (integer block dot products,
 * block values summed in order); GEGLU and soft-cap add the device tanhf. */

/* matvec.rs:58-63 matvec_q8_0(w, rows, quantize_q8_0(x)) */
int g4a_matvec_q8_0(g4a_ctx *ctx, const uint8_t *w_dev, int64_t rows, int64_t cols, const float *x_dev,
                    int32_t n_vec, float *out_dev);
/* matvec.rs:88-103 geglu_q8_0 with gelu_tanh (ops.rs:85-89), as
 * model.rs:229-240 gated_ffn_input calls it */
int g4a_geglu_q8_0(g4a_ctx *ctx, const uint8_t *gate_dev, const uint8_t *up_dev, int64_t rows, int64_t cols,
                   const float *x_dev, int32_t n_vec, float *out_dev);
/* matvec.rs:67-80 matvec_q8_0_then with softcap (ops.rs:79-81), as
 * model.rs:438-449 logits calls it */
int g4a_matvec_q8_0_softcap(g4a_ctx *ctx, const uint8_t *w_dev, int64_t rows, int64_t cols, const float *x_dev,
                            int32_t n_vec, float cap, float *out_dev);
/* matvec.rs:36-54 quantize_q8_0 alone: n values (a multiple of 32) to
 * n/32 scales and n int8 quants. */
int g4a_quantize_q8_0(g4a_ctx *ctx, const float *x_dev, int64_t n, float *scales_dev, int8_t *quants_dev);

/* ---- E2B decoder: one token per sequence through the whole model --------
 * crates/llm-gemma4/src/impl_/model.rs:252-449 (TransformerSpec::{embed,
 * layer, logits} of Gemma4CpuModel with the default numerics) and
 * generate.rs:15-64 (generate_cpu with greedy sampling, sample.rs:27-36), for
 * many sequences at once. Every step runs on the device: the Q8_0 mat-vecs
 * above, the fused decode attention over an f32 K/V cache per owner layer,
 * and the norms, residual adds, per-layer embeddings and argmax. */

#define G4A_MAX_LAYERS 64

/* Weights of blk.N (GGUF names without the prefix; model.rs:123-141).
 * Matrices are GGUF Q8_0 bytes [out][in] in device memory; norms are f32
 * device arrays (the reference widens F32/BF16 norm tensors to f32). */
typedef struct g4a_layer_weights {
    const float *attn_norm, *attn_q_norm, *attn_k_norm, *post_attention_norm;
    const float *ffn_norm, *post_ffw_norm, *post_norm;
    const uint8_t *attn_q, *attn_k, *attn_v, *attn_output;  /* k, v unused on shared-KV layers */
    const uint8_t *ffn_gate, *ffn_up, *ffn_down;
    const uint8_t *inp_gate, *proj;                         /* per-layer embedding (ple_dim > 0) */
    float layer_output_scale;                               /* the scalar tensor; 1 when absent */
} g4a_layer_weights;

typedef struct g4a_model_weights {
    int32_t vocab_size, d_model, d_ff, ple_dim;
    float final_logit_softcap;
    const uint8_t *token_embd;     /* [vocab][d_model] Q8_0; also the tied output head */
    const float *output_norm;      /* [d_model] */
    const uint8_t *ple_token_embd; /* [vocab][n_layers * ple_dim] Q8_0 */
    const uint8_t *ple_model_proj; /* [n_layers * ple_dim][d_model] Q8_0 */
    const float *ple_proj_norm;    /* [ple_dim] */
    g4a_layer_weights layers[G4A_MAX_LAYERS];
} g4a_model_weights;

typedef struct g4a_model g4a_model;

/* Fills a device buffer with seeded synthetic weights (no reference
 * counterpart; stands in for a GGUF file): Q8_0 blocks of N(0, sigma) values
 * (n_values a multiple of 32, the buffer n_values/32*34 bytes), or f32 norm
 * scales center + spread * N(0, 1) rounded to bf16. `tensor` separates the
 * streams of different tensors of one seed. */
int g4a_synth_q8_0(g4a_ctx *ctx, uint8_t *dst_dev, int64_t n_values, uint64_t seed, uint64_t tensor, float sigma);
int g4a_synth_norm(g4a_ctx *ctx, float *dst_dev, int64_t n, uint64_t seed, uint64_t tensor, float center,
                   float spread);

/* A decoder over `w` (the pointers are borrowed and must outlive the model)
 * for up to max_seqs sequences of up to max_tokens positions each; the
 * context's hyperparameters give the layer pattern and its RoPE tables must
 * cover max_tokens positions. The model owns its K/V caches. */
int g4a_model_create(g4a_ctx *ctx, const g4a_model_weights *w, int32_t max_seqs, int32_t max_tokens,
                     g4a_model **out);
void g4a_model_destroy(g4a_model *m);
/* Gemma4CpuModel::clear_context for one sequence (its length back to 0). */
int g4a_model_clear(g4a_model *m, int32_t seq);
int g4a_model_len(const g4a_model *m, int32_t seq, int32_t *len);
/* One forward pass: token tokens_host[i] of sequence seq_ids_host[i] (ids
 * distinct) at position = that sequence's length, which then grows by one.
 * next_host (optional) receives each row's greedy token. Blocks until the
 * step is done. G4A_CONTEXT_TOO_LONG when a sequence is full. */
int g4a_model_step(g4a_model *m, int32_t n, const int32_t *seq_ids_host, const int32_t *tokens_host,
                   int32_t *next_host);
/* A prompt of `len` tokens for each of n sequences (tokens_host [n][len]),
 * appended at each sequence's length. The reference feeds a prompt through
 * transformer::prefill one token per call (transformer.rs:40-52 from
 * generate.rs:38-42); here a step takes many positions (up to a few
 * thousand rows over all sequences), every row computed as in a one-token
 * step, so the caches and logits are those of len g4a_model_step calls.
 * next_host (optional) receives each sequence's greedy token after its last
 * prompt token, and g4a_model_logits then gives those n rows. On an error
 * the chunks already done stay in the caches (g4a_model_len tells how
 * far). */
int g4a_model_prefill(g4a_model *m, int32_t n, const int32_t *seq_ids_host, const int32_t *tokens_host, int32_t len,
                      int32_t *next_host);
/* ContextMemory::view (context_memory.rs:53-69) of the model's cache: rows
 * [0, len) of `layer`'s K/V source for one sequence, [len][head_dim] f32
 * each, copied into caller device buffers on the context's stream. */
int g4a_model_kv_view(const g4a_model *m, int32_t seq, int32_t layer, int32_t len, float *keys_dev,
                      float *values_dev);
/* Device pointer to the soft-capped logits of the last step, [n][vocab]. */
int g4a_model_logits(g4a_model *m, const float **logits_dev);
/* eos_token_ids (model.rs:88,159-164: `<eos>`, and `<turn|>` for chat,
 * tokenizer.rs:127-130): g4a_model_generate keeps such a token and ends that
 * sequence (generate.rs:58-60). Empty by default, as the reference's
 * synthetic model. */
int g4a_model_set_eos(g4a_model *m, const int32_t *ids_host, int32_t n);
/* generate_cpu (generate.rs:15-64) with greedy sampling for sequences
 * 0..n-1 at once: clears them, feeds the prompts [n][prompt_len] through
 * g4a_model_prefill (the same logits as token by token), then samples up to
 * max_new tokens each into out_host [n][max_new] (the last one is not fed
 * back; a sequence that emits an eos token stops there and its later slots
 * are -1). max_context bounds prompt + generated as the reference's
 * max_context does. */
int g4a_model_generate(g4a_model *m, int32_t n, const int32_t *prompts_host, int32_t prompt_len, int32_t max_new,
                       int32_t max_context, int32_t *out_host);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif
#endif /* G4ATTN_H */
