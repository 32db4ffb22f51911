// Shared host/device definitions of the g4attn library (not part of the ABI).
#pragma once

#include <cstddef>
#include <cstdint>

#include <cuda_runtime.h>

namespace g4a {

// Launches `kernel`, with programmatic stream serialization when `pdl` is set:
// the kernel may then start while its predecessor on the stream is still
// running, so it must call ptx::pdl_wait() before it touches any memory a
// predecessor writes or reads (only constant inputs such as weights may be
// read before). Every kernel of the decoder step follows that rule.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(bool pdl, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                            Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = pdl ? attr : nullptr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Query heads per KV head served by the fused E2B kernels (idea/mod.rs:53-54:
// 8 query heads, 1 KV head).
constexpr int kHeads = 8;
// Threads of a decode CTA: one warp per query head in the q-preparation phase.
constexpr int kDecodeThreads = 256;

// One (sequence, layer) attention task of a decode call.
struct DecodeTask {
    const void *k_base;   // paged: the layer's K page pool; contiguous: row 0
    const void *v_base;
    const float *q_raw;   // [kHeads][hd] raw q of this task (or ready q)
    const float *k_raw;   // [hd] raw k of the appended token (owners only)
    const float *v_raw;
    const float *q_w;     // attn_q_norm weight [hd]
    const float *k_w;     // attn_k_norm weight [hd]
    float *out;           // [kHeads][hd]
    int32_t seq;          // row of the block table
    int32_t position;     // RoPE position of the query (and of the new key)
    int32_t lo, hi;       // rows attended: [lo, hi)
    int32_t new_row;      // cache row receiving the new token, -1 if none
    int32_t n_splits;     // work items of this task
    int32_t partial_base; // first partial slot of this task
    int32_t global;       // 1 = global RoPE table
    int32_t q_ready;      // 1 = q is already normalised and rotated
    float scale;          // score scale (1.0 in the model, model.rs:409)
    int32_t hd;           // head width of this task's layer
    const void *tmap_k;   // f16 paged caches: TMA descriptors of the layer's pools
    const void *tmap_v;
};

// One CTA's share of a task: cache rows [row_lo, row_hi).
struct DecodeItem {
    int32_t task, split, row_lo, row_hi;
};

struct DecodeParams {
    const DecodeTask *tasks;
    const DecodeItem *items;
    const int32_t *block_table;  // [n_seqs][max_pages]; nullptr = contiguous rows
    int32_t max_pages;
    int32_t page_tokens;
    const float2 *rope_local;    // [max_positions][hd_local/2] (sin, cos)
    const float2 *rope_global;   // [max_positions][hd_global/2]
    float eps;
    float *part_o;               // [slots][kHeads][hd]
    float *part_ml;              // [slots][2][kHeads] (max, sum)
    unsigned *tickets;           // [tasks] arrival counters, zero between calls
    int *err_flag;               // bit 0: non-finite softmax
    int32_t n_items;
    const int32_t *cta_start;    // f16 kernel: CTA b runs items [cta_start[b], cta_start[b+1])
    void *q_blocks;              // f16 kernel: [tasks][kQBlockBytes] q hi/lo blocks
    const int32_t *split_tasks;  // f16 kernel: tasks whose items are merged by the combine kernel
    int32_t max_rows;            // exact kernels: the most rows a task attends
    float *scores;               // exact kernels: [tasks][kHeads][max_rows]
    int32_t stall;               // f16 main kernel: the g4a_debug_stall test wait, then no work
};

// Bulk append of already processed rows, or norm+RoPE of raw rows.
struct AppendParams {
    void *k_pool, *v_pool;       // the layer's pools
    const int32_t *block_table;  // this sequence's row of the block table
    const float *k_src, *v_src;  // [n][hd]
    const float *k_w;            // k norm weight (raw mode)
    const float2 *rope;          // table of this layer kind (raw mode)
    int32_t hd, page_tokens, first_row, first_pos, n_rows, raw;
    float eps;
};

struct ViewParams {
    const void *k_pool, *v_pool;
    const int32_t *block_table;
    float *k_out, *v_out;
    int32_t hd, page_tokens, n_rows;
};

// Launchers (decode.cu).
cudaError_t launch_decode(const DecodeParams &p, int hd, int kv_f16, bool fast, cudaStream_t s);
// f32 caches in the reference's own order of operations with glibc's expf,
// so the output is the reference's bit for bit: items are (task, chunk of
// kExactRowsPerItem rows) for the scores launch; tasks 0..n_tasks-1 then get
// one CTA per (head, 128 columns). Up to kExactMaxRows rows per task.
constexpr int kExactMaxRows = 4096;
constexpr int kExactRowsPerItem = 32;
cudaError_t launch_decode_exact(const DecodeParams &p, int hd, int n_tasks, cudaStream_t s, bool pdl = false);
// K/V rows of tasks 0..n_tasks-1 (norms, RoPE at the task's position, stored
// at that row) ahead of an attention launch whose tasks have new_row = -1.
cudaError_t launch_task_append(const DecodeParams &p, int hd, int n_tasks, cudaStream_t s, bool pdl = false);
// The exact attention of a prompt chunk: tasks s*cl .. s*cl + cl - 1 are cl
// consecutive positions of one sequence (rows stored beforehand, new_row -1),
// each task's output the exact kernels' bit for bit. Scores, softmax and
// probabilities in p.scores ([tasks][heads][max_rows]). The tasks' q rows are
// normalized and rotated in place (q_raw is overwritten unless q_ready).
cudaError_t launch_prompt_exact(const DecodeParams &p, int hd, int n_tasks, int cl, cudaStream_t s, bool pdl = false);
// f16 paged caches (decode_f16_sm100.cu): persistent, TMA + tensor cores.
constexpr int kF16MaxSplits = 96;  // merge weights fit the kernel's shared buffer
constexpr size_t kQBlockBytes = 16 * 512 * 2;  // q hi/lo block of one task (f16 kernel)
// stage 0: prep, n tasks (q blocks + appended rows); stage 1: main, n
// persistent CTAs with per-CTA item lists; stage 2: combine, n split tasks.
cudaError_t launch_decode_f16(const DecodeParams &p, int stage, int n, cudaStream_t s);
inline int f16_stage_rows(int hd) { return 16384 / hd; }
cudaError_t launch_attend_generic(const float *q, const float *k, const float *v, int64_t len, int n_heads,
                                  int n_kv, int hd, float scale, float *out, int *err_flag, cudaStream_t s);
cudaError_t launch_append(const AppendParams &p, int kv_f16, cudaStream_t s);
cudaError_t launch_view(const ViewParams &p, int kv_f16, cudaStream_t s);
cudaError_t launch_lse_merge(int n_parts, const float *const *parts_o, const float *const *parts_lse,
                             int64_t rows, int n_heads, int hd, float *out, float *lse, cudaStream_t s);

// 2D TMA descriptor (128 B) over a row-major [rows][cols] 16-bit tensor with
// 64 x box_rows boxes and the 128-byte swizzle. dtype: 0 bf16, 1 f16.
bool encode_tmap_2d(void *map, int dtype, const void *base, uint64_t cols, uint64_t rows, uint32_t box_rows);
// 2D descriptor over [outer][inner] elements of 1 (u8), 2 (u16) or 4 (f32)
// bytes, rows row_bytes apart; boxes box_inner x box_outer; optional 128-byte
// swizzle (box_inner * elem_bytes must then be 128).
bool encode_tmap_2d_raw(void *map, int elem_bytes, const void *base, uint64_t inner, uint64_t outer,
                        uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, bool swizzle128);
// Batched Q8_0 mat-vec (q8_0_gemm_sm100.cu) over pre-quantized activations
// xq [n_vec][cols] int8, xs [n_vec][cols/32] f32; kind as q8_run. Needs cols
// a multiple of 256 and 16-byte aligned pointers; returns false when the
// shape does not fit (the caller falls back).
bool q8_gemm_fits(int kind, const uint8_t *w, const uint8_t *w2, int64_t rows, int64_t cols, const int8_t *xq,
                  const float *xs);
cudaError_t q8_gemm_run(int kind, const uint8_t *w, const uint8_t *w2, int64_t rows, int64_t cols, const int8_t *xq,
                        const float *xs, int32_t n_vec, float cap, float *out, int *d_err, cudaStream_t st, bool pdl);

// Prefill (prefill_sm100.cu): per-context scratch and the launcher behind
// g4a_prefill. Returns a g4a_status and points *msg at a description.
// Q8_0 mat-vec family (q8_0_sm100.cu); kind 0 plain, 1 GEGLU (w2 = up), 2 soft-cap.
// With pli (small batches, one pass): the input quantized is gelu(x) * pli
// (vector v's per-layer input at pli + v * pli_stride), the PLE gate of
// model.rs:426-428 fused into the `proj` mat-vec.
// With extra (kind 0, small batches, one pass): up to two more matrices of
// the same width over the same input in the same launch (q, k and v).
struct Q8Seg {
    const uint8_t *w;
    int64_t rows;
    float *out;  // [n_vec][rows]
};
int q8_run(int kind, const uint8_t *w, const uint8_t *w2, int64_t rows, int64_t cols, const float *x, int32_t n_vec,
           float cap, float *out, int8_t *xq, float *xs, int *d_err, int n_sm, cudaStream_t st, const char **msg,
           bool pdl = false, const float *pli = nullptr, int32_t pli_stride = 0, const Q8Seg *extra = nullptr,
           int n_extra = 0);

// E2B decoder step (e2b_sm100.cu).
// One layer of the model as the attention planner sees it; the caches are
// [max_seqs][max_tokens][hd] f32 of the layer's KV source.
struct E2bLayerDesc {
    const float *q_w, *k_w;
    float *k_cache, *v_cache;
    int32_t hd, global, owner;
};
struct E2bPlanArgs {
    const E2bLayerDesc *layers;
    int32_t n_layers, n, task_stride;
    const int32_t *seqs, *pos;
    int32_t max_tokens, window, rows_per_item, max_splits_local, max_splits_global;
    const float *q, *k, *v;
    float *att;
    DecodeTask *tasks;  // [n_layers][task_stride]
    DecodeItem *items_local, *items_global;
    unsigned long long *best;  // [n_best] argmax slots, zeroed here
    int32_t n_best;
    int32_t fused_append;      // 1: each attention task stores its token's K/V row; 0: stored before
};
cudaError_t e2b_synth_q8(void *dst, int64_t n_blocks, uint64_t seed, uint64_t tensor, float sigma, cudaStream_t st);
cudaError_t e2b_synth_norm(float *dst, int64_t n, uint64_t seed, uint64_t tensor, float center, float spread,
                           cudaStream_t st);
cudaError_t e2b_embed(const uint8_t *table, int d, const int32_t *tokens, int n, float scale, float *x, cudaStream_t st,
                      bool pdl = false);
cudaError_t e2b_ple_inputs(const float *P, const uint8_t *table, const int32_t *tokens, const float *w, int L, int ple,
                           float ps, float ts, float is, float eps, float *out, int n, cudaStream_t st, bool pdl = false);
cudaError_t e2b_resid(float *x, const float *y, const float *w_post, float post, const float *w_next, int d, float eps,
                      int8_t *xq, float *xs, int n, cudaStream_t st, bool pdl = false);
cudaError_t e2b_gelu_quant(const float *gate, const float *pli, int layer, int L, int ple, int8_t *xq, float *xs, int n,
                           cudaStream_t st, bool pdl = false);
cudaError_t e2b_argmax(const float *logits, int64_t vocab, int n, unsigned long long *best, cudaStream_t st,
                       bool pdl = false);
cudaError_t e2b_plan(const E2bPlanArgs &a, cudaStream_t st);
// Rows rows[j] of the quantized activations xq [.][cols] / xs [.][cols/32]
// copied to row j of xq_out / xs_out, j < n (the rows whose logits a step
// returns).
cudaError_t e2b_gather_rows(const int8_t *xq, const float *xs, int cols, const int32_t *rows, int n, int8_t *xq_out,
                            float *xs_out, cudaStream_t st, bool pdl = false);

struct PrefillScratch;
PrefillScratch *prefill_scratch_new();
void prefill_scratch_free(PrefillScratch *s);
// stall: the g4a_debug_stall test wait in every CTA pair instead of the work;
// reserve_sms: SMs the persistent kernel leaves free (for a collective that
// runs beside it on another stream)
int prefill_run(PrefillScratch *s, int *d_err, int32_t n, const struct g4a_prefill_problem *problems,
                cudaStream_t st, const char **msg, bool stall = false, int reserve_sms = 0);

// Key/value-shard context-parallel merge (cp_kernels.cu): partial results of
// one rank as row segments [t0, t1) of the sequence, o [t1-t0][8][hd] and
// lse [t1-t0][8] (natural log).
constexpr int kCpMaxSegs = 8;
struct CpSeg {
    int32_t t0, t1;
    const float *o;
    const float *lse;
};
struct CpSegs {
    CpSeg s[kCpMaxSegs];
    int32_t n;
};
cudaError_t launch_cp_rowmax(const CpSegs &segs, int32_t T, float *m, cudaStream_t st);
cudaError_t launch_cp_pack(const CpSegs &segs, const float *m, int32_t W, int32_t c, int32_t hd, float *packed,
                           cudaStream_t st);
cudaError_t launch_cp_finish(const float *recv, int32_t rows, int32_t hd, float *out, cudaStream_t st);

}  // namespace g4a
