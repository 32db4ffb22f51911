/*
 * CPU ORACLE — test infrastructure only.
 *
 * A plain-C restatement of gemma4-rs's f32 attention arithmetic, used by the
 * parity tests, by `__graft_entry__.smoke()` and by `bench.py`'s CPU-baseline
 * leg as the checker / reported baseline. Nothing in the product path (the
 * CUDA library under gemma4-rs_b200/) links or calls this code.
 *
 * Every function cites the reference file:line it restates (paths relative to
 * the gemma4-rs workspace root). The reference is Rust and cannot be built in
 * this environment (no rustc/cargo), so this restatement is pinned by the
 * reference's own known-answer tests (crates/llm-backend-cpu/tests/ops_smoke.rs,
 * crates/llm-gemma4/tests/layer_pattern.rs, crates/llm-eng/src/context_memory.rs
 * tests), reproduced in tests/test_oracle_known_answers.py.  Attention outputs
 * themselves have no golden vectors in the reference; libm (sinf/cosf/expf/
 * powf) results are the platform's, so parity is unpinned at that boundary
 * beyond the stated tolerances.
 */
#ifndef G4A_ORACLE_H
#define G4A_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Error codes mirror crates/llm-eng/src/error.rs:3-15 (EngError). */
enum {
    ORC_OK = 0,
    ORC_CONTEXT_TOO_LONG = 1, /* EngError::ContextTooLong */
    ORC_MISSING_LAYER = 2,    /* EngError::MissingLayer */
    ORC_COMPUTE = 4,          /* EngError::Compute(invalid inputs) */
    ORC_NONFINITE = 5,        /* EngError::Compute("softmax input is not finite") */
    ORC_BAD_LAYER = 6         /* KvShareError (eng/mod.rs:38-43) */
};

/* ---- numeric primitives: crates/llm-backend-cpu/src/ops.rs ---- */
int orc_rms_norm(const float *x, size_t n, const float *weight, float eps, float *out);
float orc_dot_f32(const float *a, const float *b, size_t n);
int orc_softmax_f32(const float *x, size_t n, float *out);
int orc_rope_neox(float *x, size_t len, size_t position, float base, size_t n_rot,
                  const float *freq_factors, size_t n_factors);

/* ---- hyperparameters and policies: crates/llm-gemma4/src/{idea,eng}/mod.rs ---- */
typedef struct orc_hparams {
    int32_t n_layers, n_heads, n_kv_heads, head_dim_local, head_dim_global;
    int32_t sliding_window, shared_kv_layers;
    float local_rope_base, global_rope_base, global_p, rms_norm_eps;
} orc_hparams;

void orc_hparams_e2b(orc_hparams *hp);
int orc_layer_is_global(const orc_hparams *hp, int32_t layer);
int32_t orc_head_dim(const orc_hparams *hp, int32_t layer);
int orc_kv_source_layer(const orc_hparams *hp, int32_t layer, int32_t *source, int32_t *err_detail);
void orc_windowed_len(size_t seq_len, size_t window, size_t *lo, size_t *hi);
void orc_proportional_rope_freq_factors(size_t head_dim, float p, float *out);

/* ---- attention: crates/llm-gemma4/src/impl_/model.rs:307-366 ---- */
int orc_attend(const float *q, const float *keys, const float *values, size_t len,
               size_t n_heads, size_t n_kv_heads, size_t head_dim, float scale, float *out);

/* ---- worker pool: crates/llm-backend-cpu/src/pool.rs ---- */
int orc_pool_threads(void);
int orc_pool_init(int threads);

/* ---- per-layer K/V memory: crates/llm-eng/src/context_memory.rs ---- */
typedef struct orc_kv orc_kv;
orc_kv *orc_kv_create(void);
void orc_kv_destroy(orc_kv *kv);
void orc_kv_clear(orc_kv *kv);
int orc_kv_append(orc_kv *kv, size_t layer, const float *k, const float *v, size_t width);
int orc_kv_append_rows(orc_kv *kv, size_t layer, const float *k, const float *v, size_t width, size_t n);
int orc_kv_view(const orc_kv *kv, size_t layer, size_t len, const float **keys,
                const float **values, size_t *width, size_t *max_len);

/* ---- the attention block of one layer, model.rs:393-410 without projections ----
 * kv_store: 0 = keep f32 (the reference's storage), 1 = round stored K/V to
 * IEEE binary16 (round-to-nearest-even) to model a half-precision device
 * cache. The arithmetic itself stays the reference's f32 arithmetic. */
int orc_attention_block(orc_kv *kv, const orc_hparams *hp, int32_t layer, size_t position,
                        const float *q_raw, const float *k_raw, const float *v_raw,
                        const float *q_norm_w, const float *k_norm_w,
                        const float *rope_freqs, int kv_store, float *out);

/* NEOX RoPE sin/cos of pair i at a position, exactly as rope_neox builds them
 * (ops.rs:150-159): writes half = n_rot/2 (sin, cos) pairs. */
void orc_rope_sincos(size_t position, float base, size_t n_rot, const float *freq_factors,
                     float *sin_out, float *cos_out);

/* Storage roundings used to feed identical inputs to oracle and device. */
float orc_round_f16(float x);
float orc_round_bf16(float x);

/* Batched helper for tests: causal / sliding-window attention of T query
 * positions over T keys, each position exactly as the reference's
 * token-at-a-time prefill does it (generate.rs:37-41 → model.rs:407-410). */
int orc_prefill_attend(const float *q, const float *k, const float *v, size_t T, size_t n_heads,
                       size_t head_dim, size_t window, float *out);

/* ---- Q8_0 mat-vec: crates/llm-backend-cpu/src/matvec.rs ----
 * Weights are GGUF Q8_0 rows: cols/32 blocks of (f16 scale little-endian,
 * 32 int8 values). The activation is quantized first (quantize_q8_0), then
 * every row is an int8 dot product per block, scaled, summed over blocks in
 * order. All functions return ORC_COMPUTE on shape errors. */
int orc_quantize_q8_0(const float *x, size_t n, float *scales, int8_t *quants);
int orc_matvec_q8_0(const uint8_t *w, size_t rows, size_t cols, const float *scales, const int8_t *quants,
                    float *out);
int orc_geglu_q8_0(const uint8_t *gate, const uint8_t *up, size_t rows, size_t cols, const float *scales,
                   const int8_t *quants, float *out);
int orc_matvec_q8_0_softcap(const uint8_t *w, size_t rows, size_t cols, const float *scales,
                            const int8_t *quants, float cap, float *out);
float orc_gelu_tanh(float x);
float orc_softcap(float v, float cap);
int orc_dequant_q8_0(const uint8_t *bytes, size_t n_bytes, float *out);
/* The reference test file's fixtures (crates/llm-backend-cpu/tests/matvec.rs). */
void orc_test_values(uint64_t seed, size_t len, float *out);
void orc_test_q8_0_bytes(const float *w, size_t n, uint8_t *out);

/* ---- the E2B decoder, one token per call: crates/llm-gemma4/src/impl_/model.rs:252-449 ----
 * Weights in the reference's GGUF layout: Q8_0 matrices (rows of
 * cols/32 blocks) and f32 norm scales. The output head is tied to the token
 * embeddings (model.rs:247-250). The K/V memory is an orc_kv. */
typedef struct orc_dec_layer_w {
    const uint8_t *attn_q, *attn_k, *attn_v, *attn_output, *ffn_gate, *ffn_up, *ffn_down, *inp_gate, *proj;
    const float *attn_norm, *attn_q_norm, *attn_k_norm, *post_attention_norm, *ffn_norm, *post_ffw_norm, *post_norm;
    float layer_output_scale; /* model.rs:433-435; 1.0 when absent */
} orc_dec_layer_w;

typedef struct orc_dec_w {
    int32_t d_model, vocab, ple_dim, d_ff;
    float final_logit_softcap;
    const uint8_t *token_embd, *ple_token_embd, *ple_model_proj;
    const float *ple_proj_norm, *output_norm, *rope_freqs;
    orc_dec_layer_w layers[64];
} orc_dec_w;

/* Forward pass of `token` at `position` (model.rs:376-449 through
 * transformer::prefill / decode_step): writes vocab logits. */
int orc_dec_forward(orc_kv *kv, const orc_hparams *hp, const orc_dec_w *w, int32_t token, size_t position,
                    float *logits);
/* sample.rs:27-36 with temperature 0: index of the largest logit under
 * total_cmp, the last one on ties. */
int32_t orc_argmax_total(const float *x, size_t n);

#ifdef __cplusplus
}
#endif
#endif
