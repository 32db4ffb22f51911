// Host-logic check of the decoder's step scheduling (gemma4-rs_b200/csrc/
// model_host.cpp) without a GPU: the host files are linked with host
// stand-ins for the CUDA runtime (cuda_host_stubs.h) and with recording
// stand-ins for the kernel launchers, and the public g4a_model_* calls are
// checked against what they must launch:
//  * g4a_model_prefill: chunks of at most the model's row capacity, each
//    sequence's positions consecutive and sequence-major, tokens in order,
//    K/V rows stored ahead of the attention (no fused append) with the tiled
//    prompt attention, the head only for each sequence's last row of the
//    last chunk; one position per chunk falls back to decode steps;
//  * rejected calls launch nothing and leave the lengths;
//  * g4a_model_generate with eos ids: a sequence keeps its eos token and
//    stops (generate.rs:58-60), the later steps hold the other sequences,
//    its later output slots are -1.
// The argmax stand-in picks token (131 * seq + 17 * position + 5) mod vocab
// for each row, so the expected tokens are known. Prints "ok" and exits 0,
// or the first violation and exits 1.
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

#include "g4attn.h"
#include "internal.h"
#include "cuda_host_stubs.h"

namespace {

constexpr int kVocab = 1000;

struct Step {
    int n = 0, n_best = 0, fused = 0, prompt_cl = 0, exact = 0;
    std::vector<int32_t> seqs, pos, toks, gather;
};
std::vector<Step> steps;

int32_t pick(int32_t seq, int32_t pos) { return (131 * seq + 17 * pos + 5) % kVocab; }

}  // namespace

namespace g4a {
cudaError_t launch_view(const ViewParams &, int, cudaStream_t) { return cudaSuccess; }
int prefill_run(PrefillScratch *, int *, int32_t, const g4a_prefill_problem *, cudaStream_t, const char **, bool, int) { return 0; }
cudaError_t launch_append(const AppendParams &, int, cudaStream_t) { return cudaSuccess; }
cudaError_t launch_decode(const DecodeParams &, int, int, bool, cudaStream_t) { return cudaSuccess; }
bool encode_tmap_2d(void *, int, const void *, uint64_t, uint64_t, uint32_t) { return true; }
cudaError_t launch_lse_merge(int, const float *const *, const float *const *, int64_t, int, int, float *, float *,
                             cudaStream_t) {
    return cudaSuccess;
}
cudaError_t launch_decode_f16(const DecodeParams &, int, int, cudaStream_t) { return cudaSuccess; }
PrefillScratch *prefill_scratch_new() { return nullptr; }
void prefill_scratch_free(PrefillScratch *) {}
cudaError_t launch_attend_generic(const float *, const float *, const float *, int64_t, int, int, int, float, float *,
                                  int *, cudaStream_t) {
    return cudaSuccess;
}
int q8_run(int, const uint8_t *, const uint8_t *, int64_t, int64_t, const float *, int32_t, float, float *, int8_t *,
           float *, int *, int, cudaStream_t, const char **, bool, const float *, int32_t, const Q8Seg *, int) {
    return 0;
}
cudaError_t e2b_synth_q8(void *, int64_t, uint64_t, uint64_t, float, cudaStream_t) { return cudaSuccess; }
cudaError_t e2b_synth_norm(float *, int64_t, uint64_t, uint64_t, float, float, cudaStream_t) { return cudaSuccess; }
cudaError_t e2b_ple_inputs(const float *, const uint8_t *, const int32_t *, const float *, int, int, float, float, float,
                           float, float *, int, cudaStream_t, bool) {
    return cudaSuccess;
}
cudaError_t e2b_resid(float *, const float *, const float *, float, const float *, int, float, int8_t *, float *, int,
                      cudaStream_t, bool) {
    return cudaSuccess;
}
cudaError_t e2b_gelu_quant(const float *, const float *, int, int, int, int8_t *, float *, int, cudaStream_t, bool) {
    return cudaSuccess;
}
cudaError_t launch_task_append(const DecodeParams &, int, int, cudaStream_t, bool) { return cudaSuccess; }

// recording stand-ins
cudaError_t e2b_plan(const E2bPlanArgs &a, cudaStream_t) {
    Step s;
    s.n = a.n;
    s.n_best = a.n_best;
    s.fused = a.fused_append;
    s.seqs.assign(a.seqs, a.seqs + a.n);
    s.pos.assign(a.pos, a.pos + a.n);
    steps.push_back(s);
    return cudaSuccess;
}
cudaError_t e2b_embed(const uint8_t *, int, const int32_t *tokens, int n, float, float *, cudaStream_t, bool) {
    steps.back().toks.assign(tokens, tokens + n);
    return cudaSuccess;
}
cudaError_t launch_prompt_exact(const DecodeParams &, int, int, int cl, cudaStream_t, bool) {
    steps.back().prompt_cl = cl;
    return cudaSuccess;
}
cudaError_t launch_decode_exact(const DecodeParams &, int, int, cudaStream_t, bool) {
    steps.back().exact = 1;
    return cudaSuccess;
}
cudaError_t e2b_gather_rows(const int8_t *, const float *, int, const int32_t *rows, int n, int8_t *, float *,
                            cudaStream_t, bool) {
    steps.back().gather.assign(rows, rows + n);
    return cudaSuccess;
}
cudaError_t e2b_argmax(const float *, int64_t vocab, int n, unsigned long long *best, cudaStream_t, bool) {
    const Step &s = steps.back();
    for (int j = 0; j < n; j++) {
        const int row = s.gather.empty() ? j : s.gather[j];
        best[j] = (1ull << 32) | (unsigned long long)(pick(s.seqs[row], s.pos[row]) % vocab);
    }
    return cudaSuccess;
}
}  // namespace g4a

namespace {

#define CHECK(cond, ...)                       \
    do {                                       \
        if (!(cond)) {                         \
            std::printf("FAIL: " __VA_ARGS__); \
            std::printf("\n");                 \
            std::exit(1);                      \
        }                                      \
    } while (0)

std::vector<float> norm_buf(4096, 1.0f);
std::vector<uint8_t> mat_buf(64);

g4a_model *make_model(g4a_ctx *ctx, g4a_model_weights &w, int seqs, int tokens) {
    w = g4a_model_weights{};
    w.vocab_size = kVocab;
    w.d_model = 64;
    w.d_ff = 128;
    w.ple_dim = 32;
    w.final_logit_softcap = 30.0f;
    const uint8_t *m = mat_buf.data();
    const float *n = norm_buf.data();
    w.token_embd = m;
    w.output_norm = n;
    w.ple_token_embd = m;
    w.ple_model_proj = m;
    w.ple_proj_norm = n;
    for (int l = 0; l < 35; l++) {
        g4a_layer_weights &L = w.layers[l];
        L.attn_norm = L.attn_q_norm = L.attn_k_norm = L.post_attention_norm = n;
        L.ffn_norm = L.post_ffw_norm = L.post_norm = n;
        L.attn_q = L.attn_k = L.attn_v = L.attn_output = L.ffn_gate = L.ffn_up = L.ffn_down = m;
        L.inp_gate = L.proj = m;
        L.layer_output_scale = 1.0f;
    }
    g4a_model *model = nullptr;
    CHECK(g4a_model_create(ctx, &w, seqs, tokens, &model) == G4A_OK, "model: %s", g4a_last_error(ctx));
    return model;
}

// One prompt of len tokens for sequences ids (each at its length), through
// g4a_model_prefill with the model's row capacity `rows`; checks the steps.
void check_prefill(g4a_ctx *ctx, g4a_model *m, const std::vector<int32_t> &ids, int len, int rows, const char *what) {
    const int n = (int)ids.size();
    std::vector<int32_t> len0(n), tokens((size_t)n * len), next(n);
    for (int i = 0; i < n; i++) g4a_model_len(m, ids[i], &len0[i]);
    for (size_t e = 0; e < tokens.size(); e++) tokens[e] = (int32_t)((e * 37 + 11) % kVocab);
    steps.clear();
    CHECK(g4a_model_prefill(m, n, ids.data(), tokens.data(), len, next.data()) == G4A_OK, "%s: %s", what,
          g4a_last_error(ctx));
    const int per = rows / n > 1 ? rows / n : 1;
    int c0 = 0;
    size_t k = 0;
    for (; c0 < len; c0 += per, k++) {
        const int cl = per < len - c0 ? per : len - c0;
        const bool last = c0 + cl == len;
        CHECK(k < steps.size(), "%s: %zu steps for the prompt", what, steps.size());
        const Step &s = steps[k];
        CHECK(s.n == n * cl, "%s: chunk %zu has %d rows, want %d", what, k, s.n, n * cl);
        if (cl == 1) {
            CHECK(s.fused == 1 && s.exact == 1 && s.prompt_cl == 0 && s.n_best == n && s.gather.empty(),
                  "%s: one-position chunk %zu is not a decode step", what, k);
        } else {
            CHECK(s.fused == 0 && s.prompt_cl == cl && s.exact == 0, "%s: chunk %zu attention (fused %d, cl %d)",
                  what, k, s.fused, s.prompt_cl);
            CHECK(s.n_best == (last ? n : 0), "%s: chunk %zu returns %d rows", what, k, s.n_best);
            if (last) {
                CHECK((int)s.gather.size() == n, "%s: head rows %zu", what, s.gather.size());
                for (int i = 0; i < n; i++) CHECK(s.gather[i] == i * cl + cl - 1, "%s: head row %d", what, i);
            }
        }
        for (int i = 0; i < n; i++)
            for (int j = 0; j < cl; j++) {
                const int r = i * cl + j;
                CHECK(s.seqs[r] == ids[i] && s.pos[r] == len0[i] + c0 + j &&
                          s.toks[r] == tokens[(size_t)i * len + c0 + j],
                      "%s: chunk %zu row %d (seq %d pos %d tok %d)", what, k, r, s.seqs[r], s.pos[r], s.toks[r]);
            }
    }
    CHECK(k == steps.size(), "%s: %zu steps, want %zu", what, steps.size(), k);
    for (int i = 0; i < n; i++) {
        int32_t L = 0;
        g4a_model_len(m, ids[i], &L);
        CHECK(L == len0[i] + len, "%s: length %d after the prompt", what, L);
        CHECK(next[i] == pick(ids[i], len0[i] + len - 1), "%s: next token %d", what, next[i]);
    }
}

}  // namespace

int main() {
    setenv("G4A_NO_GRAPH", "1", 1);  // every step recorded
    g4a_hparams hp;
    g4a_hparams_e2b(&hp);
    std::vector<float> ff(hp.head_dim_global / 2);
    g4a_proportional_rope_freq_factors(hp.head_dim_global, hp.global_p, ff.data());
    g4a_ctx *ctx = nullptr;
    CHECK(g4a_ctx_create(0, &hp, ff.data(), 256, &ctx) == G4A_OK, "context");
    g4a_model_weights w;

    // one chunk holds the whole prompt (row capacity min(2048, 3 * 40))
    {
        g4a_model *m = make_model(ctx, w, 3, 40);
        int32_t one = 0, t = 7;
        CHECK(g4a_model_step(m, 1, &one, &t, nullptr) == G4A_OK, "step");  // sequence 0 holds a token
        check_prefill(ctx, m, {2, 0, 1}, 10, 120, "single chunk");
        g4a_model_destroy(m);
    }
    // several chunks of two positions, then one position per chunk
    for (int rows : {8, 4}) {
        setenv("G4A_CHUNK_ROWS", std::to_string(rows).c_str(), 1);
        g4a_model *m = make_model(ctx, w, 3, 40);
        check_prefill(ctx, m, {0, 1, 2}, 10, rows, rows == 8 ? "two-position chunks" : "one-position chunks");
        check_prefill(ctx, m, {1}, 7, rows, "a second prompt for one sequence");
        g4a_model_destroy(m);
        unsetenv("G4A_CHUNK_ROWS");
    }
    // rejected calls launch nothing
    {
        g4a_model *m = make_model(ctx, w, 2, 12);
        std::vector<int32_t> tok(26, 1), ids = {0, 1};
        steps.clear();
        CHECK(g4a_model_prefill(m, 2, ids.data(), tok.data(), 13, nullptr) == G4A_CONTEXT_TOO_LONG, "too long");
        tok[3] = kVocab;
        CHECK(g4a_model_prefill(m, 2, ids.data(), tok.data(), 5, nullptr) == G4A_COMPUTE, "bad token");
        ids = {1, 1};
        tok[3] = 1;
        CHECK(g4a_model_prefill(m, 2, ids.data(), tok.data(), 5, nullptr) == G4A_COMPUTE, "repeated sequence");
        CHECK(steps.empty(), "a rejected call launched %zu steps", steps.size());
        int32_t L = -1;
        g4a_model_len(m, 0, &L);
        CHECK(L == 0, "length %d after rejected calls", L);
        g4a_model_destroy(m);
    }
    // generate with an eos id: sequence 1 stops after its second token
    {
        g4a_model *m = make_model(ctx, w, 3, 32);
        const int n = 3, plen = 4, max_new = 6;
        std::vector<int32_t> prompts((size_t)n * plen, 3), out((size_t)n * max_new, 0);
        const int32_t eos = pick(1, plen);  // sequence 1's second generated token
        CHECK(g4a_model_set_eos(m, &eos, 1) == G4A_OK, "set eos");
        steps.clear();
        CHECK(g4a_model_generate(m, n, prompts.data(), plen, max_new, 32, out.data()) == G4A_OK, "generate: %s",
              g4a_last_error(ctx));
        for (int i = 0; i < n; i++)
            for (int k = 0; k < max_new; k++) {
                const int32_t want = (i == 1 && k > 1) ? -1 : pick(i, plen - 1 + k);
                CHECK(out[(size_t)i * max_new + k] == want, "generate: out[%d][%d] = %d, want %d", i, k,
                      out[(size_t)i * max_new + k], want);
            }
        // the prompt chunk, then steps of 3, 2, 2, 2, 2 sequences (no step after the last token)
        CHECK(steps.size() == 6, "generate: %zu steps", steps.size());
        const int want_n[6] = {12, 3, 2, 2, 2, 2};
        for (int k = 0; k < 6; k++) CHECK(steps[k].n == want_n[k], "generate: step %d has %d rows", k, steps[k].n);
        CHECK(steps[2].seqs[0] == 0 && steps[2].seqs[1] == 2, "generate: sequences after the eos");
        g4a_model_destroy(m);
    }
    g4a_ctx_destroy(ctx);
    std::printf("ok\n");
    return 0;
}
