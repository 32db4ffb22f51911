// Host-logic check of the decode planner (gemma4-rs_b200/csrc/g4attn_host.cpp)
// without a GPU: the host file is compiled into this program together with
// stand-ins for the CUDA runtime calls it makes (host memory instead of
// device memory, no-op events and launches), then g4a_kv_* and the planner
// run on random batches and every plan is checked:
//  * each task's window is the reference's (eng/mod.rs:10-36) and its new
//    row is the cache length before the call;
//  * the items of a task cover its rows once, in split order, with interior
//    cuts on 64-row boundaries (f16 kernel) and at most kF16MaxSplits splits;
//  * split tasks own disjoint ranges of partial slots;
//  * the persistent-CTA table is consistent, and the longest-first
//    assignment keeps every CTA's load within one item of the least loaded.
// Prints "ok <plans>" and exits 0, or the first violation and exits 1.
#include "g4attn_host.cpp"

#include <cstdio>
#include <random>

#include "cuda_host_stubs.h"

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
}  // namespace g4a

namespace {

#define CHECK(cond, ...)                      \
    do {                                      \
        if (!(cond)) {                        \
            std::printf("FAIL: " __VA_ARGS__); \
            std::printf("\n");                \
            return false;                     \
        }                                     \
    } while (0)

int64_t item_cost(const Plan &plan, const DecodeItem &it) {  // the assignment's cost model
    const DecodeTask &t = plan.tasks[it.task];
    return (int64_t)(it.row_hi - it.row_lo) * (t.hd / 256) + 64 + (t.n_splits > 1 ? 32 : 0);
}

bool check_plan(const Plan &plan, const g4a_hparams &hp, int n, const std::vector<int32_t> &pos,
                const std::vector<int64_t> &len_before, bool f16) {
    CHECK((int)plan.tasks.size() == 2 * n, "task count %zu", plan.tasks.size());
    std::vector<const DecodeItem *> all;
    for (int w = 0; w < 2; w++)
        for (const auto &it : plan.items[w]) all.push_back(&it);
    std::vector<std::vector<const DecodeItem *>> per(plan.tasks.size());
    for (const DecodeItem *it : all) {
        CHECK(it->task >= 0 && it->task < (int)plan.tasks.size(), "item task %d", it->task);
        per[it->task].push_back(it);
    }
    std::vector<char> slot_used(std::max(plan.slots, 1), 0);
    for (size_t ti = 0; ti < plan.tasks.size(); ti++) {
        const DecodeTask &t = plan.tasks[ti];
        const int j = (int)ti % n;
        const bool global = t.hd == 512;
        const int64_t hi = (int64_t)pos[j] + 1, lo = global ? 0 : std::max<int64_t>(0, hi - hp.sliding_window);
        CHECK(t.lo == lo && t.hi == hi, "task %zu window [%d,%d) want [%lld,%lld)", ti, t.lo, t.hi, (long long)lo,
              (long long)hi);
        CHECK(t.new_row == len_before[ti], "task %zu new row %d want %lld", ti, t.new_row, (long long)len_before[ti]);
        auto its = per[ti];
        std::sort(its.begin(), its.end(), [](const DecodeItem *a, const DecodeItem *b) { return a->split < b->split; });
        CHECK((int)its.size() == t.n_splits && t.n_splits >= 1, "task %zu has %zu items, n_splits %d", ti, its.size(),
              t.n_splits);
        if (f16) CHECK(t.n_splits <= kF16MaxSplits, "task %zu splits %d", ti, t.n_splits);
        int32_t at = t.lo;
        for (int s = 0; s < t.n_splits; s++) {
            CHECK(its[s]->split == s && its[s]->row_lo == at, "task %zu split %d starts at %d, want %d", ti, s,
                  its[s]->row_lo, at);
            CHECK(its[s]->row_hi >= its[s]->row_lo, "task %zu split %d empty range", ti, s);
            if (f16 && s + 1 < t.n_splits) CHECK(its[s]->row_hi % 64 == 0, "task %zu cut %d unaligned", ti, its[s]->row_hi);
            at = its[s]->row_hi;
        }
        CHECK(at == t.hi, "task %zu covered up to %d of %d", ti, at, t.hi);
        if (t.n_splits > 1) {
            CHECK(t.partial_base >= 0 && t.partial_base + t.n_splits <= plan.slots, "task %zu slots out of range", ti);
            for (int s = 0; s < t.n_splits; s++) {
                CHECK(!slot_used[t.partial_base + s], "slot %d used twice", t.partial_base + s);
                slot_used[t.partial_base + s] = 1;
            }
        }
    }
    if (!f16) return true;
    CHECK(plan.items[1].empty(), "f16 plan keeps items by width");
    const int n_items = (int)plan.items[0].size();
    const int n_ctas = (int)plan.cta_start.size() - 1;
    CHECK(n_ctas == std::max(1, std::min(148, n_items)), "%d CTAs for %d items", n_ctas, n_items);
    CHECK(plan.cta_start[0] == 0 && plan.cta_start[n_ctas] == n_items, "start table ends");
    int64_t lmin = INT64_MAX, lmax = 0, cmax = 0;
    for (int b = 0; b < n_ctas; b++) {
        CHECK(plan.cta_start[b] <= plan.cta_start[b + 1], "start table not monotone at %d", b);
        int64_t load = 0;
        for (int i = plan.cta_start[b]; i < plan.cta_start[b + 1]; i++) {
            const int64_t c = item_cost(plan, plan.items[0][i]);
            load += c;
            cmax = std::max(cmax, c);
        }
        lmin = std::min(lmin, load);
        lmax = std::max(lmax, load);
    }
    CHECK(lmax - lmin <= cmax, "CTA loads %lld..%lld, largest item %lld", (long long)lmin, (long long)lmax,
          (long long)cmax);
    return true;
}

}  // namespace

int main() {
    g4a_hparams hp;
    g4a_hparams_e2b(&hp);
    std::vector<float> ff(hp.head_dim_global / 2);
    g4a_proportional_rope_freq_factors(hp.head_dim_global, hp.global_p, ff.data());
    g4a_ctx *ctx = nullptr;
    if (g4a_ctx_create(0, &hp, ff.data(), 4224, &ctx)) {
        std::printf("FAIL: context\n");
        return 1;
    }
    std::mt19937 rng(2026);
    std::vector<float> rows((size_t)4096 * 512, 0.0f), w(512, 1.0f);
    int plans = 0;
    const int32_t layers[2] = {13, 14};
    const int edge[] = {1, 2, 63, 64, 65, 511, 512, 513, 4095, 4096};
    for (int trial = 0; trial < 24; trial++) {
        const bool f16 = trial % 3 != 2;
        const int n = trial < 4 ? 1 + trial : 1 + (int)(rng() % 64);
        g4a_kv *kv = nullptr;
        if (g4a_kv_create(ctx, n, 4160, 64, 0, f16 ? G4A_KV_F16 : G4A_KV_F32, layers, 2, &kv)) {
            std::printf("FAIL: cache: %s\n", g4a_last_error(ctx));
            return 1;
        }
        std::vector<int32_t> pos(n), seqs(n);
        for (int s = 0; s < n; s++) seqs[s] = s;
        std::shuffle(seqs.begin(), seqs.end(), rng);
        for (int j = 0; j < n; j++) {
            const int L = (rng() % 4) == 0 ? edge[rng() % 10] : 1 + (int)(rng() % 4096);
            pos[j] = L - 1;
            for (int l = 0; l < 2; l++)
                if (L - 1 > 0 &&
                    g4a_kv_append_tokens(kv, seqs[j], layers[l], rows.data(), rows.data(), w.data(), L - 1)) {
                    std::printf("FAIL: append: %s\n", g4a_last_error(ctx));
                    return 1;
                }
        }
        std::vector<float> q((size_t)n * 8 * 512), k((size_t)n * 512), o(q.size());
        g4a_decode_layer L[2] = {{13, q.data(), k.data(), k.data(), w.data(), w.data(), o.data()},
                                 {14, q.data(), k.data(), k.data(), w.data(), w.data(), o.data()}};
        for (int step = 0; step < 3; step++) {
            std::vector<int64_t> before(2 * n);
            for (int i = 0; i < 2; i++)
                for (int j = 0; j < n; j++) g4a_kv_len(kv, seqs[j], layers[i], &before[(size_t)i * n + j]);
            Plan &plan = scratch_plan();
            if (build_decode(ctx, kv, 2, L, n, seqs.data(), pos.data(), plan)) {
                std::printf("FAIL: plan: %s\n", g4a_last_error(ctx));
                return 1;
            }
            if (!check_plan(plan, hp, n, pos, before, f16)) {
                std::printf("(trial %d, step %d, %d sequences, %s)\n", trial, step, n, f16 ? "f16" : "f32");
                return 1;
            }
            plans++;
            for (auto &p : pos) p++;
        }
        g4a_kv_destroy(kv);
    }
    g4a_ctx_destroy(ctx);
    std::printf("ok %d\n", plans);
    return 0;
}
