// Decode-side kernels of g4attn for sm_100a:
//   * fused q/k RMSNorm + NEOX RoPE + KV append + split-KV attention with an
//     in-kernel log-sum-exp combine (the last CTA of a task merges), replacing
//     crates/llm-gemma4/src/impl_/model.rs:393-410 and :326-366;
//   * the bulk append / view kernels behind ContextMemory
//     (crates/llm-eng/src/context_memory.rs:44-69);
//   * a generic attend kernel for shapes other than E2B's 8:1 heads;
//   * the log-sum-exp merge of partial results.
//
// Arithmetic notes. RMSNorm follows ops.rs:45-56: squares in f32, summed in
// f64, mean cast to f32, scale = 1/sqrt(mean + eps) with IEEE sqrt and
// division, then (x * scale) * w. RoPE uses (sin, cos) tables built on the
// host exactly as ops.rs:150-159 builds its angles, and applies them with
// round-to-nearest multiplies and adds that are never fused, so q and the
// stored k/v match the reference bit for bit. Attention sums in a different
// order than the reference (within the 1e-4 decode tolerance).
#include <cuda_fp16.h>
#include <math_constants.h>

#include "internal.h"
#include "libm_glibc.cuh"
#include "sm100_ptx.cuh"

namespace g4a {
namespace {

constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ float load_elem(const float *p) { return *p; }
__device__ __forceinline__ float load_elem(const __half *p) { return __half2float(*p); }
__device__ __forceinline__ void store_elem(float *p, float v) { *p = v; }
__device__ __forceinline__ void store_elem(__half *p, float v) { *p = __float2half_rn(v); }
__device__ __forceinline__ float round_to(float v, const float *) { return v; }
__device__ __forceinline__ float round_to(float v, const __half *) { return __half2float(__float2half_rn(v)); }

__device__ __forceinline__ double warp_sum_f64(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, o));
    return v;
}

// Row r of a cache layer: paged (block table) or contiguous.
template <typename KT>
__device__ __forceinline__ const KT *row_ptr(const void *base, const int32_t *bt, int page_tokens, int hd, int r) {
    size_t idx;
    if (bt) {
        int page = __ldg(bt + r / page_tokens);
        idx = ((size_t)page * page_tokens + (r % page_tokens)) * hd;
    } else {
        idx = (size_t)r * hd;
    }
    return reinterpret_cast<const KT *>(base) + idx;
}

// RMSNorm (+ optional weight) and optional NEOX RoPE of one head held by a
// warp: lane owns elements lane + 32*k. Returns the values in x.
template <int HD>
__device__ __forceinline__ void norm_rope_warp(float (&x)[HD / 32], const float *w, const float2 *rope_row,
                                               float eps, int lane) {
    constexpr int PL = HD / 32;
    double ss = 0.0;
#pragma unroll
    for (int k = 0; k < PL; k++) {
        float sq = __fmul_rn(x[k], x[k]);
        ss += (double)sq;
    }
    ss = warp_sum_f64(ss);
    float mean = (float)(ss / (double)HD);
    float scale = 1.0f / sqrtf(mean + eps);
#pragma unroll
    for (int k = 0; k < PL; k++) {
        float y = __fmul_rn(x[k], scale);
        if (w) y = __fmul_rn(y, __ldg(w + lane + 32 * k));
        x[k] = y;
    }
    if (rope_row) {
#pragma unroll
        for (int k = 0; k < PL / 2; k++) {
            float2 sc = __ldg(rope_row + lane + 32 * k);  // (sin, cos)
            float a = x[k], b = x[k + PL / 2];
            x[k] = __fsub_rn(__fmul_rn(a, sc.y), __fmul_rn(b, sc.x));
            x[k + PL / 2] = __fadd_rn(__fmul_rn(a, sc.x), __fmul_rn(b, sc.y));
        }
    }
}

// Sum 8 per-lane partials across the warp. On return, lanes with
// (lane & 3) == 0 hold the total of head ((lane>>4)&1)*4 + ((lane>>3)&1)*2 + ((lane>>2)&1).
__device__ __forceinline__ float reduce8(float (&v)[kHeads], int lane) {
    {
        const bool up = lane & 16;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            float send = up ? v[j] : v[j + 4];
            float keep = up ? v[j + 4] : v[j];
            v[j] = keep + __shfl_xor_sync(kFull, send, 16);
        }
    }
    {
        const bool up = lane & 8;
#pragma unroll
        for (int j = 0; j < 2; j++) {
            float send = up ? v[j] : v[j + 2];
            float keep = up ? v[j + 2] : v[j];
            v[j] = keep + __shfl_xor_sync(kFull, send, 8);
        }
    }
    {
        const bool up = lane & 4;
        float send = up ? v[0] : v[1];
        float keep = up ? v[1] : v[0];
        v[0] = keep + __shfl_xor_sync(kFull, send, 4);
    }
    float r = v[0];
    r += __shfl_xor_sync(kFull, r, 2);
    r += __shfl_xor_sync(kFull, r, 1);
    return r;
}

__device__ __forceinline__ int reduce8_head(int lane) {
    return ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
}

// Fused decode attention: one CTA per work item (a contiguous range of cache
// rows of one task). 8 warps; rows are processed in blocks of BLK with an
// online softmax; partials of split tasks are merged by the last CTA.
template <int HD, typename KT>
__global__ void __launch_bounds__(kDecodeThreads) decode_kernel(DecodeParams p) {
    constexpr int BLK = 64;
    constexpr int PL = HD / 32;        // elements per lane in a warp-owned row
    constexpr int CPT = HD / kDecodeThreads;  // output columns per thread
    __shared__ __align__(16) float q_s[kHeads][HD];
    __shared__ float s_s[kHeads][BLK];
    __shared__ __align__(16) float knew_s[HD];
    __shared__ __align__(16) float vnew_s[HD];
    __shared__ float alpha_s[kHeads], m_s[kHeads], l_s[kHeads];
    __shared__ const KT *krow_s[BLK], *vrow_s[BLK];  // this block's row addresses
    __shared__ int last_s;

    const DecodeItem it = p.items[blockIdx.x];
    if (it.task < 0) return;  // an unused slot of a fixed-size (captured) launch
    const DecodeTask &tk = p.tasks[it.task];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int32_t *bt = p.block_table ? p.block_table + (size_t)tk.seq * p.max_pages : nullptr;
    const float2 *rope = tk.global ? p.rope_global : p.rope_local;

    // ---- q: norm + RoPE (model.rs:395-396), one warp per head ----
    {
        float x[PL];
        const float *src = tk.q_raw + (size_t)warp * HD;
#pragma unroll
        for (int k = 0; k < PL; k++) x[k] = __ldg(src + lane + 32 * k);
        if (!tk.q_ready) norm_rope_warp<HD>(x, tk.q_w, rope + (size_t)tk.position * (HD / 2), p.eps, lane);
#pragma unroll
        for (int k = 0; k < PL; k++) q_s[warp][lane + 32 * k] = x[k];
    }
    // ---- the appended token (model.rs:400-405): only the CTA holding its row ----
    // A row appended past the attended range (position < cache length, as
    // the reference permits) is still stored, by the task's last item.
    const bool has_new = tk.new_row >= 0 && ((tk.new_row >= it.row_lo && tk.new_row < it.row_hi) ||
                                             (it.split == tk.n_splits - 1 && tk.new_row >= it.row_hi));
    if (has_new && warp < 2) {
        float x[PL];
        const float *src = warp == 0 ? tk.k_raw : tk.v_raw;
#pragma unroll
        for (int k = 0; k < PL; k++) x[k] = __ldg(src + lane + 32 * k);
        if (warp == 0)
            norm_rope_warp<HD>(x, tk.k_w, rope + (size_t)tk.position * (HD / 2), p.eps, lane);
        else
            norm_rope_warp<HD>(x, nullptr, nullptr, p.eps, lane);
        KT *dst = const_cast<KT *>(row_ptr<KT>(warp == 0 ? tk.k_base : tk.v_base, bt, p.page_tokens, HD, tk.new_row));
        float *sm = warp == 0 ? knew_s : vnew_s;
#pragma unroll
        for (int k = 0; k < PL; k++) {
            store_elem(dst + lane + 32 * k, x[k]);
            sm[lane + 32 * k] = round_to(x[k], (const KT *)nullptr);
        }
    }
    if (threadIdx.x < kHeads) {
        m_s[threadIdx.x] = -CUDART_INF_F;
        l_s[threadIdx.x] = 0.0f;
    }
    float acc[kHeads][CPT];
#pragma unroll
    for (int h = 0; h < kHeads; h++)
#pragma unroll
        for (int u = 0; u < CPT; u++) acc[h][u] = 0.0f;
    bool bad = false;
    __syncthreads();

    for (int b0 = it.row_lo; b0 < it.row_hi; b0 += BLK) {
        const int nb = min(BLK, it.row_hi - b0);
        // Row addresses first (one block-table read per row, in parallel), so
        // that the row loads below do not each wait for their page number.
        if (threadIdx.x < nb) {
            krow_s[threadIdx.x] = row_ptr<KT>(tk.k_base, bt, p.page_tokens, HD, b0 + threadIdx.x);
            vrow_s[threadIdx.x] = row_ptr<KT>(tk.v_base, bt, p.page_tokens, HD, b0 + threadIdx.x);
        }
        __syncthreads();
        // ---- scores: warp w takes rows w, w+8, ... of the block ----
#pragma unroll 4
        for (int r = warp; r < nb; r += kHeads) {
            const int row = b0 + r;
            float part[kHeads];
#pragma unroll
            for (int h = 0; h < kHeads; h++) part[h] = 0.0f;
            if (row == tk.new_row) {
#pragma unroll
                for (int k = 0; k < PL; k++) {
                    const int e = lane + 32 * k;
                    const float kv = knew_s[e];
#pragma unroll
                    for (int h = 0; h < kHeads; h++) part[h] = fmaf(q_s[h][e], kv, part[h]);
                }
            } else {
                const KT *krow = krow_s[r];
#pragma unroll
                for (int k = 0; k < PL; k++) {
                    const int e = lane + 32 * k;
                    const float kv = load_elem(krow + e);
#pragma unroll
                    for (int h = 0; h < kHeads; h++) part[h] = fmaf(q_s[h][e], kv, part[h]);
                }
            }
            const float tot = reduce8(part, lane);
            if ((lane & 3) == 0) s_s[reduce8_head(lane)][r] = tot * tk.scale;
        }
        __syncthreads();
        // ---- online softmax update, warp h owns head h ----
        {
            const int h = warp;
            float s0 = lane < nb ? s_s[h][lane] : -CUDART_INF_F;
            float s1 = lane + 32 < nb ? s_s[h][lane + 32] : -CUDART_INF_F;
            if (isnan(s0) || s0 == CUDART_INF_F || isnan(s1) || s1 == CUDART_INF_F) bad = true;
            const float bmax = warp_max(fmaxf(s0, s1));
            const float m_old = m_s[h];
            const float m_new = fmaxf(m_old, bmax);
            float p0 = 0.0f, p1 = 0.0f, alpha = 1.0f;
            if (m_new != -CUDART_INF_F) {
                p0 = expf(s0 - m_new);
                p1 = expf(s1 - m_new);
                alpha = expf(m_old - m_new);
            }
            const float bsum = warp_sum(p0 + p1);
            if (lane < nb) s_s[h][lane] = p0;
            if (lane + 32 < nb) s_s[h][lane + 32] = p1;
            __syncwarp();
            if (lane == 0) {
                alpha_s[h] = alpha;
                m_s[h] = m_new;
                l_s[h] = l_s[h] * alpha + bsum;
            }
        }
        __syncthreads();
        // ---- O += P V: thread owns columns threadIdx.x + 256*u ----
#pragma unroll
        for (int h = 0; h < kHeads; h++) {
            const float a = alpha_s[h];
#pragma unroll
            for (int u = 0; u < CPT; u++) acc[h][u] *= a;
        }
#pragma unroll 16
        for (int r = 0; r < nb; r++) {
            const int row = b0 + r;
            float v[CPT];
            if (row == tk.new_row) {
#pragma unroll
                for (int u = 0; u < CPT; u++) v[u] = vnew_s[threadIdx.x + kDecodeThreads * u];
            } else {
                const KT *vrow = vrow_s[r];
#pragma unroll
                for (int u = 0; u < CPT; u++) v[u] = load_elem(vrow + threadIdx.x + kDecodeThreads * u);
            }
#pragma unroll
            for (int h = 0; h < kHeads; h++) {
                const float pr = s_s[h][r];
#pragma unroll
                for (int u = 0; u < CPT; u++) acc[h][u] = fmaf(pr, v[u], acc[h][u]);
            }
        }
        __syncthreads();
    }
    if (bad) atomicOr(p.err_flag, 1);

    if (tk.n_splits == 1) {
#pragma unroll
        for (int h = 0; h < kHeads; h++) {
            const float l = l_s[h];
            if (threadIdx.x == 0 && !(l > 0.0f)) atomicOr(p.err_flag, 1);
#pragma unroll
            for (int u = 0; u < CPT; u++) tk.out[(size_t)h * HD + threadIdx.x + kDecodeThreads * u] = acc[h][u] / l;
        }
        return;
    }
    // ---- split task: publish the partial, the last arriving CTA merges ----
    const int slot = tk.partial_base + it.split;
    float *po = p.part_o + (size_t)slot * kHeads * HD;
#pragma unroll
    for (int h = 0; h < kHeads; h++)
#pragma unroll
        for (int u = 0; u < CPT; u++) po[(size_t)h * HD + threadIdx.x + kDecodeThreads * u] = acc[h][u];
    if (threadIdx.x < kHeads) {
        p.part_ml[(size_t)slot * 2 * kHeads + threadIdx.x] = m_s[threadIdx.x];
        p.part_ml[(size_t)slot * 2 * kHeads + kHeads + threadIdx.x] = l_s[threadIdx.x];
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned prev = atomicAdd(p.tickets + it.task, 1u);
        last_s = prev == (unsigned)(tk.n_splits - 1);
    }
    __syncthreads();
    if (!last_s) return;
    __threadfence();
    // Merge: per (split, head) weights computed in parallel into shared
    // memory (q_s is free now), then every thread sums its columns over the
    // splits in split order.
    const int ns = tk.n_splits;
    const float *pml = p.part_ml + (size_t)tk.partial_base * 2 * kHeads;
    const float *pall = p.part_o + (size_t)tk.partial_base * kHeads * HD;
    float *wsm = &q_s[0][0];  // [ns][8] weights, then [8] 1/L; ns*8+8 <= 8*HD
    {
        const int h = warp;
        float M = -CUDART_INF_F;
        for (int s = lane; s < ns; s += 32) M = fmaxf(M, __ldcg(pml + (size_t)s * 2 * kHeads + h));
        M = warp_max(M);
        float L = 0.0f;
        for (int s = lane; s < ns; s += 32) {
            const float ms = __ldcg(pml + (size_t)s * 2 * kHeads + h);
            const float w = ms == -CUDART_INF_F ? 0.0f : expf(ms - M);
            wsm[s * kHeads + h] = w;
            L = fmaf(__ldcg(pml + (size_t)s * 2 * kHeads + kHeads + h), w, L);
        }
        L = warp_sum(L);
        if (lane == 0) {
            wsm[ns * kHeads + h] = 1.0f / L;
            if (!(L > 0.0f)) atomicOr(p.err_flag, 1);
        }
    }
    __syncthreads();
    // Each thread owns kHeads*HD/256 output elements and walks the splits in
    // order, loading all of its elements of a split (and of the next one) at
    // once: a few rounds of independent loads instead of one round per element.
    constexpr int EPT = kHeads * HD / kDecodeThreads;
    float o[EPT];
#pragma unroll
    for (int q = 0; q < EPT; q++) o[q] = 0.0f;
#pragma unroll 2
    for (int s = 0; s < ns; s++) {
        const float *ps = pall + (size_t)s * kHeads * HD + threadIdx.x;
        float x[EPT];
#pragma unroll
        for (int q = 0; q < EPT; q++) x[q] = __ldcg(ps + kDecodeThreads * q);
#pragma unroll
        for (int q = 0; q < EPT; q++) o[q] = fmaf(x[q], wsm[s * kHeads + (threadIdx.x + kDecodeThreads * q) / HD], o[q]);
    }
#pragma unroll
    for (int q = 0; q < EPT; q++) {
        const int e = threadIdx.x + kDecodeThreads * q;
        tk.out[e] = o[q] * wsm[ns * kHeads + e / HD];
    }
    if (threadIdx.x == 0) p.tickets[it.task] = 0u;  // ready for the next call
}

// Attention in the reference's order of operations (model.rs:323-343
// attend_head; ops.rs:62-76 dot_f32, :105-127 softmax_f32), so that each
// output is the reference's bit for bit, in two launches:
//   scores  one CTA per (task, chunk of kExactChunk rows): q norm + RoPE, the
//           append (the CTA holding the new row), the chunk's K rows staged
//           in shared memory, then one thread per (head, row):
//           dot_f32 = 16 accumulators (element i into accumulator i % 16,
//           multiply then add), summed in order from -0.0, times the scale;
//   pv      one CTA per (task, 128 value columns): per head max, p_j =
//           exp(s_j - max) / sum with glibc's expf and the sum sequential in
//           key order from -0.0, then out = sum_j p_j * v_j in key order from
//           +0.0 (multiply then add), one thread per column for all eight
//           heads (each V row read once); with few tasks, one CTA per head.
// The q/k norms, RoPE and the stored rows are the fused kernel's (bit-exact).
constexpr int kExactChunk = 32;
constexpr int kPvCols = 128;

template <int HD>
__global__ void __launch_bounds__(kDecodeThreads) exact_scores_kernel(DecodeParams p) {
    ptx::pdl_trigger();
    ptx::pdl_wait();
    constexpr int PL = HD / 32;
    constexpr int KS = HD + 4;  // padded row stride: the 8 lanes of a float4 phase hit distinct banks
    extern __shared__ float4 k_s4[];  // [kExactChunk][KS]
    float *k_s = reinterpret_cast<float *>(k_s4);
    __shared__ __align__(16) float q_s[kHeads][HD];

    const DecodeItem it = p.items[blockIdx.x];
    if (it.task < 0) return;  // an unused slot of a fixed-size (captured) launch
    const DecodeTask &tk = p.tasks[it.task];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int32_t *bt = p.block_table ? p.block_table + (size_t)tk.seq * p.max_pages : nullptr;
    const float2 *rope = tk.global ? p.rope_global : p.rope_local;
    const int nr = it.row_hi - it.row_lo;
    {
        float x[PL];
        const float *src = tk.q_raw + (size_t)warp * HD;
#pragma unroll
        for (int k = 0; k < PL; k++) x[k] = __ldg(src + lane + 32 * k);
        if (!tk.q_ready) norm_rope_warp<HD>(x, tk.q_w, rope + (size_t)tk.position * (HD / 2), p.eps, lane);
#pragma unroll
        for (int k = 0; k < PL; k++) q_s[warp][lane + 32 * k] = x[k];
    }
    const bool in_chunk = tk.new_row >= it.row_lo && tk.new_row < it.row_hi;
    const bool has_new = tk.new_row >= 0 && (in_chunk || (it.split == tk.n_splits - 1 && tk.new_row >= it.row_hi));
    if (has_new && warp < 2) {
        float x[PL];
        const float *src = warp == 0 ? tk.k_raw : tk.v_raw;
#pragma unroll
        for (int k = 0; k < PL; k++) x[k] = __ldg(src + lane + 32 * k);
        if (warp == 0)
            norm_rope_warp<HD>(x, tk.k_w, rope + (size_t)tk.position * (HD / 2), p.eps, lane);
        else
            norm_rope_warp<HD>(x, nullptr, nullptr, p.eps, lane);
        float *dst = const_cast<float *>(row_ptr<float>(warp == 0 ? tk.k_base : tk.v_base, bt, p.page_tokens, HD,
                                                        tk.new_row));
#pragma unroll
        for (int k = 0; k < PL; k++) dst[lane + 32 * k] = x[k];
        if (warp == 0 && in_chunk) {
            float *ks = k_s + (size_t)(tk.new_row - it.row_lo) * KS;
#pragma unroll
            for (int k = 0; k < PL; k++) ks[lane + 32 * k] = x[k];
        }
    }
    // the chunk's other K rows, every load of the chunk in flight at once
    for (int e = threadIdx.x; e < nr * (HD / 4); e += kDecodeThreads) {
        const int r = e / (HD / 4), c = e - r * (HD / 4);
        if (it.row_lo + r == tk.new_row) continue;
        const float4 v = *(reinterpret_cast<const float4 *>(row_ptr<float>(tk.k_base, bt, p.page_tokens, HD,
                                                                            it.row_lo + r)) + c);
        *reinterpret_cast<float4 *>(k_s + (size_t)r * KS + 4 * c) = v;
    }
    __syncthreads();
    // thread = (head warp, row lane)
    if (lane < nr) {
        const float *kr = k_s + (size_t)lane * KS;
        const float *qh = q_s[warp];
        float acc[16];
#pragma unroll
        for (int l = 0; l < 16; l++) acc[l] = 0.0f;
#pragma unroll 2
        for (int m = 0; m < HD / 16; m++) {
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const float4 kv = *reinterpret_cast<const float4 *>(kr + 16 * m + 4 * c);
                const float4 qv = *reinterpret_cast<const float4 *>(qh + 16 * m + 4 * c);
                acc[4 * c + 0] = __fadd_rn(acc[4 * c + 0], __fmul_rn(qv.x, kv.x));
                acc[4 * c + 1] = __fadd_rn(acc[4 * c + 1], __fmul_rn(qv.y, kv.y));
                acc[4 * c + 2] = __fadd_rn(acc[4 * c + 2], __fmul_rn(qv.z, kv.z));
                acc[4 * c + 3] = __fadd_rn(acc[4 * c + 3], __fmul_rn(qv.w, kv.w));
            }
        }
        float sum = -0.0f;
#pragma unroll
        for (int l = 0; l < 16; l++) sum = __fadd_rn(sum, acc[l]);
        p.scores[((size_t)it.task * kHeads + warp) * p.max_rows + (it.row_lo - tk.lo + lane)] = __fmul_rn(sum, tk.scale);
    }
}

// The same per (task, head, 128 columns): more CTAs for few tasks (one
// sequence), each V row then read once per head.
template <int HD>
__global__ void __launch_bounds__(kPvCols) exact_pv_head_kernel(DecodeParams p) {
    ptx::pdl_trigger();
    ptx::pdl_wait();
    constexpr int CH = HD / kPvCols;
    extern __shared__ float pr[];  // [max_rows]
    __shared__ float red[kPvCols / 32];
    __shared__ int flag_s;
    const int task = blockIdx.x / (kHeads * CH);
    const int h = (blockIdx.x / CH) % kHeads, chunk = blockIdx.x % CH;
    const DecodeTask &tk = p.tasks[task];
    const int32_t *bt = p.block_table ? p.block_table + (size_t)tk.seq * p.max_pages : nullptr;
    const int rows = tk.hi - tk.lo, t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const float *sc = p.scores + ((size_t)task * kHeads + h) * p.max_rows;
    float m = -CUDART_INF_F;
    bool finite = true;
    for (int r = t; r < rows; r += kPvCols) {
        const float v = sc[r];
        pr[r] = v;
        finite = finite && isfinite(v);
        m = fmaxf(m, v);
    }
    m = warp_max(m);
    finite = __all_sync(kFull, finite);
    if (t == 0) flag_s = 1;
    if (lane == 0) red[warp] = m;
    __syncthreads();
    if (lane == 0 && !finite) flag_s = 0;
    m = red[0];
#pragma unroll
    for (int w = 1; w < kPvCols / 32; w++) m = fmaxf(m, red[w]);
    for (int r = t; r < rows; r += kPvCols) pr[r] = glibc::expf(__fsub_rn(pr[r], m));
    __syncthreads();
    if (t == 0) {
        float total = -0.0f;
        for (int r = 0; r < rows; r++) total = __fadd_rn(total, pr[r]);
        if (!flag_s || !isfinite(total) || total == 0.0f) {  // softmax_f32's error
            if (chunk == 0) atomicOr(p.err_flag, 1);
            total = CUDART_NAN_F;
        }
        red[0] = total;
    }
    __syncthreads();
    const float total = red[0];
    for (int r = t; r < rows; r += kPvCols) pr[r] = __fdiv_rn(pr[r], total);
    __syncthreads();
    const int col = chunk * kPvCols + t;
    float acc = 0.0f;
    int r = 0;
    for (; r + 16 <= rows; r += 16) {
        float v[16];
#pragma unroll
        for (int u = 0; u < 16; u++) v[u] = row_ptr<float>(tk.v_base, bt, p.page_tokens, HD, tk.lo + r + u)[col];
#pragma unroll
        for (int u = 0; u < 16; u++) acc = __fadd_rn(acc, __fmul_rn(pr[r + u], v[u]));
    }
    for (; r < rows; r++) acc = __fadd_rn(acc, __fmul_rn(pr[r], row_ptr<float>(tk.v_base, bt, p.page_tokens, HD, tk.lo + r)[col]));
    tk.out[(size_t)h * HD + col] = acc;
}

template <int HD>
__global__ void __launch_bounds__(kPvCols) exact_pv_kernel(DecodeParams p) {
    ptx::pdl_trigger();
    ptx::pdl_wait();
    constexpr int CH = HD / kPvCols;  // column chunks per task
    extern __shared__ float pr[];     // [kHeads][max_rows]: scores, then probabilities
    __shared__ float tot_s[kHeads];
    __shared__ int bad_s[kHeads];
    const int task = blockIdx.x / CH, chunk = blockIdx.x % CH;
    const DecodeTask &tk = p.tasks[task];
    const int32_t *bt = p.block_table ? p.block_table + (size_t)tk.seq * p.max_pages : nullptr;
    const int rows = tk.hi - tk.lo, t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const float *sc = p.scores + (size_t)task * kHeads * p.max_rows;
    for (int i = t; i < kHeads * p.max_rows; i += kPvCols) {
        const int h = i / p.max_rows, r = i - h * p.max_rows;
        if (r < rows) pr[i] = sc[i];
    }
    __syncthreads();
    // softmax_f32 per head: warp w takes heads w and w + 4
    for (int h = warp; h < kHeads; h += kPvCols / 32) {
        float *ph = pr + (size_t)h * p.max_rows;
        float m = -CUDART_INF_F;
        bool finite = true;
        for (int r = lane; r < rows; r += 32) {
            finite = finite && isfinite(ph[r]);
            m = fmaxf(m, ph[r]);
        }
        m = warp_max(m);
        finite = __all_sync(kFull, finite);
        for (int r = lane; r < rows; r += 32) ph[r] = glibc::expf(__fsub_rn(ph[r], m));
        __syncwarp();
        if (lane == 0) {
            float total = -0.0f;  // sequential in key order, as f32 Sum
            for (int r = 0; r < rows; r++) total = __fadd_rn(total, ph[r]);
            const bool bad = !finite || !isfinite(total) || total == 0.0f;
            bad_s[h] = bad;
            tot_s[h] = bad ? CUDART_NAN_F : total;
        }
        __syncwarp();
        const float total = tot_s[h];
        for (int r = lane; r < rows; r += 32) ph[r] = __fdiv_rn(ph[r], total);
    }
    __syncthreads();
    if (t < kHeads && chunk == 0 && bad_s[t]) atomicOr(p.err_flag, 1);
    // out[h][col] = sum_j p[h][j] * v[j][col] in key order; each V row is
    // loaded once and serves the eight heads
    const int col = chunk * kPvCols + t;
    float acc[kHeads];
#pragma unroll
    for (int h = 0; h < kHeads; h++) acc[h] = 0.0f;
    int r = 0;
    for (; r + 8 <= rows; r += 8) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; u++) v[u] = row_ptr<float>(tk.v_base, bt, p.page_tokens, HD, tk.lo + r + u)[col];
#pragma unroll
        for (int u = 0; u < 8; u++)
#pragma unroll
            for (int h = 0; h < kHeads; h++)
                acc[h] = __fadd_rn(acc[h], __fmul_rn(pr[(size_t)h * p.max_rows + r + u], v[u]));
    }
    for (; r < rows; r++) {
        const float v = row_ptr<float>(tk.v_base, bt, p.page_tokens, HD, tk.lo + r)[col];
#pragma unroll
        for (int h = 0; h < kHeads; h++) acc[h] = __fadd_rn(acc[h], __fmul_rn(pr[(size_t)h * p.max_rows + r], v));
    }
#pragma unroll
    for (int h = 0; h < kHeads; h++) tk.out[(size_t)h * HD + col] = acc[h];
}

// Few tasks (a batch of a few sequences): the whole attention of one
// (task, head) in one CTA, in the same order of operations as the two
// kernels above: q norm + RoPE of the head, the new row's k/v (stored by the
// head-0 CTA; every CTA uses its own copy for that row), then K in chunks of
// kExactChunk rows staged in shared memory by cp.async (double-buffered):
// eight threads per row each run two of dot_f32's sixteen accumulators, one
// thread per row sums them in order; softmax_f32 with glibc's expf and the
// sequential sum; then V in chunks the same way, one thread per column.
constexpr int kHeadThreads = 256;

template <int HD>
__global__ void __launch_bounds__(kHeadThreads) exact_head_kernel(DecodeParams p) {
    ptx::pdl_trigger();
    ptx::pdl_wait();
    constexpr int PL = HD / 32, KS = HD + 4, RC = kExactChunk, CPT = HD / kHeadThreads;
    extern __shared__ float4 dyn4[];
    float *buf = reinterpret_cast<float *>(dyn4);  // [2][RC][KS]
    float *sc = buf + 2 * RC * KS;                 // [max_rows]
    float *accs = sc + p.max_rows;                 // [RC][17]
    __shared__ __align__(16) float q_s[HD];
    __shared__ __align__(16) float knew_s[HD];
    __shared__ __align__(16) float vnew_s[HD];
    __shared__ float red[kHeadThreads / 32];
    __shared__ int flag_s;
    const int task = blockIdx.x / kHeads, h = blockIdx.x % kHeads;
    const DecodeTask &tk = p.tasks[task];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int32_t *bt = p.block_table ? p.block_table + (size_t)tk.seq * p.max_pages : nullptr;
    const float2 *rope = tk.global ? p.rope_global : p.rope_local;
    const int lo = tk.lo, rows = tk.hi - tk.lo;
    if (warp == 0) {
        float x[PL];
        const float *src = tk.q_raw + (size_t)h * HD;
#pragma unroll
        for (int k = 0; k < PL; k++) x[k] = __ldg(src + lane + 32 * k);
        if (!tk.q_ready) norm_rope_warp<HD>(x, tk.q_w, rope + (size_t)tk.position * (HD / 2), p.eps, lane);
#pragma unroll
        for (int k = 0; k < PL; k++) q_s[lane + 32 * k] = x[k];
    } else if (tk.new_row >= 0 && warp < 3) {
        float x[PL];
        const float *src = warp == 1 ? tk.k_raw : tk.v_raw;
#pragma unroll
        for (int k = 0; k < PL; k++) x[k] = __ldg(src + lane + 32 * k);
        if (warp == 1)
            norm_rope_warp<HD>(x, tk.k_w, rope + (size_t)tk.position * (HD / 2), p.eps, lane);
        else
            norm_rope_warp<HD>(x, nullptr, nullptr, p.eps, lane);
        float *sm = warp == 1 ? knew_s : vnew_s;
        float *dst = h == 0 ? const_cast<float *>(row_ptr<float>(warp == 1 ? tk.k_base : tk.v_base, bt, p.page_tokens,
                                                                 HD, tk.new_row))
                            : nullptr;
#pragma unroll
        for (int k = 0; k < PL; k++) {
            sm[lane + 32 * k] = x[k];
            if (dst) dst[lane + 32 * k] = x[k];
        }
    }
    if (tid == 0) flag_s = rows > 0 && rows <= p.max_rows;
    __syncthreads();
    if (!flag_s) {  // more rows than the launch's score buffer: report, skip
        if (tid == 0 && h == 0) atomicOr(p.err_flag, 4);
        return;
    }
    const int n_chunks = (rows + RC - 1) / RC;
    // rows [c*RC, ...) of K (which = 0) or V (1) into buffer b; the new row from shared memory
    auto stage = [&](int which, int c, int b) {
        const int r0 = c * RC, nr = min(RC, rows - r0);
        float *dst = buf + (size_t)b * RC * KS;
        for (int e = tid; e < nr * (HD / 4); e += kHeadThreads) {
            const int r = e / (HD / 4), q4 = e - r * (HD / 4);
            const int row = lo + r0 + r;
            float *d = dst + (size_t)r * KS + 4 * q4;
            if (row == tk.new_row)
                *reinterpret_cast<float4 *>(d) = reinterpret_cast<const float4 *>(which ? vnew_s : knew_s)[q4];
            else
                ptx::cp_async16(d, row_ptr<float>(which ? tk.v_base : tk.k_base, bt, p.page_tokens, HD, row) + 4 * q4);
        }
        ptx::cp_async_commit();
    };
    // ---- scores ----
    stage(0, 0, 0);
    for (int c = 0; c < n_chunks; c++) {
        if (c + 1 < n_chunks) {
            stage(0, c + 1, (c + 1) & 1);
            ptx::cp_async_wait<1>();
        } else {
            ptx::cp_async_wait<0>();
        }
        __syncthreads();
        const int r0 = c * RC, nr = min(RC, rows - r0);
        const float *kb = buf + (size_t)(c & 1) * RC * KS;
        {
            const int r = tid >> 3, sub = tid & 7;  // accumulators 2 sub, 2 sub + 1
            if (r < nr) {
                const float *kr = kb + (size_t)r * KS;
                float a0 = 0.0f, a1 = 0.0f;
#pragma unroll 8
                for (int m = 0; m < HD / 16; m++) {
                    const float2 kv = *reinterpret_cast<const float2 *>(kr + 16 * m + 2 * sub);
                    const float2 qv = *reinterpret_cast<const float2 *>(q_s + 16 * m + 2 * sub);
                    a0 = __fadd_rn(a0, __fmul_rn(qv.x, kv.x));
                    a1 = __fadd_rn(a1, __fmul_rn(qv.y, kv.y));
                }
                accs[r * 17 + 2 * sub] = a0;
                accs[r * 17 + 2 * sub + 1] = a1;
            }
        }
        __syncthreads();
        if (tid < nr) {
            float s = -0.0f;
#pragma unroll
            for (int l = 0; l < 16; l++) s = __fadd_rn(s, accs[tid * 17 + l]);
            sc[r0 + tid] = __fmul_rn(s, tk.scale);
        }
        __syncthreads();  // the buffer is restaged two chunks on
    }
    // V's first chunk streams in while the softmax runs
    stage(1, 0, 0);
    // ---- softmax_f32 (ops.rs:105-127) ----
    float m = -CUDART_INF_F;
    bool finite = true;
    for (int r = tid; r < rows; r += kHeadThreads) {
        finite = finite && isfinite(sc[r]);
        m = fmaxf(m, sc[r]);
    }
    m = warp_max(m);
    finite = __all_sync(kFull, finite);
    if (lane == 0) red[warp] = m;
    if (tid == 0) flag_s = 1;
    __syncthreads();
    if (lane == 0 && !finite) flag_s = 0;
    m = red[0];
#pragma unroll
    for (int w = 1; w < kHeadThreads / 32; w++) m = fmaxf(m, red[w]);
    for (int r = tid; r < rows; r += kHeadThreads) sc[r] = glibc::expf(__fsub_rn(sc[r], m));
    __syncthreads();
    if (tid == 0) {
        float total = -0.0f;
        for (int r = 0; r < rows; r++) total = __fadd_rn(total, sc[r]);
        if (!flag_s || !isfinite(total) || total == 0.0f) {
            atomicOr(p.err_flag, 1);
            total = CUDART_NAN_F;
        }
        red[0] = total;
    }
    __syncthreads();
    const float total = red[0];
    for (int r = tid; r < rows; r += kHeadThreads) sc[r] = __fdiv_rn(sc[r], total);
    // ---- out = sum_j p_j v_j in key order ----
    float acc[CPT];
#pragma unroll
    for (int u = 0; u < CPT; u++) acc[u] = 0.0f;
    for (int c = 0; c < n_chunks; c++) {
        if (c + 1 < n_chunks) {
            stage(1, c + 1, (c + 1) & 1);
            ptx::cp_async_wait<1>();
        } else {
            ptx::cp_async_wait<0>();
        }
        __syncthreads();
        const int r0 = c * RC, nr = min(RC, rows - r0);
        const float *vb = buf + (size_t)(c & 1) * RC * KS;
        for (int r = 0; r < nr; r++) {
            const float pr = sc[r0 + r];
#pragma unroll
            for (int u = 0; u < CPT; u++)
                acc[u] = __fadd_rn(acc[u], __fmul_rn(pr, vb[(size_t)r * KS + tid + kHeadThreads * u]));
        }
        __syncthreads();
    }
#pragma unroll
    for (int u = 0; u < CPT; u++) tk.out[(size_t)h * HD + tid + kHeadThreads * u] = acc[u];
}

// Generic attend for any (n_heads, n_kv, hd <= 1024): one CTA per query
// head, online softmax over blocks of 256 rows. Used for shapes the fused
// E2B kernels do not serve (e.g. the reference's small synthetic models).
__global__ void __launch_bounds__(256) attend_generic_kernel(const float *q, const float *keys, const float *values,
                                                             int64_t len, int n_heads, int n_kv, int hd,
                                                             float scale, float *out, int *err_flag) {
    constexpr int BLK = 256;
    __shared__ float q_s[1024];
    __shared__ float p_s[BLK];
    __shared__ float red_s[32];
    const int h = blockIdx.x;
    const int kvh = h * n_kv / n_heads;
    const int width = n_kv * hd;
    for (int e = threadIdx.x; e < hd; e += blockDim.x) q_s[e] = q[(size_t)h * hd + e];
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    float m = -CUDART_INF_F, l = 0.0f;
    bool bad = false;
    __syncthreads();
    for (int64_t b0 = 0; b0 < len; b0 += BLK) {
        const int nb = (int)min((int64_t)BLK, len - b0);
        float s = -CUDART_INF_F;
        if ((int)threadIdx.x < nb) {
            const float *k = keys + (size_t)(b0 + threadIdx.x) * width + (size_t)kvh * hd;
            float d = 0.0f;
            for (int e = 0; e < hd; e++) d = fmaf(q_s[e], k[e], d);
            s = d * scale;
            if (isnan(s) || s == CUDART_INF_F) bad = true;
        }
        // block max
        float bm = warp_max(s);
        if ((threadIdx.x & 31) == 0) red_s[threadIdx.x >> 5] = bm;
        __syncthreads();
        if (threadIdx.x < 32) {
            float v = threadIdx.x < blockDim.x / 32 ? red_s[threadIdx.x] : -CUDART_INF_F;
            v = warp_max(v);
            if (threadIdx.x == 0) red_s[0] = v;
        }
        __syncthreads();
        const float m_new = fmaxf(m, red_s[0]);
        __syncthreads();
        float pr = 0.0f, alpha = 1.0f;
        if (m_new != -CUDART_INF_F) {
            pr = (int)threadIdx.x < nb ? expf(s - m_new) : 0.0f;
            alpha = expf(m - m_new);
        }
        p_s[threadIdx.x] = pr;
        float bs = warp_sum(pr);
        if ((threadIdx.x & 31) == 0) red_s[threadIdx.x >> 5] = bs;
        __syncthreads();
        if (threadIdx.x < 32) {
            float v = threadIdx.x < blockDim.x / 32 ? red_s[threadIdx.x] : 0.0f;
            v = warp_sum(v);
            if (threadIdx.x == 0) red_s[0] = v;
        }
        __syncthreads();
        l = l * alpha + red_s[0];
        m = m_new;
        for (int u = 0; u < 4; u++) {
            const int c = threadIdx.x + 256 * u;
            if (c >= hd) break;
            float a = acc[u] * alpha;
            for (int r = 0; r < nb; r++)
                a = fmaf(p_s[r], values[(size_t)(b0 + r) * width + (size_t)kvh * hd + c], a);
            acc[u] = a;
        }
        __syncthreads();
    }
    if (bad || !(l > 0.0f)) atomicOr(err_flag, 1);
    for (int u = 0; u < 4; u++) {
        const int c = threadIdx.x + 256 * u;
        if (c < hd) out[(size_t)h * hd + c] = acc[u] / l;
    }
}

// Bulk append: one warp per (row, K|V). Raw mode applies k-norm + RoPE to K
// and the unweighted norm to V (model.rs:402-404); otherwise rows are stored
// as given.
template <int HD, typename KT>
__global__ void __launch_bounds__(64) append_kernel(AppendParams p) {
    constexpr int PL = HD / 32;
    const int row = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float *src = (warp == 0 ? p.k_src : p.v_src) + (size_t)row * HD;
    float x[PL];
#pragma unroll
    for (int k = 0; k < PL; k++) x[k] = src[lane + 32 * k];
    if (p.raw) {
        if (warp == 0)
            norm_rope_warp<HD>(x, p.k_w, p.rope + (size_t)(p.first_pos + row) * (HD / 2), p.eps, lane);
        else
            norm_rope_warp<HD>(x, nullptr, nullptr, p.eps, lane);
    }
    const int r = p.first_row + row;
    const int page = p.block_table[r / p.page_tokens];
    KT *dst = reinterpret_cast<KT *>(warp == 0 ? p.k_pool : p.v_pool) +
              ((size_t)page * p.page_tokens + (r % p.page_tokens)) * HD;
#pragma unroll
    for (int k = 0; k < PL; k++) store_elem(dst + lane + 32 * k, x[k]);
}

// ---- prompt chunks ----------------------------------------------------------
// A prompt chunk holds, for each of its sequences, cl consecutive positions:
// tasks s*cl .. s*cl + cl - 1 of sequence s, their K/V rows already stored
// (task_append_kernel). The queries of one sequence read the same key and
// value rows, so a CTA serves a block of kPromptQ consecutive queries x 8
// heads from each staged row. Per (query, head) the arithmetic is that of the
// exact kernels above, in the same order, so the bits are the same:
//   scores  dot_f32's 16 accumulators, lane l summing q[16m+l] * k[16m+l]
//           over m (multiply then add, from +0.0), the lanes added in order
//           from -0.0, times the scale;
//   softmax max, glibc's expf, the sequential sum, the division;
//   pv      out += p_j * v_j in key order from +0.0 (multiply then add).
// The PV loop runs over the union of the block's key ranges; a key outside a
// query's range has p = 0, and adding the zero product leaves the (never
// negative-zero) accumulator's bits unchanged.
constexpr int kPromptQ = 8;                  // queries per block
constexpr int kPromptQH = kPromptQ * kHeads;  // 64 (query, head) rows
constexpr int kPromptKeys = 8;               // keys per staged chunk (scores)
constexpr int kPromptRed = 16;               // floats per (row, key) of the lane table
constexpr int kPromptPvKeys = 32;            // keys per staged chunk (pv)

struct PromptBlock {
    int t0, nq;
};
__device__ __forceinline__ PromptBlock prompt_block(int b, int cl) {
    const int bps = (cl + kPromptQ - 1) / kPromptQ;
    const int seq = b / bps, q0 = (b - seq * bps) * kPromptQ;
    return {seq * cl + q0, min(kPromptQ, cl - q0)};
}

// q-norm and RoPE of every task's q (model.rs:395-396), in place, once per
// task (the scores kernel's CTAs of a block then read it ready): one CTA per
// task, warp h on head h; the exact kernels' arithmetic.
template <int HD>
__global__ void __launch_bounds__(256) prompt_q_kernel(DecodeParams p) {
    ptx::pdl_trigger();
    ptx::pdl_wait();
    constexpr int PL = HD / 32;
    const DecodeTask &tk = p.tasks[blockIdx.x];
    if (tk.q_ready) return;
    const int h = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float *q = const_cast<float *>(tk.q_raw) + (size_t)h * HD;
    const float2 *rope = tk.global ? p.rope_global : p.rope_local;
    float x[PL];
#pragma unroll
    for (int k = 0; k < PL; k++) x[k] = q[lane + 32 * k];
    norm_rope_warp<HD>(x, tk.q_w, rope + (size_t)tk.position * (HD / 2), p.eps, lane);
#pragma unroll
    for (int k = 0; k < PL; k++) q[lane + 32 * k] = x[k];
}

// grid (blocks, splits): CTA (b, y) takes key chunks y, y + splits, ... of
// block b. 256 threads: warp w holds query w's eight heads; within a warp,
// lanes 0-15 and 16-31 take keys 0-3 and 4-7 of the chunk, lane & 15 being
// the dot_f32 accumulator lane.
template <int HD>
__global__ void __launch_bounds__(256) prompt_scores_kernel(DecodeParams p, int cl) {
    ptx::pdl_trigger();
    ptx::pdl_wait();
    constexpr int KS = HD + 4;
    extern __shared__ float4 dyn4[];
    // q rows unpadded (their reads are broadcasts), key rows padded so that
    // the two half-warps' rows fall in different banks: two CTAs per SM at
    // width 256
    float *q_s = reinterpret_cast<float *>(dyn4);  // [64][HD]
    float *k_s = q_s + kPromptQH * HD;            // [2][kPromptKeys][KS]
    float *red = k_s + 2 * kPromptKeys * KS;      // [64 * kPromptKeys][kPromptRed]
    // blocks in reverse: the longest key ranges (latest positions) start first
    const PromptBlock blk = prompt_block(gridDim.x - 1 - blockIdx.x, cl);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const DecodeTask &first = p.tasks[blk.t0];
    const int klo = first.lo, khi = p.tasks[blk.t0 + blk.nq - 1].hi;
    const int n_chunks = (khi - klo + kPromptKeys - 1) / kPromptKeys;
    if ((int)blockIdx.y >= n_chunks) return;  // uniform over the CTA, before any barrier
    const int32_t *bt = p.block_table ? p.block_table + (size_t)first.seq * p.max_pages : nullptr;
    // q rows, normalized and rotated by prompt_q_kernel; zeros past the block
    for (int e = tid; e < kPromptQH * (HD / 4); e += 256) {
        const int r = e / (HD / 4), q4 = e - r * (HD / 4), q = r / kHeads;
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (q < blk.nq)
            v = *reinterpret_cast<const float4 *>(p.tasks[blk.t0 + q].q_raw + (size_t)(r - q * kHeads) * HD + 4 * q4);
        *reinterpret_cast<float4 *>(q_s + (size_t)r * HD + 4 * q4) = v;
    }
    auto stage = [&](int c, int b) {
        const int r0 = klo + c * kPromptKeys, nr = min(kPromptKeys, khi - r0);
        float *dst = k_s + (size_t)b * kPromptKeys * KS;
        for (int e = tid; e < kPromptKeys * (HD / 4); e += 256) {
            const int r = e / (HD / 4), q4 = e - r * (HD / 4);
            float *d = dst + (size_t)r * KS + 4 * q4;
            if (r < nr)
                ptx::cp_async16(d, row_ptr<float>(first.k_base, bt, p.page_tokens, HD, r0 + r) + 4 * q4);
            else
                *reinterpret_cast<float4 *>(d) = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
        ptx::cp_async_commit();
    };
    // the two (query, head) rows whose sums this thread writes: pair tid and
    // tid + 256 of each chunk's table, i.e. rows tid / 8 and tid / 8 + 32
    int s_lo[2], s_hi[2];
    float s_scale[2], *s_row[2];
#pragma unroll
    for (int u = 0; u < 2; u++) {
        const int qh = tid / kPromptKeys + 32 * u, q = qh / kHeads;
        s_lo[u] = 0;
        s_hi[u] = 0;
        s_scale[u] = 1.0f;
        s_row[u] = p.scores;
        if (q < blk.nq) {
            const DecodeTask &tk = p.tasks[blk.t0 + q];
            s_lo[u] = tk.lo;
            s_hi[u] = tk.hi;
            s_scale[u] = tk.scale;
            s_row[u] = p.scores + ((size_t)(blk.t0 + q) * kHeads + (qh - q * kHeads)) * p.max_rows;
        }
    }
    const int kg = lane >> 4, l = lane & 15;
    const float *qb = q_s + (size_t)(warp * kHeads) * HD + l;
    int b = 0;
    stage(blockIdx.y, 0);
    for (int c = blockIdx.y; c < n_chunks; c += gridDim.y) {
        if (c + (int)gridDim.y < n_chunks) {
            stage(c + gridDim.y, b ^ 1);
            ptx::cp_async_wait<1>();
        } else {
            ptx::cp_async_wait<0>();
        }
        __syncthreads();
        const float *kb = k_s + ((size_t)b * kPromptKeys + kg * 4) * KS + l;
        float acc[kHeads][4];
#pragma unroll
        for (int j = 0; j < kHeads; j++)
#pragma unroll
            for (int i = 0; i < 4; i++) acc[j][i] = 0.0f;
#pragma unroll 2
        for (int m = 0; m < HD / 16; m++) {
            float qv[kHeads], kv[4];
#pragma unroll
            for (int j = 0; j < kHeads; j++) qv[j] = qb[j * HD + 16 * m];
#pragma unroll
            for (int i = 0; i < 4; i++) kv[i] = kb[i * KS + 16 * m];
#pragma unroll
            for (int j = 0; j < kHeads; j++)
#pragma unroll
                for (int i = 0; i < 4; i++) acc[j][i] = __fadd_rn(acc[j][i], __fmul_rn(qv[j], kv[i]));
        }
#pragma unroll
        for (int j = 0; j < kHeads; j++)
#pragma unroll
            for (int i = 0; i < 4; i++)
                red[((warp * kHeads + j) * kPromptKeys + kg * 4 + i) * kPromptRed + l] = acc[j][i];
        __syncthreads();
        // lanes added in order; thread tid takes the pairs tid and tid + 256
        // of the table (its two rows and key fixed, set up before the loop)
        const int k = klo + c * kPromptKeys + (tid & (kPromptKeys - 1));
#pragma unroll
        for (int u = 0; u < 2; u++) {
            if (k < s_lo[u] || k >= s_hi[u]) continue;  // also rows past the block (empty range)
            const float4 *rp = reinterpret_cast<const float4 *>(red + (size_t)(tid + 256 * u) * kPromptRed);
            float sum = -0.0f;
#pragma unroll
            for (int w = 0; w < 4; w++) {
                const float4 v = rp[w];
                sum = __fadd_rn(sum, v.x);
                sum = __fadd_rn(sum, v.y);
                sum = __fadd_rn(sum, v.z);
                sum = __fadd_rn(sum, v.w);
            }
            s_row[u][k - s_lo[u]] = __fmul_rn(sum, s_scale[u]);
        }
        __syncthreads();  // the lane table and this chunk's buffer are rewritten next
        b ^= 1;
    }
}

// softmax_f32 (ops.rs:105-127) of every (task, head) row of the scores, in
// place: one warp per row; the same arithmetic as the exact kernels. The
// sequential sum runs in key order over chunks of 128 keys held four per
// lane: each value is broadcast in turn and every lane adds them all, so no
// lane waits on a memory load per element.
__global__ void __launch_bounds__(256) prompt_softmax_kernel(DecodeParams p, int n_rows) {
    ptx::pdl_trigger();
    ptx::pdl_wait();
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= n_rows) return;
    const DecodeTask &tk = p.tasks[row / kHeads];
    const int rows = tk.hi - tk.lo;
    float *s = p.scores + (size_t)row * p.max_rows;
    float m = -CUDART_INF_F;
    bool finite = true;
    for (int r = lane; r < rows; r += 32) {
        const float v = s[r];
        finite = finite && isfinite(v);
        m = fmaxf(m, v);
    }
    m = warp_max(m);
    finite = __all_sync(kFull, finite);
    float total = -0.0f;
    for (int c0 = 0; c0 < rows; c0 += 128) {
        float e[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int r = c0 + 32 * u + lane;
            e[u] = 0.0f;
            if (r < rows) {
                e[u] = glibc::expf(__fsub_rn(s[r], m));
                s[r] = e[u];
            }
        }
        const int nr = min(128, rows - c0);
#pragma unroll
        for (int u = 0; u < 4; u++)
#pragma unroll
            for (int j = 0; j < 32; j++) {
                const float v = __shfl_sync(kFull, e[u], j);
                if (32 * u + j < nr) total = __fadd_rn(total, v);
            }
    }
    if (!finite || !isfinite(total) || total == 0.0f) {
        if (lane == 0) atomicOr(p.err_flag, 1);
        total = CUDART_NAN_F;
    }
    for (int r = lane; r < rows; r += 32) s[r] = __fdiv_rn(s[r], total);
}

// grid (blocks, HD / 64), 256 threads: warp w accumulates query w over 64
// columns, lane = a pair of columns, all eight heads (each key's eight
// probabilities one broadcast per warp); V rows and the probabilities of the
// block's 64 rows are staged per chunk of kPromptPvKeys keys.
constexpr int kPromptPvCols = 64;

template <int HD>
__global__ void __launch_bounds__(256) prompt_pv_kernel(DecodeParams p, int cl) {
    ptx::pdl_trigger();
    ptx::pdl_wait();
    constexpr int VC = kPromptPvCols, KC = kPromptPvKeys;
    extern __shared__ float4 dyn4[];
    float *v_s = reinterpret_cast<float *>(dyn4);  // [2][KC][VC]
    float *p_s = v_s + 2 * KC * VC;                // [2][KC][64]
    const PromptBlock blk = prompt_block(gridDim.x - 1 - blockIdx.x, cl);  // longest ranges first
    const int col0 = blockIdx.y * VC;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const DecodeTask &first = p.tasks[blk.t0];
    const int klo = first.lo, khi = p.tasks[blk.t0 + blk.nq - 1].hi;
    const int n_chunks = (khi - klo + KC - 1) / KC;
    const int32_t *bt = p.block_table ? p.block_table + (size_t)first.seq * p.max_pages : nullptr;
    // probability gather: thread = (row gq, keys gk .. gk + 7 of the chunk)
    const int gq = tid & (kPromptQH - 1), gk = (tid / kPromptQH) * 8;
    const int gq_q = gq / kHeads;
    int g_lo = 0, g_hi = 0;
    const float *g_row = p.scores;
    if (gq_q < blk.nq) {
        const DecodeTask &gt = p.tasks[blk.t0 + gq_q];
        g_lo = gt.lo;
        g_hi = gt.hi;
        g_row = p.scores + ((size_t)(blk.t0 + gq_q) * kHeads + (gq - gq_q * kHeads)) * p.max_rows;
    }
    float pf[8];
    auto load_p = [&](int c) {
        const int k0 = klo + c * KC + gk;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int k = k0 + j;
            pf[j] = (k >= g_lo && k < g_hi) ? g_row[k - g_lo] : 0.0f;
        }
    };
    auto store_p = [&](int b) {
        float *d = p_s + (size_t)b * KC * kPromptQH;
#pragma unroll
        for (int j = 0; j < 8; j++) d[(gk + j) * kPromptQH + gq] = pf[j];
    };
    auto stage_v = [&](int c, int b) {
        const int r0 = klo + c * KC, nr = min(KC, khi - r0);
        float *dst = v_s + (size_t)b * KC * VC;
        for (int e = tid; e < KC * (VC / 4); e += 256) {
            const int r = e / (VC / 4), q4 = e - r * (VC / 4);
            float *d = dst + (size_t)r * VC + 4 * q4;
            if (r < nr)
                ptx::cp_async16(d, row_ptr<float>(first.v_base, bt, p.page_tokens, HD, r0 + r) + col0 + 4 * q4);
            else
                *reinterpret_cast<float4 *>(d) = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
        ptx::cp_async_commit();
    };
    float acc[kHeads][2];
#pragma unroll
    for (int h = 0; h < kHeads; h++) acc[h][0] = acc[h][1] = 0.0f;
    load_p(0);
    store_p(0);
    stage_v(0, 0);
    int b = 0;
    for (int c = 0; c < n_chunks; c++) {
        const bool more = c + 1 < n_chunks;
        if (more) {
            stage_v(c + 1, b ^ 1);
            load_p(c + 1);
            ptx::cp_async_wait<1>();
        } else {
            ptx::cp_async_wait<0>();
        }
        __syncthreads();
        const float *vb = v_s + (size_t)b * KC * VC + 2 * lane;
        const float *pb = p_s + (size_t)b * KC * kPromptQH + warp * kHeads;
#pragma unroll 8
        for (int k = 0; k < KC; k++) {  // key order
            const float2 v = *reinterpret_cast<const float2 *>(vb + (size_t)k * VC);
            const float4 p0 = *reinterpret_cast<const float4 *>(pb + (size_t)k * kPromptQH);
            const float4 p1 = *reinterpret_cast<const float4 *>(pb + (size_t)k * kPromptQH + 4);
            const float pp[kHeads] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
            for (int h = 0; h < kHeads; h++) {
                acc[h][0] = __fadd_rn(acc[h][0], __fmul_rn(pp[h], v.x));
                acc[h][1] = __fadd_rn(acc[h][1], __fmul_rn(pp[h], v.y));
            }
        }
        __syncthreads();  // both buffers of this chunk are free
        if (more) store_p(b ^ 1);
        b ^= 1;
    }
    if (warp < blk.nq) {
        const DecodeTask &tk = p.tasks[blk.t0 + warp];
#pragma unroll
        for (int h = 0; h < kHeads; h++)
            *reinterpret_cast<float2 *>(tk.out + (size_t)h * HD + col0 + 2 * lane) = make_float2(acc[h][0], acc[h][1]);
    }
}

// The K/V rows of a step's tokens stored before any attention of the step
// reads them (a prompt chunk holds several positions of one sequence): k-norm
// and RoPE of K, the unweighted norm of V (model.rs:398-404), the arithmetic
// of the attention kernels' own append, so the rows are the same bits. One
// CTA of two warps per task; a task without k_raw (a layer reading another
// layer's cache) stores nothing. The row is the task's position.
template <int HD>
__global__ void __launch_bounds__(64) task_append_kernel(DecodeParams p) {
    ptx::pdl_trigger();
    ptx::pdl_wait();
    constexpr int PL = HD / 32;
    const DecodeTask &tk = p.tasks[blockIdx.x];
    if (!tk.k_raw) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int32_t *bt = p.block_table ? p.block_table + (size_t)tk.seq * p.max_pages : nullptr;
    const float2 *rope = tk.global ? p.rope_global : p.rope_local;
    float x[PL];
    const float *src = warp == 0 ? tk.k_raw : tk.v_raw;
#pragma unroll
    for (int k = 0; k < PL; k++) x[k] = __ldg(src + lane + 32 * k);
    if (warp == 0)
        norm_rope_warp<HD>(x, tk.k_w, rope + (size_t)tk.position * (HD / 2), p.eps, lane);
    else
        norm_rope_warp<HD>(x, nullptr, nullptr, p.eps, lane);
    float *dst =
        const_cast<float *>(row_ptr<float>(warp == 0 ? tk.k_base : tk.v_base, bt, p.page_tokens, HD, tk.position));
#pragma unroll
    for (int k = 0; k < PL; k++) dst[lane + 32 * k] = x[k];
}

template <typename KT>
__global__ void append_any_kernel(AppendParams p) {
    const int row = blockIdx.x;
    const int r = p.first_row + row;
    const int page = p.block_table[r / p.page_tokens];
    const size_t off = ((size_t)page * p.page_tokens + (r % p.page_tokens)) * p.hd;
    for (int e = threadIdx.x; e < p.hd; e += blockDim.x) {
        store_elem(reinterpret_cast<KT *>(p.k_pool) + off + e, p.k_src[(size_t)row * p.hd + e]);
        store_elem(reinterpret_cast<KT *>(p.v_pool) + off + e, p.v_src[(size_t)row * p.hd + e]);
    }
}

template <typename KT>
__global__ void view_kernel(ViewParams p) {
    const int r = blockIdx.x;
    const int page = p.block_table[r / p.page_tokens];
    const size_t off = ((size_t)page * p.page_tokens + (r % p.page_tokens)) * p.hd;
    for (int e = threadIdx.x; e < p.hd; e += blockDim.x) {
        p.k_out[(size_t)r * p.hd + e] = load_elem(reinterpret_cast<const KT *>(p.k_pool) + off + e);
        p.v_out[(size_t)r * p.hd + e] = load_elem(reinterpret_cast<const KT *>(p.v_pool) + off + e);
    }
}

constexpr int kMaxMergeParts = 16;
struct MergeArgs {
    const float *o[kMaxMergeParts];
    const float *lse[kMaxMergeParts];
};

// out = sum_i exp(lse_i - L) out_i, L = log(sum_i exp(lse_i)); one CTA per
// (row, head).
__global__ void lse_merge_kernel(MergeArgs a, int n_parts, int hd, float *out, float *lse) {
    const size_t rh = blockIdx.x;  // row * n_heads + head
    float M = -CUDART_INF_F;
    for (int i = 0; i < n_parts; i++) M = fmaxf(M, a.lse[i][rh]);
    float L = 0.0f;
    float w[kMaxMergeParts];
    for (int i = 0; i < n_parts; i++) {
        w[i] = M == -CUDART_INF_F ? 0.0f : expf(a.lse[i][rh] - M);
        L += w[i];
    }
    const float inv = L > 0.0f ? 1.0f / L : 0.0f;
    for (int c = threadIdx.x; c < hd; c += blockDim.x) {
        float o = 0.0f;
        for (int i = 0; i < n_parts; i++) o = fmaf(w[i], a.o[i][rh * hd + c], o);
        out[rh * hd + c] = o * inv;
    }
    if (lse && threadIdx.x == 0) lse[rh] = L > 0.0f ? M + logf(L) : -CUDART_INF_F;
}

}  // namespace

cudaError_t launch_decode(const DecodeParams &p, int hd, int kv_f16, bool /*fast*/, cudaStream_t s) {
    if (p.n_items == 0) return cudaSuccess;
    dim3 grid(p.n_items), block(kDecodeThreads);
    if (hd == 256) {
        if (kv_f16) decode_kernel<256, __half><<<grid, block, 0, s>>>(p);
        else decode_kernel<256, float><<<grid, block, 0, s>>>(p);
    } else if (hd == 512) {
        if (kv_f16) decode_kernel<512, __half><<<grid, block, 0, s>>>(p);
        else decode_kernel<512, float><<<grid, block, 0, s>>>(p);
    } else {
        return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_decode_exact(const DecodeParams &p, int hd, int n_tasks, cudaStream_t s, bool pdl) {
    if (p.n_items == 0 || n_tasks == 0) return cudaSuccess;
    if (p.max_rows <= 0 || p.max_rows > kExactMaxRows || !p.scores) return cudaErrorInvalidValue;
    if (n_tasks * kHeads <= 148) {  // few tasks: one launch, a CTA per (task, head)
        const size_t smem = ((size_t)2 * kExactChunk * (hd + 4) + p.max_rows + kExactChunk * 17) * sizeof(float);
        if (hd == 256) {
            cudaFuncSetAttribute(exact_head_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            return launch_k(pdl, exact_head_kernel<256>, dim3(n_tasks * kHeads), dim3(kHeadThreads), smem, s, p);
        }
        if (hd == 512) {
            cudaFuncSetAttribute(exact_head_kernel<512>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            return launch_k(pdl, exact_head_kernel<512>, dim3(n_tasks * kHeads), dim3(kHeadThreads), smem, s, p);
        }
        return cudaErrorInvalidValue;
    }
    const size_t pv_smem = (size_t)kHeads * p.max_rows * sizeof(float);
    if (pv_smem > 48 * 1024) {
        cudaFuncSetAttribute(exact_pv_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pv_smem);
        cudaFuncSetAttribute(exact_pv_kernel<512>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pv_smem);
    }
    // few tasks: a CTA per head as well, so that the GPU has work to spread
    const bool per_head = n_tasks * (hd / kPvCols) < 148;
    const size_t head_smem = (size_t)p.max_rows * sizeof(float);
    if (hd == 256) {
        const size_t smem = (size_t)kExactChunk * (256 + 4) * sizeof(float);
        cudaFuncSetAttribute(exact_scores_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        cudaError_t e = launch_k(pdl, exact_scores_kernel<256>, dim3(p.n_items), dim3(kDecodeThreads), smem, s, p);
        if (e == cudaSuccess)
            e = per_head ? launch_k(pdl, exact_pv_head_kernel<256>, dim3(n_tasks * kHeads * (256 / kPvCols)),
                                    dim3(kPvCols), head_smem, s, p)
                         : launch_k(pdl, exact_pv_kernel<256>, dim3(n_tasks * (256 / kPvCols)), dim3(kPvCols),
                                    pv_smem, s, p);
        if (e != cudaSuccess) return e;
    } else if (hd == 512) {
        const size_t smem = (size_t)kExactChunk * (512 + 4) * sizeof(float);
        cudaFuncSetAttribute(exact_scores_kernel<512>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        cudaError_t e = launch_k(pdl, exact_scores_kernel<512>, dim3(p.n_items), dim3(kDecodeThreads), smem, s, p);
        if (e == cudaSuccess)
            e = per_head ? launch_k(pdl, exact_pv_head_kernel<512>, dim3(n_tasks * kHeads * (512 / kPvCols)),
                                    dim3(kPvCols), head_smem, s, p)
                         : launch_k(pdl, exact_pv_kernel<512>, dim3(n_tasks * (512 / kPvCols)), dim3(kPvCols),
                                    pv_smem, s, p);
        if (e != cudaSuccess) return e;
    } else {
        return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

template <int HD>
cudaError_t launch_prompt_hd(const DecodeParams &p, int n_tasks, int cl, int n_blocks, int splits, cudaStream_t s,
                             bool pdl) {
    constexpr int KS = HD + 4;
    const size_t sc_smem = ((size_t)kPromptQH * HD + 2 * kPromptKeys * KS + kPromptQH * kPromptKeys * kPromptRed) *
                           sizeof(float);
    const size_t pv_smem = (size_t)2 * kPromptPvKeys * (kPromptPvCols + kPromptQH) * sizeof(float);
    cudaFuncSetAttribute(prompt_scores_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sc_smem);
    cudaError_t e = launch_k(pdl, prompt_q_kernel<HD>, dim3(n_tasks), dim3(32 * kHeads), 0, s, p);
    if (e == cudaSuccess)
        e = launch_k(pdl, prompt_scores_kernel<HD>, dim3(n_blocks, splits), dim3(256), sc_smem, s, p, cl);
    if (e == cudaSuccess)
        e = launch_k(pdl, prompt_softmax_kernel, dim3(n_tasks), dim3(256), 0, s, p, n_tasks * kHeads);
    if (e == cudaSuccess)
        e = launch_k(pdl, prompt_pv_kernel<HD>, dim3(n_blocks, HD / kPromptPvCols), dim3(256), pv_smem, s, p, cl);
    return e;
}

cudaError_t launch_prompt_exact(const DecodeParams &p, int hd, int n_tasks, int cl, cudaStream_t s, bool pdl) {
    if (n_tasks == 0) return cudaSuccess;
    if (cl < 1 || n_tasks % cl || p.max_rows <= 0 || p.max_rows > kExactMaxRows || !p.scores)
        return cudaErrorInvalidValue;
    const int n_blocks = (n_tasks / cl) * ((cl + kPromptQ - 1) / kPromptQ);
    // key chunks of one block: at most max_rows rows; splits spread them over
    // about four CTAs per SM in all (a CTA with no chunk exits at once)
    const int max_chunks = (p.max_rows + kPromptKeys - 1) / kPromptKeys;
    int splits = (4 * 148 + n_blocks - 1) / n_blocks;
    splits = splits < 1 ? 1 : (splits > max_chunks ? max_chunks : splits);
    if (hd == 256) return launch_prompt_hd<256>(p, n_tasks, cl, n_blocks, splits, s, pdl);
    if (hd == 512) return launch_prompt_hd<512>(p, n_tasks, cl, n_blocks, splits, s, pdl);
    return cudaErrorInvalidValue;
}

cudaError_t launch_task_append(const DecodeParams &p, int hd, int n_tasks, cudaStream_t s, bool pdl) {
    if (n_tasks == 0) return cudaSuccess;
    if (hd == 256) return launch_k(pdl, task_append_kernel<256>, dim3(n_tasks), dim3(64), 0, s, p);
    if (hd == 512) return launch_k(pdl, task_append_kernel<512>, dim3(n_tasks), dim3(64), 0, s, p);
    return cudaErrorInvalidValue;
}

cudaError_t launch_attend_generic(const float *q, const float *k, const float *v, int64_t len, int n_heads, int n_kv,
                                  int hd, float scale, float *out, int *err_flag, cudaStream_t s) {
    attend_generic_kernel<<<n_heads, 256, 0, s>>>(q, k, v, len, n_heads, n_kv, hd, scale, out, err_flag);
    return cudaGetLastError();
}

cudaError_t launch_append(const AppendParams &p, int kv_f16, cudaStream_t s) {
    if (p.n_rows == 0) return cudaSuccess;
    if (p.hd == 256 || p.hd == 512) {
        if (p.hd == 256) {
            if (kv_f16) append_kernel<256, __half><<<p.n_rows, 64, 0, s>>>(p);
            else append_kernel<256, float><<<p.n_rows, 64, 0, s>>>(p);
        } else {
            if (kv_f16) append_kernel<512, __half><<<p.n_rows, 64, 0, s>>>(p);
            else append_kernel<512, float><<<p.n_rows, 64, 0, s>>>(p);
        }
    } else {
        if (p.raw) return cudaErrorInvalidValue;
        if (kv_f16) append_any_kernel<__half><<<p.n_rows, 128, 0, s>>>(p);
        else append_any_kernel<float><<<p.n_rows, 128, 0, s>>>(p);
    }
    return cudaGetLastError();
}

cudaError_t launch_view(const ViewParams &p, int kv_f16, cudaStream_t s) {
    if (p.n_rows == 0) return cudaSuccess;
    if (kv_f16) view_kernel<__half><<<p.n_rows, 128, 0, s>>>(p);
    else view_kernel<float><<<p.n_rows, 128, 0, s>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_lse_merge(int n_parts, const float *const *parts_o, const float *const *parts_lse, int64_t rows,
                             int n_heads, int hd, float *out, float *lse, cudaStream_t s) {
    if (n_parts < 1 || n_parts > kMaxMergeParts) return cudaErrorInvalidValue;
    MergeArgs a{};
    for (int i = 0; i < n_parts; i++) {
        a.o[i] = parts_o[i];
        a.lse[i] = parts_lse[i];
    }
    const int64_t n = rows * n_heads;
    if (n == 0) return cudaSuccess;
    lse_merge_kernel<<<(unsigned)n, 128, 0, s>>>(a, n_parts, hd, out, lse);
    return cudaGetLastError();
}

}  // namespace g4a
