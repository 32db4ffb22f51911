// Paged decode attention over an f16 KV cache on sm_100a.
//
// Replaces, for batched decoding, crates/llm-gemma4/src/impl_/model.rs:393-410
// (q/k norms, RoPE, append, view, window, attend) and :326-366 (attend_head).
// Fused per (sequence, layer) task: q RMSNorm + RoPE, the appended token's
// k/v norm + RoPE + store, attention over the window of the paged cache, and
// for split tasks a log-sum-exp merge by the last CTA to finish.
//
// Structure (one persistent CTA per SM, items taken round-robin):
//   warp 4      producer: for every 64 KB stage (S rows of K and of V, S =
//               16384 / head width, page-aligned so a stage never crosses a
//               page) it issues head_width/64 TMA box loads per tensor into a
//               3-slot ring (64 x S boxes, 128-byte swizzle, no multicast).
//   warps 0-3   q prep (2 heads per warp), the new row, then per stage:
//               S = Q K^T on tensor cores (mma.sync m16n8k16, f16 inputs, f32
//               accumulate): the 16 MMA rows are the 8 heads' q split into a
//               high and a low f16 half, so the two partial scores add up to
//               the f32 score to about 2^-22 relative; keys are split across
//               the 4 warps. The stage's softmax statistics are computed by
//               every warp (same inputs, same result), P is split hi/lo the
//               same way, and O^T += V^T P^T runs with the head dimension split
//               across the warps (O stays in 32 registers per thread).
// Accuracy: within 1e-4 of the reference's f32 attention on the same f16 rows.
// All mbarrier waits are bounded; a time-out sets bit 2 of the error flag and
// the CTA leaves its loops at the next common barrier.
#include <cuda.h>
#include <cuda_fp16.h>
#include <math_constants.h>

#include "internal.h"
#include "sm100_ptx.cuh"

namespace g4a {
namespace {

constexpr int kWarpsC = 4;                 // compute warps
constexpr int kThreadsF16 = 32 * (kWarpsC + 1);
constexpr int kSlots = 3;
constexpr int kStageBytes = 65536;         // K + V of one stage
constexpr uint32_t kPollLimit = 1u << 22;

template <int HD>
struct F16Cfg {
    static constexpr int S = 16384 / HD;          // rows per stage: 64 (hd 256) or 32 (hd 512)
    static constexpr int kBoxBytes = S * 128;     // one 64-column box of S rows
    static constexpr int kBoxes = HD / 64;
    static constexpr int kKeysPerWarp = S / kWarpsC;   // 16 or 8
    static constexpr int kNT = kKeysPerWarp / 8;       // QK n-tiles per warp
    static constexpr int kKS = HD / 16;                // k-steps over the head width
    static constexpr int kMT = HD / 16 / kWarpsC;      // PV m-tiles per warp
    static constexpr int kPVK = S / 16;                // PV k-steps per stage
    static constexpr int kSmemQ = 16 * HD * 2;         // hi/lo q, f16
    static_assert(2 * kBoxes * kBoxBytes == kStageBytes, "a stage is 32 KB of K and 32 KB of V");
    static_assert(S <= 64, "score buffer holds 64 keys per head");
    static constexpr int kSmemBytes = kSlots * kStageBytes + kSmemQ + 2 * 8 * 64 * 4 + 2 * HD * 2 + 1024 + 1024;
};

struct F16Bars {
    uint64_t full[kSlots];
    uint64_t empty[kSlots];
    int abort;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t &r0, uint32_t &r1) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack2(__half lo, __half hi) {
    return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}
__device__ __forceinline__ void compute_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Byte offset of element (row, col) inside a stage tensor stored as HD/64
// boxes of [S rows][128 B] with the 128-byte swizzle (16-byte chunk index
// XOR row % 8).
template <int HD>
__device__ __forceinline__ uint32_t box_off(int row, int col) {
    using C = F16Cfg<HD>;
    const int box = col >> 6, chunk = (col >> 3) & 7;
    return box * C::kBoxBytes + row * 128 + ((chunk ^ (row & 7)) << 4) + (col & 7) * 2;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// RMSNorm (+weight) and optional NEOX RoPE of one head held by a warp, lane
// owning elements lane + 32 k; the same operation order as the oracle.
template <int HD>
__device__ __forceinline__ void norm_rope(float (&x)[HD / 32], const float *w, const float2 *rope_row, float eps,
                                          int lane) {
    constexpr int PL = HD / 32;
    double ss = 0.0;
#pragma unroll
    for (int k = 0; k < PL; k++) ss += (double)__fmul_rn(x[k], x[k]);
    ss = warp_sum_d(ss);
    const float mean = (float)(ss / (double)HD);
    const float scale = 1.0f / sqrtf(mean + eps);
#pragma unroll
    for (int k = 0; k < PL; k++) {
        float y = __fmul_rn(x[k], scale);
        if (w) y = __fmul_rn(y, __ldg(w + lane + 32 * k));
        x[k] = y;
    }
    if (rope_row) {
#pragma unroll
        for (int k = 0; k < PL / 2; k++) {
            const float2 sc = __ldg(rope_row + lane + 32 * k);
            const float a = x[k], b = x[k + PL / 2];
            x[k] = __fsub_rn(__fmul_rn(a, sc.y), __fmul_rn(b, sc.x));
            x[k + PL / 2] = __fadd_rn(__fmul_rn(a, sc.x), __fmul_rn(b, sc.y));
        }
    }
}

template <int HD>
__global__ void __launch_bounds__(kThreadsF16, 1) decode_f16_kernel(DecodeParams p) {
    using C = F16Cfg<HD>;
    constexpr int S = C::S;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *stages = smem;                                 // kSlots x 64 KB
    uint8_t *q_smem = stages + kSlots * kStageBytes;        // [16][HD] f16, swizzled
    float *s_smem = reinterpret_cast<float *>(q_smem + C::kSmemQ);  // [2][8][S]
    __half *new_kv = reinterpret_cast<__half *>(s_smem + 2 * 8 * 64);  // k then v, [HD] each
    F16Bars *bars = reinterpret_cast<F16Bars *>(new_kv + 2 * HD);
    __shared__ int last_s;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kSlots; i++) {
            ptx::mbar_init(&bars->full[i], 1);
            ptx::mbar_init(&bars->empty[i], kWarpsC);
        }
        bars->abort = 0;
        ptx::fence_mbar_init();
    }
    __syncthreads();
    volatile int *abort = &bars->abort;

    if (warp == kWarpsC) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            uint32_t st = 0;  // global stage counter across items
            for (int item = blockIdx.x; item < p.n_items && !*abort; item += gridDim.x) {
                const DecodeItem it = p.items[item];
                const DecodeTask &tk = p.tasks[it.task];
                const int32_t *bt = p.block_table + (size_t)tk.seq * p.max_pages;
                const int first = it.row_lo / S * S;
                for (int r0 = first; r0 < it.row_hi; r0 += S, st++) {
                    const int slot = st % kSlots;
                    const uint32_t ph = (st / kSlots) & 1u;
                    bool got = false;
                    for (uint32_t i = 0; i < kPollLimit; i++) {
                        if (ptx::mbar_try_wait(&bars->empty[slot], ph ^ 1u)) {
                            got = true;
                            break;
                        }
                        if ((i & 1023) == 1023 && *abort) break;
                    }
                    if (!got) {
                        if (!*abort) atomicOr(p.err_flag, 4);
                        *abort = 1;
                        break;
                    }
                    const int page = __ldg(bt + r0 / p.page_tokens);
                    const int y = page * p.page_tokens + (r0 % p.page_tokens);
                    uint8_t *dst = stages + slot * kStageBytes;
                    ptx::mbar_arrive_expect_tx(&bars->full[slot], kStageBytes);
#pragma unroll
                    for (int c = 0; c < C::kBoxes; c++) {
                        ptx::tma_load_2d(dst + c * C::kBoxBytes, tk.tmap_k, &bars->full[slot], 64 * c, y);
                        ptx::tma_load_2d(dst + kStageBytes / 2 + c * C::kBoxBytes, tk.tmap_v, &bars->full[slot],
                                         64 * c, y);
                    }
                }
            }
            // every issued load lands before the CTA may exit
            for (uint32_t s2 = (st > kSlots ? st - kSlots : 0); s2 < st; s2++) {
                for (uint32_t i = 0; i < kPollLimit && !ptx::mbar_try_wait(&bars->full[s2 % kSlots], (s2 / kSlots) & 1u);
                     i++) {
                }
            }
        }
        return;
    }

    // ---------------------------------------------------------------- compute
    const uint32_t q_base = ptx::smem_u32(q_smem);
    const uint32_t st_base = ptx::smem_u32(stages);
    uint32_t st = 0;
    for (int item = blockIdx.x; item < p.n_items; item += gridDim.x) {
        const DecodeItem it = p.items[item];
        const DecodeTask &tk = p.tasks[it.task];
        const float2 *rope = tk.global ? p.rope_global : p.rope_local;
        // -- q: norm + RoPE (model.rs:395-396), hi/lo f16 split into smem
        for (int hh = 0; hh < 2; hh++) {
            const int h = warp * 2 + hh;
            float x[HD / 32];
#pragma unroll
            for (int k = 0; k < HD / 32; k++) x[k] = __ldg(tk.q_raw + (size_t)h * HD + lane + 32 * k);
            if (!tk.q_ready) norm_rope<HD>(x, tk.q_w, rope + (size_t)tk.position * (HD / 2), p.eps, lane);
#pragma unroll
            for (int k = 0; k < HD / 32; k++) {
                const int col = lane + 32 * k;
                const float v = x[k] * tk.scale;
                const __half hi = __float2half_rn(v);
                const __half lo = __float2half_rn(v - __half2float(hi));
                const int chunk = col >> 3;
                *reinterpret_cast<__half *>(q_smem + h * HD * 2 + (((chunk ^ (h & 7)) << 4) | ((col & 7) * 2))) = hi;
                const int r2 = h + 8;
                *reinterpret_cast<__half *>(q_smem + r2 * HD * 2 + (((chunk ^ (r2 & 7)) << 4) | ((col & 7) * 2))) = lo;
            }
        }
        // -- the appended token (model.rs:400-405), by the item holding its row
        const bool has_new = tk.new_row >= 0 && ((tk.new_row >= it.row_lo && tk.new_row < it.row_hi) ||
                                                 (it.split == tk.n_splits - 1 && tk.new_row >= it.row_hi));
        if (has_new && warp < 2) {
            float x[HD / 32];
            const float *src = warp == 0 ? tk.k_raw : tk.v_raw;
#pragma unroll
            for (int k = 0; k < HD / 32; k++) x[k] = __ldg(src + lane + 32 * k);
            if (warp == 0)
                norm_rope<HD>(x, tk.k_w, rope + (size_t)tk.position * (HD / 2), p.eps, lane);
            else
                norm_rope<HD>(x, nullptr, nullptr, p.eps, lane);
            const int32_t *bt = p.block_table + (size_t)tk.seq * p.max_pages;
            const int page = bt[tk.new_row / p.page_tokens];
            __half *dst = const_cast<__half *>(reinterpret_cast<const __half *>(warp == 0 ? tk.k_base : tk.v_base)) +
                          ((size_t)page * p.page_tokens + (tk.new_row % p.page_tokens)) * HD;
#pragma unroll
            for (int k = 0; k < HD / 32; k++) {
                const __half h16 = __float2half_rn(x[k]);
                dst[lane + 32 * k] = h16;
                new_kv[warp * HD + lane + 32 * k] = h16;
            }
        }
        compute_bar();
        // -- A fragments of Q (hi rows 0-7, lo rows 8-15) for every k-step
        uint32_t qa[C::kKS][4];
#pragma unroll
        for (int ks = 0; ks < C::kKS; ks++) {
            const int row = (lane & 7) + ((lane >> 3) & 1) * 8;
            const int chunk = ks * 2 + (lane >> 4);
            ldsm_x4(q_base + row * HD * 2 + ((chunk ^ (row & 7)) << 4), qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3]);
        }
        // per-head running stats for head g (identical in every warp)
        float m_run = -CUDART_INF_F, l_run = 0.0f;
        float acc[C::kMT][4];
#pragma unroll
        for (int mt = 0; mt < C::kMT; mt++)
#pragma unroll
            for (int i = 0; i < 4; i++) acc[mt][i] = 0.0f;
        bool bad = false;
        const int first = it.row_lo / S * S;
        bool aborted = false;
        for (int r0 = first; r0 < it.row_hi; r0 += S, st++) {
            const int slot = st % kSlots;
            const uint32_t ph = (st / kSlots) & 1u;
            bool got = false;
            for (uint32_t i = 0; i < kPollLimit; i++) {
                if (ptx::mbar_try_wait(&bars->full[slot], ph)) {
                    got = true;
                    break;
                }
                if ((i & 1023) == 1023 && *abort) break;
            }
            if (!got && !*abort) {
                atomicOr(p.err_flag, 4);
                *abort = 1;
            }
            const uint32_t kb = st_base + slot * kStageBytes;
            const uint32_t vb = kb + kStageBytes / 2;
            uint8_t *vgen = stages + slot * kStageBytes + kStageBytes / 2;
            uint8_t *kgen = stages + slot * kStageBytes;
            // rows of this stage outside [row_lo, row_hi) are masked; their V
            // rows are zeroed (a masked weight is 0, and 0 * garbage could be
            // NaN); the appended row is patched in from the computed values.
            const bool partial = r0 < it.row_lo || r0 + S > it.row_hi;
            const bool patch = tk.new_row >= r0 && tk.new_row < r0 + S && tk.new_row >= it.row_lo &&
                               tk.new_row < it.row_hi;
            if (got && (partial || patch)) {
                for (int e = threadIdx.x; e < S * (HD / 8); e += 32 * kWarpsC) {
                    const int row = e / (HD / 8), c8 = (e % (HD / 8)) * 8;
                    const int r = r0 + row;
                    if (r < it.row_lo || r >= it.row_hi) {
                        *reinterpret_cast<uint4 *>(vgen + box_off<HD>(row, c8)) = make_uint4(0, 0, 0, 0);
                    } else if (r == tk.new_row) {
                        *reinterpret_cast<uint4 *>(kgen + box_off<HD>(row, c8)) =
                            *reinterpret_cast<const uint4 *>(new_kv + c8);
                        *reinterpret_cast<uint4 *>(vgen + box_off<HD>(row, c8)) =
                            *reinterpret_cast<const uint4 *>(new_kv + HD + c8);
                    }
                }
                // these generic-proxy writes must be ordered before the TMA
                // that later refills this slot
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            }
            compute_bar();
            if (*abort) {
                aborted = true;
                break;
            }
            float *s_buf = s_smem + (st & 1) * 8 * 64;
            // -- S = Q K^T for this warp's keys
            {
                float sc[C::kNT][4];
#pragma unroll
                for (int n = 0; n < C::kNT; n++)
#pragma unroll
                    for (int i = 0; i < 4; i++) sc[n][i] = 0.0f;
                const int key0 = warp * C::kKeysPerWarp;
#pragma unroll
                for (int ks = 0; ks < C::kKS; ks++) {
                    if constexpr (C::kNT == 2) {
                        // matrices: keys key0..+7 at d 16ks, +8; keys key0+8..+15 at d 16ks, +8
                        const int row = key0 + (lane & 7) + ((lane >> 4) << 3);
                        const int col = ks * 16 + ((lane >> 3) & 1) * 8;
                        uint32_t b0, b1, b2, b3;
                        ldsm_x4(kb + box_off<HD>(row, col), b0, b1, b2, b3);
                        mma16816(sc[0], qa[ks], b0, b1);
                        mma16816(sc[1], qa[ks], b2, b3);
                    } else {
                        const int row = key0 + (lane & 7);
                        const int col = ks * 16 + ((lane >> 3) & 1) * 8;
                        uint32_t b0, b1;
                        ldsm_x2(kb + box_off<HD>(row, col), b0, b1);
                        mma16816(sc[0], qa[ks], b0, b1);
                    }
                }
#pragma unroll
                for (int n = 0; n < C::kNT; n++) {
#pragma unroll
                    for (int j = 0; j < 2; j++) {
                        const int key = key0 + n * 8 + 2 * t + j;
                        const int r = r0 + key;
                        float s = sc[n][j] + sc[n][j + 2];  // hi + lo rows
                        if (r < it.row_lo || r >= it.row_hi) s = -CUDART_INF_F;
                        else if (isnan(s) || s == CUDART_INF_F) bad = true;
                        s_buf[g * 64 + key] = s;
                    }
                }
            }
            compute_bar();
            // -- online softmax of head g over this stage (every warp alike)
            float pv[C::kPVK][4];
            float smax = -CUDART_INF_F;
#pragma unroll
            for (int kk = 0; kk < C::kPVK; kk++) {
                pv[kk][0] = s_buf[g * 64 + kk * 16 + 2 * t];
                pv[kk][1] = s_buf[g * 64 + kk * 16 + 2 * t + 1];
                pv[kk][2] = s_buf[g * 64 + kk * 16 + 2 * t + 8];
                pv[kk][3] = s_buf[g * 64 + kk * 16 + 2 * t + 9];
#pragma unroll
                for (int i = 0; i < 4; i++) smax = fmaxf(smax, pv[kk][i]);
            }
            smax = fmaxf(smax, __shfl_xor_sync(0xffffffffu, smax, 1));
            smax = fmaxf(smax, __shfl_xor_sync(0xffffffffu, smax, 2));
            const float m_new = fmaxf(m_run, smax);
            const float alpha = m_new == -CUDART_INF_F ? 1.0f : expf(m_run - m_new);
            float lsum = 0.0f;
            uint32_t bhi[C::kPVK][2], blo[C::kPVK][2];
#pragma unroll
            for (int kk = 0; kk < C::kPVK; kk++) {
                __half hi[4], lo[4];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const float e = m_new == -CUDART_INF_F ? 0.0f : expf(pv[kk][i] - m_new);
                    lsum += e;
                    hi[i] = __float2half_rn(e);
                    lo[i] = __float2half_rn(e - __half2float(hi[i]));
                }
                bhi[kk][0] = pack2(hi[0], hi[1]);
                bhi[kk][1] = pack2(hi[2], hi[3]);
                blo[kk][0] = pack2(lo[0], lo[1]);
                blo[kk][1] = pack2(lo[2], lo[3]);
            }
            lsum += __shfl_xor_sync(0xffffffffu, lsum, 1);
            lsum += __shfl_xor_sync(0xffffffffu, lsum, 2);
            l_run = l_run * alpha + lsum;
            m_run = m_new;
            // -- O^T += V^T P^T for this warp's head-dimension quarter
            const float a0 = __shfl_sync(0xffffffffu, alpha, 8 * t);      // head 2t
            const float a1 = __shfl_sync(0xffffffffu, alpha, 8 * t + 4);  // head 2t+1
#pragma unroll
            for (int mt = 0; mt < C::kMT; mt++) {
                acc[mt][0] *= a0;
                acc[mt][1] *= a1;
                acc[mt][2] *= a0;
                acc[mt][3] *= a1;
            }
#pragma unroll
            for (int kk = 0; kk < C::kPVK; kk++) {
#pragma unroll
                for (int mt = 0; mt < C::kMT; mt++) {
                    const int dm = (warp * C::kMT + mt) * 16;
                    const int row = kk * 16 + (lane & 7) + ((lane >> 4) << 3);
                    const int col = dm + ((lane >> 3) & 1) * 8;
                    uint32_t a[4];
                    ldsm_x4_t(vb + box_off<HD>(row, col), a[0], a[1], a[2], a[3]);
                    mma16816(acc[mt], a, bhi[kk][0], bhi[kk][1]);
                    mma16816(acc[mt], a, blo[kk][0], blo[kk][1]);
                }
            }
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(&bars->empty[slot]);
        }
        if (aborted) return;
        if (bad) atomicOr(p.err_flag, 1);
        // ---- output: O[h][d] for h = 2t, 2t+1 and d = dm + g (+8)
        const float l0 = __shfl_sync(0xffffffffu, l_run, 8 * t), l1 = __shfl_sync(0xffffffffu, l_run, 8 * t + 4);
        if (tk.n_splits == 1) {
            const float i0 = 1.0f / l0, i1 = 1.0f / l1;
#pragma unroll
            for (int mt = 0; mt < C::kMT; mt++) {
                const int dm = (warp * C::kMT + mt) * 16;
                tk.out[(2 * t) * HD + dm + g] = acc[mt][0] * i0;
                tk.out[(2 * t + 1) * HD + dm + g] = acc[mt][1] * i1;
                tk.out[(2 * t) * HD + dm + g + 8] = acc[mt][2] * i0;
                tk.out[(2 * t + 1) * HD + dm + g + 8] = acc[mt][3] * i1;
            }
            if (warp == 0 && t == 0 && !(l_run > 0.0f)) atomicOr(p.err_flag, 1);
            continue;
        }
        const int slot_p = tk.partial_base + it.split;
        float *po = p.part_o + (size_t)slot_p * kHeads * 512;
#pragma unroll
        for (int mt = 0; mt < C::kMT; mt++) {
            const int dm = (warp * C::kMT + mt) * 16;
            po[(2 * t) * HD + dm + g] = acc[mt][0];
            po[(2 * t + 1) * HD + dm + g] = acc[mt][1];
            po[(2 * t) * HD + dm + g + 8] = acc[mt][2];
            po[(2 * t + 1) * HD + dm + g + 8] = acc[mt][3];
        }
        if (warp == 0 && t == 0) {
            p.part_ml[(size_t)slot_p * 2 * kHeads + g] = m_run;
            p.part_ml[(size_t)slot_p * 2 * kHeads + kHeads + g] = l_run;
        }
        __threadfence();
        compute_bar();
        if (threadIdx.x == 0) last_s = atomicAdd(p.tickets + it.task, 1u) == (unsigned)(tk.n_splits - 1);
        compute_bar();
        if (last_s) {
            __threadfence();
            // merge: weights per (split, head) in parallel, then each thread
            // sums its columns over the splits
            const int ns = tk.n_splits;
            const float *pml = p.part_ml + (size_t)tk.partial_base * 2 * kHeads;
            const float *pall = p.part_o + (size_t)tk.partial_base * kHeads * 512;
            float *wsm = s_smem;  // reuse: [ns][8] weights then [8] 1/L, ns <= 96
            for (int h = warp; h < kHeads; h += kWarpsC) {
                float M = -CUDART_INF_F;
                for (int s = lane; s < ns; s += 32) M = fmaxf(M, __ldcg(pml + (size_t)s * 2 * kHeads + h));
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
                float L = 0.0f;
                for (int s = lane; s < ns; s += 32) {
                    const float ms = __ldcg(pml + (size_t)s * 2 * kHeads + h);
                    const float w = ms == -CUDART_INF_F ? 0.0f : expf(ms - M);
                    wsm[s * 8 + h] = w;
                    L = fmaf(__ldcg(pml + (size_t)s * 2 * kHeads + kHeads + h), w, L);
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
                if (lane == 0) {
                    wsm[ns * 8 + h] = 1.0f / L;
                    if (!(L > 0.0f)) atomicOr(p.err_flag, 1);
                }
            }
            compute_bar();
            for (int e = threadIdx.x; e < kHeads * HD; e += 32 * kWarpsC) {
                const int h = e / HD;
                float o = 0.0f;
                for (int s = 0; s < ns; s++) o = fmaf(__ldcg(pall + (size_t)s * kHeads * 512 + e), wsm[s * 8 + h], o);
                tk.out[e] = o * wsm[ns * 8 + h];
            }
            if (threadIdx.x == 0) p.tickets[it.task] = 0u;
            compute_bar();
        }
    }
}

}  // namespace

int decode_f16_smem_bytes(int hd) { return hd == 256 ? F16Cfg<256>::kSmemBytes : F16Cfg<512>::kSmemBytes; }

cudaError_t launch_decode_f16(const DecodeParams &p, int hd, int n_sm, cudaStream_t s) {
    if (p.n_items == 0) return cudaSuccess;
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(decode_f16_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             F16Cfg<256>::kSmemBytes);
        cudaFuncSetAttribute(decode_f16_kernel<512>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             F16Cfg<512>::kSmemBytes);
        attr = true;
    }
    const int grid = p.n_items < n_sm ? p.n_items : n_sm;
    if (hd == 256)
        decode_f16_kernel<256><<<grid, kThreadsF16, F16Cfg<256>::kSmemBytes, s>>>(p);
    else if (hd == 512)
        decode_f16_kernel<512><<<grid, kThreadsF16, F16Cfg<512>::kSmemBytes, s>>>(p);
    else
        return cudaErrorInvalidValue;
    return cudaGetLastError();
}

}  // namespace g4a
