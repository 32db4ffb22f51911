// Paged decode attention over an f16 KV cache on sm_100a.
//
// Replaces, for batched decoding, crates/llm-gemma4/src/impl_/model.rs:393-410
// (q/k norms, RoPE, append, view, window, attend) and :326-366 (attend_head).
// Sliding (256-wide) and global (512-wide) layers run in the same launches.
//
// Three kernels per step:
//   prep     one CTA per (sequence, layer) task: q RMSNorm + RoPE, split into
//            a high and a low f16 half and stored in the layout the main
//            kernel's shared memory uses; on KV-owning layers the new token's
//            k (norm + RoPE) and v (norm) are stored into the paged cache.
//   main     one persistent CTA per SM, items (row ranges of tasks) assigned
//            by the host longest-processing-time first.
//            warp 8    producer: per item one bulk copy of the task's q block,
//                      then every 64 KB stage (S rows of K and of V, S = 16384
//                      / head width, page-aligned) as head_width/64 TMA box
//                      loads per tensor (64 columns x S rows, 128-byte
//                      swizzle, no multicast) into a 3-slot ring.
//            warps 0-7 S = Q K^T with mma.sync m16n8k16 (f16 in, f32
//                      accumulate); the 16 MMA rows are the hi and lo halves
//                      of the 8 heads' q, so the two partial scores add up to
//                      the f32 score to about 2^-22 relative. Warp w takes key
//                      half w/4 and head-dimension quarter w%4 (MMA chains 4
//                      deep); quarter sums meet in shared memory; every warp
//                      computes the stage's softmax statistics (same inputs,
//                      same result), splits P hi/lo the same way and
//                      accumulates O^T += V^T P^T for its eighth of the head
//                      dimension. Items of split tasks store (O, max, sum).
//   combine  one CTA per split task: log-sum-exp merge of its items.
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

constexpr int kWarpsC = 8;                      // compute warps
constexpr int kThreadsF16 = 32 * (kWarpsC + 1);
constexpr int kSlots = 3;
constexpr int kStageBytes = 65536;              // K + V of one stage
// q hi/lo block at [0, 16 KB), two score-partial buffers at [16 KB, 32 KB):
// the same places for both head widths, so the producer's copy of the next
// item's q never lands on partials the compute warps are still reading.
constexpr int kQRegion = 16384;
constexpr int kRegionBytes = 32768;
constexpr uint32_t kPollLimit = 1u << 22;

template <int HD>
struct F16Cfg {
    static constexpr int S = 16384 / HD;        // rows per stage: 64 (hd 256) or 32 (hd 512)
    static constexpr int kBoxBytes = S * 128;   // one 64-column box of S rows
    static constexpr int kBoxes = HD / 64;
    static constexpr int kKeysQ = S / 4;        // keys per QK warp (a key quarter)
    static constexpr int kNT = kKeysQ / 8;      // QK n-tiles per warp: 2 or 1
    static constexpr int kKSH = HD / 32;        // k-steps per head-dimension half: 8 or 16
    static constexpr int kNCH = 4 / kNT;        // accumulator chains per n-tile (4 chains of 4)
    static constexpr int kMT = HD / 128;        // PV m-tiles per warp (an eighth of hd): 2 or 4
    static constexpr int kPVK = S / 16;         // PV k-steps per stage
    static constexpr int kQBytes = 16 * HD * 2; // hi/lo q, f16
    // [half][head][key ^ 4*head] f32, one buffer: the XOR keeps the
    // partial-score accesses at most 2-way bank-conflicted
    static constexpr int kSPartBytes = 2 * 8 * S * 4;
    static_assert(2 * kBoxes * kBoxBytes == kStageBytes, "a stage is 32 KB of K and 32 KB of V");
    static_assert(kQBytes <= kQRegion && kQRegion + 2 * kSPartBytes <= kRegionBytes, "region layout");
    static_assert(kKSH % kNCH == 0, "chains divide the k-steps");
};

constexpr int kSmemBytes = kSlots * kStageBytes + kRegionBytes + 128 + 1024;

struct F16Bars {
    uint64_t full[kSlots];
    uint64_t empty[kSlots];
    uint64_t q_full, q_empty;
    int abort;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
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
// Programmatic dependent launch: a kernel launched with the programmatic
// stream-serialization attribute may start before its predecessor ends; it
// must wait here before touching what the predecessor writes. Without the
// attribute both instructions do nothing.
__device__ __forceinline__ void wait_prerequisite() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void release_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// named barrier of the 8 compute warps (the producer never takes part)
__device__ __forceinline__ void compute_bar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     ptx::smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(ptx::smem_u32(bar))
                 : "memory");
}

// Byte offset of element (row, col) inside a stage tensor stored as HD/64
// boxes of [S rows][128 B] with the 128-byte swizzle (16-byte chunk index
// XOR row % 8).
template <int HD>
__device__ __forceinline__ uint32_t box_off(int row, int col) {
    using C = F16Cfg<HD>;
    const int box = col >> 6, chunk = (col >> 3) & 7;
    return box * C::kBoxBytes + row * 128 + ((chunk ^ (row & 7)) << 4) + (col & 7) * 2;
}

// Byte offset of (row, col) in a [16][HD] f16 q block: 16-byte chunks of a
// row XOR-ed with row % 8 (conflict-free ldmatrix).
template <int HD>
__device__ __forceinline__ uint32_t q_off(int row, int col) {
    return row * HD * 2 + ((((col >> 3) ^ (row & 7))) << 4) + (col & 7) * 2;
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

// norm_rope with the weight and the RoPE row fetched before the reduction,
// so the three global reads overlap.
template <int HD>
__device__ __forceinline__ void norm_rope_pre(float (&x)[HD / 32], const float *w, const float2 *rope_row, float eps,
                                              int lane) {
    constexpr int PL = HD / 32;
    float wv[PL];
    float2 sc[PL / 2];
#pragma unroll
    for (int k = 0; k < PL; k++) wv[k] = w ? __ldg(w + lane + 32 * k) : 1.0f;
#pragma unroll
    for (int k = 0; k < PL / 2; k++) sc[k] = rope_row ? __ldg(rope_row + lane + 32 * k) : make_float2(0.f, 1.f);
    double ss = 0.0;
#pragma unroll
    for (int k = 0; k < PL; k++) ss += (double)__fmul_rn(x[k], x[k]);
    ss = warp_sum_d(ss);
    const float mean = (float)(ss / (double)HD);
    const float scale = 1.0f / sqrtf(mean + eps);
#pragma unroll
    for (int k = 0; k < PL; k++) {
        float y = __fmul_rn(x[k], scale);
        if (w) y = __fmul_rn(y, wv[k]);
        x[k] = y;
    }
    if (rope_row) {
#pragma unroll
        for (int k = 0; k < PL / 2; k++) {
            const float a = x[k], b = x[k + PL / 2];
            x[k] = __fsub_rn(__fmul_rn(a, sc[k].y), __fmul_rn(b, sc[k].x));
            x[k + PL / 2] = __fadd_rn(__fmul_rn(a, sc[k].x), __fmul_rn(b, sc[k].y));
        }
    }
}

// ---------------------------------------------------------------------------
// prep: q hi/lo blocks and the appended rows
// ---------------------------------------------------------------------------

template <int HD>
__device__ __forceinline__ void prep_task(const DecodeParams &p, const DecodeTask &tk, int task) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float2 *rope = (tk.global ? p.rope_global : p.rope_local) + (size_t)tk.position * (HD / 2);
    uint8_t *qblk = reinterpret_cast<uint8_t *>(p.q_blocks) + (size_t)task * kQBlockBytes;
    if (warp < kHeads) {  // q of head `warp` (model.rs:395-396)
        const int h = warp;
        float x[HD / 32];
#pragma unroll
        for (int k = 0; k < HD / 32; k++) x[k] = __ldg(tk.q_raw + (size_t)h * HD + lane + 32 * k);
        if (!tk.q_ready) norm_rope_pre<HD>(x, tk.q_w, rope, p.eps, lane);
#pragma unroll
        for (int k = 0; k < HD / 32; k++) {
            const int col = lane + 32 * k;
            const float v = x[k] * tk.scale;
            const __half hi = __float2half_rn(v);
            const __half lo = __float2half_rn(v - __half2float(hi));
            *reinterpret_cast<__half *>(qblk + q_off<HD>(h, col)) = hi;
            *reinterpret_cast<__half *>(qblk + q_off<HD>(h + 8, col)) = lo;
        }
    }
    // the appended token (model.rs:400-405): k on warp 8, v on warp 9, beside
    // the q heads rather than after two of them
    if (tk.new_row >= 0 && warp >= kHeads) {
        const bool is_k = warp == kHeads;
        float x[HD / 32];
        const float *src = is_k ? tk.k_raw : tk.v_raw;
#pragma unroll
        for (int k = 0; k < HD / 32; k++) x[k] = __ldg(src + lane + 32 * k);
        if (is_k)
            norm_rope_pre<HD>(x, tk.k_w, rope, p.eps, lane);
        else
            norm_rope_pre<HD>(x, nullptr, nullptr, p.eps, lane);
        const int32_t *bt = p.block_table + (size_t)tk.seq * p.max_pages;
        const int page = bt[tk.new_row / p.page_tokens];
        __half *dst = const_cast<__half *>(reinterpret_cast<const __half *>(is_k ? tk.k_base : tk.v_base)) +
                      ((size_t)page * p.page_tokens + (tk.new_row % p.page_tokens)) * HD;
#pragma unroll
        for (int k = 0; k < HD / 32; k++) dst[lane + 32 * k] = __float2half_rn(x[k]);
    }
}

constexpr int kPrepThreads = 32 * (kHeads + 2);  // a warp per q head, one for k, one for v
__global__ void __launch_bounds__(kPrepThreads) decode_f16_prep(DecodeParams p) {
    release_dependents();  // the main kernel may be scheduled now; it waits for our writes
    const DecodeTask &tk = p.tasks[blockIdx.x];
    if (tk.hd == 256) prep_task<256>(p, tk, blockIdx.x);
    else prep_task<512>(p, tk, blockIdx.x);
}

// ---------------------------------------------------------------------------
// main
// ---------------------------------------------------------------------------

struct Shared {
    uint8_t *stages;
    uint8_t *region;   // q hi/lo block, then two score-partial buffers
    F16Bars *bars;
};

__device__ __forceinline__ bool wait_poll(uint64_t *bar, uint32_t parity, volatile int *abort, int *err) {
    for (uint32_t i = 0; i < kPollLimit; i++) {
        if (ptx::mbar_try_wait(bar, parity)) return true;
        if ((i & 1023) == 1023 && *abort) return false;
    }
    if (!*abort) atomicOr(err, 4);
    *abort = 1;
    return false;
}

// Producer side of one item: its q block, then its stages.
// Stages are issued first; the q block (written by the prep kernel) follows
// once the stages that fit in the ring are under way, and any stage holding
// an appended row (also written by prep) waits for the prep kernel to end.
template <int HD>
__device__ __forceinline__ bool produce_item(const DecodeParams &p, const DecodeItem &it, const DecodeTask &tk,
                                             const Shared &sh, uint32_t &st, uint32_t ic, bool &prereq_done) {
    using C = F16Cfg<HD>;
    volatile int *abort = &sh.bars->abort;
    bool q_issued = false;
    auto issue_q = [&]() -> bool {
        if (!prereq_done) {
            wait_prerequisite();
            prereq_done = true;
        }
        if (!wait_poll(&sh.bars->q_empty, (ic & 1u) ^ 1u, abort, p.err_flag)) return false;
        ptx::mbar_arrive_expect_tx(&sh.bars->q_full, C::kQBytes);
        bulk_load(sh.region, reinterpret_cast<const uint8_t *>(p.q_blocks) + (size_t)it.task * kQBlockBytes,
                  C::kQBytes, &sh.bars->q_full);
        q_issued = true;
        return true;
    };
    const int32_t *bt = p.block_table + (size_t)tk.seq * p.max_pages;
    const int first = it.row_lo / C::S * C::S;
    int issued = 0;
    for (int r0 = first; r0 < it.row_hi; r0 += C::S, st++, issued++) {
        const int slot = st % kSlots;
        if (!q_issued && issued == kSlots - 1 && !issue_q()) return false;
        if (!prereq_done && tk.new_row >= r0 && tk.new_row < r0 + C::S) {
            wait_prerequisite();
            prereq_done = true;
        }
        if (!wait_poll(&sh.bars->empty[slot], ((st / kSlots) & 1u) ^ 1u, abort, p.err_flag)) return false;
        const int page = __ldg(bt + r0 / p.page_tokens);
        const int y = page * p.page_tokens + (r0 % p.page_tokens);
        uint8_t *dst = sh.stages + slot * kStageBytes;
        ptx::mbar_arrive_expect_tx(&sh.bars->full[slot], kStageBytes);
#pragma unroll
        for (int c = 0; c < C::kBoxes; c++) {
            ptx::tma_load_2d(dst + c * C::kBoxBytes, tk.tmap_k, &sh.bars->full[slot], 64 * c, y);
            ptx::tma_load_2d(dst + kStageBytes / 2 + c * C::kBoxBytes, tk.tmap_v, &sh.bars->full[slot], 64 * c, y);
        }
    }
    if (!q_issued && !issue_q()) return false;
    return true;
}

// Compute side of one item. Returns false if the CTA aborted.
template <int HD>
__device__ __forceinline__ bool compute_item(const DecodeParams &p, const DecodeItem &it, const DecodeTask &tk,
                                             const Shared &sh, uint32_t &st, uint32_t ic) {
    using C = F16Cfg<HD>;
    constexpr int S = C::S;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int kq = warp >> 1, dh = warp & 1;  // QK: key quarter, head-dimension half
    volatile int *abort = &sh.bars->abort;
    float *s_part = reinterpret_cast<float *>(sh.region + kQRegion);

    // -- A fragments of this warp's half of q, then hand the q buffer back
    const bool qok = wait_poll(&sh.bars->q_full, ic & 1u, abort, p.err_flag);
    const uint32_t q_base = ptx::smem_u32(sh.region);
    uint32_t qa[C::kKSH][4];
#pragma unroll
    for (int i = 0; i < C::kKSH; i++) {
        const int ks = dh * C::kKSH + i;
        const int row = (lane & 7) + ((lane >> 3) & 1) * 8;
        const int col = ks * 16 + (lane >> 4) * 8;
        ldsm_x4(q_base + q_off<HD>(row, col), qa[i][0], qa[i][1], qa[i][2], qa[i][3]);
    }
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive(&sh.bars->q_empty);
    if (!qok) {
        compute_bar();
        return false;
    }
    float m_run = -CUDART_INF_F, l_run = 0.0f;  // head g, identical in every warp
    float acc[C::kMT][4];
#pragma unroll
    for (int mt = 0; mt < C::kMT; mt++)
#pragma unroll
        for (int i = 0; i < 4; i++) acc[mt][i] = 0.0f;
    constexpr float kLog2e = 1.4426950408889634f;
    const uint32_t st_base = ptx::smem_u32(sh.stages);

    for (int r0 = it.row_lo / S * S; r0 < it.row_hi; r0 += S, st++) {
        const int slot = st % kSlots;
        const bool got = wait_poll(&sh.bars->full[slot], (st / kSlots) & 1u, abort, p.err_flag);
        const uint32_t kb = st_base + slot * kStageBytes;
        const uint32_t vb = kb + kStageBytes / 2;
        // Rows outside [row_lo, row_hi) are masked and their V rows zeroed (a
        // zero weight times stale data could be NaN). Same decision in every warp.
        const bool partial = r0 < it.row_lo || r0 + S > it.row_hi;
        if (partial) {
            if (got) {
                uint8_t *vgen = sh.stages + slot * kStageBytes + kStageBytes / 2;
                for (int e = threadIdx.x; e < S * (HD / 8); e += 32 * kWarpsC) {
                    const int row = e / (HD / 8), c8 = (e % (HD / 8)) * 8;
                    const int r = r0 + row;
                    if (r < it.row_lo || r >= it.row_hi)
                        *reinterpret_cast<uint4 *>(vgen + box_off<HD>(row, c8)) = make_uint4(0, 0, 0, 0);
                }
                // generic-proxy writes, ordered before the TMA that refills the slot
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            }
            compute_bar();
        }
        float *sp = s_part + (st & 1) * (C::kSPartBytes / 4);
        // -- partial S = Q K^T over this warp's half of the head width
        {
            float sc[C::kNT][C::kNCH][4];
#pragma unroll
            for (int n = 0; n < C::kNT; n++)
#pragma unroll
                for (int c = 0; c < C::kNCH; c++)
#pragma unroll
                    for (int i = 0; i < 4; i++) sc[n][c][i] = 0.0f;
            const int key0 = kq * C::kKeysQ;
            if constexpr (C::kNT == 2) {
#pragma unroll
                for (int i = 0; i < C::kKSH; i++) {
                    // matrices: keys +0..7 at d 16ks, 16ks+8; keys +8..15 likewise
                    const int ks = dh * C::kKSH + i;
                    const int row = key0 + (lane & 7) + ((lane >> 4) << 3);
                    const int col = ks * 16 + ((lane >> 3) & 1) * 8;
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4(kb + box_off<HD>(row, col), b0, b1, b2, b3);
                    mma16816(sc[0][i % C::kNCH], qa[i], b0, b1);
                    mma16816(sc[1][i % C::kNCH], qa[i], b2, b3);
                }
            } else {
#pragma unroll
                for (int i = 0; i < C::kKSH; i += 2) {
                    // matrices: keys +0..7 at d 16ks, +8, +16, +24 (two k-steps)
                    const int ks = dh * C::kKSH + i;
                    const int row = key0 + (lane & 7);
                    const int col = ks * 16 + (lane >> 3) * 8;
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4(kb + box_off<HD>(row, col), b0, b1, b2, b3);
                    mma16816(sc[0][i % C::kNCH], qa[i], b0, b1);
                    mma16816(sc[0][(i + 1) % C::kNCH], qa[i + 1], b2, b3);
                }
            }
#pragma unroll
            for (int n = 0; n < C::kNT; n++)
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    float s = 0.0f;
#pragma unroll
                    for (int c = 0; c < C::kNCH; c++) s += sc[n][c][j] + sc[n][c][j + 2];  // hi + lo rows
                    sp[(dh * 8 + g) * S + ((key0 + n * 8 + 2 * t + j) ^ (4 * g))] = s * kLog2e;
                }
        }
        compute_bar();
        if (*abort) return false;
        // -- online softmax of head g over this stage (every warp alike), in
        // base-2 units: the scores carry a factor log2(e)
        float pv[C::kPVK][4];
        float smax = -CUDART_INF_F;
#pragma unroll
        for (int kk = 0; kk < C::kPVK; kk++)
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int key = kk * 16 + 2 * t + (i & 1) + (i >> 1) * 8;
                const int kx = key ^ (4 * g);
                float s = sp[g * S + kx] + sp[(8 + g) * S + kx];
                if (partial && (r0 + key < it.row_lo || r0 + key >= it.row_hi)) s = -CUDART_INF_F;
                pv[kk][i] = s;
                smax = fmaxf(smax, s);
            }
        smax = fmaxf(smax, __shfl_xor_sync(0xffffffffu, smax, 1));
        smax = fmaxf(smax, __shfl_xor_sync(0xffffffffu, smax, 2));
        // A NaN or +inf score makes the sum NaN, which the output check reports.
        const float m_new = fmaxf(m_run, smax);
        const float alpha = m_new == -CUDART_INF_F ? 1.0f : ptx::ex2(m_run - m_new);
        float lsum = 0.0f;
        uint32_t bhi[C::kPVK][2], blo[C::kPVK][2];
#pragma unroll
        for (int kk = 0; kk < C::kPVK; kk++) {
            __half hi[4], lo[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float e = ptx::ex2(pv[kk][i] - m_new);  // ex2(-inf) = 0
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
        // -- O^T += V^T P^T for this warp's eighth of the head width
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
        for (int kk = 0; kk < C::kPVK; kk++)
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
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&sh.bars->empty[slot]);
    }
    // ---- O[h][d] for h = 2t, 2t+1 and d = dm + g (+8): final, or a partial
    const float l0 = __shfl_sync(0xffffffffu, l_run, 8 * t), l1 = __shfl_sync(0xffffffffu, l_run, 8 * t + 4);
    const bool final_out = tk.n_splits == 1;
    float *dst = final_out ? tk.out : p.part_o + (size_t)(tk.partial_base + it.split) * kHeads * 512;
    const float i0 = final_out ? 1.0f / l0 : 1.0f, i1 = final_out ? 1.0f / l1 : 1.0f;
#pragma unroll
    for (int mt = 0; mt < C::kMT; mt++) {
        const int dm = (warp * C::kMT + mt) * 16;
        dst[(2 * t) * HD + dm + g] = acc[mt][0] * i0;
        dst[(2 * t + 1) * HD + dm + g] = acc[mt][1] * i1;
        dst[(2 * t) * HD + dm + g + 8] = acc[mt][2] * i0;
        dst[(2 * t + 1) * HD + dm + g + 8] = acc[mt][3] * i1;
    }
    if (warp == 0 && t == 0) {
        if (final_out) {
            if (!(l_run > 0.0f) || !(l_run < CUDART_INF_F)) atomicOr(p.err_flag, 1);
        } else {
            const size_t slot_p = (size_t)(tk.partial_base + it.split);
            p.part_ml[slot_p * 2 * kHeads + g] = m_run;
            p.part_ml[slot_p * 2 * kHeads + kHeads + g] = l_run;
        }
    }
    return true;
}

__global__ void __launch_bounds__(kThreadsF16, 1) decode_f16_kernel(DecodeParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Shared sh;
    sh.stages = smem;
    sh.region = smem + kSlots * kStageBytes;
    sh.bars = reinterpret_cast<F16Bars *>(sh.region + kRegionBytes);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kSlots; i++) {
            ptx::mbar_init(&sh.bars->full[i], 1);
            ptx::mbar_init(&sh.bars->empty[i], kWarpsC);
        }
        ptx::mbar_init(&sh.bars->q_full, 1);
        ptx::mbar_init(&sh.bars->q_empty, kWarpsC);
        sh.bars->abort = 0;
        ptx::fence_mbar_init();
    }
    __syncthreads();
    release_dependents();  // the combine kernel may be scheduled; it waits for our end
    if (p.stall) {
        // g4a_debug_stall: a bounded wait on a bit of the error word that
        // nothing sets, before any load; the time-out is recorded as a
        // stalled ring wait would record it, and the CTA does no work
        if (threadIdx.x == 0 && !ptx::stall_wait(p.err_flag, 1 << 30, 2000000ull)) atomicOr(p.err_flag, 4);
        return;
    }
    const int i0 = p.cta_start[blockIdx.x], i1 = p.cta_start[blockIdx.x + 1];
    uint32_t st = 0;  // stage counter over this CTA's items
    if (warp == kWarpsC) {
        if (lane == 0) {
            uint32_t ic = 0;
            bool prereq_done = false;
            for (int i = i0; i < i1 && !sh.bars->abort; i++, ic++) {
                const DecodeItem it = p.items[i];
                const DecodeTask &tk = p.tasks[it.task];
                const bool ok = tk.hd == 256 ? produce_item<256>(p, it, tk, sh, st, ic, prereq_done)
                                             : produce_item<512>(p, it, tk, sh, st, ic, prereq_done);
                if (!ok) break;
            }
            if (!prereq_done) wait_prerequisite();
            // every issued load lands before the CTA may exit
            for (uint32_t s2 = (st > kSlots ? st - kSlots : 0); s2 < st; s2++)
                for (uint32_t i = 0; i < kPollLimit && !ptx::mbar_try_wait(&sh.bars->full[s2 % kSlots], (s2 / kSlots) & 1u);
                     i++) {
                }
            if (ic > 0)
                for (uint32_t i = 0; i < kPollLimit && !ptx::mbar_try_wait(&sh.bars->q_full, (ic - 1) & 1u); i++) {
                }
        }
        return;
    }
    uint32_t ic = 0;
    for (int i = i0; i < i1; i++, ic++) {
        const DecodeItem it = p.items[i];
        const DecodeTask &tk = p.tasks[it.task];
        const bool ok = tk.hd == 256 ? compute_item<256>(p, it, tk, sh, st, ic)
                                     : compute_item<512>(p, it, tk, sh, st, ic);
        if (!ok) return;
    }
}

// ---------------------------------------------------------------------------
// combine: out = sum_i w_i O_i / sum_i w_i l_i, w_i = exp(m_i - max_j m_j)
// ---------------------------------------------------------------------------

// max values of the partials are in base-2 units (scores times log2 e).
// One block per (task, head). Warp w takes the 128-column chunk w % C (C = hd
// / 128; lane = 4 columns) and the splits s = w / C, w / C + G, ... (G = 8 /
// C); it loads them as float4 in rounds of kCombineRound, the next round in
// flight while the current one is summed, and the G warp sums of a chunk meet
// in shared memory. The first round is loaded before the weights are known.
constexpr int kCombineChunk = 128;  // columns per warp
constexpr int kCombineRound = 6;    // float4 loads in flight per thread and round
__global__ void __launch_bounds__(256) decode_f16_combine(DecodeParams p) {
    wait_prerequisite();  // every partial of the main kernel is written
    const int task = p.split_tasks[blockIdx.x >> 3];
    const int h = blockIdx.x & 7;
    const DecodeTask &tk = p.tasks[task];
    const int ns = tk.n_splits, hd = tk.hd;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nc = hd / kCombineChunk, chunk = warp % nc, sg = warp / nc, G = 8 / nc;
    __shared__ float wsm[kF16MaxSplits + 1];
    __shared__ float4 red[8][32];
    const float *pml = p.part_ml + (size_t)tk.partial_base * 2 * kHeads;
    const float *pcol =
        p.part_o + (size_t)tk.partial_base * kHeads * 512 + (size_t)h * hd + chunk * kCombineChunk + 4 * lane;
    const int mine = ns > sg ? (ns - sg + G - 1) / G : 0;  // splits of this warp
    const int rounds = (mine + kCombineRound - 1) / kCombineRound;
    auto load = [&](float4 (&v)[kCombineRound], int r) {
#pragma unroll
        for (int k = 0; k < kCombineRound; k++) {
            const int i = r * kCombineRound + k;
            v[k] = i < mine ? __ldcg(reinterpret_cast<const float4 *>(pcol + (size_t)(sg + G * i) * kHeads * 512))
                            : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    };
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    auto accumulate = [&](const float4 (&v)[kCombineRound], int r) {
#pragma unroll
        for (int k = 0; k < kCombineRound; k++) {
            const int i = r * kCombineRound + k;
            if (i < mine) {
                const float w = wsm[sg + G * i];
                o.x = fmaf(v[k].x, w, o.x);
                o.y = fmaf(v[k].y, w, o.y);
                o.z = fmaf(v[k].z, w, o.z);
                o.w = fmaf(v[k].w, w, o.w);
            }
        }
    };
    float4 a[kCombineRound], b[kCombineRound];
    if (rounds > 0) load(a, 0);
    if (warp == 0) {
        float mv[3], lv[3];
        float M = -CUDART_INF_F;
#pragma unroll
        for (int k = 0; k < 3; k++) {  // ns <= 96
            const int s = lane + 32 * k;
            mv[k] = s < ns ? pml[(size_t)s * 2 * kHeads + h] : -CUDART_INF_F;
            lv[k] = s < ns ? pml[(size_t)s * 2 * kHeads + kHeads + h] : 0.0f;
            M = fmaxf(M, mv[k]);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
        float L = 0.0f;
#pragma unroll
        for (int k = 0; k < 3; k++) {
            const int s = lane + 32 * k;
            const float w = mv[k] == -CUDART_INF_F ? 0.0f : exp2f(mv[k] - M);
            if (s < ns) wsm[s] = w;
            L = fmaf(lv[k], w, L);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
        if (lane == 0) {
            wsm[ns] = 1.0f / L;
            if (!(L > 0.0f) || !(L < CUDART_INF_F)) atomicOr(p.err_flag, 1);
        }
    }
    __syncthreads();
    for (int r = 0; r < rounds; r += 2) {
        if (r + 1 < rounds) load(b, r + 1);
        accumulate(a, r);
        if (r + 2 < rounds) load(a, r + 2);
        if (r + 1 < rounds) accumulate(b, r + 1);
    }
    red[warp][lane] = o;
    __syncthreads();
    if (sg == 0) {
        float4 t = o;
        for (int g = 1; g < G; g++) {
            const float4 u = red[chunk + nc * g][lane];
            t.x += u.x;
            t.y += u.y;
            t.z += u.z;
            t.w += u.w;
        }
        const float inv = wsm[ns];
        float *dst = tk.out + (size_t)h * hd + chunk * kCombineChunk + 4 * lane;
        const float4 r = make_float4(t.x * inv, t.y * inv, t.z * inv, t.w * inv);
        if ((reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
            *reinterpret_cast<float4 *>(dst) = r;
        } else {
            dst[0] = r.x;
            dst[1] = r.y;
            dst[2] = r.z;
            dst[3] = r.w;
        }
    }
}

}  // namespace

cudaError_t launch_decode_f16(const DecodeParams &p, int stage, int n, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(decode_f16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
        attr = true;
    }
    if (stage == 0) {
        decode_f16_prep<<<n, kPrepThreads, 0, s>>>(p);
        return cudaGetLastError();
    }
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute pdl[1];
    pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = pdl;
    cfg.numAttrs = 1;
    cfg.stream = s;
    if (stage == 1) {
        cfg.gridDim = dim3(n);
        cfg.blockDim = dim3(kThreadsF16);
        cfg.dynamicSmemBytes = kSmemBytes;
        return cudaLaunchKernelEx(&cfg, decode_f16_kernel, p);
    }
    cfg.gridDim = dim3(n * kHeads);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = 0;
    return cudaLaunchKernelEx(&cfg, decode_f16_combine, p);
}

}  // namespace g4a
