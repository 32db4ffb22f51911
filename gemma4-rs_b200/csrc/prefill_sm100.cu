// Causal / sliding-window prefill attention on sm_100a tensor cores.
//
// Replaces the reference's token-at-a-time prompt processing, in which query
// position t runs crates/llm-gemma4/src/impl_/model.rs:326-366 (attend) over
// keys [max(0, t+1-window), t] (crates/llm-gemma4/src/eng/mod.rs:10-36), with
// one batched kernel over bf16 inputs and f32 accumulation.
//
// Tiling. A cluster of two CTAs (a "pair", one per SM) owns 32 query tokens x
// 8 heads = 256 rows and runs the CTA-pair form of tcgen05.mma (M = 256):
// each CTA holds 128 rows (16 tokens x 8 heads) of Q in its shared memory and
// of S and O in its TMEM, and each CTA loads only HALF of every K/V tile (its
// 64 of the tile's 128 keys for S = Q K^T, its 128 of the pair's 256 output
// columns for O += P V); the tensor cores of the pair exchange the B halves.
// All 8 heads of a row tile share the single KV head (grouped-query reuse, no
// multicast anywhere). Head width 512 runs two pairs per row tile, one per
// 256-wide half of the output, each recomputing S over the full width.
//
// Roles (352 threads per CTA):
//   warp 0      TMA producer: Q once, then K and V in stages of two or four
//               boxes (each 64 columns x 64 rows, 128-byte swizzle) under
//               one barrier, through a ring, in the fixed order K(0), K(1),
//               V(0), K(2), V(1), ... Both CTAs fill the same stage sequence;
//               every load signals the LEADER CTA's stage barrier, which
//               expects the pair's bytes. Few, large stages keep the barrier
//               waits of the MMA threads rare.
//   warp 1      allocates 512 TMEM columns (pair allocation); in the leader,
//               one thread issues S(j) = Q K(j)^T (bf16, f32 in TMEM,
//               double-buffered 2 x 128 columns).
//   warp 10     in the leader, one thread issues O += P(j) V(j) (P fp16 from
//               TMEM, V fp16 from shared memory, N = 256, f32 accumulator in
//               TMEM columns 0-255). Two issuing threads keep the tensor pipe
//               fed while either one waits on a barrier: a barrier wait in
//               the issuing thread stalls its MMA stream for about a hundred
//               cycles, as long as an M = 128, N = 128 MMA.
//   warps 2-9   softmax on the CTA's own rows: two threads per TMEM lane
//               (row), each over 64 of the tile's 128 scores; mask (edge
//               tiles only), row max agreed through a shared-memory mailbox,
//               one FFMA + EX2 per score, P written back into the S columns
//               as fp16, then an arrive on the leader's P barrier; the
//               running max is rescaled lazily (only when it grows by more
//               than 2^15); the epilogue divides by the row sum and stores
//               f32, each thread 128 of the 256 output columns.
// Every mbarrier wait is bounded; on time-out the CTA records an error flag,
// drains what it can, frees TMEM and exits (after the pair's final cluster
// barrier, so that no MMA still reads its shared memory).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <math_constants.h>

#include <algorithm>
#include <climits>
#include <cstdlib>
#include <cstring>
#include <unordered_map>
#include <vector>

#include "../../include/g4attn.h"
#include "internal.h"
#include "sm100_ptx.cuh"

namespace g4a {
namespace {

constexpr int kRows = 128;            // rows per CTA: 16 tokens x 8 heads
constexpr int kTokensPerCta = 16;
constexpr int kTokensPerPair = 32;
constexpr int kKeysPerTile = 128;     // N of S for the pair
constexpr int kDV = 256;              // output columns per pair
constexpr int kQBoxBytes = 128 * 128; // 64 bf16 columns x 128 rows
constexpr int kBoxBytes = 64 * 128;   // 64 columns x 64 rows (bf16 / fp16)
constexpr int kOutBoxBytes = 128 * 128;  // 32 f32 columns x 128 rows
constexpr int kThreads = 352;
constexpr int kPvWarp = 10;
constexpr int kSoftmaxWarps = 8;     // warps 2-9
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 0, kColS0 = 256, kColS1 = 384;
constexpr uint32_t kWaitLimit = 1u << 22;  // polls; far above any legitimate wait
constexpr uint16_t kBothCtas = 0x3;

struct alignas(64) ProblemDev {
    CUtensorMap tq, tk, tv;  // Q [n_q*8, hd] bf16 (128-row boxes), K [n_kv, hd] bf16, V [n_kv, hd] fp16 (64-row boxes)
    CUtensorMap to;          // out [n_q*8, hd] f32, 32-column x 128-row boxes, 128-byte swizzle
    CUtensorMap tk32;        // K with 32-row boxes (the persistent kernel's 64-key tiles at width 512)
    int32_t hd, window, n_q, q_pos0, n_kv, kv_pos0;
    float *out;
    float *lse;
};

struct WorkItem {
    int32_t problem, q_tile, dv_half, kv_tile_lo, n_kv_tiles, pad;  // q_tile: 32-token tile of the pair
};

template <int HD>
struct Cfg {
    static constexpr int kQBoxes = HD / 64;    // Q boxes per CTA
    // A stage is kStageBoxes boxes under one barrier: K(j) is HD/64 boxes
    // (64 keys x 64 columns each), V(j) four (2 key halves x 2 column atoms,
    // atoms adjacent). Width 512 keeps 16 KB stages (Q takes 128 KB of shared
    // memory), width 256 takes 32 KB stages: one wait each for K(j) and V(j).
    static constexpr int kStageBoxes = HD == 256 ? 4 : 2;
    static constexpr int kStageBytes = kStageBoxes * kBoxBytes;
    static constexpr int kKStages = HD / 64 / kStageBoxes;
    static constexpr int kVStages = 4 / kStageBoxes;
    static constexpr int kRing = HD == 256 ? 4 : 5;  // stages
    static constexpr int kSmemQ = kQBoxes * kQBoxBytes;
    static constexpr int kSmemRing = kRing * kStageBytes;
    static constexpr int kSmemBytes = kSmemQ + kSmemRing + 5120 /*barriers, mailboxes*/ + 1024 /*alignment slack*/;
    static_assert(kSmemBytes <= 227 * 1024, "shared memory");
    static_assert(kSmemQ + kSmemRing >= 8 * kOutBoxBytes, "output staging reuses the Q and K/V stages");
    // Position of the first stage of K(j) / V(j) in the push sequence
    // K(0), K(1), V(0), K(2), V(1), ..., K(n-1), V(n-2), V(n-1).
    __device__ static int k_pos(int j) { return j == 0 ? 0 : kKStages + (j - 1) * (kKStages + kVStages); }
    __device__ static int v_pos(int j, int n) {
        return kKStages + j * (kKStages + kVStages) + (j + 1 < n ? kKStages : 0);
    }
};

struct alignas(8) Mailbox {
    int seq;  // tile index the value belongs to
    float v;
};

struct Barriers {
    Mailbox box[2][2][128];  // [seq parity][column half][row]
    uint64_t q_full;         // leader: both CTAs' Q bytes
    uint64_t s_full[2];      // both: S buffer ready (pair commit)
    uint64_t p_full[2];      // leader: one arrival per softmax warp of each CTA
    uint64_t o_done[2];      // both: PV of the tile in this S buffer done (pair commit): O
                             // updated, P buffer free. A wait by phase parity is exact
                             // only while its barrier is at most one phase behind the
                             // awaited one; a barrier per S buffer keeps that true.
    uint64_t mma_done;       // both: every MMA of the pair done (one commit per issuer)
    uint64_t ring_full[8];   // leader: both CTAs' bytes of the stage
    uint64_t ring_empty[8];  // both: stage consumed (pair commit)
    uint32_t tmem_base;
    int abort;
    int k_seen;              // leader: tiles whose K stages the S issuer has seen land
};

static_assert(sizeof(Barriers) <= 5120, "barrier region");

// Bounded wait: false if another role aborted or the limit ran out (which
// aborts the CTA and records bit 1 of the error flag).
template <bool kCluster = false>
__device__ __forceinline__ bool wait_bar(uint64_t *bar, uint32_t parity, volatile int *abort, int *err) {
    for (uint32_t i = 0; i < kWaitLimit; i++) {
        if (kCluster ? ptx::mbar_try_wait_cluster(bar, parity) : ptx::mbar_try_wait(bar, parity)) return true;
        if ((i & 1023) == 1023 && *abort) return false;
    }
    *abort = 1;
    atomicOr(err, 2);
    return false;
}

// One work item on one CTA pair (both CTAs call this with the same item).
// g4a_debug_stall: both CTAs of every pair skip the item after the leader's
// bounded wait on a bit of the error word that nothing sets (no barrier,
// TMEM or load touched yet), recording the time-out as a stalled wait would.
__device__ __forceinline__ void stall_item(int *err) {
    if (threadIdx.x == 0 && ptx::cluster_ctarank() == 0 && !ptx::stall_wait(err, 1 << 30, 2000000ull))
        atomicOr(err, 2);
}

// 2^x on the FMA pipe, for part of the softmax's exponentials (the MUFU pipe
// takes 16 per clock per SM, the FMA pipe 128 operations): x = n + f with n
// rounded to the nearest integer by the 1.5 * 2^23 addition trick and f in
// [-0.5, 0.5]; 2^f by a cubic whose coefficients were fitted for this kernel
// (minimax of the relative error, 7.5e-5, below the fp16 rounding of P);
// 2^n added to the exponent bits. Below -125 the result is 0, as the
// hardware's flushed ex2 gives for masked (-inf) scores.
__device__ __forceinline__ float ex2_fma(float x) {
    const float xc = fmaxf(x, -125.0f);
    const float t = xc + 12582912.0f;
    const int n = __float_as_int(t) - 0x4B400000;
    const float f = xc - (t - 12582912.0f);
    const float p = fmaf(fmaf(fmaf(0.05517149f, f, 0.24261093f), f, 0.69326097f), f, 0.99992806f);
    const float r = __int_as_float(__float_as_int(p) + (n << 23));
    return x < -125.0f ? 0.0f : r;
}

// ex2_fma on a pair, with packed fp32 arithmetic: the same operations in the
// same order (each lane rounds as the scalar form), except that x below -125
// is clamped there, giving 2^-125 * p(f) instead of 0. That value rounds to 0
// in fp16 P, and its share of a row sum (which is at least 1 once a key is
// visible) is below 1e-36; a row that sees no key keeps its -inf maximum, so
// its output stays 0 and its lse -inf.
__device__ __forceinline__ float2 ex2_fma2(float2 x) {
    const float2 xc = make_float2(fmaxf(x.x, -125.0f), fmaxf(x.y, -125.0f));
    const float2 magic = make_float2(12582912.0f, 12582912.0f);
    const float2 t = ptx::add2(xc, magic);
    const float2 f = ptx::sub2(xc, ptx::sub2(t, magic));
    float2 p = ptx::fma2(make_float2(0.05517149f, 0.05517149f), f, make_float2(0.24261093f, 0.24261093f));
    p = ptx::fma2(p, f, make_float2(0.69326097f, 0.69326097f));
    p = ptx::fma2(p, f, make_float2(0.99992806f, 0.99992806f));
    // t's low mantissa bits hold n + 2^22 and 0x4B400000 << 23 wraps to 0, so
    // (t bits << 23) adds n to p's exponent
    return make_float2(__int_as_float(__float_as_int(p.x) + (__float_as_int(t.x) << 23)),
                       __int_as_float(__float_as_int(p.y) + (__float_as_int(t.y) << 23)));
}

// Maximum of N values by three-input max instructions (depth log3 N).
template <int N> __device__ __forceinline__ float max_tree(const float (&v)[N]) {
    if constexpr (N == 1) {
        return v[0];
    } else if constexpr (N == 2) {
        return fmaxf(v[0], v[1]);
    } else {
        constexpr int M = N / 3, R = N - 3 * M;
        float t[M + R];
#pragma unroll
        for (int c = 0; c < M; c++) t[c] = ptx::max3(v[3 * c], v[3 * c + 1], v[3 * c + 2]);
#pragma unroll
        for (int c = 0; c < R; c++) t[M + c] = v[3 * M + c];
        return max_tree<M + R>(t);
    }
}

// Bounded wait until a progress counter of another issuing thread of this
// CTA reaches `target` (false on abort or time-out, as wait_bar).
__device__ __forceinline__ bool wait_count(const int *counter, int target, volatile int *abort, int *err) {
    const uint32_t a = ptx::smem_u32(counter);
    for (uint32_t i = 0; i < kWaitLimit; i++) {
        int v;
        asm volatile("ld.volatile.shared.b32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
        if (v >= target) {
            __threadfence_block();
            return true;
        }
        if ((i & 1023) == 1023 && *abort) return false;
    }
    *abort = 1;
    atomicOr(err, 2);
    return false;
}
__device__ __forceinline__ void set_count(int *counter, int v) {
    asm volatile("st.volatile.shared.b32 [%0], %1;" ::"r"(ptx::smem_u32(counter)), "r"(v) : "memory");
}

template <int HD>
__device__ __forceinline__ void prefill_item(const ProblemDev *__restrict__ problems, const WorkItem it, int *err) {
    using C = Cfg<HD>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *q_smem = smem;
    uint8_t *ring = smem + C::kSmemQ;
    Barriers *bars = reinterpret_cast<Barriers *>(ring + C::kSmemRing);
    volatile int *abort = &bars->abort;

    const uint32_t rank = ptx::cluster_ctarank();  // 0 = leader
    const ProblemDev &pb = problems[it.problem];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_tiles = it.n_kv_tiles;

    if (threadIdx.x == 0) {
        ptx::mbar_init(&bars->q_full, 1);
        for (int i = 0; i < 2; i++) {
            ptx::mbar_init(&bars->s_full[i], 1);
            ptx::mbar_init(&bars->p_full[i], 2 * kSoftmaxWarps);
            ptx::mbar_init(&bars->o_done[i], 1);
        }
        ptx::mbar_init(&bars->mma_done, 2);
        for (int i = 0; i < C::kRing; i++) {
            ptx::mbar_init(&bars->ring_full[i], 1);
            ptx::mbar_init(&bars->ring_empty[i], 1);
        }
        bars->abort = 0;
        bars->k_seen = 0;
        ptx::fence_mbar_init();
    }
    for (int i = threadIdx.x; i < 2 * 2 * kRows; i += blockDim.x)
        bars->box[i / (2 * kRows)][(i / kRows) & 1][i % kRows] = Mailbox{-1, 0.0f};
    if (warp == 1) {
        ptx::tmem_alloc2(&bars->tmem_base, kTmemCols);
        ptx::tmem_relinquish2();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::cluster_sync();  // barrier inits of both CTAs visible before any remote signal
    ptx::tc_fence_after();
    const uint32_t tmem = bars->tmem_base;

    // slot / phase of push-sequence position pos
    auto slot_of = [](int pos) { return pos % C::kRing; };
    auto phase_of = [](int pos) { return (uint32_t)(pos / C::kRing) & 1u; };

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0 && n_tiles > 0) {
            ptx::prefetch_tmap(&pb.tq);
            ptx::prefetch_tmap(&pb.tk);
            ptx::prefetch_tmap(&pb.tv);
            ptx::prefetch_tmap(&pb.to);
            if (rank == 0) ptx::mbar_arrive_expect_tx(&bars->q_full, 2 * C::kSmemQ);
            const uint32_t q_full_l = ptx::mapa(&bars->q_full, 0);
            for (int c = 0; c < C::kQBoxes; c++)
                ptx::tma_load_2d_pair(q_smem + c * kQBoxBytes, &pb.tq, q_full_l, 64 * c,
                                      it.q_tile * 2 * kRows + (int)rank * kRows);
            int slot = 0;
            uint32_t phase = 0;
            uint32_t issued = 0;  // bit s: slot s received at least one load
            bool ok = true;
            // one stage: box b at (xs[b], ys[b])
            auto push = [&](const CUtensorMap *m, const int *xs, const int *ys) {
                if (!ok) return;
                if (!wait_bar(&bars->ring_empty[slot], phase ^ 1u, abort, err)) {
                    ok = false;
                    return;
                }
                if (rank == 0) ptx::mbar_arrive_expect_tx(&bars->ring_full[slot], 2 * C::kStageBytes);
                const uint32_t bar_l = ptx::mapa(&bars->ring_full[slot], 0);
                for (int b = 0; b < C::kStageBoxes; b++)
                    ptx::tma_load_2d_pair(ring + slot * C::kStageBytes + b * kBoxBytes, m, bar_l, xs[b], ys[b]);
                issued |= 1u << slot;
                if (++slot == C::kRing) {
                    slot = 0;
                    phase ^= 1u;
                }
            };
            // K: this CTA's 64 keys of the tile, all HD columns
            auto push_k = [&](int j) {
                const int y = (it.kv_tile_lo + j) * kKeysPerTile + 64 * (int)rank;
                for (int st = 0; st < C::kKStages; st++) {
                    int xs[C::kStageBoxes], ys[C::kStageBoxes];
                    for (int b = 0; b < C::kStageBoxes; b++) {
                        xs[b] = 64 * (st * C::kStageBoxes + b);
                        ys[b] = y;
                    }
                    push(&pb.tk, xs, ys);
                }
            };
            // V: this CTA's 128 output columns (two 64-column atoms) of both
            // 64-key halves; box q = 2 * key half + atom
            auto push_v = [&](int j) {
                const int x = it.dv_half * kDV + 128 * (int)rank;
                const int y = (it.kv_tile_lo + j) * kKeysPerTile;
                for (int st = 0; st < C::kVStages; st++) {
                    int xs[C::kStageBoxes], ys[C::kStageBoxes];
                    for (int b = 0; b < C::kStageBoxes; b++) {
                        const int q = st * C::kStageBoxes + b;
                        xs[b] = x + 64 * (q & 1);
                        ys[b] = y + 64 * (q >> 1);
                    }
                    push(&pb.tv, xs, ys);
                }
            };
            push_k(0);
            for (int j = 0; j < n_tiles && ok; j++) {
                if (j + 1 < n_tiles) push_k(j + 1);
                push_v(j);
            }
            // Drain (leader): every load of both CTAs signals the leader's
            // barriers; no TMA write may land after the pair exits. Normally
            // the MMA threads already waited for every load; after an abort,
            // wait here (bounded) for Q and for each slot's latest load.
            if (rank == 0) {
                for (uint32_t i = 0; i < kWaitLimit && !ptx::mbar_try_wait(&bars->q_full, 0); i++) {
                }
                if (!ok || *abort) {
                    for (int s = 0; s < C::kRing; s++) {
                        if (!(issued >> s & 1u)) continue;
                        const uint32_t ph = s < slot ? phase : phase ^ 1u;
                        for (uint32_t i = 0; i < kWaitLimit && !ptx::mbar_try_wait(&bars->ring_full[s], ph); i++) {
                        }
                    }
                }
            }
            // Non-leader after an abort: its loads signal the leader's barriers,
            // which the leader may not have armed for a stage it never reached,
            // so their completion cannot be observed from here; the CTA lets
            // 200 us of the global timer pass (far above any load's latency)
            // before it may exit.
            if (rank != 0 && (!ok || *abort)) {
                const uint64_t t0 = ptx::globaltimer_ns();
                while (ptx::globaltimer_ns() - t0 < 200000ull) __nanosleep(2000);
            }
        }
    } else if (warp == 1 || warp == kPvWarp) {
        // ------------------------------------------------------------ MMA issuers (leader)
        // Base descriptors: the address field holds (address >> 4) in its low
        // 14 bits and every operand lies below 256 KB of shared memory, so a
        // byte offset is added as (offset >> 4) without a carry out of it.
        const uint64_t q_desc = ptx::smem_desc(ptx::smem_u32(q_smem), 16, 1024);
        const uint64_t k_desc = ptx::smem_desc(ptx::smem_u32(ring), 16, 1024);
        const uint64_t v_desc = ptx::smem_desc(ptx::smem_u32(ring), kBoxBytes, 1024);
        if (lane == 0 && rank == 0) {
            bool ok = n_tiles > 0 && wait_bar(&bars->q_full, 0, abort, err);
            if (warp == 1) {
                // S(j) = Q K(j)^T into S buffer j&1, once PV(j-2) has read P(j-2) from it
                constexpr uint32_t kIdescS = ptx::idesc_f16(1, 1, 0, 2 * kRows, kKeysPerTile);
                for (int j = 0; j < n_tiles && ok; j++) {
                    if (j >= 2 && !wait_bar(&bars->o_done[j & 1], (uint32_t)((j - 2) >> 1) & 1u, abort, err)) {
                        ok = false;
                        break;
                    }
                    ptx::tc_fence_after();
                    const uint32_t d = tmem + ((j & 1) ? kColS1 : kColS0);
                    const int pos = C::k_pos(j);
                    for (int st = 0; st < C::kKStages && ok; st++) {
                        const int slot = slot_of(pos + st);
                        if (!wait_bar(&bars->ring_full[slot], phase_of(pos + st), abort, err)) {
                            ok = false;
                            break;
                        }
                        ptx::tc_fence_after();
#pragma unroll
                        for (int b = 0; b < C::kStageBoxes; b++) {
                            const uint64_t kd = k_desc + (uint64_t)((slot * C::kStageBytes + b * kBoxBytes) >> 4);
                            const uint64_t qd = q_desc + (uint64_t)((C::kStageBoxes * st + b) * (kQBoxBytes >> 4));
                            ptx::mma2_ss(d, qd, kd, kIdescS, (st | b) != 0);
#pragma unroll
                            for (int kk = 1; kk < 4; kk++) ptx::mma2_ss(d, qd + 2 * kk, kd + 2 * kk, kIdescS, 1);
                        }
                        ptx::mma2_commit_pair(&bars->ring_empty[slot], kBothCtas);
                    }
                    set_count(&bars->k_seen, j + 1);
                    if (ok) ptx::mma2_commit_pair(&bars->s_full[j & 1], kBothCtas);
                }
            } else {
                // O += P(j) V(j) once the softmax of both CTAs published P(j)
                constexpr uint32_t kIdescPV = ptx::idesc_f16(0, 0, 1, 2 * kRows, kDV);
                for (int j = 0; j < n_tiles && ok; j++) {
                    if (!wait_bar<true>(&bars->p_full[j & 1], (uint32_t)(j >> 1) & 1u, abort, err)) {
                        ok = false;
                        break;
                    }
                    // Width 512 (5-stage ring, 4 K stages per tile): V(j)'s second
                    // slot last held K(j+1)'s first stage. A parity wait on that
                    // slot is exact only once that earlier fill has landed, which
                    // the S issuer has seen when it has waited for K(j+1).
                    if (HD == 512 && j + 1 < n_tiles && !wait_count(&bars->k_seen, j + 2, abort, err)) {
                        ok = false;
                        break;
                    }
                    const int pos = C::v_pos(j, n_tiles);
                    for (int c = 0; c < C::kVStages && ok; c++)
                        ok = wait_bar(&bars->ring_full[slot_of(pos + c)], phase_of(pos + c), abort, err);
                    if (!ok) break;
                    ptx::tc_fence_after();
                    const uint32_t p_tmem = tmem + ((j & 1) ? kColS1 : kColS0);
                    // keys 16ks.. live in V half h = ks/4: box 2h of the V sequence (the
                    // next box holds its second column atom)
                    const uint64_t vd0 = v_desc + (uint64_t)((slot_of(pos) * C::kStageBytes) >> 4);
                    const uint64_t vd1 =
                        v_desc + (uint64_t)((slot_of(pos + 2 / C::kStageBoxes) * C::kStageBytes +
                                             (2 % C::kStageBoxes) * kBoxBytes) >> 4);
                    ptx::mma2_ts(tmem + kColO, p_tmem, vd0, kIdescPV, j > 0);
#pragma unroll
                    for (int ks = 1; ks < kKeysPerTile / 16; ks++)
                        ptx::mma2_ts(tmem + kColO, p_tmem + 8 * ks, (ks < 4 ? vd0 : vd1) + (2048 >> 4) * (ks & 3),
                                     kIdescPV, 1);
                    for (int c = 0; c < C::kVStages; c++)
                        ptx::mma2_commit_pair(&bars->ring_empty[slot_of(pos + c)], kBothCtas);
                    ptx::mma2_commit_pair(&bars->o_done[j & 1], kBothCtas);
                }
            }
            // Every MMA this thread issued completes before either CTA
            // releases TMEM or exits (mma_done expects one commit per issuer).
            ptx::mma2_commit_pair(&bars->mma_done, kBothCtas);
            for (uint32_t i = 0; i < kWaitLimit && !ptx::mbar_try_wait(&bars->mma_done, 0); i++) {
            }
        } else if (warp == 1 && lane == 0 && n_tiles > 0) {
            // non-leader: wait (bounded) for the leader's final commits
            for (uint32_t i = 0; i < kWaitLimit && !ptx::mbar_try_wait(&bars->mma_done, 0); i++) {
                if ((i & 1023) == 1023 && *abort) break;
            }
        }
    } else {
        // ------------------------------------------------------------ softmax + epilogue
        // Two warpgroups: warp w reaches TMEM lanes 32*(w%4).., so warps w and
        // w+4 share a quadrant of rows and split each row's 128 scores (and
        // its 256 output columns) in halves. They agree on the row max
        // through a per-row shared-memory mailbox (no named barrier, so that
        // either side can give up alone after a bounded wait).
        const int quad = warp & 3;                  // TMEM lane quadrant this warp may access
        const int half = (warp - 2) >> 2;           // column half of S and of O
        const int row = quad * 32 + lane;           // tile row = TMEM lane
        const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
        const int tok0 = it.q_tile * kTokensPerPair + (int)rank * kTokensPerCta;  // this CTA's first token
        const int tok = tok0 + row / 8;
        const int head = row % 8;
        const bool row_valid = tok < pb.n_q;
        const int qpos = pb.q_pos0 + tok;
        // visible key indices of this row: [vis_lo, vis_hi]
        const int vis_hi = min(qpos - pb.kv_pos0, pb.n_kv - 1);
        const int vis_lo = pb.window > 0 ? qpos - pb.window + 1 - pb.kv_pos0 : INT_MIN / 2;
        // this CTA's first and last query positions (rows past n_q included)
        const int q_first = pb.q_pos0 + tok0;
        const int q_last = q_first + kTokensPerCta - 1;
        const float kLog2e = 1.4426950408889634f;
        const uint32_t p_full_l0 = ptx::mapa(&bars->p_full[0], 0), p_full_l1 = ptx::mapa(&bars->p_full[1], 0);
        float m_used = -CUDART_INF_F;  // running reference max, log2 units
        float l = 0.0f;                // this half's row sum
        bool ok = true;
        Mailbox *my_box = &bars->box[0][half][row];
        Mailbox *other_box = &bars->box[0][half ^ 1][row];
        // Post (seq, v) and read the partner's value for the same seq.
        auto swap = [&](int seq, float v, float *out) -> bool {
            const int par = seq & 1;
            const uint32_t mine = ptx::smem_u32(my_box + par * 2 * kRows);
            const uint32_t theirs = ptx::smem_u32(other_box + par * 2 * kRows);
            // one 8-byte scalar store: the partner sees seq and value together
            const uint64_t word = (uint64_t)(uint32_t)seq | ((uint64_t)__float_as_uint(v) << 32);
            asm volatile("st.volatile.shared.b64 [%0], %1;" ::"r"(mine), "l"(word) : "memory");
            for (uint32_t i = 0; i < kWaitLimit; i++) {
                uint64_t t;
                asm volatile("ld.volatile.shared.b64 %0, [%1];" : "=l"(t) : "r"(theirs) : "memory");
                if ((int)(uint32_t)t == seq) {
                    *out = __uint_as_float((uint32_t)(t >> 32));
                    return true;
                }
                if ((i & 255) == 255 && *abort) return false;
            }
            *abort = 1;
            atomicOr(err, 2);
            return false;
        };
        // tcgen05.ld/st are warp-collective (.sync.aligned): every branch that
        // contains one is decided by a warp vote, never per row.
        for (int j = 0; j < n_tiles && ok; j++) {
            if (!__all_sync(0xffffffffu, wait_bar(&bars->s_full[j & 1], (uint32_t)(j >> 1) & 1u, abort, err))) {
                ok = false;
                break;
            }
            ptx::tc_fence_after();
            const uint32_t s_addr = tmem + lane_addr + ((j & 1) ? kColS1 : kColS0);
            uint32_t r0[32], r1[32];
            ptx::tmem_ld32(s_addr + 64 * half, r0);
            ptx::tmem_ld32(s_addr + 64 * half + 32, r1);
            ptx::tmem_wait_ld();
            ptx::tmem_ld_fence(r0);
            ptx::tmem_ld_fence(r1);
            float s[64];
#pragma unroll
            for (int i = 0; i < 32; i++) {
                s[i] = __uint_as_float(r0[i]);
                s[32 + i] = __uint_as_float(r1[i]);
            }
            const int k0 = (it.kv_tile_lo + j) * kKeysPerTile;  // first key index of the tile
            // Masking only where some key of the tile is invisible to some row of this CTA.
            const int kp0 = pb.kv_pos0 + k0;
            const bool edge = k0 + kKeysPerTile > pb.n_kv || kp0 + kKeysPerTile - 1 > q_first ||
                              (pb.window > 0 && q_last - kp0 >= pb.window);
            if (edge) {
                const int kb = k0 + 64 * half;
                const int lo = vis_lo - kb, hi = vis_hi - kb;  // visible i in [lo, hi]
#pragma unroll
                for (int i = 0; i < 64; i++) s[i] = (i >= lo && i <= hi) ? s[i] : -CUDART_INF_F;
            }
            // row max as a tree (depth 6, not a chain of 63)
            float mt[32];
#pragma unroll
            for (int c = 0; c < 32; c++) mt[c] = fmaxf(s[c], s[c + 32]);
#pragma unroll
            for (int w = 16; w >= 1; w >>= 1)
#pragma unroll
                for (int c = 0; c < w; c++) mt[c] = fmaxf(mt[c], mt[c + w]);
            float mx = mt[0];
            float mo;
            if (!__all_sync(0xffffffffu, swap(j, mx, &mo))) {
                ok = false;
                break;
            }
            mx = fmaxf(mx, mo) * kLog2e;
            // Lazy rescale: move this row's reference max only when the tile
            // max exceeds it by more than 15 (log2 units), so that P stays at
            // or below 2^15 and fits fp16 (max 65504). With scores of unit-RMS
            // rows spread over tens of bits, a smaller margin would rescale O
            // on most tiles; this one rarely does.
            const bool grow = mx > m_used + 15.0f;
            const bool o_live = grow && m_used != -CUDART_INF_F;  // O holds weights of the old max
            const float f = o_live ? ptx::ex2(m_used - mx) : 1.0f;
            if (grow) m_used = mx;
            // p = 2^(s*log2e - m); masked scores are -inf and give 0. A row
            // with no visible key so far keeps m = -inf; subtract 0 then.
            const float neg_m = m_used == -CUDART_INF_F ? 0.0f : -m_used;
            uint32_t pk[32];
            // row sum in 8 partial sums, then a tree
            float rs[8];
#pragma unroll
            for (int k = 0; k < 8; k++) rs[k] = 0.0f;
#pragma unroll
            for (int i = 0; i < 32; i++) {
                // half of the exponentials on the MUFU pipe, half on the FMA pipe
                const float x0 = fmaf(s[2 * i], kLog2e, neg_m), x1 = fmaf(s[2 * i + 1], kLog2e, neg_m);
                const float p0 = (i & 1) ? ex2_fma(x0) : ptx::ex2(x0);
                const float p1 = (i & 1) ? ex2_fma(x1) : ptx::ex2(x1);
                rs[(2 * i) & 7] += p0;
                rs[(2 * i + 1) & 7] += p1;
                pk[i] = ptx::pack_half2(p0, p1);
            }
            l = l * f + (((rs[0] + rs[1]) + (rs[2] + rs[3])) + ((rs[4] + rs[5]) + (rs[6] + rs[7])));
            // P (fp16 pairs) goes over the first 64 columns of this S buffer;
            // half 1's columns 32-63 were read by half 0 before it posted its
            // max, which half 1 has seen.
            ptx::tmem_st32(s_addr + 32 * half, pk);
            // O rescale after P is out of the registers: the wait for PV(j-1)
            // then overlaps the exponentials above. PV(j) reads neither O's
            // new scale nor P(j) before the arrive below.
            if (__any_sync(0xffffffffu, o_live)) {
                if (!__all_sync(0xffffffffu,
                                wait_bar(&bars->o_done[(j - 1) & 1], (uint32_t)((j - 1) >> 1) & 1u, abort, err))) {
                    ok = false;
                    break;
                }
                ptx::tc_fence_after();
                // this thread's 128 columns of O, 64 at a time
#pragma unroll 1
                for (int c = 0; c < kDV / 128; c++) {
                    uint32_t r0[32], r1[32];
                    const uint32_t o_addr = tmem + lane_addr + kColO + 128 * half + 64 * c;
                    ptx::tmem_ld32(o_addr, r0);
                    ptx::tmem_ld32(o_addr + 32, r1);
                    ptx::tmem_wait_ld();
                    ptx::tmem_ld_fence(r0);
                    ptx::tmem_ld_fence(r1);
#pragma unroll
                    for (int i = 0; i < 32; i++) {
                        r0[i] = __float_as_uint(__uint_as_float(r0[i]) * f);
                        r1[i] = __float_as_uint(__uint_as_float(r1[i]) * f);
                    }
                    ptx::tmem_st32(o_addr, r0);
                    ptx::tmem_st32(o_addr + 32, r1);
                }
            }
            ptx::tmem_wait_st();
            ptx::tc_fence_before();
            // one arrival per warp on the leader's barrier (release, cluster scope)
            // once every lane's P is in TMEM
            __syncwarp();
            if (lane == 0) {  // the leader's own warps arrive locally (CTA-scope release)
                if (rank == 0) ptx::mbar_arrive(&bars->p_full[j & 1]);
                else ptx::mbar_arrive_cl((j & 1) ? p_full_l1 : p_full_l0);
            }
        }
        // ---- epilogue: O / l, staged in shared memory, written by TMA ----
        float lo_ = 0.0f;
        if (ok && !__all_sync(0xffffffffu, swap(n_tiles, l, &lo_))) ok = false;
        l += lo_;
        if (ok && n_tiles > 0 &&
            !__all_sync(0xffffffffu,
                        wait_bar(&bars->o_done[(n_tiles - 1) & 1], (uint32_t)((n_tiles - 1) >> 1) & 1u, abort, err)))
            ok = false;
        ptx::tc_fence_after();
        // The CTA's Q and K/V stages are idle by now (every load was consumed,
        // every MMA reading them completed), so O / l is staged there as eight
        // 32-column x 128-row f32 boxes in the 128-byte-swizzled layout (16-byte
        // chunk j of row r at chunk j ^ (r % 8)) and written by TMA stores: full
        // lines to L2 instead of 16-byte pieces of 128 different rows.
        uint8_t *stage = smem;
        if (ok) {
            const float inv = l > 0.0f ? 1.0f / l : 0.0f;
#pragma unroll 1
            for (int c = 0; c < kDV / 64; c++) {
                uint32_t r[32];
                if (n_tiles > 0) {
                    ptx::tmem_ld32(tmem + lane_addr + kColO + 128 * half + 32 * c, r);
                    ptx::tmem_wait_ld();
                    ptx::tmem_ld_fence(r);
                } else {
#pragma unroll
                    for (int i = 0; i < 32; i++) r[i] = 0u;
                }
                uint8_t *row_p = stage + (4 * half + c) * kOutBoxBytes + row * 128;
#pragma unroll
                for (int jj = 0; jj < 8; jj++) {
                    const float4 v = make_float4(__uint_as_float(r[4 * jj]) * inv, __uint_as_float(r[4 * jj + 1]) * inv,
                                                 __uint_as_float(r[4 * jj + 2]) * inv,
                                                 __uint_as_float(r[4 * jj + 3]) * inv);
                    *reinterpret_cast<float4 *>(row_p + ((jj ^ (row & 7)) << 4)) = v;
                }
            }
            if (row_valid && pb.lse && it.dv_half == 0 && half == 0)
                pb.lse[(size_t)tok * 8 + head] = l > 0.0f ? (m_used + log2f(l)) * 0.6931471805599453f : -CUDART_INF_F;
        }
        ptx::fence_proxy_async_smem();
        // All eight softmax warps reach this barrier on every path (an aborted
        // warp only skips its staging writes above).
        ptx::named_bar_sync(1, 256);
        if (threadIdx.x == 64 && !*abort && tok0 < pb.n_q) {
            // rows past n_q * 8 are clipped by the tensor map; a box starting past them is not issued
            for (int k = 0; k < 8; k++)
                ptx::tma_store_2d(&pb.to, stage + k * kOutBoxBytes, it.dv_half * kDV + 32 * k, tok0 * 8);
            ptx::bulk_commit_group();
            ptx::bulk_wait_read_all();
        }
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::cluster_sync();  // no MMA or load of the pair still touches either CTA
    if (warp == 1) {
        __syncwarp();
        ptx::tc_fence_after();
        ptx::tmem_dealloc2(tmem, kTmemCols);
    }
}

template <int HD>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    prefill_kernel(const ProblemDev *__restrict__ problems, const WorkItem *__restrict__ items, int *err, int stall) {
    if (stall) return stall_item(err);
    prefill_item<HD>(problems, items[blockIdx.x >> 1], err);
}

// Items of both head widths in one grid (a prompt's sliding and global layers
// together), taken longest first: the width is the item's problem's.
constexpr int kSmemMixed = Cfg<256>::kSmemBytes > Cfg<512>::kSmemBytes ? Cfg<256>::kSmemBytes : Cfg<512>::kSmemBytes;
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    prefill_kernel_mixed(const ProblemDev *__restrict__ problems, const WorkItem *__restrict__ items, int *err,
                         int stall) {
    if (stall) return stall_item(err);
    const WorkItem it = items[blockIdx.x >> 1];
    if (problems[it.problem].hd == 256) prefill_item<256>(problems, it, err);
    else prefill_item<512>(problems, it, err);
}

// ---------------------------------------------------------------------------
// Persistent form: one CTA pair per two SMs runs a host-assigned list of work
// items (longest-processing-time first), its pipeline running on from item to
// item. Roles as above, plus four epilogue warps (11-14, one thread per TMEM
// lane) that read an item's O from TMEM, divide by the row sums and store it
// straight to global memory while the next item's Q loads, its first S tiles
// are computed and its first softmax runs; only the next item's first PV
// waits for them (barrier o_free). The row sums and maxima pass from the
// softmax warps to the epilogue warps through shared memory (stats, two
// buffers by item parity). Tile-indexed barriers and buffers use a tile
// counter that runs over all items of the pair, ring positions a stage
// counter over all items; items without a visible key load nothing and only
// write zeros (and lse -inf).
// ---------------------------------------------------------------------------

constexpr int kThreadsP = 480;
constexpr int kEpiWarp0 = 11;

struct PBars {
    Mailbox box[2][2][128];   // [exchange parity][column half][row]
    float2 stats[2][128];     // (running max in log2 units, row sum) per row, by item parity
    uint64_t q_full;          // leader: both CTAs' Q bytes of an item
    uint64_t q_empty;         // both: the item's last S MMA done (pair commit): Q smem free
    uint64_t s_full[2];
    uint64_t p_full[2];
    uint64_t o_done[2];
    uint64_t o_free;          // leader: one arrival per epilogue warp of each CTA: an item's O read out of TMEM
    uint64_t stats_full[2];   // both: 128 softmax arrivals (stats of an item written)
    uint64_t stats_free[2];   // both: 128 epilogue arrivals (stats of an item read)
    uint64_t mma_done;
    uint64_t ring_full[8];
    uint64_t ring_empty[8];
    uint32_t tmem_base;
    int abort;
    int k_seen;               // leader: K stages the S issuer has seen land (over the pair's tiles)
    int v_seen;               // leader: tiles whose V stages the PV issuer has seen land
};
static_assert(sizeof(PBars) <= 8192, "persistent barrier region");

// Epilogue staging: per epilogue warp 32 rows x 16 f32 columns, the 16-byte
// chunks of row r at chunk index k ^ ((r >> 1) & 3) (conflict-free writes of
// one row per lane and reads of 8 rows per instruction)
constexpr int kEpiWarps = 4;
constexpr int kEpiStageBytes = kEpiWarps * 32 * 16 * 4;

// Persistent-kernel tiling: KEYS keys per tile (the N of S). Width 256 takes
// 128-key tiles (its ring holds two tiles). Width 512 takes 64 or 128: with 64
// each CTA stages 32 KB of K (32 keys x 512 columns, boxes of 32 rows) and
// 16 KB of V (64 keys x its 128 output columns) per tile, so that the 5-slot
// ring holds K(j+1), V(j) and K(j+2) together; with 128 a tile's 96 KB exceed
// the 80 KB ring, but each tile carries twice the tensor work per softmax
// round trip.
template <int HD, int KEYS>
struct CfgP {
    static constexpr int kKeys = KEYS;                  // N of S for the pair
    static constexpr int kKeysCta = kKeys / 2;         // K rows each CTA loads
    static constexpr int kKBoxBytes = kKeysCta * 128;  // one 64-column box of those rows
    static constexpr int kQBoxes = Cfg<HD>::kQBoxes;
    static constexpr int kRing = Cfg<HD>::kRing;
    static constexpr int kStageBytes = Cfg<HD>::kStageBytes;
    static constexpr int kKBoxesPerStage = kStageBytes / kKBoxBytes;
    static constexpr int kKStages = HD / 64 / kKBoxesPerStage;
    static constexpr int kVBoxesPerStage = kStageBytes / kBoxBytes;       // V boxes: 64 keys x 64 columns
    static constexpr int kVStages = 2 * (kKeys / 64) / kVBoxesPerStage;   // 2 column atoms per 64 keys
    static constexpr int kScores = kKeys / 2;                             // scores per softmax thread
    static constexpr int kSmemQ = Cfg<HD>::kSmemQ;
    static constexpr int kSmemRing = kRing * kStageBytes;
    static constexpr int kSmemBytes = kSmemQ + kSmemRing + 8192 + kEpiStageBytes + 1024;
    static_assert(kSmemBytes <= 227 * 1024, "shared memory");
    static_assert(kKStages * kKBoxesPerStage * 64 == HD && kVStages >= 1, "stage layout");
    // A tile's stages exceed the ring (width 512, 128 keys): a slot is refilled
    // before every consumer has waited on its previous fill, and two progress
    // counters keep each parity wait exact.
    static constexpr bool kSeen = kKStages + kVStages > kRing;
    __device__ static int k_pos(int j) { return j == 0 ? 0 : kKStages + (j - 1) * (kKStages + kVStages); }
    __device__ static int v_pos(int j, int n) {
        return kKStages + j * (kKStages + kVStages) + (j + 1 < n ? kKStages : 0);
    }
};

template <int HD, int KEYS>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreadsP, 1)
    prefill_persistent(const ProblemDev *__restrict__ problems, const WorkItem *__restrict__ items,
                       const int32_t *__restrict__ pair_start, int *err, int stall, int wait_v) {
    // A launch that follows this one in the stream (the other head width of
    // the same call) may take SMs as this launch's pairs exit.
    ptx::pdl_trigger();
    if (stall) {
        stall_item(err);
        ptx::pdl_wait();
        return;
    }
    using C = CfgP<HD, KEYS>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *q_smem = smem;
    uint8_t *ring = smem + C::kSmemQ;
    PBars *bars = reinterpret_cast<PBars *>(ring + C::kSmemRing);
    volatile int *abort = &bars->abort;

    const uint32_t rank = ptx::cluster_ctarank();  // 0 = leader
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pair = blockIdx.x >> 1;
    const int i0 = pair_start[pair], i1 = pair_start[pair + 1];

    if (threadIdx.x == 0) {
        ptx::mbar_init(&bars->q_full, 1);
        ptx::mbar_init(&bars->q_empty, 1);
        for (int i = 0; i < 2; i++) {
            ptx::mbar_init(&bars->s_full[i], 1);
            ptx::mbar_init(&bars->p_full[i], 2 * kSoftmaxWarps);
            ptx::mbar_init(&bars->o_done[i], 1);
            ptx::mbar_init(&bars->stats_full[i], kRows);
            ptx::mbar_init(&bars->stats_free[i], kRows);
        }
        ptx::mbar_init(&bars->o_free, 2 * kEpiWarps);
        ptx::mbar_init(&bars->mma_done, 2);
        for (int i = 0; i < C::kRing; i++) {
            ptx::mbar_init(&bars->ring_full[i], 1);
            ptx::mbar_init(&bars->ring_empty[i], 1);
        }
        bars->abort = 0;
        bars->k_seen = 0;
        bars->v_seen = 0;
        ptx::fence_mbar_init();
    }
    for (int i = threadIdx.x; i < 2 * 2 * kRows; i += blockDim.x)
        bars->box[i / (2 * kRows)][(i / kRows) & 1][i % kRows] = Mailbox{-1, 0.0f};
    if (warp == 1) {
        ptx::tmem_alloc2(&bars->tmem_base, kTmemCols);
        ptx::tmem_relinquish2();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::cluster_sync();  // barrier inits of both CTAs visible before any remote signal
    ptx::tc_fence_after();
    const uint32_t tmem = bars->tmem_base;

    auto slot_of = [](int pos) { return pos % C::kRing; };
    auto phase_of = [](int pos) { return (uint32_t)(pos / C::kRing) & 1u; };

    if (warp == 0) {
        // ------------------------------------------------------------ producer (both CTAs)
        if (lane == 0) {
            int slot = 0;
            uint32_t phase = 0;
            uint32_t issued = 0;  // bit s: slot s received at least one load
            uint32_t qk = 0;      // items with keys so far (Q loads issued)
            bool ok = true;
            for (int i = i0; i < i1 && ok; i++) {
                const WorkItem it = items[i];
                const int n_tiles = it.n_kv_tiles;
                if (n_tiles == 0) continue;
                const ProblemDev &pb = problems[it.problem];
                ptx::prefetch_tmap(&pb.tq);
                ptx::prefetch_tmap(C::kKeysCta == 32 ? &pb.tk32 : &pb.tk);
                ptx::prefetch_tmap(&pb.tv);
                // Q of this item once the previous item's last S MMA has read the old Q
                if (qk > 0 && !wait_bar(&bars->q_empty, (qk - 1) & 1u, abort, err)) {
                    ok = false;
                    break;
                }
                if (rank == 0) ptx::mbar_arrive_expect_tx(&bars->q_full, 2 * C::kSmemQ);
                const uint32_t q_full_l = ptx::mapa(&bars->q_full, 0);
                for (int c = 0; c < C::kQBoxes; c++)
                    ptx::tma_load_2d_pair(q_smem + c * kQBoxBytes, &pb.tq, q_full_l, 64 * c,
                                          it.q_tile * 2 * kRows + (int)rank * kRows);
                // the next item's Q into L2 meanwhile (its load waits for this
                // item's last S, then reads L2 instead of HBM)
                for (int n = i + 1; n < i1; n++) {
                    const WorkItem nx = items[n];
                    if (nx.n_kv_tiles == 0) continue;
                    const CUtensorMap *ntq = &problems[nx.problem].tq;
                    for (int c = 0; c < C::kQBoxes; c++)
                        ptx::tma_prefetch_l2_2d(ntq, 64 * c, nx.q_tile * 2 * kRows + (int)rank * kRows);
                    break;
                }
                qk++;
                // one stage of n boxes of box_bytes each, box b at (xs[b], ys[b])
                auto push = [&](const CUtensorMap *m, const int *xs, const int *ys, int n, int box_bytes) {
                    if (!ok) return;
                    if (!wait_bar(&bars->ring_empty[slot], phase ^ 1u, abort, err)) {
                        ok = false;
                        return;
                    }
                    if (rank == 0) ptx::mbar_arrive_expect_tx(&bars->ring_full[slot], 2 * C::kStageBytes);
                    const uint32_t bar_l = ptx::mapa(&bars->ring_full[slot], 0);
                    for (int b = 0; b < n; b++)
                        ptx::tma_load_2d_pair(ring + slot * C::kStageBytes + b * box_bytes, m, bar_l, xs[b], ys[b]);
                    issued |= 1u << slot;
                    if (++slot == C::kRing) {
                        slot = 0;
                        phase ^= 1u;
                    }
                };
                // K: this CTA's kKeysCta keys of the tile, all HD columns (width 512:
                // the map with 32-row boxes)
                const CUtensorMap *tk = C::kKeysCta == 32 ? &pb.tk32 : &pb.tk;
                auto push_k = [&](int j) {
                    const int y = (it.kv_tile_lo + j) * C::kKeys + C::kKeysCta * (int)rank;
                    for (int st = 0; st < C::kKStages; st++) {
                        int xs[C::kKBoxesPerStage], ys[C::kKBoxesPerStage];
                        for (int b = 0; b < C::kKBoxesPerStage; b++) {
                            xs[b] = 64 * (st * C::kKBoxesPerStage + b);
                            ys[b] = y;
                        }
                        push(tk, xs, ys, C::kKBoxesPerStage, C::kKBoxBytes);
                    }
                };
                // V: this CTA's 128 output columns (two 64-column atoms) of the
                // tile's 64-key halves; box q = 2 * key half + atom
                auto push_v = [&](int j) {
                    if (wait_v) {  // V comes from the conversion this launch may overlap
                        ptx::pdl_wait();
                        wait_v = 0;
                    }
                    const int x = it.dv_half * kDV + 128 * (int)rank;
                    const int y = (it.kv_tile_lo + j) * C::kKeys;
                    for (int st = 0; st < C::kVStages; st++) {
                        int xs[C::kVBoxesPerStage], ys[C::kVBoxesPerStage];
                        for (int b = 0; b < C::kVBoxesPerStage; b++) {
                            const int q = st * C::kVBoxesPerStage + b;
                            xs[b] = x + 64 * (q & 1);
                            ys[b] = y + 64 * (q >> 1);
                        }
                        push(&pb.tv, xs, ys, C::kVBoxesPerStage, kBoxBytes);
                    }
                };
                push_k(0);
                for (int j = 0; j < n_tiles && ok; j++) {
                    if (j + 1 < n_tiles) push_k(j + 1);
                    push_v(j);
                }
            }
            // Drain (leader): every load of both CTAs signals the leader's
            // barriers; no TMA write may land after the pair exits. Normally
            // the MMA threads already waited for every load; after an abort,
            // wait here (bounded) for the last Q and each slot's latest load.
            if (rank == 0 && qk > 0) {
                for (uint32_t i = 0; i < kWaitLimit && !ptx::mbar_try_wait(&bars->q_full, (qk - 1) & 1u); i++) {
                }
                if (!ok || *abort) {
                    for (int s = 0; s < C::kRing; s++) {
                        if (!(issued >> s & 1u)) continue;
                        const uint32_t ph = s < slot ? phase : phase ^ 1u;
                        for (uint32_t i = 0; i < kWaitLimit && !ptx::mbar_try_wait(&bars->ring_full[s], ph); i++) {
                        }
                    }
                }
            }
            // Non-leader after an abort: its loads signal the leader's barriers,
            // which the leader may not have armed for a stage it never reached,
            // so their completion cannot be observed from here; the CTA lets
            // 200 us of the global timer pass (far above any load's latency)
            // before it may exit.
            if (rank != 0 && (!ok || *abort)) {
                const uint64_t t0 = ptx::globaltimer_ns();
                while (ptx::globaltimer_ns() - t0 < 200000ull) __nanosleep(2000);
            }
        }
    } else if (warp == 1 || warp == kPvWarp) {
        // ------------------------------------------------------------ MMA issuers (leader)
        const uint64_t q_desc = ptx::smem_desc(ptx::smem_u32(q_smem), 16, 1024);
        const uint64_t k_desc = ptx::smem_desc(ptx::smem_u32(ring), 16, 1024);
        const uint64_t v_desc = ptx::smem_desc(ptx::smem_u32(ring), kBoxBytes, 1024);
        if (lane == 0 && rank == 0) {
            bool ok = true;
            uint32_t g = 0;    // tile counter over the pair's items
            uint32_t qk = 0;   // items with keys so far
            int pos_base = 0;  // push-sequence position of the item's first stage
            for (int i = i0; i < i1 && ok; i++) {
                const int n_tiles = items[i].n_kv_tiles;
                if (n_tiles == 0) continue;
                if (warp == 1) {
                    // S(g) = Q K^T into S buffer g&1, once PV(g-2) has read P(g-2) from it
                    constexpr uint32_t kIdescS = ptx::idesc_f16(1, 1, 0, 2 * kRows, C::kKeys);
                    if (!wait_bar(&bars->q_full, qk & 1u, abort, err)) {
                        ok = false;
                        break;
                    }
                    for (int j = 0; j < n_tiles && ok; j++, g++) {
                        if (g >= 2 && !wait_bar(&bars->o_done[g & 1], ((g - 2) >> 1) & 1u, abort, err)) {
                            ok = false;
                            break;
                        }
                        // K(0)'s last stage takes the slot of the previous item's last
                        // V stage; its parity wait is exact once the PV issuer has
                        // seen that V stage land
                        if (C::kSeen && j == 0 && g >= 1 && !wait_count(&bars->v_seen, (int)g, abort, err)) {
                            ok = false;
                            break;
                        }
                        ptx::tc_fence_after();
                        const uint32_t d = tmem + ((g & 1) ? kColS1 : kColS0);
                        const int pos = pos_base + C::k_pos(j);
                        for (int st = 0; st < C::kKStages && ok; st++) {
                            const int slot = slot_of(pos + st);
                            if (!wait_bar(&bars->ring_full[slot], phase_of(pos + st), abort, err)) {
                                ok = false;
                                break;
                            }
                            if (C::kSeen) set_count(&bars->k_seen, (int)(g * C::kKStages) + st + 1);
                            ptx::tc_fence_after();
#pragma unroll
                            for (int b = 0; b < C::kKBoxesPerStage; b++) {
                                const uint64_t kd =
                                    k_desc + (uint64_t)((slot * C::kStageBytes + b * C::kKBoxBytes) >> 4);
                                const uint64_t qd =
                                    q_desc + (uint64_t)((C::kKBoxesPerStage * st + b) * (kQBoxBytes >> 4));
                                ptx::mma2_ss(d, qd, kd, kIdescS, (st | b) != 0);
#pragma unroll
                                for (int kk = 1; kk < 4; kk++) ptx::mma2_ss(d, qd + 2 * kk, kd + 2 * kk, kIdescS, 1);
                            }
                            ptx::mma2_commit_pair(&bars->ring_empty[slot], kBothCtas);
                        }
                        if (ok) ptx::mma2_commit_pair(&bars->s_full[g & 1], kBothCtas);
                    }
                    // the item's Q is free once its last S MMA completes
                    if (ok) ptx::mma2_commit_pair(&bars->q_empty, kBothCtas);
                } else {
                    // O += P(g) V(g) once the softmax of both CTAs published P(g);
                    // the item's first PV also waits for the previous item's O to
                    // be read out by the epilogue warps of both CTAs
                    constexpr uint32_t kIdescPV = ptx::idesc_f16(0, 0, 1, 2 * kRows, kDV);
                    for (int j = 0; j < n_tiles && ok; j++, g++) {
                        if (!wait_bar<true>(&bars->p_full[g & 1], (g >> 1) & 1u, abort, err)) {
                            ok = false;
                            break;
                        }
                        if (j == 0 && qk > 0 && !wait_bar(&bars->o_free, (qk - 1) & 1u, abort, err)) {
                            ok = false;
                            break;
                        }
                        // V(j)'s second slot last held K(j+1)'s first stage when a tile
                        // exceeds the ring: the wait needs only that stage seen (PV(j)
                        // then runs between S(j+1)'s stages); otherwise every slot's
                        // previous fill has landed before its next parity wait (both
                        // checked by a randomized model of the protocol)
                        if (C::kSeen && j + 1 < n_tiles &&
                            !wait_count(&bars->k_seen, (int)((g + 1) * C::kKStages) + 1, abort, err)) {
                            ok = false;
                            break;
                        }
                        const int pos = pos_base + C::v_pos(j, n_tiles);
                        for (int c = 0; c < C::kVStages && ok; c++)
                            ok = wait_bar(&bars->ring_full[slot_of(pos + c)], phase_of(pos + c), abort, err);
                        if (!ok) break;
                        if (C::kSeen) set_count(&bars->v_seen, (int)g + 1);
                        ptx::tc_fence_after();
                        const uint32_t p_tmem = tmem + ((g & 1) ? kColS1 : kColS0);
                        // keys 16 ks.. are in V box vb = 2 * (ks / 4) (its 64-key half,
                        // first column atom; the next box holds the second atom), 16
                        // rows of 128 bytes per k-step
#pragma unroll
                        for (int ks = 0; ks < C::kKeys / 16; ks++) {
                            const int vb = 2 * (ks / 4);
                            const uint64_t vd =
                                v_desc + (uint64_t)((slot_of(pos + vb / C::kVBoxesPerStage) * C::kStageBytes +
                                                     (vb % C::kVBoxesPerStage) * kBoxBytes) >> 4) +
                                (uint64_t)((2048 >> 4) * (ks & 3));
                            ptx::mma2_ts(tmem + kColO, p_tmem + 8 * ks, vd, kIdescPV, (j > 0 || ks > 0) ? 1u : 0u);
                        }
                        for (int c = 0; c < C::kVStages; c++)
                            ptx::mma2_commit_pair(&bars->ring_empty[slot_of(pos + c)], kBothCtas);
                        ptx::mma2_commit_pair(&bars->o_done[g & 1], kBothCtas);
                    }
                }
                qk++;
                pos_base += n_tiles * (C::kKStages + C::kVStages);
            }
            // Every MMA this thread issued completes before either CTA
            // releases TMEM or exits (mma_done expects one commit per issuer).
            ptx::mma2_commit_pair(&bars->mma_done, kBothCtas);
            for (uint32_t i = 0; i < kWaitLimit && !ptx::mbar_try_wait(&bars->mma_done, 0); i++) {
            }
        } else if (warp == 1 && lane == 0) {
            // non-leader: wait (bounded) for the leader's final commits
            for (uint32_t i = 0; i < kWaitLimit && !ptx::mbar_try_wait(&bars->mma_done, 0); i++) {
                if ((i & 1023) == 1023 && *abort) break;
            }
        }
    } else if (warp < kEpiWarp0) {
        // ------------------------------------------------------------ softmax (warps 2-9)
        const int quad = warp & 3;
        const int half = (warp - 2) >> 2;
        const int row = quad * 32 + lane;
        const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
        const float kLog2e = 1.4426950408889634f;
        const uint32_t p_full_l0 = ptx::mapa(&bars->p_full[0], 0), p_full_l1 = ptx::mapa(&bars->p_full[1], 0);
        Mailbox *my_box = &bars->box[0][half][row];
        Mailbox *other_box = &bars->box[0][half ^ 1][row];
        uint32_t e = 0;  // exchanges with the partner thread so far (both halves make the same sequence)
        // Post (e, v) and read the partner's value for the same exchange.
        auto swap = [&](float v, float *out) -> bool {
            const int seq = (int)e;
            const int par = seq & 1;
            e++;
            const uint32_t mine = ptx::smem_u32(my_box + par * 2 * kRows);
            const uint32_t theirs = ptx::smem_u32(other_box + par * 2 * kRows);
            const uint64_t word = (uint64_t)(uint32_t)seq | ((uint64_t)__float_as_uint(v) << 32);
            asm volatile("st.volatile.shared.b64 [%0], %1;" ::"r"(mine), "l"(word) : "memory");
            for (uint32_t i = 0; i < kWaitLimit; i++) {
                uint64_t t;
                asm volatile("ld.volatile.shared.b64 %0, [%1];" : "=l"(t) : "r"(theirs) : "memory");
                if ((int)(uint32_t)t == seq) {
                    *out = __uint_as_float((uint32_t)(t >> 32));
                    return true;
                }
                if ((i & 255) == 255 && *abort) return false;
            }
            *abort = 1;
            atomicOr(err, 2);
            return false;
        };
        bool ok = true;
        uint32_t g = 0, qk = 0;
        for (int i = i0; i < i1 && ok; i++) {
            const WorkItem it = items[i];
            const int n_tiles = it.n_kv_tiles;
            if (n_tiles == 0) continue;
            // the problem's fields in registers for the item (the inline asm's
            // memory clobbers would otherwise reload them from global memory)
            const ProblemDev &pb = problems[it.problem];
            const int kv_pos0 = pb.kv_pos0, n_kv = pb.n_kv, window = pb.window;
            const int tok0 = it.q_tile * kTokensPerPair + (int)rank * kTokensPerCta;
            const int qpos = pb.q_pos0 + tok0 + row / 8;
            const int vis_hi = min(qpos - kv_pos0, n_kv - 1);
            const int vis_lo = window > 0 ? qpos - window + 1 - kv_pos0 : INT_MIN / 2;
            const int q_first = pb.q_pos0 + tok0;
            const int q_last = q_first + kTokensPerCta - 1;
            float m_used = -CUDART_INF_F;
            float l = 0.0f;
            for (int j = 0; j < n_tiles && ok; j++, g++) {
                if (!__all_sync(0xffffffffu, wait_bar(&bars->s_full[g & 1], (g >> 1) & 1u, abort, err))) {
                    ok = false;
                    break;
                }
                ptx::tc_fence_after();
                const uint32_t s_addr = tmem + lane_addr + ((g & 1) ? kColS1 : kColS0);
                // this thread's kSc scores: columns [kSc * half, kSc * half + kSc) of S
                constexpr int kSc = C::kScores;
                float s[kSc];
#pragma unroll
                for (int q = 0; q < kSc / 32; q++) {
                    uint32_t r0[32];
                    ptx::tmem_ld32(s_addr + kSc * half + 32 * q, r0);
                    ptx::tmem_wait_ld();
                    ptx::tmem_ld_fence(r0);
#pragma unroll
                    for (int c = 0; c < 32; c++) s[32 * q + c] = __uint_as_float(r0[c]);
                }
                const int k0 = (it.kv_tile_lo + j) * C::kKeys;
                const int kp0 = kv_pos0 + k0;
                const bool edge = k0 + C::kKeys > n_kv || kp0 + C::kKeys - 1 > q_first ||
                                  (window > 0 && q_last - kp0 >= window);
                if (edge) {
                    const int kb = k0 + kSc * half;
                    const int lo = vis_lo - kb, hi = vis_hi - kb;  // visible columns: lo <= c <= hi
                    // a warp's 32 rows are 4 tokens: the sides that cut into the
                    // tile agree across it, and a one-sided mask takes 2 instructions
                    const bool cut_lo = __any_sync(0xffffffffu, lo > 0);
                    const bool cut_hi = __any_sync(0xffffffffu, hi < kSc - 1);
                    if (cut_lo && cut_hi) {
#pragma unroll
                        for (int c = 0; c < kSc; c++) s[c] = (c >= lo && c <= hi) ? s[c] : -CUDART_INF_F;
                    } else if (cut_hi) {
#pragma unroll
                        for (int c = 0; c < kSc; c++) s[c] = c <= hi ? s[c] : -CUDART_INF_F;
                    } else if (cut_lo) {
#pragma unroll
                        for (int c = 0; c < kSc; c++) s[c] = c >= lo ? s[c] : -CUDART_INF_F;
                    }
                }
                float mx = max_tree<kSc>(s);
                float mo;
                if (!__all_sync(0xffffffffu, swap(mx, &mo))) {
                    ok = false;
                    break;
                }
                mx = fmaxf(mx, mo) * kLog2e;
                // lazy rescale with a 2^15 margin (P <= 2^15 fits fp16)
                const bool grow = mx > m_used + 15.0f;
                const bool o_live = grow && m_used != -CUDART_INF_F;
                const float f = o_live ? ptx::ex2(m_used - mx) : 1.0f;
                if (grow) m_used = mx;
                const float neg_m = m_used == -CUDART_INF_F ? 0.0f : -m_used;
                // pairs of scores in packed fp32: x = s log2e - m, P = 2^x (5 of
                // every 8 pairs on the MUFU pipe, the rest on the FMA pipe), the
                // row sum in 4 packed partial sums. P (fp16 pairs) goes over the
                // first kSc / 2 columns of this half's part of the S buffer, 16
                // columns at a time, each store issued as soon as its pairs are
                // packed (the next pairs' exponentials overlap its latency); the
                // columns half 1 writes were read by half 0 before it posted its max.
                const float2 scale = make_float2(kLog2e, kLog2e), shift = make_float2(neg_m, neg_m);
                float2 rs[4];
#pragma unroll
                for (int k = 0; k < 4; k++) rs[k] = make_float2(0.0f, 0.0f);
#pragma unroll
                for (int q = 0; q < kSc / 32; q++) {
                    uint32_t pk[16];
#pragma unroll
                    for (int cc = 0; cc < 16; cc++) {
                        const int c = 16 * q + cc;
                        const float2 x = ptx::fma2(make_float2(s[2 * c], s[2 * c + 1]), scale, shift);
                        const float2 pr = (c & 7) < 5 ? make_float2(ptx::ex2(x.x), ptx::ex2(x.y)) : ex2_fma2(x);
                        rs[c & 3] = ptx::add2(rs[c & 3], pr);
                        pk[cc] = ptx::pack_half2(pr.x, pr.y);
                    }
                    ptx::tmem_st16(s_addr + (kSc / 2) * half + 16 * q, pk);
                }
                const float2 rsum = ptx::add2(ptx::add2(rs[0], rs[1]), ptx::add2(rs[2], rs[3]));
                l = l * f + (rsum.x + rsum.y);
                if (__any_sync(0xffffffffu, o_live)) {
                    // O holds this item's earlier tiles (j >= 1): wait for PV(g-1)
                    if (!__all_sync(0xffffffffu, wait_bar(&bars->o_done[(g - 1) & 1], ((g - 1) >> 1) & 1u, abort, err))) {
                        ok = false;
                        break;
                    }
                    ptx::tc_fence_after();
#pragma unroll 1
                    for (int c = 0; c < kDV / 128; c++) {
                        uint32_t o0[32], o1[32];
                        const uint32_t o_addr = tmem + lane_addr + kColO + 128 * half + 64 * c;
                        ptx::tmem_ld32(o_addr, o0);
                        ptx::tmem_ld32(o_addr + 32, o1);
                        ptx::tmem_wait_ld();
                        ptx::tmem_ld_fence(o0);
                        ptx::tmem_ld_fence(o1);
                        const float2 f2 = make_float2(f, f);
#pragma unroll
                        for (int k = 0; k < 32; k += 2) {
                            float2 a0 = ptx::mul2(make_float2(__uint_as_float(o0[k]), __uint_as_float(o0[k + 1])), f2);
                            float2 a1 = ptx::mul2(make_float2(__uint_as_float(o1[k]), __uint_as_float(o1[k + 1])), f2);
                            o0[k] = __float_as_uint(a0.x);
                            o0[k + 1] = __float_as_uint(a0.y);
                            o1[k] = __float_as_uint(a1.x);
                            o1[k + 1] = __float_as_uint(a1.y);
                        }
                        ptx::tmem_st32(o_addr, o0);
                        ptx::tmem_st32(o_addr + 32, o1);
                    }
                }
                ptx::tmem_wait_st();
                ptx::tc_fence_before();
                __syncwarp();
                if (lane == 0) {  // the leader's own warps arrive locally (CTA-scope release)
                    if (rank == 0) ptx::mbar_arrive(&bars->p_full[g & 1]);
                    else ptx::mbar_arrive_cl((g & 1) ? p_full_l1 : p_full_l0);
                }
            }
            if (!ok) break;
            // the item's row sums meet; its stats go to the epilogue warps
            float lo_ = 0.0f;
            if (!__all_sync(0xffffffffu, swap(l, &lo_))) {
                ok = false;
                break;
            }
            l += lo_;
            // Only half 0 writes the stats, so only it waits for their slot: the
            // epilogue may release the slot's next use (this item's stats) as soon
            // as half 0 posts them, and a parity wait of half 1 would then find
            // the barrier two phases on.
            if (half == 0 && qk >= 2 &&
                !__all_sync(0xffffffffu, wait_bar(&bars->stats_free[qk & 1], ((qk - 2) >> 1) & 1u, abort, err))) {
                ok = false;
                break;
            }
            if (half == 0) {
                bars->stats[qk & 1][row] = make_float2(m_used, l);
                ptx::mbar_arrive(&bars->stats_full[qk & 1]);
            }
            qk++;
        }
    } else {
        // ------------------------------------------------------------ epilogue (warps 11-14)
        // Warp w reaches TMEM lanes 32 * (w % 4).. (the rows of this CTA it
        // writes); thread t reads its own row's statistics, and the 256 output
        // columns are read 32 at a time and divided by the row sums.
        const int quad = warp & 3;
        const int row = quad * 32 + lane;
        const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
        const uint32_t o_free_l = ptx::mapa(&bars->o_free, 0);
        bool ok = true;
        uint32_t g = 0, qk = 0;
        for (int i = i0; i < i1 && ok; i++) {
            const WorkItem it = items[i];
            const int n_tiles = it.n_kv_tiles;
            const ProblemDev &pb = problems[it.problem];
            const int tok0 = it.q_tile * kTokensPerPair + (int)rank * kTokensPerCta;  // this CTA's first token
            // rows [tok0 * 8, tok0 * 8 + 128) of the [n_q * 8][HD] output; this warp's rows quad * 32 ..
            float *out_rows = pb.out + (size_t)tok0 * 8 * HD + it.dv_half * kDV;
            const int valid_rows = min(kRows, (pb.n_q - tok0) * 8);  // rows of tokens below n_q
            if (n_tiles == 0) {  // no visible key: zeros, lse -inf
                if (row < valid_rows) {
                    float *dst = out_rows + (size_t)row * HD;
                    for (int c = 0; c < kDV / 4; c++) reinterpret_cast<float4 *>(dst)[c] = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (pb.lse && it.dv_half == 0) pb.lse[(size_t)tok0 * 8 + row] = -CUDART_INF_F;
                }
                continue;
            }
            const uint32_t g_last = g + (uint32_t)n_tiles - 1;
            g += (uint32_t)n_tiles;
            if (!__all_sync(0xffffffffu, wait_bar(&bars->stats_full[qk & 1], (qk >> 1) & 1u, abort, err))) {
                ok = false;
                break;
            }
            const float2 st = bars->stats[qk & 1][row];
            ptx::mbar_arrive(&bars->stats_free[qk & 1]);
            if (!__all_sync(0xffffffffu, wait_bar(&bars->o_done[g_last & 1], (g_last >> 1) & 1u, abort, err))) {
                ok = false;
                break;
            }
            ptx::tc_fence_after();
            const float inv = st.y > 0.0f ? 1.0f / st.y : 0.0f;
            // Stores straight from registers: with the 16x256b TMEM shape, lanes
            // 4 g .. 4 g + 3 hold 8 consecutive columns (32 bytes) of one row, so
            // each 8-byte store completes a sector with its 3 neighbours, and no
            // staging in shared memory competes with the tensor core's operand
            // reads. Lane t writes rows 8 k + t / 4 (k = 0..3) of the warp's 32.
            const int tr = lane >> 2, tc = 2 * (lane & 3);
            float rinv[4];
#pragma unroll
            for (int k = 0; k < 4; k++) rinv[k] = __shfl_sync(0xffffffffu, inv, 8 * k + tr);
            // chunk c (32 columns): lo holds rows 0-15 of the warp's 32, hi rows 16-31
            auto load = [&](int c, uint32_t(&lo)[16], uint32_t(&hi)[16]) {
                ptx::tmem_ld16x256_x4(tmem + lane_addr + kColO + 32 * c, lo);
                ptx::tmem_ld16x256_x4(tmem + lane_addr + (16u << 16) + kColO + 32 * c, hi);
            };
            auto emit = [&](const uint32_t(&lo)[16], const uint32_t(&hi)[16], int c) {
#pragma unroll
                for (int sh = 0; sh < 2; sh++) {
                    const uint32_t(&r)[16] = sh ? hi : lo;
#pragma unroll
                    for (int k = 0; k < 4; k++) {
#pragma unroll
                        for (int e = 0; e < 2; e++) {  // e = 1: the row 8 below
                            const int orow = quad * 32 + 16 * sh + 8 * e + tr;
                            const float w = rinv[2 * sh + e];
                            if (orow < valid_rows)
                                *reinterpret_cast<float2 *>(out_rows + (size_t)orow * HD + 32 * c + 8 * k + tc) =
                                    make_float2(__uint_as_float(r[4 * k + 2 * e]) * w,
                                                __uint_as_float(r[4 * k + 2 * e + 1]) * w);
                        }
                    }
                }
            };
            // Two register sets: the TMEM loads of the next chunk are in flight
            // while the current one is stored. O is free for the next item once
            // the last chunk is in registers.
            uint32_t a0[16], a1[16], b0[16], b1[16];
            load(0, a0, a1);
            ptx::tmem_wait_ld();
            ptx::tmem_ld_fence16(a0);
            ptx::tmem_ld_fence16(a1);
#pragma unroll 1
            for (int c = 0; c < kDV / 32; c += 2) {
                load(c + 1, b0, b1);
                emit(a0, a1, c);
                ptx::tmem_wait_ld();
                ptx::tmem_ld_fence16(b0);
                ptx::tmem_ld_fence16(b1);
                const bool more = c + 2 < kDV / 32;
                if (more) {
                    load(c + 2, a0, a1);
                } else {
                    // every column of O is in registers: the next item's first PV may overwrite it
                    ptx::tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        if (rank == 0) ptx::mbar_arrive(&bars->o_free);
                        else ptx::mbar_arrive_cl(o_free_l);
                    }
                }
                emit(b0, b1, c + 1);
                if (more) {
                    ptx::tmem_wait_ld();
                    ptx::tmem_ld_fence16(a0);
                    ptx::tmem_ld_fence16(a1);
                }
            }
            if (row < valid_rows && pb.lse && it.dv_half == 0)
                pb.lse[(size_t)tok0 * 8 + row] = st.y > 0.0f ? (st.x + log2f(st.y)) * 0.6931471805599453f : -CUDART_INF_F;
            qk++;
        }
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::cluster_sync();  // no MMA or load of the pair still touches either CTA
    if (warp == 1) {
        __syncwarp();
        ptx::tc_fence_after();
        ptx::tmem_dealloc2(tmem, kTmemCols);
    }
    // Launched behind the other width: finish only after it (later work in the
    // stream then follows both launches); a no-op for a plain launch.
    ptx::pdl_wait();
}

// bf16 -> fp16 copies of up to kMaxSegs V arrays in one launch (blockIdx.y =
// segment); 8 elements per thread and step. Every count is a multiple of 8
// (a head width) and every address 16-byte aligned (checked on the host).
constexpr int kMaxSegs = 32;
struct ConvSegs {
    const __nv_bfloat16 *src[kMaxSegs];
    __half *dst[kMaxSegs];
    uint64_t n8[kMaxSegs];  // elements / 8
};

__global__ void bf16_to_f16_kernel(ConvSegs segs) {
    ptx::pdl_trigger();  // a prefill launched behind it may start; it waits before reading V
    const int sg = blockIdx.y;
    const uint4 *src = reinterpret_cast<const uint4 *>(segs.src[sg]);
    uint4 *dst = reinterpret_cast<uint4 *>(segs.dst[sg]);
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < segs.n8[sg];
         i += (uint64_t)gridDim.x * blockDim.x) {
        uint4 v = src[i];
        uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162 *>(&w[k]);
            const __half2 h = __floats2half2_rn(__bfloat162float(b.x), __bfloat162float(b.y));
            w[k] = *reinterpret_cast<const uint32_t *>(&h);
        }
        dst[i] = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

}  // namespace

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                    const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// The driver's tensor-map encoder, looked up at run time so that the library
// loads (for symbol checks) on machines without a driver.
static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

bool encode_tmap_2d(void *map, int dtype, const void *base, uint64_t cols, uint64_t rows, uint32_t box_rows) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const CUtensorMapDataType dt = dtype == 1 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * 2};
    const cuuint32_t box[2] = {64, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(reinterpret_cast<CUtensorMap *>(map), dt, 2, const_cast<void *>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool encode_tmap_2d_raw(void *map, int elem_bytes, const void *base, uint64_t inner, uint64_t outer,
                        uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, bool swizzle128) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const CUtensorMapDataType dt = elem_bytes == 1   ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                   : elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16
                                                     : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    return enc(reinterpret_cast<CUtensorMap *>(map), dt, 2, const_cast<void *>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Output map: f32 [rows, cols], 32-column x 128-row boxes, 128-byte swizzle.
static bool encode_out_f32(CUtensorMap *map, const float *base, uint64_t cols, uint64_t rows) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * 4};
    const cuuint32_t box[2] = {32, 128};
    const cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// One prepared problem list: what a launch of it needs on the device (the
// problem table, the work list, the fp16 copies of its V arrays) and the
// V-conversion launches. Everything launched from here reads only buffers this
// struct owns or the caller's pointers in the list, so an equal list means an
// equal launch.
struct Prepared {
    std::vector<g4a_prefill_problem> key;
    ProblemDev *d_problems = nullptr;
    WorkItem *d_items = nullptr;
    __half *v16 = nullptr;
    struct ConvLaunch {
        ConvSegs segs;
        unsigned bx;
        int cnt;
    };
    std::vector<ConvLaunch> conv;  // the width-512 sources' launches first, then width 256's
    size_t n_conv_wide = 0;
    size_t n_work[2] = {0, 0};
    bool mixed = false;  // both widths in one launch (the items in one cost order)
    // persistent launches: per width, n_pairs CTA pairs, pair p running the
    // items [pair_start[p], pair_start[p + 1]) of that width's list
    bool persistent = false;
    int keys512 = 128;  // key tile of the width-512 persistent launch
    int reserve = 0;    // SMs left free (part of the cache key)
    int32_t *d_pair_start = nullptr;  // width 256's table, then width 512's
    int n_pairs[2] = {0, 0};
    uint64_t used = 0;   // call counter at the last use
};

// Host-side state the prefill keeps in the context between calls.
struct PrefillScratch {
    bool attr_set = false;
    int n_sm = 0;          // of the device, read on the first call
    int persistent = -1;   // 1: persistent CTA pairs, 0: a CTA pair per item (G4A_PREFILL_KERNEL)
    int keys512 = 128;     // key tile of the persistent width-512 kernel (G4A_PREFILL_KEYS512: 64 or 128)
    // Tensor maps by (kind, base, columns, rows): the encoder is a driver call
    // per map, and repeated calls (a model's layers, every prompt of a batch)
    // name the same buffers.
    struct MapKey {
        int kind;
        const void *base;
        uint64_t cols, rows;
        bool operator==(const MapKey &o) const {
            return kind == o.kind && base == o.base && cols == o.cols && rows == o.rows;
        }
    };
    struct MapHash {
        size_t operator()(const MapKey &k) const {
            return std::hash<const void *>()(k.base) ^ (k.cols * 0x9E3779B97F4A7C15ull) ^ (k.rows << 7) ^ (size_t)k.kind;
        }
    };
    std::unordered_map<MapKey, CUtensorMap, MapHash> maps;
    // The last few problem lists, prepared: a call that repeats one exactly (a
    // model's prompt loop, a benchmark, the alternating lists of a
    // context-parallel schedule) skips validation, map encoding, work-list
    // construction and uploads.
    static constexpr int kCached = 8;
    Prepared cache[kCached];
    uint64_t calls = 0;
};

static void free_prepared(Prepared &p) {
    cudaFree(p.d_problems);
    cudaFree(p.d_items);
    cudaFree(p.v16);
    cudaFree(p.d_pair_start);
    p = Prepared();
}

static cudaError_t launch_prepared(PrefillScratch *S, const Prepared &P, int *d_err, cudaStream_t st,
                                   bool stall) {
    for (const auto &c : P.conv) bf16_to_f16_kernel<<<dim3(c.bx, c.cnt), 256, 0, st>>>(c.segs);
    if (!S->attr_set) {
        cudaFuncSetAttribute(prefill_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<256>::kSmemBytes);
        cudaFuncSetAttribute(prefill_kernel<512>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<512>::kSmemBytes);
        cudaFuncSetAttribute(prefill_kernel_mixed, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMixed);
        cudaFuncSetAttribute(prefill_persistent<256, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             CfgP<256, 128>::kSmemBytes);
        cudaFuncSetAttribute(prefill_persistent<512, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             CfgP<512, 64>::kSmemBytes);
        cudaFuncSetAttribute(prefill_persistent<512, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             CfgP<512, 128>::kSmemBytes);
        S->attr_set = true;
    }
    if (P.persistent) {
        // Programmatic stream serialization: the width-256 launch starts while
        // the width-256 V conversion (the last conversion launch) runs and waits
        // for it before its first V load; width 512 follows width 256, taking
        // SMs as its pairs finish (its V, converted first, is complete by then).
        // Alone, width 512 follows the conversions the same way width 256 does.
        const bool narrow_conv = P.conv.size() > P.n_conv_wide;
        const int st_flag = (int)stall;
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute pdl[1];
        pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        pdl[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = pdl;
        cfg.stream = st;
        cfg.blockDim = dim3(kThreadsP);
        if (P.n_pairs[0]) {
            cfg.numAttrs = narrow_conv ? 1 : 0;
            cfg.gridDim = dim3(2 * (unsigned)P.n_pairs[0]);
            cfg.dynamicSmemBytes = CfgP<256, 128>::kSmemBytes;
            const cudaError_t e = cudaLaunchKernelEx(&cfg, prefill_persistent<256, 128>, (const ProblemDev *)P.d_problems,
                                                     (const WorkItem *)P.d_items, (const int32_t *)P.d_pair_start, d_err,
                                                     st_flag, narrow_conv ? 1 : 0);
            if (e != cudaSuccess) return e;
        }
        if (P.n_pairs[1]) {
            const bool first = P.n_pairs[0] == 0;
            const int wait_v = first && !P.conv.empty() ? 1 : 0;
            cfg.numAttrs = !first || wait_v ? 1 : 0;
            cfg.gridDim = dim3(2 * (unsigned)P.n_pairs[1]);
            const WorkItem *items = P.d_items + P.n_work[0];
            const int32_t *starts = P.d_pair_start + P.n_pairs[0] + 1;
            if (P.keys512 == 64) {
                cfg.dynamicSmemBytes = CfgP<512, 64>::kSmemBytes;
                return cudaLaunchKernelEx(&cfg, prefill_persistent<512, 64>, (const ProblemDev *)P.d_problems, items,
                                          starts, d_err, st_flag, wait_v);
            }
            cfg.dynamicSmemBytes = CfgP<512, 128>::kSmemBytes;
            return cudaLaunchKernelEx(&cfg, prefill_persistent<512, 128>, (const ProblemDev *)P.d_problems, items, starts,
                                      d_err, st_flag, wait_v);
        }
        return cudaSuccess;
    }
    // two CTAs (one cluster) per work item
    if (P.mixed) {
        prefill_kernel_mixed<<<2 * (unsigned)(P.n_work[0] + P.n_work[1]), kThreads, kSmemMixed, st>>>(
            P.d_problems, P.d_items, d_err, (int)stall);
        return cudaGetLastError();
    }
    if (P.n_work[0])
        prefill_kernel<256><<<2 * (unsigned)P.n_work[0], kThreads, Cfg<256>::kSmemBytes, st>>>(
            P.d_problems, P.d_items, d_err, (int)stall);
    if (P.n_work[1])
        prefill_kernel<512><<<2 * (unsigned)P.n_work[1], kThreads, Cfg<512>::kSmemBytes, st>>>(
            P.d_problems, P.d_items + P.n_work[0], d_err, (int)stall);
    return cudaGetLastError();
}

// kind 0: bf16 Q (128-row boxes), 1: bf16 K (64-row boxes), 2: fp16 V (64-row boxes), 3: f32 output
static bool cached_map(PrefillScratch *S, int kind, const void *base, uint64_t cols, uint64_t rows, CUtensorMap *out) {
    const PrefillScratch::MapKey key{kind, base, cols, rows};
    auto f = S->maps.find(key);
    if (f != S->maps.end()) {
        *out = f->second;
        return true;
    }
    bool ok;
    if (kind == 3) ok = encode_out_f32(out, static_cast<const float *>(base), cols, rows);
    else ok = encode_tmap_2d(out, kind == 2 ? 1 : 0, base, cols, rows, kind == 0 ? kRows : kind == 4 ? 32 : 64);
    if (!ok) return false;
    if (S->maps.size() > 4096) S->maps.clear();
    S->maps.emplace(key, *out);
    return true;
}

PrefillScratch *prefill_scratch_new() { return new PrefillScratch(); }
void prefill_scratch_free(PrefillScratch *s) {
    if (!s) return;
    for (auto &p : s->cache) free_prepared(p);
    delete s;
}

// Validates, converts V to fp16, builds tensor maps and the work list, and
// launches one kernel per head width. Returns a g4a_status; *msg names the
// failure.
int prefill_run(PrefillScratch *S, int *d_err, int32_t n, const g4a_prefill_problem *pr, cudaStream_t st,
                const char **msg, bool stall, int reserve_sms) {
    *msg = "";
    if (n < 0 || (n > 0 && !pr)) {
        *msg = "invalid prefill problem list";
        return G4A_COMPUTE;
    }
    S->calls++;
    for (auto &P : S->cache) {
        if (P.used && P.key.size() == (size_t)n && P.reserve == reserve_sms &&
            (n == 0 || std::memcmp(pr, P.key.data(), (size_t)n * sizeof(g4a_prefill_problem)) == 0)) {
            P.used = S->calls;
            const cudaError_t e = launch_prepared(S, P, d_err, st, stall);
            if (e != cudaSuccess) {
                *msg = cudaGetErrorString(e);
                return G4A_CUDA;
            }
            return G4A_OK;
        }
    }
    // a new list: prepared into the least recently used slot (its buffers may
    // still be read by queued launches, so the stream drains first)
    Prepared *slot = &S->cache[0];
    for (auto &P : S->cache)
        if (P.used < slot->used) slot = &P;
    if (slot->used) {
        cudaStreamSynchronize(st);
        free_prepared(*slot);
    }
    Prepared &P = *slot;
    // distinct V arrays -> fp16 copies, each sized for the most rows any problem reads
    std::vector<const void *> v_src;
    std::vector<size_t> v_len;
    std::vector<char> v_wide;  // read by a width-512 problem
    for (int32_t i = 0; i < n; i++) {
        const g4a_prefill_problem &p = pr[i];
        if (p.head_dim != 256 && p.head_dim != 512) {
            *msg = "prefill head width must be 256 or 512";
            return G4A_COMPUTE;
        }
        if (p.n_q < 0 || p.n_kv < 0 || p.window < 0 || p.q_pos0 < 0 || p.kv_pos0 < 0 ||
            (int64_t)p.n_q * 8 > INT32_MAX) {
            *msg = "invalid prefill shape";
            return G4A_COMPUTE;
        }
        if (p.n_q > 0 && (!p.q_dev || !p.out_dev)) {
            *msg = "null prefill query or output";
            return G4A_COMPUTE;
        }
        if (p.n_kv > 0 && (!p.k_dev || !p.v_dev)) {
            *msg = "null prefill keys or values";
            return G4A_COMPUTE;
        }
        const uintptr_t al = (uintptr_t)p.q_dev | (uintptr_t)p.k_dev | (uintptr_t)p.v_dev | (uintptr_t)p.out_dev;
        if (al & 15u) {
            *msg = "prefill buffers must be 16-byte aligned";
            return G4A_COMPUTE;
        }
        if (p.n_kv > 0) {
            const size_t k = std::find(v_src.begin(), v_src.end(), p.v_dev) - v_src.begin();
            if (k == v_src.size()) {
                v_src.push_back(p.v_dev);
                v_len.push_back(0);
                v_wide.push_back(0);
            }
            v_len[k] = std::max(v_len[k], (size_t)p.n_kv * p.head_dim);
            v_wide[k] |= p.head_dim == 512;
        }
    }
    std::vector<size_t> v_off(v_src.size(), 0);
    size_t v_total = 0;
    for (size_t k = 0; k < v_src.size(); k++) {
        v_off[k] = v_total;
        v_total += v_len[k];  // multiples of 256 elements: every copy stays 16-byte aligned
    }
    cudaError_t e = cudaMalloc(&P.v16, std::max<size_t>(v_total, 1) * sizeof(__half));
    if (e != cudaSuccess) {
        free_prepared(P);
        *msg = cudaGetErrorString(e);
        return G4A_CUDA;
    }
    // conversion launches by width group: the sources any width-512 problem
    // reads first, so that a launch never mixes the groups
    for (int wide = 1; wide >= 0; wide--) {
        std::vector<size_t> grp;
        for (size_t k = 0; k < v_src.size(); k++)
            if ((v_wide[k] != 0) == (wide != 0)) grp.push_back(k);
        for (size_t k0 = 0; k0 < grp.size(); k0 += kMaxSegs) {
            ConvSegs segs{};
            const int cnt = (int)std::min<size_t>(kMaxSegs, grp.size() - k0);
            uint64_t most = 0;
            for (int q = 0; q < cnt; q++) {
                const size_t k = grp[k0 + q];
                segs.src[q] = reinterpret_cast<const __nv_bfloat16 *>(v_src[k]);
                segs.dst[q] = P.v16 + v_off[k];
                segs.n8[q] = v_len[k] / 8;
                most = std::max(most, segs.n8[q]);
            }
            const unsigned bx = (unsigned)std::min<uint64_t>((most + 255) / 256, 1024);
            P.conv.push_back({segs, bx, cnt});
        }
        if (wide) P.n_conv_wide = P.conv.size();
    }
    if (S->persistent < 0) {
        const char *mode = getenv("G4A_PREFILL_KERNEL");  // measurement switch: "item" or "persistent"
        S->persistent = !(mode && std::strcmp(mode, "item") == 0);
        const char *keys = getenv("G4A_PREFILL_KEYS512");  // measurement switch: "64" or "128"
        S->keys512 = keys && std::strcmp(keys, "64") == 0 ? 64 : 128;
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&S->n_sm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || S->n_sm < 2)
            S->n_sm = 148;
    }
    std::vector<ProblemDev> hp(std::max(n, 1));
    std::vector<WorkItem> work[2];
    for (int32_t i = 0; i < n; i++) {
        const g4a_prefill_problem &p = pr[i];
        ProblemDev &d = hp[i];
        std::memset(&d, 0, sizeof d);
        const bool wide_tiles = S->persistent == 1 && p.head_dim == 512 && S->keys512 == 64;
        d.hd = p.head_dim;
        d.window = p.window;
        d.n_q = p.n_q;
        d.q_pos0 = p.q_pos0;
        d.n_kv = p.n_kv;
        d.kv_pos0 = p.kv_pos0;
        d.out = p.out_dev;
        d.lse = p.lse_dev;
        if (p.n_q == 0) continue;
        if (!cached_map(S, 0, p.q_dev, p.head_dim, (uint64_t)p.n_q * 8, &d.tq)) {
            *msg = "cuTensorMapEncodeTiled failed for Q";
            free_prepared(P);
            return G4A_CUDA;
        }
        if (!cached_map(S, 3, p.out_dev, p.head_dim, (uint64_t)p.n_q * 8, &d.to)) {
            *msg = "cuTensorMapEncodeTiled failed for the output";
            free_prepared(P);
            return G4A_CUDA;
        }
        if (p.n_kv > 0) {
            size_t k = std::find(v_src.begin(), v_src.end(), p.v_dev) - v_src.begin();
            if (!cached_map(S, 1, p.k_dev, p.head_dim, p.n_kv, &d.tk) ||
                !cached_map(S, 2, P.v16 + v_off[k], p.head_dim, p.n_kv, &d.tv) ||
                (wide_tiles && !cached_map(S, 4, p.k_dev, p.head_dim, p.n_kv, &d.tk32))) {
                *msg = "cuTensorMapEncodeTiled failed for K/V";
                free_prepared(P);
                return G4A_CUDA;
            }
        }
        const int n_qt = (p.n_q + kTokensPerPair - 1) / kTokensPerPair;
        // key tile of this problem's items: 64 keys for width 512 in the
        // persistent kernel when it runs 64-key tiles, else 128
        const int tile_keys = wide_tiles ? 64 : kKeysPerTile;
        for (int t = 0; t < n_qt; t++) {
            const int64_t q_lo = (int64_t)p.q_pos0 + (int64_t)t * kTokensPerPair;
            const int64_t q_hi = (int64_t)p.q_pos0 + std::min<int64_t>((int64_t)(t + 1) * kTokensPerPair, p.n_q) - 1;
            int64_t k_lo = p.window > 0 ? q_lo - p.window + 1 : 0;  // first key position any row may see
            int64_t klo = std::max<int64_t>(0, k_lo - p.kv_pos0);
            int64_t khi = std::min<int64_t>((int64_t)p.n_kv - 1, q_hi - p.kv_pos0);
            WorkItem w{};
            w.problem = i;
            w.q_tile = t;
            if (khi < klo) {
                w.kv_tile_lo = 0;
                w.n_kv_tiles = 0;
            } else {
                w.kv_tile_lo = (int32_t)(klo / tile_keys);
                w.n_kv_tiles = (int32_t)(khi / tile_keys) - w.kv_tile_lo + 1;
            }
            for (int h = 0; h < p.head_dim / kDV; h++) {
                w.dv_half = h;
                work[p.head_dim == 512].push_back(w);
            }
        }
    }
    // Largest work first: the block scheduler then fills SMs longest-first.
    // With both widths, one launch takes every item in one order, an item's
    // cost being its key tiles times 2 (width 256: S and PV of 256 columns)
    // or 3 (a 256-column half of width 512 recomputes the 512-wide S).
    for (auto &w : work)
        std::stable_sort(w.begin(), w.end(),
                         [](const WorkItem &a, const WorkItem &b) { return a.n_kv_tiles > b.n_kv_tiles; });
    const size_t n_items = work[0].size() + work[1].size();
    P.persistent = S->persistent == 1;
    P.keys512 = S->keys512;
    P.mixed = !P.persistent && !work[0].empty() && !work[1].empty();
    std::vector<int32_t> pair_start;
    if (P.persistent) {
        // Longest-processing-time assignment per width: an item costs its key
        // tiles times 4 (width 256: S and PV over 128 keys) or 3 per 64 keys
        // (a half of width 512, which recomputes the 512-wide S), plus 4 for
        // its Q load and epilogue;
        // items go longest first to the least loaded pair, and each pair's
        // list is stored in assignment order.
        for (int w = 0; w < 2; w++) {
            std::vector<WorkItem> &list = work[w];
            const int n_pairs =
                (int)std::min<size_t>(list.size(), (size_t)std::max(1, (S->n_sm - std::max(0, reserve_sms)) / 2));
            P.n_pairs[w] = n_pairs;
            const int base = (int)pair_start.size();
            pair_start.resize(base + n_pairs + 1, 0);
            if (n_pairs == 0) continue;
            const int tile_cost = w == 0 ? 4 : S->keys512 == 64 ? 3 : 6;
            auto cost = [&](const WorkItem &it) { return (int64_t)it.n_kv_tiles * tile_cost + 4; };
            std::vector<int64_t> load(n_pairs, 0);
            std::vector<int> owner(list.size());
            std::vector<int> count(n_pairs, 0);
            for (size_t k = 0; k < list.size(); k++) {  // list is longest first
                int best = 0;
                for (int q = 1; q < n_pairs; q++)
                    if (load[q] < load[best]) best = q;
                owner[k] = best;
                load[best] += cost(list[k]);
                count[best]++;
            }
            for (int q = 0; q < n_pairs; q++) pair_start[base + q + 1] = pair_start[base + q] + count[q];
            std::vector<int> fill(pair_start.begin() + base, pair_start.begin() + base + n_pairs);
            std::vector<WorkItem> ordered(list.size());
            for (size_t k = 0; k < list.size(); k++) ordered[fill[owner[k]]++] = list[k];
            list.swap(ordered);
        }
        if ((e = cudaMalloc(&P.d_pair_start, pair_start.size() * sizeof(int32_t))) != cudaSuccess ||
            (e = cudaMemcpyAsync(P.d_pair_start, pair_start.data(), pair_start.size() * sizeof(int32_t),
                                 cudaMemcpyHostToDevice, st)) != cudaSuccess) {
            free_prepared(P);
            *msg = cudaGetErrorString(e);
            return G4A_CUDA;
        }
    }
    if ((e = cudaMalloc(&P.d_problems, hp.size() * sizeof(ProblemDev))) != cudaSuccess ||
        (e = cudaMalloc(&P.d_items, std::max<size_t>(n_items, 1) * sizeof(WorkItem))) != cudaSuccess) {
        free_prepared(P);
        *msg = cudaGetErrorString(e);
        return G4A_CUDA;
    }
    std::vector<WorkItem> all(work[0]);
    all.insert(all.end(), work[1].begin(), work[1].end());
    if (P.mixed) {
        auto cost = [&](const WorkItem &w) { return w.n_kv_tiles * (hp[w.problem].hd == 512 ? 3 : 2); };
        std::stable_sort(all.begin(), all.end(), [&](const WorkItem &a, const WorkItem &b) { return cost(a) > cost(b); });
    }
    // stream-ordered uploads from pageable memory (staged by the driver before
    // the call returns)
    if ((e = cudaMemcpyAsync(P.d_problems, hp.data(), hp.size() * sizeof(ProblemDev), cudaMemcpyHostToDevice, st)) !=
            cudaSuccess ||
        (n_items && (e = cudaMemcpyAsync(P.d_items, all.data(), n_items * sizeof(WorkItem), cudaMemcpyHostToDevice,
                                         st)) != cudaSuccess)) {
        free_prepared(P);
        *msg = cudaGetErrorString(e);
        return G4A_CUDA;
    }
    P.n_work[0] = work[0].size();
    P.n_work[1] = work[1].size();
    P.key.assign(pr, pr + n);
    P.reserve = reserve_sms;
    P.used = S->calls;
    if ((e = launch_prepared(S, P, d_err, st, stall)) != cudaSuccess) {
        *msg = cudaGetErrorString(e);
        return G4A_CUDA;
    }
    return G4A_OK;
}

}  // namespace g4a
