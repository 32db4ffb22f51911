// Q8_0 mat-vec on sm_100a: the projections that feed attention (and the FFN
// and output head) in the reference's default numerics, restated for the GPU:
//   * quantize_q8_0 (crates/llm-backend-cpu/src/matvec.rs:36-54): per block of
//     32 values, scale = max|x| / 127, stored as f16; quants = round-half-even
//     of x * (1 / scale), saturated to int8;
//   * dot_q8_0 (matvec.rs:137-150): per block an exact int32 dot product of
//     the weight and activation quants (dp4a), times (w_scale * x_scale), and
//     the block values summed over the row IN BLOCK ORDER starting from -0.0
//     (Rust's f32 Sum), so the result is the reference's bit for bit;
//   * matvec_q8_0 (:58-63), geglu_q8_0 with gelu_tanh (:88-103, ops.rs:85-89)
//     and matvec_q8_0_then with softcap (:67-80, ops.rs:79-81).
//
// Weights stay in the GGUF Q8_0 byte layout the reference reads (rows of
// cols/32 blocks of [f16 scale, 32 x int8]); nothing is repacked. The kernel
// streams them: persistent CTAs (several per SM) take tiles of consecutive
// rows (one contiguous span of bytes, about 16 KB) through a 4-stage ring of
// 1-D bulk copies, so the weights cross HBM once per call whatever the number
// of activation vectors (up to 8 per pass). Roles per CTA:
//   warps 0-7  every block's dot product and value, into a double-buffered
//              shared-memory table (one padded row per matrix row);
//   warp 8     the bulk copies;
//   warp 9     the in-order sums, one lane per (vector, row), overlapping the
//              next tile's dot products.
// Hand-offs are mbarriers (stage full / empty, table full / empty); no
// barrier spans the CTA inside the loop.
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdint>

#include "../../include/g4attn.h"
#include "internal.h"
#include "libm_glibc.cuh"
#include "sm100_ptx.cuh"

namespace g4a {
namespace {

constexpr int kQ8Block = 32;
constexpr int kQ8BlockBytes = 34;
constexpr int kMaxVec = 8;
constexpr int kStages = 4;
constexpr int kConsumers = 256;         // warps 0-7: block dot products
constexpr int kProducerWarp = 8;        // bulk copies
constexpr int kSumWarp = 9;             // in-order row sums
constexpr int kThreadsQ8 = kConsumers + 64;
constexpr uint32_t kQ8WaitLimit = 1u << 24;
constexpr int64_t kStageTarget = 16 * 1024;  // weight bytes per stage


enum { KIND_PLAIN = 0, KIND_GEGLU = 1, KIND_SOFTCAP = 2 };
constexpr int kMaxSeg = 3;

// ops.rs:85-89, left to right, no fused multiply-adds.
__device__ __forceinline__ float gelu_tanh(float x) {
    const float sqrt_2_over_pi = 0.7978846f, coef_a = 0.044715f;
    const float inner = __fmul_rn(__fmul_rn(sqrt_2_over_pi, x), __fadd_rn(1.0f, __fmul_rn(__fmul_rn(coef_a, x), x)));
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, glibc::tanhf(inner)));
}

// ops.rs:79-81
__device__ __forceinline__ float softcap(float v, float cap) {
    return __fmul_rn(glibc::tanhf(__fmul_rn(v, __fdiv_rn(1.0f, cap))), cap);
}

// One warp per block of 32 values: matvec.rs:36-54.
__global__ void __launch_bounds__(256) q8_quantize_kernel(const float *__restrict__ x, int64_t n_blocks,
                                                          float *__restrict__ scales, int8_t *__restrict__ quants) {
    ptx::pdl_trigger();
    ptx::pdl_wait();
    const int64_t b = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (b >= n_blocks) return;  // whole warps exit together
    const float v = x[b * kQ8Block + lane];
    float m = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float scale = __fdiv_rn(m, 127.0f);
    const float inverse = scale == 0.0f ? 0.0f : __fdiv_rn(1.0f, scale);
    float q = rintf(__fmul_rn(v, inverse));
    q = q != q ? 0.0f : fminf(fmaxf(q, -128.0f), 127.0f);  // Rust's saturating `as i8`
    quants[b * kQ8Block + lane] = (int8_t)(int)q;
    if (lane == 0) scales[b] = __half2float(__float2half_rn(scale));
}

struct Q8Params {
    const uint8_t *w;      // [rows][row_len] Q8_0 bytes
    const uint8_t *w2;     // second matrix (GEGLU up), same shape
    const int8_t *xq;      // [n_vec][cols] activation quants
    const float *xs;       // [n_vec][cols / 32] activation scales
    const float *xf;       // [n_vec][cols] f32 activations quantized in the prologue (then xq/xs unused)
    const float *pli;      // with xf: quantize gelu(xf) * the layer's per-layer input instead (model.rs:426-428)
    int32_t pli_stride;    // floats between consecutive vectors' per-layer inputs
    float *out;            // [n_vec][rows]
    int64_t rows;
    int32_t cols, row_len, n_vec, tile_rows, n_tiles, kind;
    float cap;
    int *err;
    // Up to three matrices of the same width over one input in one launch
    // (q, k, v): row tiles are numbered across them; segment i holds tiles
    // [seg_tile0[i], seg_tile0[i + 1]). Segment 0 is (w, rows, out).
    int32_t n_seg;
    const uint8_t *seg_w[kMaxSeg];
    float *seg_out[kMaxSeg];
    int64_t seg_rows[kMaxSeg];
    int32_t seg_tile0[kMaxSeg + 1];
};

// Block b of a row at `row` (shared memory, row start 16-byte aligned): the
// f16 scale and the 32 int8 quants as 8 words, from 9 aligned word reads.
__device__ __forceinline__ float load_block(const uint8_t *row, int b, uint32_t (&q)[8]) {
    const int off = b * kQ8BlockBytes;  // even
    const uint32_t *w = reinterpret_cast<const uint32_t *>(row + (off & ~3));
    uint32_t r[9];
#pragma unroll
    for (int k = 0; k < 9; k++) r[k] = w[k];
    // Odd blocks start 2 bytes into a word: the scale is the upper half of
    // word 0 and the quants are words 1-8; even blocks have the scale in the
    // lower half and the quants straddle words. Neighbouring lanes differ in
    // parity, so this is done without a branch: a clamped funnel shift by 32
    // returns the upper word, by 16 the straddling one.
    const uint32_t sh = (off & 2) ? 32u : 16u;
    const uint32_t sbits = (r[0] >> (sh - 16u)) & 0xffffu;
#pragma unroll
    for (int k = 0; k < 8; k++) q[k] = __funnelshift_rc(r[k], r[k + 1], sh);
    return __half2float(__ushort_as_half((unsigned short)sbits));
}

__device__ __forceinline__ float block_value(const uint32_t (&wq)[8], float ws, const int8_t *xq, float xs) {
    const uint4 x0 = reinterpret_cast<const uint4 *>(xq)[0], x1 = reinterpret_cast<const uint4 *>(xq)[1];
    const uint32_t x[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
    int dot = 0;
#pragma unroll
    for (int k = 0; k < 8; k++) dot = __dp4a((int)wq[k], (int)x[k], dot);
    return __fmul_rn(__int2float_rn(dot), __fmul_rn(ws, xs));  // exact dot (|dot| < 2^24)
}

// Activation quants in shared memory: 48 bytes per block of 32, read as two
// 16-byte loads; the eight lanes of a quarter warp then cover 32 distinct
// banks (block stride of 12 words).
constexpr int kXqStride = 48;

struct Q8Shared {
    uint64_t full[kStages], empty[kStages];  // weight stages: producer -> compute warps
    uint64_t vfull[2], vempty[2];            // block-value buffers: compute warps -> sum warp
};

// Shared-memory layout of one launch (host and device agree on it):
// ring [stages][n_mat][mat_bytes] | x quants [n_vec][nb][36 B] | x scales [n_vec][nb]
// | block values [2][n_mat][n_vec][tile_rows][nb + 1] f32 | barriers (16-byte aligned).
// The block-value rows are padded by one float so that the sum warp's lanes
// (one row each) read different banks.
struct Q8Layout {
    size_t mat_bytes, xq, xs, vals, vals_buf, bars, total;
    __host__ __device__ Q8Layout(int n_mat, int n_vec, int cols, int tile_rows) {
        const size_t nb = (size_t)cols / kQ8Block;
        mat_bytes = ((size_t)tile_rows * nb * kQ8BlockBytes + 127) & ~(size_t)127;
        xq = (size_t)kStages * n_mat * mat_bytes;
        xs = xq + (size_t)n_vec * nb * kXqStride;
        vals = xs + (size_t)n_vec * nb * 4;
        vals_buf = (size_t)n_mat * n_vec * tile_rows * (nb + 1);  // floats per buffer
        bars = (vals + 2 * vals_buf * 4 + 15) & ~(size_t)15;
        total = bars + sizeof(Q8Shared);
    }
};

// Bounded mbarrier wait; a time-out sets the error bit and returns (the
// caller goes on, so that every barrier still receives its arrivals).
__device__ __forceinline__ void q8_wait(uint64_t *bar, uint32_t parity, int *err) {
    for (uint32_t i = 0; i < kQ8WaitLimit; i++)
        if (ptx::mbar_try_wait(bar, parity)) return;
    atomicOr(err, 2);
}

__global__ void __launch_bounds__(kThreadsQ8, 3) q8_matvec_kernel(Q8Params p) {
    extern __shared__ __align__(128) uint8_t sm[];
    const int nb = p.cols / kQ8Block;
    const int nbp = nb + 1;
    const int n_mat = p.kind == KIND_GEGLU ? 2 : 1;
    const Q8Layout L(n_mat, p.n_vec, p.cols, p.tile_rows);
    uint8_t *ring = sm;
    int8_t *xq_s = reinterpret_cast<int8_t *>(sm + L.xq);
    float *xs_s = reinterpret_cast<float *>(sm + L.xs);
    float *val_s = reinterpret_cast<float *>(sm + L.vals);
    Q8Shared *bars = reinterpret_cast<Q8Shared *>(sm + L.bars);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) {
            ptx::mbar_init(&bars->full[s], 1);
            ptx::mbar_init(&bars->empty[s], kConsumers / 32);
        }
        for (int b = 0; b < 2; b++) {
            ptx::mbar_init(&bars->vfull[b], kConsumers / 32);
            ptx::mbar_init(&bars->vempty[b], 1);
        }
        ptx::fence_mbar_init();
    }
    __syncthreads();
    // The weights are constant: the producer starts streaming them at once,
    // even before the grid this one depends on has finished. Everything that
    // reads or writes the activations and outputs waits for it (the compute
    // warps below; the sum warp only after them).
    ptx::pdl_trigger();

    const int my_tiles = p.n_tiles > (int)blockIdx.x ? (p.n_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    // tile k of this CTA: its segment, first row and row count
    auto rows_of = [&](int k, int64_t *r0, int *seg) {
        const int t = (int)blockIdx.x + k * (int)gridDim.x;
        int sg = 0;
        while (sg + 1 < p.n_seg && t >= p.seg_tile0[sg + 1]) sg++;
        *seg = sg;
        *r0 = (int64_t)(t - p.seg_tile0[sg]) * p.tile_rows;
        const int64_t rows = p.seg_rows[sg];
        return (int)(rows - *r0 < p.tile_rows ? rows - *r0 : p.tile_rows);
    };

    if (warp == kProducerWarp) {
        // ---------------------------------------------------------------- producer
        if (lane == 0) {
            for (int k = 0; k < my_tiles; k++) {
                const int s = k % kStages;
                if (k >= kStages) q8_wait(&bars->empty[s], ((uint32_t)(k / kStages) & 1u) ^ 1u, p.err);
                int64_t r0;
                int sg;
                const int rows_here = rows_of(k, &r0, &sg);
                const uint32_t bytes = (uint32_t)rows_here * p.row_len;
                ptx::mbar_arrive_expect_tx(&bars->full[s], bytes * n_mat);
                ptx::bulk_load_1d(ring + (size_t)s * n_mat * L.mat_bytes, p.seg_w[sg] + r0 * p.row_len, bytes,
                                  &bars->full[s]);
                if (n_mat == 2)
                    ptx::bulk_load_1d(ring + (size_t)s * n_mat * L.mat_bytes + L.mat_bytes, p.w2 + r0 * p.row_len,
                                      bytes, &bars->full[s]);
            }
            // No copy may land after the CTA exits: wait (bounded) for the
            // last stages issued (normally long consumed already).
            for (int k = max(0, my_tiles - kStages); k < my_tiles; k++)
                q8_wait(&bars->full[k % kStages], (uint32_t)(k / kStages) & 1u, p.err);
        }
    } else if (warp == kSumWarp) {
        // ---------------------------------------------------------------- in-order sums
        // lane = (vector, row): the block values of the row in block order,
        // from -0.0 (Rust's f32 Sum), loads of each group of 8 issued first
        for (int k = 0; k < my_tiles; k++) {
            const int buf = k & 1;
            q8_wait(&bars->vfull[buf], (uint32_t)(k >> 1) & 1u, p.err);
            int64_t r0;
            int sg;
            const int rows_here = rows_of(k, &r0, &sg);
            const int64_t seg_rows = p.seg_rows[sg];
            float *seg_out = p.seg_out[sg];
            const float *vals_k = val_s + (size_t)buf * L.vals_buf;
            for (int e = lane; e < p.n_vec * rows_here; e += 32) {
                const int v = e / rows_here, r = e - v * rows_here;
                float sums[2];
                for (int m = 0; m < n_mat; m++) {
                    const float *vr = vals_k + (((size_t)m * p.n_vec + v) * p.tile_rows + r) * nbp;
                    float sum = -0.0f;
                    int b = 0;
                    for (; b + 8 <= nb; b += 8) {
                        float x[8];
#pragma unroll
                        for (int i = 0; i < 8; i++) x[i] = vr[b + i];
#pragma unroll
                        for (int i = 0; i < 8; i++) sum = __fadd_rn(sum, x[i]);
                    }
                    for (; b < nb; b++) sum = __fadd_rn(sum, vr[b]);
                    sums[m] = sum;
                }
                float res = sums[0];
                if (p.kind == KIND_GEGLU) res = __fmul_rn(gelu_tanh(sums[0]), sums[1]);
                else if (p.kind == KIND_SOFTCAP) res = softcap(sums[0], p.cap);
                seg_out[(size_t)v * seg_rows + r0 + r] = res;
            }
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(&bars->vempty[buf]);
        }
    } else {
        // ---------------------------------------------------------------- block dot products
        ptx::pdl_wait();
        if (p.xf) {
            // matvec.rs:36-54 on the f32 inputs, a float4 per thread: the 8
            // consecutive lanes of a block of 32 share its maximum
            const int total = p.n_vec * p.cols / 4;
            for (int base = warp * 32; base < total; base += kConsumers) {
                const int e = base + lane;
                const bool in = e < total;  // whole groups of 8 (cols a multiple of 32)
                float4 v = in ? __ldg(reinterpret_cast<const float4 *>(p.xf) + e) : make_float4(0.f, 0.f, 0.f, 0.f);
                if (p.pli && in) {  // the PLE gate: gelu(gate) * per-layer input
                    const int vec = e / (p.cols / 4), c4 = e - vec * (p.cols / 4);
                    const float4 g = __ldg(reinterpret_cast<const float4 *>(p.pli + (size_t)vec * p.pli_stride) + c4);
                    v.x = __fmul_rn(gelu_tanh(v.x), g.x);
                    v.y = __fmul_rn(gelu_tanh(v.y), g.y);
                    v.z = __fmul_rn(gelu_tanh(v.z), g.z);
                    v.w = __fmul_rn(gelu_tanh(v.w), g.w);
                }
                float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
                m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
                m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
                m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
                const float scale = __fdiv_rn(m, 127.0f);
                const float inverse = scale == 0.0f ? 0.0f : __fdiv_rn(1.0f, scale);
                auto q = [&](float x) {
                    float r = rintf(__fmul_rn(x, inverse));
                    r = r != r ? 0.0f : fminf(fmaxf(r, -128.0f), 127.0f);
                    return (uint32_t)(uint8_t)(int8_t)(int)r;
                };
                if (in) {
                    const int blk = e >> 3, k = e & 7;
                    reinterpret_cast<uint32_t *>(xq_s)[blk * (kXqStride / 4) + k] =
                        q(v.x) | (q(v.y) << 8) | (q(v.z) << 16) | (q(v.w) << 24);
                    if (k == 0) xs_s[blk] = __half2float(__float2half_rn(scale));
                }
            }
        } else {
            // activation quants (padded to 48 bytes per block) and scales, once per CTA
            for (int i = threadIdx.x; i < p.n_vec * p.cols / 4; i += kConsumers) {
                const int blk = i >> 3, k = i & 7;  // word k of block blk (over all vectors)
                reinterpret_cast<uint32_t *>(xq_s)[blk * (kXqStride / 4) + k] =
                    reinterpret_cast<const uint32_t *>(p.xq)[i];
            }
            for (int i = threadIdx.x; i < p.n_vec * nb; i += kConsumers) xs_s[i] = p.xs[i];
        }
        ptx::named_bar_sync(1, kConsumers);
        const int step_r = kConsumers / nb, step_b = kConsumers - (kConsumers / nb) * nb;  // 256 = step_r*nb + step_b
        // One vector and at most 256 blocks per row: thread t owns block column
        // t % nb for the whole call (its activation quants and scale live in
        // registers) and walks rows t / nb, + G, + 2G, ... (G = 256 / nb).
        const bool column_mode = p.n_vec == 1 && nb <= kConsumers;
        const int G = column_mode ? kConsumers / nb : 0;
        const int my_b = column_mode ? (int)threadIdx.x % nb : 0;
        const int my_g = column_mode ? (int)threadIdx.x / nb : 0;
        uint32_t xw[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        float my_xs = 0.0f;
        if (column_mode && my_g < G) {
            const uint4 x0 = reinterpret_cast<const uint4 *>(xq_s + (size_t)my_b * kXqStride)[0];
            const uint4 x1 = reinterpret_cast<const uint4 *>(xq_s + (size_t)my_b * kXqStride)[1];
            xw[0] = x0.x, xw[1] = x0.y, xw[2] = x0.z, xw[3] = x0.w, xw[4] = x1.x, xw[5] = x1.y, xw[6] = x1.z,
            xw[7] = x1.w;
            my_xs = xs_s[my_b];
        }
        for (int k = 0; k < my_tiles; k++) {
            const int s = k % kStages, buf = k & 1;
            q8_wait(&bars->full[s], (uint32_t)(k / kStages) & 1u, p.err);
            if (k >= 2) q8_wait(&bars->vempty[buf], (uint32_t)((k - 2) >> 1) & 1u, p.err);
            int64_t r0;
            int sg;
            const int rows_here = rows_of(k, &r0, &sg);
            const uint8_t *stage = ring + (size_t)s * n_mat * L.mat_bytes;
            float *vals_k = val_s + (size_t)buf * L.vals_buf;
            if (column_mode) {
                if (my_g < G) {
                    for (int m = 0; m < n_mat; m++) {
                        const uint8_t *wrow = stage + (size_t)m * L.mat_bytes + (size_t)my_g * p.row_len;
                        float *vout = vals_k + ((size_t)m * p.tile_rows + my_g) * nbp + my_b;
                        for (int r = my_g; r < rows_here; r += G) {
                            uint32_t wq[8];
                            const float ws = load_block(wrow, my_b, wq);
                            int dot = 0;
#pragma unroll
                            for (int k2 = 0; k2 < 8; k2++) dot = __dp4a((int)wq[k2], (int)xw[k2], dot);
                            *vout = __fmul_rn(__int2float_rn(dot), __fmul_rn(ws, my_xs));
                            wrow += (size_t)G * p.row_len;
                            vout += (size_t)G * nbp;
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) {
                    ptx::mbar_arrive(&bars->empty[s]);
                    ptx::mbar_arrive(&bars->vfull[buf]);
                }
                continue;
            }
            // (m, r, b) of element threadIdx.x + 256 j, stepped without divisions
            int m = 0, r = threadIdx.x / nb, b = threadIdx.x - (threadIdx.x / nb) * nb;
            while (r >= rows_here && m < n_mat) r -= rows_here, m++;
            while (m < n_mat) {
                uint32_t wq[8];
                const float ws = load_block(stage + (size_t)m * L.mat_bytes + (size_t)r * p.row_len, b, wq);
                for (int v = 0; v < p.n_vec; v++)
                    vals_k[(((size_t)m * p.n_vec + v) * p.tile_rows + r) * nbp + b] =
                        block_value(wq, ws, xq_s + ((size_t)v * nb + b) * kXqStride, xs_s[v * nb + b]);
                b += step_b;
                r += step_r;
                if (b >= nb) b -= nb, r++;
                while (r >= rows_here && m < n_mat) r -= rows_here, m++;
            }
            __syncwarp();
            if (lane == 0) {
                ptx::mbar_arrive(&bars->empty[s]);   // this warp no longer reads the stage
                ptx::mbar_arrive(&bars->vfull[buf]); // this warp's block values are written
            }
        }
    }
    __syncthreads();
}

// Rows whose byte length is not a multiple of 16 (cols not a multiple of
// 256): one warp per (vector, row), blocks read byte-wise from global memory,
// lane 0 adds the block values in order.
__global__ void __launch_bounds__(256) q8_matvec_generic_kernel(Q8Params p) {
    ptx::pdl_trigger();
    ptx::pdl_wait();
    const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (gw >= p.rows * p.n_vec) return;
    const int v = (int)(gw / p.rows);
    const int64_t row = gw - (int64_t)v * p.rows;
    const int nb = p.cols / kQ8Block;
    const int n_mat = p.kind == KIND_GEGLU ? 2 : 1;
    float sums[2] = {-0.0f, -0.0f};
    for (int m = 0; m < n_mat; m++) {
        const uint8_t *w = (m ? p.w2 : p.w) + row * p.row_len;
        for (int b0 = 0; b0 < nb; b0 += 32) {
            const int b = b0 + lane;
            float val = 0.0f;
            if (b < nb) {
                const uint8_t *blk = w + (size_t)b * kQ8BlockBytes;
                const float ws = __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
                const int8_t *xq = p.xq + (size_t)v * p.cols + b * kQ8Block;
                int dot = 0;
                for (int i = 0; i < kQ8Block; i++) dot += (int)(int8_t)blk[2 + i] * (int)xq[i];
                val = __fmul_rn(__int2float_rn(dot), __fmul_rn(ws, p.xs[(size_t)v * nb + b]));
            }
            const int n = min(32, nb - b0);
            for (int i = 0; i < n; i++) {
                const float x = __shfl_sync(0xffffffffu, val, i);
                if (lane == 0) sums[m] = __fadd_rn(sums[m], x);
            }
        }
    }
    if (lane == 0) {
        float r = sums[0];
        if (p.kind == KIND_GEGLU) r = __fmul_rn(gelu_tanh(sums[0]), sums[1]);
        else if (p.kind == KIND_SOFTCAP) r = softcap(sums[0], p.cap);
        p.out[(size_t)v * p.rows + row] = r;
    }
}

}  // namespace

// Quantizes x ([n_vec][cols] f32) into the caller's scratch, then runs the
// mat-vec of `kind` (0 plain, 1 GEGLU with w2, 2 soft-cap) into out
// ([n_vec][rows]). With x == nullptr the scratch already holds the quantized
// activations (several projections of one input). Returns a g4a_status;
// *msg names a failure.
int q8_run(int kind, const uint8_t *w, const uint8_t *w2, int64_t rows, int64_t cols, const float *x, int32_t n_vec,
           float cap, float *out, int8_t *xq, float *xs, int *d_err, int n_sm, cudaStream_t st, const char **msg,
           bool pdl, const float *pli, int32_t pli_stride, const Q8Seg *extra, int n_extra) {
    *msg = "";
    if (n_extra < 0 || n_extra > kMaxSeg - 1 || (n_extra && (kind != KIND_PLAIN || !extra))) {
        *msg = "invalid extra mat-vec segments";
        return G4A_COMPUTE;
    }
    const int64_t nb = cols / kQ8Block;
    const int64_t n_blocks = nb * n_vec;
    const int n_mat = kind == KIND_GEGLU ? 2 : 1;
    const int64_t row_len = nb * kQ8BlockBytes;
    const bool aligned = ((uintptr_t)w % 16 == 0) && (!w2 || (uintptr_t)w2 % 16 == 0) && ((uintptr_t)x % 16 == 0);
    const bool fast = rows > 0 && aligned && row_len % 16 == 0 && row_len * n_mat <= kStageTarget &&
                      Q8Layout(n_mat, 1, (int)cols, 1).total <= 227 * 1024;
    // One pass of the streaming kernel quantizes its own inputs; otherwise
    // (several passes, the generic kernel, or quantization alone) a separate
    // kernel fills xq/xs first.
    // Many vectors: the tensor-core kernel over quantized activations.
    const bool gemm = n_vec > kMaxVec && rows > 0 && q8_gemm_fits(kind, w, w2, rows, cols, xq, xs);
    const bool fused_quant = !gemm && x && fast && n_vec <= kMaxVec &&
                             Q8Layout(n_mat, n_vec, (int)cols, (int)std::max<int64_t>(1, std::min<int64_t>(
                                 32, kStageTarget / (row_len * n_mat)))).total <= 227 * 1024;
    if (x && n_blocks > 0 && !fused_quant) {
        const int64_t threads = n_blocks * 32;
        const cudaError_t e = launch_k(pdl, q8_quantize_kernel, dim3((unsigned)((threads + 255) / 256)), dim3(256), 0,
                                       st, x, n_blocks, xs, xq);
        if (e != cudaSuccess) {
            *msg = cudaGetErrorString(e);
            return G4A_CUDA;
        }
    }
    if (pli && !fused_quant) {
        *msg = "the gelu-gate input needs the single-pass streaming kernel";
        return G4A_COMPUTE;
    }
    if (n_extra && (!fast || gemm || n_vec > kMaxVec)) {
        *msg = "several matrices in one launch need the single-pass streaming kernel";
        return G4A_COMPUTE;
    }
    if (rows == 0) return cudaGetLastError() == cudaSuccess ? G4A_OK : G4A_CUDA;
    if (gemm) {
        const cudaError_t e = q8_gemm_run(kind, w, w2, rows, cols, xq, xs, n_vec, cap, out, d_err, st, pdl);
        if (e != cudaSuccess) {
            *msg = cudaGetErrorString(e);
            return G4A_CUDA;
        }
        return G4A_OK;
    }
    Q8Params p{};
    p.w = w;
    p.w2 = w2;
    p.rows = rows;
    p.cols = (int32_t)cols;
    p.row_len = (int32_t)row_len;
    p.kind = kind;
    p.cap = cap;
    p.err = d_err;
    if (!fast) {
        p.xq = xq;
        p.xs = xs;
        p.out = out;
        p.n_vec = n_vec;
        const int64_t threads = rows * n_vec * 32;
        const cudaError_t e = launch_k(pdl, q8_matvec_generic_kernel, dim3((unsigned)((threads + 255) / 256)),
                                       dim3(256), 0, st, p);
        if (e != cudaSuccess) {
            *msg = cudaGetErrorString(e);
            return G4A_CUDA;
        }
    } else {
        static bool attr_set = false;  // per process; the attribute is per function
        if (!attr_set) {
            cudaFuncSetAttribute(q8_matvec_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
            attr_set = true;
        }
        // rows per stage: as many as fit the stage target (about 16 KB, up to
        // 32 rows); several CTAs per SM keep enough copies in flight
        p.tile_rows = (int32_t)std::max<int64_t>(1, std::min<int64_t>(32, kStageTarget / (row_len * n_mat)));
        // segments: (w, rows, out) and the extra matrices, tiles numbered across them
        p.n_seg = 1 + n_extra;
        int64_t n_tiles = 0;
        for (int sg = 0; sg < p.n_seg; sg++) {
            const int64_t seg_rows = sg == 0 ? rows : extra[sg - 1].rows;
            p.seg_w[sg] = sg == 0 ? w : extra[sg - 1].w;
            p.seg_rows[sg] = seg_rows;
            p.seg_tile0[sg] = (int32_t)n_tiles;
            n_tiles += (seg_rows + p.tile_rows - 1) / p.tile_rows;
            if (sg > 0 && (!p.seg_w[sg] || (uintptr_t)p.seg_w[sg] % 16 || !extra[sg - 1].out || seg_rows <= 0)) {
                *msg = "invalid extra mat-vec segment";
                return G4A_COMPUTE;
            }
        }
        if (n_tiles > INT32_MAX) {
            *msg = "Q8_0 mat-vec too large";
            return G4A_COMPUTE;
        }
        p.seg_tile0[p.n_seg] = (int32_t)n_tiles;
        p.n_tiles = (int32_t)n_tiles;
        for (int32_t v0 = 0; v0 < n_vec;) {
            int g = std::min<int32_t>(kMaxVec, n_vec - v0);
            while (g > 1 && Q8Layout(n_mat, g, (int)cols, p.tile_rows).total > 227 * 1024) g--;
            if (Q8Layout(n_mat, g, (int)cols, p.tile_rows).total > 227 * 1024) {
                *msg = "Q8_0 row too wide for the streaming kernel";
                return G4A_COMPUTE;
            }
            p.n_vec = g;
            p.xq = xq + (size_t)v0 * cols;
            p.xs = xs + (size_t)v0 * nb;
            p.xf = fused_quant ? x + (size_t)v0 * cols : nullptr;
            p.pli = pli;
            p.pli_stride = pli_stride;
            p.out = out + (size_t)v0 * rows;
            for (int sg = 0; sg < p.n_seg; sg++)
                p.seg_out[sg] = (sg == 0 ? out : extra[sg - 1].out) + (size_t)v0 * p.seg_rows[sg];
            // as many resident CTAs per SM as shared memory allows (up to 4):
            // more warps hide the shared-memory latency of the block dots
            const size_t smem = Q8Layout(n_mat, g, (int)cols, p.tile_rows).total;
            int per_sm = 1;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, q8_matvec_kernel, kThreadsQ8, smem) != cudaSuccess ||
                per_sm < 1)
                per_sm = 1;
            const int grid = (int)std::min<int64_t>(n_tiles, (int64_t)std::max(1, n_sm) * std::min(per_sm, 4));
            const cudaError_t e = launch_k(pdl, q8_matvec_kernel, dim3(grid), dim3(kThreadsQ8), smem, st, p);
            if (e != cudaSuccess) {
                *msg = cudaGetErrorString(e);
                return G4A_CUDA;
            }
            v0 += g;
        }
    }
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        *msg = cudaGetErrorString(e);
        return G4A_CUDA;
    }
    return G4A_OK;
}

}  // namespace g4a
