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
// streams them: persistent CTAs take tiles of consecutive rows (one
// contiguous span of bytes) through a 4-stage ring of 1-D bulk copies, so the
// weights cross HBM once per call whatever the number of activation vectors
// (up to 8 per pass). Warps 0-7 compute every block value of a tile into
// shared memory; then one thread per (vector, row) adds them in order.
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdint>

#include "../../include/g4attn.h"
#include "internal.h"
#include "sm100_ptx.cuh"

namespace g4a {
namespace {

constexpr int kQ8Block = 32;
constexpr int kQ8BlockBytes = 34;
constexpr int kMaxVec = 8;
constexpr int kStages = 4;
constexpr int kStageBytes = 32 * 1024;  // per stage (split between the matrices of a GEGLU)
constexpr int kConsumers = 256;         // warps 0-7
constexpr int kThreadsQ8 = kConsumers + 32;
constexpr uint32_t kQ8WaitLimit = 1u << 24;

enum { KIND_PLAIN = 0, KIND_GEGLU = 1, KIND_SOFTCAP = 2 };

// ops.rs:85-89, left to right, no fused multiply-adds.
__device__ __forceinline__ float gelu_tanh(float x) {
    const float sqrt_2_over_pi = 0.7978846f, coef_a = 0.044715f;
    const float inner = __fmul_rn(__fmul_rn(sqrt_2_over_pi, x), __fadd_rn(1.0f, __fmul_rn(__fmul_rn(coef_a, x), x)));
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(inner)));
}

// ops.rs:79-81
__device__ __forceinline__ float softcap(float v, float cap) {
    return __fmul_rn(tanhf(__fmul_rn(v, __fdiv_rn(1.0f, cap))), cap);
}

// One warp per block of 32 values: matvec.rs:36-54.
__global__ void __launch_bounds__(256) q8_quantize_kernel(const float *__restrict__ x, int64_t n_blocks,
                                                          float *__restrict__ scales, int8_t *__restrict__ quants) {
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
    float *out;            // [n_vec][rows]
    int64_t rows;
    int32_t cols, row_len, n_vec, tile_rows, n_tiles, kind;
    float cap;
    int *err;
};

// Block b of a row at `row` (shared memory, row start 16-byte aligned): the
// f16 scale and the 32 int8 quants as 8 words, from 9 aligned word reads.
__device__ __forceinline__ float load_block(const uint8_t *row, int b, uint32_t (&q)[8]) {
    const int off = b * kQ8BlockBytes;  // even
    const uint32_t *w = reinterpret_cast<const uint32_t *>(row + (off & ~3));
    uint32_t r[9];
#pragma unroll
    for (int k = 0; k < 9; k++) r[k] = w[k];
    uint32_t sbits;
    if (off & 2) {  // scale in the upper half of word 0, quants aligned from word 1
        sbits = r[0] >> 16;
#pragma unroll
        for (int k = 0; k < 8; k++) q[k] = r[k + 1];
    } else {        // scale in the lower half, quants start two bytes into word 0
        sbits = r[0] & 0xffffu;
#pragma unroll
        for (int k = 0; k < 8; k++) q[k] = __funnelshift_r(r[k], r[k + 1], 16);
    }
    return __half2float(__ushort_as_half((unsigned short)sbits));
}

__device__ __forceinline__ float block_value(const uint32_t (&wq)[8], float ws, const int8_t *xq, float xs) {
    const uint32_t *x = reinterpret_cast<const uint32_t *>(xq);
    int dot = 0;
#pragma unroll
    for (int k = 0; k < 8; k++) dot = __dp4a((int)wq[k], (int)x[k], dot);
    return __fmul_rn(__int2float_rn(dot), __fmul_rn(ws, xs));  // exact dot (|dot| < 2^24)
}

struct Q8Shared {
    uint64_t full[kStages], empty[kStages];
    int bad;
};

// Shared-memory layout of one launch (host and device agree on it):
// ring [stages][n_mat][mat_bytes] | x quants [n_vec][cols] | x scales [n_vec][nb]
// | block values [n_mat][n_vec][tile_rows][nb] f32 | barriers (8-byte aligned).
struct Q8Layout {
    size_t mat_bytes, xq, xs, vals, bars, total;
    __host__ __device__ Q8Layout(int n_mat, int n_vec, int cols, int tile_rows) {
        const size_t nb = (size_t)cols / kQ8Block;
        mat_bytes = (size_t)kStageBytes / n_mat;
        xq = (size_t)kStages * n_mat * mat_bytes;
        xs = xq + (size_t)n_vec * cols;
        vals = xs + (size_t)n_vec * nb * 4;
        bars = (vals + (size_t)n_mat * n_vec * tile_rows * nb * 4 + 15) & ~(size_t)15;
        total = bars + sizeof(Q8Shared);
    }
};

__global__ void __launch_bounds__(kThreadsQ8, 1) q8_matvec_kernel(Q8Params p) {
    extern __shared__ __align__(128) uint8_t sm[];
    const int nb = p.cols / kQ8Block;
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
            ptx::mbar_init(&bars->empty[s], 1);
        }
        bars->bad = 0;
        ptx::fence_mbar_init();
    }
    // activation quants and scales, once per CTA
    for (int i = threadIdx.x; i < p.n_vec * p.cols / 16; i += blockDim.x)
        reinterpret_cast<uint4 *>(xq_s)[i] = reinterpret_cast<const uint4 *>(p.xq)[i];
    for (int i = threadIdx.x; i < p.n_vec * nb; i += blockDim.x) xs_s[i] = p.xs[i];
    __syncthreads();

    const int my_tiles = p.n_tiles > (int)blockIdx.x ? (p.n_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    if (warp == kConsumers / 32) {
        // ---------------------------------------------------------------- producer
        if (lane == 0) {
            int issued = 0;
            for (int k = 0; k < my_tiles; k++) {
                const int s = k % kStages;
                const uint32_t ph = (uint32_t)(k / kStages) & 1u;
                bool ok = true;
                if (k >= kStages) {
                    uint32_t i = 0;
                    while (!ptx::mbar_try_wait(&bars->empty[s], ph ^ 1u) && ++i < kQ8WaitLimit) {
                    }
                    ok = i < kQ8WaitLimit;
                }
                if (!ok) {
                    atomicOr(p.err, 2);
                    break;
                }
                const int64_t t = (int64_t)blockIdx.x + (int64_t)k * gridDim.x;
                const int64_t r0 = t * p.tile_rows;
                const int rows_here = (int)(p.rows - r0 < p.tile_rows ? p.rows - r0 : p.tile_rows);
                const uint32_t bytes = (uint32_t)rows_here * p.row_len;
                ptx::mbar_arrive_expect_tx(&bars->full[s], bytes * n_mat);
                ptx::bulk_load_1d(ring + (size_t)s * n_mat * L.mat_bytes, p.w + r0 * p.row_len, bytes, &bars->full[s]);
                if (n_mat == 2)
                    ptx::bulk_load_1d(ring + (size_t)s * n_mat * L.mat_bytes + L.mat_bytes, p.w2 + r0 * p.row_len,
                                      bytes, &bars->full[s]);
                issued = k + 1;
            }
            // No copy may land after the CTA exits: wait (bounded) for the
            // last stages issued (normally long consumed already).
            for (int k = max(0, issued - kStages); k < issued; k++)
                for (uint32_t i = 0;
                     i < kQ8WaitLimit && !ptx::mbar_try_wait(&bars->full[k % kStages], (uint32_t)(k / kStages) & 1u); i++) {
                }
        }
    } else {
        // ---------------------------------------------------------------- consumers
        for (int k = 0; k < my_tiles; k++) {
            const int s = k % kStages;
            const uint32_t ph = (uint32_t)(k / kStages) & 1u;
            uint32_t i = 0;
            while (!ptx::mbar_try_wait(&bars->full[s], ph) && ++i < kQ8WaitLimit) {
            }
            if (i >= kQ8WaitLimit) atomicOr(&bars->bad, 1);
            ptx::named_bar_sync(1, kConsumers);  // consumers only: the producer warp never joins
            if (*(volatile int *)&bars->bad) {
                if (threadIdx.x == 0) atomicOr(p.err, 2);
                break;
            }
            const int64_t t = (int64_t)blockIdx.x + (int64_t)k * gridDim.x;
            const int64_t r0 = t * p.tile_rows;
            const int rows_here = (int)(p.rows - r0 < p.tile_rows ? p.rows - r0 : p.tile_rows);
            const uint8_t *stage = ring + (size_t)s * n_mat * L.mat_bytes;
            // every (matrix, row, block): its value for every vector
            const int n_blocks = n_mat * rows_here * nb;
            for (int e = threadIdx.x; e < n_blocks; e += kConsumers) {
                const int m = e / (rows_here * nb);
                const int rb = e - m * rows_here * nb;
                const int r = rb / nb, b = rb - r * nb;
                uint32_t wq[8];
                const float ws = load_block(stage + (size_t)m * L.mat_bytes + (size_t)r * p.row_len, b, wq);
                for (int v = 0; v < p.n_vec; v++)
                    val_s[(((size_t)m * p.n_vec + v) * p.tile_rows + r) * nb + b] =
                        block_value(wq, ws, xq_s + (size_t)v * p.cols + b * kQ8Block, xs_s[v * nb + b]);
            }
            ptx::named_bar_sync(1, kConsumers);
            // the stage's bytes are no longer read: hand it back to the producer
            if (threadIdx.x == 0) ptx::mbar_arrive(&bars->empty[s]);
            // one thread per (vector, row): the blocks in order, from -0.0
            for (int e = threadIdx.x; e < p.n_vec * rows_here; e += kConsumers) {
                const int v = e / rows_here, r = e - v * rows_here;
                const float *vals = val_s + ((size_t)v * p.tile_rows + r) * nb;
                float sum = -0.0f;
                for (int b = 0; b < nb; b++) sum = __fadd_rn(sum, vals[b]);
                if (p.kind == KIND_GEGLU) {
                    const float *vals2 = val_s + (((size_t)p.n_vec + v) * p.tile_rows + r) * nb;
                    float sum2 = -0.0f;
                    for (int b = 0; b < nb; b++) sum2 = __fadd_rn(sum2, vals2[b]);
                    sum = __fmul_rn(gelu_tanh(sum), sum2);
                } else if (p.kind == KIND_SOFTCAP) {
                    sum = softcap(sum, p.cap);
                }
                p.out[(size_t)v * p.rows + r0 + r] = sum;
            }
            ptx::named_bar_sync(1, kConsumers);  // val_s is rewritten by the next tile
        }
    }
    __syncthreads();
}

// Rows whose byte length is not a multiple of 16 (cols not a multiple of
// 256): one warp per (vector, row), blocks read byte-wise from global memory,
// lane 0 adds the block values in order.
__global__ void __launch_bounds__(256) q8_matvec_generic_kernel(Q8Params p) {
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
// ([n_vec][rows]). Returns a g4a_status; *msg names a failure.
int q8_run(int kind, const uint8_t *w, const uint8_t *w2, int64_t rows, int64_t cols, const float *x, int32_t n_vec,
           float cap, float *out, int8_t *xq, float *xs, int *d_err, int n_sm, cudaStream_t st, const char **msg) {
    *msg = "";
    const int64_t nb = cols / kQ8Block;
    const int64_t n_blocks = nb * n_vec;
    if (n_blocks > 0) {
        const int64_t threads = n_blocks * 32;
        q8_quantize_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(x, n_blocks, xs, xq);
    }
    if (rows == 0) return cudaGetLastError() == cudaSuccess ? G4A_OK : G4A_CUDA;
    const int n_mat = kind == KIND_GEGLU ? 2 : 1;
    const int64_t row_len = nb * kQ8BlockBytes;
    const bool aligned = ((uintptr_t)w % 16 == 0) && (!w2 || (uintptr_t)w2 % 16 == 0);
    const bool fast = aligned && row_len % 16 == 0 && row_len <= kStageBytes / n_mat;
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
        q8_matvec_generic_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(p);
    } else {
        static bool attr_set = false;  // per process; the attribute is per function
        if (!attr_set) {
            cudaFuncSetAttribute(q8_matvec_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
            attr_set = true;
        }
        p.tile_rows = (int32_t)std::max<int64_t>(1, std::min<int64_t>(32, (kStageBytes / n_mat) / row_len));
        const int64_t n_tiles = (rows + p.tile_rows - 1) / p.tile_rows;
        if (n_tiles > INT32_MAX) {
            *msg = "Q8_0 mat-vec too large";
            return G4A_COMPUTE;
        }
        p.n_tiles = (int32_t)n_tiles;
        const int grid = (int)std::min<int64_t>(n_tiles, std::max(1, n_sm));
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
            p.out = out + (size_t)v0 * rows;
            q8_matvec_kernel<<<grid, kThreadsQ8, Q8Layout(n_mat, g, (int)cols, p.tile_rows).total, st>>>(p);
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
