// Q8_0 mat-vec for many activation vectors at once (the batched decoder's
// projections), with the reference's results bit for bit
// (crates/llm-backend-cpu/src/matvec.rs:137-150 dot_q8_0 per vector):
//   out[v][r] = sum over blocks b, in block order from -0.0, of
//               (float)dot_i32(wq[r][b], xq[v][b]) * (ws[r][b] * xs[v][b]).
//
// One block of 32 int8 products is exactly the K = 32 of the int8 tensor-core
// instruction mma.sync.m16n8k32.s8.s8.s32, so each instruction yields the
// exact block dot products of a 16-row x 8-vector tile; the scaling and the
// ordered sum follow in registers, block after block. That per-block f32
// work (five operations per result, against one instruction per 128 results
// for the products) bounds the kernel whatever the tensor unit, so the
// register-accumulator form is used rather than TMEM accumulators, which
// would add a TMEM read per block on the same path.
//
// Tiles: 64 rows x 64 vectors per CTA, 8 blocks (256 columns) per stage.
// Weights stay in the GGUF layout: a 2-D TMA box of 64 rows x 272 bytes (8
// blocks of [f16 scale, 32 quants]) per stage; activation quants come in two
// 128-byte-swizzled boxes of 64 vectors x 128 bytes, their f32 scales in a
// 64 x 8 box. Warp 8 issues the copies; warps 0-7 (4 along rows, 2 along
// vectors, a 16 x 32 tile each) run the products and the block sums.
#include <cuda.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "../../include/g4attn.h"
#include "internal.h"
#include "libm_glibc.cuh"
#include "sm100_ptx.cuh"

namespace g4a {
namespace {

constexpr int kBM = 64, kBN = 64, kKB = 8;    // rows, vectors, Q8_0 blocks per stage
constexpr int kMmaWarps = 8;                  // 4 (rows) x 2 (vectors)
constexpr int kGemmThreads = kMmaWarps * 32 + 32;
constexpr int kRowBytes = kKB * 34;           // 272: one row's 8 blocks
constexpr int kAStage = kBM * kRowBytes;      // 17,408
constexpr int kBStage = kBN * kKB * 32;       // 16,384: two swizzled halves of 64 x 128 B
constexpr int kSStage = kBN * kKB * 4;        // 2,048
constexpr uint32_t kGemmWaitLimit = 1u << 24;

enum { KIND_PLAIN = 0, KIND_GEGLU = 1, KIND_SOFTCAP = 2 };

struct __align__(64) GemmParams {
    CUtensorMap ta, ta2, tb, ts;  // weights (u16 view), up weights (GEGLU), activation quants (u8), scales (f32)
    float *out;                   // [n_vec][rows]
    int64_t rows;
    int32_t n_vec, nb, kind, stages;
    float cap;
    int *err;
};

__device__ __forceinline__ void gemm_wait(uint64_t *bar, uint32_t parity, int *err) {
    for (uint32_t i = 0; i < kGemmWaitLimit; i++)
        if (ptx::mbar_try_wait(bar, parity)) return;
    atomicOr(err, 2);
}

__device__ __forceinline__ void mma_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %10, %10, %10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
}

// Four quant bytes of a weight row at byte offset `off` of its stage row
// (off = 2 mod 4 for even blocks: two aligned words and a funnel shift).
__device__ __forceinline__ uint32_t a_word(const uint8_t *row, int off) {
    if (off & 2) {
        const uint32_t *w = reinterpret_cast<const uint32_t *>(row + (off - 2));
        return __funnelshift_r(w[0], w[1], 16);
    }
    return *reinterpret_cast<const uint32_t *>(row + off);
}

// (float)i exactly for |i| < 2^22 (a block dot is at most 32 * 128 * 128)
__device__ __forceinline__ float i2f_exact(int i) {
    return __fsub_rn(__int_as_float(0x4B400000 + i), 12582912.0f);
}

// ops.rs:85-89 and :79-81, glibc's tanh
__device__ __forceinline__ float gelu_tanh(float x) {
    const float inner = __fmul_rn(__fmul_rn(0.7978846f, x), __fadd_rn(1.0f, __fmul_rn(__fmul_rn(0.044715f, x), x)));
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, glibc::tanhf(inner)));
}
__device__ __forceinline__ float softcap(float v, float cap) {
    return __fmul_rn(glibc::tanhf(__fmul_rn(v, __fdiv_rn(1.0f, cap))), cap);
}

__global__ void __launch_bounds__(kGemmThreads, 1) q8_gemm_kernel(const __grid_constant__ GemmParams p) {
    extern __shared__ __align__(1024) uint8_t sm_raw[];
    // the swizzled boxes need 1024-byte aligned destinations
    uint8_t *sm = sm_raw + ((1024u - (ptx::smem_u32(sm_raw) & 1023u)) & 1023u);
    const int n_mat = p.kind == KIND_GEGLU ? 2 : 1;
    // stage: [B 16 KB (1024-aligned for the swizzle)][A][A2][S], padded to 1 KB
    const int stage_bytes = ((kBStage + n_mat * kAStage + kSStage) + 1023) & ~1023;
    uint64_t *full = reinterpret_cast<uint64_t *>(sm + (size_t)p.stages * stage_bytes);
    uint64_t *empty = full + p.stages;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int v0 = blockIdx.x * kBN;
    const int64_t r0 = (int64_t)blockIdx.y * kBM;
    const int n_kt = p.nb / kKB;

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.stages; s++) {
            ptx::mbar_init(&full[s], 1);
            ptx::mbar_init(&empty[s], kMmaWarps);
        }
        ptx::fence_mbar_init();
    }
    __syncthreads();
    ptx::pdl_trigger();

    if (warp == kMmaWarps) {
        // ------------------------------------------------------------ copies
        if (lane == 0) {
            const uint32_t bytes = (uint32_t)(kBStage + n_mat * kAStage + kSStage);
            // The weights are constant: the first stages' weight boxes go out
            // before waiting for the grid that produced the activations.
            const int pre = n_kt < p.stages ? n_kt : p.stages;
            for (int k = 0; k < pre; k++) {
                uint8_t *st = sm + (size_t)k * stage_bytes;
                ptx::mbar_arrive_expect_tx(&full[k], bytes);
                ptx::tma_load_2d(st + kBStage, &p.ta, &full[k], k * kKB * 17, (int32_t)r0);
                if (n_mat == 2) ptx::tma_load_2d(st + kBStage + kAStage, &p.ta2, &full[k], k * kKB * 17, (int32_t)r0);
            }
            ptx::pdl_wait();
            for (int k = 0; k < n_kt; k++) {
                const int s = k % p.stages;
                uint8_t *st = sm + (size_t)s * stage_bytes;
                if (k >= pre) {
                    gemm_wait(&empty[s], ((uint32_t)(k / p.stages) & 1u) ^ 1u, p.err);
                    ptx::mbar_arrive_expect_tx(&full[s], bytes);
                    ptx::tma_load_2d(st + kBStage, &p.ta, &full[s], k * kKB * 17, (int32_t)r0);
                    if (n_mat == 2)
                        ptx::tma_load_2d(st + kBStage + kAStage, &p.ta2, &full[s], k * kKB * 17, (int32_t)r0);
                }
                ptx::tma_load_2d(st, &p.tb, &full[s], k * kKB * 32, v0);
                ptx::tma_load_2d(st + kBStage / 2, &p.tb, &full[s], k * kKB * 32 + 128, v0);
                ptx::tma_load_2d(st + kBStage + n_mat * kAStage, &p.ts, &full[s], k * kKB, v0);
            }
            // no copy may land after the CTA exits
            for (int k = n_kt - p.stages < 0 ? 0 : n_kt - p.stages; k < n_kt; k++)
                gemm_wait(&full[k % p.stages], (uint32_t)(k / p.stages) & 1u, p.err);
        }
        return;
    }
    // ---------------------------------------------------------------- products
    const int wm = warp & 3, wn = warp >> 2;
    const int g = lane >> 2, t = lane & 3;
    const int ra = wm * 16 + g;  // this thread's rows in the tile: ra, ra + 8
    float acc[2][4][4];          // [matrix][n8 tile][fragment element]
#pragma unroll
    for (int m = 0; m < 2; m++)
#pragma unroll
        for (int j = 0; j < 4; j++)
#pragma unroll
            for (int e = 0; e < 4; e++) acc[m][j][e] = -0.0f;  // Rust's f32 Sum starts from -0.0
    for (int k = 0; k < n_kt; k++) {
        const int s = k % p.stages;
        const uint8_t *st = sm + (size_t)s * stage_bytes;
        gemm_wait(&full[s], (uint32_t)(k / p.stages) & 1u, p.err);
        const uint8_t *bq = st;
        const float *xs = reinterpret_cast<const float *>(st + kBStage + n_mat * kAStage);
#pragma unroll 2
        for (int kb = 0; kb < kKB; kb++) {
            // activation fragments and scales of the four n8 tiles
            uint32_t b[4][2];
            float xsc[4][2];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int v = wn * 32 + j * 8 + g;  // the vector this lane feeds to the product
                const uint8_t *row = bq + (kb >> 2) * (kBStage / 2) + v * 128;
                const int c = (kb & 3) * 2;
                b[j][0] = *reinterpret_cast<const uint32_t *>(row + (((c) ^ (v & 7)) << 4) + 4 * t);
                b[j][1] = *reinterpret_cast<const uint32_t *>(row + (((c + 1) ^ (v & 7)) << 4) + 4 * t);
                const int vo = wn * 32 + j * 8 + 2 * t;  // the vectors of this lane's results
                xsc[j][0] = xs[vo * kKB + kb];
                xsc[j][1] = xs[(vo + 1) * kKB + kb];
            }
#pragma unroll
            for (int m = 0; m < 2; m++) {
                if (m == n_mat) break;
                const uint8_t *A = st + kBStage + m * kAStage;
                const uint8_t *row0 = A + (size_t)ra * kRowBytes, *row1 = row0 + 8 * kRowBytes;
                const int off = kb * 34;
                uint32_t a[4];
                a[0] = a_word(row0, off + 2 + 4 * t);
                a[1] = a_word(row1, off + 2 + 4 * t);
                a[2] = a_word(row0, off + 18 + 4 * t);
                a[3] = a_word(row1, off + 18 + 4 * t);
                const float ws0 = __half2float(*reinterpret_cast<const __half *>(row0 + off));
                const float ws1 = __half2float(*reinterpret_cast<const __half *>(row1 + off));
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    int d[4];
                    mma_s8(d, a, b[j][0], b[j][1]);
                    // d: (row ra, vector 2t), (ra, 2t+1), (ra+8, 2t), (ra+8, 2t+1)
                    acc[m][j][0] = __fadd_rn(acc[m][j][0], __fmul_rn(i2f_exact(d[0]), __fmul_rn(ws0, xsc[j][0])));
                    acc[m][j][1] = __fadd_rn(acc[m][j][1], __fmul_rn(i2f_exact(d[1]), __fmul_rn(ws0, xsc[j][1])));
                    acc[m][j][2] = __fadd_rn(acc[m][j][2], __fmul_rn(i2f_exact(d[2]), __fmul_rn(ws1, xsc[j][0])));
                    acc[m][j][3] = __fadd_rn(acc[m][j][3], __fmul_rn(i2f_exact(d[3]), __fmul_rn(ws1, xsc[j][1])));
                }
            }
        }
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&empty[s]);
    }
    // results: out[v][r]
#pragma unroll
    for (int j = 0; j < 4; j++)
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const int64_t r = r0 + ra + (e >> 1) * 8;
            const int v = v0 + wn * 32 + j * 8 + 2 * t + (e & 1);
            if (r >= p.rows || v >= p.n_vec) continue;
            float res = acc[0][j][e];
            if (p.kind == KIND_GEGLU) res = __fmul_rn(gelu_tanh(acc[0][j][e]), acc[1][j][e]);
            else if (p.kind == KIND_SOFTCAP) res = softcap(res, p.cap);
            p.out[(int64_t)v * p.rows + r] = res;
        }
}

size_t gemm_smem(int n_mat, int stages) {
    const size_t stage_bytes = ((kBStage + n_mat * kAStage + kSStage) + 1023) & ~(size_t)1023;
    return 1024 + stages * stage_bytes + 2 * stages * sizeof(uint64_t);  // + alignment slack
}

}  // namespace

bool q8_gemm_fits(int kind, const uint8_t *w, const uint8_t *w2, int64_t rows, int64_t cols, const int8_t *xq,
                  const float *xs) {
    return rows > 0 && cols > 0 && cols % (kKB * 32) == 0 && (uintptr_t)w % 16 == 0 &&
           (kind != KIND_GEGLU || (w2 && (uintptr_t)w2 % 16 == 0)) && (uintptr_t)xq % 16 == 0 &&
           (uintptr_t)xs % 16 == 0 && rows <= (int64_t)kBM * 65535;
}

cudaError_t q8_gemm_run(int kind, const uint8_t *w, const uint8_t *w2, int64_t rows, int64_t cols, const int8_t *xq,
                        const float *xs, int32_t n_vec, float cap, float *out, int *d_err, cudaStream_t st, bool pdl) {
    const int n_mat = kind == KIND_GEGLU ? 2 : 1;
    const int64_t nb = cols / 32, row_len = nb * 34;
    GemmParams p;
    bool ok = encode_tmap_2d_raw(&p.ta, 2, w, (uint64_t)row_len / 2, (uint64_t)rows, (uint64_t)row_len, kKB * 17, kBM,
                                 false);
    if (n_mat == 2)
        ok = ok && encode_tmap_2d_raw(&p.ta2, 2, w2, (uint64_t)row_len / 2, (uint64_t)rows, (uint64_t)row_len, kKB * 17,
                                      kBM, false);
    else
        p.ta2 = p.ta;
    ok = ok && encode_tmap_2d_raw(&p.tb, 1, xq, (uint64_t)cols, (uint64_t)n_vec, (uint64_t)cols, 128, kBN, true);
    ok = ok && encode_tmap_2d_raw(&p.ts, 4, xs, (uint64_t)nb, (uint64_t)n_vec, (uint64_t)nb * 4, kKB, kBN, false);
    if (!ok) return cudaErrorInvalidValue;
    p.out = out;
    p.rows = rows;
    p.n_vec = n_vec;
    p.nb = (int32_t)nb;
    p.kind = kind;
    p.cap = cap;
    p.err = d_err;
    p.stages = n_mat == 2 ? 3 : 4;
    const size_t smem = gemm_smem(n_mat, p.stages);
    static bool attr_set = false;
    if (!attr_set) {
        cudaFuncSetAttribute(q8_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        attr_set = true;
    }
    const dim3 grid((unsigned)((n_vec + kBN - 1) / kBN), (unsigned)((rows + kBM - 1) / kBM));
    return launch_k(pdl, q8_gemm_kernel, grid, dim3(kGemmThreads), smem, st, p);
}

}  // namespace g4a
