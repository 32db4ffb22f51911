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
// Tiles: 64 rows x 64, 32 or 16 vectors per CTA (the widest that still
// gives two CTAs per SM; at most 32 for GEGLU's two matrices), 8 blocks (256
// columns) per stage, two CTAs per SM.
// Weights stay in the GGUF layout: a 2-D TMA box of 64 rows x 272 bytes (8
// blocks of [f16 scale, 32 quants]) per stage; activation quants come in two
// 128-byte-swizzled boxes of 128 bytes per vector, their f32 scales in a
// vectors x 8 box. Warp 8 issues the copies; warps 0-7 (4 along rows, 2
// along vectors) run the products and the block sums. All of a block's
// products are issued before its scaling, so their latency overlaps; the
// activation fragments come by ldmatrix from the swizzled rows, and the
// conversion and scaling run on pairs (sm_100 f32x2 instructions, each lane
// rounded as the scalar operation) ahead of scalar in-order sums, since the
// per-result f32 work is what bounds the kernel.
#include <cuda.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "../../include/g4attn.h"
#include "internal.h"
#include "libm_glibc.cuh"
#include "sm100_ptx.cuh"

namespace g4a {
namespace {

constexpr int kBM = 64, kKB = 8;              // rows, Q8_0 blocks per stage
constexpr int kMmaWarps = 8;                  // 4 (rows) x 2 (vectors)
constexpr int kGemmThreads = kMmaWarps * 32 + 32;
constexpr int kRowBytes = kKB * 34;           // 272: one row's 8 blocks
constexpr int kAStage = kBM * kRowBytes;      // 17,408
constexpr uint32_t kGemmWaitLimit = 1u << 24;
constexpr int kMagic = 0x4B400000;            // 1.5 * 2^23 as f32 bits

enum { KIND_PLAIN = 0, KIND_GEGLU = 1, KIND_SOFTCAP = 2 };

struct __align__(64) GemmParams {
    CUtensorMap ta, ta2, tb, ts;  // weights (u16 view), up weights (GEGLU), activation quants (u8), scales (f32)
    float *out;                   // [n_vec][rows]
    int64_t rows;
    int32_t n_vec, nb, kind, stages;
    float cap;
    int *err;
};

// Stage layout for a tile of BN vectors: [B: BN x 256 B, two 128-byte
// swizzled halves (1024-aligned)][A][A2][S: BN x 8 f32], padded to 1 KB.
__host__ __device__ constexpr int b_stage(int bn) { return bn * kKB * 32; }
__host__ __device__ constexpr int s_stage(int bn) { return bn * kKB * 4; }
__host__ __device__ constexpr int stage_bytes(int bn, int n_mat) {
    return ((b_stage(bn) + n_mat * kAStage + s_stage(bn)) + 1023) & ~1023;
}

__device__ __forceinline__ void gemm_wait(uint64_t *bar, uint32_t parity, int *err) {
    for (uint32_t i = 0; i < kGemmWaitLimit; i++)
        if (ptx::mbar_try_wait(bar, parity)) return;
    atomicOr(err, 2);
}

// d = a * b + magic: the exact block dot plus 1.5 * 2^23 in the low bits of
// an f32 pattern, so that (float)dot = as_float(d) - 1.5 * 2^23 exactly
// (|dot| <= 32 * 128 * 128 < 2^22), one subtraction instead of a conversion.
__device__ __forceinline__ void mma_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %10, %10, %10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(kMagic));
}
// Pairs of f32 in one 64-bit register for the sm_100 f32x2 instructions:
// each lane is an IEEE round-to-nearest operation, as the scalar one, at
// half the instruction count. Only multiplies and subtractions whose results
// feed no add are paired: a paired multiply-then-add may be contracted.
__device__ __forceinline__ uint64_t pk(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ uint64_t pki(int lo, int hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
    return r;
}
__device__ __forceinline__ float2 upk(uint64_t v) {
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
    return r;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t sub2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}

// Four 8 x 16-byte matrices from shared memory: lane l gives the address of
// row l % 8 of matrix l / 8 and receives bytes 4(l % 4)..+3 of row l / 4 of
// each, which is the B fragment of mma.m16n8k32 for the vector of that row.
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t (&r)[2], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(addr));
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

// ops.rs:85-89 and :79-81, glibc's tanh
__device__ __forceinline__ float gelu_tanh(float x) {
    const float inner = __fmul_rn(__fmul_rn(0.7978846f, x), __fadd_rn(1.0f, __fmul_rn(__fmul_rn(0.044715f, x), x)));
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, glibc::tanhf(inner)));
}
__device__ __forceinline__ float softcap(float v, float cap) {
    return __fmul_rn(glibc::tanhf(__fmul_rn(v, __fdiv_rn(1.0f, cap))), cap);
}

// NJ n8 tiles per warp: a CTA covers 64 rows x (16 * NJ) vectors; NMAT
// weight matrices (2: GEGLU's gate and up).
template <int NJ, int NMAT>
__global__ void __launch_bounds__(kGemmThreads, 2) q8_gemm_kernel(const __grid_constant__ GemmParams p) {
    constexpr int BN = 16 * NJ;
    constexpr int BST = b_stage(BN);
    extern __shared__ __align__(1024) uint8_t sm_raw[];
    // the swizzled boxes need 1024-byte aligned destinations
    uint8_t *sm = sm_raw + ((1024u - (ptx::smem_u32(sm_raw) & 1023u)) & 1023u);
    constexpr int n_mat = NMAT;
    const int sb = stage_bytes(BN, n_mat);
    uint64_t *full = reinterpret_cast<uint64_t *>(sm + (size_t)p.stages * sb);
    uint64_t *empty = full + p.stages;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int v0 = blockIdx.x * BN;
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
            const uint32_t bytes = (uint32_t)(BST + n_mat * kAStage + s_stage(BN));
            // The weights are constant: the first stages' weight boxes go out
            // before waiting for the grid that produced the activations.
            const int pre = n_kt < p.stages ? n_kt : p.stages;
            for (int k = 0; k < pre; k++) {
                uint8_t *st = sm + (size_t)k * sb;
                ptx::mbar_arrive_expect_tx(&full[k], bytes);
                ptx::tma_load_2d(st + BST, &p.ta, &full[k], k * kKB * 17, (int32_t)r0);
                if (n_mat == 2) ptx::tma_load_2d(st + BST + kAStage, &p.ta2, &full[k], k * kKB * 17, (int32_t)r0);
            }
            ptx::pdl_wait();
            for (int k = 0; k < n_kt; k++) {
                const int s = k % p.stages;
                uint8_t *st = sm + (size_t)s * sb;
                if (k >= pre) {
                    gemm_wait(&empty[s], ((uint32_t)(k / p.stages) & 1u) ^ 1u, p.err);
                    ptx::mbar_arrive_expect_tx(&full[s], bytes);
                    ptx::tma_load_2d(st + BST, &p.ta, &full[s], k * kKB * 17, (int32_t)r0);
                    if (n_mat == 2) ptx::tma_load_2d(st + BST + kAStage, &p.ta2, &full[s], k * kKB * 17, (int32_t)r0);
                }
                ptx::tma_load_2d(st, &p.tb, &full[s], k * kKB * 32, v0);
                ptx::tma_load_2d(st + BST / 2, &p.tb, &full[s], k * kKB * 32 + 128, v0);
                ptx::tma_load_2d(st + BST + n_mat * kAStage, &p.ts, &full[s], k * kKB, v0);
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
    // accumulators: [matrix][n8 tile][(row ra | ra + 8) x (vector 2t | 2t + 1)]
    float acc[NMAT][NJ][4];
    const uint64_t magic = pk(12582912.0f, 12582912.0f);
#pragma unroll
    for (int m = 0; m < NMAT; m++)
#pragma unroll
        for (int j = 0; j < NJ; j++)
#pragma unroll
            for (int e = 0; e < 4; e++) acc[m][j][e] = -0.0f;  // Rust's f32 Sum starts from -0.0
    // ldmatrix row of this lane: matrix lane / 8 (tile j + mm / 2, half mm % 2), row lane % 8
    const int mm = lane >> 3, rr = lane & 7;
    for (int k = 0; k < n_kt; k++) {
        const int s = k % p.stages;
        const uint8_t *st = sm + (size_t)s * sb;
        gemm_wait(&full[s], (uint32_t)(k / p.stages) & 1u, p.err);
        const float *xs = reinterpret_cast<const float *>(st + BST + n_mat * kAStage);
        const uint32_t bst = ptx::smem_u32(st);
        // fully unrolled (every offset an immediate) where the registers allow
        constexpr int kUnroll = NJ * NMAT >= 4 ? 4 : kKB;
#pragma unroll kUnroll
        for (int kb = 0; kb < kKB; kb++) {
            // activation fragments (ldmatrix from the swizzled rows) and scales
            uint32_t b[NJ][2];
            const int c = (kb & 3) * 2;
            const uint32_t half = bst + (kb >> 2) * (BST / 2);
            if constexpr (NJ == 1) {
                const int v = wn * 8 + rr;
                uint32_t r2[2];
                ldsm_x2(r2, half + v * 128 + (((c + (mm & 1)) ^ rr) << 4));
                b[0][0] = r2[0];
                b[0][1] = r2[1];
            } else {
#pragma unroll
                for (int j = 0; j < NJ; j += 2) {
                    const int v = wn * 8 * NJ + (j + (mm >> 1)) * 8 + rr;
                    uint32_t r4[4];
                    ldsm_x4(r4, half + v * 128 + (((c + (mm & 1)) ^ rr) << 4));
                    b[j][0] = r4[0];
                    b[j][1] = r4[1];
                    b[j + 1][0] = r4[2];
                    b[j + 1][1] = r4[3];
                }
            }
            uint64_t xsc[NJ];
#pragma unroll
            for (int j = 0; j < NJ; j++) {
                const int vo = wn * 8 * NJ + j * 8 + 2 * t;  // the vectors of this lane's results
                xsc[j] = pk(xs[vo * kKB + kb], xs[(vo + 1) * kKB + kb]);
            }
#pragma unroll
            for (int m = 0; m < NMAT; m++) {
                const uint8_t *row0 = st + BST + m * kAStage + (size_t)ra * kRowBytes;
                const uint8_t *row1 = row0 + 8 * kRowBytes;
                const int off = kb * 34;
                uint32_t a[4];
                a[0] = a_word(row0, off + 2 + 4 * t);
                a[1] = a_word(row1, off + 2 + 4 * t);
                a[2] = a_word(row0, off + 18 + 4 * t);
                a[3] = a_word(row1, off + 18 + 4 * t);
                const float ws0 = __half2float(*reinterpret_cast<const __half *>(row0 + off));
                const float ws1 = __half2float(*reinterpret_cast<const __half *>(row1 + off));
                const uint64_t w0 = pk(ws0, ws0), w1 = pk(ws1, ws1);
                int d[NJ][4];
#pragma unroll
                for (int j = 0; j < NJ; j++) mma_s8(d[j], a, b[j][0], b[j][1]);
                // d[j]: (row ra, vector 2t), (ra, 2t+1), (ra+8, 2t), (ra+8, 2t+1);
                // acc + (float)dot * (w_scale * x_scale), as dot_q8_0: the
                // conversion and both products on pairs, the sum scalar (a
                // paired multiply followed by a paired add may be fused into
                // one rounding; the scalar add.rn never is)
#pragma unroll
                for (int j = 0; j < NJ; j++) {
                    const float2 t0 = upk(mul2(sub2(pki(d[j][0], d[j][1]), magic), mul2(w0, xsc[j])));
                    const float2 t1 = upk(mul2(sub2(pki(d[j][2], d[j][3]), magic), mul2(w1, xsc[j])));
                    acc[m][j][0] = __fadd_rn(acc[m][j][0], t0.x);
                    acc[m][j][1] = __fadd_rn(acc[m][j][1], t0.y);
                    acc[m][j][2] = __fadd_rn(acc[m][j][2], t1.x);
                    acc[m][j][3] = __fadd_rn(acc[m][j][3], t1.y);
                }
            }
        }
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&empty[s]);
    }
    // results: out[v][r]
#pragma unroll
    for (int j = 0; j < NJ; j++)
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int64_t r = r0 + ra + h * 8;
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const int v = v0 + wn * 8 * NJ + j * 8 + 2 * t + e;
                if (r >= p.rows || v >= p.n_vec) continue;
                const float gate = acc[0][j][2 * h + e];
                float res = gate;
                if constexpr (NMAT == 2) res = __fmul_rn(gelu_tanh(gate), acc[NMAT - 1][j][2 * h + e]);
                else if (p.kind == KIND_SOFTCAP) res = softcap(gate, p.cap);
                p.out[(int64_t)v * p.rows + r] = res;
            }
        }
}

// The most stages (2-4) that leave room for two CTAs per SM.
int gemm_stages(int bn, int n_mat) {
    int st = 4;
    while (st > 2 && 1024 + (size_t)st * stage_bytes(bn, n_mat) + 64 > 113 * 1024) st--;
    return st;
}

template <int NJ, int NMAT>
cudaError_t gemm_launch(GemmParams &p, int64_t rows, int32_t n_vec, cudaStream_t st, bool pdl) {
    constexpr int BN = 16 * NJ;
    p.stages = gemm_stages(BN, NMAT);
    const size_t smem = 1024 + (size_t)p.stages * stage_bytes(BN, NMAT) + 2 * p.stages * sizeof(uint64_t);
    static bool attr_set = false;
    if (!attr_set) {
        cudaFuncSetAttribute(q8_gemm_kernel<NJ, NMAT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        attr_set = true;
    }
    const dim3 grid((unsigned)((n_vec + BN - 1) / BN), (unsigned)((rows + kBM - 1) / kBM));
    return launch_k(pdl, q8_gemm_kernel<NJ, NMAT>, grid, dim3(kGemmThreads), smem, st, p);
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
    // vector tile (64, 32 or 16 vectors): the least estimated time, waves of
    // two CTAs per SM times the tile's work over its relative efficiency
    // (wider tiles reuse each weight fragment for more vectors; measured on
    // the E2B shapes)
    const int64_t row_tiles = (rows + kBM - 1) / kBM;
    int nj = 1;
    double best = 1e300;
    for (int cand = n_mat == 2 ? 2 : 4; cand >= 1; cand >>= 1) {
        const double eff = cand == 4 ? 1.0 : cand == 2 ? 0.8 : 0.55;
        const int64_t ctas = row_tiles * ((n_vec + 16 * cand - 1) / (16 * cand));
        const double waves = (double)((ctas + 2 * 148 - 1) / (2 * 148));
        const double cost = waves * cand / eff;
        if (cost < best - 1e-9) best = cost, nj = cand;
    }
    GemmParams p;
    bool ok = encode_tmap_2d_raw(&p.ta, 2, w, (uint64_t)row_len / 2, (uint64_t)rows, (uint64_t)row_len, kKB * 17, kBM,
                                 false);
    if (n_mat == 2)
        ok = ok && encode_tmap_2d_raw(&p.ta2, 2, w2, (uint64_t)row_len / 2, (uint64_t)rows, (uint64_t)row_len, kKB * 17,
                                      kBM, false);
    else
        p.ta2 = p.ta;
    ok = ok && encode_tmap_2d_raw(&p.tb, 1, xq, (uint64_t)cols, (uint64_t)n_vec, (uint64_t)cols, 128, 16 * nj, true);
    ok = ok && encode_tmap_2d_raw(&p.ts, 4, xs, (uint64_t)nb, (uint64_t)n_vec, (uint64_t)nb * 4, kKB, 16 * nj, false);
    if (!ok) return cudaErrorInvalidValue;
    p.out = out;
    p.rows = rows;
    p.n_vec = n_vec;
    p.nb = (int32_t)nb;
    p.kind = kind;
    p.cap = cap;
    p.err = d_err;
    if (n_mat == 2) return nj == 2 ? gemm_launch<2, 2>(p, rows, n_vec, st, pdl) : gemm_launch<1, 2>(p, rows, n_vec, st, pdl);
    if (nj == 4) return gemm_launch<4, 1>(p, rows, n_vec, st, pdl);
    if (nj == 2) return gemm_launch<2, 1>(p, rows, n_vec, st, pdl);
    return gemm_launch<1, 1>(p, rows, n_vec, st, pdl);
}

}  // namespace g4a
