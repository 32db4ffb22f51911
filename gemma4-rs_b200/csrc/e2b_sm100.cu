// Kernels of the E2B decoder step around attention and the Q8_0 mat-vecs
// (crates/llm-gemma4/src/impl_/model.rs:252-449): the token embedding, the
// per-layer embedding inputs, the residual adds fused with the RMSNorm that
// follows and with the Q8_0 quantization of the next projection's input, the
// PLE gate, the greedy argmax, the per-step attention plan, and a seeded
// generator of synthetic weights in the GGUF layout the reference reads.
//
// RMSNorm follows ops.rs:45-56: squares in f32, summed in f64 (a block
// reduction here instead of the reference's sequential sum; the f32 mean
// after the cast agrees unless the two f64 sums straddle an f32 rounding
// boundary), scale = 1 / sqrt(mean + eps) in f32, y = (x * scale) * w. The
// quantization is matvec.rs:36-54 as in the Q8_0 kernels. Every f32 step is
// a round-to-nearest intrinsic, never a fused multiply-add, and tanh is
// glibc's, so each value is the reference's bit for bit.
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#include <cstdint>

#include "internal.h"
#include "libm_glibc.cuh"

namespace g4a {
namespace {

constexpr int kQ8Block = 32;
constexpr int kQ8BlockBytes = 34;
constexpr int kRowThreads = 256;
constexpr int kMaxRow = 4096;  // widest row a fused row kernel holds in shared memory

// ---- synthetic weights ---------------------------------------------------

__device__ __forceinline__ uint64_t mix64(uint64_t z) {  // splitmix64 finaliser
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// A standard normal from one counter (Box-Muller on two 24-bit uniforms).
__device__ __forceinline__ float normal_at(uint64_t seed, uint64_t tensor, uint64_t index) {
    const uint64_t h = mix64(seed ^ mix64(tensor * 0x100000001B3ull + index));
    const float u1 = ((float)(uint32_t)(h >> 40) + 1.0f) * (1.0f / 16777216.0f);  // (0, 1]
    const float u2 = (float)(uint32_t)(h & 0xFFFFFFu) * (1.0f / 16777216.0f);       // [0, 1)
    return sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
}

// Q8_0 blocks of N(0, sigma) values, quantized as the reference's test
// fixture quantizes weights (crates/llm-backend-cpu/tests/matvec.rs:21-31):
// scale = max|w| / 127 stored as f16, q = round-half-away(w / scale).
__global__ void synth_q8_kernel(uint8_t *dst, int64_t n_blocks, uint64_t seed, uint64_t tensor, float sigma) {
    const int64_t blk = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (blk >= n_blocks) return;  // whole warps
    const float w = sigma * normal_at(seed, tensor, (uint64_t)blk * kQ8Block + lane);
    float m = fabsf(w);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float scale = m / 127.0f;
    float q = roundf(w / scale);
    q = q != q ? 0.0f : fminf(fmaxf(q, -128.0f), 127.0f);
    // The block's 34 bytes as 17 little-endian halfwords (the block start is
    // 2-byte aligned): halfword 0 the f16 scale, halfword k the quants of
    // lanes 2k-2 and 2k-1.
    const uint32_t qb = (uint32_t)(uint8_t)(int8_t)(int)q;
    const uint32_t hi = __shfl_down_sync(0xffffffffu, qb, 1);
    uint16_t *h = reinterpret_cast<uint16_t *>(dst + blk * kQ8BlockBytes);
    if ((lane & 1) == 0) h[1 + lane / 2] = (uint16_t)(qb | (hi << 8));
    if (lane == 0) h[0] = __half_as_ushort(__float2half_rn(scale));
}

// Norm scales: center + spread * N(0, 1), rounded to bf16 (stored as f32,
// as the reference widens BF16 norm tensors).
__global__ void synth_norm_kernel(float *dst, int64_t n, uint64_t seed, uint64_t tensor, float center, float spread) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float v = center + spread * normal_at(seed, tensor, (uint64_t)i);
    dst[i] = __bfloat162float(__float2bfloat16_rn(v));
}

// ---- row helpers (one CTA per sequence row) -------------------------------

__device__ __forceinline__ double block_sum_f64(double v, double *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();  // red may still be read by a previous call
    if (lane == 0) red[warp] = v;
    __syncthreads();
    double t = 0.0;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) t += red[i];
    return t;
}

// ops.rs:45-56 scale of a row (every thread returns it)
__device__ __forceinline__ float rms_scale(const float *x, int n, float eps, double *red) {
    double ss = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss += (double)__fmul_rn(x[i], x[i]);
    const double sum = block_sum_f64(ss, red);
    const float mean = (float)(sum / (double)n);
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
}

// matvec.rs:36-54 on a row in shared memory, a warp per block of 32
__device__ __forceinline__ void quantize_row(const float *a, int n, int8_t *xq, float *xs) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int b = warp; b < n / kQ8Block; b += nw) {
        const float v = a[b * kQ8Block + lane];
        float m = fabsf(v);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        const float scale = __fdiv_rn(m, 127.0f);
        const float inverse = scale == 0.0f ? 0.0f : __fdiv_rn(1.0f, scale);
        float q = rintf(__fmul_rn(v, inverse));
        q = q != q ? 0.0f : fminf(fmaxf(q, -128.0f), 127.0f);  // Rust's saturating `as i8`
        xq[b * kQ8Block + lane] = (int8_t)(int)q;
        if (lane == 0) xs[b] = __half2float(__float2half_rn(scale));
    }
}

__device__ __forceinline__ float q8_elem(const uint8_t *row, int64_t e) {  // dequant.rs:13-24
    const uint8_t *blk = row + (e / kQ8Block) * kQ8BlockBytes;
    const float sc = __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
    return __fmul_rn((float)(int8_t)blk[2 + e % kQ8Block], sc);
}

// ---- decoder step kernels ---------------------------------------------------

// model.rs:376-384: the token's embedding row times sqrt(d_model)
__global__ void embed_kernel(const uint8_t *__restrict__ table, int d, const int32_t *__restrict__ tokens, float scale,
                             float *__restrict__ x) {
    const int s = blockIdx.x;
    const uint8_t *row = table + (int64_t)tokens[s] * (d / kQ8Block) * kQ8BlockBytes;
    for (int i = threadIdx.x; i < d; i += blockDim.x) x[(int64_t)s * d + i] = __fmul_rn(q8_elem(row, i), scale);
}

// model.rs:252-270: per layer slice of `ple` values,
// (rms_norm(P * ps, w) + table[token] * ts) * is
__global__ void ple_inputs_kernel(const float *__restrict__ P, const uint8_t *__restrict__ table,
                                  const int32_t *__restrict__ tokens, const float *__restrict__ w, int L, int ple,
                                  float ps, float ts, float is, float eps, float *__restrict__ out) {
    __shared__ double red[32];
    __shared__ float scaled[1024];
    const int s = blockIdx.x / L, l = blockIdx.x % L;
    const int64_t width = (int64_t)L * ple;
    const float *p = P + (int64_t)s * width + (int64_t)l * ple;
    for (int i = threadIdx.x; i < ple; i += blockDim.x) scaled[i] = __fmul_rn(p[i], ps);
    __syncthreads();
    const float sc = rms_scale(scaled, ple, eps, red);
    const uint8_t *row = table + (int64_t)tokens[s] * (width / kQ8Block) * kQ8BlockBytes;
    for (int i = threadIdx.x; i < ple; i += blockDim.x) {
        const int64_t e = (int64_t)l * ple + i;
        const float normed = __fmul_rn(__fmul_rn(scaled[i], sc), w[i]);
        out[(int64_t)s * width + e] = __fmul_rn(__fadd_rn(normed, __fmul_rn(q8_elem(row, e), ts)), is);
    }
}

// The residual step of the layer and the input of the next projection:
//   y given:   x = (x + rms_norm(y, w_post)) [* post]   (model.rs:412-413,
//              419-420, 430-435)
//   then:      a = w_next ? rms_norm(x, w_next) : x      (:392, :415, :438)
//              xq, xs = quantize_q8_0(a)
struct ResidArgs {
    float *x;
    const float *y, *w_post, *w_next;
    int8_t *xq;
    float *xs;
    int d;
    float eps, post;
};

__global__ void __launch_bounds__(kRowThreads) resid_kernel(ResidArgs a) {
    __shared__ double red[32];
    __shared__ float v[kMaxRow];
    const int s = blockIdx.x, d = a.d;
    float *xr = a.x + (int64_t)s * d;
    if (a.y) {
        const float *yr = a.y + (int64_t)s * d;
        const float sc = rms_scale(yr, d, a.eps, red);
        for (int i = threadIdx.x; i < d; i += blockDim.x) {
            float t = __fadd_rn(xr[i], __fmul_rn(__fmul_rn(yr[i], sc), a.w_post[i]));
            if (a.post != 1.0f) t = __fmul_rn(t, a.post);
            v[i] = t;
            xr[i] = t;
        }
    } else {
        for (int i = threadIdx.x; i < d; i += blockDim.x) v[i] = xr[i];
    }
    __syncthreads();
    if (a.w_next) {
        const float sc = rms_scale(v, d, a.eps, red);
        for (int i = threadIdx.x; i < d; i += blockDim.x) v[i] = __fmul_rn(__fmul_rn(v[i], sc), a.w_next[i]);
        __syncthreads();
    }
    quantize_row(v, d, a.xq + (int64_t)s * d, a.xs + (int64_t)s * (d / kQ8Block));
}

// ops.rs:85-89 gelu_tanh, left to right without fused multiply-adds
__device__ __forceinline__ float gelu_tanh(float x) {
    const float inner = __fmul_rn(__fmul_rn(0.7978846f, x), __fadd_rn(1.0f, __fmul_rn(__fmul_rn(0.044715f, x), x)));
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, glibc::tanhf(inner)));
}

// model.rs:426-428: gelu(gate) * this layer's per-layer input, quantized for
// the `proj` mat-vec
__global__ void __launch_bounds__(kRowThreads) gelu_quant_kernel(const float *__restrict__ gate,
                                                                 const float *__restrict__ pli, int layer, int L,
                                                                 int ple, int8_t *xq, float *xs) {
    __shared__ float v[1024];
    const int s = blockIdx.x;
    for (int i = threadIdx.x; i < ple; i += blockDim.x)
        v[i] = __fmul_rn(gelu_tanh(gate[(int64_t)s * ple + i]), pli[((int64_t)s * L + layer) * ple + i]);
    __syncthreads();
    quantize_row(v, ple, xq + (int64_t)s * ple, xs + (int64_t)s * (ple / kQ8Block));
}

// Greedy sampling (crates/llm-eng/src/sample.rs:27-36): the maximum under
// f32::total_cmp, the last index among equal maxima (Iterator::max_by). The
// total order as an unsigned key, packed above the index, so one unsigned
// maximum decides both.
__device__ __forceinline__ uint32_t total_key(float f) {
    int32_t b = __float_as_int(f);
    b ^= (int32_t)(((uint32_t)(b >> 31)) >> 1);
    return (uint32_t)b ^ 0x80000000u;
}

__global__ void __launch_bounds__(1024) argmax_kernel(const float *__restrict__ logits, int64_t vocab,
                                                      int32_t *__restrict__ out) {
    __shared__ unsigned long long best_s[32];
    const float *row = logits + (int64_t)blockIdx.x * vocab;
    unsigned long long best = 0;
    for (int64_t i = threadIdx.x; i < vocab; i += blockDim.x) {
        const unsigned long long packed = ((unsigned long long)total_key(row[i]) << 32) | (unsigned long long)i;
        best = packed > best ? packed : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
    }
    if ((threadIdx.x & 31) == 0) best_s[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int i = 1; i < (int)(blockDim.x >> 5); i++) best = best_s[i] > best ? best_s[i] : best;
        out[blockIdx.x] = (int32_t)(best & 0xFFFFFFFFull);
    }
}

// The attention tasks of one step, on the device so that a captured step
// replays at any position: task (layer l, row i) attends sequence seqs[i] at
// position pos[i] over the cache of l's source layer (eng/mod.rs:71-90),
// rows [pos + 1 - window, pos + 1) on sliding layers and [0, pos + 1) on
// global ones (eng/mod.rs:10-36), appending row pos on owner layers. Items
// split each task's rows in pieces of rows_per_item; unused item slots get
// task -1 (the kernel returns at once for them).
__global__ void e2b_plan_kernel(E2bPlanArgs a) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    const int n_tasks = a.n_layers * a.n;
    if (t < n_tasks) {
        const int l = t / a.n, i = t % a.n;
        const E2bLayerDesc &ld = a.layers[l];
        const int pos = a.pos[i], seq = a.seqs[i];
        const int hi = pos + 1, lo = ld.global ? 0 : max(0, hi - a.window);
        DecodeTask tk{};
        const size_t cache_row0 = (size_t)seq * a.max_tokens * ld.hd;
        tk.k_base = ld.k_cache + cache_row0;
        tk.v_base = ld.v_cache + cache_row0;
        tk.q_raw = a.q + (size_t)i * kHeads * ld.hd;
        tk.k_raw = ld.owner ? a.k + (size_t)i * ld.hd : nullptr;
        tk.v_raw = ld.owner ? a.v + (size_t)i * ld.hd : nullptr;
        tk.q_w = ld.q_w;
        tk.k_w = ld.k_w;
        tk.out = a.att + (size_t)i * kHeads * ld.hd;
        tk.seq = seq;
        tk.position = pos;
        tk.lo = lo;
        tk.hi = hi;
        tk.new_row = ld.owner ? pos : -1;
        tk.n_splits = (hi - lo + a.rows_per_item - 1) / a.rows_per_item;
        tk.partial_base = i * (ld.global ? a.max_splits_global : a.max_splits_local);
        tk.global = ld.global;
        tk.q_ready = 0;
        tk.scale = 1.0f;  // model.rs:409
        tk.hd = ld.hd;
        a.tasks[(size_t)l * a.task_stride + i] = tk;
        return;
    }
    const int u = t - n_tasks;
    const int n_local = a.n * a.max_splits_local, n_global = a.n * a.max_splits_global;
    if (u >= n_local + n_global) return;
    const bool global = u >= n_local;
    const int ms = global ? a.max_splits_global : a.max_splits_local;
    const int v = global ? u - n_local : u;
    const int i = v / ms, s = v % ms;
    const int hi = a.pos[i] + 1, lo = global ? 0 : max(0, hi - a.window);
    const int r0 = lo + s * a.rows_per_item;
    DecodeItem it;
    it.task = r0 < hi ? i : -1;
    it.split = s;
    it.row_lo = r0;
    it.row_hi = min(hi, r0 + a.rows_per_item);
    (global ? a.items_global : a.items_local)[v] = it;
}

}  // namespace

// ---- launchers -------------------------------------------------------------

cudaError_t e2b_synth_q8(void *dst, int64_t n_blocks, uint64_t seed, uint64_t tensor, float sigma, cudaStream_t st) {
    if (n_blocks == 0) return cudaSuccess;
    synth_q8_kernel<<<(unsigned)((n_blocks * 32 + 255) / 256), 256, 0, st>>>(static_cast<uint8_t *>(dst), n_blocks,
                                                                          seed, tensor, sigma);
    return cudaGetLastError();
}

cudaError_t e2b_synth_norm(float *dst, int64_t n, uint64_t seed, uint64_t tensor, float center, float spread,
                           cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    synth_norm_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(dst, n, seed, tensor, center, spread);
    return cudaGetLastError();
}

cudaError_t e2b_embed(const uint8_t *table, int d, const int32_t *tokens, int n, float scale, float *x, cudaStream_t st) {
    embed_kernel<<<n, kRowThreads, 0, st>>>(table, d, tokens, scale, x);
    return cudaGetLastError();
}

cudaError_t e2b_ple_inputs(const float *P, const uint8_t *table, const int32_t *tokens, const float *w, int L, int ple,
                           float ps, float ts, float is, float eps, float *out, int n, cudaStream_t st) {
    if (ple > 1024) return cudaErrorInvalidValue;
    ple_inputs_kernel<<<n * L, kRowThreads, 0, st>>>(P, table, tokens, w, L, ple, ps, ts, is, eps, out);
    return cudaGetLastError();
}

cudaError_t e2b_resid(float *x, const float *y, const float *w_post, float post, const float *w_next, int d, float eps,
                      int8_t *xq, float *xs, int n, cudaStream_t st) {
    if (d > kMaxRow || d % kQ8Block) return cudaErrorInvalidValue;
    ResidArgs a{x, y, w_post, w_next, xq, xs, d, eps, post};
    resid_kernel<<<n, kRowThreads, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t e2b_gelu_quant(const float *gate, const float *pli, int layer, int L, int ple, int8_t *xq, float *xs, int n,
                           cudaStream_t st) {
    if (ple > 1024 || ple % kQ8Block) return cudaErrorInvalidValue;
    gelu_quant_kernel<<<n, kRowThreads, 0, st>>>(gate, pli, layer, L, ple, xq, xs);
    return cudaGetLastError();
}

cudaError_t e2b_argmax(const float *logits, int64_t vocab, int n, int32_t *out, cudaStream_t st) {
    argmax_kernel<<<n, 1024, 0, st>>>(logits, vocab, out);
    return cudaGetLastError();
}

cudaError_t e2b_plan(const E2bPlanArgs &a, cudaStream_t st) {
    const int total = a.n_layers * a.n + a.n * (a.max_splits_local + a.max_splits_global);
    if (total == 0) return cudaSuccess;
    e2b_plan_kernel<<<(total + 255) / 256, 256, 0, st>>>(a);
    return cudaGetLastError();
}

}  // namespace g4a
