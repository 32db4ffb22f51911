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
#include "sm100_ptx.cuh"

namespace g4a {
namespace {

constexpr int kQ8Block = 32;
constexpr int kQ8BlockBytes = 34;
constexpr int kRowThreads = 256;
constexpr int kMaxRow = 4096;  // widest row of the fused row kernels (one float4 per thread)

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

__device__ __forceinline__ float q8_elem(const uint8_t *row, int64_t e) {  // dequant.rs:13-24
    const uint8_t *blk = row + (e / kQ8Block) * kQ8BlockBytes;
    const float sc = __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
    return __fmul_rn((float)(int8_t)blk[2 + e % kQ8Block], sc);
}

// ---- decoder step kernels ---------------------------------------------------

// model.rs:376-384: the token's embedding row times sqrt(d_model)
__global__ void embed_kernel(const uint8_t *__restrict__ table, int d, const int32_t *__restrict__ tokens, float scale,
                             float *__restrict__ x) {
    ptx::pdl_trigger();  // a dependent may launch; it waits for this grid itself
    ptx::pdl_wait();
    const int s = blockIdx.x;
    const uint8_t *row = table + (int64_t)tokens[s] * (d / kQ8Block) * kQ8BlockBytes;
    for (int i = threadIdx.x; i < d; i += blockDim.x) x[(int64_t)s * d + i] = __fmul_rn(q8_elem(row, i), scale);
}

// model.rs:252-270: per layer slice of `ple` values,
// (rms_norm(P * ps, w) + table[token] * ts) * is
__global__ void ple_inputs_kernel(const float *__restrict__ P, const uint8_t *__restrict__ table,
                                  const int32_t *__restrict__ tokens, const float *__restrict__ w, int L, int ple,
                                  float ps, float ts, float is, float eps, float *__restrict__ out) {
    ptx::pdl_trigger();  // a dependent may launch; it waits for this grid itself
    ptx::pdl_wait();
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

// matvec.rs:36-54 for the four values a thread holds; the 8 consecutive
// threads of a block of 32 share its maximum through shuffles.
__device__ __forceinline__ void quant4(float4 v, int t, bool on, int8_t *xq_row, float *xs_row) {
    float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
    const float scale = __fdiv_rn(m, 127.0f);
    const float inverse = scale == 0.0f ? 0.0f : __fdiv_rn(1.0f, scale);
    auto q = [&](float x) {
        float r = rintf(__fmul_rn(x, inverse));
        r = r != r ? 0.0f : fminf(fmaxf(r, -128.0f), 127.0f);  // Rust's saturating `as i8`
        return (uint32_t)(uint8_t)(int8_t)(int)r;
    };
    if (!on) return;  // a whole group of 8 past the row's end (d a multiple of 32)
    reinterpret_cast<uint32_t *>(xq_row)[t] = q(v.x) | (q(v.y) << 8) | (q(v.z) << 16) | (q(v.w) << 24);
    if ((t & 7) == 0) xs_row[t >> 3] = __half2float(__float2half_rn(scale));
}

__device__ __forceinline__ double sq4(float4 v) {  // the f32 squares, widened and summed in f64
    double s = (double)__fmul_rn(v.x, v.x);
    s += (double)__fmul_rn(v.y, v.y);
    s += (double)__fmul_rn(v.z, v.z);
    s += (double)__fmul_rn(v.w, v.w);
    return s;
}

__device__ __forceinline__ float scale_of(double sum, int n, float eps) {  // ops.rs:50-51
    const float mean = (float)(sum / (double)n);
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
}

// One CTA per row, one float4 per thread (d / 4 threads, rounded up to
// whole warps): no loops, two block reductions at most.
__global__ void __launch_bounds__(1024) resid_kernel(ResidArgs a) {
    ptx::pdl_trigger();  // a dependent may launch; it waits for this grid itself
    ptx::pdl_wait();
    __shared__ double red[32];
    const int s = blockIdx.x, d = a.d, t = threadIdx.x;
    const bool on = 4 * t < d;
    float4 *xr = reinterpret_cast<float4 *>(a.x + (int64_t)s * d);
    const float4 zero = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    float4 v;
    if (a.y) {
        const float4 y = on ? __ldg(reinterpret_cast<const float4 *>(a.y + (int64_t)s * d) + t) : zero;
        const float4 x = on ? xr[t] : zero;
        const float4 w = on ? __ldg(reinterpret_cast<const float4 *>(a.w_post) + t) : zero;
        const float sc = scale_of(block_sum_f64(sq4(y), red), d, a.eps);
        v.x = __fadd_rn(x.x, __fmul_rn(__fmul_rn(y.x, sc), w.x));
        v.y = __fadd_rn(x.y, __fmul_rn(__fmul_rn(y.y, sc), w.y));
        v.z = __fadd_rn(x.z, __fmul_rn(__fmul_rn(y.z, sc), w.z));
        v.w = __fadd_rn(x.w, __fmul_rn(__fmul_rn(y.w, sc), w.w));
        if (a.post != 1.0f) {
            v.x = __fmul_rn(v.x, a.post);
            v.y = __fmul_rn(v.y, a.post);
            v.z = __fmul_rn(v.z, a.post);
            v.w = __fmul_rn(v.w, a.post);
        }
        if (on) xr[t] = v;
    } else {
        v = on ? xr[t] : zero;
    }
    if (a.w_next) {
        const float4 w = on ? __ldg(reinterpret_cast<const float4 *>(a.w_next) + t) : zero;
        const float sc = scale_of(block_sum_f64(sq4(v), red), d, a.eps);
        v.x = __fmul_rn(__fmul_rn(v.x, sc), w.x);
        v.y = __fmul_rn(__fmul_rn(v.y, sc), w.y);
        v.z = __fmul_rn(__fmul_rn(v.z, sc), w.z);
        v.w = __fmul_rn(__fmul_rn(v.w, sc), w.w);
    }
    quant4(v, t, on, a.xq + (int64_t)s * d, a.xs + (int64_t)s * (d / kQ8Block));
}

// ops.rs:85-89 gelu_tanh, left to right without fused multiply-adds
__device__ __forceinline__ float gelu_tanh(float x) {
    const float inner = __fmul_rn(__fmul_rn(0.7978846f, x), __fadd_rn(1.0f, __fmul_rn(__fmul_rn(0.044715f, x), x)));
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, glibc::tanhf(inner)));
}

// model.rs:426-428: gelu(gate) * this layer's per-layer input, quantized for
// the `proj` mat-vec; one float4 per thread
__global__ void __launch_bounds__(256) gelu_quant_kernel(const float *__restrict__ gate, const float *__restrict__ pli,
                                                         int layer, int L, int ple, int8_t *xq, float *xs) {
    ptx::pdl_trigger();  // a dependent may launch; it waits for this grid itself
    ptx::pdl_wait();
    const int s = blockIdx.x, t = threadIdx.x;
    const float4 g = __ldg(reinterpret_cast<const float4 *>(gate + (int64_t)s * ple) + t);
    const float4 e = __ldg(reinterpret_cast<const float4 *>(pli + ((int64_t)s * L + layer) * ple) + t);
    float4 v;
    v.x = __fmul_rn(gelu_tanh(g.x), e.x);
    v.y = __fmul_rn(gelu_tanh(g.y), e.y);
    v.z = __fmul_rn(gelu_tanh(g.z), e.z);
    v.w = __fmul_rn(gelu_tanh(g.w), e.w);
    quant4(v, t, true, xq + (int64_t)s * ple, xs + (int64_t)s * (ple / kQ8Block));
}

// Greedy sampling (crates/llm-eng/src/sample.rs:27-36): the maximum under
// f32::total_cmp, the last index among equal maxima (Iterator::max_by). The
// total order as an unsigned key, packed above the index, so one unsigned
// maximum decides both; each CTA scans a chunk of the row and folds its
// result into the row's slot with a 64-bit atomic maximum (slots zeroed by
// the step's plan kernel).
__device__ __forceinline__ uint32_t total_key(float f) {
    int32_t b = __float_as_int(f);
    b ^= (int32_t)(((uint32_t)(b >> 31)) >> 1);
    return (uint32_t)b ^ 0x80000000u;
}

constexpr int kArgmaxChunk = 4096;

__global__ void __launch_bounds__(256) argmax_kernel(const float *__restrict__ logits, int64_t vocab,
                                                     unsigned long long *__restrict__ best) {
    ptx::pdl_trigger();  // a dependent may launch; it waits for this grid itself
    ptx::pdl_wait();
    __shared__ unsigned long long best_s[8];
    const int s = blockIdx.y;
    const float *row = logits + (int64_t)s * vocab;
    const int64_t i0 = (int64_t)blockIdx.x * kArgmaxChunk;
    const int64_t i1 = i0 + kArgmaxChunk < vocab ? i0 + kArgmaxChunk : vocab;
    unsigned long long b = 0;
    for (int64_t i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
        const unsigned long long packed = ((unsigned long long)total_key(row[i]) << 32) | (unsigned long long)i;
        b = packed > b ? packed : b;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, b, o);
        b = other > b ? other : b;
    }
    if ((threadIdx.x & 31) == 0) best_s[threadIdx.x >> 5] = b;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int i = 1; i < (int)(blockDim.x >> 5); i++) b = best_s[i] > b ? best_s[i] : b;
        atomicMax(best + s, b);
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
    ptx::pdl_trigger();  // a dependent may launch; it waits for this grid itself
    ptx::pdl_wait();
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    const int n_tasks = a.n_layers * a.n;
    if (t < a.n_best) a.best[t] = 0;
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
        tk.new_row = ld.owner && a.fused_append ? pos : -1;
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

// Row rows[blockIdx.x] of xq/xs to row blockIdx.x of xq_out/xs_out; cols is
// a multiple of 32, so a row is cols/16 16-byte pieces and cols/32 scales.
__global__ void gather_rows_kernel(const int8_t *__restrict__ xq, const float *__restrict__ xs, int cols,
                                   const int32_t *__restrict__ rows, int8_t *__restrict__ xq_out,
                                   float *__restrict__ xs_out) {
    ptx::pdl_trigger();
    ptx::pdl_wait();
    const int j = blockIdx.x, r = rows[j];
    const int4 *src = reinterpret_cast<const int4 *>(xq + (size_t)r * cols);
    int4 *dst = reinterpret_cast<int4 *>(xq_out + (size_t)j * cols);
    for (int e = threadIdx.x; e < cols / 16; e += blockDim.x) dst[e] = src[e];
    for (int e = threadIdx.x; e < cols / kQ8Block; e += blockDim.x)
        xs_out[(size_t)j * (cols / kQ8Block) + e] = xs[(size_t)r * (cols / kQ8Block) + e];
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

cudaError_t e2b_embed(const uint8_t *table, int d, const int32_t *tokens, int n, float scale, float *x, cudaStream_t st,
                      bool pdl) {
    return launch_k(pdl, embed_kernel, dim3(n), dim3(kRowThreads), 0, st, table, d, tokens, scale, x);
}

cudaError_t e2b_ple_inputs(const float *P, const uint8_t *table, const int32_t *tokens, const float *w, int L, int ple,
                           float ps, float ts, float is, float eps, float *out, int n, cudaStream_t st, bool pdl) {
    if (ple > 1024) return cudaErrorInvalidValue;
    return launch_k(pdl, ple_inputs_kernel, dim3(n * L), dim3(kRowThreads), 0, st, P, table, tokens, w, L, ple, ps, ts,
                    is, eps, out);
}

cudaError_t e2b_resid(float *x, const float *y, const float *w_post, float post, const float *w_next, int d, float eps,
                      int8_t *xq, float *xs, int n, cudaStream_t st, bool pdl) {
    if (d > kMaxRow || d % kQ8Block) return cudaErrorInvalidValue;
    ResidArgs a{x, y, w_post, w_next, xq, xs, d, eps, post};
    return launch_k(pdl, resid_kernel, dim3(n), dim3((d / 4 + 31) / 32 * 32), 0, st, a);
}

cudaError_t e2b_gelu_quant(const float *gate, const float *pli, int layer, int L, int ple, int8_t *xq, float *xs, int n,
                           cudaStream_t st, bool pdl) {
    if (ple > 1024 || ple % 128) return cudaErrorInvalidValue;  // whole warps of float4s
    return launch_k(pdl, gelu_quant_kernel, dim3(n), dim3(ple / 4), 0, st, gate, pli, layer, L, ple, xq, xs);
}

cudaError_t e2b_argmax(const float *logits, int64_t vocab, int n, unsigned long long *best, cudaStream_t st,
                       bool pdl) {
    const dim3 grid((unsigned)((vocab + kArgmaxChunk - 1) / kArgmaxChunk), (unsigned)n);
    return launch_k(pdl, argmax_kernel, grid, dim3(256), 0, st, logits, vocab, best);
}

cudaError_t e2b_gather_rows(const int8_t *xq, const float *xs, int cols, const int32_t *rows, int n, int8_t *xq_out,
                            float *xs_out, cudaStream_t st, bool pdl) {
    if (n == 0) return cudaSuccess;
    if (cols % kQ8Block) return cudaErrorInvalidValue;
    return launch_k(pdl, gather_rows_kernel, dim3(n), dim3(kRowThreads), 0, st, xq, xs, cols, rows, xq_out, xs_out);
}

cudaError_t e2b_plan(const E2bPlanArgs &a, cudaStream_t st) {
    const int total = a.n_layers * a.n + a.n * (a.max_splits_local + a.max_splits_global);
    if (total == 0) return cudaSuccess;
    e2b_plan_kernel<<<(total + 255) / 256, 256, 0, st>>>(a);
    return cudaGetLastError();
}

}  // namespace g4a
