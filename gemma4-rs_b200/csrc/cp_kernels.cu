// Element-wise kernels of the key/value-shard context-parallel prefill
// (g4a_cp_prefill, schedule G4A_CP_KV_SHARDS).
//
// Each rank holds partial attention results of its own two key chunks for
// query rows of the whole sequence, as up to kCpMaxSegs row segments, each a
// normalised output O [rows][8][hd] and its natural-log sum of exponentials
// L [rows][8] from g4a_prefill. The cross-rank merge is
//   M   = max over ranks and segments of L        (all-reduce MAX, [T][8])
//   w_k = exp(L_k - M)
//   O   = sum_k w_k O_k / sum_k w_k               (reduce-scatter SUM)
// The reference computes the same attention one position at a time over all
// earlier keys (crates/llm-gemma4/src/impl_/generate.rs:37-41 into
// model.rs:326-366, global range eng/mod.rs:33-35); the merge is the
// log-sum-exp identity of a softmax over a union of disjoint key sets.
#include <cuda_runtime.h>
#include <math_constants.h>

#include "internal.h"

namespace g4a {
namespace {

constexpr int kCpHeads = 8;

__device__ __forceinline__ float seg_weight(float lse, float m) {
    return lse == -CUDART_INF_F ? 0.0f : __expf(lse - m);
}

// m[t][h] = max over the segments covering row t of their L (-inf if none).
__global__ void cp_rowmax_kernel(CpSegs segs, int32_t T, float *m) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)T * kCpHeads) return;
    const int32_t t = (int32_t)(idx / kCpHeads);
    const int h = (int)(idx % kCpHeads);
    float v = -CUDART_INF_F;
    for (int k = 0; k < segs.n; k++)
        if (t >= segs.s[k].t0 && t < segs.s[k].t1) v = fmaxf(v, segs.s[k].lse[(int64_t)(t - segs.s[k].t0) * kCpHeads + h]);
    m[idx] = v;
}

// One CTA per packed row. Packed rows are in reduce-scatter order: for rank
// s = 0..W-1 its chunk s, then its chunk 2W-1-s, c rows each; a packed row
// holds sum_k w_k O_k (8 x hd floats) then sum_k w_k (8 floats).
__global__ void __launch_bounds__(256) cp_pack_kernel(CpSegs segs, const float *__restrict__ m, int32_t W, int32_t c,
                                                      int32_t hd, float *__restrict__ packed) {
    const int64_t pr = blockIdx.x;
    const int32_t s = (int32_t)(pr / (2 * (int64_t)c));
    const int32_t j = (int32_t)((pr / c) & 1);
    const int32_t i = (int32_t)(pr % c);
    const int32_t chunk = j == 0 ? s : 2 * W - 1 - s;
    const int32_t t = chunk * c + i;
    const int64_t stride = (int64_t)kCpHeads * hd + kCpHeads;
    __shared__ float ws[kCpMaxSegs][kCpHeads];
    __shared__ const float *rows[kCpMaxSegs];
    __shared__ int n_cover;
    if (threadIdx.x == 0) {
        int n = 0;
        for (int k = 0; k < segs.n; k++) {
            if (t < segs.s[k].t0 || t >= segs.s[k].t1) continue;
            const int64_t r = t - segs.s[k].t0;
            rows[n] = segs.s[k].o + r * kCpHeads * hd;
            for (int h = 0; h < kCpHeads; h++) ws[n][h] = seg_weight(segs.s[k].lse[r * kCpHeads + h], m[(int64_t)t * kCpHeads + h]);
            n++;
        }
        n_cover = n;
    }
    __syncthreads();
    const int n = n_cover;
    float *dst = packed + pr * stride;
    const int n4 = kCpHeads * hd / 4;
    for (int e = threadIdx.x; e < n4; e += blockDim.x) {
        const int h = (4 * e) / hd;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int k = 0; k < n; k++) {
            const float4 o = reinterpret_cast<const float4 *>(rows[k])[e];
            const float w = ws[k][h];
            acc.x = fmaf(w, o.x, acc.x);
            acc.y = fmaf(w, o.y, acc.y);
            acc.z = fmaf(w, o.z, acc.z);
            acc.w = fmaf(w, o.w, acc.w);
        }
        reinterpret_cast<float4 *>(dst)[e] = acc;
    }
    if (threadIdx.x < kCpHeads) {
        float w = 0.0f;
        for (int k = 0; k < n; k++) w += ws[k][threadIdx.x];
        dst[kCpHeads * hd + threadIdx.x] = w;
    }
}

// out[r][h][:] = X[r][h][:] / w[r][h] for this rank's 2c rows.
__global__ void __launch_bounds__(256) cp_finish_kernel(const float *__restrict__ recv, int32_t hd,
                                                        float *__restrict__ out) {
    const int64_t r = blockIdx.x;
    const int64_t stride = (int64_t)kCpHeads * hd + kCpHeads;
    const float *src = recv + r * stride;
    float *dst = out + r * kCpHeads * hd;
    const int n4 = kCpHeads * hd / 4;
    for (int e = threadIdx.x; e < n4; e += blockDim.x) {
        const float w = src[kCpHeads * hd + (4 * e) / hd];
        const float inv = w > 0.0f ? 1.0f / w : 0.0f;
        float4 x = reinterpret_cast<const float4 *>(src)[e];
        x.x *= inv;
        x.y *= inv;
        x.z *= inv;
        x.w *= inv;
        reinterpret_cast<float4 *>(dst)[e] = x;
    }
}

}  // namespace

cudaError_t launch_cp_rowmax(const CpSegs &segs, int32_t T, float *m, cudaStream_t st) {
    const int64_t n = (int64_t)T * kCpHeads;
    if (n == 0) return cudaSuccess;
    cp_rowmax_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(segs, T, m);
    return cudaGetLastError();
}

cudaError_t launch_cp_pack(const CpSegs &segs, const float *m, int32_t W, int32_t c, int32_t hd, float *packed,
                           cudaStream_t st) {
    const int64_t rows = 2 * (int64_t)W * c;
    if (rows == 0) return cudaSuccess;
    cp_pack_kernel<<<(unsigned)rows, 256, 0, st>>>(segs, m, W, c, hd, packed);
    return cudaGetLastError();
}

cudaError_t launch_cp_finish(const float *recv, int32_t rows, int32_t hd, float *out, cudaStream_t st) {
    if (rows == 0) return cudaSuccess;
    cp_finish_kernel<<<(unsigned)rows, 256, 0, st>>>(recv, hd, out);
    return cudaGetLastError();
}

}  // namespace g4a
