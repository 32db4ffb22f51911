// g4a_attend_static: grouped-query attention for one query position (the
// E2B shape: 8 query heads over 1 KV head, head width 256 or 512) that
// allocates no device memory when called.
//
// Who needs it: callers that cannot call cudaMalloc at the time they attend,
// for instance a serving process that hands (nearly) all device memory to its
// own pools at start-up and keeps none back for libraries, or code paths where
// the device synchronisation that cudaMalloc / cudaFree can imply is not
// acceptable. Everything this call needs beyond the caller's inputs and
// output lives in one file-scope device array, g4a_attend_scratch, of
// kScratchBytes (about 1 MiB): every GPU that loads this library holds it
// until the process exits.
//
// Set-up: the device is the one cuda_stream belongs to (the current device
// for the legacy default stream). The first call on a device makes it current
// for the moment of the call, looks up the array's device address there
// (cudaGetSymbolAddress) and keeps it; make that first call before any stream
// capture. Later calls reuse the address. The address is not looked up again
// after cudaDeviceReset, so do not call this after resetting a device.
//
// Sharing: all calls on a device use the same array, which keeps the last
// call's contents. The arrival counter that must start at zero is cleared by
// each call (an async memset on the caller's stream, the only reset: the
// kernel never clears it). Calls that overlap on the GPU (different streams,
// or a second call before the first finished on another stream) race on the
// array; serialise them on one stream.
#include <cuda_runtime.h>
#include <math_constants.h>

#include <algorithm>
#include <mutex>

#include "../../include/g4attn.h"

namespace {

constexpr int kHeadsS = 8;
constexpr int kMaxHd = 512;
constexpr int kMaxSplits = 64;  // row ranges merged through the scratch array
constexpr int kThreadsS = 256;
constexpr size_t kPartOFloats = (size_t)kMaxSplits * kHeadsS * kMaxHd;
constexpr size_t kPartMLFloats = (size_t)kMaxSplits * 2 * kHeadsS;
constexpr size_t kScratchBytes = (kPartOFloats + kPartMLFloats) * sizeof(float) + 256;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g4a_attend_scratch[kScratchBytes];

__device__ __forceinline__ float wsum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float wmax(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// One CTA per row range [len*s/n, len*(s+1)/n) of the keys; online softmax in
// blocks of 64 rows; the last CTA to arrive merges the partials in split
// order.
template <int HD>
__global__ void __launch_bounds__(kThreadsS) attend_static_kernel(const float *__restrict__ q,
                                                                  const float *__restrict__ keys,
                                                                  const float *__restrict__ values, int64_t len,
                                                                  int n_splits, float scale, float *__restrict__ out,
                                                                  unsigned char *scratch) {
    constexpr int BLK = 64;
    constexpr int PL = HD / 32;
    constexpr int CPT = HD / kThreadsS;
    __shared__ float q_s[kHeadsS][HD];
    __shared__ float p_s[kHeadsS][BLK];
    __shared__ float alpha_s[kHeadsS], m_s[kHeadsS], l_s[kHeadsS];
    __shared__ int last_s;
    float *part_o = reinterpret_cast<float *>(scratch);
    float *part_ml = part_o + kPartOFloats;
    unsigned *ticket = reinterpret_cast<unsigned *>(part_ml + kPartMLFloats);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int s = blockIdx.x;
    const int64_t lo = len * s / n_splits, hi = len * (s + 1) / n_splits;
    for (int e = threadIdx.x; e < kHeadsS * HD; e += kThreadsS) q_s[e / HD][e % HD] = q[e];
    if (threadIdx.x < kHeadsS) {
        m_s[threadIdx.x] = -CUDART_INF_F;
        l_s[threadIdx.x] = 0.0f;
    }
    float acc[kHeadsS][CPT];
#pragma unroll
    for (int h = 0; h < kHeadsS; h++)
#pragma unroll
        for (int u = 0; u < CPT; u++) acc[h][u] = 0.0f;
    __syncthreads();
    for (int64_t b0 = lo; b0 < hi; b0 += BLK) {
        const int nb = (int)min((int64_t)BLK, hi - b0);
        // scores: warp w takes rows w, w+8, ...; each lane a strided slice
        for (int r = warp; r < nb; r += kHeadsS) {
            const float *k = keys + (size_t)(b0 + r) * HD;
            float part[kHeadsS];
#pragma unroll
            for (int h = 0; h < kHeadsS; h++) part[h] = 0.0f;
#pragma unroll
            for (int i = 0; i < PL; i++) {
                const float kv = k[lane + 32 * i];
#pragma unroll
                for (int h = 0; h < kHeadsS; h++) part[h] = fmaf(q_s[h][lane + 32 * i], kv, part[h]);
            }
#pragma unroll
            for (int h = 0; h < kHeadsS; h++) {
                const float t = wsum(part[h]);
                if (lane == 0) p_s[h][r] = t * scale;
            }
        }
        __syncthreads();
        {  // online softmax, warp h owns head h
            const int h = warp;
            const float s0 = lane < nb ? p_s[h][lane] : -CUDART_INF_F;
            const float s1 = lane + 32 < nb ? p_s[h][lane + 32] : -CUDART_INF_F;
            const float m_old = m_s[h];
            const float m_new = fmaxf(m_old, wmax(fmaxf(s0, s1)));
            const float p0 = expf(s0 - m_new), p1 = expf(s1 - m_new);
            const float alpha = expf(m_old - m_new);
            const float bs = wsum((lane < nb ? p0 : 0.0f) + (lane + 32 < nb ? p1 : 0.0f));
            if (lane < nb) p_s[h][lane] = p0;
            if (lane + 32 < nb) p_s[h][lane + 32] = p1;
            __syncwarp();
            if (lane == 0) {
                alpha_s[h] = alpha;
                m_s[h] = m_new;
                l_s[h] = l_s[h] * alpha + bs;
            }
        }
        __syncthreads();
#pragma unroll
        for (int h = 0; h < kHeadsS; h++)
#pragma unroll
            for (int u = 0; u < CPT; u++) acc[h][u] *= alpha_s[h];
        for (int r = 0; r < nb; r++) {
            const float *v = values + (size_t)(b0 + r) * HD;
            float vv[CPT];
#pragma unroll
            for (int u = 0; u < CPT; u++) vv[u] = v[threadIdx.x + kThreadsS * u];
#pragma unroll
            for (int h = 0; h < kHeadsS; h++)
#pragma unroll
                for (int u = 0; u < CPT; u++) acc[h][u] = fmaf(p_s[h][r], vv[u], acc[h][u]);
        }
        __syncthreads();
    }
    if (n_splits == 1) {
#pragma unroll
        for (int h = 0; h < kHeadsS; h++)
#pragma unroll
            for (int u = 0; u < CPT; u++) out[h * HD + threadIdx.x + kThreadsS * u] = acc[h][u] / l_s[h];
        return;
    }
    float *po = part_o + (size_t)s * kHeadsS * kMaxHd;
#pragma unroll
    for (int h = 0; h < kHeadsS; h++)
#pragma unroll
        for (int u = 0; u < CPT; u++) po[h * kMaxHd + threadIdx.x + kThreadsS * u] = acc[h][u];
    if (threadIdx.x < kHeadsS) {
        part_ml[s * 2 * kHeadsS + threadIdx.x] = m_s[threadIdx.x];
        part_ml[s * 2 * kHeadsS + kHeadsS + threadIdx.x] = l_s[threadIdx.x];
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last_s = atomicAdd(ticket, 1u) == (unsigned)(n_splits - 1);
    __syncthreads();
    if (!last_s) return;
    __threadfence();
    for (int h = 0; h < kHeadsS; h++) {
        float M = -CUDART_INF_F;
        for (int i = 0; i < n_splits; i++) M = fmaxf(M, __ldcg(part_ml + i * 2 * kHeadsS + h));
        float L = 0.0f, o[CPT];
#pragma unroll
        for (int u = 0; u < CPT; u++) o[u] = 0.0f;
        for (int i = 0; i < n_splits; i++) {
            const float w = expf(__ldcg(part_ml + i * 2 * kHeadsS + h) - M);
            L = fmaf(__ldcg(part_ml + i * 2 * kHeadsS + kHeadsS + h), w, L);
#pragma unroll
            for (int u = 0; u < CPT; u++)
                o[u] = fmaf(__ldcg(part_o + ((size_t)i * kHeadsS + h) * kMaxHd + threadIdx.x + kThreadsS * u), w, o[u]);
        }
#pragma unroll
        for (int u = 0; u < CPT; u++) out[h * HD + threadIdx.x + kThreadsS * u] = o[u] / L;
    }
}

std::mutex g_setup_mu;
unsigned char *g_scratch[kMaxDevices] = {};

// Device address of g4a_attend_scratch on device `dev`, looked up (with dev
// current) on the first call for that device.
cudaError_t scratch_for_device(int dev, unsigned char **out) {
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_setup_mu);
    if (!g_scratch[dev]) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g4a_attend_scratch);
        if (e != cudaSuccess) return e;
        g_scratch[dev] = static_cast<unsigned char *>(p);
    }
    *out = g_scratch[dev];
    return cudaSuccess;
}

// Makes the stream's device current for the life of the object and restores
// the caller's device afterwards.
struct DeviceOfStream {
    int prev = -1, dev = -1;
    cudaError_t err = cudaSuccess;
    explicit DeviceOfStream(cudaStream_t st) {
        if ((err = cudaGetDevice(&prev)) != cudaSuccess) return;
        if ((err = cudaStreamGetDevice(st, &dev)) != cudaSuccess) return;
        if (dev != prev) err = cudaSetDevice(dev);
    }
    ~DeviceOfStream() {
        if (prev >= 0 && dev >= 0 && dev != prev) cudaSetDevice(prev);
    }
};

}  // namespace

extern "C" int g4a_attend_static(void *cuda_stream, const float *q_dev, const float *keys_dev,
                                 const float *values_dev, int64_t len, int32_t n_heads, int32_t n_kv_heads,
                                 int32_t head_dim, float scale, float *out_dev) {
    if (n_heads != kHeadsS || n_kv_heads != 1 || (head_dim != 256 && head_dim != 512))
        return G4A_COMPUTE;  // the static scratch holds 8 heads x at most 512 columns per row range
    if (len < 0 || !q_dev || !out_dev) return G4A_COMPUTE;
    if (len == 0) return G4A_NONFINITE;  // empty softmax, as the reference's attend
    if (!keys_dev || !values_dev) return G4A_COMPUTE;
    cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
    const DeviceOfStream on(st);
    if (on.err != cudaSuccess) return G4A_CUDA;
    unsigned char *scratch = nullptr;
    if (scratch_for_device(on.dev, &scratch) != cudaSuccess) return G4A_CUDA;
    const int n_splits = (int)std::min<int64_t>(kMaxSplits, std::max<int64_t>(1, (len + 31) / 32));
    unsigned *ticket = reinterpret_cast<unsigned *>(scratch + (kPartOFloats + kPartMLFloats) * sizeof(float));
    if (cudaMemsetAsync(ticket, 0, sizeof(unsigned), st) != cudaSuccess) return G4A_CUDA;
    // cudaLaunchKernelEx reports this launch's own error (not one left over
    // from an earlier call in the process)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)n_splits);
    cfg.blockDim = dim3(kThreadsS);
    cfg.stream = st;
    const cudaError_t e =
        head_dim == 256
            ? cudaLaunchKernelEx(&cfg, attend_static_kernel<256>, q_dev, keys_dev, values_dev, len, n_splits, scale,
                                 out_dev, scratch)
            : cudaLaunchKernelEx(&cfg, attend_static_kernel<512>, q_dev, keys_dev, values_dev, len, n_splits, scale,
                                 out_dev, scratch);
    return e == cudaSuccess ? G4A_OK : G4A_CUDA;
}
