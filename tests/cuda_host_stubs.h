// Host stand-ins for the CUDA runtime calls of the library's host files
// (host memory for device and pinned memory, copies as memcpy, no-op events,
// streams and graphs, 148 SMs), for checks of the host logic without a GPU.
// Include in exactly one translation unit of a check program.
#pragma once
#include <cstdlib>
#include <cstring>

#include <cuda_runtime.h>

extern "C" {
cudaError_t cudaDeviceGetAttribute(int *v, cudaDeviceAttr, int) {
    *v = 148;
    return cudaSuccess;
}
cudaError_t cudaEventCreate(cudaEvent_t *e) {
    *e = reinterpret_cast<cudaEvent_t>(std::malloc(8));
    return cudaSuccess;
}
cudaError_t cudaEventCreateWithFlags(cudaEvent_t *e, unsigned) { return cudaEventCreate(e); }
cudaError_t cudaEventDestroy(cudaEvent_t e) {
    std::free(e);
    return cudaSuccess;
}
cudaError_t cudaEventElapsedTime(float *ms, cudaEvent_t, cudaEvent_t) {
    *ms = 0.0f;
    return cudaSuccess;
}
cudaError_t cudaEventRecord(cudaEvent_t, cudaStream_t) { return cudaSuccess; }
cudaError_t cudaEventSynchronize(cudaEvent_t) { return cudaSuccess; }
cudaError_t cudaFree(void *p) {
    std::free(p);
    return cudaSuccess;
}
cudaError_t cudaFreeHost(void *p) { return cudaFree(p); }
const char *cudaGetErrorString(cudaError_t) { return "host stand-in"; }
cudaError_t cudaMalloc(void **p, size_t n) {
    *p = std::aligned_alloc(256, (n + 255) / 256 * 256);
    return *p ? cudaSuccess : cudaErrorMemoryAllocation;
}
cudaError_t cudaHostAlloc(void **p, size_t n, unsigned) { return cudaMalloc(p, n); }
cudaError_t cudaMemcpy(void *d, const void *s, size_t n, cudaMemcpyKind) {
    std::memcpy(d, s, n);
    return cudaSuccess;
}
cudaError_t cudaMemcpyAsync(void *d, const void *s, size_t n, cudaMemcpyKind k, cudaStream_t) {
    return cudaMemcpy(d, s, n, k);
}
cudaError_t cudaMemset(void *d, int v, size_t n) {
    std::memset(d, v, n);
    return cudaSuccess;
}
cudaError_t cudaMemsetAsync(void *d, int v, size_t n, cudaStream_t) { return cudaMemset(d, v, n); }
cudaError_t cudaSetDevice(int) { return cudaSuccess; }
cudaError_t cudaStreamSynchronize(cudaStream_t) { return cudaSuccess; }
cudaError_t cudaDeviceSynchronize() { return cudaSuccess; }
cudaError_t cudaStreamCreateWithFlags(cudaStream_t *s, unsigned) {
    *s = reinterpret_cast<cudaStream_t>(std::malloc(8));
    return cudaSuccess;
}
cudaError_t cudaStreamDestroy(cudaStream_t s) {
    std::free(s);
    return cudaSuccess;
}
cudaError_t cudaStreamWaitEvent(cudaStream_t, cudaEvent_t, unsigned) { return cudaSuccess; }
// every host pointer is pageable to the stand-ins (the copy path of g4a_decode_host)
cudaError_t cudaPointerGetAttributes(cudaPointerAttributes *a, const void *) {
    *a = cudaPointerAttributes{};
    a->type = cudaMemoryTypeUnregistered;
    return cudaSuccess;
}
cudaError_t cudaGetLastError() { return cudaSuccess; }
cudaError_t cudaStreamBeginCapture(cudaStream_t, cudaStreamCaptureMode) { return cudaSuccess; }
cudaError_t cudaStreamEndCapture(cudaStream_t, cudaGraph_t *g) {
    *g = reinterpret_cast<cudaGraph_t>(std::malloc(8));
    return cudaSuccess;
}
cudaError_t cudaGraphInstantiate(cudaGraphExec_t *e, cudaGraph_t, unsigned long long) {
    *e = reinterpret_cast<cudaGraphExec_t>(std::malloc(8));
    return cudaSuccess;
}
cudaError_t cudaGraphDestroy(cudaGraph_t g) {
    std::free(g);
    return cudaSuccess;
}
cudaError_t cudaGraphExecDestroy(cudaGraphExec_t e) {
    std::free(e);
    return cudaSuccess;
}
cudaError_t cudaGraphLaunch(cudaGraphExec_t, cudaStream_t) { return cudaSuccess; }
}
