// Roofline denominators measured on the device itself: the L2 read bandwidth (a buffer that
// stays resident in L2, streamed with 16-byte loads that bypass L1) and the int8 tensor-core
// rate of tcgen05.mma.kind::i8 (t2sx_tc.cu).  Measurement entry points of the C ABI; the
// reference has no counterpart.
#include "../../include/t2sx.h"
#include "t2sx_kernels.cuh"

#include <cuda_runtime.h>

#include <cstdio>

using namespace t2sx;

int t2sx_set_error(int code, const char* msg);

namespace {

// Grid-stride read of n16 16-byte words with ld.global.cg (cached in L2 only), eight independent
// loads in flight per thread; the xor of everything read decides a store that never happens
// for the zero-filled buffer, so the loads are kept.
__global__ void __launch_bounds__(256) k_l2_read(const int4* __restrict__ p, int64_t n16, int* __restrict__ sink) {
    constexpr int U = 8;
    int x = 0;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (; i + (U - 1) * stride < n16; i += U * stride) {
        int4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u)
            asm volatile("ld.global.cg.v4.s32 {%0, %1, %2, %3}, [%4];\n"
                         : "=r"(v[u].x), "=r"(v[u].y), "=r"(v[u].z), "=r"(v[u].w)
                         : "l"(p + i + u * stride));
#pragma unroll
        for (int u = 0; u < U; ++u) x ^= v[u].x ^ v[u].y ^ v[u].z ^ v[u].w;
    }
    for (; i < n16; i += stride) {
        int4 v;
        asm volatile("ld.global.cg.v4.s32 {%0, %1, %2, %3}, [%4];\n" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p + i));
        x ^= v.x ^ v.y ^ v.z ^ v.w;
    }
    if (x == 0x5A5A5A5A) sink[0] = x;
}

#define PCK(x)                                                                          \
    do {                                                                                \
        cudaError_t e_ = (x);                                                           \
        if (e_ != cudaSuccess) {                                                        \
            char m_[200];                                                               \
            snprintf(m_, sizeof(m_), "%s: %s", #x, cudaGetErrorString(e_));             \
            rc = t2sx_set_error(T2SX_ERR_CUDA, m_);                                     \
            goto done;                                                                  \
        }                                                                               \
    } while (0)

}  // namespace

extern "C" int t2sx_probe_l2_read(int32_t device, int64_t bytes, int32_t iters, double* gbs) {
    if (!gbs || bytes < (1 << 20) || bytes > ((int64_t)1 << 30) || iters <= 0 || iters > 100000)
        return t2sx_set_error(T2SX_ERR_INVALID, "t2sx_probe_l2_read: bad arguments");
    DeviceGuard dg_;
    if (dg_.set(device) != cudaSuccess) return t2sx_set_error(T2SX_ERR_CUDA, "t2sx_probe_l2_read: cudaSetDevice failed");
    int rc = T2SX_OK, n_sm = 0;
    void* buf = nullptr;
    int* sink = nullptr;
    cudaStream_t st = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    float ms = 0.0f;
    const int64_t n16 = bytes / 16;
    PCK(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, device));
    PCK(cudaMalloc(&buf, (size_t)n16 * 16));
    PCK(cudaMalloc(&sink, 4));
    PCK(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    PCK(cudaMemsetAsync(buf, 0, (size_t)n16 * 16, st));
    PCK(cudaEventCreate(&e0));
    PCK(cudaEventCreate(&e1));
    for (int w = 0; w < 3; ++w) k_l2_read<<<n_sm * 8, 256, 0, st>>>((const int4*)buf, n16, sink);   // into L2
    PCK(cudaEventRecord(e0, st));
    for (int it = 0; it < iters; ++it) k_l2_read<<<n_sm * 8, 256, 0, st>>>((const int4*)buf, n16, sink);
    PCK(cudaEventRecord(e1, st));
    PCK(cudaEventSynchronize(e1));
    PCK(cudaGetLastError());
    PCK(cudaEventElapsedTime(&ms, e0, e1));
    *gbs = (double)n16 * 16.0 * iters / ((double)ms * 1e-3) / 1e9;
done:
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    if (st) cudaStreamDestroy(st);
    if (buf) cudaFree(buf);
    if (sink) cudaFree(sink);
    return rc;
}

extern "C" int t2sx_probe_i8_mma(int32_t device, int32_t iters, int32_t issuers, double* tops) {
    if (!tops || iters <= 0 || iters > (1 << 22) || issuers < 1 || issuers > 2)
        return t2sx_set_error(T2SX_ERR_INVALID, "t2sx_probe_i8_mma: bad arguments");
    DeviceGuard dg_;
    if (dg_.set(device) != cudaSuccess) return t2sx_set_error(T2SX_ERR_CUDA, "t2sx_probe_i8_mma: cudaSetDevice failed");
    int rc = T2SX_OK, ctas = 0;
    int32_t* err = nullptr;
    int32_t herr = 0;
    cudaStream_t st = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    float ms = 0.0f;
    PCK(cudaMalloc(&err, 4));
    PCK(cudaMemset(err, 0, 4));
    PCK(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    PCK(cudaEventCreate(&e0));
    PCK(cudaEventCreate(&e1));
    if (!probe_i8_mma(iters / 8 > 0 ? iters / 8 : 1, issuers, err, st, &ctas)) {   // warm-up
        rc = t2sx_set_error(T2SX_ERR_CUDA, "t2sx_probe_i8_mma: launch failed");
        goto done;
    }
    PCK(cudaEventRecord(e0, st));
    if (!probe_i8_mma(iters, issuers, err, st, &ctas)) {
        rc = t2sx_set_error(T2SX_ERR_CUDA, "t2sx_probe_i8_mma: launch failed");
        goto done;
    }
    PCK(cudaEventRecord(e1, st));
    PCK(cudaEventSynchronize(e1));
    PCK(cudaGetLastError());
    PCK(cudaMemcpy(&herr, err, 4, cudaMemcpyDeviceToHost));
    if (herr) {
        rc = t2sx_set_error(T2SX_ERR_TIMEOUT, "t2sx_probe_i8_mma: a wait ran out");
        goto done;
    }
    PCK(cudaEventElapsedTime(&ms, e0, e1));
    // one MMA: 2 * 128 * 256 * 32 integer operations
    *tops = (double)ctas * issuers * iters * 4.0 * (2.0 * 128 * 256 * 32) / ((double)ms * 1e-3) / 1e12;
done:
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    if (st) cudaStreamDestroy(st);
    if (err) cudaFree(err);
    return rc;
}
