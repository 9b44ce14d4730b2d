// t2sx_matmul_noalloc: the isolated matmul without any device allocation.
//
// Who needs it: callers that must not call cudaMalloc at the time they run a matmul -- for
// example a streaming TTS server's per-request synthesis thread (cudaMalloc can synchronise the
// whole device and stall every other stream on it), or an application embedding this library that
// has already reserved the device's memory budget for itself and forbids further allocations.
// t2sx_matmul allocates its activation-quantisation scratch on first use; this variant instead
// uses one fixed scratch array that lives in the library's own device image.
//
// The scratch is a file-scope __device__ array of T2SX_NOALLOC_MAX_ELEMS activation elements
// (about 4.5 MiB); every GPU that loads the library holds it until the process exits.  All calls
// on a device share it and it keeps the previous call's contents, so calls that overlap on the
// GPU (on different streams, or from different host threads) race and must be serialised by the
// caller.  Nothing in it has to start at zero: each call's quantisation kernel writes every byte
// that the same call's matmul kernel reads.
#include "../../include/t2sx.h"
#include "t2sx_kernels.cuh"

#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

using namespace t2sx;

// int8 (or f16) activation values, then per-32-element scales, then per-32-element sums
static constexpr size_t kQBytes = (size_t)T2SX_NOALLOC_MAX_ELEMS * 2;
static constexpr size_t kDBytes = (size_t)T2SX_NOALLOC_MAX_ELEMS / 32 * 4;
static constexpr size_t kScratchBytes = kQBytes + kDBytes + kDBytes;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kScratchBytes];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
void* g_scratch_ptr[kMaxDevices] = {};   // device address of g_noalloc_scratch, per device
}  // namespace

// Internal helpers of t2sx_api.cu (weight handle fields, the thread's error message).
int32_t t2sx_weight_device_of(const t2sx_weight* w);
const DevW* t2sx_weight_devw_of(const t2sx_weight* w);
int t2sx_set_error(int code, const char* msg);
int32_t* t2sx_weight_err_of(const t2sx_weight* w);

extern "C" int t2sx_matmul_noalloc(t2sx_weight* w, const float* x_dev, int64_t M, const float* bias_dev, float* y_dev,
                                   void* stream) {
    if (!w || !x_dev || !y_dev || M <= 0) return t2sx_set_error(T2SX_ERR_INVALID, "t2sx_matmul_noalloc: bad arguments");
    const int32_t dev = t2sx_weight_device_of(w);
    const DevW* W = t2sx_weight_devw_of(w);
    // M is bounded before the product is formed, so M * K cannot overflow
    if (M > (int64_t)T2SX_NOALLOC_MAX_ELEMS / W->K) {
        char msg[160];
        snprintf(msg, sizeof(msg), "t2sx_matmul_noalloc: M = %lld rows of K = %d exceed the fixed scratch of %d activation elements",
                 (long long)M, W->K, (int)T2SX_NOALLOC_MAX_ELEMS);
        return t2sx_set_error(T2SX_ERR_INVALID, msg);
    }
    if (dev < 0 || dev >= kMaxDevices) return t2sx_set_error(T2SX_ERR_INVALID, "t2sx_matmul_noalloc: device index out of range");
    DeviceGuard dg_;   // the caller's current device is restored on return
    if (dg_.set(dev) != cudaSuccess) return t2sx_set_error(T2SX_ERR_CUDA, "t2sx_matmul_noalloc: cudaSetDevice failed");
    void* base = nullptr;
    {
        // One-time set-up per device, done by the first call on that device with the device
        // current: the host-side symbol is only a stand-in, the kernels need the device address
        // of this device's copy of the array.  Make the first call before any stream capture.
        std::lock_guard<std::mutex> lk(g_setup_mu);
        if (!g_scratch_ptr[dev]) {
            void* p = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
            if (e != cudaSuccess || !p) return t2sx_set_error(T2SX_ERR_CUDA, "t2sx_matmul_noalloc: cudaGetSymbolAddress failed");
            g_scratch_ptr[dev] = p;
        }
        base = g_scratch_ptr[dev];
    }
    cudaStream_t st = (cudaStream_t)stream;
    ErrScope es_(t2sx_weight_err_of(w));   // the weight's error word (allocated with the weight)
    uint8_t* p = (uint8_t*)base;
    ActQ a;
    a.q = (int8_t*)p;
    a.h = (uint16_t*)p;
    a.d = (float*)(p + kQBytes);
    a.bs = (int32_t*)(p + kQBytes + kDBytes);
    quantize_act(W->type, x_dev, (int)M, W->K, a, st);
    matmul(*W, a, (int)M, bias_dev, 0, y_dev, st);
    if (cudaGetLastError() != cudaSuccess) return t2sx_set_error(T2SX_ERR_CUDA, "t2sx_matmul_noalloc: launch failed");
    return T2SX_OK;
}
