/* Minimal ggml type shim (see ggml.h): the CUDA backend of the T2S drop-in.  A backend is one
 * CUDA device; models and sessions made with it run there.  Returns NULL when the device does
 * not exist (no GPU, or device >= the device count). */
#ifndef T2S_GGML_CUDA_SHIM_H
#define T2S_GGML_CUDA_SHIM_H
#include "ggml-backend.h"
#ifdef __cplusplus
extern "C" {
#endif
GGML_SHIM_API ggml_backend_t ggml_backend_cuda_init(int device);
GGML_SHIM_API int ggml_backend_cuda_get_device_count(void);
#ifdef __cplusplus
}
#endif
#endif
