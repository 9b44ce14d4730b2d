/*
 * Minimal ggml type shim (see ggml.h): the backend calls a caller of the T2S interface makes
 * (tests/t2s/test_t2s_infer.cpp:186-399 of the reference), implemented over libt2sx.
 *   ggml_backend_t             a CUDA device (ggml_backend_cuda_init in ggml-cuda.h)
 *   ggml_backend_tensor_set    writes a session input (token ids, noise, seen mask, prefill rows)
 *   ggml_backend_tensor_get    reads an output or a view (sampled/greedy tokens, final-layer rows
 *                              y, the f16 KV cache of a layer, kv_pos, positions, masks)
 *   ggml_backend_graph_compute runs a session's decode step or flex plan on the device
 * Out-of-range offsets, writes to read-only views and unknown graphs abort with a message, as
 * GGML_ASSERT does.
 */
#ifndef T2S_GGML_BACKEND_SHIM_H
#define T2S_GGML_BACKEND_SHIM_H
#include "ggml.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct ggml_backend* ggml_backend_t;
typedef struct ggml_backend_buffer* ggml_backend_buffer_t;

GGML_SHIM_API void ggml_backend_tensor_set(struct ggml_tensor* tensor, const void* data, size_t offset, size_t size);
GGML_SHIM_API void ggml_backend_tensor_get(const struct ggml_tensor* tensor, void* data, size_t offset, size_t size);
GGML_SHIM_API enum ggml_status ggml_backend_graph_compute(ggml_backend_t backend, struct ggml_cgraph* graph);
GGML_SHIM_API const char* ggml_backend_name(ggml_backend_t backend);
GGML_SHIM_API void ggml_backend_free(ggml_backend_t backend);

#ifdef __cplusplus
}
#endif
#endif
