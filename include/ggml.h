/*
 * Minimal ggml type shim for the T2S drop-in (include/gpt_sovits/t2s.h) -- not ggml.
 *
 * GPT-SoVITS.cpp's T2S interface exposes ggml types in its structs and signatures
 * (include/gpt_sovits/t2s.h:3-5 of the reference).  This header declares the handful of them a
 * caller of that interface touches -- enum ggml_type, ggml_fp16_t, struct ggml_tensor (ne, nb,
 * type, data, name), the opaque context/graph handles, GGML_ASSERT and the f16 conversions -- so
 * code written against the reference header compiles here.  There is no tensor algebra: the
 * tensors a session hands out are views of its CUDA state (see ggml-backend.h for get/set).
 * The enum values are the GGUF on-disk type ids (a file-format constant).
 */
#ifndef T2S_GGML_SHIM_H
#define T2S_GGML_SHIM_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define GGML_SHIM_API __attribute__((visibility("default")))
#else
#define GGML_SHIM_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define GGML_MAX_DIMS 4
#define GGML_MAX_NAME 64

typedef uint16_t ggml_fp16_t;

enum ggml_type {
    GGML_TYPE_F32 = 0,
    GGML_TYPE_F16 = 1,
    GGML_TYPE_Q4_0 = 2,
    GGML_TYPE_Q4_1 = 3,
    GGML_TYPE_Q5_0 = 6,
    GGML_TYPE_Q5_1 = 7,
    GGML_TYPE_Q8_0 = 8,
    GGML_TYPE_Q8_1 = 9,
    GGML_TYPE_Q4_K = 12,
    GGML_TYPE_I32 = 26,
};

enum ggml_status {
    GGML_STATUS_ALLOC_FAILED = -2,
    GGML_STATUS_FAILED = -1,
    GGML_STATUS_SUCCESS = 0,
    GGML_STATUS_ABORTED = 1,
};

struct ggml_context;   /* opaque: owner of a set of tensors */
struct ggml_cgraph;    /* opaque: a session's decode step or flex plan */

/* A tensor handed out by the T2S interface.  ne/nb/type/name describe it as ggml would; the
 * storage behind `data` is host memory of the session (inputs, outputs) or absent (KV caches,
 * masks and weights live on the device); read and write it through ggml_backend_tensor_get /
 * ggml_backend_tensor_set only. */
struct ggml_tensor {
    enum ggml_type type;
    int64_t ne[GGML_MAX_DIMS];
    size_t nb[GGML_MAX_DIMS];
    void* data;
    char name[GGML_MAX_NAME];
    /* this implementation: what the tensor is a view of (not part of ggml's layout) */
    int t2s_kind;
    int t2s_index;
    void* t2s_owner;
};

GGML_SHIM_API int64_t ggml_nelements(const struct ggml_tensor* t);
GGML_SHIM_API size_t ggml_nbytes(const struct ggml_tensor* t);
GGML_SHIM_API size_t ggml_type_size(enum ggml_type type);
GGML_SHIM_API int64_t ggml_blck_size(enum ggml_type type);
GGML_SHIM_API const char* ggml_type_name(enum ggml_type type);
GGML_SHIM_API float ggml_fp16_to_fp32(ggml_fp16_t h);
GGML_SHIM_API ggml_fp16_t ggml_fp32_to_fp16(float f);
GGML_SHIM_API void ggml_abort(const char* file, int line, const char* fmt, ...);

#define GGML_ASSERT(x)                                                        \
    do {                                                                      \
        if (!(x)) ggml_abort(__FILE__, __LINE__, "GGML_ASSERT(%s) failed", #x); \
    } while (0)

#ifdef __cplusplus
}
#endif
#endif
