/* Minimal ggml type shim (see ggml.h): the graph allocator handle of the T2S session structs.
 * Nothing allocates through it here; the session owns its device memory. */
#ifndef T2S_GGML_ALLOC_SHIM_H
#define T2S_GGML_ALLOC_SHIM_H
#include "ggml.h"
typedef struct ggml_gallocr* ggml_gallocr_t;
#endif
