// The backend-creation helper of the reference's T2S tests (tests/common/test_backend.h there),
// with its one line changed for this implementation: the backend is a CUDA device
// (ggml_backend_cuda_init from include/ggml-cuda.h) instead of ggml's CPU or Metal backend.
#pragma once
#include "ggml-backend.h"
#include "ggml-cuda.h"

static inline ggml_backend_t create_test_backend() { return ggml_backend_cuda_init(0); }
