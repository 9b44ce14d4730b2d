// Kernel launchers of the T2S decode path (host-side declarations).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <utility>

namespace t2sx {

// With T2SX_PDL=1 in the environment, or inside a PdlScope(true) (the one- and two-row layer
// chain), kernels are launched with programmatic stream serialization (PDL): a kernel may start
// while its predecessor runs and waits for it before touching data it produced (see pdl_wait in
// t2sx_math.cuh for what may be read before the wait).
bool pdl_enabled();
// Launches made on this host thread while a PdlScope(true) lives carry the attribute as well.
struct PdlScope {
    explicit PdlScope(bool on);
    ~PdlScope();
    PdlScope(const PdlScope&) = delete;
    PdlScope& operator=(const PdlScope&) = delete;
    bool prev;
};

// Makes `dev` the calling thread's current CUDA device for the lifetime of the guard and puts the
// caller's device back afterwards, so an entry point never changes the device a host thread
// works on (a host may keep other models on other devices in the same thread).
struct DeviceGuard {
    DeviceGuard() = default;
    DeviceGuard(const DeviceGuard&) = delete;
    DeviceGuard& operator=(const DeviceGuard&) = delete;
    cudaError_t set(int dev) {
        cudaError_t e = cudaGetDevice(&prev);
        if (e != cudaSuccess) return e;
        if (prev == dev) return cudaSuccess;
        e = cudaSetDevice(dev);
        restore = (e == cudaSuccess);
        return e;
    }
    ~DeviceGuard() {
        if (restore) cudaSetDevice(prev);
    }
    int prev = 0;
    bool restore = false;
};

// Device error word of the entry point running on this host thread (the session's flag, or the
// isolated weight's): kernels that can give up a bounded wait store a code there.  An ErrScope
// sets it for the launches made (or captured) while it lives.
int32_t* current_err_word();
struct ErrScope {
    explicit ErrScope(int32_t* word);
    ~ErrScope();
    ErrScope(const ErrScope&) = delete;
    ErrScope& operator=(const ErrScope&) = delete;
    int32_t* prev;
};
// Test stall of the tensor-core matmul for launches made from now on: cycles > 0 bounds its
// barrier waits by `cycles` and makes its fold warps first wait on a barrier that nothing
// completes (so the error path runs); 0 = normal operation with the built-in bound (about one
// second).  Set only through the test hook of the C ABI.
long long tc_test_wait_cycles();
void set_tc_test_wait_cycles(long long cycles);

// One-time set-up per device (function attributes such as the dynamic shared-memory limit apply
// to the device that is current when they are set): ensure() runs setup(dev, &value) once for the
// current device, under a mutex, and reports whether it succeeded; value is what setup stored.
struct PerDeviceOnce {
    static constexpr int kMaxDevices = 64;
    template <class F>
    bool ensure(F&& setup, int* value_out = nullptr) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return false;
        std::lock_guard<std::mutex> lk(mu);
        if (state[dev] == 0) state[dev] = setup(dev, &value[dev]) ? 1 : -1;
        if (value_out) *value_out = value[dev];
        return state[dev] == 1;
    }
    std::mutex mu;
    signed char state[kMaxDevices] = {};   // 0 not yet, 1 usable, -1 set-up failed
    int value[kMaxDevices] = {};
};

template <typename... KArgs, typename... Args>
inline void launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// GGUF tensor types.  Q5_0 only occurs in files: the loader expands it to the Q8_0 layout (int8
// values and a per-block scale), whose kernels compute its dot exactly as ggml does.
enum WType : int { W_F32 = 0, W_F16 = 1, W_Q4_0 = 2, W_Q5_0 = 6, W_Q8_0 = 8, W_Q4_K = 12 };

// A linear weight [N rows][K] repacked for the device.
//   Q8_0: q8 [N][K] int8, d [N][K/32] f32 (the f16 block scales widened)
//   Q4_0: q4 [N][K/32][16] (ggml nibble order: low nibble j -> element j, high -> j+16), d as Q8_0
//   Q4_K: q4 [N][K/256][128] (ggml order), d, dmin [N][K/256] f32, scm [N][K/256][16] = the
//         eight 6-bit sub-block scales then the eight 6-bit mins
//   F16 : h [N][K];  F32: f [N][K]
struct DevW {
    int type = -1, N = 0, K = 0;
    const int8_t* q8 = nullptr;
    const int8_t* tcw = nullptr;   // Q4_K: int8 planes [3][tc_npad][K] for the tcgen05 path (see repack)
    int tc_npad = 0;
    const uint8_t* q4 = nullptr;
    const float* d = nullptr;
    const float* dmin = nullptr;
    const uint8_t* scm = nullptr;
    const uint16_t* h = nullptr;
    const float* f = nullptr;
};

// Activations converted to a weight type's dot type (ggml vec_dot_type):
//   Q8_0/Q4_0 weights -> q [M][K] int8 + d [M][K/32] (f16-rounded scales as f32)
//   Q4_K weights      -> q [M][K] int8 + d [M][K/256] f32 + bs [M][K/32] (sum of each 32 group)
//   F16 weights       -> h [M][K];  F32 weights -> f [M][K] (the input itself)
struct ActQ {
    int8_t* q = nullptr;
    float* d = nullptr;
    int32_t* bs = nullptr;
    uint16_t* h = nullptr;
    const float* f = nullptr;
};

// Paged f16 KV cache, layer-major: page p holds kPage positions, and each layer's slices of all
// n_pages pages are one contiguous region (an attention launch reads one layer, so its pages lie
// in n_pages * 128 KB of address space instead of spread over the whole pool);
// element (layer, p, kv, head, pos, dim) at
//   pool[(((((size_t)layer * n_pages + p) * 2 + kv) * kHeads + head) * kPage + pos) * kHeadDim + dim]
struct KVView {
    uint16_t* pool = nullptr;
    const int32_t* ptab = nullptr;  // [n_slots][max_pages]
    int max_pages = 0;
    int n_layer = 0;
    int n_pages = 0;                // pages in the pool
};

// Per-row routing of one forward pass (rows = tokens of this pass).
struct Rows {
    const int32_t* slot = nullptr;  // [T] slot of the row
    int32_t* pos = nullptr;         // [T] KV position written by the row
    int32_t* L = nullptr;           // [T] attended prefix length
    const int32_t* cap = nullptr;   // [n_slots] capacity (positions) of the slot
    int32_t* err = nullptr;         // device error flag (bounds)
};

// Output of the QKV projection routed by rows: Q as f16 [T][512], K and V as f16 into the pages.
struct QKVStore {
    Rows rows;
    KVView kv;
    int layer = 0;
    uint16_t* q16 = nullptr;
};

// Work done by the last CTA of a small-M (<= 32 rows) matmul after all its outputs are written:
// kind 1: y_out = LN(resid + y) * g + beta, plus y_out in dot type qtype into qo;
// kind 2: y (M x N) in dot type qtype into qo.
struct Tail {
    int kind = 0;
    const float* resid = nullptr;
    const float* g = nullptr;
    const float* beta = nullptr;
    float eps = 1e-5f;
    float* y_out = nullptr;
    int qtype = -1;
    ActQ qo;
    int32_t* counter = nullptr;   // zero-initialised; reset by the tail
};

struct Epi {
    const QKVStore* qkv = nullptr;
    const Tail* tail = nullptr;
    // The activations are only in a.f (f32): Q8_0/Q4_0 weights for at most 8 rows quantise them
    // inside the few-row kernel; otherwise matmul converts them (quantize_act) first.
    bool quant_in = false;
};

void quantize_act(int wtype, const float* x, int M, int K, ActQ& a, cudaStream_t st);
// Input of a few-row matmul that starts with y_out = LN(a + b) * g + beta (rows of kD; CTA 0
// stores y_out).
constexpr int kLnRows = 2;
struct LnIn {
    const float* a = nullptr;
    const float* b = nullptr;
    const float* g = nullptr;
    const float* beta = nullptr;
    float eps = 1e-5f;
    float* y_out = nullptr;
};
// false (nothing launched) unless Q8_0/Q4_0 weights with K == kD and 1..kLnRows rows
bool matmul_ln(const DevW& W, const LnIn& ln, int M, const float* bias, int relu, float* y, const QKVStore* qkv,
               cudaStream_t st);
void matmul(const DevW& W, const ActQ& a, int M, const float* bias, int relu, float* y, cudaStream_t st,
            const Epi& epi = Epi());
// tcgen05 path (TMA-fed, TMEM accumulators; Q4_K weights) for large M; false if not supported.
// int8 tensor-core peak probe (t2sx_tc.cu): one launch on every SM; false if not launchable
bool probe_i8_mma(int iters, int issuers, int32_t* err, cudaStream_t st, int* ctas);
bool matmul_tc(const DevW& W, const ActQ& a, int M, const float* bias, int relu, float* y, const QKVStore* qkv,
               cudaStream_t st);
// Rows from which matmul() takes the tcgen05 path (T2SX_TC_MIN_ROWS overrides).
int tc_min_rows();
// mma.sync path with 32-weight-row tiles for M <= 32 (enough CTAs when there are few rows).
bool matmul_mma_narrow(const DevW& W, const ActQ& a, int M, const float* bias, int relu, float* y, const QKVStore* qkv,
                       cudaStream_t st);
// Quantised weights, 33 to T2SX_SK_MAX_ROWS rows: split-K tiles; false: nothing launched.
bool matmul_sk_mid(const DevW& W, const ActQ& a, int M, const float* bias, int relu, float* y, const QKVStore* qkv,
                   cudaStream_t st);
// F16 weights, 1-256 rows, K a multiple of 256 up to 2048: split-K tiles; false: nothing launched.
bool matmul_f16_sk(const DevW& W, const ActQ& a, int M, const float* bias, int relu, float* y, const QKVStore* qkv,
                   cudaStream_t st);
// Rows from which matmul() takes the narrow mma.sync path instead of the per-row kernel
// (T2SX_NARROW_MIN_ROWS overrides).
int narrow_min_rows();
// Tensor-core path (mma.sync s8) for M > 32; false if the shape is not supported.
bool matmul_mma(const DevW& W, const ActQ& a, int M, const float* bias, int relu, float* y, const QKVStore* qkv,
                cudaStream_t st);
void embed_decode(int T, const int32_t* row_slot, const int32_t* token_in, const int32_t* n_pos,
                  const int32_t* audio_off, const uint16_t* emb16, const float* emb32, int emb_rows,
                  const float* pe, int pe_rows, float alpha, Rows rows, float* x, int qtype, ActQ qo, cudaStream_t st);
void attention_decode(int T, const uint16_t* q16, Rows rows, KVView kv, int layer, float scale, float* out, int qtype,
                      ActQ qo, cudaStream_t st);
void attention_rows(int T, int row0, const int2* groups, int n_groups, const uint16_t* q16, Rows rows, KVView kv, int layer,
                    float scale, float* out, int qtype, ActQ qo, cudaStream_t st);
// y = LN(a + b) * g + beta over T rows of kD (and y in dot type qtype into qo).  With a programmatic
// launch a is read before the wait: it must have been written two or more launches back.
void residual_layernorm(int T, const float* a, const float* b, const float* g, const float* beta, float eps,
                        float* y, int qtype, ActQ qo, cudaStream_t st);
// Logit given to EOS when EOS is masked (finite, so the masked-lerp filters stay finite).
constexpr float kEosMasked = -1.0e30f;
void sample_greedy(int T, const float* logits, int V, const int32_t* row_slot, const uint8_t* seen, float rp,
                   float inv_rp, int eos_mask, int eos, int32_t* tok_out, int32_t* greedy_out, cudaStream_t st);
struct SamplerArgs {
    int top_k;
    float top_p;
    float inv_t;       // 1 / max(temperature, 1e-5)
    float rp, inv_rp;  // repetition penalty and its reciprocal
    int eos_mask, eos;
    const float* noise;  // [rows][V] Exp(1) noise by sorted position, or null (greedy)
};
void sample_full(int T, const float* logits, int V, const int32_t* row_slot, const uint8_t* seen, const SamplerArgs& a,
                 int32_t* tok_out, int32_t* greedy_out, cudaStream_t st);
void advance(int T, const int32_t* row_slot, const int32_t* tok, int32_t* token_in, int32_t* n_pos, uint8_t* seen,
             int V, int32_t* ring, int ring_len, int32_t* ring_step, cudaStream_t st);
// extract-latent: im2col of the width-2 stride-2 Conv1d (cols [To][2C]) and the nearest-code pick
void im2col_k2s2(int To, int C, const float* x, float* cols, cudaStream_t st);
void code_argmax(int To, int NC, const float* score, const float* half_norm, int32_t* codes, cudaStream_t st);
void gather_rows(int n, const float* src, const int32_t* idx, int ld, float* dst, cudaStream_t st);
void embed_prefill_rows(int T_text, int T_prompt, const int32_t* phones, const int32_t* sem, const float* bert_proj,
                        const uint16_t* text16, const float* text32, const uint16_t* audio16, const float* audio32,
                        const float* pe, float alpha_t, float alpha_a, float* x, cudaStream_t st);

}  // namespace t2sx
