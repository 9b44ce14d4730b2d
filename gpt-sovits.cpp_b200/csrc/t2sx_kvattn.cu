// Isolated batched attention over a paged f16 KV cache (one layer).
//
// The reference computes attention inside t2s_attention_block_forward (src/t2s/block.cpp:575-608)
// on its session cache; these entry points run the attention kernel of the decode step and the
// prefill (k_attn_decode) on a stand-alone cache, so the attention can be checked and measured on
// its own at batched-attention shapes (many sequences, long prefixes, causal prefill rows).
// Pages have the session layout with one layer: element (page, kv, head, pos, dim) at
// (((page * 2 + kv) * 16 + head) * 64 + pos) * 32 + dim; sequence s owns pages
// [s * pages_per_seq, (s + 1) * pages_per_seq).
#include "../../include/t2sx.h"
#include "t2sx_kernels.cuh"
#include "t2sx_math.cuh"

#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <memory>
#include <vector>

using namespace t2sx;

int t2sx_set_error(int code, const char* msg);

namespace {

// K and V rows [len][16][32] (staged on the device) -> positions pos0.. of sequence seq
__global__ void k_kv_scatter(int len, int pos0, int seq, const uint16_t* __restrict__ k, const uint16_t* __restrict__ v,
                             KVView kv) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;   // one thread per (position, head, 8 dims)
    if (i >= len * kHeads * 4) return;
    const int p = i / (kHeads * 4), h = (i / 4) % kHeads, d0 = (i % 4) * 8;
    const int pos = pos0 + p;
    const int page = kv.ptab[(size_t)seq * kv.max_pages + pos / kPage];
    const size_t src = ((size_t)p * kHeads + h) * kHeadDim + d0;
#pragma unroll
    for (int which = 0; which < 2; ++which) {
        const size_t dst = ((((size_t)page * 2 + which) * kHeads + h) * kPage + pos % kPage) * kHeadDim + d0;
        *reinterpret_cast<uint4*>(kv.pool + dst) = *reinterpret_cast<const uint4*>((which ? v : k) + src);
    }
}

}  // namespace

struct t2sx_kvcache {
    int device = 0, n_seqs = 0, max_len = 0, pages_per_seq = 0;
    uint16_t* pool = nullptr;
    int32_t* ptab = nullptr;
    int32_t* cap = nullptr;
    int32_t* err = nullptr;
    uint16_t* stage = nullptr;   // K then V rows of one write
    size_t stage_rows = 0;
    int32_t* rows_mem = nullptr;  // slot [cap_rows], L [cap_rows], groups [cap_rows] of int2
    size_t cap_rows = 0;
    cudaStream_t st = nullptr;
};

#define KCK(x)                                                                                          \
    do {                                                                                                \
        cudaError_t e_ = (x);                                                                           \
        if (e_ != cudaSuccess) {                                                                        \
            char m_[256];                                                                               \
            snprintf(m_, sizeof(m_), "%s: %s", #x, cudaGetErrorString(e_));                             \
            return t2sx_set_error(T2SX_ERR_CUDA, m_);                                                   \
        }                                                                                               \
    } while (0)

static void kv_release(t2sx_kvcache* c) {
    if (!c) return;
    DeviceGuard dg_;
    dg_.set(c->device);
    if (c->st) cudaStreamSynchronize(c->st);
    cudaFree(c->pool); cudaFree(c->ptab); cudaFree(c->cap); cudaFree(c->err); cudaFree(c->stage); cudaFree(c->rows_mem);
    if (c->st) cudaStreamDestroy(c->st);
    delete c;
}

extern "C" int t2sx_kvcache_create(int32_t device, int32_t n_seqs, int32_t max_len, t2sx_kvcache** out) {
    if (!out || n_seqs <= 0 || max_len <= 0 || (int64_t)n_seqs * max_len > (int64_t)1 << 31)
        return t2sx_set_error(T2SX_ERR_INVALID, "t2sx_kvcache_create: bad arguments");
    *out = nullptr;
    DeviceGuard dg_;
    KCK(dg_.set(device));
    std::unique_ptr<t2sx_kvcache, void (*)(t2sx_kvcache*)> c(new t2sx_kvcache(), kv_release);
    c->device = device; c->n_seqs = n_seqs; c->max_len = max_len;
    c->pages_per_seq = (max_len + kPage - 1) / kPage;
    const size_t npages = (size_t)n_seqs * c->pages_per_seq;
    const size_t page_elems = (size_t)2 * kHeads * kPage * kHeadDim;
    if (cudaMalloc(&c->pool, npages * page_elems * 2) != cudaSuccess) {
        cudaGetLastError();
        return t2sx_set_error(T2SX_ERR_OOM, "t2sx_kvcache_create: out of device memory for the pages");
    }
    KCK(cudaMemset(c->pool, 0, npages * page_elems * 2));
    std::vector<int32_t> pt(npages), cap(n_seqs, c->pages_per_seq * kPage);
    for (size_t i = 0; i < npages; ++i) pt[i] = (int32_t)i;
    KCK(cudaMalloc(&c->ptab, npages * 4));
    KCK(cudaMemcpy(c->ptab, pt.data(), npages * 4, cudaMemcpyHostToDevice));
    KCK(cudaMalloc(&c->cap, (size_t)n_seqs * 4));
    KCK(cudaMemcpy(c->cap, cap.data(), (size_t)n_seqs * 4, cudaMemcpyHostToDevice));
    KCK(cudaMalloc(&c->err, 4));
    KCK(cudaMemset(c->err, 0, 4));
    KCK(cudaStreamCreateWithFlags(&c->st, cudaStreamNonBlocking));
    *out = c.release();
    return T2SX_OK;
}

extern "C" void t2sx_kvcache_free(t2sx_kvcache* c) { kv_release(c); }

extern "C" int t2sx_kvcache_write(t2sx_kvcache* c, int32_t seq, int32_t pos0, int32_t len, const uint16_t* k,
                                  const uint16_t* v) {
    if (!c || !k || !v || seq < 0 || seq >= c->n_seqs || pos0 < 0 || len <= 0 || (int64_t)pos0 + len > c->max_len)
        return t2sx_set_error(T2SX_ERR_INVALID, "t2sx_kvcache_write: bad arguments");
    DeviceGuard dg_;
    KCK(dg_.set(c->device));
    const size_t row = (size_t)kHeads * kHeadDim;
    if (c->stage_rows < (size_t)len) {
        KCK(cudaStreamSynchronize(c->st));
        cudaFree(c->stage);
        c->stage = nullptr;
        c->stage_rows = 0;
        KCK(cudaMalloc(&c->stage, (size_t)len * row * 2 * 2));
        c->stage_rows = (size_t)len;
    }
    KCK(cudaMemcpyAsync(c->stage, k, (size_t)len * row * 2, cudaMemcpyHostToDevice, c->st));
    KCK(cudaMemcpyAsync(c->stage + (size_t)len * row, v, (size_t)len * row * 2, cudaMemcpyHostToDevice, c->st));
    KVView kv;
    kv.pool = c->pool; kv.ptab = c->ptab; kv.max_pages = c->pages_per_seq; kv.n_layer = 1;
    kv.n_pages = c->n_seqs * c->pages_per_seq;
    const int threads = len * kHeads * 4;
    k_kv_scatter<<<(threads + 255) / 256, 256, 0, c->st>>>(len, pos0, seq, c->stage, c->stage + (size_t)len * row, kv);
    KCK(cudaGetLastError());
    KCK(cudaStreamSynchronize(c->st));
    return T2SX_OK;
}

// Routes rows (sequence, prefix length) to the device; returns the Rows view.
static int kv_rows(t2sx_kvcache* c, int32_t n, const int32_t* seqs, const int32_t* lens, Rows* r, cudaStream_t st) {
    for (int32_t i = 0; i < n; ++i)
        if (seqs[i] < 0 || seqs[i] >= c->n_seqs || lens[i] <= 0 || lens[i] > c->max_len)
            return t2sx_set_error(T2SX_ERR_INVALID, "attention rows: sequence id or length out of range");
    if (c->cap_rows < (size_t)n) {
        KCK(cudaStreamSynchronize(st));
        KCK(cudaStreamSynchronize(c->st));
        cudaFree(c->rows_mem);
        c->rows_mem = nullptr;
        c->cap_rows = 0;
        KCK(cudaMalloc(&c->rows_mem, (size_t)n * 4 * 4));   // slot, L, then up to n groups of (first row, rows)
        c->cap_rows = (size_t)n;
    }
    KCK(cudaMemcpyAsync(c->rows_mem, seqs, (size_t)n * 4, cudaMemcpyHostToDevice, st));
    KCK(cudaMemcpyAsync(c->rows_mem + c->cap_rows, lens, (size_t)n * 4, cudaMemcpyHostToDevice, st));
    Rows rows;
    rows.slot = c->rows_mem;
    rows.L = c->rows_mem + c->cap_rows;
    rows.pos = nullptr;
    rows.cap = c->cap;
    rows.err = c->err;
    *r = rows;
    return T2SX_OK;
}

static int kv_attn(t2sx_kvcache* c, int32_t n, const int32_t* seqs, const int32_t* lens, const uint16_t* q, float* out,
                   void* stream, bool grouped) {
    if (!c || n <= 0 || !seqs || !lens || !q || !out) return t2sx_set_error(T2SX_ERR_INVALID, "attention: bad arguments");
    DeviceGuard dg_;
    KCK(dg_.set(c->device));
    cudaStream_t st = (cudaStream_t)stream;
    Rows rows;
    int rc = kv_rows(c, n, seqs, lens, &rows, st);
    if (rc) return rc;
    KVView kv;
    kv.pool = c->pool; kv.ptab = c->ptab; kv.max_pages = c->pages_per_seq; kv.n_layer = 1;
    kv.n_pages = c->n_seqs * c->pages_per_seq;
    const float scale = 1.0f / sqrtf((float)kHeadDim);
    int n_groups = 0;
    if (grouped && n >= 64) {
        // runs of up to 16 consecutive rows of one sequence (the rows of a prompt)
        std::vector<int2> g;
        for (int r = 0; r < n;) {
            int k = 1;
            while (r + k < n && k < 16 && seqs[r + k] == seqs[r]) ++k;
            g.push_back(make_int2(r, k));
            r += k;
        }
        KCK(cudaMemcpyAsync(c->rows_mem + 2 * c->cap_rows, g.data(), g.size() * sizeof(int2), cudaMemcpyHostToDevice, st));
        n_groups = (int)g.size();
    }
    attention_rows(n, 0, reinterpret_cast<const int2*>(c->rows_mem + 2 * c->cap_rows), n_groups, q, rows, kv, 0, scale, out, -1,
                   ActQ(), st);
    KCK(cudaGetLastError());
    return T2SX_OK;
}

extern "C" int t2sx_kvcache_attn_decode(t2sx_kvcache* c, int32_t n, const int32_t* seqs, const int32_t* lens,
                                        const uint16_t* q, float* out, void* stream) {
    return kv_attn(c, n, seqs, lens, q, out, stream, false);
}

extern "C" int t2sx_kvcache_attn_prefill(t2sx_kvcache* c, int32_t n, const int32_t* seqs, const int32_t* lens,
                                         const uint16_t* q, float* out, void* stream) {
    // the same result as t2sx_kvcache_attn_decode; consecutive rows of one sequence share the staged K/V
    return kv_attn(c, n, seqs, lens, q, out, stream, true);
}
