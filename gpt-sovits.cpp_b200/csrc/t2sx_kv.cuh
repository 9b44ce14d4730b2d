// Paged KV cache addressing and f16 row loads shared by the attention and matmul kernels.
#pragma once
#include "t2sx_kernels.cuh"
#include "t2sx_math.cuh"

namespace t2sx {

// Element offset of (layer, page, K|V, head, position in page, dim 0) in the page pool (layer-major).
__device__ __forceinline__ size_t kv_off(const KVView& kv, int page, int layer, int which, int head, int pos_in_page) {
    return (((((size_t)layer * kv.n_pages + page) * 2 + which) * kHeads + head) * kPage + pos_in_page) * kHeadDim;
}

// Elements of one page (K and V of every head) and of its K (or V) half: kv_off is linear in the
// page, so a kernel can hold (layer, head) fixed in a base pointer and add page and position.
constexpr size_t kPageElems = (size_t)2 * kHeads * kPage * kHeadDim;
constexpr int kHalfPageElems = kHeads * kPage * kHeadDim;
__device__ __forceinline__ const uint16_t* kv_head_base(const KVView& kv, int layer, int head) {
    return kv.pool + kv_off(kv, 0, layer, 0, head, 0);
}

// cp.async copies global -> shared (16 or 4 bytes; a false `valid` copies nothing and zero-fills),
// grouped per thread by commit; wait until at most N of this thread's groups are pending.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    const int n = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(n));
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem, bool valid) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    const int n = valid ? 4 : 0;
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(s), "l"(gmem), "r"(n));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// 32 f16 values (four 16-byte chunks, in order) -> f32
__device__ __forceinline__ void unpack_row32(const uint4 (&u4)[4], float* out) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const uint32_t w[4] = {u4[c].x, u4[c].y, u4[c].z, u4[c].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            out[c * 8 + 2 * e] = h2f((uint16_t)(w[e] & 0xffffu));
            out[c * 8 + 2 * e + 1] = h2f((uint16_t)(w[e] >> 16));
        }
    }
}

// four 16-byte chunks -> 16 words of packed f16 pairs, in order
__device__ __forceinline__ void words16(const uint4 (&u4)[4], uint32_t (&w)[16]) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        w[4 * c] = u4[c].x; w[4 * c + 1] = u4[c].y; w[4 * c + 2] = u4[c].z; w[4 * c + 3] = u4[c].w;
    }
}

// 32 consecutive f16 values at p (16-byte aligned) as 16 packed pairs
__device__ __forceinline__ void load_row32_h(const uint16_t* p, uint32_t (&w)[16]) {
    const uint4* p4 = reinterpret_cast<const uint4*>(p);
    const uint4 u[4] = {p4[0], p4[1], p4[2], p4[3]};
    words16(u, w);
}

// 32 consecutive f16 values at p (16-byte aligned) -> f32
__device__ __forceinline__ void load_row32(const uint16_t* p, float* out) {
    const uint4* p4 = reinterpret_cast<const uint4*>(p);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const uint4 u = p4[c];
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            out[c * 8 + 2 * e] = h2f((uint16_t)(w[e] & 0xffffu));
            out[c * 8 + 2 * e + 1] = h2f((uint16_t)(w[e] >> 16));
        }
    }
}

// QKV projection output element (row m, column n) -> Q as f16 for attention, K / V as f16 into
// the row's cache page (ggml_set_rows into an F16 cache, block.cpp:557-573).
__device__ __forceinline__ void qkv_store(const QKVStore& e, int m, int n, float v) {
    const uint16_t h = f2h(v);
    if (n < kD) { e.q16[(size_t)m * kD + n] = h; return; }
    const int pos = e.rows.pos[m];
    const int s = e.rows.slot[m];
    if (pos < 0 || pos >= e.rows.cap[s]) return;
    const int page = e.kv.ptab[(size_t)s * e.kv.max_pages + pos / kPage];
    const int which = (n - kD) / kD, j = (n - kD) % kD;
    e.kv.pool[kv_off(e.kv, page, e.layer, which, j / kHeadDim, pos % kPage) + (j % kHeadDim)] = h;
}

// qkv_store in two steps, for kernels that look the destination up ahead of the dot products:
// qkv_dest gives row m's cache page and position ((-1, 0): no K/V store, as qkv_store skips a
// position outside the slot's capacity).  Its capacity and page-table loads are independent
// (the page-table index is clamped), so they cost one round trip after the position and slot.
__device__ __forceinline__ int2 qkv_dest(const QKVStore& e, int pos, int s) {
    const int pg = min(max(pos, 0) / kPage, e.kv.max_pages - 1);
    const int cap = e.rows.cap[s];
    const int page = e.kv.ptab[(size_t)s * e.kv.max_pages + pg];
    return (pos < 0 || pos >= cap) ? make_int2(-1, 0) : make_int2(page, pos);
}

__device__ __forceinline__ void qkv_store_at(const QKVStore& e, int m, int n, float v, int2 dst) {
    const uint16_t h = f2h(v);
    if (n < kD) { e.q16[(size_t)m * kD + n] = h; return; }
    if (dst.x < 0) return;
    const int which = (n - kD) / kD, j = (n - kD) % kD;
    e.kv.pool[kv_off(e.kv, dst.x, e.layer, which, j / kHeadDim, dst.y % kPage) + (j % kHeadDim)] = h;
}

}  // namespace t2sx
