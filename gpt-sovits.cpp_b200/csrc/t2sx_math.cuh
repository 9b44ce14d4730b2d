// Device arithmetic of the T2S decode path.
//
// Every reduction in the kernels follows one fixed evaluation order so that results are
// reproducible bit for bit (the CPU oracle restates the same order).  All code here is
// compiled with --fmad=false: a fused multiply-add appears only where it is written as
// __fmaf_rn, everything else rounds after each operation.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

namespace t2sx {

constexpr int kD = 512;        // d_model
constexpr int kHeads = 16;
constexpr int kHeadDim = 32;
constexpr int kPage = 64;      // KV positions per page
constexpr int kAttnLanes = 32;   // decode attention: position lanes per (row, head)

// e^x: Cody-Waite reduction x = k*ln2 + r (ln2 split in a 16-bit head and a tail so k*head
// is exact), e^r from its Taylor series to degree 7 in Horner form with fused multiply-adds,
// scaled by 2^k assembled from exponent bits.  Arguments <= -87 (and -inf, NaN) give 0; the
// kernels only evaluate e^(s - max) <= 1.
__device__ __forceinline__ float t2s_expf(float x) {
    if (!(x > -87.0f)) return 0.0f;
    if (x > 88.0f) return __int_as_float(0x7f800000);
    const float kf = rintf(__fmul_rn(x, 1.44269502162933349609375f));
    float r = __fmaf_rn(kf, -0.693145751953125f, x);
    r = __fmaf_rn(kf, -1.428606765330187045037746429443359375e-06f, r);
    float p = 1.98412701138295233249664306640625e-04f;
    p = __fmaf_rn(p, r, 1.3888889225199818611145019531250e-03f);
    p = __fmaf_rn(p, r, 8.3333337679505348205566406250000e-03f);
    p = __fmaf_rn(p, r, 4.1666667908430099487304687500000e-02f);
    p = __fmaf_rn(p, r, 1.6666667163372039794921875000000e-01f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const int k = (int)kf;
    return __fmul_rn(p, __int_as_float((k + 127) << 23));
}

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }

// Online softmax state of one attention lane.
struct AttnState {
    float m, l, o[kHeadDim];
};

__device__ __forceinline__ void st_empty(AttnState& s) {
    s.m = __int_as_float(0xff800000);
    s.l = 0.0f;
#pragma unroll
    for (int d = 0; d < kHeadDim; ++d) s.o[d] = 0.0f;
}

// Fold one key position (score s, value row v as f32) into the state.
__device__ __forceinline__ void st_update(AttnState& st, float s, const float* v) {
    // the weight before the branch (fsub(m, s) = -fsub(s, m) exactly): lanes that take the two
    // sides apart share the exponential
    const float t = t2s_expf(-fabsf(__fsub_rn(s, st.m)));
    if (s > st.m) {
        st.m = s;
        st.l = __fmaf_rn(st.l, t, 1.0f);
#pragma unroll
        for (int d = 0; d < kHeadDim; ++d) st.o[d] = __fmaf_rn(st.o[d], t, v[d]);
    } else {
        st.l = __fadd_rn(st.l, t);
#pragma unroll
        for (int d = 0; d < kHeadDim; ++d) st.o[d] = __fmaf_rn(t, v[d], st.o[d]);
    }
}

// st_update with the value row as 16 packed f16 pairs, converted element by element inside the
// update (the same values and operations as st_update on the converted row).
__device__ __forceinline__ void st_update_h(AttnState& st, float s, const uint32_t (&vw)[kHeadDim / 2]) {
    const float t = t2s_expf(-fabsf(__fsub_rn(s, st.m)));
    if (s > st.m) {
        st.m = s;
        st.l = __fmaf_rn(st.l, t, 1.0f);
#pragma unroll
        for (int w = 0; w < kHeadDim / 2; ++w) {
            st.o[2 * w] = __fmaf_rn(st.o[2 * w], t, h2f((uint16_t)(vw[w] & 0xffffu)));
            st.o[2 * w + 1] = __fmaf_rn(st.o[2 * w + 1], t, h2f((uint16_t)(vw[w] >> 16)));
        }
    } else {
        st.l = __fadd_rn(st.l, t);
#pragma unroll
        for (int w = 0; w < kHeadDim / 2; ++w) {
            st.o[2 * w] = __fmaf_rn(t, h2f((uint16_t)(vw[w] & 0xffffu)), st.o[2 * w]);
            st.o[2 * w + 1] = __fmaf_rn(t, h2f((uint16_t)(vw[w] >> 16)), st.o[2 * w + 1]);
        }
    }
}

// Symmetric merge of two states: merge(A,B) == merge(B,A) bit for bit.
__device__ __forceinline__ void st_merge_scalars(float mA, float lA, float mB, float lB, float& M, float& a,
                                                 float& b, float& l, bool& empty) {
    M = fmaxf(mA, mB);
    empty = (M == __int_as_float(0xff800000));
    a = empty ? 0.0f : t2s_expf(__fsub_rn(mA, M));
    b = empty ? 0.0f : t2s_expf(__fsub_rn(mB, M));
    l = empty ? 0.0f : __fadd_rn(__fmul_rn(lA, a), __fmul_rn(lB, b));
}

// Two steps of an fma chain on packed f16 pairs: c = fma(a.lo, b.lo, c), then c = fma(a.hi, b.hi, c)
// (element 2i in the low half of word i).  sm_100's mixed-precision fma takes the f16 operands as
// they are (their conversion to f32 is exact) and rounds once, so each step is the same value as
// __fmaf_rn(h2f(a), h2f(b), c), without the two conversions.
__device__ __forceinline__ float fma_h2(uint32_t a2, uint32_t b2, float c) {
    asm("{\n.reg .f16 al, ah, bl, bh;\nmov.b32 {al, ah}, %1;\nmov.b32 {bl, bh}, %2;\n"
        "fma.rn.f32.f16 %0, al, bl, %0;\nfma.rn.f32.f16 %0, ah, bh, %0;\n}\n"
        : "+f"(c)
        : "r"(a2), "r"(b2));
    return c;
}

// 32-term dot of an f16 query with an f16 key row, both held as 16 packed f16 pairs: four
// sequential fma chains of 8 terms (the products of two f16 values are exact in f32), summed
// pairwise as (c0 + c1) + (c2 + c3).
__device__ __forceinline__ float dot32_h(const uint32_t (&q)[16], const uint32_t (&k)[16]) {
    float c[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        float s = 0.0f;
#pragma unroll
        for (int w = 4 * j; w < 4 * j + 4; ++w) s = fma_h2(q[w], k[w], s);
        c[j] = s;
    }
    return __fadd_rn(__fadd_rn(c[0], c[1]), __fadd_rn(c[2], c[3]));
}

}  // namespace t2sx

namespace t2sx {

// ---- warp-level quantisation of activations (the rules of the k_quant_* kernels) ----------

__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
    return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

// Q8_0 of one 32-element block held one value per lane (x86 AVX2 rule of ggml's
// quantize_row_q8_0): amax, d = amax/127 stored as f16, id = 127/amax, q = rint(v*id).
// Lane 0 writes the scale (as the f32 value of the f16) to *d_slot.
__device__ __forceinline__ int q8_0_lane(float v, float* d_slot, int lane) {
    const float a = warp_max_f(fabsf(v));
    const float dd = __fdiv_rn(a, 127.0f);
    const float id = (a != 0.0f) ? __fdiv_rn(127.0f, a) : 0.0f;
    float r = rintf(__fmul_rn(v, id));
    r = fminf(fmaxf(r, -128.0f), 127.0f);
    if (lane == 0) *d_slot = __half2float(__float2half_rn(dd));
    return (int)r;
}

// q8_0_lane's rule for a whole 32-element block in one thread (the |x| maximum is the same in
// any order, so it is taken as a tree): the block's bytes as the activation buffer holds them
// (little-endian, elements 0-15 in lo, 16-31 in hi) and its f16-rounded scale.
__device__ __forceinline__ void q8_0_block_regs(const float4 (&x4)[8], int4& lo, int4& hi, float& d) {
    float v[32];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        v[4 * i] = x4[i].x; v[4 * i + 1] = x4[i].y; v[4 * i + 2] = x4[i].z; v[4 * i + 3] = x4[i].w;
    }
    float t[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) t[i] = fmaxf(fabsf(v[i]), fabsf(v[i + 16]));
#pragma unroll
    for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
        for (int i = 0; i < w; ++i) t[i] = fmaxf(t[i], t[i + w]);
    const float a = t[0];
    const float dd = __fdiv_rn(a, 127.0f);
    const float id = (a != 0.0f) ? __fdiv_rn(127.0f, a) : 0.0f;
    int w[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        uint32_t p = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            float r = rintf(__fmul_rn(v[4 * j + k], id));
            r = fminf(fmaxf(r, -128.0f), 127.0f);
            p |= ((uint32_t)(int)r & 0xffu) << (8 * k);
        }
        w[j] = (int)p;
    }
    lo = make_int4(w[0], w[1], w[2], w[3]);
    hi = make_int4(w[4], w[5], w[6], w[7]);
    d = __half2float(__float2half_rn(dd));
}

// the same from 32 floats at x (16-byte aligned)
__device__ __forceinline__ void q8_0_block_thread(const float* __restrict__ x, int4& lo, int4& hi, float& d) {
    float4 x4[8];
    const float4* xp = reinterpret_cast<const float4*>(x);
#pragma unroll
    for (int i = 0; i < 8; ++i) x4[i] = xp[i];
    q8_0_block_regs(x4, lo, hi, d);
}

// Running (|x| max, signed value, first index) of a Q8_K block (ggml quantize_row_q8_K_ref).
struct AbsMax {
    float a, m;
    int i;
};
__device__ __forceinline__ void absmax_take(AbsMax& s, float v, int idx) {
    const float a = fabsf(v);
    if (a > s.a || (a == s.a && a > 0.0f && idx < s.i)) { s.a = a; s.m = v; s.i = idx; }
}
__device__ __forceinline__ void absmax_merge(AbsMax& s, const AbsMax& o) {
    if (o.a > s.a || (o.a == s.a && o.i < s.i)) s = o;
}
__device__ __forceinline__ AbsMax absmax_warp(AbsMax s) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        AbsMax o;
        o.a = __shfl_xor_sync(0xffffffffu, s.a, off);
        o.m = __shfl_xor_sync(0xffffffffu, s.m, off);
        o.i = __shfl_xor_sync(0xffffffffu, s.i, off);
        absmax_merge(s, o);
    }
    return s;
}
// iscale = -127/max of the block (0 for an all-zero block); d = 1/iscale (0 for all-zero).
__device__ __forceinline__ float q8k_iscale(const AbsMax& s) { return s.a == 0.0f ? 0.0f : __fdiv_rn(-127.0f, s.m); }
__device__ __forceinline__ float q8k_d(float iscale) { return iscale == 0.0f ? 0.0f : __fdiv_rn(1.0f, iscale); }
__device__ __forceinline__ int q8k_q(float iscale, float v) {
    if (iscale == 0.0f) return 0;
    const float r = rintf(__fmul_rn(iscale, v));
    return r > 127.0f ? 127 : (int)r;
}

}  // namespace t2sx

namespace t2sx {
// Programmatic dependent launch (sm_90+): `pdl_trigger` lets the next kernel in the stream begin
// launching; `pdl_wait` blocks until the preceding kernel has completed and its writes are
// visible.  Every kernel triggers only after its own wait, so a kernel that starts early overlaps
// its predecessor alone: before pdl_wait it may read constants (weights, page tables, K/V of
// earlier steps) and data of kernels two or more launches back, never its predecessor's output.
// Both are no-ops when the kernel was launched without the programmatic-serialization attribute.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
}  // namespace t2sx
