// T2S decode-path oracle -- TEST INFRASTRUCTURE ONLY (see t2s_oracle.h).
//
// Restates, from operator definitions, what the reference's ggml CPU graph computes for one
// T2S layer / step, and fixes the float evaluation order of every reduction.  The CUDA
// library reproduces these orders exactly, so GPU and oracle agree bit for bit.
//
// Reference call sites followed (paths inside zpeng11/GPT-SoVITS.cpp):
//   decode embedding      src/t2s/session.cpp:337-344   x = emb[tok] + pe[pos]*alpha
//   PE table              src/t2s/session.cpp:33-53     [sin_j, cos_j] pairs, host libm
//   attention layer       src/t2s/block.cpp:513-637     QKV, set_rows, flash-attn, out-proj,
//                                                       post-norm LN1, FFN(ReLU), post-norm LN2
//   sampler               src/t2s/block.cpp:117-138,221,273-348 (repetition penalty, argmax)
//   prefill embedding     src/t2s/block.cpp:424-511
//   prefill mask / offset src/t2s/session.cpp:773-784,819-824
//   decode advance        src/t2s/session.cpp:247-284
//   GGUF names / defaults src/t2s/loader.cpp:39-134, python/convert_t2s_to_gguf.py:95-228
//
// ggml semantics restated (ggml itself is absent from the reference snapshot):
//   mul_mat     the f32 activation row is converted to the weight type's dot type first:
//               Q8_0, Q5_0 and Q4_0 weights -> Q8_0 activations (x86 AVX2 rule: id = 127/amax,
//               round-half-even, scale stored f16); Q4_K -> Q8_K (ggml reference rule: scale
//               -127/max, f32); F16 -> f16 (round-half-even); F32 stays f32.  Per block the
//               integer dot is exact.  Float order (fixed here): blocks in increasing order,
//               acc = fma(d_w*d_x, (float)isum, acc); Q4_K keeps a separate fma accumulator for
//               the min terms and adds the two at the end; F16/F32 sum each 32-element block
//               with a sequential fma chain and add block sums in order.
//   norm        ggml_norm with double (ggml_float) sums; summation order fixed as 32 lanes of
//               strided sequential sums combined by an xor butterfly.
//   flash_attn  K/V rounded to f16 by set_rows, Q rounded to f16; score = 32-term dot (4
//               sequential fma chains of 8, summed pairwise) * (1/sqrt(32)); softmax-weighted V
//               accumulated in f32 with the online (running-max) update.  Every row (decode and
//               prefill): 32 position lanes (lane = pos mod 32) merged by an xor butterfly.
//               ggml's F16-V kernel keeps its VKQ accumulator in f16; this order keeps f32.
//   exp         own Cody-Waite + degree-7 Taylor polynomial (t2s_expf below), identical on GPU.
#include "t2s_oracle.h"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>
#include <map>
#include <algorithm>
#ifdef _OPENMP
#include <omp.h>
#endif

// ============================================================================================
// f16 conversion (IEEE 754 binary16, round-to-nearest-even)
// ============================================================================================
static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

static inline float h2f(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1f;
    const uint32_t man = h & 0x3ffu;
    if (exp == 0) {
        // zero or subnormal: man * 2^-24, exact in f32
        float v = (float)man * 5.9604644775390625e-08f;
        return u2f(f2u(v) | sign);
    }
    if (exp == 31) return u2f(sign | 0x7f800000u | (man << 13));
    return u2f(sign | ((exp + 112) << 23) | (man << 13));
}

static inline uint16_t f2h(float f) {
    const uint32_t u = f2u(f);
    const uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    const uint32_t au = u & 0x7fffffffu;
    if (au >= 0x7f800000u) {  // inf or nan
        return (uint16_t)(sign | 0x7c00u | (au > 0x7f800000u ? 0x200u : 0u));
    }
    if (au >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);  // rounds to >= 65520 -> inf
    const int e = (int)(au >> 23) - 127;
    if (e >= -14) {
        // normal f16: keep 10 mantissa bits, round half to even on the 13 dropped bits
        uint32_t man = au & 0x7fffffu;
        uint32_t hexp = (uint32_t)(e + 15);
        uint32_t val = (hexp << 10) | (man >> 13);
        uint32_t rem = man & 0x1fffu;
        if (rem > 0x1000u || (rem == 0x1000u && (val & 1u))) val += 1;  // may carry into exp
        return (uint16_t)(sign | val);
    }
    // subnormal f16 (or zero): value = round(|f| * 2^24) * 2^-24
    if (e < -25) return sign;  // |f| < 2^-25 rounds to zero (2^-25 exactly ties to even 0)
    uint32_t man = (au & 0x7fffffu) | 0x800000u;  // 24-bit significand, value man * 2^(e-23)
    int shift = -e - 1;  // bits to drop so that result unit is 2^-24: (e-23) + shift = -24
    // shift in [14, 24]
    uint32_t q = man >> shift;
    uint32_t rem = man & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (q & 1u))) q += 1;
    return (uint16_t)(sign | q);
}

// ============================================================================================
// exp: Cody-Waite range reduction x = k*ln2 + r with ln2 = LN2_HI + LN2_LO (LN2_HI has 16
// significant bits so k*LN2_HI is exact), e^r by its Taylor series to degree 7 evaluated with
// fused multiply-adds, then scaled by 2^k built from exponent bits.  Arguments below -87 give 0
// (all uses are softmax weights e^(s - max) <= 1).
// ============================================================================================
static inline float t2s_expf(float x) {
    if (!(x > -87.0f)) return 0.0f;          // also -inf and NaN
    if (x > 88.0f) return INFINITY;
    const float kf = rintf(x * 1.44269502162933349609375f);      // log2(e) rounded to f32
    float r = fmaf(kf, -0.693145751953125f, x);                  // LN2_HI
    r = fmaf(kf, -1.428606765330187045037746429443359375e-06f, r);  // LN2_LO
    float p = 1.98412701138295233249664306640625e-04f;           // 1/5040
    p = fmaf(p, r, 1.3888889225199818611145019531250e-03f);       // 1/720
    p = fmaf(p, r, 8.3333337679505348205566406250000e-03f);       // 1/120
    p = fmaf(p, r, 4.1666667908430099487304687500000e-02f);       // 1/24
    p = fmaf(p, r, 1.6666667163372039794921875000000e-01f);       // 1/6
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    const int k = (int)kf;
    return p * u2f((uint32_t)(k + 127) << 23);
}

// ============================================================================================
// quantisation formats
// ============================================================================================
struct BlkQ8 { float d; int8_t qs[32]; };                    // activation Q8_0 (d = f16 value)
struct BlkQ8K { float d; int8_t qs[256]; int16_t bsums[16]; };

static inline uint16_t rd16(const uint8_t* p) { uint16_t v; memcpy(&v, p, 2); return v; }

static void q4k_scale_min(const uint8_t* sc, int j, int& s, int& m) {
    if (j < 4) { s = sc[j] & 63; m = sc[j + 4] & 63; }
    else {
        s = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
        m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
    }
}

// Element i (0..31) of a Q5_0 block as a signed integer in [-16, 15] (ggml dequantize_row_q5_0:
// elements j and j + 16 share byte j of qs, low and high nibble; bit j / j + 16 of qh is the fifth bit).
static int q5_0_value(const uint8_t* blk, int i) {
    uint32_t qh;
    memcpy(&qh, blk + 2, 4);
    const int j = i & 15;
    const int lo = (i < 16) ? (blk[6 + j] & 0xF) : (blk[6 + j] >> 4);
    return (lo | (int)(((qh >> i) & 1u) << 4)) - 16;
}

int64_t orc_row_bytes(int type, int64_t n) {
    switch (type) {
        case ORC_F32: return n * 4;
        case ORC_F16: return n * 2;
        case ORC_Q8_0: return n / 32 * 34;
        case ORC_Q4_0: return n / 32 * 18;
        case ORC_Q5_0: return n / 32 * 22;
        case ORC_Q4_K: return n / 256 * 144;
    }
    return -1;
}

void orc_dequantize(int type, const void* data, int64_t n, float* out) {
    const uint8_t* p = (const uint8_t*)data;
    switch (type) {
        case ORC_F32: memcpy(out, p, n * 4); break;
        case ORC_F16: for (int64_t i = 0; i < n; ++i) out[i] = h2f(rd16(p + 2 * i)); break;
        case ORC_Q8_0:
            for (int64_t b = 0; b < n / 32; ++b) {
                const uint8_t* blk = p + b * 34;
                float d = h2f(rd16(blk));
                for (int i = 0; i < 32; ++i) out[b * 32 + i] = (float)(int8_t)blk[2 + i] * d;
            }
            break;
        case ORC_Q4_0:
            for (int64_t b = 0; b < n / 32; ++b) {
                const uint8_t* blk = p + b * 18;
                float d = h2f(rd16(blk));
                for (int i = 0; i < 16; ++i) {
                    out[b * 32 + i] = (float)((blk[2 + i] & 0xF) - 8) * d;
                    out[b * 32 + 16 + i] = (float)((blk[2 + i] >> 4) - 8) * d;
                }
            }
            break;
        case ORC_Q5_0:   // ggml block_q5_0: f16 d, uint32 qh (fifth bits), 16 bytes of low nibbles
            for (int64_t b = 0; b < n / 32; ++b) {
                const uint8_t* blk = p + b * 22;
                float d = h2f(rd16(blk));
                for (int i = 0; i < 32; ++i) out[b * 32 + i] = (float)q5_0_value(blk, i) * d;
            }
            break;
        case ORC_Q4_K:
            for (int64_t b = 0; b < n / 256; ++b) {
                const uint8_t* blk = p + b * 144;
                float d = h2f(rd16(blk)), dmin = h2f(rd16(blk + 2));
                const uint8_t* sc = blk + 4;
                const uint8_t* qs = blk + 16;
                for (int c = 0; c < 4; ++c) {
                    int s1, m1, s2, m2;
                    q4k_scale_min(sc, 2 * c, s1, m1);
                    q4k_scale_min(sc, 2 * c + 1, s2, m2);
                    const float d1 = d * (float)s1, mm1 = dmin * (float)m1;
                    const float d2 = d * (float)s2, mm2 = dmin * (float)m2;
                    for (int l = 0; l < 32; ++l) {
                        out[b * 256 + 64 * c + l] = d1 * (float)(qs[32 * c + l] & 0xF) - mm1;
                        out[b * 256 + 64 * c + 32 + l] = d2 * (float)(qs[32 * c + l] >> 4) - mm2;
                    }
                }
            }
            break;
    }
}

// Activation -> Q8_0, x86 AVX2 rule of ggml's quantize_row_q8_0: amax over the block,
// d = amax/127 stored as f16, id = 127/amax (0 if amax == 0), q = round-half-even(x*id).
static void quant_q8_0(const float* x, int64_t n, BlkQ8* out, uint8_t* raw) {
    for (int64_t b = 0; b < n / 32; ++b) {
        const float* xb = x + b * 32;
        float amax = 0.0f;
        for (int i = 0; i < 32; ++i) { float a = fabsf(xb[i]); if (a > amax) amax = a; }
        const float d = amax / 127.0f;
        const uint16_t dh = f2h(d);
        const float id = (amax != 0.0f) ? 127.0f / amax : 0.0f;
        int8_t q[32];
        for (int i = 0; i < 32; ++i) {
            float v = rintf(xb[i] * id);
            v = v > 127.0f ? 127.0f : (v < -128.0f ? -128.0f : v);
            q[i] = (int8_t)v;
        }
        if (out) { out[b].d = h2f(dh); memcpy(out[b].qs, q, 32); }
        if (raw) { memcpy(raw + b * 34, &dh, 2); memcpy(raw + b * 34 + 2, q, 32); }
    }
}

// Activation -> Q8_K, ggml quantize_row_q8_K_ref rule: max = signed value of largest |x|
// (first occurrence), iscale = -127/max, q = min(127, round-half-even(iscale*x)), d = 1/iscale.
static void quant_q8_K(const float* x, int64_t n, BlkQ8K* out) {
    for (int64_t b = 0; b < n / 256; ++b) {
        const float* xb = x + b * 256;
        float amax = 0.0f, mx = 0.0f;
        for (int i = 0; i < 256; ++i) { float a = fabsf(xb[i]); if (a > amax) { amax = a; mx = xb[i]; } }
        BlkQ8K& o = out[b];
        if (amax == 0.0f) { o.d = 0.0f; memset(o.qs, 0, 256); memset(o.bsums, 0, 32); continue; }
        const float iscale = -127.0f / mx;
        for (int i = 0; i < 256; ++i) {
            float v = rintf(iscale * xb[i]);
            o.qs[i] = (int8_t)(v > 127.0f ? 127 : (int)v);
        }
        for (int j = 0; j < 16; ++j) {
            int s = 0;
            for (int i = 0; i < 16; ++i) s += o.qs[16 * j + i];
            o.bsums[j] = (int16_t)s;
        }
        o.d = 1.0f / iscale;
    }
}

void orc_quantize_q8_0(const float* x, int64_t n, uint8_t* out) { quant_q8_0(x, n, nullptr, out); }
void orc_quantize_q8_K(const float* x, int64_t n, uint8_t* out) {
    std::vector<BlkQ8K> q(n / 256);
    quant_q8_K(x, n, q.data());
    for (size_t b = 0; b < q.size(); ++b) {
        uint8_t* o = out + b * 292;
        memcpy(o, &q[b].d, 4); memcpy(o + 4, q[b].qs, 256); memcpy(o + 260, q[b].bsums, 32);
    }
}

// Quantised activation row, prepared once per row for a given weight type.
struct ActRow {
    int type = -1;
    std::vector<BlkQ8> q8;
    std::vector<BlkQ8K> q8k;
    std::vector<float> f;   // f32 values of f16-rounded (F16) or raw (F32) activations
};

static void prep_act(int wtype, const float* x, int64_t K, ActRow& a) {
    a.type = wtype;
    if (wtype == ORC_Q8_0 || wtype == ORC_Q4_0 || wtype == ORC_Q5_0) { a.q8.resize(K / 32); quant_q8_0(x, K, a.q8.data(), nullptr); }
    else if (wtype == ORC_Q4_K) { a.q8k.resize(K / 256); quant_q8_K(x, K, a.q8k.data()); }
    else if (wtype == ORC_F16) { a.f.resize(K); for (int64_t i = 0; i < K; ++i) a.f[i] = h2f(f2h(x[i])); }
    else { a.f.assign(x, x + K); }
}

// Canonical dot of one weight row with one prepared activation row.
static float qdot(int wtype, const uint8_t* w, int64_t K, const ActRow& a) {
    if (wtype == ORC_Q8_0) {
        float acc = 0.0f;
        for (int64_t b = 0; b < K / 32; ++b) {
            const uint8_t* wb = w + b * 34;
            const int8_t* qw = (const int8_t*)(wb + 2);
            int isum = 0;
            for (int i = 0; i < 32; ++i) isum += (int)qw[i] * (int)a.q8[b].qs[i];
            const float dd = h2f(rd16(wb)) * a.q8[b].d;
            acc = fmaf(dd, (float)isum, acc);
        }
        return acc;
    }
    if (wtype == ORC_Q4_0) {
        float acc = 0.0f;
        for (int64_t b = 0; b < K / 32; ++b) {
            const uint8_t* wb = w + b * 18;
            int isum = 0;
            for (int i = 0; i < 16; ++i) {
                isum += ((int)(wb[2 + i] & 0xF) - 8) * (int)a.q8[b].qs[i];
                isum += ((int)(wb[2 + i] >> 4) - 8) * (int)a.q8[b].qs[16 + i];
            }
            const float dd = h2f(rd16(wb)) * a.q8[b].d;
            acc = fmaf(dd, (float)isum, acc);
        }
        return acc;
    }
    if (wtype == ORC_Q5_0) {   // ggml_vec_dot_q5_0_q8_0: integer block dot, then the Q8_0 fold
        float acc = 0.0f;
        for (int64_t b = 0; b < K / 32; ++b) {
            const uint8_t* wb = w + b * 22;
            int isum = 0;
            for (int i = 0; i < 32; ++i) isum += q5_0_value(wb, i) * (int)a.q8[b].qs[i];
            const float dd = h2f(rd16(wb)) * a.q8[b].d;
            acc = fmaf(dd, (float)isum, acc);
        }
        return acc;
    }
    if (wtype == ORC_Q4_K) {
        float acc_a = 0.0f, acc_m = 0.0f;
        for (int64_t b = 0; b < K / 256; ++b) {
            const uint8_t* wb = w + b * 144;
            const BlkQ8K& x = a.q8k[b];
            const uint8_t* sc = wb + 4;
            const uint8_t* qs = wb + 16;
            int sumi_a = 0, sumi_m = 0;
            for (int j = 0; j < 8; ++j) {
                int s, m;
                q4k_scale_min(sc, j, s, m);
                const int c = j >> 1, sh = (j & 1) * 4;
                int isum = 0;
                for (int l = 0; l < 32; ++l) isum += (int)((qs[32 * c + l] >> sh) & 0xF) * (int)x.qs[32 * j + l];
                sumi_a += s * isum;
                sumi_m += m * ((int)x.bsums[2 * j] + (int)x.bsums[2 * j + 1]);
            }
            const float d = x.d * h2f(rd16(wb));
            const float dmin = -x.d * h2f(rd16(wb + 2));
            acc_a = fmaf(d, (float)sumi_a, acc_a);
            acc_m = fmaf(dmin, (float)sumi_m, acc_m);
        }
        return acc_a + acc_m;
    }
    // F16 / F32: per 32-element block a sequential fma chain from zero, block sums added in order
    float acc = 0.0f;
    for (int64_t b = 0; b < K / 32; ++b) {
        float s = 0.0f;
        for (int i = 0; i < 32; ++i) {
            const int64_t k = b * 32 + i;
            const float wv = (wtype == ORC_F16) ? h2f(rd16(w + 2 * k)) : u2f(f2u(((const float*)w)[k]));
            s = fmaf(wv, a.f[k], s);
        }
        acc = acc + s;
    }
    return acc;
}

// A quantised weight row unpacked once per matmul call into plain int8 values and per-block
// scales, so the per-activation-row dot is a contiguous int8 x int8 loop.  The integer block sums
// and the float fold (operands and order) are exactly those of qdot above; only the unpacking of
// the nibbles / 5th bits / 6-bit scales moves out of the per-row loop.
struct WRowX {
    std::vector<int8_t> q;      // [K] element values (Q4_0: nibble - 8; Q5_0: 5-bit - 16; Q4_K: 0..15)
    std::vector<float> dw;      // Q8_0/Q4_0/Q5_0: f16 block scale as f32 [K/32]
    std::vector<int> sc, mn;    // Q4_K: 6-bit scale / min of each 32-element sub-block [K/32]
    std::vector<float> d, dmin; // Q4_K: super-block d / dmin as f32 [K/256]
};

static void expand_row(int wtype, const uint8_t* w, int64_t K, WRowX& e) {
    e.q.resize(K);
    if (wtype == ORC_Q4_K) {
        e.sc.resize(K / 32); e.mn.resize(K / 32); e.d.resize(K / 256); e.dmin.resize(K / 256);
        for (int64_t b = 0; b < K / 256; ++b) {
            const uint8_t* wb = w + b * 144;
            e.d[b] = h2f(rd16(wb)); e.dmin[b] = h2f(rd16(wb + 2));
            const uint8_t* qs = wb + 16;
            for (int j = 0; j < 8; ++j) {
                q4k_scale_min(wb + 4, j, e.sc[b * 8 + j], e.mn[b * 8 + j]);
                const int c = j >> 1, sh = (j & 1) * 4;
                for (int l = 0; l < 32; ++l) e.q[b * 256 + 32 * j + l] = (int8_t)((qs[32 * c + l] >> sh) & 0xF);
            }
        }
        return;
    }
    e.dw.resize(K / 32);
    for (int64_t b = 0; b < K / 32; ++b) {
        int8_t* q = &e.q[b * 32];
        if (wtype == ORC_Q8_0) {
            const uint8_t* wb = w + b * 34;
            e.dw[b] = h2f(rd16(wb));
            memcpy(q, wb + 2, 32);
        } else if (wtype == ORC_Q4_0) {
            const uint8_t* wb = w + b * 18;
            e.dw[b] = h2f(rd16(wb));
            for (int i = 0; i < 16; ++i) { q[i] = (int8_t)((wb[2 + i] & 0xF) - 8); q[16 + i] = (int8_t)((wb[2 + i] >> 4) - 8); }
        } else {   // Q5_0
            const uint8_t* wb = w + b * 22;
            e.dw[b] = h2f(rd16(wb));
            for (int i = 0; i < 32; ++i) q[i] = (int8_t)q5_0_value(wb, i);
        }
    }
}

static inline int dot32_i8(const int8_t* a, const int8_t* b) {
    int s = 0;
    for (int i = 0; i < 32; ++i) s += (int)a[i] * (int)b[i];
    return s;
}

static float qdot_x(int wtype, const WRowX& e, int64_t K, const ActRow& a) {
    if (wtype == ORC_Q4_K) {
        float acc_a = 0.0f, acc_m = 0.0f;
        for (int64_t b = 0; b < K / 256; ++b) {
            const BlkQ8K& x = a.q8k[b];
            int sumi_a = 0, sumi_m = 0;
            for (int j = 0; j < 8; ++j) {
                const int isum = dot32_i8(&e.q[b * 256 + 32 * j], &x.qs[32 * j]);
                sumi_a += e.sc[b * 8 + j] * isum;
                sumi_m += e.mn[b * 8 + j] * ((int)x.bsums[2 * j] + (int)x.bsums[2 * j + 1]);
            }
            const float d = x.d * e.d[b];
            const float dmin = -x.d * e.dmin[b];
            acc_a = fmaf(d, (float)sumi_a, acc_a);
            acc_m = fmaf(dmin, (float)sumi_m, acc_m);
        }
        return acc_a + acc_m;
    }
    float acc = 0.0f;
    for (int64_t b = 0; b < K / 32; ++b) {
        const int isum = dot32_i8(&e.q[b * 32], a.q8[b].qs);
        const float dd = e.dw[b] * a.q8[b].d;
        acc = fmaf(dd, (float)isum, acc);
    }
    return acc;
}

// ---- ggml-order dot products ---------------------------------------------------------------
// The float folds of ggml's generic (scalar) vec_dot kernels, restated from their published
// definitions: the same integer block sums as above, folded the way those kernels fold them.
//   Q8_0 x Q8_0 : sumf += (float)sumi * (d_w * d_x)
//   Q4_0 x Q8_0 : sumf += ((float)sumi * d_w) * d_x
//   Q5_0 x Q8_0 : sumf += (d_w * d_x) * (float)sumi
//   Q4_K x Q8_K : per super-block eight integer lane sums aux[l] (element e -> lane e % 8) of
//                 scale_j * q_w * q_x; sums[l] += (d_w * d_x) * aux[l]; sumf -= (dmin_w * d_x) * sumi_m;
//                 after the last super-block sumf += sums[0..7] in order
//   F16 x F16   : double sum of the f32 products, rounded to f32 once
//   F32 x F32   : double sum of the f32 products, rounded to f32 once
// These are the ISA-independent forms; ggml's SIMD builds split the sums over vector lanes
// differently per instruction set, so no single order is "the" ggml order.
static float qdot_x_ggml(int wtype, const WRowX& e, int64_t K, const ActRow& a) {
    if (wtype == ORC_Q4_K) {
        float sums[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        float sumf = 0.0f;
        for (int64_t b = 0; b < K / 256; ++b) {
            const BlkQ8K& x = a.q8k[b];
            int aux[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            for (int j = 0; j < 8; ++j)
                for (int l = 0; l < 32; ++l)
                    aux[l & 7] += e.sc[b * 8 + j] * ((int)e.q[b * 256 + 32 * j + l] * (int)x.qs[32 * j + l]);
            int sumi = 0;
            for (int j = 0; j < 16; ++j) sumi += (int)x.bsums[j] * e.mn[b * 8 + j / 2];
            const float d = e.d[b] * x.d;
            for (int l = 0; l < 8; ++l) sums[l] = sums[l] + d * (float)aux[l];
            const float dmin = e.dmin[b] * x.d;
            sumf = sumf - dmin * (float)sumi;
        }
        for (int l = 0; l < 8; ++l) sumf = sumf + sums[l];
        return sumf;
    }
    float sumf = 0.0f;
    for (int64_t b = 0; b < K / 32; ++b) {
        const float sumi = (float)dot32_i8(&e.q[b * 32], a.q8[b].qs);
        const float dw = e.dw[b], dx = a.q8[b].d;
        float t;
        if (wtype == ORC_Q8_0) t = sumi * (dw * dx);
        else if (wtype == ORC_Q4_0) t = (sumi * dw) * dx;
        else t = (dw * dx) * sumi;   // Q5_0
        sumf = sumf + t;
    }
    return sumf;
}

static float fdot_ggml(int wtype, const uint8_t* w, int64_t K, const ActRow& a) {
    double sumf = 0.0;
    for (int64_t k = 0; k < K; ++k) {
        const float wv = (wtype == ORC_F16) ? h2f(rd16(w + 2 * k)) : ((const float*)w)[k];
        sumf += (double)(wv * a.f[k]);
    }
    return (float)sumf;
}

static int matmul_impl(int wtype, const void* w, int64_t N, int64_t K, const float* x, int64_t M, float* y, int ggml_order) {
    const int64_t rb = orc_row_bytes(wtype, K);
    if (rb <= 0) return -1;
    std::vector<ActRow> acts(M);
    for (int64_t m = 0; m < M; ++m) prep_act(wtype, x + m * K, K, acts[m]);
    const bool quant = wtype == ORC_Q8_0 || wtype == ORC_Q4_0 || wtype == ORC_Q5_0 || wtype == ORC_Q4_K;
    if (ggml_order) {
        #pragma omp parallel
        {
            WRowX e;
            #pragma omp for schedule(static)
            for (int64_t n = 0; n < N; ++n) {
                const uint8_t* wr = (const uint8_t*)w + n * rb;
                if (quant) expand_row(wtype, wr, K, e);
                for (int64_t m = 0; m < M; ++m)
                    y[m * N + n] = quant ? qdot_x_ggml(wtype, e, K, acts[m]) : fdot_ggml(wtype, wr, K, acts[m]);
            }
        }
        return 0;
    }
    if (!quant || M < 2) {
        #pragma omp parallel for schedule(static)
        for (int64_t n = 0; n < N; ++n)
            for (int64_t m = 0; m < M; ++m)
                y[m * N + n] = qdot(wtype, (const uint8_t*)w + n * rb, K, acts[m]);
        return 0;
    }
    #pragma omp parallel
    {
        WRowX e;
        #pragma omp for schedule(static)
        for (int64_t n = 0; n < N; ++n) {
            expand_row(wtype, (const uint8_t*)w + n * rb, K, e);
            for (int64_t m = 0; m < M; ++m) y[m * N + n] = qdot_x(wtype, e, K, acts[m]);
        }
    }
    return 0;
}

int orc_matmul(int wtype, const void* w, int64_t N, int64_t K, const float* x, int64_t M, float* y) {
    return matmul_impl(wtype, w, N, K, x, M, y, 0);
}
int orc_matmul_ggml(int wtype, const void* w, int64_t N, int64_t K, const float* x, int64_t M, float* y) {
    return matmul_impl(wtype, w, N, K, x, M, y, 1);
}

// ============================================================================================
// LayerNorm (ggml_norm + mul + add), double sums in the fixed 32-lane butterfly order
// ============================================================================================
static double lanes_sum(double* lane) {
    double t[32];
    for (int off = 16; off >= 1; off >>= 1) {
        for (int l = 0; l < 32; ++l) t[l] = lane[l] + lane[l ^ off];
        memcpy(lane, t, sizeof(t));
    }
    return lane[0];
}

void orc_layernorm(const float* x, const float* g, const float* b, int n, float eps, float* y) {
    double lane[32] = {0};
    for (int l = 0; l < 32; ++l)
        for (int t = 0; t < n / 32; ++t) lane[l] += (double)x[l + 32 * t];
    const float mean = (float)(lanes_sum(lane) / (double)n);
    std::vector<float> v(n);
    for (int i = 0; i < n; ++i) v[i] = x[i] - mean;
    double lane2[32] = {0};
    for (int l = 0; l < 32; ++l)
        for (int t = 0; t < n / 32; ++t) { const float vv = v[l + 32 * t] * v[l + 32 * t]; lane2[l] += (double)vv; }
    const float var = (float)(lanes_sum(lane2) / (double)n);
    const float scale = 1.0f / sqrtf(var + eps);
    for (int i = 0; i < n; ++i) y[i] = (v[i] * scale) * g[i] + b[i];
}

// ggml_norm as its CPU kernel defines it: sequential double sums, mean and variance rounded to
// f32, y = (x - mean) * (1/sqrtf(var + eps)); then ggml_mul by gamma and ggml_add of beta.
static void layernorm_ggml(const float* x, const float* g, const float* b, int n, float eps, float* y) {
    double sum = 0.0;
    for (int i = 0; i < n; ++i) sum += (double)x[i];
    const float mean = (float)(sum / (double)n);
    double sum2 = 0.0;
    for (int i = 0; i < n; ++i) { const float v = x[i] - mean; y[i] = v; sum2 += (double)(v * v); }
    const float var = (float)(sum2 / (double)n);
    const float scale = 1.0f / sqrtf(var + eps);
    for (int i = 0; i < n; ++i) y[i] = (y[i] * scale) * g[i] + b[i];
}

// ============================================================================================
// attention
// ============================================================================================
struct AttnState { float m, l, o[32]; };
static inline void st_empty(AttnState& s) { s.m = -INFINITY; s.l = 0.0f; for (int d = 0; d < 32; ++d) s.o[d] = 0.0f; }

static inline float dot32(const float* q, const uint16_t* k) {
    float c[4];
    for (int j = 0; j < 4; ++j) {
        float s = 0.0f;
        for (int d = 8 * j; d < 8 * j + 8; ++d) s = fmaf(q[d], h2f(k[d]), s);
        c[j] = s;
    }
    return (c[0] + c[1]) + (c[2] + c[3]);
}

static inline void st_update(AttnState& st, float s, const uint16_t* v) {
    if (s > st.m) {
        const float t = t2s_expf(st.m - s);
        st.m = s;
        st.l = fmaf(st.l, t, 1.0f);
        for (int d = 0; d < 32; ++d) st.o[d] = fmaf(st.o[d], t, h2f(v[d]));
    } else {
        const float t = t2s_expf(s - st.m);
        st.l = st.l + t;
        for (int d = 0; d < 32; ++d) st.o[d] = fmaf(t, h2f(v[d]), st.o[d]);
    }
}

static inline AttnState st_merge(const AttnState& A, const AttnState& B) {
    AttnState R;
    const float M = fmaxf(A.m, B.m);
    if (M == -INFINITY) { st_empty(R); return R; }
    const float a = t2s_expf(A.m - M), b = t2s_expf(B.m - M);
    R.m = M;
    R.l = A.l * a + B.l * b;
    for (int d = 0; d < 32; ++d) R.o[d] = A.o[d] * a + B.o[d] * b;
    return R;
}

static const float kAttnScale = 1.0f / sqrtf(32.0f);
static const int kAttnLanes = 32;

// q holds the f32 values of the f16-rounded query.  32 position lanes (lane = position mod 32,
// ascending within a lane), merged in the order of an xor butterfly (partners 16, 8, 4, 2, 1).
static void attn_decode_head(const float* q, const uint16_t* k, const uint16_t* v, int L,
                             int64_t stride, float* out) {
    AttnState lane[kAttnLanes];
    for (auto& s : lane) st_empty(s);
    for (int i = 0; i < L; ++i) {
        const float s = dot32(q, k + i * stride) * kAttnScale;
        st_update(lane[i % kAttnLanes], s, v + i * stride);
    }
    for (int off = 16; off >= 1; off >>= 1) {
        AttnState t[kAttnLanes];
        for (int l = 0; l < kAttnLanes; ++l) t[l] = st_merge(lane[l], lane[l ^ off]);
        for (int l = 0; l < kAttnLanes; ++l) lane[l] = t[l];
    }
    const AttnState& R = lane[0];
    const float inv = 1.0f / R.l;
    for (int d = 0; d < 32; ++d) out[d] = R.o[d] * inv;
}

// ggml_flash_attn_ext's CPU kernel for one query row and head, as it defines it: positions in
// increasing order, score = double sum of the f32 products q_d * k_d rounded to f32, times the
// scale; online softmax with libm expf (M running maximum, S running sum: S = S * ms + vs); the
// V accumulator VKQ is f16 for an F16 cache (every rescale and every multiply-add rounded back to
// f16) and f32 for an F32 cache; out = VKQ * (1/S).  q holds f16-rounded values for an F16 cache
// and the raw f32 values for an F32 cache.  kf/vf: F32 cache rows (used when k16 is null).
static void attn_head_ggml(const float* q, const uint16_t* k16, const uint16_t* v16, const float* kf, const float* vf,
                           int L, int64_t stride, float* out) {
    float M = -INFINITY, S = 0.0f;
    uint16_t vkq16[32];
    float vkq32[32];
    for (int d = 0; d < 32; ++d) { vkq16[d] = 0; vkq32[d] = 0.0f; }
    for (int i = 0; i < L; ++i) {
        double acc = 0.0;
        if (k16) for (int d = 0; d < 32; ++d) acc += (double)(q[d] * h2f(k16[i * stride + d]));
        else for (int d = 0; d < 32; ++d) acc += (double)(q[d] * kf[i * stride + d]);
        float s = (float)acc * kAttnScale;
        s = s + 0.0f;   // the mask value of a visible position
        const float Mold = M;
        float ms = 1.0f, vs = 1.0f;
        if (s > M) {
            M = s;
            ms = expf(Mold - M);
            if (v16) for (int d = 0; d < 32; ++d) vkq16[d] = f2h(h2f(vkq16[d]) * ms);
            else for (int d = 0; d < 32; ++d) vkq32[d] = vkq32[d] * ms;
        } else {
            vs = expf(s - M);
        }
        if (v16) for (int d = 0; d < 32; ++d) vkq16[d] = f2h(h2f(vkq16[d]) + h2f(v16[i * stride + d]) * vs);
        else for (int d = 0; d < 32; ++d) vkq32[d] = vkq32[d] + vf[i * stride + d] * vs;
        S = S * ms + vs;
    }
    const float inv = (S == 0.0f) ? 0.0f : 1.0f / S;
    for (int d = 0; d < 32; ++d) out[d] = (v16 ? h2f(vkq16[d]) : vkq32[d]) * inv;
}

void orc_attn_decode(const float* q, const uint16_t* k, const uint16_t* v, int L, float* out) {
    float qh[32];
    for (int d = 0; d < 32; ++d) qh[d] = h2f(f2h(q[d]));
    attn_decode_head(qh, k, v, L, 32, out);
}
// Batched attention rows (the per-head functions above, positions strided by 16 heads x 32 dims).
// Used for batched-attention shapes (many sessions attending over a paged f16 cache).
void orc_attn_rows(int n, const int* seqs, const int* lens, const uint16_t* q16, const uint16_t* k,
                   const uint16_t* v, int max_len, float* out) {
#pragma omp parallel for schedule(dynamic, 4)
    for (int64_t rh = 0; rh < (int64_t)n * 16; ++rh) {
        const int r = (int)(rh / 16), h = (int)(rh % 16);
        float qh[32];
        for (int d = 0; d < 32; ++d) qh[d] = h2f(q16[(size_t)r * 512 + h * 32 + d]);
        const size_t base = ((size_t)seqs[r] * max_len) * 512 + (size_t)h * 32;
        attn_decode_head(qh, k + base, v + base, lens[r], 512, out + (size_t)r * 512 + h * 32);
    }
}

float orc_expf(float x) { return t2s_expf(x); }
uint16_t orc_f32_to_f16(float x) { return f2h(x); }
float orc_f16_to_f32(uint16_t h) { return h2f(h); }

// PE row (session.cpp:33-53; same expression as ggml_timestep_embedding for block.cpp:350-401)
void orc_pe_row(int pos, int d_model, float* out) {
    const int half = d_model / 2;
    for (int j = 0; j < half; ++j) {
        const float freq = std::exp(-std::log((float)10000) * (float)j / (float)half);
        const float arg = (float)pos * freq;
        out[2 * j] = std::sin(arg);
        out[2 * j + 1] = std::cos(arg);
    }
}

// ============================================================================================
// GGUF reader
// ============================================================================================
struct Tensor { std::string name; int type; int64_t ne[4]; int nd; uint64_t off; const uint8_t* data = nullptr; };

struct Model {
    std::vector<uint8_t> file;
    std::map<std::string, Tensor> tensors;
    uint32_t hp[9] = {512, 512, 16, 2048, 24, 1025, 732, 1024, 192};
    struct Layer {
        const Tensor *qkv_w, *qkv_b, *out_w, *out_b, *ln1_w, *ln1_b, *up_w, *up_b, *down_w, *down_b, *ln2_w, *ln2_b;
    };
    std::vector<Layer> layers;
    const Tensor *text_emb, *bert_w, *bert_b, *text_alpha, *audio_emb, *audio_alpha, *lm_head;
    const Tensor *ssl_w = nullptr, *ssl_b = nullptr, *codebook = nullptr;   // extract-latent
};

struct Rd {
    const uint8_t* p; size_t n, o = 0; bool ok = true;
    template <class T> T get() { T v{}; if (o + sizeof(T) > n) { ok = false; return v; } memcpy(&v, p + o, sizeof(T)); o += sizeof(T); return v; }
    std::string str() { uint64_t l = get<uint64_t>(); if (!ok || o + l > n) { ok = false; return ""; } std::string s((const char*)p + o, l); o += l; return s; }
    void skip(uint32_t t) {
        static const int sz[] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
        if (t == 8) { str(); return; }
        if (t == 9) { uint32_t et = get<uint32_t>(); uint64_t c = get<uint64_t>(); for (uint64_t i = 0; i < c && ok; ++i) skip(et); return; }
        if (t > 12) { ok = false; return; }
        o += sz[t]; if (o > n) ok = false;
    }
};

static const float* fdata(const Tensor* t) { return (const float*)t->data; }

void* orc_model_load(const char* path) {
    FILE* f = fopen(path, "rb");
    if (!f) return nullptr;
    Model* m = new Model();
    fseek(f, 0, SEEK_END); long sz = ftell(f); fseek(f, 0, SEEK_SET);
    m->file.resize(sz);
    if (fread(m->file.data(), 1, sz, f) != (size_t)sz) { fclose(f); delete m; return nullptr; }
    fclose(f);
    Rd r{m->file.data(), m->file.size()};
    if (r.get<uint32_t>() != 0x46554747u) { delete m; return nullptr; }
    uint32_t ver = r.get<uint32_t>();
    if (ver < 2) { delete m; return nullptr; }
    uint64_t nt = r.get<uint64_t>(), nkv = r.get<uint64_t>();
    uint32_t align = 32;
    static const char* keys[9] = {"t2s.embedding_dim", "t2s.hidden_dim", "t2s.head", "t2s.linear_units", "t2s.n_layer",
                                  "t2s.vocab_size", "t2s.phoneme_vocab_size", "t2s.eos", "sovits.inter_channels"};
    for (uint64_t i = 0; i < nkv && r.ok; ++i) {
        std::string k = r.str();
        uint32_t t = r.get<uint32_t>();
        bool used = false;
        for (int j = 0; j < 9; ++j) if (k == keys[j] && t == 4) { m->hp[j] = r.get<uint32_t>(); used = true; }
        if (k == "general.alignment" && t == 4) { align = r.get<uint32_t>(); used = true; }
        if (!used) r.skip(t);
    }
    std::vector<Tensor> tl;
    for (uint64_t i = 0; i < nt && r.ok; ++i) {
        Tensor t;
        t.name = r.str();
        t.nd = (int)r.get<uint32_t>();
        for (int d = 0; d < 4; ++d) t.ne[d] = 1;
        for (int d = 0; d < t.nd && d < 4; ++d) t.ne[d] = (int64_t)r.get<uint64_t>();
        t.type = (int)r.get<uint32_t>();
        t.off = r.get<uint64_t>();
        tl.push_back(t);
    }
    if (!r.ok) { delete m; return nullptr; }
    size_t data0 = (r.o + align - 1) / align * align;
    for (auto& t : tl) {
        int64_t n = t.ne[0] * t.ne[1] * t.ne[2] * t.ne[3];
        int64_t bytes = orc_row_bytes(t.type, t.ne[0]) * (n / t.ne[0]);
        if (data0 + t.off + bytes > m->file.size()) { delete m; return nullptr; }
        t.data = m->file.data() + data0 + t.off;
        m->tensors[t.name] = t;
    }
    auto get = [&](const std::string& n) -> const Tensor* { auto it = m->tensors.find(n); return it == m->tensors.end() ? nullptr : &it->second; };
    const int nl = (int)m->hp[4];
    m->layers.resize(nl);
    for (int i = 0; i < nl; ++i) {
        auto p = "attention." + std::to_string(i) + ".";
        auto& L = m->layers[i];
        L.qkv_w = get(p + "qkv_w"); L.qkv_b = get(p + "qkv_b"); L.out_w = get(p + "out_proj_w"); L.out_b = get(p + "out_proj_b");
        L.ln1_w = get(p + "ln1_w"); L.ln1_b = get(p + "ln1_b"); L.up_w = get(p + "ffn_up_w"); L.up_b = get(p + "ffn_up_b");
        L.down_w = get(p + "ffn_down_w"); L.down_b = get(p + "ffn_down_b"); L.ln2_w = get(p + "ln2_w"); L.ln2_b = get(p + "ln2_b");
        if (!L.qkv_w || !L.qkv_b || !L.out_w || !L.out_b || !L.ln1_w || !L.ln1_b || !L.up_w || !L.up_b || !L.down_w ||
            !L.down_b || !L.ln2_w || !L.ln2_b) { delete m; return nullptr; }
    }
    m->text_emb = get("encoder.text_embedding"); m->bert_w = get("encoder.bert_proj_w"); m->bert_b = get("encoder.bert_proj_b");
    m->text_alpha = get("encoder.text_pos_alpha"); m->audio_emb = get("encoder.audio_embedding");
    m->audio_alpha = get("encoder.audio_pos_alpha"); m->lm_head = get("sampler.lm_head_w");
    m->ssl_w = get("extract_latent.ssl_proj_w"); m->ssl_b = get("extract_latent.ssl_proj_b");
    m->codebook = get("extract_latent.codebook");
    if (!m->text_emb || !m->bert_w || !m->bert_b || !m->text_alpha || !m->audio_emb || !m->audio_alpha || !m->lm_head) { delete m; return nullptr; }
    return m;
}

void orc_model_free(void* model) { delete (Model*)model; }

int orc_model_info(void* model, uint32_t* hp, int32_t* types) {
    Model* m = (Model*)model;
    for (int i = 0; i < 9; ++i) hp[i] = m->hp[i];
    if (types) {
        types[0] = m->layers[0].qkv_w->type; types[1] = m->lm_head->type;
        types[2] = m->audio_emb->type; types[3] = m->bert_w->type;
    }
    return 0;
}

// ============================================================================================
// session
// ============================================================================================
struct Session {
    Model* m;
    int n_slots, cap;
    std::vector<int> n_pos, audio_off;
    std::vector<std::vector<uint16_t>> K, V;   // [slot*L + layer] -> [cap][d]
    std::vector<float> pe;                     // [cap][d]
    // evaluation order, per operator: bit 0 the matmul folds, bit 1 LayerNorm, bit 2 flash
    // attention; a set bit follows ggml's CPU operator definition, a clear bit the canonical
    // order above (what the CUDA kernels reproduce)
    int ggml_order = 0;
    int kv_f32 = 0;                            // 1: F32 KV cache (the reference's default type)
    std::vector<std::vector<float>> Kf, Vf;    // F32 cache rows when kv_f32
};

static int g_threads = 0;
void orc_set_threads(int n) { g_threads = n; }

void* orc_session_new(void* model, int n_slots, int capacity) {
    Model* m = (Model*)model;
    if (n_slots <= 0 || capacity <= 0) return nullptr;
    Session* s = new Session();
    s->m = m; s->n_slots = n_slots; s->cap = capacity;
    s->n_pos.assign(n_slots, 0); s->audio_off.assign(n_slots, 0);
    const int d = (int)m->hp[1], nl = (int)m->hp[4];
    s->K.resize((size_t)n_slots * nl); s->V.resize((size_t)n_slots * nl);
    for (auto& k : s->K) k.assign((size_t)capacity * d, 0);
    for (auto& v : s->V) v.assign((size_t)capacity * d, 0);
    s->pe.resize((size_t)capacity * d);
    for (int p = 0; p < capacity; ++p) orc_pe_row(p, d, &s->pe[(size_t)p * d]);
    return s;
}
void orc_session_free(void* sess) { delete (Session*)sess; }
int orc_slot_release(void* sess, int slot) {
    Session* S = (Session*)sess;
    if (slot < 0 || slot >= S->n_slots) return -1;
    S->n_pos[slot] = 0;
    S->audio_off[slot] = 0;
    return 0;
}

int orc_slot_n_pos(void* sess, int slot) { return ((Session*)sess)->n_pos[slot]; }

int orc_session_set_mode(void* sess, int ggml_order, int kv_f32) {
    Session* S = (Session*)sess;
    for (int i = 0; i < S->n_slots; ++i) if (S->n_pos[i] != 0) return -1;   // set before any prefill
    S->ggml_order = (ggml_order & 7) | (kv_f32 ? 7 : 0);
    S->kv_f32 = kv_f32 ? 1 : 0;
    if (S->kv_f32 && S->Kf.empty()) {
        const size_t n = S->K.size(), per = (size_t)S->cap * S->m->hp[1];
        S->Kf.assign(n, std::vector<float>(per, 0.0f));
        S->Vf.assign(n, std::vector<float>(per, 0.0f));
    }
    return 0;
}

static void matmul_rows(const Tensor* W, const Tensor* bias, const float* x, int64_t M, float* y, int ggml_order = 0) {
    const int64_t K = W->ne[0], N = W->ne[1];
    matmul_impl(W->type, W->data, N, K, x, M, y, ggml_order);
    if (bias) {
        const float* b = fdata(bias);
        for (int64_t m = 0; m < M; ++m) for (int64_t n = 0; n < N; ++n) y[m * N + n] = y[m * N + n] + b[n];
    }
}

// Rows of one forward pass: row r belongs to slot[r], writes KV position pos[r], attends to
// prefix [0, L[r]) of its slot (32 position lanes per head, butterfly merge).
static void forward_rows(Session* S, int64_t T, const int* slot, const int* pos, const int* L,
                         float* x /* [T][d], in/out */) {
    Model* m = S->m;
    const int d = (int)m->hp[1], nl = (int)m->hp[4], F = (int)m->hp[3], H = (int)m->hp[2];
    const int hd = d / H;
    std::vector<float> qkv((size_t)T * 3 * d), attn((size_t)T * d), o((size_t)T * d), r((size_t)T * d),
        ln1((size_t)T * d), h((size_t)T * F), f((size_t)T * d);
    const int go = S->ggml_order & 1, go_norm = S->ggml_order & 2, go_attn = S->ggml_order & 4, f32kv = S->kv_f32;
    auto norm = [&](const float* in, const Tensor* g, const Tensor* b, float* out) {
        if (go_norm) layernorm_ggml(in, fdata(g), fdata(b), d, 1e-5f, out);
        else orc_layernorm(in, fdata(g), fdata(b), d, 1e-5f, out);
    };
    for (int li = 0; li < nl; ++li) {
        const Model::Layer& Lw = m->layers[li];
        matmul_rows(Lw.qkv_w, Lw.qkv_b, x, T, qkv.data(), go);
        // set_rows: K and V into the cache (f16, or f32 for an F32 cache)
        for (int64_t t = 0; t < T; ++t) {
            const size_t cs = (size_t)slot[t] * nl + li, off = (size_t)pos[t] * d;
            for (int i = 0; i < d; ++i) {
                const float kv_k = qkv[t * 3 * d + d + i], kv_v = qkv[t * 3 * d + 2 * d + i];
                if (f32kv) { S->Kf[cs][off + i] = kv_k; S->Vf[cs][off + i] = kv_v; }
                S->K[cs][off + i] = f2h(kv_k);
                S->V[cs][off + i] = f2h(kv_v);
            }
        }
        #pragma omp parallel for schedule(dynamic)
        for (int64_t th = 0; th < T * H; ++th) {
            const int64_t t = th / H; const int hh = (int)(th % H);
            const size_t cs = (size_t)slot[t] * nl + li;
            float qh[32];
            for (int i = 0; i < hd; ++i) {
                const float qv = qkv[t * 3 * d + hh * hd + i];
                qh[i] = f32kv ? qv : h2f(f2h(qv));   // an F16 cache takes an f16 query
            }
            float* o_th = &attn[t * d + hh * hd];
            if (f32kv)
                attn_head_ggml(qh, nullptr, nullptr, &S->Kf[cs][hh * hd], &S->Vf[cs][hh * hd], L[t], d, o_th);
            else if (go_attn)
                attn_head_ggml(qh, &S->K[cs][hh * hd], &S->V[cs][hh * hd], nullptr, nullptr, L[t], d, o_th);
            else
                attn_decode_head(qh, &S->K[cs][hh * hd], &S->V[cs][hh * hd], L[t], d, o_th);
        }
        matmul_rows(Lw.out_w, Lw.out_b, attn.data(), T, o.data(), go);
        for (int64_t i = 0; i < T * d; ++i) r[i] = x[i] + o[i];
        for (int64_t t = 0; t < T; ++t) norm(&r[t * d], Lw.ln1_w, Lw.ln1_b, &ln1[t * d]);
        matmul_rows(Lw.up_w, Lw.up_b, ln1.data(), T, h.data(), go);
        for (auto& v : h) v = (v > 0.0f) ? v : 0.0f;
        matmul_rows(Lw.down_w, Lw.down_b, h.data(), T, f.data(), go);
        for (int64_t i = 0; i < T * d; ++i) r[i] = ln1[i] + f[i];
        for (int64_t t = 0; t < T; ++t) norm(&r[t * d], Lw.ln2_w, Lw.ln2_b, &x[t * d]);
    }
}

// Logit given to EOS when EOS is masked (a harness rule: the reference sampler has no EOS
// input).  Finite, so that ggml's masked-lerp filters (base + m*(fill - base)) stay finite.
static const float kEosMasked = -1.0e30f;
static const float kMaskLogit = -1.0e10f;   // block.cpp:10

struct SamplerCfg { int top_k; float top_p; float temperature; float rp; int eos_mask; };

// Repetition penalty (block.cpp:117-138) as ggml's op sequence, then the EOS rule.
static void penalise(Model* m, float* logits, const float* seen, float rp, int eos_mask) {
    const int V = (int)m->hp[5];
    if (seen && rp != 1.0f) {
        const float inv = 1.0f / rp;
        for (int v = 0; v < V; ++v) {
            const float l = logits[v];
            const float pos = l * inv, neg = l * rp;
            const float negm = (-l > 0.0f) ? 1.0f : 0.0f;
            const float sel = pos + negm * (neg - pos);
            const float s = (seen[v] > 0.0f) ? 1.0f : 0.0f;
            logits[v] = l + s * (sel - l);
        }
    }
    if (eos_mask && (int)m->hp[7] < V) logits[m->hp[7]] = kEosMasked;
}

// Greedy pick (block.cpp:221, 319-323): the first index of the maximum.
static int32_t pick_greedy(Model* m, float* logits, const float* seen, float rp, int eos_mask) {
    const int V = (int)m->hp[5];
    penalise(m, logits, seen, rp, eos_mask);
    int best = 0;
    for (int v = 1; v < V; ++v) if (logits[v] > logits[best]) best = v;
    return best;
}

// ggml_soft_max over n values: e^(x - max) with the own exp, double sum (32 strided lanes
// combined by an xor butterfly), scale by (float)(1/sum).
static void softmax_canon(const float* x, int n, float* p) {
    float mx = x[0];
    for (int i = 1; i < n; ++i) if (x[i] > mx) mx = x[i];
    double lane[32] = {0};
    for (int i = 0; i < n; ++i) {
        p[i] = t2s_expf(x[i] - mx);
        lane[i % 32] += (double)p[i];
    }
    const float inv = (float)(1.0 / lanes_sum(lane));
    for (int i = 0; i < n; ++i) p[i] = p[i] * inv;
}

// Full sampler chain of one row (block.cpp:52-115, 191-271): penalty, descending argsort (ties
// by lower index), top-p on the sorted softmax (sequential f32 cumsum, first token above the
// threshold kept), temperature, top-k by pivot, softmax, argmax of probs / noise, where noise is
// indexed by sorted position as in the reference graph.  Returns the sampled token.
static int32_t sample_row(Model* m, const float* logits_in, const float* seen, const float* noise,
                          const SamplerCfg& c, int32_t* greedy_out) {
    const int V = (int)m->hp[5];
    std::vector<float> l(logits_in, logits_in + V);
    penalise(m, l.data(), seen, c.rp, c.eos_mask);
    std::vector<int> idx(V);
    for (int i = 0; i < V; ++i) idx[i] = i;
    std::sort(idx.begin(), idx.end(), [&](int a, int b) { return l[a] > l[b] || (l[a] == l[b] && a < b); });
    *greedy_out = idx[0];
    if (!noise) return idx[0];
    std::vector<float> s(V), p(V);
    for (int i = 0; i < V; ++i) s[i] = l[idx[i]];
    if (c.top_p < 1.0f && V > 1) {
        softmax_canon(s.data(), V, p.data());
        float cum = 0.0f;
        int cut = V;
        for (int i = 0; i < V; ++i) {
            cum = cum + p[i];
            if (cum - c.top_p > 0.0f) { cut = i + 1; break; }
        }
        for (int i = cut; i < V; ++i) s[i] = s[i] + (kMaskLogit - s[i]);
    }
    const float inv_t = 1.0f / fmaxf(c.temperature, 1.0e-5f);
    for (int i = 0; i < V; ++i) s[i] = s[i] * inv_t;
    if (c.top_k > 0 && c.top_k < V) {
        const float pivot = s[c.top_k - 1];
        for (int i = 0; i < V; ++i) if (pivot - s[i] > 0.0f) s[i] = s[i] + (kMaskLogit - s[i]);
    }
    softmax_canon(s.data(), V, p.data());
    int best = 0;
    float best_v = p[0] / noise[0];
    for (int i = 1; i < V; ++i) {
        const float sc = p[i] / noise[i];
        if (sc > best_v) { best_v = sc; best = i; }
    }
    return idx[best];
}

int orc_sample(void* model, int n, const float* logits, const float* seen, const float* noise, int top_k, float top_p,
               float temperature, float rp, int eos_mask, int32_t* sampled, int32_t* greedy) {
    Model* m = (Model*)model;
    const int V = (int)m->hp[5];
    const SamplerCfg c{top_k, top_p, temperature, rp, eos_mask};
    for (int r = 0; r < n; ++r)
        sampled[r] = sample_row(m, logits + (size_t)r * V, seen ? seen + (size_t)r * V : nullptr,
                                noise ? noise + (size_t)r * V : nullptr, c, &greedy[r]);
    return 0;
}

int orc_prefill(void* sess, int slot, const float* x, int nq, int T_prompt, int eos_mask, int32_t* token_out, float* logits_out,
                float* y_out) {
    Session* S = (Session*)sess;
    Model* m = S->m;
    const int d = (int)m->hp[1];
    if (slot < 0 || slot >= S->n_slots || nq <= 0 || S->n_pos[slot] != 0 || nq > S->cap) return -1;
    const int T_text = nq - T_prompt;
    if (T_text < 0) return -1;
    std::vector<int> sl(nq, slot), pos(nq), L(nq);
    for (int j = 0; j < nq; ++j) { pos[j] = j; L[j] = (j < T_text) ? T_text : (j + 1); }
    std::vector<float> xs(x, x + (size_t)nq * d);
#ifdef _OPENMP
    if (g_threads > 0) omp_set_num_threads(g_threads);
#endif
    forward_rows(S, nq, sl.data(), pos.data(), L.data(), xs.data());
    if (y_out) memcpy(y_out, xs.data(), sizeof(float) * xs.size());
    std::vector<float> logits(m->hp[5]);
    matmul_rows(m->lm_head, nullptr, &xs[(size_t)(nq - 1) * d], 1, logits.data(), S->ggml_order & 1);
    if (logits_out) memcpy(logits_out, logits.data(), sizeof(float) * logits.size());
    *token_out = pick_greedy(m, logits.data(), nullptr, 1.0f, eos_mask);
    S->n_pos[slot] = nq;
    S->audio_off[slot] = T_text;
    return 0;
}

// Forward of one decode step for n slots; fills logits [n][V] and advances n_pos.
static int decode_forward(Session* S, int n, const int32_t* slots, const int32_t* tokens_in, std::vector<float>& logits) {
    Model* m = S->m;
    const int d = (int)m->hp[1], V = (int)m->hp[5];
#ifdef _OPENMP
    if (g_threads > 0) omp_set_num_threads(g_threads);
#endif
    std::vector<float> x((size_t)n * d);
    std::vector<int> sl(n), pos(n), L(n);
    const float alpha = fdata(m->audio_alpha)[0];
    for (int i = 0; i < n; ++i) {
        const int s = slots[i];
        if (s < 0 || s >= S->n_slots || S->n_pos[s] <= 0 || S->n_pos[s] >= S->cap) return -1;
        if (tokens_in[i] < 0 || tokens_in[i] >= (int)m->audio_emb->ne[1]) return -1;
        const int pe_pos = S->n_pos[s] - S->audio_off[s];
        if (pe_pos < 0 || pe_pos >= S->cap) return -1;
        const uint8_t* er = m->audio_emb->data + (size_t)tokens_in[i] * orc_row_bytes(m->audio_emb->type, d);
        std::vector<float> e(d);
        orc_dequantize(m->audio_emb->type, er, d, e.data());
        for (int k = 0; k < d; ++k) x[(size_t)i * d + k] = e[k] + S->pe[(size_t)pe_pos * d + k] * alpha;
        sl[i] = s; pos[i] = S->n_pos[s]; L[i] = S->n_pos[s] + 1;
    }
    forward_rows(S, n, sl.data(), pos.data(), L.data(), x.data());
    logits.assign((size_t)n * V, 0.0f);
    matmul_rows(m->lm_head, nullptr, x.data(), n, logits.data(), S->ggml_order & 1);
    for (int i = 0; i < n; ++i) S->n_pos[slots[i]] += 1;
    return 0;
}

int orc_decode_step(void* sess, int n, const int32_t* slots, const int32_t* tokens_in, const float* seen, float rp,
                    int eos_mask, int32_t* tokens_out, float* logits_out) {
    Session* S = (Session*)sess;
    const int V = (int)S->m->hp[5];
    std::vector<float> logits;
    if (decode_forward(S, n, slots, tokens_in, logits)) return -1;
    if (logits_out) memcpy(logits_out, logits.data(), sizeof(float) * logits.size());
    for (int i = 0; i < n; ++i)
        tokens_out[i] = pick_greedy(S->m, &logits[(size_t)i * V], seen ? seen + (size_t)i * V : nullptr, rp, eos_mask);
    return 0;
}

int orc_decode_step2(void* sess, int n, const int32_t* slots, const int32_t* tokens_in, const float* seen,
                     const float* noise, int top_k, float top_p, float temperature, float rp, int eos_mask,
                     int32_t* sampled_out, int32_t* greedy_out, float* logits_out) {
    Session* S = (Session*)sess;
    std::vector<float> logits;
    if (decode_forward(S, n, slots, tokens_in, logits)) return -1;
    if (logits_out) memcpy(logits_out, logits.data(), sizeof(float) * logits.size());
    return orc_sample(S->m, n, logits.data(), seen, noise, top_k, top_p, temperature, rp, eos_mask, sampled_out, greedy_out);
}

int orc_read_kv(void* sess, int slot, int layer, int which, uint16_t* out) {
    Session* S = (Session*)sess;
    const int d = (int)S->m->hp[1], nl = (int)S->m->hp[4];
    const auto& src = which ? S->V[(size_t)slot * nl + layer] : S->K[(size_t)slot * nl + layer];
    memcpy(out, src.data(), sizeof(uint16_t) * (size_t)S->n_pos[slot] * d);
    return S->n_pos[slot];
}

// Extract-latent (sovits_extract_latent_block_forward, src/t2s/block.cpp:140-189): prompt semantic
// codes from HuBERT frames.  ggml_conv_1d(k = 2, s = 2, p = 0) is im2col in f16 (frames rounded to
// f16, row j = ic * 2 + k of output frame t is x[2t + k][ic]) times the f16 kernel rows
// [oc][ic][k]: the F16 matmul with 1536-long rows; then + bias; then score = codebook (F32
// matmul) - 0.5 * ||E_c||^2 with ||E_c||^2 = sum of the f32 squares in a sequential double sum
// (ggml_sqr, ggml_sum_rows, ggml_scale, ggml_sub); code = first index of the max (ggml_argmax).
int orc_extract_latent(void* model, const float* hubert, int T, int32_t* codes_out) {
    Model* m = (Model*)model;
    if (!m->ssl_w || !m->ssl_b || !m->codebook || T < 2) return -1;
    const int C = 768, K = 2 * C, NC = (int)m->codebook->ne[1];
    if (m->ssl_w->ne[0] != 2 || m->ssl_w->ne[1] != C || m->ssl_w->ne[2] != C || m->codebook->ne[0] != C) return -1;
    const int To = (T - 2) / 2 + 1;
    std::vector<float> cols((size_t)To * K), ssl((size_t)To * C), score((size_t)To * NC);
    for (int t = 0; t < To; ++t)
        for (int ic = 0; ic < C; ++ic)
            for (int k = 0; k < 2; ++k) cols[(size_t)t * K + ic * 2 + k] = hubert[(size_t)(2 * t + k) * C + ic];
    orc_matmul(m->ssl_w->type, m->ssl_w->data, C, K, cols.data(), To, ssl.data());
    const float* b = fdata(m->ssl_b);
    for (int t = 0; t < To; ++t) for (int o = 0; o < C; ++o) ssl[(size_t)t * C + o] = ssl[(size_t)t * C + o] + b[o];
    orc_matmul(m->codebook->type, m->codebook->data, NC, C, ssl.data(), To, score.data());
    const float* E = fdata(m->codebook);
    std::vector<float> half_norm(NC);
    for (int c = 0; c < NC; ++c) {
        double sum = 0.0;
        for (int d = 0; d < C; ++d) { const float e = E[(size_t)c * C + d]; sum += (double)(e * e); }
        half_norm[c] = (float)sum * 0.5f;
    }
    for (int t = 0; t < To; ++t) {
        int best = 0;
        float bv = score[(size_t)t * NC] - half_norm[0];
        for (int c = 1; c < NC; ++c) {
            const float v = score[(size_t)t * NC + c] - half_norm[c];
            if (v > bv) { bv = v; best = c; }
        }
        codes_out[t] = best;
    }
    return To;
}

int orc_embed_prefill(void* model, const int32_t* phones, const float* bert, int T_text, const int32_t* sem, int T_prompt,
                      float* x_out) {
    Model* m = (Model*)model;
    const int d = (int)m->hp[1];
    const int64_t bk = m->bert_w->ne[0];
    std::vector<float> bp((size_t)T_text * d);
    if (T_text > 0) matmul_rows(m->bert_w, m->bert_b, bert, T_text, bp.data());
    const float at = fdata(m->text_alpha)[0], aa = fdata(m->audio_alpha)[0];
    std::vector<float> e(d), pe(d);
    (void)bk;
    for (int t = 0; t < T_text; ++t) {
        if (phones[t] < 0 || phones[t] >= (int)m->text_emb->ne[1]) return -1;
        orc_dequantize(m->text_emb->type, m->text_emb->data + (size_t)phones[t] * orc_row_bytes(m->text_emb->type, d), d, e.data());
        orc_pe_row(t, d, pe.data());
        for (int k = 0; k < d; ++k) x_out[(size_t)t * d + k] = (e[k] + bp[(size_t)t * d + k]) + pe[k] * at;
    }
    for (int t = 0; t < T_prompt; ++t) {
        if (sem[t] < 0 || sem[t] >= (int)m->audio_emb->ne[1]) return -1;
        orc_dequantize(m->audio_emb->type, m->audio_emb->data + (size_t)sem[t] * orc_row_bytes(m->audio_emb->type, d), d, e.data());
        orc_pe_row(t, d, pe.data());
        for (int k = 0; k < d; ++k) x_out[(size_t)(T_text + t) * d + k] = e[k] + pe[k] * aa;
    }
    return 0;
}
