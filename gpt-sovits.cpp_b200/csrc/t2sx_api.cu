// C ABI of the B200 T2S decode path: GGUF loading and repacking, the paged-KV session manager,
// prefill orchestration and the CUDA-graph decode step.  Declarations and the reference
// interface each entry point replaces: include/t2sx.h.
#include "../../include/t2sx.h"
#include "t2sx_kernels.cuh"
#include "t2sx_math.cuh"

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

using namespace t2sx;

// ============================================================================================
// errors
// ============================================================================================
static thread_local std::string g_err;

static int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

#define CK(expr)                                                                                  \
    do {                                                                                          \
        cudaError_t e_ = (expr);                                                                  \
        if (e_ != cudaSuccess)                                                                    \
            return fail(e_ == cudaErrorMemoryAllocation ? T2SX_ERR_OOM : T2SX_ERR_CUDA, "%s: %s (%s:%d)", \
                        #expr, cudaGetErrorString(e_), __FILE__, __LINE__);                       \
    } while (0)

extern "C" const char* t2sx_last_error(void) { return g_err.c_str(); }
extern "C" int t2sx_version(void) { return 1; }
extern "C" int t2sx_device_count(int32_t* n) {
    int c = 0;
    CK(cudaGetDeviceCount(&c));
    *n = c;
    return T2SX_OK;
}

// ============================================================================================
// host helpers
// ============================================================================================
static float host_h2f(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1f, man = h & 0x3ffu;
    uint32_t u;
    if (exp == 0) {
        float v = (float)man * 5.9604644775390625e-08f;
        memcpy(&u, &v, 4);
        u |= sign;
    } else if (exp == 31) {
        u = sign | 0x7f800000u | (man << 13);
    } else {
        u = sign | ((exp + 112) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &u, 4);
    return f;
}

// Sine PE row p (session.cpp:33-53): [sin(p f_j), cos(p f_j)] with f_j = e^(-ln(10000) j / 256).
static void pe_row(int p, float* out) {
    const int half = kD / 2;
    for (int j = 0; j < half; ++j) {
        const float freq = std::exp(-std::log((float)10000) * (float)j / (float)half);
        const float arg = (float)p * freq;
        out[2 * j] = std::sin(arg);
        out[2 * j + 1] = std::cos(arg);
    }
}

static int64_t row_bytes(int type, int64_t n) {
    switch (type) {
        case W_F32: return n * 4;
        case W_F16: return n * 2;
        case W_Q8_0: return n % 32 ? -1 : n / 32 * 34;
        case W_Q4_0: return n % 32 ? -1 : n / 32 * 18;
        case W_Q5_0: return n % 32 ? -1 : n / 32 * 22;
        case W_Q4_K: return n % 256 ? -1 : n / 256 * 144;
    }
    return -1;
}

// ============================================================================================
// device arena (one allocation for all weights)
// ============================================================================================
struct Arena {
    char* base = nullptr;
    size_t size = 0, used = 0;
    std::vector<std::pair<size_t, std::vector<uint8_t>>> staged;  // offset, bytes
    size_t reserve(size_t n) {
        const size_t off = (used + 255) & ~(size_t)255;
        used = off + n;
        return off;
    }
    size_t add(std::vector<uint8_t>&& bytes) {
        const size_t off = reserve(bytes.size());
        staged.emplace_back(off, std::move(bytes));
        return off;
    }
};

template <class T>
static std::vector<uint8_t> as_bytes(const std::vector<T>& v) {
    std::vector<uint8_t> b(v.size() * sizeof(T));
    if (!b.empty()) memcpy(b.data(), v.data(), b.size());
    return b;
}

// Offsets of a repacked weight inside the arena (resolved to pointers after upload).
struct WOff {
    int type = -1, N = 0, K = 0;
    int tc_npad = 0;
    size_t q8 = SIZE_MAX, tcw = SIZE_MAX, q4 = SIZE_MAX, d = SIZE_MAX, dmin = SIZE_MAX, scm = SIZE_MAX, h = SIZE_MAX, f = SIZE_MAX;
};

static bool repack_weight(int type, const uint8_t* src, int64_t N, int64_t K, Arena& ar, WOff& w) {
    w.type = type; w.N = (int)N; w.K = (int)K;
    if (type == W_Q8_0) {
        std::vector<int8_t> q((size_t)N * K);
        std::vector<float> d((size_t)N * (K / 32));
        for (int64_t n = 0; n < N; ++n)
            for (int64_t b = 0; b < K / 32; ++b) {
                const uint8_t* blk = src + (n * (K / 32) + b) * 34;
                uint16_t hd; memcpy(&hd, blk, 2);
                d[n * (K / 32) + b] = host_h2f(hd);
                memcpy(&q[n * K + b * 32], blk + 2, 32);
            }
        w.q8 = ar.add(as_bytes(q)); w.d = ar.add(as_bytes(d));
    } else if (type == W_Q5_0) {
        // ggml block_q5_0 (f16 d, uint32 qh of fifth bits, 16 bytes of low nibbles; elements j and
        // j + 16 share byte j) -> the Q8_0 layout: int8 value in [-16, 15] and f32 d per block.  The
        // ggml dot with Q8_0 activations (integer block sum, then the scale fold) is the Q8_0 one.
        std::vector<int8_t> q((size_t)N * K);
        std::vector<float> d((size_t)N * (K / 32));
        for (int64_t n = 0; n < N; ++n)
            for (int64_t b = 0; b < K / 32; ++b) {
                const uint8_t* blk = src + (n * (K / 32) + b) * 22;
                uint16_t hd; memcpy(&hd, blk, 2);
                uint32_t qh; memcpy(&qh, blk + 2, 4);
                d[n * (K / 32) + b] = host_h2f(hd);
                for (int i = 0; i < 32; ++i) {
                    const int j = i & 15;
                    const int lo = (i < 16) ? (blk[6 + j] & 0xF) : (blk[6 + j] >> 4);
                    q[n * K + b * 32 + i] = (int8_t)((lo | (int)(((qh >> i) & 1u) << 4)) - 16);
                }
            }
        w.type = W_Q8_0;
        w.q8 = ar.add(as_bytes(q)); w.d = ar.add(as_bytes(d));
    } else if (type == W_Q4_0) {
        std::vector<uint8_t> q((size_t)N * (K / 2));
        std::vector<float> d((size_t)N * (K / 32));
        for (int64_t n = 0; n < N; ++n)
            for (int64_t b = 0; b < K / 32; ++b) {
                const uint8_t* blk = src + (n * (K / 32) + b) * 18;
                uint16_t hd; memcpy(&hd, blk, 2);
                d[n * (K / 32) + b] = host_h2f(hd);
                memcpy(&q[(n * (K / 32) + b) * 16], blk + 2, 16);
            }
        w.q4 = ar.add(std::move(q)); w.d = ar.add(as_bytes(d));
    } else if (type == W_Q4_K) {
        const int64_t nsb = K / 256;
        std::vector<uint8_t> q((size_t)N * nsb * 128), scm((size_t)N * nsb * 16);
        std::vector<float> d((size_t)N * nsb), dm((size_t)N * nsb);
        for (int64_t n = 0; n < N; ++n)
            for (int64_t b = 0; b < nsb; ++b) {
                const uint8_t* blk = src + (n * nsb + b) * 144;
                uint16_t hd, hm; memcpy(&hd, blk, 2); memcpy(&hm, blk + 2, 2);
                d[n * nsb + b] = host_h2f(hd);
                dm[n * nsb + b] = host_h2f(hm);
                const uint8_t* sc = blk + 4;
                uint8_t* o = &scm[(n * nsb + b) * 16];
                for (int j = 0; j < 8; ++j) {
                    int s, m;
                    if (j < 4) { s = sc[j] & 63; m = sc[j + 4] & 63; }
                    else {
                        s = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
                        m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
                    }
                    o[j] = (uint8_t)s; o[8 + j] = (uint8_t)m;
                }
                memcpy(&q[(n * nsb + b) * 128], blk + 16, 128);
            }
        // Planes for the tcgen05 path, int8 [3][Npad][K] in element order (Npad = N rounded up to
        // 128, padding rows zero): p = sc_j * q with sub-block j of the element, plane 0 = p & 127,
        // plane 1 = p >> 7, plane 2 = mn_j.  Then for activation block values x:
        //   sum_k plane0*x + 128 * sum_k plane1*x = sum_j sc_j * (sum_{k in j} q*x)   and
        //   sum_k plane2*x = sum_j mn_j * (sum_{k in j} x),
        // the two integer sums of the Q4_K dot, exactly.  Within a super-block, byte j of 32-byte
        // chunk c holds element 64c + j (low nibble, sub-block 2c) and 64c + 32 + j (high, 2c + 1).
        const int64_t Npad = (N + 127) / 128 * 128;
        std::vector<int8_t> x((size_t)3 * Npad * K, 0);
        for (int64_t n = 0; n < N; ++n)
            for (int64_t b = 0; b < nsb; ++b) {
                const uint8_t* o = &scm[(n * nsb + b) * 16];
                for (int c = 0; c < 4; ++c)
                    for (int j = 0; j < 32; ++j) {
                        const uint8_t v = q[(n * nsb + b) * 128 + c * 32 + j];
                        for (int h = 0; h < 2; ++h) {
                            const int sub = 2 * c + h, e = c * 64 + h * 32 + j;
                            const int p = o[sub] * ((h ? v >> 4 : v) & 15);
                            const size_t at = (size_t)n * K + b * 256 + e;
                            x[at] = (int8_t)(p & 127);
                            x[(size_t)Npad * K + at] = (int8_t)(p >> 7);
                            x[(size_t)2 * Npad * K + at] = (int8_t)o[8 + sub];
                        }
                    }
            }
        w.q4 = ar.add(std::move(q)); w.d = ar.add(as_bytes(d)); w.dmin = ar.add(as_bytes(dm)); w.scm = ar.add(std::move(scm));
        w.tcw = ar.add(as_bytes(x)); w.tc_npad = (int)Npad;
    } else if (type == W_F16) {
        std::vector<uint8_t> b(src, src + (size_t)N * K * 2);
        w.h = ar.add(std::move(b));
    } else if (type == W_F32) {
        std::vector<uint8_t> b(src, src + (size_t)N * K * 4);
        w.f = ar.add(std::move(b));
    } else {
        return false;
    }
    return true;
}

static DevW resolve(const WOff& o, char* base) {
    DevW w;
    w.type = o.type; w.N = o.N; w.K = o.K;
    auto P = [&](size_t off) -> char* { return off == SIZE_MAX ? nullptr : base + off; };
    w.q8 = (const int8_t*)P(o.q8); w.tcw = (const int8_t*)P(o.tcw); w.tc_npad = o.tc_npad; w.q4 = (const uint8_t*)P(o.q4); w.d = (const float*)P(o.d);
    w.dmin = (const float*)P(o.dmin); w.scm = (const uint8_t*)P(o.scm); w.h = (const uint16_t*)P(o.h);
    w.f = (const float*)P(o.f);
    return w;
}

// ============================================================================================
// GGUF (v2/v3) reader
// ============================================================================================
struct GTensor { int type = -1; int nd = 0; int64_t ne[4] = {1, 1, 1, 1}; uint64_t off = 0; const uint8_t* data = nullptr; };

struct GFile {
    std::vector<uint8_t> buf;
    std::map<std::string, GTensor> t;
    std::map<std::string, uint32_t> u32;
};

struct Cur {
    const uint8_t* p; size_t n, o = 0; bool ok = true;
    template <class T> T get() { T v{}; if (o + sizeof(T) > n) { ok = false; return v; } memcpy(&v, p + o, sizeof(T)); o += sizeof(T); return v; }
    std::string str() { const uint64_t l = get<uint64_t>(); if (!ok || l > n - o) { ok = false; return ""; } std::string s((const char*)p + o, l); o += l; return s; }
    void skip(uint32_t ty, int depth = 0) {
        static const int sz[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
        if (!ok || depth > 4) { ok = false; return; }
        if (ty == 8) { str(); return; }
        if (ty == 9) {
            const uint32_t et = get<uint32_t>();
            const uint64_t c = get<uint64_t>();
            if (et != 8 && et != 9 && et <= 12) {
                const uint64_t bytes = c * (uint64_t)sz[et];
                if (c != 0 && bytes / c != (uint64_t)sz[et]) { ok = false; return; }
                if (bytes > n - o) { ok = false; return; }
                o += bytes;
                return;
            }
            for (uint64_t i = 0; i < c && ok; ++i) skip(et, depth + 1);
            return;
        }
        if (ty > 12) { ok = false; return; }
        if ((size_t)sz[ty] > n - o) { ok = false; return; }
        o += sz[ty];
    }
};

static int gguf_read(const char* path, GFile& g) {
    FILE* f = fopen(path, "rb");
    if (!f) return fail(T2SX_ERR_IO, "t2sx_model_load: cannot open '%s'", path);
    fseek(f, 0, SEEK_END);
    const long sz = ftell(f);
    fseek(f, 0, SEEK_SET);
    if (sz <= 0) { fclose(f); return fail(T2SX_ERR_IO, "t2sx_model_load: empty file '%s'", path); }
    g.buf.resize((size_t)sz);
    const size_t rd = fread(g.buf.data(), 1, (size_t)sz, f);
    fclose(f);
    if (rd != (size_t)sz) return fail(T2SX_ERR_IO, "t2sx_model_load: short read on '%s'", path);
    Cur c{g.buf.data(), g.buf.size()};
    if (c.get<uint32_t>() != 0x46554747u) return fail(T2SX_ERR_FORMAT, "'%s' is not a GGUF file", path);
    const uint32_t ver = c.get<uint32_t>();
    if (ver < 2 || ver > 3) return fail(T2SX_ERR_FORMAT, "unsupported GGUF version %u", ver);
    const uint64_t nt = c.get<uint64_t>(), nkv = c.get<uint64_t>();
    if (nt > (1u << 20) || nkv > (1u << 20)) return fail(T2SX_ERR_FORMAT, "GGUF header counts out of range");
    uint32_t align = 32;
    for (uint64_t i = 0; i < nkv && c.ok; ++i) {
        const std::string k = c.str();
        const uint32_t ty = c.get<uint32_t>();
        if (ty == 4) {
            const uint32_t v = c.get<uint32_t>();
            g.u32[k] = v;
            if (k == "general.alignment") align = v;
        } else {
            c.skip(ty);
        }
    }
    if (align == 0 || (align & (align - 1))) return fail(T2SX_ERR_FORMAT, "bad GGUF alignment %u", align);
    std::vector<std::pair<std::string, GTensor>> tl;
    for (uint64_t i = 0; i < nt && c.ok; ++i) {
        GTensor t;
        std::string name = c.str();
        t.nd = (int)c.get<uint32_t>();
        if (t.nd < 1 || t.nd > 4) { c.ok = false; break; }
        for (int d = 0; d < t.nd; ++d) t.ne[d] = (int64_t)c.get<uint64_t>();
        t.type = (int)c.get<uint32_t>();
        t.off = c.get<uint64_t>();
        tl.emplace_back(std::move(name), t);
    }
    if (!c.ok) return fail(T2SX_ERR_FORMAT, "truncated GGUF header in '%s'", path);
    const size_t data0 = (c.o + align - 1) / align * align;
    for (auto& kv : tl) {
        GTensor& t = kv.second;
        for (int d = 0; d < 4; ++d)
            if (t.ne[d] <= 0 || t.ne[d] > (1ll << 32)) return fail(T2SX_ERR_FORMAT, "tensor '%s' has bad shape", kv.first.c_str());
        const int64_t rb = row_bytes(t.type, t.ne[0]);
        if (rb < 0) return fail(T2SX_ERR_FORMAT, "tensor '%s' has unsupported type %d", kv.first.c_str(), t.type);
        const uint64_t bytes = (uint64_t)rb * (uint64_t)(t.ne[1] * t.ne[2] * t.ne[3]);
        if (data0 + t.off < data0 || data0 + t.off + bytes > g.buf.size())
            return fail(T2SX_ERR_FORMAT, "tensor '%s' data out of file bounds", kv.first.c_str());
        t.data = g.buf.data() + data0 + t.off;
        g.t[kv.first] = t;
    }
    return T2SX_OK;
}

// ============================================================================================
// model
// ============================================================================================
struct LayerW {
    WOff qkv, out, up, down;
    size_t qkv_b, out_b, ln1_w, ln1_b, up_b, down_b, ln2_w, ln2_b;
};
struct LayerD {
    DevW qkv, out, up, down;
    const float *qkv_b, *out_b, *ln1_w, *ln1_b, *up_b, *down_b, *ln2_w, *ln2_b;
};

struct t2sx_model {
    int device = 0;
    // A model freed while sessions still use it is released when the last of them is freed.
    std::mutex mu;
    int live_sessions = 0;
    bool free_requested = false;
    uint32_t hp[9] = {512, 512, 16, 2048, 24, 1025, 732, 1024, 192};
    int32_t wtypes[4] = {-1, -1, -1, -1};
    char* arena = nullptr;
    size_t arena_bytes = 0;
    std::vector<LayerD> layers;
    DevW lm_head, bert;
    const float* bert_b = nullptr;
    const uint16_t* audio16 = nullptr; const float* audio32 = nullptr; int audio_rows = 0;
    const uint16_t* text16 = nullptr; const float* text32 = nullptr; int text_rows = 0;
    float alpha_text = 1.0f, alpha_audio = 1.0f;
    // extract-latent: Conv1d(768, 768, k=2, s=2) as a 768 x 1536 weight, the codebook as an
    // n_codes x 768 weight, and 0.5 * ||E_c||^2 per code
    DevW ssl_w, codebook;
    const float* ssl_b = nullptr;
    const float* code_half_norm = nullptr;
    int n_codes = 0;
    // GGUF type and shape of every tensor of the file (t2sx_model_tensor_info)
    struct TInfo { int type; int nd; int64_t ne[4]; };
    std::map<std::string, TInfo> tinfo;
};

static const float* fptr(char* base, size_t off) { return (const float*)(base + off); }

extern "C" int t2sx_model_load(const char* path, int32_t device, t2sx_model** out) {
    if (!path || !out) return fail(T2SX_ERR_INVALID, "t2sx_model_load: null argument");
    *out = nullptr;
    int ndev = 0;
    CK(cudaGetDeviceCount(&ndev));
    if (device < 0 || device >= ndev) return fail(T2SX_ERR_INVALID, "t2sx_model_load: device %d of %d", device, ndev);
    GFile g;
    int rc = gguf_read(path, g);
    if (rc) return rc;
    std::unique_ptr<t2sx_model> m(new t2sx_model());
    m->device = device;
    static const char* keys[9] = {"t2s.embedding_dim", "t2s.hidden_dim", "t2s.head", "t2s.linear_units", "t2s.n_layer",
                                  "t2s.vocab_size", "t2s.phoneme_vocab_size", "t2s.eos", "sovits.inter_channels"};
    for (int i = 0; i < 9; ++i) { auto it = g.u32.find(keys[i]); if (it != g.u32.end()) m->hp[i] = it->second; }
    if (m->hp[1] != (uint32_t)kD || m->hp[2] != (uint32_t)kHeads || m->hp[0] != (uint32_t)kD)
        return fail(T2SX_ERR_FORMAT, "unsupported T2S shape d=%u heads=%u (this build: d=512, 16 heads)", m->hp[1], m->hp[2]);
    const int nl = (int)m->hp[4], ff = (int)m->hp[3], V = (int)m->hp[5];
    if (nl <= 0 || nl > 256 || ff <= 0 || ff % 256 || V <= 0) return fail(T2SX_ERR_FORMAT, "bad hparams");
    // the few-row matmul keeps a row's 32-element block sums in shared memory (at most 64)
    if (ff > 2048) return fail(T2SX_ERR_FORMAT, "unsupported FFN width %d (this build: at most 2048)", ff);
    // the full sampler sorts a row's logits in shared memory (2048 entries)
    if (V > 2048) return fail(T2SX_ERR_FORMAT, "unsupported vocabulary size %d (this build: at most 2048)", V);
    auto need = [&](const std::string& n, int64_t ne0, int64_t ne1, const GTensor** t) -> int {
        auto it = g.t.find(n);
        if (it == g.t.end()) return fail(T2SX_ERR_FORMAT, "tensor '%s' not found in GGUF", n.c_str());
        if (it->second.ne[0] != ne0 || it->second.ne[1] != ne1)
            return fail(T2SX_ERR_FORMAT, "tensor '%s' has shape {%lld,%lld}, expected {%lld,%lld}", n.c_str(),
                        (long long)it->second.ne[0], (long long)it->second.ne[1], (long long)ne0, (long long)ne1);
        *t = &it->second;
        return T2SX_OK;
    };
    Arena ar;
    auto add_f32 = [&](const GTensor* t, size_t& off) -> int {
        const int64_t n = t->ne[0] * t->ne[1];
        std::vector<float> v((size_t)n);
        if (t->type == W_F32) memcpy(v.data(), t->data, n * 4);
        else if (t->type == W_F16) { for (int64_t i = 0; i < n; ++i) { uint16_t h; memcpy(&h, t->data + 2 * i, 2); v[i] = host_h2f(h); } }
        else return fail(T2SX_ERR_FORMAT, "1-D tensor with type %d", t->type);
        off = ar.add(as_bytes(v));
        return T2SX_OK;
    };
    auto add_w = [&](const GTensor* t, WOff& w) -> int {
        if (!repack_weight(t->type, t->data, t->ne[1], t->ne[0], ar, w))
            return fail(T2SX_ERR_FORMAT, "weight type %d unsupported", t->type);
        return T2SX_OK;
    };
    std::vector<LayerW> lw(nl);
    for (int i = 0; i < nl; ++i) {
        const std::string p = "attention." + std::to_string(i) + ".";
        const GTensor *qkv, *qkv_b, *ow, *ob, *l1w, *l1b, *uw, *ub, *dw, *db, *l2w, *l2b;
        if ((rc = need(p + "qkv_w", kD, 3 * kD, &qkv)) || (rc = need(p + "qkv_b", 3 * kD, 1, &qkv_b)) ||
            (rc = need(p + "out_proj_w", kD, kD, &ow)) || (rc = need(p + "out_proj_b", kD, 1, &ob)) ||
            (rc = need(p + "ln1_w", kD, 1, &l1w)) || (rc = need(p + "ln1_b", kD, 1, &l1b)) ||
            (rc = need(p + "ffn_up_w", kD, ff, &uw)) || (rc = need(p + "ffn_up_b", ff, 1, &ub)) ||
            (rc = need(p + "ffn_down_w", ff, kD, &dw)) || (rc = need(p + "ffn_down_b", kD, 1, &db)) ||
            (rc = need(p + "ln2_w", kD, 1, &l2w)) || (rc = need(p + "ln2_b", kD, 1, &l2b)))
            return rc;
        LayerW& L = lw[i];
        if ((rc = add_w(qkv, L.qkv)) || (rc = add_w(ow, L.out)) || (rc = add_w(uw, L.up)) || (rc = add_w(dw, L.down)) ||
            (rc = add_f32(qkv_b, L.qkv_b)) || (rc = add_f32(ob, L.out_b)) || (rc = add_f32(l1w, L.ln1_w)) ||
            (rc = add_f32(l1b, L.ln1_b)) || (rc = add_f32(ub, L.up_b)) || (rc = add_f32(db, L.down_b)) ||
            (rc = add_f32(l2w, L.ln2_w)) || (rc = add_f32(l2b, L.ln2_b)))
            return rc;
        if (i == 0) m->wtypes[0] = qkv->type;
    }
    const GTensor *lm, *te, *bw, *bb, *ta, *ae, *aa;
    if ((rc = need("sampler.lm_head_w", kD, V, &lm)) || (rc = need("encoder.text_embedding", kD, m->hp[6], &te)) ||
        (rc = need("encoder.bert_proj_w", 1024, kD, &bw)) || (rc = need("encoder.bert_proj_b", kD, 1, &bb)) ||
        (rc = need("encoder.text_pos_alpha", 1, 1, &ta)) || (rc = need("encoder.audio_embedding", kD, V, &ae)) ||
        (rc = need("encoder.audio_pos_alpha", 1, 1, &aa)))
        return rc;
    for (const char* n : {"extract_latent.ssl_proj_w", "extract_latent.ssl_proj_b", "extract_latent.codebook"})
        if (!g.t.count(n)) return fail(T2SX_ERR_FORMAT, "tensor '%s' not found in GGUF", n);
    // extract-latent (block.cpp:140-189): kernel {2, 768, 768} = 768 rows of [ic][k], codebook
    // {768, n_codes} kept f32 (convert_t2s_to_gguf.py keeps it un-quantised)
    const GTensor* sw = &g.t.at("extract_latent.ssl_proj_w");
    const GTensor* sbias = &g.t.at("extract_latent.ssl_proj_b");
    const GTensor* cb = &g.t.at("extract_latent.codebook");
    if (sw->ne[0] != 2 || sw->ne[1] != 768 || sw->ne[2] != 768 || sbias->ne[0] != 768 || sbias->ne[1] != 1 ||
        cb->ne[0] != 768 || cb->type != W_F32 || cb->ne[1] < 1)
        return fail(T2SX_ERR_FORMAT, "extract_latent tensors have unexpected shapes or types");
    WOff swo, cbo;
    if (!repack_weight(sw->type, sw->data, 768, 1536, ar, swo) || !repack_weight(W_F32, cb->data, cb->ne[1], 768, ar, cbo))
        return fail(T2SX_ERR_FORMAT, "extract_latent weight type %d unsupported", sw->type);
    size_t sbo;
    if ((rc = add_f32(sbias, sbo))) return rc;
    size_t hno;
    {
        // ggml_sqr, ggml_sum_rows (sequential double sum of the f32 squares), ggml_scale(0.5)
        std::vector<float> hn((size_t)cb->ne[1]);
        const float* E = (const float*)cb->data;
        for (int64_t c = 0; c < cb->ne[1]; ++c) {
            double sum = 0.0;
            for (int d = 0; d < 768; ++d) { const float e = E[c * 768 + d]; sum += (double)(e * e); }
            hn[c] = (float)sum * 0.5f;
        }
        hno = ar.add(as_bytes(hn));
    }
    WOff lmo, bwo;
    size_t bbo;
    if ((rc = add_w(lm, lmo)) || (rc = add_w(bw, bwo)) || (rc = add_f32(bb, bbo))) return rc;
    if ((te->type != W_F16 && te->type != W_F32) || (ae->type != W_F16 && ae->type != W_F32))
        return fail(T2SX_ERR_FORMAT, "embedding tables must be F16 or F32");
    const size_t teo = ar.add(std::vector<uint8_t>(te->data, te->data + row_bytes(te->type, kD) * te->ne[1]));
    const size_t aeo = ar.add(std::vector<uint8_t>(ae->data, ae->data + row_bytes(ae->type, kD) * ae->ne[1]));
    auto scalar = [&](const GTensor* t) { if (t->type == W_F32) { float v; memcpy(&v, t->data, 4); return v; } uint16_t h; memcpy(&h, t->data, 2); return host_h2f(h); };
    m->alpha_text = scalar(ta);
    m->alpha_audio = scalar(aa);
    m->wtypes[1] = lm->type; m->wtypes[2] = ae->type; m->wtypes[3] = bw->type;

    DeviceGuard dg_;
    CK(dg_.set(device));
    char* base = nullptr;
    CK(cudaMalloc(&base, ar.used));
    m->arena = base;
    m->arena_bytes = ar.used;
    for (auto& s : ar.staged) {
        cudaError_t e = cudaMemcpy(base + s.first, s.second.data(), s.second.size(), cudaMemcpyHostToDevice);
        if (e != cudaSuccess) { cudaFree(base); m->arena = nullptr; return fail(T2SX_ERR_CUDA, "weight upload: %s", cudaGetErrorString(e)); }
    }
    m->layers.resize(nl);
    for (int i = 0; i < nl; ++i) {
        LayerD& D = m->layers[i];
        const LayerW& L = lw[i];
        D.qkv = resolve(L.qkv, base); D.out = resolve(L.out, base); D.up = resolve(L.up, base); D.down = resolve(L.down, base);
        D.qkv_b = fptr(base, L.qkv_b); D.out_b = fptr(base, L.out_b); D.ln1_w = fptr(base, L.ln1_w); D.ln1_b = fptr(base, L.ln1_b);
        D.up_b = fptr(base, L.up_b); D.down_b = fptr(base, L.down_b); D.ln2_w = fptr(base, L.ln2_w); D.ln2_b = fptr(base, L.ln2_b);
    }
    m->lm_head = resolve(lmo, base);
    m->bert = resolve(bwo, base);
    m->bert_b = fptr(base, bbo);
    if (te->type == W_F16) m->text16 = (const uint16_t*)(base + teo); else m->text32 = (const float*)(base + teo);
    if (ae->type == W_F16) m->audio16 = (const uint16_t*)(base + aeo); else m->audio32 = (const float*)(base + aeo);
    m->text_rows = (int)te->ne[1];
    m->audio_rows = (int)ae->ne[1];
    m->ssl_w = resolve(swo, base);
    m->codebook = resolve(cbo, base);
    m->ssl_b = fptr(base, sbo);
    m->code_half_norm = fptr(base, hno);
    m->n_codes = (int)cb->ne[1];
    for (const auto& kv : g.t) {
        t2sx_model::TInfo ti{kv.second.type, kv.second.nd, {kv.second.ne[0], kv.second.ne[1], kv.second.ne[2], kv.second.ne[3]}};
        m->tinfo[kv.first] = ti;
    }
    *out = m.release();
    return T2SX_OK;
}

static void release_model(t2sx_model* m) {
    DeviceGuard dg_;
    dg_.set(m->device);
    if (m->arena) cudaFree(m->arena);
    delete m;
}

extern "C" void t2sx_model_free(t2sx_model* m) {
    if (!m) return;
    {
        std::lock_guard<std::mutex> lk(m->mu);
        if (m->free_requested) return;
        m->free_requested = true;
        if (m->live_sessions > 0) return;   // released by the last t2sx_session_free
    }
    release_model(m);
}

extern "C" int t2sx_model_hparams(const t2sx_model* m, uint32_t* hp, int32_t* wtypes) {
    if (!m) return fail(T2SX_ERR_INVALID, "null model");
    if (hp) for (int i = 0; i < 9; ++i) hp[i] = m->hp[i];
    if (wtypes) for (int i = 0; i < 4; ++i) wtypes[i] = m->wtypes[i];
    return T2SX_OK;
}

extern "C" int t2sx_model_device_bytes(const t2sx_model* m, uint64_t* bytes) {
    if (!m || !bytes) return fail(T2SX_ERR_INVALID, "null argument");
    *bytes = m->arena_bytes;
    return T2SX_OK;
}

// ============================================================================================
// session
// ============================================================================================
struct Work {
    int cap = 0;
    void* mem = nullptr;
    size_t bytes = 0;
    float *x, *qkv, *attn, *o, *ln1, *h, *f, *logits, *xl;
    uint16_t *q16, *ah;
    int8_t* aq;
    float* ad;
    int32_t *abs, *row_slot, *row_pos, *row_L, *tok, *lastrow, *greedy;
    int2* grp;          // prefill row groups of the pass (first row, rows): consecutive rows of one slot
    int n_grp = 0;      // groups of the current pass (0: the per-row attention kernels only)
    int grp_row0 = 0;   // first row covered by the groups
};

static size_t work_bytes(int R, int V, int ff) {
    size_t b = 0;
    auto add = [&](size_t n) { b += (n + 255) & ~(size_t)255; };
    add((size_t)R * kD * 4); add((size_t)R * 3 * kD * 4); add((size_t)R * kD * 4); add((size_t)R * kD * 4);
    add((size_t)R * kD * 4); add((size_t)R * ff * 4); add((size_t)R * kD * 4); add((size_t)R * V * 4); add((size_t)R * kD * 4);
    add((size_t)R * kD * 2); add((size_t)R * ff * 2); add((size_t)R * ff); add((size_t)R * (ff / 32) * 4);
    add((size_t)R * (ff / 32) * 4);
    for (int i = 0; i < 6; ++i) add((size_t)R * 4);
    add((size_t)R * 8);
    return b;
}

static int work_alloc(Work& w, int R, int V, int ff) {
    if (w.cap >= R) return T2SX_OK;
    if (w.mem) { cudaFree(w.mem); w.mem = nullptr; w.cap = 0; }
    const size_t bytes = work_bytes(R, V, ff);
    CK(cudaMalloc(&w.mem, bytes));
    w.bytes = bytes;
    char* p = (char*)w.mem;
    auto take = [&](size_t n) { char* r = p; p += (n + 255) & ~(size_t)255; return r; };
    w.x = (float*)take((size_t)R * kD * 4); w.qkv = (float*)take((size_t)R * 3 * kD * 4);
    w.attn = (float*)take((size_t)R * kD * 4); w.o = (float*)take((size_t)R * kD * 4);
    w.ln1 = (float*)take((size_t)R * kD * 4); w.h = (float*)take((size_t)R * ff * 4);
    w.f = (float*)take((size_t)R * kD * 4); w.logits = (float*)take((size_t)R * V * 4); w.xl = (float*)take((size_t)R * kD * 4);
    w.q16 = (uint16_t*)take((size_t)R * kD * 2); w.ah = (uint16_t*)take((size_t)R * ff * 2);
    w.aq = (int8_t*)take((size_t)R * ff); w.ad = (float*)take((size_t)R * (ff / 32) * 4);
    w.abs = (int32_t*)take((size_t)R * (ff / 32) * 4);
    w.row_slot = (int32_t*)take((size_t)R * 4); w.row_pos = (int32_t*)take((size_t)R * 4);
    w.row_L = (int32_t*)take((size_t)R * 4); w.tok = (int32_t*)take((size_t)R * 4); w.lastrow = (int32_t*)take((size_t)R * 4);
    w.greedy = (int32_t*)take((size_t)R * 4);
    w.grp = (int2*)take((size_t)R * 8);
    w.cap = R;
    return T2SX_OK;
}

struct t2sx_session {
    const t2sx_model* m = nullptr;
    int device = 0;
    bool counted = false;          // holds a reference on the model
    int n_slots = 0, slot_size = 0, pages_per_slot = 0, n_layer = 0, V = 0, ff = 0;
    t2sx_sampler_config cfg{};
    cudaStream_t st = nullptr;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    // KV pages
    uint16_t* pool = nullptr;
    size_t pool_bytes = 0;
    int32_t* ptab = nullptr;                 // device [n_slots][pages_per_slot]
    std::vector<int32_t> ptab_h;
    std::vector<int32_t> free_pages;
    // slot state (device + host mirrors)
    int32_t *n_pos = nullptr, *audio_off = nullptr, *token_in = nullptr, *cap = nullptr, *err = nullptr;
    uint8_t* seen = nullptr;
    float* pe = nullptr;
    std::vector<int32_t> n_pos_h, audio_off_h;
    // work buffers
    Work dec, pre;
    int dec_rows = 0;          // rows of the captured decode graph
    bool dec_dirty = true;     // active set changed since the last capture
    cudaGraphExec_t graph = nullptr;
    int32_t* ring = nullptr;
    int32_t* ring_step = nullptr;
    int ring_len = 256;
    int graph_kernels = 0;         // kernel nodes in the captured step graph
    int32_t* scratch_i = nullptr;  // [n_slots]
    int32_t* tail_ctr = nullptr;   // ticket of the last-CTA matmul tails (self-resetting)
    int last_rows = 0;             // rows of the last logits
    const float* last_logits = nullptr;
    int last_hidden_rows = 0;      // rows of the last pass's final-layer output
    const float* last_hidden = nullptr;
    const int32_t* last_greedy = nullptr;
    float* noise = nullptr;        // [n_slots][V] Exp(1) noise by sorted position (stochastic sampling)
    bool noise_on = false;
    bool graph_noise = false;      // sampler kind captured in the step graph
    float last_ms = 0.0f;
    std::vector<int32_t> active;   // slots in row order
    int graph_gen = 0;             // bumped whenever the step graph is instantiated
    // t2sx_decode_step_host with tokens in and out: one graph (pinned token copies, scatter,
    // ring reset, timing events, the step, the token copy back) built for graph_gen
    cudaGraphExec_t host_graph = nullptr;
    int host_gen = -1;
    int32_t* pin_in = nullptr;     // [n_slots] pinned
    int32_t* pin_out = nullptr;    // [n_slots] pinned
};

static Rows rows_of(t2sx_session* s, Work& w) {
    Rows r;
    r.slot = w.row_slot; r.pos = w.row_pos; r.L = w.row_L; r.cap = s->cap; r.err = s->err;
    return r;
}

static KVView kv_of(t2sx_session* s) {
    KVView v;
    v.pool = s->pool; v.ptab = s->ptab; v.max_pages = s->pages_per_slot; v.n_layer = s->n_layer;
    v.n_pages = s->n_slots * s->pages_per_slot;
    return v;
}

static ActQ act_of(Work& w) {
    ActQ a;
    a.q = w.aq; a.d = w.ad; a.bs = w.abs; a.h = w.ah;
    return a;
}

static const float kAttnScale = 1.0f / sqrtf((float)kHeadDim);

static ActQ act_for(Work& w, const float* f32_input) {
    ActQ a = act_of(w);
    a.f = f32_input;   // read directly by F32-weight matmuls
    return a;
}

// The post-norm layers over T rows (block.cpp:513-637).  On entry w.x holds the input rows (f32)
// and the activation buffer holds them in layer 0's QKV dot type; on exit w.x holds the output
// rows and, when final_qtype >= 0, the activation buffer holds them in that dot type.  For one or
// two rows the residual + LayerNorm runs at the start of the matmul that consumes it (Q8_0/Q4_0
// QKV and FFN-up weights) or in the last CTA of the preceding matmul (other weight types);
// otherwise it is its own kernel.
// Rows up to which the residual + LayerNorm runs as the last CTA's tail of the preceding matmul
// (T2SX_LN_TAIL_ROWS overrides; 0 = always a separate kernel).
static int tail_rows() {
    static const int v = [] {
        const char* e = getenv("T2SX_LN_TAIL_ROWS");
        return e ? atoi(e) : 2;
    }();
    return v;
}

// Prefill row groups of rows [row0, T) (rs = slot of each row): up to 16 consecutive rows of one
// slot each, uploaded to w.grp.  Fewer than 64 such rows: no groups (the per-row kernels serve).
static int set_row_groups(t2sx_session* s, Work& w, int T, int row0, const std::vector<int32_t>& rs) {
    w.n_grp = 0;
    w.grp_row0 = row0;
    if (T - row0 < 64) return T2SX_OK;
    std::vector<int2> g;
    for (int r = row0; r < T;) {
        int n = 1;
        while (r + n < T && n < 16 && rs[r + n] == rs[r]) ++n;
        g.push_back(make_int2(r, n));
        r += n;
    }
    CK(cudaMemcpyAsync(w.grp, g.data(), g.size() * sizeof(int2), cudaMemcpyHostToDevice, s->st));
    w.n_grp = (int)g.size();
    return T2SX_OK;
}

// Programmatic launches for the one- and two-row layer chain (T2SX_PDL_SMALL=0: off).
static bool pdl_small() {
    static const bool v = [] {
        const char* e = getenv("T2SX_PDL_SMALL");
        return !(e && e[0] == '0');
    }();
    return v;
}

// Rows up to which the general layer chain is launched programmatically as well (T2SX_PDL_ROWS;
// 0 = only the one- and two-row chain): its split-K matmuls fetch their weight slices and the
// split attention its page numbers and earlier positions' K/V before waiting on the predecessor.
// 32 sessions, Q4_0, 500 steps: 1.029 -> 0.889 ms per step.
static int pdl_rows() {
    static const int v = [] {
        const char* e = getenv("T2SX_PDL_ROWS");
        return e ? atoi(e) : 32;
    }();
    return v;
}

// The LayerNorm-prologue matmuls take Q8_0/Q4_0 QKV and FFN-up weights (Q5_0 is held as Q8_0).
static bool ln_prologue_ok(const t2sx_model* m) {
    for (const LayerD& L : m->layers)
        if ((L.qkv.type != W_Q8_0 && L.qkv.type != W_Q4_0) || (L.up.type != W_Q8_0 && L.up.type != W_Q4_0)) return false;
    return true;
}

// head / head_out (optional): the logits matmul that follows the layers.  Returns true when it
// has been run here (the one- and two-row path with Q8_0/Q4_0 logits weights: the last layer's
// second LayerNorm is its prologue); the caller runs it otherwise.
static bool run_layers(t2sx_session* s, Work& w, int T, bool decode, int final_qtype, const DevW* head = nullptr,
                       float* head_out = nullptr) {
    const t2sx_model* m = s->m;
    Rows rows = rows_of(s, w);
    KVView kv = kv_of(s);
    // last-CTA LayerNorm tails: at most tail_rows() rows (the tail runs on one CTA)
    const bool small = T <= tail_rows();
    const int nl = s->n_layer;
    if (small && T <= kLnRows && ln_prologue_ok(m)) {
        // each norm runs at the start of the matmul that consumes it (matmul_ln): the QKV
        // projection of layer l > 0 normalises the previous layer's FFN output, the FFN up
        // projection the attention output; the last layer's second norm is its own kernel.
        // The chain's kernels are launched programmatically (T2SX_PDL_SMALL=0 turns that off):
        // each fetches its weights (the attention its page numbers and earlier positions' K/V)
        // while its predecessor finishes.
        const LayerD& Z = m->layers[nl - 1];
        const bool fuse_head = head && head_out && head->K == kD && (head->type == W_Q8_0 || head->type == W_Q4_0);
        {
            PdlScope pdl(pdl_small());
            for (int l = 0; l < nl; ++l) {
                const LayerD& L = m->layers[l];
                QKVStore qs;
                qs.rows = rows;
                qs.kv = kv;
                qs.layer = l;
                qs.q16 = w.q16;
                if (l == 0) {
                    Epi e_qkv;
                    e_qkv.qkv = &qs;
                    matmul(L.qkv, act_for(w, w.x), T, L.qkv_b, 0, nullptr, s->st, e_qkv);
                } else {
                    const LayerD& P = m->layers[l - 1];
                    LnIn n2;
                    n2.a = w.ln1; n2.b = w.f; n2.g = P.ln2_w; n2.beta = P.ln2_b; n2.y_out = w.x;
                    matmul_ln(L.qkv, n2, T, L.qkv_b, 0, nullptr, &qs, s->st);
                }
                attention_rows(T, w.grp_row0, w.grp, w.n_grp, w.q16, rows, kv, l, kAttnScale, w.attn, L.out.type, act_of(w), s->st);
                matmul(L.out, act_for(w, w.attn), T, L.out_b, 0, w.o, s->st);
                LnIn n1;
                n1.a = w.x; n1.b = w.o; n1.g = L.ln1_w; n1.beta = L.ln1_b; n1.y_out = w.ln1;
                matmul_ln(L.up, n1, T, L.up_b, 1, w.h, nullptr, s->st);
                Epi e3;
                e3.quant_in = true;
                matmul(L.down, act_for(w, w.h), T, L.down_b, 0, w.f, s->st, e3);
            }
            if (fuse_head) {
                LnIn nz;
                nz.a = w.ln1; nz.b = w.f; nz.g = Z.ln2_w; nz.beta = Z.ln2_b; nz.y_out = w.x;
                matmul_ln(*head, nz, T, nullptr, 0, head_out, nullptr, s->st);
            }
        }   // (the final norm alone is launched without the attribute)
        if (fuse_head) return true;
        residual_layernorm(T, w.ln1, w.f, Z.ln2_w, Z.ln2_b, 1e-5f, w.x, final_qtype, act_of(w), s->st);
        return false;
    }
    PdlScope pdl(T <= pdl_rows());
    for (int l = 0; l < nl; ++l) {
        const LayerD& L = m->layers[l];
        const int next_q = (l + 1 < nl) ? m->layers[l + 1].qkv.type : final_qtype;
        QKVStore qs;
        qs.rows = rows;
        qs.kv = kv;
        qs.layer = l;
        qs.q16 = w.q16;
        Epi e_qkv;
        e_qkv.qkv = &qs;
        matmul(L.qkv, act_for(w, w.x), T, L.qkv_b, 0, nullptr, s->st, e_qkv);
        // decode and prefill rows alike: the row attends to positions [0, L) of its slot
        attention_rows(T, w.grp_row0, w.grp, w.n_grp, w.q16, rows, kv, l, kAttnScale, w.attn, L.out.type, act_of(w), s->st);
        if (small) {
            Tail t1;
            t1.kind = 1; t1.resid = w.x; t1.g = L.ln1_w; t1.beta = L.ln1_b; t1.eps = 1e-5f; t1.y_out = w.ln1;
            t1.qtype = L.up.type; t1.qo = act_of(w); t1.counter = s->tail_ctr;
            Epi e1;
            e1.tail = &t1;
            matmul(L.out, act_for(w, w.attn), T, L.out_b, 0, w.o, s->st, e1);
            matmul(L.up, act_for(w, w.ln1), T, L.up_b, 1, w.h, s->st);
            Tail t3;
            t3.kind = 1; t3.resid = w.ln1; t3.g = L.ln2_w; t3.beta = L.ln2_b; t3.eps = 1e-5f; t3.y_out = w.x;
            t3.qtype = next_q; t3.qo = act_of(w); t3.counter = s->tail_ctr;
            Epi e3;
            e3.tail = &t3;
            e3.quant_in = true;   // the FFN rows' conversion (Q8_0: inside the down projection)
            matmul(L.down, act_for(w, w.h), T, L.down_b, 0, w.f, s->st, e3);
        } else {
            matmul(L.out, act_for(w, w.attn), T, L.out_b, 0, w.o, s->st);
            residual_layernorm(T, w.x, w.o, L.ln1_w, L.ln1_b, 1e-5f, w.ln1, L.up.type, act_of(w), s->st);
            matmul(L.up, act_for(w, w.ln1), T, L.up_b, 1, w.h, s->st);
            ActQ a = act_of(w);
            quantize_act(L.down.type, w.h, T, s->ff, a, s->st);
            matmul(L.down, act_for(w, w.h), T, L.down_b, 0, w.f, s->st);
            residual_layernorm(T, w.ln1, w.f, L.ln2_w, L.ln2_b, 1e-5f, w.x, next_q, act_of(w), s->st);
        }
    }
    return false;
}

static void free_session(t2sx_session* s) {
    if (!s) return;
    DeviceGuard dg_;
    dg_.set(s->device);
    if (s->st) cudaStreamSynchronize(s->st);
    if (s->graph) cudaGraphExecDestroy(s->graph);
    if (s->host_graph) cudaGraphExecDestroy(s->host_graph);
    if (s->pin_in) cudaFreeHost(s->pin_in);
    if (s->pin_out) cudaFreeHost(s->pin_out);
    for (void* p : {(void*)s->pool, (void*)s->ptab, (void*)s->n_pos, (void*)s->audio_off, (void*)s->token_in, (void*)s->cap,
                    (void*)s->err, (void*)s->seen, (void*)s->pe, (void*)s->dec.mem, (void*)s->pre.mem, (void*)s->ring,
                    (void*)s->ring_step, (void*)s->scratch_i, (void*)s->noise, (void*)s->tail_ctr})
        if (p) cudaFree(p);
    if (s->ev0) cudaEventDestroy(s->ev0);
    if (s->ev1) cudaEventDestroy(s->ev1);
    if (s->st) cudaStreamDestroy(s->st);
    t2sx_model* m = const_cast<t2sx_model*>(s->m);
    const bool counted = s->counted;
    delete s;
    if (m && counted) {
        bool release = false;
        {
            std::lock_guard<std::mutex> lk(m->mu);
            release = (--m->live_sessions == 0) && m->free_requested;
        }
        if (release) release_model(m);
    }
}

extern "C" int t2sx_session_create(const t2sx_model* m, uint32_t n_slots, uint32_t slot_size, const t2sx_sampler_config* cfg,
                                   t2sx_session** out) {
    if (!m || !out) return fail(T2SX_ERR_INVALID, "t2sx_session_create: null argument");
    *out = nullptr;
    if (n_slots == 0 || slot_size == 0) return fail(T2SX_ERR_INVALID, "t2sx_session_create: n_batch and slot_size must be > 0");
    if (n_slots > (1u << 20) || slot_size > (1u << 20)) return fail(T2SX_ERR_INVALID, "t2sx_session_create: sizes too large");
    DeviceGuard dg_;
    CK(dg_.set(m->device));
    t2sx_session* s = new t2sx_session();
    s->m = m;
    s->device = m->device;
    {
        std::lock_guard<std::mutex> lk(const_cast<t2sx_model*>(m)->mu);
        if (m->free_requested) { delete s; return fail(T2SX_ERR_STATE, "t2sx_session_create: model already freed"); }
        ++const_cast<t2sx_model*>(m)->live_sessions;
        s->counted = true;
    }
    s->n_slots = (int)n_slots; s->slot_size = (int)slot_size;
    s->pages_per_slot = (int)((slot_size + kPage - 1) / kPage);
    s->n_layer = (int)m->hp[4]; s->V = (int)m->hp[5]; s->ff = (int)m->hp[3];
    if (cfg) s->cfg = *cfg;
    else { s->cfg.top_k = 15; s->cfg.top_p = 1.0f; s->cfg.temperature = 1.0f; s->cfg.repetition_penalty = 1.35f; s->cfg.eos_mask = 0; }
    if (!(s->cfg.repetition_penalty > 0.0f)) { delete s; return fail(T2SX_ERR_INVALID, "repetition_penalty must be > 0"); }
    int rc = T2SX_OK;
    auto ck = [&](cudaError_t e, const char* what) {
        if (e != cudaSuccess && rc == T2SX_OK)
            rc = fail(e == cudaErrorMemoryAllocation ? T2SX_ERR_OOM : T2SX_ERR_CUDA, "t2sx_session_create: %s: %s", what, cudaGetErrorString(e));
    };
    ck(cudaStreamCreateWithFlags(&s->st, cudaStreamNonBlocking), "stream");
    ck(cudaEventCreate(&s->ev0), "event"); ck(cudaEventCreate(&s->ev1), "event");
    const size_t page_elems = (size_t)s->n_layer * 2 * kHeads * kPage * kHeadDim;
    const size_t npages = (size_t)n_slots * s->pages_per_slot;
    s->pool_bytes = npages * page_elems * 2;
    ck(cudaMalloc(&s->pool, s->pool_bytes), "KV pages");
    ck(cudaMalloc(&s->ptab, npages * 4), "page table");
    ck(cudaMalloc(&s->n_pos, n_slots * 4), "state"); ck(cudaMalloc(&s->audio_off, n_slots * 4), "state");
    ck(cudaMalloc(&s->token_in, n_slots * 4), "state"); ck(cudaMalloc(&s->cap, n_slots * 4), "state");
    ck(cudaMalloc(&s->err, 4), "state"); ck(cudaMalloc(&s->scratch_i, n_slots * 4), "state");
    ck(cudaMalloc(&s->ring_step, 4), "state");
    ck(cudaMalloc(&s->tail_ctr, 4), "state");
    if (s->cfg.repetition_penalty != 1.0f) ck(cudaMalloc(&s->seen, (size_t)n_slots * s->V), "seen mask");
    ck(cudaMalloc(&s->pe, (size_t)slot_size * kD * 4), "PE table");
    if (rc) { free_session(s); return rc; }
    std::vector<float> pe((size_t)slot_size * kD);
    for (uint32_t p = 0; p < slot_size; ++p) pe_row((int)p, &pe[(size_t)p * kD]);
    ck(cudaMemcpy(s->pe, pe.data(), pe.size() * 4, cudaMemcpyHostToDevice), "PE upload");
    s->ptab_h.assign(npages, -1);
    ck(cudaMemset(s->ptab, 0xff, npages * 4), "memset");
    ck(cudaMemset(s->n_pos, 0, n_slots * 4), "memset"); ck(cudaMemset(s->audio_off, 0, n_slots * 4), "memset");
    ck(cudaMemset(s->token_in, 0, n_slots * 4), "memset"); ck(cudaMemset(s->cap, 0, n_slots * 4), "memset");
    ck(cudaMemset(s->err, 0, 4), "memset");
    ck(cudaMemset(s->tail_ctr, 0, 4), "memset");
    if (s->seen) ck(cudaMemset(s->seen, 0, (size_t)n_slots * s->V), "memset");
    if (rc) { free_session(s); return rc; }
    s->free_pages.resize(npages);
    for (size_t i = 0; i < npages; ++i) s->free_pages[i] = (int32_t)(npages - 1 - i);
    s->n_pos_h.assign(n_slots, 0);
    s->audio_off_h.assign(n_slots, 0);
    *out = s;
    return T2SX_OK;
}

extern "C" void t2sx_session_free(t2sx_session* s) { free_session(s); }

extern "C" int t2sx_session_find_free_slot(const t2sx_session* s) {
    if (!s) return -1;
    for (int i = 0; i < s->n_slots; ++i) if (s->n_pos_h[i] == 0) return i;
    return -1;
}

extern "C" int t2sx_session_slot_n_pos(const t2sx_session* s, int32_t slot) {
    if (!s || slot < 0 || slot >= s->n_slots) return -1;
    return s->n_pos_h[slot];
}

extern "C" int t2sx_session_slot_audio_offset(const t2sx_session* s, int32_t slot) {
    if (!s || slot < 0 || slot >= s->n_slots) return -1;
    return s->audio_off_h[slot];
}

extern "C" int t2sx_session_device_bytes(const t2sx_session* s, uint64_t* bytes) {
    if (!s || !bytes) return fail(T2SX_ERR_INVALID, "null argument");
    *bytes = s->pool_bytes + s->dec.bytes + s->pre.bytes + (size_t)s->slot_size * kD * 4;
    return T2SX_OK;
}

static void rebuild_active(t2sx_session* s) {
    s->active.clear();
    for (int i = 0; i < s->n_slots; ++i) if (s->n_pos_h[i] > 0) s->active.push_back(i);
    s->dec_dirty = true;
}

extern "C" int t2sx_session_slot_release(t2sx_session* s, int32_t slot) {
    if (!s || slot < 0 || slot >= s->n_slots) return fail(T2SX_ERR_INVALID, "t2sx_session_slot_release: bad slot %d", slot);
    DeviceGuard dg_;
    CK(dg_.set(s->m->device));
    CK(cudaStreamSynchronize(s->st));
    for (int p = 0; p < s->pages_per_slot; ++p) {
        int32_t& pg = s->ptab_h[(size_t)slot * s->pages_per_slot + p];
        if (pg >= 0) { s->free_pages.push_back(pg); pg = -1; }
    }
    const int32_t zero = 0;
    CK(cudaMemcpy(s->ptab + (size_t)slot * s->pages_per_slot, &s->ptab_h[(size_t)slot * s->pages_per_slot],
                  (size_t)s->pages_per_slot * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(s->n_pos + slot, &zero, 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(s->audio_off + slot, &zero, 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(s->cap + slot, &zero, 4, cudaMemcpyHostToDevice));
    s->n_pos_h[slot] = 0;
    s->audio_off_h[slot] = 0;
    rebuild_active(s);
    return T2SX_OK;
}

extern "C" int t2sx_embed_prefill(t2sx_session* s, const int32_t* phones, const float* bert, int32_t T_text, const int32_t* sem,
                                  int32_t T_prompt, float* x_out, int32_t x_out_on_device) {
    if (!s || !x_out || T_text < 0 || T_prompt < 0 || T_text + T_prompt <= 0 || (T_text && (!phones || !bert)) ||
        (T_prompt && !sem))
        return fail(T2SX_ERR_INVALID, "t2sx_embed_prefill: bad arguments");
    const t2sx_model* m = s->m;
    const int T = T_text + T_prompt;
    if (T > s->slot_size) return fail(T2SX_ERR_INVALID, "t2sx_embed_prefill: %d rows exceed slot_size %d (PE table)", T, s->slot_size);
    for (int i = 0; i < T_text; ++i) if (phones[i] < 0 || phones[i] >= m->text_rows) return fail(T2SX_ERR_INVALID, "phoneme id %d out of range", phones[i]);
    for (int i = 0; i < T_prompt; ++i) if (sem[i] < 0 || sem[i] >= m->audio_rows) return fail(T2SX_ERR_INVALID, "semantic id %d out of range", sem[i]);
    DeviceGuard dg_;
    CK(dg_.set(m->device));
    ErrScope es_(s->err);   // bounded-wait failures of this call's kernels land here
    int rc = work_alloc(s->pre, T_text > 0 ? (T_text * 2 > T ? T_text * 2 : T) : T, s->V, s->ff);
    if (rc) return rc;
    Work& w = s->pre;
    // ids in row_slot / row_pos scratch, BERT features in h (T_text x 1024 <= T x ff), projection in o
    int32_t* d_ph = w.row_slot; int32_t* d_sem = w.row_pos;
    if (T_text) CK(cudaMemcpyAsync(d_ph, phones, T_text * 4, cudaMemcpyHostToDevice, s->st));
    if (T_prompt) CK(cudaMemcpyAsync(d_sem, sem, T_prompt * 4, cudaMemcpyHostToDevice, s->st));
    if (T_text) {
        CK(cudaMemcpyAsync(w.h, bert, (size_t)T_text * 1024 * 4, cudaMemcpyHostToDevice, s->st));
        ActQ a = act_for(w, w.h);
        quantize_act(m->bert.type, w.h, T_text, 1024, a, s->st);
        matmul(m->bert, a, T_text, m->bert_b, 0, w.o, s->st);
    }
    float* dst = x_out_on_device ? x_out : w.x;
    embed_prefill_rows(T_text, T_prompt, d_ph, d_sem, w.o, m->text16, m->text32, m->audio16, m->audio32, s->pe,
                       m->alpha_text, m->alpha_audio, dst, s->st);
    CK(cudaGetLastError());
    if (!x_out_on_device) CK(cudaMemcpyAsync(x_out, w.x, (size_t)T * kD * 4, cudaMemcpyDeviceToHost, s->st));
    CK(cudaStreamSynchronize(s->st));
    return T2SX_OK;
}

static int check_err_flag(t2sx_session* s) {
    int32_t e = 0;
    CK(cudaMemcpy(&e, s->err, 4, cudaMemcpyDeviceToHost));
    if (e) {
        const int32_t z = 0;
        CK(cudaMemcpy(s->err, &z, 4, cudaMemcpyHostToDevice));
        if (e == 3) return fail(T2SX_ERR_TIMEOUT, "a tensor-core matmul gave up waiting; the pass's outputs are NaN");
        return fail(T2SX_ERR_BOUNDS, "a slot ran past its KV capacity");
    }
    return T2SX_OK;
}

static void run_sampler(t2sx_session* s, int T, const float* logits, const int32_t* row_slot, const uint8_t* seen,
                        int32_t* tok, int32_t* greedy);

// Rows of one prefill pass at most (the prefill work buffers are sized for this many).
static const int64_t kChunk = 32768;

// Validates the prefill part of a plan (t2s_session_flex_advance checks, session.cpp:461-540).
static int check_prefill(t2sx_session* s, int32_t n, const int32_t* slots, const int32_t* n_query, const int32_t* t_prompt,
                         std::vector<char>& used, const char* who) {
    for (int i = 0; i < n; ++i) {
        const int sl = slots[i];
        if (sl < 0 || sl >= s->n_slots || used[sl]) return fail(T2SX_ERR_INVALID, "%s: bad or repeated slot %d", who, sl);
        used[sl] = 1;
        if (s->n_pos_h[sl] != 0) return fail(T2SX_ERR_STATE, "%s: slot %d is not idle (n_pos=%d)", who, sl, s->n_pos_h[sl]);
        if (n_query[i] <= 0 || n_query[i] > s->slot_size) return fail(T2SX_ERR_INVALID, "%s: n_query %d out of range", who, n_query[i]);
        if (t_prompt[i] < 0 || n_query[i] < t_prompt[i])
            return fail(T2SX_ERR_INVALID, "%s: n_query < ref_T_prompt (audio_offset would be negative)", who);
        if ((int64_t)s->free_pages.size() < (int64_t)(i + 1) * s->pages_per_slot) return fail(T2SX_ERR_OOM, "%s: out of KV pages", who);
    }
    return T2SX_OK;
}

// Gives each slot its pages from the free list (a slot holds slot_size positions).
static int assign_pages(t2sx_session* s, int32_t n, const int32_t* slots) {
    for (int i = 0; i < n; ++i) {
        const int sl = slots[i];
        for (int p = 0; p < s->pages_per_slot; ++p) {
            s->ptab_h[(size_t)sl * s->pages_per_slot + p] = s->free_pages.back();
            s->free_pages.pop_back();
        }
        CK(cudaMemcpyAsync(s->ptab + (size_t)sl * s->pages_per_slot, &s->ptab_h[(size_t)sl * s->pages_per_slot],
                           (size_t)s->pages_per_slot * 4, cudaMemcpyHostToDevice, s->st));
        const int32_t cap = s->slot_size;
        CK(cudaMemcpyAsync(s->cap + sl, &cap, 4, cudaMemcpyHostToDevice, s->st));
    }
    CK(cudaStreamSynchronize(s->st));
    return T2SX_OK;
}

// Slot state after its prefill: n_pos = n_query, audio_offset = n_query - T_prompt, the first
// token as the next input and as the only seen token.
static int finish_prefill(t2sx_session* s, int sl, int nq, int tp, int32_t tok) {
    s->n_pos_h[sl] = nq;
    s->audio_off_h[sl] = nq - tp;
    CK(cudaMemcpyAsync(s->n_pos + sl, &s->n_pos_h[sl], 4, cudaMemcpyHostToDevice, s->st));
    CK(cudaMemcpyAsync(s->audio_off + sl, &s->audio_off_h[sl], 4, cudaMemcpyHostToDevice, s->st));
    CK(cudaMemcpyAsync(s->token_in + sl, &tok, 4, cudaMemcpyHostToDevice, s->st));
    if (s->seen) {
        CK(cudaMemsetAsync(s->seen + (size_t)sl * s->V, 0, s->V, s->st));
        const uint8_t one = 1;
        CK(cudaMemcpyAsync(s->seen + (size_t)sl * s->V + tok, &one, 1, cudaMemcpyHostToDevice, s->st));
    }
    return T2SX_OK;
}

extern "C" int t2sx_prefill(t2sx_session* s, int32_t n, const int32_t* slots, const int32_t* n_query, const int32_t* t_prompt,
                            const float* x, int32_t x_on_device, int32_t* tokens_out) {
    if (!s || n <= 0 || !slots || !n_query || !t_prompt || !x) return fail(T2SX_ERR_INVALID, "t2sx_prefill: bad arguments");
    std::vector<char> used(s->n_slots, 0);
    {
        const int rc0 = check_prefill(s, n, slots, n_query, t_prompt, used, "t2sx_prefill");
        if (rc0) return rc0;
    }
    const t2sx_model* m = s->m;
    DeviceGuard dg_;
    CK(dg_.set(m->device));
    ErrScope es_(s->err);   // bounded-wait failures of this call's kernels land here
    int rc;
    if ((rc = assign_pages(s, n, slots))) return rc;
    // process slots in chunks of at most kChunk rows
    std::vector<int32_t> toks(n, 0);
    int64_t xoff = 0;
    for (int i0 = 0; i0 < n;) {
        int i1 = i0;
        int64_t rows = 0;
        while (i1 < n && (rows == 0 || rows + n_query[i1] <= kChunk)) rows += n_query[i1++];
        const int T = (int)rows, ns = i1 - i0;
        if ((rc = work_alloc(s->pre, T > ns ? T : ns, s->V, s->ff))) return rc;
        Work& w = s->pre;
        std::vector<int32_t> rs(T), rp(T), rl(T), last(ns);
        int r = 0;
        for (int i = i0; i < i1; ++i) {
            const int T_text = n_query[i] - t_prompt[i];
            for (int j = 0; j < n_query[i]; ++j, ++r) {
                rs[r] = slots[i]; rp[r] = j; rl[r] = (j < T_text) ? T_text : (j + 1);
            }
            last[i - i0] = r - 1;
        }
        CK(cudaMemcpyAsync(w.row_slot, rs.data(), T * 4, cudaMemcpyHostToDevice, s->st));
        CK(cudaMemcpyAsync(w.row_pos, rp.data(), T * 4, cudaMemcpyHostToDevice, s->st));
        CK(cudaMemcpyAsync(w.row_L, rl.data(), T * 4, cudaMemcpyHostToDevice, s->st));
        CK(cudaMemcpyAsync(w.lastrow, last.data(), ns * 4, cudaMemcpyHostToDevice, s->st));
        CK(cudaMemcpyAsync(w.x, x + xoff * kD, (size_t)T * kD * 4, x_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, s->st));
        {
            ActQ a0 = act_of(w);
            quantize_act(m->layers[0].qkv.type, w.x, T, kD, a0, s->st);
        }
        if ((rc = set_row_groups(s, w, T, 0, rs))) return rc;
        run_layers(s, w, T, false, -1);
        w.n_grp = 0;
        // sampler on each slot's last row
        gather_rows(ns, w.x, w.lastrow, kD, w.xl, s->st);
        ActQ a = act_for(w, w.xl);
        quantize_act(m->lm_head.type, w.xl, ns, kD, a, s->st);
        matmul(m->lm_head, a, ns, nullptr, 0, w.logits, s->st);
        for (int i = i0; i < i1; ++i) rs[i - i0] = slots[i];
        CK(cudaMemcpyAsync(w.row_slot, rs.data(), ns * 4, cudaMemcpyHostToDevice, s->st));
        run_sampler(s, ns, w.logits, w.row_slot, nullptr, w.tok, w.greedy);
        CK(cudaGetLastError());
        CK(cudaMemcpyAsync(toks.data() + i0, w.tok, ns * 4, cudaMemcpyDeviceToHost, s->st));
        CK(cudaStreamSynchronize(s->st));
        s->last_rows = ns;
        s->last_logits = w.logits;
        s->last_greedy = w.greedy;
        s->last_hidden_rows = T;
        s->last_hidden = w.x;
        xoff += rows;
        i0 = i1;
    }
    if ((rc = check_err_flag(s))) return rc;
    for (int i = 0; i < n; ++i) {
        if ((rc = finish_prefill(s, slots[i], n_query[i], t_prompt[i], toks[i]))) return rc;
        if (tokens_out) tokens_out[i] = toks[i];
    }
    CK(cudaStreamSynchronize(s->st));
    rebuild_active(s);
    return T2SX_OK;
}

// Sampler of one pass: the greedy argmax kernel, or the full chain when noise is set.
static void run_sampler(t2sx_session* s, int T, const float* logits, const int32_t* row_slot, const uint8_t* seen,
                        int32_t* tok, int32_t* greedy) {
    const t2sx_model* m = s->m;
    const float rp = s->cfg.repetition_penalty;
    if (!s->noise_on) {
        sample_greedy(T, logits, s->V, row_slot, seen, rp, 1.0f / rp, s->cfg.eos_mask, (int)m->hp[7], tok, greedy, s->st);
        return;
    }
    SamplerArgs a;
    a.top_k = s->cfg.top_k;
    a.top_p = s->cfg.top_p;
    a.inv_t = 1.0f / fmaxf(s->cfg.temperature, 1.0e-5f);
    a.rp = rp;
    a.inv_rp = 1.0f / rp;
    a.eos_mask = s->cfg.eos_mask;
    a.eos = (int)m->hp[7];
    a.noise = s->noise;
    sample_full(T, logits, s->V, row_slot, seen, a, tok, greedy, s->st);
}

// Record one decode step for the active rows on s->st (captured into the step graph).
static void enqueue_step(t2sx_session* s) {
    const t2sx_model* m = s->m;
    Work& w = s->dec;
    const int T = (int)s->active.size();
    Rows rows = rows_of(s, w);
    embed_decode(T, w.row_slot, s->token_in, s->n_pos, s->audio_off, m->audio16, m->audio32, m->audio_rows, s->pe, s->slot_size,
                 m->alpha_audio, rows, w.x, m->layers[0].qkv.type, act_of(w), s->st);
    if (!run_layers(s, w, T, true, m->lm_head.type, &m->lm_head, w.logits))
        matmul(m->lm_head, act_for(w, w.x), T, nullptr, 0, w.logits, s->st);
    run_sampler(s, T, w.logits, w.row_slot, s->seen, w.tok, w.greedy);
    advance(T, w.row_slot, w.tok, s->token_in, s->n_pos, s->seen, s->V, s->ring, s->ring_len, s->ring_step, s->st);
}

static int prepare_decode(t2sx_session* s, int n_steps) {
    const int T = (int)s->active.size();
    if (T == 0) return fail(T2SX_ERR_STATE, "decode: no active slot (prefill first)");
    for (int sl : s->active)
        if (s->n_pos_h[sl] + n_steps > s->slot_size)
            return fail(T2SX_ERR_BOUNDS, "decode: slot %d would exceed slot_size %d (n_pos=%d, steps=%d)", sl, s->slot_size,
                        s->n_pos_h[sl], n_steps);
    int rc;
    if ((rc = work_alloc(s->dec, s->n_slots, s->V, s->ff))) return rc;
    if (!s->ring) CK(cudaMalloc(&s->ring, (size_t)s->ring_len * s->n_slots * 4));
    if (s->dec_dirty) {
        CK(cudaMemcpyAsync(s->dec.row_slot, s->active.data(), T * 4, cudaMemcpyHostToDevice, s->st));
        CK(cudaStreamSynchronize(s->st));
        CK(cudaGetLastError());
        if (s->graph && (s->dec_rows != T || s->graph_noise != s->noise_on)) { cudaGraphExecDestroy(s->graph); s->graph = nullptr; }
        if (!s->graph) {
            cudaGraph_t g;
            CK(cudaStreamBeginCapture(s->st, cudaStreamCaptureModeThreadLocal));
            enqueue_step(s);
            cudaError_t e = cudaStreamEndCapture(s->st, &g);
            if (e != cudaSuccess) return fail(T2SX_ERR_CUDA, "decode graph capture: %s", cudaGetErrorString(e));
            e = cudaGetLastError();
            if (e != cudaSuccess) { cudaGraphDestroy(g); return fail(T2SX_ERR_CUDA, "decode step launch during capture: %s", cudaGetErrorString(e)); }
            size_t nn = 0;
            cudaGraphGetNodes(g, nullptr, &nn);
            std::vector<cudaGraphNode_t> nodes(nn);
            if (nn) cudaGraphGetNodes(g, nodes.data(), &nn);
            s->graph_kernels = 0;
            for (auto nd : nodes) {
                cudaGraphNodeType ty;
                if (cudaGraphNodeGetType(nd, &ty) == cudaSuccess && ty == cudaGraphNodeTypeKernel) ++s->graph_kernels;
            }
            e = cudaGraphInstantiate(&s->graph, g, 0);
            cudaGraphDestroy(g);
            if (e != cudaSuccess) { s->graph = nullptr; return fail(T2SX_ERR_CUDA, "decode graph instantiate: %s", cudaGetErrorString(e)); }
            s->dec_rows = T;
            s->graph_noise = s->noise_on;
            ++s->graph_gen;
        }
        s->dec_dirty = false;
    }
    return T2SX_OK;
}

static int launch_steps(t2sx_session* s, int n_steps) {
    CK(cudaEventRecord(s->ev0, s->st));
    for (int i = 0; i < n_steps; ++i) CK(cudaGraphLaunch(s->graph, s->st));
    CK(cudaEventRecord(s->ev1, s->st));
    for (int sl : s->active) s->n_pos_h[sl] += n_steps;
    s->last_rows = (int)s->active.size();
    s->last_logits = s->dec.logits;
    s->last_greedy = s->dec.greedy;
    s->last_hidden_rows = (int)s->active.size();
    s->last_hidden = s->dec.x;
    return T2SX_OK;
}

extern "C" int t2sx_decode_async(t2sx_session* s, int32_t n_steps) {
    if (!s || n_steps < 0) return fail(T2SX_ERR_INVALID, "t2sx_decode_async: bad arguments");
    if (n_steps == 0) return T2SX_OK;
    DeviceGuard dg_;
    CK(dg_.set(s->m->device));
    ErrScope es_(s->err);   // bounded-wait failures of this call's kernels land here
    {
        const cudaError_t stale = cudaGetLastError();
        if (stale != cudaSuccess) return fail(T2SX_ERR_CUDA, "pending CUDA error before decode: %s", cudaGetErrorString(stale));
    }
    int rc;
    if ((rc = prepare_decode(s, n_steps))) return rc;
    CK(cudaMemsetAsync(s->ring_step, 0, 4, s->st));
    return launch_steps(s, n_steps);
}

extern "C" int t2sx_synchronize(t2sx_session* s) {
    if (!s) return fail(T2SX_ERR_INVALID, "null session");
    DeviceGuard dg_;
    CK(dg_.set(s->m->device));
    CK(cudaStreamSynchronize(s->st));
    CK(cudaEventElapsedTime(&s->last_ms, s->ev0, s->ev1));
    return check_err_flag(s);
}

extern "C" int t2sx_decode(t2sx_session* s, int32_t n_steps, int32_t* tokens_out) {
    if (!s || n_steps < 0) return fail(T2SX_ERR_INVALID, "t2sx_decode: bad arguments");
    if (n_steps == 0) return T2SX_OK;
    DeviceGuard dg_;
    CK(dg_.set(s->m->device));
    ErrScope es_(s->err);   // bounded-wait failures of this call's kernels land here
    {
        const cudaError_t stale = cudaGetLastError();
        if (stale != cudaSuccess) return fail(T2SX_ERR_CUDA, "pending CUDA error before decode: %s", cudaGetErrorString(stale));
    }
    int rc;
    if ((rc = prepare_decode(s, n_steps))) return rc;
    const int T = (int)s->active.size();
    float total = 0.0f;
    for (int done = 0; done < n_steps;) {
        const int k = (n_steps - done) < s->ring_len ? (n_steps - done) : s->ring_len;
        CK(cudaMemsetAsync(s->ring_step, 0, 4, s->st));
        if ((rc = launch_steps(s, k))) return rc;
        if (tokens_out)
            CK(cudaMemcpyAsync(tokens_out + (size_t)done * T, s->ring, (size_t)k * T * 4, cudaMemcpyDeviceToHost, s->st));
        CK(cudaStreamSynchronize(s->st));
        float ms = 0.0f;
        CK(cudaEventElapsedTime(&ms, s->ev0, s->ev1));
        total += ms;
        done += k;
    }
    s->last_ms = total;
    return check_err_flag(s);
}

__global__ void k_scatter_tokens(int T, const int32_t* row_slot, const int32_t* tok, int32_t* token_in) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r < T) token_in[row_slot[r]] = tok[r];
}

// The host-step graph (T2SX_HOST_GRAPH=0: separate copies and launches, as before).
static bool host_graph_on() {
    static const bool v = [] {
        const char* e = getenv("T2SX_HOST_GRAPH");
        return !(e && e[0] == '0');
    }();
    return v;
}

// Captures, for the current step graph, the whole host step: pinned tokens -> device, scatter to
// the slots, ring reset, timing event, the step, timing event, next tokens -> pinned.
static int build_host_graph(t2sx_session* s) {
    if (s->host_graph && s->host_gen == s->graph_gen) return T2SX_OK;
    if (s->host_graph) { cudaGraphExecDestroy(s->host_graph); s->host_graph = nullptr; }
    if (!s->pin_in) CK(cudaHostAlloc((void**)&s->pin_in, (size_t)s->n_slots * 4, cudaHostAllocDefault));
    if (!s->pin_out) CK(cudaHostAlloc((void**)&s->pin_out, (size_t)s->n_slots * 4, cudaHostAllocDefault));
    const int T = (int)s->active.size();
    cudaGraph_t g;
    CK(cudaStreamBeginCapture(s->st, cudaStreamCaptureModeThreadLocal));
    cudaMemcpyAsync(s->scratch_i, s->pin_in, (size_t)T * 4, cudaMemcpyHostToDevice, s->st);
    k_scatter_tokens<<<(T + 255) / 256, 256, 0, s->st>>>(T, s->dec.row_slot, s->scratch_i, s->token_in);
    cudaMemsetAsync(s->ring_step, 0, 4, s->st);
    cudaEventRecordWithFlags(s->ev0, s->st, cudaEventRecordExternal);   // (event-record nodes, not capture markers)
    enqueue_step(s);
    cudaEventRecordWithFlags(s->ev1, s->st, cudaEventRecordExternal);
    cudaMemcpyAsync(s->pin_out, s->dec.tok, (size_t)T * 4, cudaMemcpyDeviceToHost, s->st);
    cudaError_t e = cudaStreamEndCapture(s->st, &g);
    if (e != cudaSuccess) return fail(T2SX_ERR_CUDA, "host step graph capture: %s", cudaGetErrorString(e));
    e = cudaGetLastError();
    if (e != cudaSuccess) { cudaGraphDestroy(g); return fail(T2SX_ERR_CUDA, "host step graph: %s", cudaGetErrorString(e)); }
    e = cudaGraphInstantiate(&s->host_graph, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) { s->host_graph = nullptr; return fail(T2SX_ERR_CUDA, "host step graph instantiate: %s", cudaGetErrorString(e)); }
    s->host_gen = s->graph_gen;
    return T2SX_OK;
}

extern "C" int t2sx_decode_step_host(t2sx_session* s, const int32_t* tokens_in, int32_t* tokens_out) {
    if (!s) return fail(T2SX_ERR_INVALID, "null session");
    DeviceGuard dg_;
    CK(dg_.set(s->m->device));
    ErrScope es_(s->err);   // bounded-wait failures of this call's kernels land here
    {
        const cudaError_t stale = cudaGetLastError();
        if (stale != cudaSuccess) return fail(T2SX_ERR_CUDA, "pending CUDA error before decode: %s", cudaGetErrorString(stale));
    }
    int rc;
    if ((rc = prepare_decode(s, 1))) return rc;
    const int T = (int)s->active.size();
    if (tokens_in)
        for (int i = 0; i < T; ++i)
            if (tokens_in[i] < 0 || tokens_in[i] >= s->m->audio_rows) return fail(T2SX_ERR_INVALID, "token id %d out of range", tokens_in[i]);
    if (tokens_in && tokens_out && host_graph_on()) {
        // one launch per step: the tokens pass through session-owned pinned buffers
        if ((rc = build_host_graph(s))) return rc;
        memcpy(s->pin_in, tokens_in, (size_t)T * 4);
        CK(cudaGraphLaunch(s->host_graph, s->st));
        for (int sl : s->active) s->n_pos_h[sl] += 1;
        s->last_rows = T;
        s->last_logits = s->dec.logits;
        s->last_greedy = s->dec.greedy;
        s->last_hidden_rows = T;
        s->last_hidden = s->dec.x;
        CK(cudaStreamSynchronize(s->st));
        memcpy(tokens_out, s->pin_out, (size_t)T * 4);
        CK(cudaEventElapsedTime(&s->last_ms, s->ev0, s->ev1));
        return T2SX_OK;
    }
    if (tokens_in) {
        CK(cudaMemcpyAsync(s->scratch_i, tokens_in, T * 4, cudaMemcpyHostToDevice, s->st));
        k_scatter_tokens<<<(T + 255) / 256, 256, 0, s->st>>>(T, s->dec.row_slot, s->scratch_i, s->token_in);
        CK(cudaGetLastError());
    }
    CK(cudaMemsetAsync(s->ring_step, 0, 4, s->st));
    if ((rc = launch_steps(s, 1))) return rc;
    if (tokens_out) CK(cudaMemcpyAsync(tokens_out, s->dec.tok, T * 4, cudaMemcpyDeviceToHost, s->st));
    CK(cudaStreamSynchronize(s->st));
    CK(cudaEventElapsedTime(&s->last_ms, s->ev0, s->ev1));
    return T2SX_OK;
}

// One pass over a mixed plan (the flex graph of session.cpp:461-859 with decode and prefill slots):
// rows [0, n_dec) are one decode step of the listed slots, then each prefill slot's n_query rows.
// The layers run once over all rows; the sampler picks a token for every decode row and for the
// last row of every prefill slot.  Per-row arithmetic is the one of t2sx_decode_step_host and
// t2sx_prefill, so the tokens equal those of the two separate passes.
extern "C" int t2sx_flex_step(t2sx_session* s, int32_t n_dec, const int32_t* dec_slots, const int32_t* dec_tokens,
                              int32_t n_pre, const int32_t* pre_slots, const int32_t* n_query, const int32_t* t_prompt,
                              const float* x, int32_t* tokens_out) {
    if (!s || n_dec < 0 || n_pre < 0 || n_dec + n_pre == 0 || (n_dec && (!dec_slots || !dec_tokens)) ||
        (n_pre && (!pre_slots || !n_query || !t_prompt || !x)))
        return fail(T2SX_ERR_INVALID, "t2sx_flex_step: bad arguments");
    const t2sx_model* m = s->m;
    std::vector<char> used(s->n_slots, 0);
    int64_t T64 = n_dec;
    for (int i = 0; i < n_dec; ++i) {
        const int sl = dec_slots[i];
        if (sl < 0 || sl >= s->n_slots || used[sl]) return fail(T2SX_ERR_INVALID, "t2sx_flex_step: bad or repeated slot %d", sl);
        used[sl] = 1;
        if (s->n_pos_h[sl] == 0) return fail(T2SX_ERR_STATE, "t2sx_flex_step: decode of an idle slot %d", sl);
        if (s->n_pos_h[sl] + 1 > s->slot_size)
            return fail(T2SX_ERR_BOUNDS, "t2sx_flex_step: slot %d would exceed slot_size %d", sl, s->slot_size);
        if (dec_tokens[i] < 0 || dec_tokens[i] >= m->audio_rows) return fail(T2SX_ERR_INVALID, "token id %d out of range", dec_tokens[i]);
    }
    int rc;
    if ((rc = check_prefill(s, n_pre, pre_slots, n_query, t_prompt, used, "t2sx_flex_step"))) return rc;
    for (int i = 0; i < n_pre; ++i) T64 += n_query[i];
    if (T64 > kChunk) return fail(T2SX_ERR_INVALID, "t2sx_flex_step: %lld rows in one pass (at most %lld)", (long long)T64, (long long)kChunk);
    const int T = (int)T64, ns = n_dec + n_pre;
    DeviceGuard dg_;
    CK(dg_.set(m->device));
    ErrScope es_(s->err);   // bounded-wait failures of this call's kernels land here
    {
        const cudaError_t stale = cudaGetLastError();
        if (stale != cudaSuccess) return fail(T2SX_ERR_CUDA, "pending CUDA error before the pass: %s", cudaGetErrorString(stale));
    }
    if ((rc = assign_pages(s, n_pre, pre_slots))) return rc;
    if ((rc = work_alloc(s->pre, T, s->V, s->ff))) return rc;
    Work& w = s->pre;
    std::vector<int32_t> rs(T), rp(T), rl(T), last(ns), samp(ns);
    int r = 0;
    for (int i = 0; i < n_dec; ++i, ++r) {
        rs[r] = dec_slots[i]; rp[r] = s->n_pos_h[dec_slots[i]]; rl[r] = rp[r] + 1;
        last[i] = r; samp[i] = dec_slots[i];
    }
    for (int i = 0; i < n_pre; ++i) {
        const int T_text = n_query[i] - t_prompt[i];
        for (int j = 0; j < n_query[i]; ++j, ++r) {
            rs[r] = pre_slots[i]; rp[r] = j; rl[r] = (j < T_text) ? T_text : (j + 1);
        }
        last[n_dec + i] = r - 1; samp[n_dec + i] = pre_slots[i];
    }
    CK(cudaMemcpyAsync(w.row_slot, rs.data(), T * 4, cudaMemcpyHostToDevice, s->st));
    CK(cudaMemcpyAsync(w.row_pos, rp.data(), T * 4, cudaMemcpyHostToDevice, s->st));
    CK(cudaMemcpyAsync(w.row_L, rl.data(), T * 4, cudaMemcpyHostToDevice, s->st));
    CK(cudaMemcpyAsync(w.lastrow, last.data(), ns * 4, cudaMemcpyHostToDevice, s->st));
    if (n_pre) CK(cudaMemcpyAsync(w.x + (size_t)n_dec * kD, x, (size_t)(T - n_dec) * kD * 4, cudaMemcpyHostToDevice, s->st));
    if (n_dec) {
        CK(cudaMemcpyAsync(s->scratch_i, dec_tokens, n_dec * 4, cudaMemcpyHostToDevice, s->st));
        k_scatter_tokens<<<(n_dec + 255) / 256, 256, 0, s->st>>>(n_dec, w.row_slot, s->scratch_i, s->token_in);
        embed_decode(n_dec, w.row_slot, s->token_in, s->n_pos, s->audio_off, m->audio16, m->audio32, m->audio_rows, s->pe,
                     s->slot_size, m->alpha_audio, rows_of(s, w), w.x, m->layers[0].qkv.type, act_of(w), s->st);
    }
    {
        ActQ a0 = act_of(w);
        quantize_act(m->layers[0].qkv.type, w.x, T, kD, a0, s->st);
    }
    if ((rc = set_row_groups(s, w, T, n_dec, rs))) return rc;
    run_layers(s, w, T, false, -1);
    w.n_grp = 0;
    gather_rows(ns, w.x, w.lastrow, kD, w.xl, s->st);
    ActQ a = act_for(w, w.xl);
    quantize_act(m->lm_head.type, w.xl, ns, kD, a, s->st);
    matmul(m->lm_head, a, ns, nullptr, 0, w.logits, s->st);
    // the prefill rows sample with an empty seen set, as in t2sx_prefill
    for (int i = 0; s->seen && i < n_pre; ++i) CK(cudaMemsetAsync(s->seen + (size_t)pre_slots[i] * s->V, 0, s->V, s->st));
    CK(cudaMemcpyAsync(w.row_slot, samp.data(), ns * 4, cudaMemcpyHostToDevice, s->st));
    run_sampler(s, ns, w.logits, w.row_slot, s->seen, w.tok, w.greedy);
    // decode rows: token_in, n_pos + 1 and the seen set, as in the decode step
    if (n_dec) advance(n_dec, w.row_slot, w.tok, s->token_in, s->n_pos, s->seen, s->V, nullptr, 0, s->ring_step, s->st);
    CK(cudaGetLastError());
    std::vector<int32_t> toks(ns, 0);
    CK(cudaMemcpyAsync(toks.data(), w.tok, ns * 4, cudaMemcpyDeviceToHost, s->st));
    CK(cudaStreamSynchronize(s->st));
    s->last_rows = ns;
    s->last_logits = w.logits;
    s->last_greedy = w.greedy;
    s->last_hidden_rows = T;
    s->last_hidden = w.x;
    if ((rc = check_err_flag(s))) return rc;
    for (int i = 0; i < n_dec; ++i) s->n_pos_h[dec_slots[i]] += 1;
    for (int i = 0; i < n_pre; ++i)
        if ((rc = finish_prefill(s, pre_slots[i], n_query[i], t_prompt[i], toks[n_dec + i]))) return rc;
    CK(cudaStreamSynchronize(s->st));
    if (tokens_out) std::copy(toks.begin(), toks.end(), tokens_out);
    if (n_pre) rebuild_active(s);
    return T2SX_OK;
}

extern "C" int t2sx_active_slots(t2sx_session* s, int32_t* slots, int32_t* n) {
    if (!s || !n) return fail(T2SX_ERR_INVALID, "null argument");
    *n = (int32_t)s->active.size();
    if (slots) for (size_t i = 0; i < s->active.size(); ++i) slots[i] = s->active[i];
    return T2SX_OK;
}

extern "C" int t2sx_read_logits(t2sx_session* s, float* out, int32_t max_rows, int32_t* rows) {
    if (!s || !out) return fail(T2SX_ERR_INVALID, "null argument");
    DeviceGuard dg_;
    CK(dg_.set(s->m->device));
    CK(cudaStreamSynchronize(s->st));
    const int n = s->last_rows < max_rows ? s->last_rows : max_rows;
    if (!s->last_logits) return fail(T2SX_ERR_STATE, "no logits yet");
    CK(cudaMemcpy(out, s->last_logits, (size_t)n * s->V * 4, cudaMemcpyDeviceToHost));
    if (rows) *rows = n;
    return T2SX_OK;
}

extern "C" int t2sx_read_hidden(t2sx_session* s, float* out, int32_t max_rows, int32_t* rows) {
    if (!s || !out || max_rows < 0) return fail(T2SX_ERR_INVALID, "t2sx_read_hidden: bad arguments");
    DeviceGuard dg_;
    CK(dg_.set(s->m->device));
    CK(cudaStreamSynchronize(s->st));
    if (!s->last_hidden) return fail(T2SX_ERR_STATE, "t2sx_read_hidden: no pass yet");
    const int n = s->last_hidden_rows < max_rows ? s->last_hidden_rows : max_rows;
    CK(cudaMemcpy(out, s->last_hidden, (size_t)n * kD * 4, cudaMemcpyDeviceToHost));
    if (rows) *rows = n;
    return T2SX_OK;
}

extern "C" int t2sx_model_tensor_info(const t2sx_model* m, const char* name, int32_t* type, int32_t* n_dims, int64_t* ne) {
    if (!m || !name) return fail(T2SX_ERR_INVALID, "t2sx_model_tensor_info: null argument");
    auto it = m->tinfo.find(name);
    if (it == m->tinfo.end()) return fail(T2SX_ERR_INVALID, "t2sx_model_tensor_info: no tensor '%s' in the GGUF", name);
    if (type) *type = it->second.type;
    if (n_dims) *n_dims = it->second.nd;
    if (ne) for (int i = 0; i < 4; ++i) ne[i] = it->second.ne[i];
    return T2SX_OK;
}

extern "C" int t2sx_read_kv(t2sx_session* s, int32_t slot, int32_t layer, int32_t which, uint16_t* out) {
    if (!s || !out || slot < 0 || slot >= s->n_slots || layer < 0 || layer >= s->n_layer || (which != 0 && which != 1))
        return fail(T2SX_ERR_INVALID, "t2sx_read_kv: bad arguments");
    DeviceGuard dg_;
    CK(dg_.set(s->m->device));
    CK(cudaStreamSynchronize(s->st));
    const int n = s->n_pos_h[slot];
    std::vector<uint16_t> page((size_t)kHeads * kPage * kHeadDim);
    for (int p0 = 0; p0 < n; p0 += kPage) {
        const int pg = s->ptab_h[(size_t)slot * s->pages_per_slot + p0 / kPage];
        const size_t n_pages = (size_t)s->n_slots * s->pages_per_slot;
        const size_t off = ((((size_t)layer * n_pages + pg) * 2 + which) * kHeads) * kPage * kHeadDim;
        CK(cudaMemcpy(page.data(), s->pool + off, page.size() * 2, cudaMemcpyDeviceToHost));
        for (int i = p0; i < n && i < p0 + kPage; ++i)
            for (int h = 0; h < kHeads; ++h)
                memcpy(out + (size_t)i * kD + h * kHeadDim, &page[((size_t)h * kPage + (i - p0)) * kHeadDim], kHeadDim * 2);
    }
    return T2SX_OK;
}

extern "C" int t2sx_set_seen(t2sx_session* s, int32_t slot, const uint8_t* seen) {
    if (!s || !seen || slot < 0 || slot >= s->n_slots) return fail(T2SX_ERR_INVALID, "t2sx_set_seen: bad arguments");
    if (!s->seen) return T2SX_OK;  // repetition penalty disabled: nothing to track
    DeviceGuard dg_;
    CK(dg_.set(s->m->device));
    CK(cudaMemcpyAsync(s->seen + (size_t)slot * s->V, seen, s->V, cudaMemcpyHostToDevice, s->st));
    CK(cudaStreamSynchronize(s->st));
    return T2SX_OK;
}

extern "C" int t2sx_decode_graph_kernels(t2sx_session* s, int32_t* n) {
    if (!s || !n) return fail(T2SX_ERR_INVALID, "null argument");
    *n = s->graph ? s->graph_kernels : 0;
    return T2SX_OK;
}

// Average device time of one launch of each kernel class of the decode step, replayed on the
// state left by the last decode step (all replayed kernels are idempotent there).
extern "C" int t2sx_profile_step(t2sx_session* s, int32_t iters, float* ms) {
    if (!s || !ms || iters <= 0) return fail(T2SX_ERR_INVALID, "t2sx_profile_step: bad arguments");
    if (!s->graph) return fail(T2SX_ERR_STATE, "t2sx_profile_step: run a decode step first");
    DeviceGuard dg_;
    CK(dg_.set(s->m->device));
    ErrScope es_(s->err);   // bounded-wait failures of this call's kernels land here
    const t2sx_model* m = s->m;
    Work& w = s->dec;
    const int T = (int)s->active.size();
    Rows rows = rows_of(s, w);
    KVView kv = kv_of(s);
    ActQ a = act_of(w);
    const LayerD& L = m->layers[0];
    auto timeit = [&](int idx, auto&& fn) -> int {
        fn();
        CK(cudaEventRecord(s->ev0, s->st));
        for (int i = 0; i < iters; ++i) fn();
        CK(cudaEventRecord(s->ev1, s->st));
        CK(cudaEventSynchronize(s->ev1));
        float t = 0.0f;
        CK(cudaEventElapsedTime(&t, s->ev0, s->ev1));
        ms[idx] = t / iters;
        return T2SX_OK;
    };
    int rc;
    if ((rc = timeit(0, [&] { attention_decode(T, w.q16, rows, kv, 0, kAttnScale, w.attn, L.out.type, a, s->st); }))) return rc;
    quantize_act(L.qkv.type, w.x, T, kD, a, s->st);
    if ((rc = timeit(1, [&] { matmul(L.qkv, a, T, L.qkv_b, 0, w.qkv, s->st); }))) return rc;
    if ((rc = timeit(2, [&] { matmul(L.out, a, T, L.out_b, 0, w.o, s->st); }))) return rc;
    if ((rc = timeit(3, [&] { matmul(L.up, a, T, L.up_b, 1, w.h, s->st); }))) return rc;
    if ((rc = timeit(5, [&] { matmul(m->lm_head, a, T, nullptr, 0, w.logits, s->st); }))) return rc;
    quantize_act(L.down.type, w.h, T, s->ff, a, s->st);
    if ((rc = timeit(4, [&] { matmul(L.down, a, T, L.down_b, 0, w.f, s->st); }))) return rc;
    if ((rc = timeit(6, [&] { residual_layernorm(T, w.ln1, w.f, L.ln2_w, L.ln2_b, 1e-5f, w.o, -1, a, s->st); }))) return rc;
    if ((rc = timeit(7, [&] { quantize_act(L.down.type, w.h, T, s->ff, a, s->st); }))) return rc;
    // the attention kernel alone (f32 rows, no conversion for the out-projection)
    if ((rc = timeit(8, [&] { attention_decode(T, w.q16, rows, kv, 0, kAttnScale, w.attn, -1, a, s->st); }))) return rc;
    CK(cudaGetLastError());
    return T2SX_OK;
}

extern "C" int t2sx_set_exp_noise(t2sx_session* s, const float* noise, int32_t rows) {
    if (!s || rows < 0 || rows > s->n_slots) return fail(T2SX_ERR_INVALID, "t2sx_set_exp_noise: bad arguments");
    DeviceGuard dg_;
    CK(dg_.set(s->m->device));
    const bool on = noise != nullptr && rows > 0;
    if (on) {
        if (!s->noise) CK(cudaMalloc(&s->noise, (size_t)s->n_slots * s->V * 4));
        CK(cudaMemcpyAsync(s->noise, noise, (size_t)rows * s->V * 4, cudaMemcpyHostToDevice, s->st));
        CK(cudaStreamSynchronize(s->st));
    }
    if (on != s->noise_on) { s->noise_on = on; s->dec_dirty = true; }
    return T2SX_OK;
}

extern "C" int t2sx_read_greedy(t2sx_session* s, int32_t* out, int32_t max_rows, int32_t* rows) {
    if (!s || !out) return fail(T2SX_ERR_INVALID, "null argument");
    if (!s->last_greedy) return fail(T2SX_ERR_STATE, "no pass has run yet");
    DeviceGuard dg_;
    CK(dg_.set(s->m->device));
    CK(cudaStreamSynchronize(s->st));
    const int n = s->last_rows < max_rows ? s->last_rows : max_rows;
    CK(cudaMemcpy(out, s->last_greedy, (size_t)n * 4, cudaMemcpyDeviceToHost));
    if (rows) *rows = n;
    return T2SX_OK;
}

extern "C" int t2sx_last_decode_ms(t2sx_session* s, float* ms) {
    if (!s || !ms) return fail(T2SX_ERR_INVALID, "null argument");
    *ms = s->last_ms;
    return T2SX_OK;
}

// ============================================================================================
// isolated matmul
// ============================================================================================
struct t2sx_weight {
    int device = 0;
    char* mem = nullptr;
    DevW w;
    void* act = nullptr;
    int64_t act_rows = 0;
    int32_t* err = nullptr;   // device error word of the calls on this weight (see t2sx_weight_sync)
};

extern "C" int t2sx_weight_create(int32_t device, int32_t type, const void* host_bytes, int64_t N, int64_t K, t2sx_weight** out) {
    if (!host_bytes || !out || N <= 0 || K <= 0 || row_bytes(type, K) < 0) return fail(T2SX_ERR_INVALID, "t2sx_weight_create: bad arguments");
    if (type == W_Q4_K ? K % 256 : K % 32) return fail(T2SX_ERR_INVALID, "K not a multiple of the block size");
    // the few-row kernel keeps one row's 32-element block sums in shared memory (64 of them)
    if (K > 2048) return fail(T2SX_ERR_INVALID, "t2sx_weight_create: K above 2048 is not supported");
    DeviceGuard dg_;
    CK(dg_.set(device));
    Arena ar;
    WOff wo;
    if (!repack_weight(type, (const uint8_t*)host_bytes, N, K, ar, wo)) return fail(T2SX_ERR_FORMAT, "unsupported type %d", type);
    std::unique_ptr<t2sx_weight> w(new t2sx_weight());
    w->device = device;
    CK(cudaMalloc(&w->mem, ar.used));
    for (auto& s : ar.staged) {
        cudaError_t e = cudaMemcpy(w->mem + s.first, s.second.data(), s.second.size(), cudaMemcpyHostToDevice);
        if (e != cudaSuccess) { cudaFree(w->mem); return fail(T2SX_ERR_CUDA, "upload: %s", cudaGetErrorString(e)); }
    }
    w->w = resolve(wo, w->mem);
    if (cudaMalloc(&w->err, 4) != cudaSuccess || cudaMemset(w->err, 0, 4) != cudaSuccess) {
        cudaFree(w->mem);
        if (w->err) cudaFree(w->err);
        return fail(T2SX_ERR_OOM, "t2sx_weight_create: error word");
    }
    *out = w.release();
    return T2SX_OK;
}

int32_t t2sx_weight_device_of(const t2sx_weight* w) { return w->device; }
const DevW* t2sx_weight_devw_of(const t2sx_weight* w) { return &w->w; }
int t2sx_set_error(int code, const char* msg) { return fail(code, "%s", msg); }

extern "C" void t2sx_weight_free(t2sx_weight* w) {
    if (!w) return;
    DeviceGuard dg_;
    dg_.set(w->device);
    if (w->mem) cudaFree(w->mem);
    if (w->act) cudaFree(w->act);
    if (w->err) cudaFree(w->err);
    delete w;
}

int32_t* t2sx_weight_err_of(const t2sx_weight* w) { return w->err; }

extern "C" int t2sx_weight_sync(t2sx_weight* w, void* stream) {
    if (!w) return fail(T2SX_ERR_INVALID, "t2sx_weight_sync: null weight");
    DeviceGuard dg_;
    CK(dg_.set(w->device));
    CK(cudaStreamSynchronize((cudaStream_t)stream));
    int32_t e = 0;
    CK(cudaMemcpy(&e, w->err, 4, cudaMemcpyDeviceToHost));
    if (e) {
        CK(cudaMemset(w->err, 0, 4));
        return fail(T2SX_ERR_TIMEOUT, "a tensor-core matmul on this weight gave up waiting; its outputs are NaN");
    }
    return T2SX_OK;
}

extern "C" int t2sx_test_set_tc_wait_cycles(int64_t cycles) {
    if (cycles < 0) return fail(T2SX_ERR_INVALID, "t2sx_test_set_tc_wait_cycles: negative bound");
    set_tc_test_wait_cycles((long long)cycles);
    return T2SX_OK;
}

extern "C" int t2sx_matmul(t2sx_weight* w, const float* x, int64_t M, const float* bias, float* y, void* stream) {
    if (!w || !x || !y || M <= 0 || M > (1 << 24)) return fail(T2SX_ERR_INVALID, "t2sx_matmul: bad arguments");
    DeviceGuard dg_;
    CK(dg_.set(w->device));
    ErrScope es_(w->err);   // bounded-wait failures of this call's kernels land here
    cudaStream_t st = (cudaStream_t)stream;
    const int64_t K = w->w.K;
    if (w->act_rows < M) {
        if (w->act) { CK(cudaStreamSynchronize(st)); cudaFree(w->act); w->act = nullptr; }
        const size_t bytes = (size_t)M * K * 2 + 512 + (size_t)M * (K / 32) * 8 + 512;
        CK(cudaMalloc(&w->act, bytes));
        w->act_rows = M;
    }
    ActQ a;
    char* p = (char*)w->act;
    a.q = (int8_t*)p; a.h = (uint16_t*)p;
    p += ((size_t)M * K * 2 + 255) & ~(size_t)255;
    a.d = (float*)p;
    p += ((size_t)M * (K / 32) * 4 + 255) & ~(size_t)255;
    a.bs = (int32_t*)p;
    quantize_act(w->w.type, x, (int)M, (int)K, a, st);
    matmul(w->w, a, (int)M, bias, 0, y, st);
    CK(cudaGetLastError());
    return T2SX_OK;
}

// ============================================================================================
// extract-latent (t2s_session_compute_ref_emb's code extraction, session.cpp:881-1044;
// sovits_extract_latent_block_forward, block.cpp:140-189)
// ============================================================================================
extern "C" int t2sx_extract_latent(t2sx_session* s, const float* hubert, int32_t T, int32_t* codes_out) {
    if (!s || !hubert || !codes_out || T < 2 || T > (1 << 20)) return fail(T2SX_ERR_INVALID, "t2sx_extract_latent: bad arguments");
    const t2sx_model* m = s->m;
    DeviceGuard dg_;
    CK(dg_.set(m->device));
    ErrScope es_(s->err);   // bounded-wait failures of this call's kernels land here
    const int C = 768, K = 2 * C, NC = m->n_codes;
    const int To = (T - 2) / 2 + 1;
    // one scratch allocation: frames, im2col rows, their dot-type copy, conv output, scores, codes
    auto al = [](size_t n) { return (n + 255) & ~(size_t)255; };
    const size_t bx = al((size_t)T * C * 4), bc = al((size_t)To * K * 4), bq = al((size_t)To * K * 2) + al((size_t)To * (K / 32) * 8),
                 bs = al((size_t)To * C * 4), bsc = al((size_t)To * NC * 4), bk = al((size_t)To * 4);
    char* mem = nullptr;
    CK(cudaMalloc(&mem, bx + bc + bq + bs + bsc + bk));
    float* x = (float*)mem;
    float* cols = (float*)(mem + bx);
    char* qbuf = mem + bx + bc;
    float* ssl = (float*)(mem + bx + bc + bq);
    float* score = (float*)(mem + bx + bc + bq + bs);
    int32_t* codes = (int32_t*)(mem + bx + bc + bq + bs + bsc);
    ActQ a;
    a.q = (int8_t*)qbuf;
    a.h = (uint16_t*)qbuf;
    a.d = (float*)(qbuf + al((size_t)To * K * 2));
    a.bs = (int32_t*)(qbuf + al((size_t)To * K * 2) + al((size_t)To * (K / 32) * 4));
    a.f = cols;
    cudaError_t e = cudaMemcpyAsync(x, hubert, (size_t)T * C * 4, cudaMemcpyHostToDevice, s->st);
    if (e == cudaSuccess) {
        im2col_k2s2(To, C, x, cols, s->st);
        if (m->ssl_w.type != W_F32) quantize_act(m->ssl_w.type, cols, To, K, a, s->st);
        matmul(m->ssl_w, a, To, m->ssl_b, 0, ssl, s->st);
        ActQ af;
        af.f = ssl;   // the codebook is f32: the conv output is read as it is
        matmul(m->codebook, af, To, nullptr, 0, score, s->st);
        code_argmax(To, NC, score, m->code_half_norm, codes, s->st);
        e = cudaGetLastError();
        if (e == cudaSuccess) e = cudaMemcpyAsync(codes_out, codes, (size_t)To * 4, cudaMemcpyDeviceToHost, s->st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s->st);
    }
    cudaFree(mem);
    if (e != cudaSuccess) return fail(T2SX_ERR_CUDA, "t2sx_extract_latent: %s", cudaGetErrorString(e));
    return T2SX_OK;
}
