// CUDA kernels of the T2S decode path for sm_100a.
//
// Arithmetic follows the reference's ggml CPU operators (src/t2s/block.cpp:513-637 layer,
// :117-348 sampler, src/t2s/session.cpp:337-344 decode embedding) with one fixed evaluation
// order per reduction; see t2sx_math.cuh.  Built with --fmad=false.
#include "t2sx_kernels.cuh"
#include "t2sx_math.cuh"
#include "t2sx_kv.cuh"

#include <atomic>
#include <cstdlib>

namespace t2sx {

// Off unless T2SX_PDL=1 or inside a PdlScope: measured on B200 inside the step graph it slowed
// the 32-row step (early-resident dependents hold SM slots).
static thread_local bool t_pdl_scope = false;

bool pdl_enabled() {
    static const bool on = [] {
        const char* e = getenv("T2SX_PDL");
        return e && e[0] == '1';
    }();
    return on || t_pdl_scope;
}

PdlScope::PdlScope(bool on) : prev(t_pdl_scope) { t_pdl_scope = prev || on; }
PdlScope::~PdlScope() { t_pdl_scope = prev; }

static thread_local int32_t* t_err_word = nullptr;
int32_t* current_err_word() { return t_err_word; }
ErrScope::ErrScope(int32_t* word) : prev(t_err_word) { t_err_word = word; }
ErrScope::~ErrScope() { t_err_word = prev; }

static std::atomic<long long> g_tc_test_wait{0};
long long tc_test_wait_cycles() { return g_tc_test_wait.load(std::memory_order_relaxed); }
void set_tc_test_wait_cycles(long long cycles) { g_tc_test_wait.store(cycles > 0 ? cycles : 0, std::memory_order_relaxed); }

// ============================================================================================
// activation quantisation
// ============================================================================================

// Q8_0 (x86 AVX2 rule of ggml quantize_row_q8_0): one warp per 32-element block.
__global__ void k_quant_q8_0(const float* __restrict__ x, int64_t nblk, int8_t* __restrict__ q,
                             float* __restrict__ d) {
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int64_t wstride = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t b = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; b < nblk; b += wstride)
        q[b * 32 + lane] = (int8_t)q8_0_lane(x[b * 32 + lane], d + b, lane);
}

// Q8_K of one 256-element block by one warp, 8 consecutive elements per lane: q, d and the sums
// of the eight 32-element groups.  `ldcg` reads through L2 (data written by other CTAs).
__device__ __forceinline__ void quant_block_q8_K(const float* __restrict__ xb, int lane, bool ldcg,
                                                 int8_t* __restrict__ qb, float* __restrict__ d_slot,
                                                 int32_t* __restrict__ bs8) {
    const float4* p = reinterpret_cast<const float4*>(xb + lane * 8);
    const float4 x0 = ldcg ? __ldcg(p) : p[0];
    const float4 x1 = ldcg ? __ldcg(p + 1) : p[1];
    const float v[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
    AbsMax am{0.0f, 0.0f, 0x7fffffff};
#pragma unroll
    for (int i = 0; i < 8; ++i) absmax_take(am, v[i], lane * 8 + i);
    am = absmax_warp(am);
    const float iscale = q8k_iscale(am);
    int qv[8];
    int sum = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) { qv[i] = q8k_q(iscale, v[i]); sum += qv[i]; }
    if (lane == 0) *d_slot = q8k_d(iscale);
    int2 packed;
    packed.x = (qv[0] & 0xff) | ((qv[1] & 0xff) << 8) | ((qv[2] & 0xff) << 16) | ((qv[3] & 0xff) << 24);
    packed.y = (qv[4] & 0xff) | ((qv[5] & 0xff) << 8) | ((qv[6] & 0xff) << 16) | ((qv[7] & 0xff) << 24);
    *reinterpret_cast<int2*>(qb + lane * 8) = packed;
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    if ((lane & 3) == 0) bs8[lane >> 2] = sum;
}

// Q8_K (ggml quantize_row_q8_K_ref rule): one warp per 256-element block.
__global__ void k_quant_q8_K(const float* __restrict__ x, int64_t nblk, int8_t* __restrict__ q,
                             float* __restrict__ d, int32_t* __restrict__ bs) {
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int64_t wstride = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t b = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; b < nblk; b += wstride)
        quant_block_q8_K(x + b * 256, lane, false, q + b * 256, d + b, bs + b * 8);
}

// A 512-wide row held by one warp, lane l holding elements l + 32 t (t < 16), converted to the
// dot type of a weight format with the same rules as the k_quant_* kernels.  wtype < 0 or F32:
// nothing to write (an F32 matmul reads the f32 row itself).
__device__ void quant_row512_strided(const float (&y)[kD / 32], int lane, int wtype, const ActQ& o, size_t row) {
    // The blocks' warp reductions run side by side (a max, a first-index |x| max and integer sums
    // do not depend on the merge order), so their shuffles overlap instead of running block by block.
    if (wtype == W_Q8_0 || wtype == W_Q4_0) {
        // The 16 block maxima as a reduce-scatter (fmaxf is exact, so any order gives the same
        // maximum): at the rounds with partners 16, 8, 4, 2 a lane keeps the half of its blocks
        // selected by that lane bit, so lane l ends with block l >> 1, completed by partner 1.
        // Lane l then forms that block's scale and inverse (the rule of q8_0_lane, x86 AVX2
        // quantize_row_q8_0: d = amax/127 as f16, q = rint(v * 127/amax)); block t's inverse
        // comes from lane 2t.
        float a16[16], a8[8], a4[4], a2[2];
#pragma unroll
        for (int t = 0; t < 16; ++t) a16[t] = fabsf(y[t]);
        auto half_round = [&](auto& in, auto& out, int off, int n) {
            const bool hi = (lane & off) != 0;
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                if (u < n) {
                    const float keep = hi ? in[n + u] : in[u];
                    const float send = hi ? in[u] : in[n + u];
                    out[u] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, off));
                }
            }
        };
        half_round(a16, a8, 16, 8);
        half_round(a8, a4, 8, 4);
        half_round(a4, a2, 4, 2);
        float a1;
        {
            const bool hi = (lane & 2) != 0;
            const float keep = hi ? a2[1] : a2[0];
            const float send = hi ? a2[0] : a2[1];
            a1 = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, 2));
        }
        a1 = fmaxf(a1, __shfl_xor_sync(0xffffffffu, a1, 1));
        const float dd = __fdiv_rn(a1, 127.0f);
        const float id = (a1 != 0.0f) ? __fdiv_rn(127.0f, a1) : 0.0f;
#pragma unroll
        for (int t = 0; t < kD / 32; ++t) {
            const float idt = __shfl_sync(0xffffffffu, id, 2 * t);
            float r = rintf(__fmul_rn(y[t], idt));
            r = fminf(fmaxf(r, -128.0f), 127.0f);
            o.q[row * kD + 32 * t + lane] = (int8_t)(int)r;
        }
        if ((lane & 1) == 0) o.d[row * (kD / 32) + (lane >> 1)] = __half2float(__float2half_rn(dd));
    } else if (wtype == W_Q4_K) {
        constexpr int NB = kD / 256;
        AbsMax am[NB];
#pragma unroll
        for (int B = 0; B < NB; ++B) {
            am[B] = AbsMax{0.0f, 0.0f, 0x7fffffff};
#pragma unroll
            for (int k = 0; k < 8; ++k) absmax_take(am[B], y[8 * B + k], lane + 32 * k);
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1)
#pragma unroll
            for (int B = 0; B < NB; ++B) {
                AbsMax w;
                w.a = __shfl_xor_sync(0xffffffffu, am[B].a, off);
                w.m = __shfl_xor_sync(0xffffffffu, am[B].m, off);
                w.i = __shfl_xor_sync(0xffffffffu, am[B].i, off);
                absmax_merge(am[B], w);
            }
        int qv[kD / 32];
#pragma unroll
        for (int B = 0; B < NB; ++B) {
            const float iscale = q8k_iscale(am[B]);
            if (lane == 0) o.d[row * NB + B] = q8k_d(iscale);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                qv[8 * B + k] = q8k_q(iscale, y[8 * B + k]);
                o.q[row * kD + 256 * B + 32 * k + lane] = (int8_t)qv[8 * B + k];
            }
        }
        int sum[kD / 32];
#pragma unroll
        for (int t = 0; t < kD / 32; ++t) sum[t] = qv[t];
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1)
#pragma unroll
            for (int t = 0; t < kD / 32; ++t) sum[t] += __shfl_xor_sync(0xffffffffu, sum[t], off);
        if (lane == 0) {
#pragma unroll
            for (int t = 0; t < kD / 32; ++t) o.bs[row * (kD / 32) + t] = sum[t];
        }
    } else if (wtype == W_F16) {
#pragma unroll
        for (int t = 0; t < kD / 32; ++t) o.h[row * kD + 32 * t + lane] = f2h(y[t]);
    }
}

__global__ void k_quant_f16(const float* __restrict__ x, int64_t n, uint16_t* __restrict__ h) {
    pdl_wait();
    pdl_trigger();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        h[i] = f2h(x[i]);
}

static int grid_for(int64_t work, int per_block) {
    int64_t g = (work + per_block - 1) / per_block;
    if (g > 148 * 32) g = 148 * 32;
    if (g < 1) g = 1;
    return (int)g;
}

void quantize_act(int wtype, const float* x, int M, int K, ActQ& a, cudaStream_t st) {
    const int64_t n = (int64_t)M * K;
    if (wtype == W_Q8_0 || wtype == W_Q4_0) {
        launch_k(k_quant_q8_0, dim3(grid_for(n / 32, 8)), dim3(256), 0, st, x, n / 32, a.q, a.d);
    } else if (wtype == W_Q4_K) {
        launch_k(k_quant_q8_K, dim3(grid_for(n / 256, 8)), dim3(256), 0, st, x, n / 256, a.q, a.d, a.bs);
    } else if (wtype == W_F16) {
        launch_k(k_quant_f16, dim3(grid_for(n, 256)), dim3(256), 0, st, x, n, a.h);
    } else {
        a.f = x;
    }
}

// ============================================================================================
// matmul  y[m][n] = bias[n] + sum_k W[n][k] x[m][k]  in the canonical block order:
//   Q8_0/Q4_0: acc = fma(dw_b*dx_b, (float)isum_b, acc) for b = 0.. (acc starts at +0)
//   Q4_K     : per super-block, acc_a = fma(dx*dw, sumi_a, acc_a), acc_m = fma(-dx*dmin, sumi_m, acc_m);
//              result acc_a + acc_m
//   F16/F32  : per 32-block a sequential fma chain from 0; block sums added in order
// ============================================================================================

__device__ __forceinline__ int dp8(const int4& w0, const int4& w1, const int4& x0, const int4& x1) {
    int s = 0;
    s = __dp4a(w0.x, x0.x, s); s = __dp4a(w0.y, x0.y, s); s = __dp4a(w0.z, x0.z, s); s = __dp4a(w0.w, x0.w, s);
    s = __dp4a(w1.x, x1.x, s); s = __dp4a(w1.y, x1.y, s); s = __dp4a(w1.z, x1.z, s); s = __dp4a(w1.w, x1.w, s);
    return s;
}

__device__ __forceinline__ int q4lo(int w) { return __vsub4(w & 0x0F0F0F0F, 0x08080808); }
__device__ __forceinline__ int q4hi(int w) { return __vsub4((w >> 4) & 0x0F0F0F0F, 0x08080808); }

__device__ __forceinline__ float epi(float acc, const float* bias, int n, int relu) {
    float v = bias ? __fadd_rn(acc, bias[n]) : acc;
    if (relu) v = (v > 0.0f) ? v : 0.0f;
    return v;
}

constexpr int kSmallM = 32;

// y = LN(a + b) * g + beta for one row held by one warp (ggml_norm + mul + add,
// block.cpp:615-619 / :630-634): lane l sums elements l, l+32, ... in double, the lanes combine
// by an xor butterfly.  This form takes the lane's elements of a, g and beta already loaded (av,
// gv, bv: element lane + 32 t at t); `b_l2` reads b through L2 (written by other CTAs of the same
// kernel).
__device__ void ln_row_vals(const float (&av)[kD / 32], const float* __restrict__ b, bool b_l2,
                            const float (&gv)[kD / 32], const float (&bv)[kD / 32], float eps, int lane,
                            float (&out)[kD / 32]) {
    float v[kD / 32];
    double s = 0.0;
#pragma unroll
    for (int t = 0; t < kD / 32; ++t) {
        const int i = lane + 32 * t;
        v[t] = __fadd_rn(av[t], b_l2 ? __ldcg(b + i) : b[i]);
        s = __dadd_rn(s, (double)v[t]);
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) s = __dadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
    // kD is a power of two: s * (1/kD) is the same correctly rounded value as s / kD
    static_assert((kD & (kD - 1)) == 0, "kD must be a power of two");
    const float mean = __double2float_rn(__dmul_rn(s, 1.0 / kD));
    double s2 = 0.0;
#pragma unroll
    for (int t = 0; t < kD / 32; ++t) {
        v[t] = __fsub_rn(v[t], mean);
        s2 = __dadd_rn(s2, (double)__fmul_rn(v[t], v[t]));
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) s2 = __dadd_rn(s2, __shfl_xor_sync(0xffffffffu, s2, off));
    const float var = __double2float_rn(__dmul_rn(s2, 1.0 / kD));
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
#pragma unroll
    for (int t = 0; t < kD / 32; ++t) out[t] = __fadd_rn(__fmul_rn(__fmul_rn(v[t], scale), gv[t]), bv[t]);
}

// The lane's elements of a 512-wide row.
__device__ __forceinline__ void load_row_lane(const float* __restrict__ x, int lane, float (&v)[kD / 32]) {
#pragma unroll
    for (int t = 0; t < kD / 32; ++t) v[t] = x[lane + 32 * t];
}

// ln_row_vals with a, g and beta loaded here, with the row: one round trip, not one after the sums.
__device__ void ln_row_warp(const float* __restrict__ a, const float* __restrict__ b, bool b_l2,
                            const float* __restrict__ g, const float* __restrict__ beta, float eps, int lane,
                            float (&out)[kD / 32]) {
    float av[kD / 32], gv[kD / 32], bv[kD / 32];
    load_row_lane(g, lane, gv);
    load_row_lane(beta, lane, bv);
    load_row_lane(a, lane, av);
    ln_row_vals(av, b, b_l2, gv, bv, eps, lane, out);
}

// Work of the last CTA of a small-M matmul, once every CTA's output is written: residual +
// LayerNorm of the M rows (kind 1) or quantisation of the M output rows (kind 2), into the
// next matmul's dot type.
__device__ void run_tail(const Tail& tl, const float* __restrict__ y, int M, int N) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if (tl.kind == 1) {
        for (int m = warp; m < M; m += nw) {
            float out[kD / 32];
            ln_row_warp(tl.resid + (size_t)m * kD, y + (size_t)m * kD, true, tl.g, tl.beta, tl.eps, lane, out);
#pragma unroll
            for (int t = 0; t < kD / 32; ++t) tl.y_out[(size_t)m * kD + lane + 32 * t] = out[t];
            quant_row512_strided(out, lane, tl.qtype, tl.qo, (size_t)m);
        }
    } else if (tl.kind == 2) {
        if (tl.qtype == W_Q8_0 || tl.qtype == W_Q4_0) {
            const int nb = M * (N / 32);
            for (int b = warp; b < nb; b += nw)
                tl.qo.q[(size_t)b * 32 + lane] = (int8_t)q8_0_lane(__ldcg(y + (size_t)b * 32 + lane), tl.qo.d + b, lane);
        } else if (tl.qtype == W_Q4_K) {
            const int nb = M * (N / 256);
            for (int b = warp; b < nb; b += nw)
                quant_block_q8_K(y + (size_t)b * 256, lane, true, tl.qo.q + (size_t)b * 256, tl.qo.d + b,
                                 tl.qo.bs + (size_t)b * 8);
        } else if (tl.qtype == W_F16) {
            for (int i = threadIdx.x; i < M * N; i += blockDim.x) tl.qo.h[i] = f2h(__ldcg(y + i));
        }
    }
}

// Last-CTA election (threadfence + ticket): no CTA waits for another.  The last CTA runs the
// tail and resets the ticket for the next launch.
__device__ __forceinline__ void tail_if_last(const Tail& tl, const float* y, int M, int N) {
    __shared__ int s_last;
    __threadfence();   // this thread's outputs are visible device-wide before the ticket
    __syncthreads();
    if (threadIdx.x == 0) s_last = (atomicAdd(tl.counter, 1) == (int)gridDim.x - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    run_tail(tl, y, M, N);
    if (threadIdx.x == 0) *tl.counter = 0;
}

// Small-M kernel: one warp per weight row; lanes compute block partials (phase A) into shared
// memory, then lane m runs the ordered chain of row m (phase B).  Optional epilogues: QKV store
// (Q and the K/V cache append) and a last-CTA tail.
// Latency: the launch is a chain of memory round trips, so every load that does not depend on a
// dot product is issued with the weights: the bias, the K/V destination's position and slot,
// and (up to kDDM rows) the block scales, whose products phase A stages in shared memory so
// that phase B's chain reads no global memory.  The arithmetic and its order are unchanged.
constexpr int kDDM = 8;

__device__ __forceinline__ float epi_v(float acc, bool has_bias, float bv, int relu) {
    float v = has_bias ? __fadd_rn(acc, bv) : acc;
    if (relu) v = (v > 0.0f) ? v : 0.0f;
    return v;
}

template <int WT>
__device__ __forceinline__ void mm_small_row(const DevW& W, const ActQ& A, int M, const float* __restrict__ bias, int relu,
                                             float* __restrict__ y, const QKVStore* qkv, int (&s_a)[kSmallM][64],
                                             int (&s_m)[kSmallM][8], float (&s_dd)[kDDM][64], int n, int lane,
                                             bool fq = false) {
    const int K = W.K;
    const bool own = lane < M;
    const float bv = (bias && own) ? bias[n] : 0.0f;
    const bool kvcol = qkv && own && n >= kD;
    int kpos = 0, kslot = 0;
    // Loads before this point read constants (weights, bias); with a programmatic launch they
    // overlap the preceding kernel.  Every branch calls it once, before reading activations.
    auto after_wait = [&]() {
        pdl_wait();
        pdl_trigger();
        if (kvcol) { kpos = qkv->rows.pos[lane]; kslot = qkv->rows.slot[lane]; }
    };
    const bool stage_dd = M <= kDDM;
    auto finish = [&](float acc) {
        const float v_ = epi_v(acc, bias != nullptr, bv, relu);
        if (qkv) qkv_store_at(*qkv, lane, n, v_, kvcol ? qkv_dest(*qkv, kpos, kslot) : make_int2(-1, 0));
        else y[(size_t)lane * W.N + n] = v_;
    };
    if ((WT == W_Q8_0 || WT == W_Q4_0) && fq && M == 1) {
        // one row quantised here (K <= 2048: at most two blocks per lane), both blocks' weights
        // and activations fetched before any arithmetic
        const int nb = K / 32;
        int4 wq[2][2];
        float wd[2];
        float4 xv[2][8];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int b = lane + 32 * u;
            if (b < nb) {
                if (WT == W_Q8_0) {
                    const int4* wp = reinterpret_cast<const int4*>(W.q8 + (size_t)n * K + b * 32);
                    wq[u][0] = wp[0]; wq[u][1] = wp[1];
                } else {
                    wq[u][0] = *reinterpret_cast<const int4*>(W.q4 + ((size_t)n * nb + b) * 16);
                }
                wd[u] = W.d[(size_t)n * nb + b];
            }
        }
        after_wait();
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int b = lane + 32 * u;
            if (b < nb) {
                const float4* xp = reinterpret_cast<const float4*>(A.f + b * 32);
#pragma unroll
                for (int i = 0; i < 8; ++i) xv[u][i] = xp[i];
            }
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int b = lane + 32 * u;
            if (b < nb) {
                int4 w0 = wq[u][0], w1 = wq[u][1];
                if (WT == W_Q4_0) {
                    const int4 raw = wq[u][0];
                    w0 = make_int4(q4lo(raw.x), q4lo(raw.y), q4lo(raw.z), q4lo(raw.w));
                    w1 = make_int4(q4hi(raw.x), q4hi(raw.y), q4hi(raw.z), q4hi(raw.w));
                }
                int4 x0, x1;
                float ad;
                q8_0_block_regs(xv[u], x0, x1, ad);
                s_a[0][b] = dp8(w0, w1, x0, x1);
                s_dd[0][b] = __fmul_rn(wd[u], ad);
            }
        }
        __syncwarp();
        if (own) {
            float acc = 0.0f;
            for (int b = 0; b < nb; ++b) acc = __fmaf_rn(s_dd[0][b], (float)s_a[0][b], acc);
            finish(acc);
        }
    } else if (WT == W_Q8_0 || WT == W_Q4_0) {
        const int nb = K / 32;
        // the lane's first block of weights ahead of the wait
        int4 p0 = make_int4(0, 0, 0, 0), p1 = p0;
        float pd = 0.0f;
        if (lane < nb) {
            if (WT == W_Q8_0) {
                const int4* wp = reinterpret_cast<const int4*>(W.q8 + (size_t)n * K + lane * 32);
                p0 = wp[0]; p1 = wp[1];
            } else {
                p0 = *reinterpret_cast<const int4*>(W.q4 + ((size_t)n * nb + lane) * 16);
            }
            pd = W.d[(size_t)n * nb + lane];
        }
        after_wait();
        for (int b = lane; b < nb; b += 32) {
            int4 w0, w1;
            if (WT == W_Q8_0) {
                if (b == lane) { w0 = p0; w1 = p1; }
                else {
                    const int4* wp = reinterpret_cast<const int4*>(W.q8 + (size_t)n * K + b * 32);
                    w0 = wp[0]; w1 = wp[1];
                }
            } else {
                const int4 raw = b == lane ? p0 : *reinterpret_cast<const int4*>(W.q4 + ((size_t)n * nb + b) * 16);
                w0 = make_int4(q4lo(raw.x), q4lo(raw.y), q4lo(raw.z), q4lo(raw.w));
                w1 = make_int4(q4hi(raw.x), q4hi(raw.y), q4hi(raw.z), q4hi(raw.w));
            }
            const float wd = b == lane ? pd : W.d[(size_t)n * nb + b];
            for (int m = 0; m < M; ++m) {
                int4 x0, x1;
                float ad;
                if (fq) {   // the f32 rows quantised to Q8_0 here (then stage_dd holds)
                    q8_0_block_thread(A.f + (size_t)m * K + b * 32, x0, x1, ad);
                } else {
                    const int4* xp = reinterpret_cast<const int4*>(A.q + (size_t)m * K + b * 32);
                    x0 = xp[0]; x1 = xp[1];
                    ad = stage_dd ? A.d[(size_t)m * nb + b] : 0.0f;
                }
                s_a[m][b] = dp8(w0, w1, x0, x1);
                if (stage_dd) s_dd[m][b] = __fmul_rn(wd, ad);
            }
        }
        __syncwarp();
        if (own) {
            const int m = lane;
            float acc = 0.0f;
            if (stage_dd) {
                for (int b = 0; b < nb; ++b) acc = __fmaf_rn(s_dd[m][b], (float)s_a[m][b], acc);
            } else {
                for (int b = 0; b < nb; ++b) {
                    const float dd = __fmul_rn(W.d[(size_t)n * nb + b], A.d[(size_t)m * nb + b]);
                    acc = __fmaf_rn(dd, (float)s_a[m][b], acc);
                }
            }
            finish(acc);
        }
    } else if (WT == W_Q4_K) {
        after_wait();
        const int nsub = K / 32, nsb = K / 256;
        for (int t = 0; t < (nsub + 31) / 32; ++t) {
            const int j = lane + 32 * t;
            const bool act = j < nsub;
            const int sb = j >> 3, js = j & 7, c = js >> 1, hi = js & 1;
            int4 w0 = make_int4(0, 0, 0, 0), w1 = w0;
            int sc = 0, mn = 0;
            float wd = 0.0f, wdm = 0.0f;
            if (act) {
                const int4* wp = reinterpret_cast<const int4*>(W.q4 + ((size_t)n * nsb + sb) * 128 + 32 * c);
                const int4 r0 = wp[0], r1 = wp[1];
                if (hi) {
                    w0 = make_int4((r0.x >> 4) & 0x0F0F0F0F, (r0.y >> 4) & 0x0F0F0F0F, (r0.z >> 4) & 0x0F0F0F0F, (r0.w >> 4) & 0x0F0F0F0F);
                    w1 = make_int4((r1.x >> 4) & 0x0F0F0F0F, (r1.y >> 4) & 0x0F0F0F0F, (r1.z >> 4) & 0x0F0F0F0F, (r1.w >> 4) & 0x0F0F0F0F);
                } else {
                    w0 = make_int4(r0.x & 0x0F0F0F0F, r0.y & 0x0F0F0F0F, r0.z & 0x0F0F0F0F, r0.w & 0x0F0F0F0F);
                    w1 = make_int4(r1.x & 0x0F0F0F0F, r1.y & 0x0F0F0F0F, r1.z & 0x0F0F0F0F, r1.w & 0x0F0F0F0F);
                }
                const uint8_t* scm = W.scm + ((size_t)n * nsb + sb) * 16;
                sc = scm[js];
                mn = scm[8 + js];
                if (js == 0 && stage_dd) {
                    wd = W.d[(size_t)n * nsb + sb];
                    wdm = W.dmin[(size_t)n * nsb + sb];
                }
            }
            for (int m = 0; m < M; ++m) {
                int sa = 0, sm = 0;
                const float dx = (act && js == 0 && stage_dd) ? A.d[(size_t)m * nsb + sb] : 0.0f;
                if (act) {
                    const int4* xp = reinterpret_cast<const int4*>(A.q + (size_t)m * K + j * 32);
                    sa = sc * dp8(w0, w1, xp[0], xp[1]);
                    sm = mn * A.bs[(size_t)m * nsub + j];
                }
                sa += __shfl_xor_sync(0xffffffffu, sa, 1);
                sa += __shfl_xor_sync(0xffffffffu, sa, 2);
                sa += __shfl_xor_sync(0xffffffffu, sa, 4);
                sm += __shfl_xor_sync(0xffffffffu, sm, 1);
                sm += __shfl_xor_sync(0xffffffffu, sm, 2);
                sm += __shfl_xor_sync(0xffffffffu, sm, 4);
                if (act && js == 0) {
                    s_a[m][sb] = sa;
                    s_m[m][sb] = sm;
                    if (stage_dd) {
                        s_dd[m][sb] = __fmul_rn(dx, wd);
                        s_dd[m][8 + sb] = __fmul_rn(-dx, wdm);
                    }
                }
            }
        }
        __syncwarp();
        if (own) {
            const int m = lane;
            float acc_a = 0.0f, acc_m = 0.0f;
            for (int sb = 0; sb < nsb; ++sb) {
                float dd, dm;
                if (stage_dd) {
                    dd = s_dd[m][sb];
                    dm = s_dd[m][8 + sb];
                } else {
                    const float dx = A.d[(size_t)m * nsb + sb];
                    dd = __fmul_rn(dx, W.d[(size_t)n * nsb + sb]);
                    dm = __fmul_rn(-dx, W.dmin[(size_t)n * nsb + sb]);
                }
                acc_a = __fmaf_rn(dd, (float)s_a[m][sb], acc_a);
                acc_m = __fmaf_rn(dm, (float)s_m[m][sb], acc_m);
            }
            finish(__fadd_rn(acc_a, acc_m));
        }
    } else {  // F16 / F32
        after_wait();
        const int nb = K / 32;
        for (int b = lane; b < nb; b += 32) {
            float w[32];
            if (WT == W_F16) {
#pragma unroll
                for (int i = 0; i < 32; ++i) w[i] = h2f(W.h[(size_t)n * K + b * 32 + i]);
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) w[i] = W.f[(size_t)n * K + b * 32 + i];
            }
            for (int m = 0; m < M; ++m) {
                float s = 0.0f;
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const float xv = (WT == W_F16) ? h2f(A.h[(size_t)m * K + b * 32 + i]) : A.f[(size_t)m * K + b * 32 + i];
                    s = __fmaf_rn(w[i], xv, s);
                }
                s_a[m][b] = __float_as_int(s);
            }
        }
        __syncwarp();
        if (own) {
            const int m = lane;
            float acc = 0.0f;
            for (int b = 0; b < nb; ++b) acc = __fadd_rn(acc, __int_as_float(s_a[m][b]));
            finish(acc);
        }
    }
}


template <int WT>
__global__ void __launch_bounds__(128) k_mm_small(DevW W, ActQ A, int M, const float* __restrict__ bias, int relu,
                                                  float* __restrict__ y, QKVStore qkv, int use_qkv, Tail tail,
                                                  int use_tail, int fq) {
    __shared__ int s_a[4][kSmallM][64];
    __shared__ int s_m[4][kSmallM][8];
    __shared__ float s_dd[4][kDDM][64];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = blockIdx.x * 4 + warp;
    if (n < W.N) {
        if ((WT == W_Q8_0 || WT == W_Q4_0) && fq)
            mm_small_row<WT>(W, A, M, bias, relu, y, use_qkv ? &qkv : nullptr, s_a[warp], s_m[warp], s_dd[warp], n, lane, true);
        else
            mm_small_row<WT>(W, A, M, bias, relu, y, use_qkv ? &qkv : nullptr, s_a[warp], s_m[warp], s_dd[warp], n, lane);
    } else {   // (a row's warp waits inside mm_small_row)
        pdl_wait();
        pdl_trigger();
    }
    if (use_tail) tail_if_last(tail, y, M, W.N);
}

// Few-row matmul whose input is a residual + LayerNorm (ggml_norm + mul + add, block.cpp:615-619 /
// :630-634) of the preceding matmul's output: the norm runs at the start of every CTA instead of
// in the last CTA of the preceding matmul.  One warp per row normalises (ln_row_warp) and converts
// it to Q8_0 in shared memory (quant_row512_strided) while the CTA's weight loads are in flight;
// CTA 0 also stores the normalised rows (the next residual).  No ticket, no fence, and one round
// trip less than the tail.  Q8_0/Q4_0 weights, K = 512, at most 2 rows; the block sums and their
// ordered fold are those of mm_small_row.
template <int WT>
__global__ void __launch_bounds__(128) k_mm_ln(DevW W, LnIn ln, int M, const float* __restrict__ bias, int relu,
                                               float* __restrict__ y, QKVStore qkv, int use_qkv) {
    constexpr int nb = kD / 32;
    __shared__ __align__(16) int8_t s_xq[kLnRows * kD];
    __shared__ float s_xd[kLnRows * nb];
    __shared__ int s_a[4][kLnRows][nb];
    __shared__ float s_dd[4][kLnRows][nb];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = blockIdx.x * 4 + warp;
    const bool row = n < W.N;
    // this warp's weight row (block `lane`) and the epilogue's loads, issued before the norm
    int4 w0 = make_int4(0, 0, 0, 0), w1 = w0;
    float wd = 0.0f;
    if (row && lane < nb) {
        if (WT == W_Q8_0) {
            const int4* wp = reinterpret_cast<const int4*>(W.q8 + (size_t)n * kD + lane * 32);
            w0 = wp[0]; w1 = wp[1];
        } else {
            const int4 raw = *reinterpret_cast<const int4*>(W.q4 + ((size_t)n * nb + lane) * 16);
            w0 = make_int4(q4lo(raw.x), q4lo(raw.y), q4lo(raw.z), q4lo(raw.w));
            w1 = make_int4(q4hi(raw.x), q4hi(raw.y), q4hi(raw.z), q4hi(raw.w));
        }
        wd = W.d[(size_t)n * nb + lane];
    }
    const bool own = row && lane < M;
    const float bv = (bias && own) ? bias[n] : 0.0f;
    // the norm's g, beta and residual row a (written two or more launches back), and the K/V
    // cache slot of row `lane` (QKV projection above layer 0: rows placed two or more launches back)
    float ag[kD / 32], gg[kD / 32], bg[kD / 32];
    if (warp < M) {
        load_row_lane(ln.g, lane, gg);
        load_row_lane(ln.beta, lane, bg);
        load_row_lane(ln.a + (size_t)warp * kD, lane, ag);
    }
    const bool kvcol = use_qkv && own && n >= kD;
    const bool early_dst = kvcol && qkv.layer > 0;
    int2 kdst = make_int2(-1, 0);
    if (early_dst) kdst = qkv_dest(qkv, qkv.rows.pos[lane], qkv.rows.slot[lane]);
    // weights, bias and those are in flight while the preceding matmul finishes (programmatic
    // launch); below, the preceding kernel's output
    pdl_wait();
    pdl_trigger();
    if (kvcol && !early_dst) kdst = qkv_dest(qkv, qkv.rows.pos[lane], qkv.rows.slot[lane]);
    if (warp < M) {
        float o[kD / 32];
        ln_row_vals(ag, ln.b + (size_t)warp * kD, true, gg, bg, ln.eps, lane, o);
        if (blockIdx.x == 0) {
#pragma unroll
            for (int t = 0; t < kD / 32; ++t) ln.y_out[(size_t)warp * kD + lane + 32 * t] = o[t];
        }
        ActQ sq;
        sq.q = s_xq;
        sq.d = s_xd;
        quant_row512_strided(o, lane, W_Q8_0, sq, (size_t)warp);
    }
    __syncthreads();
    if (!row) return;
    if (lane < nb) {
        for (int m = 0; m < M; ++m) {
            const int4* xp = reinterpret_cast<const int4*>(s_xq + m * kD + lane * 32);
            s_a[warp][m][lane] = dp8(w0, w1, xp[0], xp[1]);
            s_dd[warp][m][lane] = __fmul_rn(wd, s_xd[m * nb + lane]);
        }
    }
    __syncwarp();
    if (own) {
        const int m = lane;
        float acc = 0.0f;
#pragma unroll
        for (int b = 0; b < nb; ++b) acc = __fmaf_rn(s_dd[warp][m][b], (float)s_a[warp][m][b], acc);
        const float v_ = epi_v(acc, bias != nullptr, bv, relu);
        if (use_qkv) qkv_store_at(qkv, m, n, v_, kdst);
        else y[(size_t)m * W.N + n] = v_;
    }
}

bool matmul_ln(const DevW& W, const LnIn& ln, int M, const float* bias, int relu, float* y, const QKVStore* qkv,
               cudaStream_t st) {
    if (M < 1 || M > kLnRows || W.K != kD || (W.type != W_Q8_0 && W.type != W_Q4_0)) return false;
    QKVStore q{};
    if (qkv) q = *qkv;
    const int grid = (W.N + 3) / 4;
    if (W.type == W_Q8_0) launch_k(k_mm_ln<W_Q8_0>, dim3(grid), dim3(128), 0, st, W, ln, M, bias, relu, y, q, qkv ? 1 : 0);
    else launch_k(k_mm_ln<W_Q4_0>, dim3(grid), dim3(128), 0, st, W, ln, M, bias, relu, y, q, qkv ? 1 : 0);
    return true;
}

int narrow_min_rows() {
    static const int v = [] {
        const char* e = getenv("T2SX_NARROW_MIN_ROWS");
        const int r = e ? atoi(e) : 8;
        return r > 0 ? r : 8;
    }();
    return v;
}

int tc_min_rows() {
    static const int v = [] {
        const char* e = getenv("T2SX_TC_MIN_ROWS");
        const int r = e ? atoi(e) : 64;
        return r > 0 ? r : 64;
    }();
    return v;
}

// F16 / F32 weights for many rows (CUDA cores): a CTA computes a 64 x 64 block of outputs (64
// weight rows x 64 activation rows), each of its 256 threads a 4 x 4 sub-block.  The arithmetic
// per output is the small kernel's: per 32-element block a chain of fmas from 0 over the
// elements in order, and the blocks added in order from 0.  Each block's weight and activation
// slices are staged in shared memory as f32, K-major, double-buffered.
template <int WT>
__global__ void __launch_bounds__(256) k_mm_fp_tile(DevW W, ActQ A, int M, const float* __restrict__ bias, int relu,
                                                     float* __restrict__ y, QKVStore qkv, int use_qkv) {
    pdl_wait();
    pdl_trigger();
    constexpr int TN = 64, TM = 64, KB = 32;
    __shared__ __align__(16) float ws[2][KB][TN];
    __shared__ __align__(16) float xs[2][KB][TM];
    const int N = W.N, K = W.K, nb = K / KB;
    const int n0 = blockIdx.x * TN, m0 = blockIdx.y * TM;
    const int tid = threadIdx.x, tn = tid & 15, tm = tid >> 4;
    // staging: thread t copies 8 consecutive elements of one row (of W and of A) per block; the
    // next block's global loads are issued before this block's fmas and stored to shared memory
    // after them
    const int lr = tid >> 2, lk = (tid & 3) * 8;
    uint4 wraw, xraw;        // F16: 8 halves each
    float4 wf0, wf1, xf0, xf1;   // F32
    auto load = [&](int b) {
        const int n = n0 + lr, m = m0 + lr, k = b * KB + lk;
        if (WT == W_F16) {
            wraw = n < N ? *reinterpret_cast<const uint4*>(W.h + (size_t)n * K + k) : make_uint4(0, 0, 0, 0);
            xraw = m < M ? *reinterpret_cast<const uint4*>(A.h + (size_t)m * K + k) : make_uint4(0, 0, 0, 0);
        } else {
            const float4 z = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            wf0 = n < N ? *reinterpret_cast<const float4*>(W.f + (size_t)n * K + k) : z;
            wf1 = n < N ? *reinterpret_cast<const float4*>(W.f + (size_t)n * K + k + 4) : z;
            xf0 = m < M ? *reinterpret_cast<const float4*>(A.f + (size_t)m * K + k) : z;
            xf1 = m < M ? *reinterpret_cast<const float4*>(A.f + (size_t)m * K + k + 4) : z;
        }
    };
    auto store = [&](int buf) {
        float wv[8], xv[8];
        if (WT == W_F16) {
            const uint32_t w4[4] = {wraw.x, wraw.y, wraw.z, wraw.w}, x4[4] = {xraw.x, xraw.y, xraw.z, xraw.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                wv[2 * i] = h2f((uint16_t)(w4[i] & 0xffffu)); wv[2 * i + 1] = h2f((uint16_t)(w4[i] >> 16));
                xv[2 * i] = h2f((uint16_t)(x4[i] & 0xffffu)); xv[2 * i + 1] = h2f((uint16_t)(x4[i] >> 16));
            }
        } else {
            wv[0] = wf0.x; wv[1] = wf0.y; wv[2] = wf0.z; wv[3] = wf0.w; wv[4] = wf1.x; wv[5] = wf1.y; wv[6] = wf1.z; wv[7] = wf1.w;
            xv[0] = xf0.x; xv[1] = xf0.y; xv[2] = xf0.z; xv[3] = xf0.w; xv[4] = xf1.x; xv[5] = xf1.y; xv[6] = xf1.z; xv[7] = xf1.w;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) { ws[buf][lk + i][lr] = wv[i]; xs[buf][lk + i][lr] = xv[i]; }
    };
    float acc[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[j][i] = 0.0f;
    load(0);
    store(0);
    __syncthreads();
    for (int b = 0; b < nb; ++b) {
        const int buf = b & 1;
        if (b + 1 < nb) load(b + 1);
        float sblk[4][4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int i = 0; i < 4; ++i) sblk[j][i] = 0.0f;
#pragma unroll
        for (int k = 0; k < KB; ++k) {
            const float4 w4 = *reinterpret_cast<const float4*>(&ws[buf][k][4 * tn]);
            const float4 x4 = *reinterpret_cast<const float4*>(&xs[buf][k][4 * tm]);
            const float wr[4] = {w4.x, w4.y, w4.z, w4.w}, xr[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int i = 0; i < 4; ++i) sblk[j][i] = __fmaf_rn(wr[j], xr[i], sblk[j][i]);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[j][i] = __fadd_rn(acc[j][i], sblk[j][i]);
        if (b + 1 < nb) store(buf ^ 1);   // buf ^ 1 was last read before the previous barrier
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = m0 + 4 * tm + i;
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int n = n0 + 4 * tn + j;
            if (n >= N) continue;
            const float v = epi(acc[j][i], bias, n, relu);
            if (use_qkv) qkv_store(qkv, m, n, v);
            else y[(size_t)m * N + n] = v;
        }
    }
}

// Rows from which F16 / F32 weights use the tiled kernel (T2SX_FP_TILE_MIN_ROWS; 0 = never).
static int fp_tile_min_rows() {
    static const int v = [] {
        const char* e = getenv("T2SX_FP_TILE_MIN_ROWS");
        return e ? atoi(e) : kSmallM + 1;
    }();
    return v;
}

static bool f16_sk_on() {
    static const bool v = [] {
        const char* e = getenv("T2SX_F16_SK");
        return !(e && e[0] == '0');
    }();
    return v;
}

void matmul(const DevW& W, const ActQ& a_in, int M, const float* bias, int relu, float* y, cudaStream_t st, const Epi& e) {
    const bool quant = W.type == W_Q8_0 || W.type == W_Q4_0 || W.type == W_Q4_K;
    ActQ a = a_in;
    // fused input quantisation: the few-row kernel is the one that runs (no narrow or tensor
    // tiles: M below their thresholds, or a tail), at most kDDM rows, 16-byte aligned rows
    const bool fq = e.quant_in && (W.type == W_Q8_0 || W.type == W_Q4_0) && M <= kDDM &&
                    (M < narrow_min_rows() || e.tail) && M < tc_min_rows() && (((uintptr_t)a.f) & 15) == 0;
    if (e.quant_in && !fq) quantize_act(W.type, a.f, M, W.K, a, st);
    if (quant && M >= tc_min_rows() && matmul_tc(W, a, M, bias, relu, y, e.qkv, st)) return;
    if (quant && M > kSmallM && matmul_sk_mid(W, a, M, bias, relu, y, e.qkv, st)) return;
    if (quant && M > kSmallM && matmul_mma(W, a, M, bias, relu, y, e.qkv, st)) return;
    if (quant && M >= narrow_min_rows() && !(e.tail && M <= kSmallM) && matmul_mma_narrow(W, a, M, bias, relu, y, e.qkv, st))
        return;
    // F16 weights at 8-256 rows: split-K tiles (T2SX_F16_SK=0: the tiled kernel / per-row kernel)
    if (W.type == W_F16 && M >= narrow_min_rows() && M <= 256 && !(e.tail && M <= kSmallM) && f16_sk_on() &&
        matmul_f16_sk(W, a, M, bias, relu, y, e.qkv, st))
        return;
    QKVStore qkv{};
    if (e.qkv) qkv = *e.qkv;
    // (16-byte loads: the f32 activations may be a caller's pointer)
    const bool fp_aligned = W.type == W_F16 ? (((uintptr_t)a.h | (uintptr_t)W.h) & 15) == 0
                                            : (((uintptr_t)a.f | (uintptr_t)W.f) & 15) == 0;
    if ((W.type == W_F16 || W.type == W_F32) && fp_tile_min_rows() > 0 && M >= fp_tile_min_rows() && W.K % 32 == 0 &&
        fp_aligned && !(e.tail && M <= kSmallM)) {
        const dim3 grid((W.N + 63) / 64, (M + 63) / 64);
        if (W.type == W_F16) launch_k(k_mm_fp_tile<W_F16>, grid, dim3(256), 0, st, W, a, M, bias, relu, y, qkv, e.qkv ? 1 : 0);
        else launch_k(k_mm_fp_tile<W_F32>, grid, dim3(256), 0, st, W, a, M, bias, relu, y, qkv, e.qkv ? 1 : 0);
        return;
    }
    Tail tail{};
    const bool use_tail = e.tail && M <= kSmallM;
    if (use_tail) tail = *e.tail;
    for (int m0 = 0; m0 < M; m0 += kSmallM) {
        const int mm = (M - m0) < kSmallM ? (M - m0) : kSmallM;
        ActQ as = a;
        const int K = W.K;
        if (as.q) as.q += (size_t)m0 * K;
        if (as.h) as.h += (size_t)m0 * K;
        if (as.f) as.f += (size_t)m0 * K;
        if (as.d) as.d += (size_t)m0 * (W.type == W_Q4_K ? K / 256 : K / 32);
        if (as.bs) as.bs += (size_t)m0 * (K / 32);
        float* yy = y ? y + (size_t)m0 * W.N : nullptr;
        QKVStore qq = qkv;
        if (e.qkv) {
            qq.rows.slot += m0;
            qq.rows.pos += m0;
            qq.rows.L += m0;
            qq.q16 += (size_t)m0 * kD;
        }
        const int grid = (W.N + 3) / 4;
        const int uq = e.qkv ? 1 : 0, ut = use_tail ? 1 : 0, ufq = fq ? 1 : 0;
        switch (W.type) {
            case W_Q8_0: launch_k(k_mm_small<W_Q8_0>, dim3(grid), dim3(128), 0, st, W, as, mm, bias, relu, yy, qq, uq, tail, ut, ufq); break;
            case W_Q4_0: launch_k(k_mm_small<W_Q4_0>, dim3(grid), dim3(128), 0, st, W, as, mm, bias, relu, yy, qq, uq, tail, ut, ufq); break;
            case W_Q4_K: launch_k(k_mm_small<W_Q4_K>, dim3(grid), dim3(128), 0, st, W, as, mm, bias, relu, yy, qq, uq, tail, ut, 0); break;
            case W_F16: launch_k(k_mm_small<W_F16>, dim3(grid), dim3(128), 0, st, W, as, mm, bias, relu, yy, qq, uq, tail, ut, 0); break;
            default: launch_k(k_mm_small<W_F32>, dim3(grid), dim3(128), 0, st, W, as, mm, bias, relu, yy, qq, uq, tail, ut, 0); break;
        }
    }
}

// ============================================================================================
// embedding, KV append, attention, LayerNorm, sampler
// ============================================================================================

// Decode embedding (session.cpp:337-344): x = emb[tok] + pe[n_pos - audio_offset] * alpha, one
// warp per row; writes x (f32, the first residual) and x in the first matmul's dot type.  Also
// fixes the row's KV position (n_pos) and attended length (n_pos + 1).
__global__ void k_embed_decode(int T, const int32_t* __restrict__ row_slot, const int32_t* __restrict__ token_in,
                               const int32_t* __restrict__ n_pos, const int32_t* __restrict__ audio_off,
                               const uint16_t* __restrict__ emb16, const float* __restrict__ emb32, int emb_rows,
                               const float* __restrict__ pe, int pe_rows, float alpha, Rows rows, float* __restrict__ x,
                               int qtype, ActQ qo) {
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (r >= T) return;
    const int s = row_slot[r];
    const int pos = n_pos[s];
    const int pp = pos - audio_off[s];
    const int tok = token_in[s];
    const bool ok = pos >= 0 && pos < rows.cap[s] && pp >= 0 && pp < pe_rows && tok >= 0 && tok < emb_rows;
    if (lane == 0) {
        rows.pos[r] = ok ? pos : -1;
        rows.L[r] = ok ? pos + 1 : 0;
        if (!ok) atomicExch(rows.err, 1);
    }
    float v[kD / 32];
#pragma unroll
    for (int t = 0; t < kD / 32; ++t) {
        const int d = lane + 32 * t;
        v[t] = 0.0f;
        if (ok) {
            const float e = emb16 ? h2f(emb16[(size_t)tok * kD + d]) : emb32[(size_t)tok * kD + d];
            v[t] = __fadd_rn(e, __fmul_rn(pe[(size_t)pp * kD + d], alpha));
        }
        x[(size_t)r * kD + d] = v[t];
    }
    quant_row512_strided(v, lane, qtype, qo, (size_t)r);
}

void embed_decode(int T, const int32_t* row_slot, const int32_t* token_in, const int32_t* n_pos,
                  const int32_t* audio_off, const uint16_t* emb16, const float* emb32, int emb_rows, const float* pe,
                  int pe_rows, float alpha, Rows rows, float* x, int qtype, ActQ qo, cudaStream_t st) {
    if (T > 0)
        launch_k(k_embed_decode, dim3((T + 3) / 4), dim3(128), 0, st, T, row_slot, token_in, n_pos, audio_off, emb16, emb32, emb_rows, pe,
                                                    pe_rows, alpha, rows, x, qtype, qo);
}

// One round of the lane merge with partner lane ^ OFF: in holds 2N values (dims whose bits
// above OFF match this lane), out receives the N whose bit OFF matches; m and l merge in full.
template <int OFF, int N>
__device__ __forceinline__ void attn_merge_round(AttnState& st, int lane, const float* in, float* out) {
    const float mB = __shfl_xor_sync(0xffffffffu, st.m, OFF);
    const float lB = __shfl_xor_sync(0xffffffffu, st.l, OFF);
    float M, a, b, l;
    bool empty;
    st_merge_scalars(st.m, st.l, mB, lB, M, a, b, l, empty);
    const bool hi = (lane & OFF) != 0;
#pragma unroll
    for (int u = 0; u < N; ++u) {
        const float keep = hi ? in[N + u] : in[u];
        const float send = hi ? in[u] : in[N + u];
        const float oB = __shfl_xor_sync(0xffffffffu, send, OFF);
        out[u] = empty ? 0.0f : __fadd_rn(__fmul_rn(keep, a), __fmul_rn(oB, b));
    }
    st.m = empty ? __int_as_float(0xff800000) : M;
    st.l = l;
}

// Merge of a warp's 32 position lanes in xor-butterfly order (partners 16, 8, 4, 2, 1; the merge
// is symmetric, so every lane ends with the same state and lane d owns output dim d), then the
// output row in the out-projection's dot type (a Q8_0 block is one head, a Q8_K block the CTA's
// eight heads: every warp of the CTA must call this for the same row), or f32 when qtype < 0.
template <int HPC>
__device__ __forceinline__ void attn_finish(AttnState& st, int r, int hg, int warp, int lane, float* __restrict__ out,
                                            int qtype, const ActQ& qo, AbsMax* s_am, float* s_is) {
    // The butterfly runs as a reduce-scatter: at the round with partner lane ^ off a lane keeps the
    // half of its dims whose bit `off` equals its own and receives the partner's values for them,
    // so after the five rounds lane d holds dim d.  Every kept value is the one the full butterfly
    // computes at that lane (the partner holds the same dims, and m, l still follow the full
    // butterfly), with 31 exchanged values per lane instead of 160.
    float o16[16], o8[8], o4[4], o2[2], mine;
    attn_merge_round<16, 16>(st, lane, st.o, o16);
    attn_merge_round<8, 8>(st, lane, o16, o8);
    attn_merge_round<4, 4>(st, lane, o8, o4);
    attn_merge_round<2, 2>(st, lane, o4, o2);
    attn_merge_round<1, 1>(st, lane, o2, &mine);
    const float val = __fmul_rn(mine, __fdiv_rn(1.0f, st.l));
    const int h = hg * HPC + warp;
    const size_t e = (size_t)r * kD + h * kHeadDim + lane;
    if (qtype == W_Q8_0 || qtype == W_Q4_0) {
        qo.q[e] = (int8_t)q8_0_lane(val, qo.d + (size_t)r * (kD / 32) + h, lane);
    } else if (qtype == W_Q4_K && HPC == 8) {
        AbsMax am{0.0f, 0.0f, 0x7fffffff};
        absmax_take(am, val, warp * kHeadDim + lane);
        am = absmax_warp(am);
        if (lane == 0) s_am[warp] = am;
        __syncthreads();
        if (threadIdx.x == 0) {
            AbsMax all = s_am[0];
            for (int w = 1; w < 8; ++w) absmax_merge(all, s_am[w]);
            const float iscale = q8k_iscale(all);
            *s_is = iscale;
            qo.d[(size_t)r * (kD / 256) + hg] = q8k_d(iscale);
        }
        __syncthreads();
        const int qv = q8k_q(*s_is, val);
        qo.q[e] = (int8_t)qv;
        const int sum = warp_sum_i(qv);
        if (lane == 0) qo.bs[(size_t)r * (kD / 32) + h] = sum;
    } else if (qtype == W_F16) {
        qo.h[e] = f2h(val);
    } else {
        out[e] = val;
    }
}

// Decode attention: one warp per (row, head), eight heads of a row per CTA.  Position lane
// t = lane folds positions t, t+32, ... with the online update; the 32 lanes merge in the
// order of an xor butterfly (partners 16, 8, 4, 2, 1).  The merge is symmetric, so every lane
// ends with the same state and lane d owns output dim d.  The output row is written in the
// out-projection's dot type (a Q8_0 block is one head, a Q8_K block the CTA's eight heads), or
// as f32 when qtype < 0.
// PF: each lane's next position's K/V rows are loaded while the current one is folded (a two-deep
// register pipeline over the lane's positions, K and V held as packed f16 pairs).
template <int HPC, bool PIPE, bool PF = false>
__global__ void __launch_bounds__(32 * HPC) k_attn_decode(const uint16_t* __restrict__ q16, Rows rows, KVView kv, int layer,
                                                          float scale, float* __restrict__ out, int qtype, ActQ qo) {
    __shared__ AbsMax s_am[8];
    __shared__ float s_is;
    // CTAs in (row, head group) order, head group fastest: the CTAs of one row run together and
    // share the address translations of its pages
    const int r = blockIdx.x / (kHeads / HPC), hg = blockIdx.x % (kHeads / HPC);
    const int warp = threadIdx.x >> 5;
    const int h = hg * HPC + warp;
    const int lane = threadIdx.x & 31;
    // the row's slot and length were written two or more launches back (read before the wait)
    const int s = rows.slot[r];
    const int L = rows.L[r];
    pdl_wait();
    pdl_trigger();
    uint32_t q[kHeadDim / 2];   // the f16 query as packed pairs (the score's mixed-precision fma chain)
    load_row32_h(q16 + (size_t)r * kD + h * kHeadDim, q);
    AttnState st;
    st_empty(st);
    const int32_t* pt = kv.ptab + (size_t)s * kv.max_pages;
    if (!PIPE && PF) {
        uint32_t kc[kHeadDim / 2], vc[kHeadDim / 2];
        auto load_pos = [&](int i, uint32_t (&kw)[kHeadDim / 2], uint32_t (&vw)[kHeadDim / 2]) {
            const int page = pt[i / kPage];
            load_row32_h(kv.pool + kv_off(kv, page, layer, 0, h, i % kPage), kw);
            load_row32_h(kv.pool + kv_off(kv, page, layer, 1, h, i % kPage), vw);
        };
        if (lane < L) load_pos(lane, kc, vc);
        for (int i = lane; i < L; i += kAttnLanes) {
            uint32_t kn[kHeadDim / 2], vn[kHeadDim / 2];
            if (i + kAttnLanes < L) load_pos(i + kAttnLanes, kn, vn);
            st_update_h(st, __fmul_rn(dot32_h(q, kc), scale), vc);
#pragma unroll
            for (int w = 0; w < kHeadDim / 2; ++w) { kc[w] = kn[w]; vc[w] = vn[w]; }
        }
    } else if (!PIPE) {
        for (int i = lane; i < L; i += kAttnLanes) {
            const int page = pt[i / kPage];
            uint32_t k[kHeadDim / 2];
            float v[kHeadDim];
            load_row32_h(kv.pool + kv_off(kv, page, layer, 0, h, i % kPage), k);
            load_row32(kv.pool + kv_off(kv, page, layer, 1, h, i % kPage), v);
            st_update(st, __fmul_rn(dot32_h(q, k), scale), v);
        }
    }
    if (PIPE) {
        // Small batches (latency-bound): each lane keeps D of its positions in flight with
        // cp.async into its own slots of a shared-memory ring ([slot][16-byte chunk][thread], so
        // a warp's reads of one chunk are bank-conflict free); the fold order is unchanged.  All
        // lanes of a warp read the same page at a step (positions lane + 32k lie in page k / 2),
        // so the row's page numbers are staged in shared memory first.
        constexpr int NT = 32 * HPC;
        constexpr int D = 16 / HPC;
        extern __shared__ __align__(16) uint8_t dsm[];
        int32_t* s_pt = reinterpret_cast<int32_t*>(dsm + D * 8 * NT * 16);
        const int np = (L + kPage - 1) / kPage;
        for (int j = threadIdx.x; j < np; j += NT) s_pt[j] = pt[j];
        __syncthreads();
        const int nk = (L - lane + kAttnLanes - 1) / kAttnLanes;   // this lane's positions
        // position lane + 32k lies in page k / 2 at lane + 32 (k & 1)
        const uint16_t* kvb = kv_head_base(kv, layer, h) + lane * kHeadDim;
        auto issue = [&](int k) {
            if (k < nk) {
                const uint16_t* kp = kvb + (size_t)s_pt[k >> 1] * kPageElems + (k & 1) * (kAttnLanes * kHeadDim);
                const uint16_t* vp = kp + kHalfPageElems;
                uint8_t* dst = dsm + (size_t)(k % D) * 8 * NT * 16 + threadIdx.x * 16;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    cp_async16(dst + c * NT * 16, kp + 8 * c, true);
                    cp_async16(dst + (4 + c) * NT * 16, vp + 8 * c, true);
                }
            }
            cp_commit();
        };
#pragma unroll
        for (int k = 0; k < D - 1; ++k) issue(k);
        for (int k = 0; k < nk; ++k) {
            asm volatile("" ::: "memory");   // the previous step's reads of that slot stay before the refill
            issue(k + D - 1);   // into the slot read in the previous step
            cp_wait<D - 1>();
            const uint8_t* src = dsm + (size_t)(k % D) * 8 * NT * 16 + threadIdx.x * 16;
            uint4 kr[4], vr[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                kr[c] = *reinterpret_cast<const uint4*>(src + c * NT * 16);
                vr[c] = *reinterpret_cast<const uint4*>(src + (4 + c) * NT * 16);
            }
            uint32_t kw[kHeadDim / 2];
            float v32[kHeadDim];
            words16(kr, kw);
            unpack_row32(vr, v32);
            st_update(st, __fmul_rn(dot32_h(q, kw), scale), v32);
        }
        cp_wait<0>();
    }
    attn_finish<HPC>(st, r, hg, warp, lane, out, qtype, qo, s_am, &s_is);
}

// Decode attention for very few rows: one CTA per (row, head), 4 threads per position lane.  With
// one warp per head the fold was a single instruction stream per SM (about 200 dependent
// instructions per position); here thread (lane group a, quarter j) of warp w folds position lane
// vl = 8w + a over dims 8j..8j+7.  The score's 32-term dot is four sequential 8-term fma chains
// summed as (c0 + c1) + (c2 + c3): thread j runs chain j and the two xor shuffles sum them in that
// order, so all four threads hold the same score and run the same online update (m, l) on their
// own 8 dims of o.  The merge keeps the butterfly partners 16, 8, 4, 2, 1 (the first two between
// warps, through shared memory) and the merge formula, so the row equals the one-warp kernel's.
constexpr int kQD = 16;   // positions per lane in flight (fewer than 4 rows)
constexpr int kQD32 = 8;  // 4-32 rows: 32 KB rings, so that all (row, head) CTAs are resident at once
                          // (32-session steps of one build: 8 deep 1.157 ms, 10 deep 1.154, 12 deep 1.165, 16 deep 1.289)

// The online-softmax step of a position lane (8 of its dims) for positions k and k + 1 (the second
// only if has1).  A position with score s against the running maximum m: a new maximum (s > m)
// takes t = e^(m - s), m = s, l = fma(l, t, 1), o = fma(o, t, v); otherwise t = e^(s - m),
// l = l + t, o = fma(t, v, o).  The running maximum does not depend on the weights, so both
// weights e^(-|s - m|) (fsub(m, s) = -fsub(s, m) exactly) are formed side by side from the maxima,
// and the updates use selects instead of branches that the lanes of a warp would take apart:
// fma(v, t, o) = fma(t, v, o), and fma(1, t, l) = l + t.
__device__ __forceinline__ void st_update8_pair(float& m, float& l, float (&o)[8], float s0, const float (&v0)[8],
                                                float s1, const float (&v1)[8], bool has1) {
    const bool g0 = s0 > m;
    const float m1 = g0 ? s0 : m;
    const bool g1 = has1 && s1 > m1;
    const float t0 = t2s_expf(-fabsf(__fsub_rn(s0, m)));
    const float t1 = t2s_expf(-fabsf(__fsub_rn(s1, m1)));
    l = __fmaf_rn(g0 ? l : 1.0f, t0, g0 ? 1.0f : l);
#pragma unroll
    for (int d = 0; d < 8; ++d) o[d] = __fmaf_rn(g0 ? o[d] : v0[d], t0, g0 ? v0[d] : o[d]);
    m = m1;
    if (has1) {
        l = __fmaf_rn(g1 ? l : 1.0f, t1, g1 ? 1.0f : l);
#pragma unroll
        for (int d = 0; d < 8; ++d) o[d] = __fmaf_rn(g1 ? o[d] : v1[d], t1, g1 ? v1[d] : o[d]);
        m = g1 ? s1 : m1;
    }
}

__device__ __forceinline__ void st_merge8(float& m, float& l, float (&o)[8], float mB, float lB, const float (&oB)[8]) {
    float M, a, b, ln;
    bool empty;
    st_merge_scalars(m, l, mB, lB, M, a, b, ln, empty);
#pragma unroll
    for (int d = 0; d < 8; ++d) o[d] = empty ? 0.0f : __fadd_rn(__fmul_rn(o[d], a), __fmul_rn(oB[d], b));
    m = empty ? __int_as_float(0xff800000) : M;
    l = ln;
}

__device__ __forceinline__ void unpack8(const uint4& u, float (&out)[8]) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        out[2 * e] = h2f((uint16_t)(w[e] & 0xffffu));
        out[2 * e + 1] = h2f((uint16_t)(w[e] >> 16));
    }
}

template <int QD>
__global__ void __launch_bounds__(128) k_attn_decode_split(const uint16_t* __restrict__ q16, Rows rows, KVView kv, int layer,
                                                          float scale, float* __restrict__ out, int qtype, ActQ qo) {
    extern __shared__ __align__(16) uint8_t dsm[];
    // [slot][K | V][thread] 16-byte chunks, then the merge exchange (10 floats per thread), the
    // output head, and the row's page numbers
    float* s_x = reinterpret_cast<float*>(dsm + QD * 2 * 128 * 16);
    float* s_val = s_x + 10 * 128;
    int32_t* s_pt = reinterpret_cast<int32_t*>(s_val + 32);
    const int r = blockIdx.x / kHeads, h = blockIdx.x % kHeads;
    const int tid = threadIdx.x, w = tid >> 5, t = tid & 31, a = t >> 2, j = t & 3;
    const int vl = 8 * w + a;
    // Before pdl_wait (a programmatic launch overlaps the preceding QKV projection): the row's slot
    // and length (written two or more launches back), its page numbers, and the K/V of every
    // position but the last T (the rows of this pass): those the QKV projection is appending.
    const int s = rows.slot[r];
    const int L = rows.L[r];
    const int T = gridDim.x / kHeads;
    const int32_t* pt = kv.ptab + (size_t)s * kv.max_pages;
    const int np = (L + kPage - 1) / kPage;
    for (int i = tid; i < np; i += 128) s_pt[i] = pt[i];
    __syncthreads();
    float m = __int_as_float(0xff800000), l = 0.0f, o[8];
#pragma unroll
    for (int d = 0; d < 8; ++d) o[d] = 0.0f;
    const int nk = (L - vl + kAttnLanes - 1) / kAttnLanes;   // this position lane's positions
    const unsigned gmask = 0xFu << (4 * a);                  // the four threads of the lane
    // position vl + 32k lies in page k / 2 at vl + 32 (k & 1)
    const uint16_t* kvb = kv_head_base(kv, layer, h) + vl * kHeadDim + 8 * j;
    // this lane's positions from step k_new on are among the last T, which the preceding QKV
    // projection may be appending (with T <= 32 at most the lane's last position)
    const int k_new = (L - T - vl <= 0) ? 0 : (L - T - vl + kAttnLanes - 1) / kAttnLanes;
    bool early = true;   // issuing before pdl_wait
    auto issue = [&](int k) {
        if (k < nk && !(early && k >= k_new)) {
            const uint16_t* kp = kvb + (size_t)s_pt[k >> 1] * kPageElems + (k & 1) * (kAttnLanes * kHeadDim);
            uint8_t* dst = dsm + (size_t)(k % QD) * 2 * 128 * 16 + tid * 16;
            cp_async16(dst, kp, true);
            cp_async16(dst + 128 * 16, kp + kHalfPageElems, true);
        }
        cp_commit();
    };
    // positions in pairs: the two scores are independent chains (computed side by side), the two
    // updates run in position order; each pair refills the two slots the previous pair read
#pragma unroll
    for (int k = 0; k < QD - 2; ++k) issue(k);
    early = false;
    pdl_wait();
    pdl_trigger();
    const uint4 q4 = *reinterpret_cast<const uint4*>(q16 + (size_t)r * kD + h * kHeadDim + 8 * j);   // f16 pairs
    for (int k = k_new; k < nk && k < QD - 2; ++k) {   // slots committed empty above: read them now
        const uint16_t* kp = kvb + (size_t)s_pt[k >> 1] * kPageElems + (k & 1) * (kAttnLanes * kHeadDim);
        uint8_t* dst = dsm + (size_t)(k % QD) * 2 * 128 * 16 + tid * 16;
        *reinterpret_cast<uint4*>(dst) = __ldcg(reinterpret_cast<const uint4*>(kp));
        *reinterpret_cast<uint4*>(dst + 128 * 16) = __ldcg(reinterpret_cast<const uint4*>(kp + kHalfPageElems));
    }
    for (int k = 0; k < nk; k += 2) {
        asm volatile("" ::: "memory");   // the previous pair's reads of those slots stay before the refill
        issue(k + QD - 2);
        issue(k + QD - 1);
        cp_wait<QD - 2>();
        const uint8_t* src0 = dsm + (size_t)(k % QD) * 2 * 128 * 16 + tid * 16;
        const uint8_t* src1 = dsm + (size_t)((k + 1) % QD) * 2 * 128 * 16 + tid * 16;
        // the 8-term chain j of each score on the f16 pairs (mixed-precision fma)
        const uint4 k0 = *reinterpret_cast<const uint4*>(src0);
        const uint4 k1 = *reinterpret_cast<const uint4*>(src1);
        float c0 = 0.0f, c1 = 0.0f;
        c0 = fma_h2(q4.x, k0.x, c0); c1 = fma_h2(q4.x, k1.x, c1);
        c0 = fma_h2(q4.y, k0.y, c0); c1 = fma_h2(q4.y, k1.y, c1);
        c0 = fma_h2(q4.z, k0.z, c0); c1 = fma_h2(q4.z, k1.z, c1);
        c0 = fma_h2(q4.w, k0.w, c0); c1 = fma_h2(q4.w, k1.w, c1);
        const float a0 = __fadd_rn(c0, __shfl_xor_sync(gmask, c0, 1));
        const float a1 = __fadd_rn(c1, __shfl_xor_sync(gmask, c1, 1));
        const float dot0 = __fadd_rn(a0, __shfl_xor_sync(gmask, a0, 2));
        const float dot1 = __fadd_rn(a1, __shfl_xor_sync(gmask, a1, 2));
        float v0[8], v1[8];
        unpack8(*reinterpret_cast<const uint4*>(src0 + 128 * 16), v0);
        unpack8(*reinterpret_cast<const uint4*>(src1 + 128 * 16), v1);
        st_update8_pair(m, l, o, __fmul_rn(dot0, scale), v0, __fmul_rn(dot1, scale), v1, k + 1 < nk);
    }
    cp_wait<0>();
    // butterfly rounds 16 and 8: partner thread tid ^ 64, then tid ^ 32
#pragma unroll
    for (int rnd = 0; rnd < 2; ++rnd) {
        const int pt_ = tid ^ (rnd == 0 ? 64 : 32);
        __syncthreads();
        s_x[tid * 10] = m;
        s_x[tid * 10 + 1] = l;
#pragma unroll
        for (int d = 0; d < 8; ++d) s_x[tid * 10 + 2 + d] = o[d];
        __syncthreads();
        float oB[8];
#pragma unroll
        for (int d = 0; d < 8; ++d) oB[d] = s_x[pt_ * 10 + 2 + d];
        st_merge8(m, l, o, s_x[pt_ * 10], s_x[pt_ * 10 + 1], oB);
    }
    // rounds 4, 2, 1: partner lane group a ^ off, the same quarter (lane t ^ 4 * off)
#pragma unroll
    for (int off = 4; off >= 1; off >>= 1) {
        const float mB = __shfl_xor_sync(0xffffffffu, m, 4 * off);
        const float lB = __shfl_xor_sync(0xffffffffu, l, 4 * off);
        float oB[8];
#pragma unroll
        for (int d = 0; d < 8; ++d) oB[d] = __shfl_xor_sync(0xffffffffu, o[d], 4 * off);
        st_merge8(m, l, o, mB, lB, oB);
    }
    // every thread now holds the merged state of its quarter; lane d of warp 0 takes dim d
    if (w == 0 && a == 0) {
        const float inv = __fdiv_rn(1.0f, l);
#pragma unroll
        for (int d = 0; d < 8; ++d) s_val[8 * j + d] = __fmul_rn(o[d], inv);
    }
    __syncthreads();
    if (w != 0) return;
    const float val = s_val[t];
    const size_t e = (size_t)r * kD + h * kHeadDim + t;
    if (qtype == W_Q8_0 || qtype == W_Q4_0) qo.q[e] = (int8_t)q8_0_lane(val, qo.d + (size_t)r * (kD / 32) + h, t);
    else if (qtype == W_F16) qo.h[e] = f2h(val);
    else out[e] = val;
}

// Prefill attention: a CTA takes a group of up to 16 consecutive rows of one slot (the rows of a
// prompt) and one head, one warp per row.  The group's K/V are staged in shared memory a page (64
// positions) at a time, double-buffered with cp.async, and every warp folds them with the decode
// kernel's lane order (lane l: positions l, l + 32, ...; page p gives its steps 2p and 2p + 1), so
// the K/V of a prompt are read once per 16 rows instead of once per row.  Staged 16-byte chunks
// are swizzled by position so that the lanes' reads of one chunk hit distinct banks.  f32 rows out.
// (Staging f32 instead, converted once for all rows, was slower: twice the shared-memory reads.)
__global__ void __launch_bounds__(512, 1) k_attn_group(const int2* __restrict__ groups, const uint16_t* __restrict__ q16,
                                                       Rows rows, KVView kv, int layer, float scale, float* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    __shared__ __align__(16) uint8_t sm[2][2][kPage * kHeadDim * 2];   // [buffer][K|V][64 positions x 64 B]
    __shared__ int s_lmax;
    const int2 gr = groups[blockIdx.x >> 4];   // (first row, rows)
    const int h = blockIdx.x & 15;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool active = warp < gr.y;
    const int r = gr.x + warp;
    const int L = active ? rows.L[r] : 0;
    if (threadIdx.x == 0) s_lmax = 0;
    __syncthreads();
    if (lane == 0 && active) atomicMax(&s_lmax, L);
    __syncthreads();
    const int Lmax = s_lmax;
    const int32_t* pt = kv.ptab + (size_t)rows.slot[gr.x] * kv.max_pages;
    uint32_t q[kHeadDim / 2] = {};   // the f16 query as packed pairs
    if (active) load_row32_h(q16 + (size_t)r * kD + h * kHeadDim, q);
    AttnState st;
    st_empty(st);
    const int npg = (Lmax + kPage - 1) / kPage;
    // thread t copies 16 bytes: K or V (t / 256), position (t / 4) % 64, chunk t % 4
    const int cw = threadIdx.x >> 8, cp = (threadIdx.x >> 2) & 63, cc = threadIdx.x & 3;
    const int coff = cp * 64 + ((cc ^ ((cp >> 1) & 3)) << 4);
    auto stage = [&](int pg, int buf) {
        const uint16_t* src = kv.pool + kv_off(kv, pt[pg], layer, cw, h, cp) + cc * 8;
        cp_async16(&sm[buf][cw][coff], src, pg * kPage + cp < Lmax);
        cp_commit();
    };
    if (npg > 0) stage(0, 0);
    const int sw = (lane >> 1) & 3;   // the swizzle of positions lane and lane + 32
    for (int pg = 0; pg < npg; ++pg) {
        if (pg + 1 < npg) stage(pg + 1, (pg + 1) & 1);
        else cp_commit();
        cp_wait<1>();
        __syncthreads();
        const int buf = pg & 1;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const int p = half * 32 + lane;
            if (pg * kPage + p < L) {
                uint4 kr[4], vr[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    kr[c] = *reinterpret_cast<const uint4*>(&sm[buf][0][p * 64 + ((c ^ sw) << 4)]);
                    vr[c] = *reinterpret_cast<const uint4*>(&sm[buf][1][p * 64 + ((c ^ sw) << 4)]);
                }
                uint32_t kw[kHeadDim / 2];
                float v32[kHeadDim];
                words16(kr, kw);
                unpack_row32(vr, v32);
                st_update(st, __fmul_rn(dot32_h(q, kw), scale), v32);
            }
        }
        __syncthreads();   // this buffer is refilled in the next step
    }
    cp_wait<0>();
    if (active) attn_finish<1>(st, r, h, 0, lane, out, -1, ActQ(), nullptr, nullptr);
}

// Attention of a pass whose rows [row0, T) are prefill rows grouped by `groups` (device, n_groups
// entries of (first row, rows), consecutive rows of one slot): rows [0, row0) by the per-row
// kernels, the groups by k_attn_group; the rows are then converted to the out-projection's dot
// type.  n_groups == 0: attention_decode.
void attention_rows(int T, int row0, const int2* groups, int n_groups, const uint16_t* q16, Rows rows, KVView kv, int layer,
                    float scale, float* out, int qtype, ActQ qo, cudaStream_t st) {
    if (n_groups <= 0 || !groups) {
        attention_decode(T, q16, rows, kv, layer, scale, out, qtype, qo, st);
        return;
    }
    if (row0 > 0) attention_decode(row0, q16, rows, kv, layer, scale, out, -1, qo, st);
    launch_k(k_attn_group, dim3(n_groups * kHeads), dim3(512), 0, st, groups, q16, rows, kv, layer, scale, out);
    if (qtype >= 0 && qtype != W_F32) quantize_act(qtype, out, T, kD, qo, st);
}

// Dynamic shared memory of the small-batch (PIPE) attention variant: the cp.async ring plus the
// row's page numbers; the kernel's limit is raised once.
template <int HPC>
static size_t attn_pipe_smem(const KVView& kv) {
    static PerDeviceOnce setup;   // the limit is raised once on each device that launches it
    setup.ensure([](int, int*) {
        return cudaFuncSetAttribute(k_attn_decode<HPC, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) ==
               cudaSuccess;
    });
    return (size_t)(16 / HPC) * 8 * (32 * HPC) * 16 + (size_t)kv.max_pages * 4;
}

// Rows below which the decode attention runs one head per CTA with 16 positions per lane in flight
// (T2SX_ATTN_PIPE1_ROWS; bs=1 step 0.940 -> 0.918 ms).
static int pipe1_rows() {
    static const int v = [] {
        const char* e = getenv("T2SX_ATTN_PIPE1_ROWS");
        return e ? atoi(e) : 4;
    }();
    return v;
}

// Below pipe1_rows() rows: the four-threads-per-lane kernel (T2SX_ATTN_SPLIT=0: one warp per head).
static bool attn_split() {
    static const bool v = [] {
        const char* e = getenv("T2SX_ATTN_SPLIT");
        return !(e && e[0] == '0');
    }();
    return v;
}

// Rows up to which the many-row attention keeps each lane's next position in flight
// (T2SX_ATTN_PF_ROWS, 0 = never).  The two-deep pipeline needs 118 registers (four CTAs per SM);
// the one-deep kernel 96 (five).  At 256 rows, 6.9 CTAs per SM, the pipeline wins (42.5 against
// 44.1 us for the best one-deep variant, the f32 score chain at four CTAs per SM); at 512 and 2048
// rows the fifth CTA per SM wins (72.2 against 76.1 us, 248.8 against 248.9 us).
static int attn_pf_rows() {
    static const int v = [] { const char* e = getenv("T2SX_ATTN_PF_ROWS"); return e ? atoi(e) : 384; }();
    return v;
}

// Up to T2SX_ATTN_PF_ROWS rows with a Q4_K out-projection, eight heads per CTA (two-deep pipeline)
// convert the row to Q8_K in place instead of a separate conversion launch (T2SX_ATTN_Q8K8=0: four
// heads per CTA and the launch).  256 rows: step 1.924 -> 1.911 ms.
static bool attn_q8k_inplace() {
    static const bool v = [] { const char* e = getenv("T2SX_ATTN_Q8K8"); return !(e && e[0] == '0'); }();
    return v;
}

// 4-32 rows (not Q4_K, whose Q8_K output spans eight heads): the four-threads-per-lane kernel as
// well (T2SX_ATTN_SPLIT32=0: two heads per CTA, one warp per head).
static bool attn_split32() {
    static const bool v = [] {
        const char* e = getenv("T2SX_ATTN_SPLIT32");
        return !(e && e[0] == '0');
    }();
    return v;
}

// The four-threads-per-lane kernel with QD positions per lane in flight (QD x 4 KB of rings).
template <int QD>
static void launch_split(int T, const uint16_t* q16, Rows rows, KVView kv, int layer, float scale, float* out,
                         int qtype, ActQ qo, cudaStream_t st) {
    static PerDeviceOnce setup;
    setup.ensure([](int, int*) {
        return cudaFuncSetAttribute(k_attn_decode_split<QD>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) ==
               cudaSuccess;
    });
    const size_t smem = (size_t)QD * 2 * 128 * 16 + (10 * 128 + 32) * 4 + (size_t)kv.max_pages * 4;
    launch_k(k_attn_decode_split<QD>, dim3(T * kHeads), dim3(128), smem, st, q16, rows, kv, layer, scale, out, qtype, qo);
}

void attention_decode(int T, const uint16_t* q16, Rows rows, KVView kv, int layer, float scale, float* out, int qtype,
                      ActQ qo, cudaStream_t st) {
    if (T <= 0) return;
    // a Q8_K output block spans eight heads, so that format needs eight heads per CTA; otherwise
    // small batches spread the heads over more CTAs
    if (qtype == W_Q4_K && T < 64) {
        launch_k((k_attn_decode<8, true>), dim3(T * (kHeads / 8)), dim3(256), attn_pipe_smem<8>(kv), st, q16, rows, kv, layer, scale, out, qtype, qo);
    } else if (qtype == W_Q4_K) {
        // many rows: four heads per CTA with an f32 row, then the Q8_K conversion as its own pass
        // (eight-head CTAs that convert in place wait on two CTA barriers per row: 8.65 -> 8.39 ms
        // for the 2048-row decode step)
        if (T <= attn_pf_rows() && attn_q8k_inplace()) {
            // eight heads per CTA write the row's Q8_K blocks in place (no conversion launch)
            launch_k((k_attn_decode<8, false, true>), dim3(T * (kHeads / 8)), dim3(256), 0, st, q16, rows, kv, layer, scale, out, qtype, qo);
            return;
        }
        if (T <= attn_pf_rows())
            launch_k((k_attn_decode<4, false, true>), dim3(T * (kHeads / 4)), dim3(128), 0, st, q16, rows, kv, layer, scale, out, -1, qo);
        else
            launch_k((k_attn_decode<4, false>), dim3(T * (kHeads / 4)), dim3(128), 0, st, q16, rows, kv, layer, scale, out, -1, qo);
        quantize_act(W_Q4_K, out, T, kD, qo, st);
    } else if (T < pipe1_rows() && T <= kAttnLanes && attn_split()) {
        // very few rows: one head per CTA, four threads per position lane (at most 32 rows: the
        // positions of a pass are then at most one per position lane, which the kernel's early
        // K/V fetch relies on)
        launch_split<kQD>(T, q16, rows, kv, layer, scale, out, qtype, qo, st);
    } else if (T >= pipe1_rows() && T <= kAttnLanes && attn_split32()) {
        // 4-32 rows: the same kernel with 8 positions per lane in flight
        launch_split<kQD32>(T, q16, rows, kv, layer, scale, out, qtype, qo, st);
    } else if (T < pipe1_rows()) {
        // very few rows: one head per CTA, 16 positions per lane in flight
        launch_k((k_attn_decode<1, true>), dim3(T * kHeads), dim3(32), attn_pipe_smem<1>(kv), st, q16, rows, kv, layer, scale, out, qtype, qo);
    } else if (T < 64) {
        launch_k((k_attn_decode<2, true>), dim3(T * (kHeads / 2)), dim3(64), attn_pipe_smem<2>(kv), st, q16, rows, kv, layer, scale, out, qtype, qo);
    } else if (T <= attn_pf_rows()) {
        launch_k((k_attn_decode<4, false, true>), dim3(T * (kHeads / 4)), dim3(128), 0, st, q16, rows, kv, layer, scale, out, qtype, qo);
    } else {
        launch_k((k_attn_decode<4, false>), dim3(T * (kHeads / 4)), dim3(128), 0, st, q16, rows, kv, layer, scale, out, qtype, qo);
    }
}

// y = LN(a + b) * g + beta, one warp per row (ln_row_vals); the row is also written in the next
// matmul's dot type when qtype >= 0.  a must have been written two or more launches back: it is
// read before the programmatic wait.
__global__ void k_residual_ln(int T, const float* __restrict__ a, const float* __restrict__ b,
                              const float* __restrict__ g, const float* __restrict__ beta, float eps,
                              float* __restrict__ y, int qtype, ActQ qo) {
    const int lane = threadIdx.x & 31;
    const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    // before the wait: g, beta and the residual rows a (callers' residuals are written two or
    // more launches back; b is the preceding matmul's output)
    float av[kD / 32], gv[kD / 32], bv[kD / 32];
    const bool live = r < T;
    if (live) {
        load_row_lane(g, lane, gv);
        load_row_lane(beta, lane, bv);
        load_row_lane(a + (size_t)r * kD, lane, av);
    }
    pdl_wait();
    pdl_trigger();
    if (!live) return;
    float out[kD / 32];
    ln_row_vals(av, b + (size_t)r * kD, false, gv, bv, eps, lane, out);
#pragma unroll
    for (int t = 0; t < kD / 32; ++t) y[(size_t)r * kD + lane + 32 * t] = out[t];
    quant_row512_strided(out, lane, qtype, qo, (size_t)r);
}

void residual_layernorm(int T, const float* a, const float* b, const float* g, const float* beta, float eps, float* y,
                        int qtype, ActQ qo, cudaStream_t st) {
    if (T > 0) launch_k(k_residual_ln, dim3((T + 3) / 4), dim3(128), 0, st, T, a, b, g, beta, eps, y, qtype, qo);
}

// Greedy token over penalised logits (block.cpp:117-138 repetition penalty as masked lerps,
// then the first index of the maximum = sorted_indices[0] of the descending argsort).
__global__ void k_sample_greedy(const float* __restrict__ logits, int V, const int32_t* __restrict__ row_slot,
                                const uint8_t* __restrict__ seen, float rp, float inv_rp, int eos_mask, int eos,
                                int32_t* __restrict__ tok_out, int32_t* __restrict__ greedy_out) {
    pdl_wait();
    pdl_trigger();
    __shared__ float s_v[8];
    __shared__ int s_i[8];
    const int r = blockIdx.x;
    const float* lg = logits + (size_t)r * V;
    const uint8_t* sn = seen ? seen + (size_t)row_slot[r] * V : nullptr;
    float best = __int_as_float(0xff800000);
    int bi = 0x7fffffff;
    for (int v = threadIdx.x; v < V; v += blockDim.x) {
        float l = lg[v];
        if (sn && rp != 1.0f) {
            const float pos = __fmul_rn(l, inv_rp), neg = __fmul_rn(l, rp);
            const float negm = (-l > 0.0f) ? 1.0f : 0.0f;
            const float sel = __fadd_rn(pos, __fmul_rn(negm, __fsub_rn(neg, pos)));
            const float s = sn[v] ? 1.0f : 0.0f;
            l = __fadd_rn(l, __fmul_rn(s, __fsub_rn(sel, l)));
        }
        if (eos_mask && v == eos) l = kEosMasked;
        if (l > best || bi == 0x7fffffff) { best = l; bi = v; }
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    if (lane == 0) { s_v[warp] = best; s_i[warp] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
            if (s_v[w] > best || (s_v[w] == best && s_i[w] < bi)) { best = s_v[w]; bi = s_i[w]; }
        tok_out[r] = bi;
        if (greedy_out) greedy_out[r] = bi;
    }
}

// ---- full sampler chain (block.cpp:52-115, 191-271) ----------------------------------------
// One CTA of 1024 threads per row: repetition penalty, descending argsort of the 1025 logits by a
// bitonic network over 2048 (key, index) pairs (ties by lower index; padding sorts last), then in
// sorted order: top-p (softmax, sequential f32 cumsum, first position above the threshold kept),
// temperature, top-k by pivot, softmax, argmax of probs / noise (noise indexed by sorted position).
constexpr int kSortN = 2048;

__device__ void softmax_block(float* s, float* p, int n, double* s_lane, float* s_scalar) {
    const int tid = threadIdx.x;
    const float mx = s[0];   // rows are sorted in descending order and filters keep position 0
    for (int i = tid; i < n; i += blockDim.x) p[i] = t2s_expf(__fsub_rn(s[i], mx));
    __syncthreads();
    if (tid < 32) {
        double acc = 0.0;
        for (int i = tid; i < n; i += 32) acc = __dadd_rn(acc, (double)p[i]);
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) acc = __dadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
        if (tid == 0) s_scalar[0] = __double2float_rn(__ddiv_rn(1.0, acc));
    }
    __syncthreads();
    const float inv = s_scalar[0];
    for (int i = tid; i < n; i += blockDim.x) p[i] = __fmul_rn(p[i], inv);
    __syncthreads();
}

__global__ void __launch_bounds__(1024) k_sample_full(const float* __restrict__ logits, int V,
                                                      const int32_t* __restrict__ row_slot,
                                                      const uint8_t* __restrict__ seen, SamplerArgs a,
                                                      int32_t* __restrict__ tok_out, int32_t* __restrict__ greedy_out) {
    pdl_wait();
    pdl_trigger();
    __shared__ float key[kSortN];
    __shared__ int idx[kSortN];
    __shared__ float prob[kSortN];
    __shared__ double s_lane[32];
    __shared__ float s_scalar[2];
    __shared__ int s_cut;
    __shared__ float s_bv[32];
    __shared__ int s_bi[32];
    const int r = blockIdx.x, tid = threadIdx.x;
    const float* lg = logits + (size_t)r * V;
    const uint8_t* sn = seen ? seen + (size_t)row_slot[r] * V : nullptr;
    for (int i = tid; i < kSortN; i += blockDim.x) {
        float l = __int_as_float(0xff800000);
        int id = 0x7fffffff;
        if (i < V) {
            l = lg[i];
            if (sn && a.rp != 1.0f) {
                const float pos = __fmul_rn(l, a.inv_rp), neg = __fmul_rn(l, a.rp);
                const float negm = (-l > 0.0f) ? 1.0f : 0.0f;
                const float sel = __fadd_rn(pos, __fmul_rn(negm, __fsub_rn(neg, pos)));
                const float sv = sn[i] ? 1.0f : 0.0f;
                l = __fadd_rn(l, __fmul_rn(sv, __fsub_rn(sel, l)));
            }
            if (a.eos_mask && i == a.eos) l = kEosMasked;
            id = i;
        }
        key[i] = l;
        idx[i] = id;
    }
    __syncthreads();
    // bitonic sort, descending by key, ascending by index on equal keys
    for (int k = 2; k <= kSortN; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int t = tid; t < kSortN / 2; t += blockDim.x) {
                const int i = 2 * t - (t & (j - 1));
                const int p = i + j;
                const float ki = key[i], kp = key[p];
                const int ii = idx[i], ip = idx[p];
                const bool i_first = (ki > kp) || (ki == kp && ii < ip);
                const bool desc = (i & k) == 0;
                if (desc != i_first) { key[i] = kp; key[p] = ki; idx[i] = ip; idx[p] = ii; }
            }
            __syncthreads();
        }
    }
    if (tid == 0) greedy_out[r] = idx[0];
    if (!a.noise) {
        if (tid == 0) tok_out[r] = idx[0];
        return;
    }
    float* s = key;
    if (a.top_p < 1.0f && V > 1) {
        softmax_block(s, prob, V, s_lane, s_scalar);
        if (tid == 0) {
            float cum = 0.0f;
            int cut = V;
            for (int i = 0; i < V; ++i) {
                cum = __fadd_rn(cum, prob[i]);
                if (__fsub_rn(cum, a.top_p) > 0.0f) { cut = i + 1; break; }
            }
            s_cut = cut;
        }
        __syncthreads();
        for (int i = s_cut + tid; i < V; i += blockDim.x) s[i] = __fadd_rn(s[i], __fsub_rn(-1.0e10f, s[i]));
        __syncthreads();
    }
    for (int i = tid; i < V; i += blockDim.x) s[i] = __fmul_rn(s[i], a.inv_t);
    __syncthreads();
    if (a.top_k > 0 && a.top_k < V) {
        const float pivot = s[a.top_k - 1];
        __syncthreads();
        for (int i = tid; i < V; i += blockDim.x)
            if (__fsub_rn(pivot, s[i]) > 0.0f) s[i] = __fadd_rn(s[i], __fsub_rn(-1.0e10f, s[i]));
        __syncthreads();
    }
    softmax_block(s, prob, V, s_lane, s_scalar);
    const float* nz = a.noise + (size_t)r * V;
    float bv = 0.0f;
    int bi = 0x7fffffff;
    for (int i = tid; i < V; i += blockDim.x) {
        const float sc = __fdiv_rn(prob[i], nz[i]);
        if (bi == 0x7fffffff || sc > bv) { bv = sc; bi = i; }
    }
    const int lane = tid & 31, warp = tid >> 5;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (oi != 0x7fffffff && (bi == 0x7fffffff || ov > bv || (ov == bv && oi < bi))) { bv = ov; bi = oi; }
    }
    if (lane == 0) { s_bv[warp] = bv; s_bi[warp] = bi; }
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
            if (s_bi[w] != 0x7fffffff && (bi == 0x7fffffff || s_bv[w] > bv || (s_bv[w] == bv && s_bi[w] < bi))) {
                bv = s_bv[w];
                bi = s_bi[w];
            }
        tok_out[r] = idx[bi];
    }
}

void sample_greedy(int T, const float* logits, int V, const int32_t* row_slot, const uint8_t* seen, float rp,
                   float inv_rp, int eos_mask, int eos, int32_t* tok_out, int32_t* greedy_out, cudaStream_t st) {
    if (T > 0) launch_k(k_sample_greedy, dim3(T), dim3(256), 0, st, logits, V, row_slot, seen, rp, inv_rp, eos_mask, eos, tok_out, greedy_out);
}

void sample_full(int T, const float* logits, int V, const int32_t* row_slot, const uint8_t* seen, const SamplerArgs& a,
                 int32_t* tok_out, int32_t* greedy_out, cudaStream_t st) {
    if (T > 0) launch_k(k_sample_full, dim3(T), dim3(1024), 0, st, logits, V, row_slot, seen, a, tok_out, greedy_out);
}

// End of a decode step (session.cpp:247-284 on the device): feed the sampled token back,
// advance n_pos, mark the token as seen, append it to the device token ring.
__global__ void k_advance(int T, const int32_t* __restrict__ row_slot, const int32_t* __restrict__ tok,
                          int32_t* __restrict__ token_in, int32_t* __restrict__ n_pos, uint8_t* __restrict__ seen, int V,
                          int32_t* __restrict__ ring, int ring_len, int32_t* __restrict__ ring_step) {
    pdl_wait();
    pdl_trigger();
    const int step = *ring_step;
    for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < T; r += gridDim.x * blockDim.x) {
        const int s = row_slot[r];
        const int t = tok[r];
        token_in[s] = t;
        n_pos[s] += 1;
        if (seen && t >= 0 && t < V) seen[(size_t)s * V + t] = 1;
        if (ring) ring[(size_t)(step % ring_len) * T + r] = t;
    }
}

__global__ void k_step_inc(int32_t* ring_step) {
    pdl_wait();
    pdl_trigger(); *ring_step += 1; }

void advance(int T, const int32_t* row_slot, const int32_t* tok, int32_t* token_in, int32_t* n_pos, uint8_t* seen,
             int V, int32_t* ring, int ring_len, int32_t* ring_step, cudaStream_t st) {
    if (T > 0) launch_k(k_advance, dim3((T + 255) / 256), dim3(256), 0, st, T, row_slot, tok, token_in, n_pos, seen, V, ring, ring_len, ring_step);
    launch_k(k_step_inc, dim3(1), dim3(1), 0, st, ring_step);
}

__global__ void k_gather_rows(int n, const float* __restrict__ src, const int32_t* __restrict__ idx, int ld,
                              float* __restrict__ dst) {
    pdl_wait();
    pdl_trigger();
    const int r = blockIdx.x;
    if (r >= n) return;
    for (int c = threadIdx.x; c < ld; c += blockDim.x) dst[(size_t)r * ld + c] = src[(size_t)idx[r] * ld + c];
}

void gather_rows(int n, const float* src, const int32_t* idx, int ld, float* dst, cudaStream_t st) {
    if (n > 0) launch_k(k_gather_rows, dim3(n), dim3(128), 0, st, n, src, idx, ld, dst);
}

// Prefill input rows (block.cpp:424-468): text row t = (emb_t + bert_proj_t) + pe[t]*alpha_t,
// audio row t = emb_a + pe[t]*alpha_a.  bert_proj already holds W*bert + b.
__global__ void k_embed_prefill(int T_text, int T_prompt, const int32_t* __restrict__ phones,
                                const int32_t* __restrict__ sem, const float* __restrict__ bert_proj,
                                const uint16_t* __restrict__ text16, const float* __restrict__ text32,
                                const uint16_t* __restrict__ audio16, const float* __restrict__ audio32,
                                const float* __restrict__ pe, float alpha_t, float alpha_a, float* __restrict__ x) {
    pdl_wait();
    pdl_trigger();
    const int r = blockIdx.x;
    for (int d = threadIdx.x; d < kD; d += blockDim.x) {
        float v;
        if (r < T_text) {
            const int id = phones[r];
            const float e = text16 ? h2f(text16[(size_t)id * kD + d]) : text32[(size_t)id * kD + d];
            v = __fadd_rn(__fadd_rn(e, bert_proj[(size_t)r * kD + d]), __fmul_rn(pe[(size_t)r * kD + d], alpha_t));
        } else {
            const int t = r - T_text;
            const int id = sem[t];
            const float e = audio16 ? h2f(audio16[(size_t)id * kD + d]) : audio32[(size_t)id * kD + d];
            v = __fadd_rn(e, __fmul_rn(pe[(size_t)t * kD + d], alpha_a));
        }
        x[(size_t)r * kD + d] = v;
    }
}

void embed_prefill_rows(int T_text, int T_prompt, const int32_t* phones, const int32_t* sem, const float* bert_proj,
                        const uint16_t* text16, const float* text32, const uint16_t* audio16, const float* audio32,
                        const float* pe, float alpha_t, float alpha_a, float* x, cudaStream_t st) {
    const int T = T_text + T_prompt;
    if (T > 0)
        launch_k(k_embed_prefill, dim3(T), dim3(128), 0, st, T_text, T_prompt, phones, sem, bert_proj, text16, text32, audio16, audio32, pe,
                                           alpha_t, alpha_a, x);
}

}  // namespace t2sx

namespace t2sx {

// ============================================================================================
// extract-latent (sovits_extract_latent_block_forward, src/t2s/block.cpp:140-189)
// ============================================================================================

// im2col of the width-2, stride-2 Conv1d: cols[t][ic * 2 + k] = x[2t + k][ic] (ggml_im2col order,
// kernel tap fastest)
__global__ void k_im2col_k2s2(int To, int C, const float* __restrict__ x, float* __restrict__ cols) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)To * C * 2) return;
    const int64_t t = i / (2 * C);
    const int j = (int)(i % (2 * C)), ic = j >> 1, k = j & 1;
    cols[i] = x[(2 * t + k) * C + ic];
}

// codes[t] = first index c of the max of score[t][c] - half_norm[c] (ggml_sub, ggml_argmax); one
// warp per frame: lanes scan c = lane, lane + 32, ... keeping their first maximum, then the
// warp keeps the larger value and, on equal values, the smaller index.
__global__ void k_code_argmax(int To, int NC, const float* __restrict__ score, const float* __restrict__ half_norm,
                              int32_t* __restrict__ codes) {
    const int lane = threadIdx.x & 31;
    const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (t >= To) return;
    float bv = __int_as_float(0xff800000);
    int bi = 0x7fffffff;
    for (int c = lane; c < NC; c += 32) {
        const float v = __fsub_rn(score[(size_t)t * NC + c], half_norm[c]);
        if (v > bv || bi == 0x7fffffff) { bv = v; bi = c; }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) codes[t] = bi;
}

void im2col_k2s2(int To, int C, const float* x, float* cols, cudaStream_t st) {
    const int64_t n = (int64_t)To * C * 2;
    if (n > 0) k_im2col_k2s2<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(To, C, x, cols);
}

void code_argmax(int To, int NC, const float* score, const float* half_norm, int32_t* codes, cudaStream_t st) {
    if (To > 0) k_code_argmax<<<(To + 3) / 4, 128, 0, st>>>(To, NC, score, half_norm, codes);
}

}  // namespace t2sx
