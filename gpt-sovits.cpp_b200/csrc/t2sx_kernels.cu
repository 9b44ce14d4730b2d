// CUDA kernels of the T2S decode path for sm_100a.
//
// Arithmetic follows the reference's ggml CPU operators (src/t2s/block.cpp:513-637 layer,
// :117-348 sampler, src/t2s/session.cpp:337-344 decode embedding) with one fixed evaluation
// order per reduction; see t2sx_math.cuh.  Built with --fmad=false.
#include "t2sx_kernels.cuh"
#include "t2sx_math.cuh"

namespace t2sx {

// ============================================================================================
// activation quantisation
// ============================================================================================

// Q8_0 (x86 AVX2 rule of ggml quantize_row_q8_0): one warp per 32-element block.
__global__ void k_quant_q8_0(const float* __restrict__ x, int64_t nblk, int8_t* __restrict__ q,
                             float* __restrict__ d) {
    const int lane = threadIdx.x & 31;
    const int64_t wstride = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t b = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; b < nblk; b += wstride) {
        const float v = x[b * 32 + lane];
        float a = fabsf(v);
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, off));
        const float dd = __fdiv_rn(a, 127.0f);
        const float id = (a != 0.0f) ? __fdiv_rn(127.0f, a) : 0.0f;
        float r = rintf(__fmul_rn(v, id));
        r = fminf(fmaxf(r, -128.0f), 127.0f);
        q[b * 32 + lane] = (int8_t)(int)r;
        if (lane == 0) d[b] = __half2float(__float2half_rn(dd));
    }
}

// Q8_K (ggml quantize_row_q8_K_ref rule): one warp per 256-element block, 8 elements per lane.
__global__ void k_quant_q8_K(const float* __restrict__ x, int64_t nblk, int8_t* __restrict__ q,
                             float* __restrict__ d, int32_t* __restrict__ bs) {
    const int lane = threadIdx.x & 31;
    const int64_t wstride = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t b = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; b < nblk; b += wstride) {
        const float4* xp = reinterpret_cast<const float4*>(x + b * 256 + lane * 8);
        const float4 x0 = xp[0], x1 = xp[1];
        const float v[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
        float amax = 0.0f, mx = 0.0f;
        int idx = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float a = fabsf(v[i]);
            if (a > amax) { amax = a; mx = v[i]; idx = lane * 8 + i; }
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
            const float oa = __shfl_xor_sync(0xffffffffu, amax, off);
            const float om = __shfl_xor_sync(0xffffffffu, mx, off);
            const int oi = __shfl_xor_sync(0xffffffffu, idx, off);
            if (oa > amax || (oa == amax && oi < idx)) { amax = oa; mx = om; idx = oi; }
        }
        int8_t qv[8];
        int sum = 0;
        if (amax == 0.0f) {
#pragma unroll
            for (int i = 0; i < 8; ++i) qv[i] = 0;
        } else {
            const float iscale = __fdiv_rn(-127.0f, mx);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float r = rintf(__fmul_rn(iscale, v[i]));
                const int iv = r > 127.0f ? 127 : (int)r;
                qv[i] = (int8_t)iv;
                sum += iv;
            }
            if (lane == 0) d[b] = __fdiv_rn(1.0f, iscale);
        }
        if (amax == 0.0f && lane == 0) d[b] = 0.0f;
        int2 packed;
        packed.x = (qv[0] & 0xff) | ((qv[1] & 0xff) << 8) | ((qv[2] & 0xff) << 16) | ((qv[3] & 0xff) << 24);
        packed.y = (qv[4] & 0xff) | ((qv[5] & 0xff) << 8) | ((qv[6] & 0xff) << 16) | ((qv[7] & 0xff) << 24);
        *reinterpret_cast<int2*>(q + b * 256 + lane * 8) = packed;
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        if ((lane & 3) == 0) bs[b * 8 + (lane >> 2)] = sum;
    }
}

__global__ void k_quant_f16(const float* __restrict__ x, int64_t n, uint16_t* __restrict__ h) {
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
        k_quant_q8_0<<<grid_for(n / 32, 8), 256, 0, st>>>(x, n / 32, a.q, a.d);
    } else if (wtype == W_Q4_K) {
        k_quant_q8_K<<<grid_for(n / 256, 8), 256, 0, st>>>(x, n / 256, a.q, a.d, a.bs);
    } else if (wtype == W_F16) {
        k_quant_f16<<<grid_for(n, 256), 256, 0, st>>>(x, n, a.h);
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

// Small-M kernel: one warp per weight row; lanes compute block partials (phase A) into shared
// memory, then lane m runs the ordered chain of row m (phase B).
template <int WT>
__global__ void __launch_bounds__(128) k_mm_small(DevW W, ActQ A, int M, const float* __restrict__ bias, int relu,
                                                  float* __restrict__ y) {
    __shared__ int s_a[4][kSmallM][64];
    __shared__ int s_m[4][kSmallM][8];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = blockIdx.x * 4 + warp;
    if (n >= W.N) return;
    const int K = W.K;
    if (WT == W_Q8_0 || WT == W_Q4_0) {
        const int nb = K / 32;
        for (int b = lane; b < nb; b += 32) {
            int4 w0, w1;
            if (WT == W_Q8_0) {
                const int4* wp = reinterpret_cast<const int4*>(W.q8 + (size_t)n * K + b * 32);
                w0 = wp[0]; w1 = wp[1];
            } else {
                const int4 raw = *reinterpret_cast<const int4*>(W.q4 + ((size_t)n * nb + b) * 16);
                w0 = make_int4(q4lo(raw.x), q4lo(raw.y), q4lo(raw.z), q4lo(raw.w));
                w1 = make_int4(q4hi(raw.x), q4hi(raw.y), q4hi(raw.z), q4hi(raw.w));
            }
            for (int m = 0; m < M; ++m) {
                const int4* xp = reinterpret_cast<const int4*>(A.q + (size_t)m * K + b * 32);
                s_a[warp][m][b] = dp8(w0, w1, xp[0], xp[1]);
            }
        }
        __syncwarp();
        if (lane < M) {
            const int m = lane;
            float acc = 0.0f;
            for (int b = 0; b < nb; ++b) {
                const float dd = __fmul_rn(W.d[(size_t)n * nb + b], A.d[(size_t)m * nb + b]);
                acc = __fmaf_rn(dd, (float)s_a[warp][m][b], acc);
            }
            y[(size_t)m * W.N + n] = epi(acc, bias, n, relu);
        }
    } else if (WT == W_Q4_K) {
        const int nsub = K / 32, nsb = K / 256;
        for (int t = 0; t < (nsub + 31) / 32; ++t) {
            const int j = lane + 32 * t;
            const bool act = j < nsub;
            const int sb = j >> 3, js = j & 7, c = js >> 1, hi = js & 1;
            int4 w0 = make_int4(0, 0, 0, 0), w1 = w0;
            int sc = 0, mn = 0;
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
            }
            for (int m = 0; m < M; ++m) {
                int sa = 0, sm = 0;
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
                if (act && js == 0) { s_a[warp][m][sb] = sa; s_m[warp][m][sb] = sm; }
            }
        }
        __syncwarp();
        if (lane < M) {
            const int m = lane;
            float acc_a = 0.0f, acc_m = 0.0f;
            for (int sb = 0; sb < nsb; ++sb) {
                const float dx = A.d[(size_t)m * nsb + sb];
                const float dd = __fmul_rn(dx, W.d[(size_t)n * nsb + sb]);
                const float dm = __fmul_rn(-dx, W.dmin[(size_t)n * nsb + sb]);
                acc_a = __fmaf_rn(dd, (float)s_a[warp][m][sb], acc_a);
                acc_m = __fmaf_rn(dm, (float)s_m[warp][m][sb], acc_m);
            }
            y[(size_t)m * W.N + n] = epi(__fadd_rn(acc_a, acc_m), bias, n, relu);
        }
    } else {  // F16 / F32
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
                s_a[warp][m][b] = __float_as_int(s);
            }
        }
        __syncwarp();
        if (lane < M) {
            const int m = lane;
            float acc = 0.0f;
            for (int b = 0; b < nb; ++b) acc = __fadd_rn(acc, __int_as_float(s_a[warp][m][b]));
            y[(size_t)m * W.N + n] = epi(acc, bias, n, relu);
        }
    }
}

// Tiled kernel for larger M: 64 weight rows x 64 activation rows per CTA, 256 threads, each a
// 4x4 register tile; K staged 4 blocks (128 elements) at a time.  Same canonical order.
template <int WT>
__global__ void __launch_bounds__(256) k_mm_tiled(DevW W, ActQ A, int M, const float* __restrict__ bias, int relu,
                                                  float* __restrict__ y) {
    constexpr int KB = 4;
    __shared__ int4 sW4[KB * 8][16];   // [k-word][n/4]
    __shared__ int4 sX4[KB * 8][16];   // [k-word][m/4]
    __shared__ float sDw[KB][64], sDx[KB][64];
    __shared__ float sDw2[64], sDm2[64], sDx2[64];
    __shared__ int sSc[KB][64], sMn[KB][64], sBs[KB][64];
    int* sW = reinterpret_cast<int*>(sW4);
    int* sX = reinterpret_cast<int*>(sX4);
    const int tid = threadIdx.x, tn = tid & 15, tm = tid >> 4;
    const int n0 = blockIdx.x * 64, m0 = blockIdx.y * 64;
    const int K = W.K, N = W.N;
    float acc[4][4], acc_m[4][4];
    int sa[4][4], smi[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) { acc[i][j] = 0.0f; acc_m[i][j] = 0.0f; sa[i][j] = 0; smi[i][j] = 0; }
    const int nstage = K / (32 * KB);
    for (int stg = 0; stg < nstage; ++stg) {
        const int kb0 = stg * KB;  // first 32-block of the stage
        // ---- stage weights ----
        for (int idx = tid; idx < 64 * KB; idx += 256) {
            const int row = idx & 63, blk = idx >> 6, n = n0 + row, b = kb0 + blk;
            int4 w0 = make_int4(0, 0, 0, 0), w1 = w0;
            if (n < N) {
                if (WT == W_Q8_0) {
                    const int4* wp = reinterpret_cast<const int4*>(W.q8 + (size_t)n * K + b * 32);
                    w0 = wp[0]; w1 = wp[1];
                } else if (WT == W_Q4_0) {
                    const int4 raw = *reinterpret_cast<const int4*>(W.q4 + ((size_t)n * (K / 32) + b) * 16);
                    w0 = make_int4(q4lo(raw.x), q4lo(raw.y), q4lo(raw.z), q4lo(raw.w));
                    w1 = make_int4(q4hi(raw.x), q4hi(raw.y), q4hi(raw.z), q4hi(raw.w));
                } else {  // Q4_K: sub-block b of the row
                    const int sb = b >> 3, js = b & 7, c = js >> 1, hi = js & 1;
                    const int4* wp = reinterpret_cast<const int4*>(W.q4 + ((size_t)n * (K / 256) + sb) * 128 + 32 * c);
                    const int4 r0 = wp[0], r1 = wp[1];
                    const int sh = hi ? 4 : 0;
                    w0 = make_int4((r0.x >> sh) & 0x0F0F0F0F, (r0.y >> sh) & 0x0F0F0F0F, (r0.z >> sh) & 0x0F0F0F0F, (r0.w >> sh) & 0x0F0F0F0F);
                    w1 = make_int4((r1.x >> sh) & 0x0F0F0F0F, (r1.y >> sh) & 0x0F0F0F0F, (r1.z >> sh) & 0x0F0F0F0F, (r1.w >> sh) & 0x0F0F0F0F);
                }
            }
            sW[(blk * 8 + 0) * 64 + row] = w0.x; sW[(blk * 8 + 1) * 64 + row] = w0.y;
            sW[(blk * 8 + 2) * 64 + row] = w0.z; sW[(blk * 8 + 3) * 64 + row] = w0.w;
            sW[(blk * 8 + 4) * 64 + row] = w1.x; sW[(blk * 8 + 5) * 64 + row] = w1.y;
            sW[(blk * 8 + 6) * 64 + row] = w1.z; sW[(blk * 8 + 7) * 64 + row] = w1.w;
            if (WT == W_Q4_K) {
                const int sb = b >> 3, js = b & 7;
                sSc[blk][row] = n < N ? W.scm[((size_t)n * (K / 256) + sb) * 16 + js] : 0;
                sMn[blk][row] = n < N ? W.scm[((size_t)n * (K / 256) + sb) * 16 + 8 + js] : 0;
            } else {
                sDw[blk][row] = n < N ? W.d[(size_t)n * (K / 32) + b] : 0.0f;
            }
        }
        // ---- stage activations ----
        for (int idx = tid; idx < 64 * KB; idx += 256) {
            const int row = idx & 63, blk = idx >> 6, m = m0 + row, b = kb0 + blk;
            int4 x0 = make_int4(0, 0, 0, 0), x1 = x0;
            if (m < M) {
                const int4* xp = reinterpret_cast<const int4*>(A.q + (size_t)m * K + b * 32);
                x0 = xp[0]; x1 = xp[1];
            }
            sX[(blk * 8 + 0) * 64 + row] = x0.x; sX[(blk * 8 + 1) * 64 + row] = x0.y;
            sX[(blk * 8 + 2) * 64 + row] = x0.z; sX[(blk * 8 + 3) * 64 + row] = x0.w;
            sX[(blk * 8 + 4) * 64 + row] = x1.x; sX[(blk * 8 + 5) * 64 + row] = x1.y;
            sX[(blk * 8 + 6) * 64 + row] = x1.z; sX[(blk * 8 + 7) * 64 + row] = x1.w;
            if (WT == W_Q4_K) sBs[blk][row] = m < M ? A.bs[(size_t)m * (K / 32) + b] : 0;
            else sDx[blk][row] = m < M ? A.d[(size_t)m * (K / 32) + b] : 0.0f;
        }
        if (WT == W_Q4_K && (kb0 & 7) == 0 && tid < 64) {
            const int n = n0 + tid, m = m0 + tid, sb = kb0 >> 3;
            sDw2[tid] = n < N ? W.d[(size_t)n * (K / 256) + sb] : 0.0f;
            sDm2[tid] = n < N ? W.dmin[(size_t)n * (K / 256) + sb] : 0.0f;
            sDx2[tid] = m < M ? A.d[(size_t)m * (K / 256) + sb] : 0.0f;
        }
        __syncthreads();
        // ---- compute ----
#pragma unroll
        for (int blk = 0; blk < KB; ++blk) {
            int is[4][4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) is[i][j] = 0;
#pragma unroll
            for (int w = 0; w < 8; ++w) {
                const int4 a = sW4[blk * 8 + w][tn];
                const int4 b = sX4[blk * 8 + w][tm];
                const int av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) is[i][j] = __dp4a(av[i], bv[j], is[i][j]);
            }
            if (WT == W_Q4_K) {
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        sa[i][j] += sSc[blk][4 * tn + i] * is[i][j];
                        smi[i][j] += sMn[blk][4 * tn + i] * sBs[blk][4 * tm + j];
                    }
            } else {
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float dd = __fmul_rn(sDw[blk][4 * tn + i], sDx[blk][4 * tm + j]);
                        acc[i][j] = __fmaf_rn(dd, (float)is[i][j], acc[i][j]);
                    }
            }
        }
        if (WT == W_Q4_K && ((kb0 + KB) & 7) == 0) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float dx = sDx2[4 * tm + j];
                    const float dd = __fmul_rn(dx, sDw2[4 * tn + i]);
                    const float dm = __fmul_rn(-dx, sDm2[4 * tn + i]);
                    acc[i][j] = __fmaf_rn(dd, (float)sa[i][j], acc[i][j]);
                    acc_m[i][j] = __fmaf_rn(dm, (float)smi[i][j], acc_m[i][j]);
                    sa[i][j] = 0; smi[i][j] = 0;
                }
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int n = n0 + 4 * tn + i;
        if (n >= N) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int m = m0 + 4 * tm + j;
            if (m >= M) continue;
            const float r = (WT == W_Q4_K) ? __fadd_rn(acc[i][j], acc_m[i][j]) : acc[i][j];
            y[(size_t)m * N + n] = epi(r, bias, n, relu);
        }
    }
}

void matmul(const DevW& W, const ActQ& a, int M, const float* bias, int relu, float* y, cudaStream_t st) {
    const bool quant = W.type == W_Q8_0 || W.type == W_Q4_0 || W.type == W_Q4_K;
    if (quant && M > kSmallM && matmul_mma(W, a, M, bias, relu, y, st)) return;
    if (quant && M > kSmallM) {
        dim3 grid((W.N + 63) / 64, (M + 63) / 64);
        switch (W.type) {
            case W_Q8_0: k_mm_tiled<W_Q8_0><<<grid, 256, 0, st>>>(W, a, M, bias, relu, y); break;
            case W_Q4_0: k_mm_tiled<W_Q4_0><<<grid, 256, 0, st>>>(W, a, M, bias, relu, y); break;
            case W_Q4_K: k_mm_tiled<W_Q4_K><<<grid, 256, 0, st>>>(W, a, M, bias, relu, y); break;
        }
        return;
    }
    for (int m0 = 0; m0 < M; m0 += kSmallM) {
        const int mm = (M - m0) < kSmallM ? (M - m0) : kSmallM;
        ActQ as = a;
        const int K = W.K;
        if (as.q) as.q += (size_t)m0 * K;
        if (as.h) as.h += (size_t)m0 * K;
        if (as.f) as.f += (size_t)m0 * K;
        if (as.d) as.d += (size_t)m0 * (W.type == W_Q4_K ? K / 256 : K / 32);
        if (as.bs) as.bs += (size_t)m0 * (K / 32);
        float* yy = y + (size_t)m0 * W.N;
        const int grid = (W.N + 3) / 4;
        switch (W.type) {
            case W_Q8_0: k_mm_small<W_Q8_0><<<grid, 128, 0, st>>>(W, as, mm, bias, relu, yy); break;
            case W_Q4_0: k_mm_small<W_Q4_0><<<grid, 128, 0, st>>>(W, as, mm, bias, relu, yy); break;
            case W_Q4_K: k_mm_small<W_Q4_K><<<grid, 128, 0, st>>>(W, as, mm, bias, relu, yy); break;
            case W_F16: k_mm_small<W_F16><<<grid, 128, 0, st>>>(W, as, mm, bias, relu, yy); break;
            default: k_mm_small<W_F32><<<grid, 128, 0, st>>>(W, as, mm, bias, relu, yy); break;
        }
    }
}

// ============================================================================================
// embedding, KV append, attention, LayerNorm, sampler
// ============================================================================================

// Decode embedding (session.cpp:337-344): x = emb[tok] + pe[n_pos - audio_offset] * alpha.
// Also fixes the row's KV position (n_pos) and attended length (n_pos + 1).
__global__ void k_embed_decode(const int32_t* __restrict__ row_slot, const int32_t* __restrict__ token_in,
                               const int32_t* __restrict__ n_pos, const int32_t* __restrict__ audio_off,
                               const uint16_t* __restrict__ emb16, const float* __restrict__ emb32,
                               int emb_rows, const float* __restrict__ pe, int pe_rows, float alpha, Rows rows,
                               float* __restrict__ x) {
    const int r = blockIdx.x;
    const int s = row_slot[r];
    const int pos = n_pos[s];
    const int pp = pos - audio_off[s];
    const int tok = token_in[s];
    const bool ok = pos >= 0 && pos < rows.cap[s] && pp >= 0 && pp < pe_rows && tok >= 0 && tok < emb_rows;
    if (threadIdx.x == 0) {
        rows.pos[r] = ok ? pos : -1;
        rows.L[r] = ok ? pos + 1 : 0;
        if (!ok) atomicExch(rows.err, 1);
    }
    for (int d = threadIdx.x; d < kD; d += blockDim.x) {
        float v = 0.0f;
        if (ok) {
            const float e = emb16 ? h2f(emb16[(size_t)tok * kD + d]) : emb32[(size_t)tok * kD + d];
            v = __fadd_rn(e, __fmul_rn(pe[(size_t)pp * kD + d], alpha));
        }
        x[(size_t)r * kD + d] = v;
    }
}

void embed_decode(int T, const int32_t* row_slot, const int32_t* token_in, const int32_t* n_pos,
                  const int32_t* audio_off, const uint16_t* emb16, const float* emb32, int emb_rows, const float* pe,
                  int pe_rows, float alpha, Rows rows, float* x, cudaStream_t st) {
    if (T > 0)
        k_embed_decode<<<T, 128, 0, st>>>(row_slot, token_in, n_pos, audio_off, emb16, emb32, emb_rows, pe, pe_rows, alpha,
                                          rows, x);
}

__device__ __forceinline__ size_t kv_off(const KVView& kv, int page, int layer, int which, int head, int pos_in_page) {
    return (((((size_t)page * kv.n_layer + layer) * 2 + which) * kHeads + head) * kPage + pos_in_page) * kHeadDim;
}

// Split the QKV projection: Q -> f16 for attention, K and V -> f16 into the paged cache
// (ggml_set_rows into an F16 cache, block.cpp:557-573).
__global__ void k_qkv_post(const float* __restrict__ qkv, Rows rows, KVView kv, int layer, uint16_t* __restrict__ q16) {
    const int r = blockIdx.x;
    const int s = rows.slot[r];
    const int pos = rows.pos[r];
    const bool ok = pos >= 0 && pos < rows.cap[s];
    const int page = ok ? kv.ptab[(size_t)s * kv.max_pages + (pos / kPage)] : -1;
    for (int i = threadIdx.x; i < 3 * kD; i += blockDim.x) {
        const uint16_t h = f2h(qkv[(size_t)r * 3 * kD + i]);
        if (i < kD) { q16[(size_t)r * kD + i] = h; continue; }
        if (page < 0) continue;
        const int which = (i - kD) / kD, j = (i - kD) % kD;
        kv.pool[kv_off(kv, page, layer, which, j / kHeadDim, pos % kPage) + (j % kHeadDim)] = h;
    }
}

void qkv_post(int T, const float* qkv, Rows rows, KVView kv, int layer, uint16_t* q16, cudaStream_t st) {
    if (T > 0) k_qkv_post<<<T, 256, 0, st>>>(qkv, rows, kv, layer, q16);
}

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

// Decode attention: one warp per (row, head), four heads of a row per CTA.  Position lane
// t = lane folds positions t, t+32, ... with the online update; the 32 lanes merge in the
// order of an xor butterfly (partners 16, 8, 4, 2, 1).  The merge is symmetric, so every lane
// ends with the same state and lane d writes output dim d.
__global__ void __launch_bounds__(128) k_attn_decode(const uint16_t* __restrict__ q16, Rows rows, KVView kv, int layer,
                                                     float scale, float* __restrict__ out) {
    const int r = blockIdx.x;
    const int h = blockIdx.y * 4 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    const int s = rows.slot[r];
    const int L = rows.L[r];
    float q[kHeadDim];
    load_row32(q16 + (size_t)r * kD + h * kHeadDim, q);
    AttnState st;
    st_empty(st);
    const int32_t* pt = kv.ptab + (size_t)s * kv.max_pages;
    for (int i = lane; i < L; i += kAttnLanes) {
        const int page = pt[i / kPage];
        const size_t kb = kv_off(kv, page, layer, 0, h, i % kPage);
        const size_t vb = kv_off(kv, page, layer, 1, h, i % kPage);
        float k[kHeadDim], v[kHeadDim];
        load_row32(kv.pool + kb, k);
        load_row32(kv.pool + vb, v);
        const float sc = __fmul_rn(dot32(q, k), scale);
        st_update(st, sc, v);
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        const float mB = __shfl_xor_sync(0xffffffffu, st.m, off);
        const float lB = __shfl_xor_sync(0xffffffffu, st.l, off);
        float M, a, b, l;
        bool empty;
        st_merge_scalars(st.m, st.l, mB, lB, M, a, b, l, empty);
#pragma unroll
        for (int d = 0; d < kHeadDim; ++d) {
            const float oB = __shfl_xor_sync(0xffffffffu, st.o[d], off);
            st.o[d] = empty ? 0.0f : __fadd_rn(__fmul_rn(st.o[d], a), __fmul_rn(oB, b));
        }
        st.m = empty ? __int_as_float(0xff800000) : M;
        st.l = l;
    }
    float mine = 0.0f;
#pragma unroll
    for (int d = 0; d < kHeadDim; ++d) if (d == lane) mine = st.o[d];
    out[(size_t)r * kD + h * kHeadDim + lane] = __fmul_rn(mine, __fdiv_rn(1.0f, st.l));
}

void attention_decode(int T, const uint16_t* q16, Rows rows, KVView kv, int layer, float scale, float* out,
                      cudaStream_t st) {
    if (T > 0) k_attn_decode<<<dim3(T, kHeads / 4), 128, 0, st>>>(q16, rows, kv, layer, scale, out);
}

// Prefill attention: one thread per (row, head) folds its prefix sequentially.
__global__ void __launch_bounds__(128) k_attn_prefill(int T, const uint16_t* __restrict__ q16, Rows rows, KVView kv,
                                                      int layer, float scale, float* __restrict__ out) {
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= T * kHeads) return;
    const int r = idx / kHeads, h = idx % kHeads;
    const int s = rows.slot[r];
    const int L = rows.L[r];
    float q[kHeadDim];
    load_row32(q16 + (size_t)r * kD + h * kHeadDim, q);
    AttnState st;
    st_empty(st);
    const int32_t* pt = kv.ptab + (size_t)s * kv.max_pages;
    for (int i = 0; i < L; ++i) {
        const int page = pt[i / kPage];
        float k[kHeadDim], v[kHeadDim];
        load_row32(kv.pool + kv_off(kv, page, layer, 0, h, i % kPage), k);
        load_row32(kv.pool + kv_off(kv, page, layer, 1, h, i % kPage), v);
        st_update(st, __fmul_rn(dot32(q, k), scale), v);
    }
    const float inv = __fdiv_rn(1.0f, st.l);
#pragma unroll
    for (int d = 0; d < kHeadDim; ++d) out[(size_t)r * kD + h * kHeadDim + d] = __fmul_rn(st.o[d], inv);
}

void attention_prefill(int T, const uint16_t* q16, Rows rows, KVView kv, int layer, float scale, float* out,
                       cudaStream_t st) {
    if (T > 0) k_attn_prefill<<<(T * kHeads + 127) / 128, 128, 0, st>>>(T, q16, rows, kv, layer, scale, out);
}

// y = LN(a + b) * g + beta (ggml_norm + mul + add, block.cpp:615-619 / :630-634).  One warp per
// row; lane l sums elements l, l+32, ... in double, lanes combine by an xor butterfly.
__global__ void k_residual_ln(int T, const float* __restrict__ a, const float* __restrict__ b,
                              const float* __restrict__ g, const float* __restrict__ beta, float eps, float* __restrict__ y) {
    const int lane = threadIdx.x & 31;
    const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (r >= T) return;
    float v[kD / 32];
    double s = 0.0;
#pragma unroll
    for (int t = 0; t < kD / 32; ++t) {
        const int i = lane + 32 * t;
        v[t] = __fadd_rn(a[(size_t)r * kD + i], b[(size_t)r * kD + i]);
        s = __dadd_rn(s, (double)v[t]);
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) s = __dadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
    const float mean = __double2float_rn(__ddiv_rn(s, (double)kD));
    double s2 = 0.0;
#pragma unroll
    for (int t = 0; t < kD / 32; ++t) {
        v[t] = __fsub_rn(v[t], mean);
        s2 = __dadd_rn(s2, (double)__fmul_rn(v[t], v[t]));
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) s2 = __dadd_rn(s2, __shfl_xor_sync(0xffffffffu, s2, off));
    const float var = __double2float_rn(__ddiv_rn(s2, (double)kD));
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
#pragma unroll
    for (int t = 0; t < kD / 32; ++t) {
        const int i = lane + 32 * t;
        y[(size_t)r * kD + i] = __fadd_rn(__fmul_rn(__fmul_rn(v[t], scale), g[i]), beta[i]);
    }
}

void residual_layernorm(int T, const float* a, const float* b, const float* g, const float* beta, float eps, float* y,
                        cudaStream_t st) {
    if (T > 0) k_residual_ln<<<(T + 3) / 4, 128, 0, st>>>(T, a, b, g, beta, eps, y);
}

// Greedy token over penalised logits (block.cpp:117-138 repetition penalty as masked lerps,
// then the first index of the maximum = sorted_indices[0] of the descending argsort).
__global__ void k_sample_greedy(const float* __restrict__ logits, int V, const int32_t* __restrict__ row_slot,
                                const uint8_t* __restrict__ seen, float rp, float inv_rp, int eos_mask, int eos,
                                int32_t* __restrict__ tok_out, int32_t* __restrict__ greedy_out) {
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
    if (T > 0) k_sample_greedy<<<T, 256, 0, st>>>(logits, V, row_slot, seen, rp, inv_rp, eos_mask, eos, tok_out, greedy_out);
}

void sample_full(int T, const float* logits, int V, const int32_t* row_slot, const uint8_t* seen, const SamplerArgs& a,
                 int32_t* tok_out, int32_t* greedy_out, cudaStream_t st) {
    if (T > 0) k_sample_full<<<T, 1024, 0, st>>>(logits, V, row_slot, seen, a, tok_out, greedy_out);
}

// End of a decode step (session.cpp:247-284 on the device): feed the sampled token back,
// advance n_pos, mark the token as seen, append it to the device token ring.
__global__ void k_advance(int T, const int32_t* __restrict__ row_slot, const int32_t* __restrict__ tok,
                          int32_t* __restrict__ token_in, int32_t* __restrict__ n_pos, uint8_t* __restrict__ seen, int V,
                          int32_t* __restrict__ ring, int ring_len, int32_t* __restrict__ ring_step) {
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

__global__ void k_step_inc(int32_t* ring_step) { *ring_step += 1; }

void advance(int T, const int32_t* row_slot, const int32_t* tok, int32_t* token_in, int32_t* n_pos, uint8_t* seen,
             int V, int32_t* ring, int ring_len, int32_t* ring_step, cudaStream_t st) {
    if (T > 0) k_advance<<<(T + 255) / 256, 256, 0, st>>>(T, row_slot, tok, token_in, n_pos, seen, V, ring, ring_len, ring_step);
    k_step_inc<<<1, 1, 0, st>>>(ring_step);
}

__global__ void k_gather_rows(int n, const float* __restrict__ src, const int32_t* __restrict__ idx, int ld,
                              float* __restrict__ dst) {
    const int r = blockIdx.x;
    if (r >= n) return;
    for (int c = threadIdx.x; c < ld; c += blockDim.x) dst[(size_t)r * ld + c] = src[(size_t)idx[r] * ld + c];
}

void gather_rows(int n, const float* src, const int32_t* idx, int ld, float* dst, cudaStream_t st) {
    if (n > 0) k_gather_rows<<<n, 128, 0, st>>>(n, src, idx, ld, dst);
}

// Prefill input rows (block.cpp:424-468): text row t = (emb_t + bert_proj_t) + pe[t]*alpha_t,
// audio row t = emb_a + pe[t]*alpha_a.  bert_proj already holds W*bert + b.
__global__ void k_embed_prefill(int T_text, int T_prompt, const int32_t* __restrict__ phones,
                                const int32_t* __restrict__ sem, const float* __restrict__ bert_proj,
                                const uint16_t* __restrict__ text16, const float* __restrict__ text32,
                                const uint16_t* __restrict__ audio16, const float* __restrict__ audio32,
                                const float* __restrict__ pe, float alpha_t, float alpha_a, float* __restrict__ x) {
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
        k_embed_prefill<<<T, 128, 0, st>>>(T_text, T_prompt, phones, sem, bert_proj, text16, text32, audio16, audio32, pe,
                                           alpha_t, alpha_a, x);
}

}  // namespace t2sx
