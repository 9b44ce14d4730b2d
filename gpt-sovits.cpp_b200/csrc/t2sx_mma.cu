// Tensor-core quantised matmul for batched rows (M > 32): y[m][n] = bias[n] + W[n] . x[m].
//
// One mma.sync.m16n8k32 (s8 x s8 -> s32, zero accumulator) computes the exact integer dot of
// one 32-element quantisation block for a 16 (weight rows) x 8 (activation rows) tile, so the
// per-block float fold of the canonical order -- acc = fma(dw_b * dx_b, (float)isum_b, acc),
// blocks in increasing order -- runs unchanged on the MMA results (Q4_K: the sub-block sums are
// combined with their 6-bit scales / mins in integers and folded once per super-block).
//
// CTA: 256 threads = 8 warps as 4 (n) x 2 (m); warp tile 32 weight rows x (8*MT) rows.
// K is staged 4 blocks (128 elements) at a time through shared memory, double buffered with
// cp.async.  Weight fragments are read straight from the ggml block bytes: a Q8_0 block row is
// the A fragment's byte order; a Q4_0 block's 16 bytes hold elements j (low nibble) and j+16
// (high nibble), i.e. exactly the a0/a2 (and a1/a3) register pairs of one 32-bit load.
#include "t2sx_kernels.cuh"

#include <cstdlib>
#include "t2sx_math.cuh"
#include "t2sx_kv.cuh"

namespace t2sx {

__device__ __forceinline__ void mma_s8(int (&c)[4], int a0, int a1, int a2, int a3, int b0, int b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

__device__ __forceinline__ int lds32(const uint8_t* p) { return *reinterpret_cast<const int*>(p); }

// exact int -> float for |i| < 2^22 (block dots of Q8_0 / Q4_0 are below 2^19)
__device__ __forceinline__ float i2f_small(int i) { return __fsub_rn(__int_as_float(0x4B400000 + i), 12582912.0f); }

constexpr int KB = 4;            // 32-element blocks per stage
constexpr int XROW = KB * 32 + 16;   // smem bytes per activation row (int8, padded)

template <int WT, int MT_, int WN_, int NSTG_ = 2, int IT_ = 2>
struct Cfg {
    static constexpr int NSTG = NSTG_;                            // cp.async ring depth (stages)
    static constexpr int MT = MT_;                                // m8 tiles per warp
    static constexpr int WN = WN_;                                // warps along the weight rows
    static constexpr int IT = IT_;                                // m16 weight-row tiles per warp
    static constexpr int NT = 64 * WN;                            // threads (WN x 2 warps)
    static constexpr int BN = 16 * IT * WN;                       // weight rows per CTA
    static constexpr int BM = 2 * 8 * MT;                         // activation rows per CTA
    static constexpr int WROW = (WT == W_Q8_0) ? KB * 32 + 16 : KB * 16 + 16;  // weight bytes per row
    static constexpr int W_BYTES = BN * WROW;
    static constexpr int X_BYTES = BM * XROW;
    static constexpr int DW_BYTES = BN * KB * 4;                  // f32 scales [n][KB] (Q4_K: d,dmin,scm)
    static constexpr int DX_BYTES = BM * KB * 4;                  // f32 [m][KB] (Q4_K: bs32 int [m][KB])
    static constexpr int K_EXTRA = (WT == W_Q4_K) ? (BN * 16 + BN * 8 + BM * 4) : 0;  // scm, d+dmin, dx8k
    static constexpr int STAGE = W_BYTES + X_BYTES + DW_BYTES + DX_BYTES + K_EXTRA;
    static constexpr int SMEM = NSTG * STAGE;
};

template <int WT, int MT_, int WN_, int NSTG_, int IT_>
__global__ void __launch_bounds__(64 * WN_) k_mm_mma(DevW W, ActQ A, int M, const float* __restrict__ bias, int relu,
                                                float* __restrict__ y, QKVStore qkv, int use_qkv) {
    using C = Cfg<WT, MT_, WN_, NSTG_, IT_>;
    constexpr int NSTG = C::NSTG;
    constexpr int MT = C::MT, BM = C::BM, WROW = C::WROW, BN = C::BN, NT = C::NT, IT = C::IT;
    extern __shared__ __align__(16) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int wn = warp % C::WN, wm = warp / C::WN;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
    const int N = W.N, K = W.K;
    const int nb32 = K / 32, nsb = K / 256;
    const int nstage = K / (32 * KB);
    pdl_wait();
    pdl_trigger();

    auto sW = [&](int buf) { return smem + buf * C::STAGE; };
    auto sX = [&](int buf) { return smem + buf * C::STAGE + C::W_BYTES; };
    auto sDw = [&](int buf) { return reinterpret_cast<float*>(smem + buf * C::STAGE + C::W_BYTES + C::X_BYTES); };
    auto sDx = [&](int buf) {
        return reinterpret_cast<float*>(smem + buf * C::STAGE + C::W_BYTES + C::X_BYTES + C::DW_BYTES);
    };
    auto sScm = [&](int buf) { return smem + buf * C::STAGE + C::W_BYTES + C::X_BYTES + C::DW_BYTES + C::DX_BYTES; };
    auto sDd = [&](int buf) { return reinterpret_cast<float*>(sScm(buf) + BN * 16); };   // [n][2] d, dmin
    auto sDx8 = [&](int buf) { return reinterpret_cast<float*>(sScm(buf) + BN * 16 + BN * 8); };

    auto load_stage = [&](int stg, int buf) {
        const int kb0 = stg * KB;
        uint8_t* w = sW(buf);
        if (WT == W_Q8_0) {
            for (int i = tid; i < BN * 8; i += NT) {
                const int row = i >> 3, c = i & 7, n = n0 + row;
                const bool ok = n < N;
                cp_async16(w + row * WROW + c * 16, ok ? (const void*)(W.q8 + (size_t)n * K + kb0 * 32 + c * 16) : (const void*)W.q8, ok);
            }
        } else if (WT == W_Q4_0) {
            for (int i = tid; i < BN * 4; i += NT) {
                const int row = i >> 2, c = i & 3, n = n0 + row;
                const bool ok = n < N;
                cp_async16(w + row * WROW + c * 16, ok ? (const void*)(W.q4 + ((size_t)n * nb32 + kb0 + c) * 16) : (const void*)W.q4, ok);
            }
        } else {  // Q4_K: half a super-block (64 nibble bytes) per row per stage
            const int sb = kb0 >> 3, half = (kb0 >> 2) & 1;
            for (int i = tid; i < BN * 4; i += NT) {
                const int row = i >> 2, c = i & 3, n = n0 + row;
                const bool ok = n < N;
                cp_async16(w + row * WROW + c * 16,
                           ok ? (const void*)(W.q4 + ((size_t)n * nsb + sb) * 128 + half * 64 + c * 16) : (const void*)W.q4, ok);
            }
            for (int i = tid; i < BN; i += NT) {
                const int n = n0 + i;
                const bool ok = n < N;
                cp_async16(sScm(buf) + i * 16, ok ? (const void*)(W.scm + ((size_t)n * nsb + sb) * 16) : (const void*)W.scm, ok);
                cp_async4(sDd(buf) + 2 * i, ok ? (const void*)(W.d + (size_t)n * nsb + sb) : (const void*)W.d, ok);
                cp_async4(sDd(buf) + 2 * i + 1, ok ? (const void*)(W.dmin + (size_t)n * nsb + sb) : (const void*)W.dmin, ok);
            }
        }
        if (WT != W_Q4_K) {
            for (int i = tid; i < BN; i += NT) {
                const int n = n0 + i;
                const bool ok = n < N;
                cp_async16(sDw(buf) + i * KB, ok ? (const void*)(W.d + (size_t)n * nb32 + kb0) : (const void*)W.d, ok);
            }
        }
        uint8_t* x = sX(buf);
        for (int i = tid; i < BM * 8; i += NT) {
            const int row = i >> 3, c = i & 7, m = m0 + row;
            const bool ok = m < M;
            cp_async16(x + row * XROW + c * 16, ok ? (const void*)(A.q + (size_t)m * K + kb0 * 32 + c * 16) : (const void*)A.q, ok);
        }
        for (int i = tid; i < BM; i += NT) {
            const int m = m0 + i;
            const bool ok = m < M;
            if (WT == W_Q4_K) {
                cp_async16(sDx(buf) + i * KB, ok ? (const void*)(A.bs + (size_t)m * nb32 + kb0) : (const void*)A.bs, ok);
                cp_async4(sDx8(buf) + i, ok ? (const void*)(A.d + (size_t)m * nsb + (kb0 >> 3)) : (const void*)A.d, ok);
            } else {
                cp_async16(sDx(buf) + i * KB, ok ? (const void*)(A.d + (size_t)m * nb32 + kb0) : (const void*)A.d, ok);
            }
        }
        cp_commit();
    };

    float acc[IT][MT][4], accm[IT][MT][4];
    int sa[IT][MT][4], sm[IT][MT][4];
#pragma unroll
    for (int i = 0; i < IT; ++i)
#pragma unroll
        for (int j = 0; j < MT; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) { acc[i][j][e] = 0.0f; accm[i][j][e] = 0.0f; sa[i][j][e] = 0; sm[i][j][e] = 0; }

    // ring of NSTG stages: stage s lives in buffer s % NSTG; every iteration commits one group
    // (empty past the end) so that waiting for all but the newest NSTG - 2 groups means stage stg
    // has landed
#pragma unroll
    for (int s0 = 0; s0 < NSTG - 1; ++s0) {
        if (s0 < nstage) load_stage(s0, s0);
        else cp_commit();
    }
    for (int stg = 0; stg < nstage; ++stg) {
        const int buf = stg % NSTG;
        cp_wait<NSTG - 2>();
        __syncthreads();   // stage stg visible to all; buffer (stg - 1) % NSTG no longer read
        {
            const int nxt = stg + NSTG - 1;
            if (nxt < nstage) load_stage(nxt, nxt % NSTG);
            else cp_commit();
        }
        const uint8_t* w = sW(buf);
        const uint8_t* x = sX(buf);
#pragma unroll
        for (int blk = 0; blk < KB; ++blk) {
            int af[IT][4];
#pragma unroll
            for (int i = 0; i < IT; ++i) {
                const int r0 = wn * (16 * IT) + i * 16 + g;
                if (WT == W_Q8_0) {
                    af[i][0] = lds32(w + r0 * WROW + blk * 32 + t * 4);
                    af[i][1] = lds32(w + (r0 + 8) * WROW + blk * 32 + t * 4);
                    af[i][2] = lds32(w + r0 * WROW + blk * 32 + 16 + t * 4);
                    af[i][3] = lds32(w + (r0 + 8) * WROW + blk * 32 + 16 + t * 4);
                } else if (WT == W_Q4_0) {
                    const int w0 = lds32(w + r0 * WROW + blk * 16 + t * 4);
                    const int w1 = lds32(w + (r0 + 8) * WROW + blk * 16 + t * 4);
                    af[i][0] = __vsub4(w0 & 0x0F0F0F0F, 0x08080808);
                    af[i][1] = __vsub4(w1 & 0x0F0F0F0F, 0x08080808);
                    af[i][2] = __vsub4((w0 >> 4) & 0x0F0F0F0F, 0x08080808);
                    af[i][3] = __vsub4((w1 >> 4) & 0x0F0F0F0F, 0x08080808);
                } else {
                    // sub-block js = 4*half + blk of the super-block; local 32-byte chunk blk>>1,
                    // nibble blk&1
                    const int lc = blk >> 1, sh = (blk & 1) * 4;
                    const int w0 = lds32(w + r0 * WROW + lc * 32 + t * 4);
                    const int w1 = lds32(w + (r0 + 8) * WROW + lc * 32 + t * 4);
                    const int w2 = lds32(w + r0 * WROW + lc * 32 + 16 + t * 4);
                    const int w3 = lds32(w + (r0 + 8) * WROW + lc * 32 + 16 + t * 4);
                    af[i][0] = (w0 >> sh) & 0x0F0F0F0F;
                    af[i][1] = (w1 >> sh) & 0x0F0F0F0F;
                    af[i][2] = (w2 >> sh) & 0x0F0F0F0F;
                    af[i][3] = (w3 >> sh) & 0x0F0F0F0F;
                }
            }
            int bf[MT][2];
#pragma unroll
            for (int j = 0; j < MT; ++j) {
                const int mr = wm * (8 * MT) + j * 8 + g;
                bf[j][0] = lds32(x + mr * XROW + blk * 32 + t * 4);
                bf[j][1] = lds32(x + mr * XROW + blk * 32 + 16 + t * 4);
            }
            int is[IT][MT][4];
#pragma unroll
            for (int i = 0; i < IT; ++i)
#pragma unroll
                for (int j = 0; j < MT; ++j)
                    mma_s8(is[i][j], af[i][0], af[i][1], af[i][2], af[i][3], bf[j][0], bf[j][1]);
            if (WT == W_Q4_K) {
                const int js = ((stg & 1) << 2) + blk;   // sub-block index within the super-block
                const uint8_t* scm = sScm(buf);
                const int* bs = reinterpret_cast<const int*>(sDx(buf));
#pragma unroll
                for (int i = 0; i < IT; ++i) {
                    const int nr = wn * (16 * IT) + i * 16 + g;
                    const int sc0 = scm[nr * 16 + js], sc1 = scm[(nr + 8) * 16 + js];
                    const int mn0 = scm[nr * 16 + 8 + js], mn1 = scm[(nr + 8) * 16 + 8 + js];
#pragma unroll
                    for (int j = 0; j < MT; ++j) {
                        const int mr = wm * (8 * MT) + j * 8 + 2 * t;
                        const int b0 = bs[mr * KB + blk], b1 = bs[(mr + 1) * KB + blk];
                        sa[i][j][0] += sc0 * is[i][j][0]; sm[i][j][0] += mn0 * b0;
                        sa[i][j][1] += sc0 * is[i][j][1]; sm[i][j][1] += mn0 * b1;
                        sa[i][j][2] += sc1 * is[i][j][2]; sm[i][j][2] += mn1 * b0;
                        sa[i][j][3] += sc1 * is[i][j][3]; sm[i][j][3] += mn1 * b1;
                    }
                }
            } else {
                const float* dw = sDw(buf);
                const float* dx = sDx(buf);
#pragma unroll
                for (int i = 0; i < IT; ++i) {
                    const int nr = wn * (16 * IT) + i * 16 + g;
                    const float w0 = dw[nr * KB + blk], w1 = dw[(nr + 8) * KB + blk];
#pragma unroll
                    for (int j = 0; j < MT; ++j) {
                        const int mr = wm * (8 * MT) + j * 8 + 2 * t;
                        const float x0 = dx[mr * KB + blk], x1 = dx[(mr + 1) * KB + blk];
                        acc[i][j][0] = __fmaf_rn(__fmul_rn(w0, x0), i2f_small(is[i][j][0]), acc[i][j][0]);
                        acc[i][j][1] = __fmaf_rn(__fmul_rn(w0, x1), i2f_small(is[i][j][1]), acc[i][j][1]);
                        acc[i][j][2] = __fmaf_rn(__fmul_rn(w1, x0), i2f_small(is[i][j][2]), acc[i][j][2]);
                        acc[i][j][3] = __fmaf_rn(__fmul_rn(w1, x1), i2f_small(is[i][j][3]), acc[i][j][3]);
                    }
                }
            }
        }
        if (WT == W_Q4_K && (stg & 1)) {   // end of a super-block: fold the integer sums
            const float* dd = sDd(buf);
            const float* dx8 = sDx8(buf);
#pragma unroll
            for (int i = 0; i < IT; ++i) {
                const int nr = wn * (16 * IT) + i * 16 + g;
                const float dw0 = dd[2 * nr], dm0 = dd[2 * nr + 1], dw1 = dd[2 * (nr + 8)], dm1 = dd[2 * (nr + 8) + 1];
#pragma unroll
                for (int j = 0; j < MT; ++j) {
                    const int mr = wm * (8 * MT) + j * 8 + 2 * t;
                    const float x0 = dx8[mr], x1 = dx8[mr + 1];
                    const float wv[4] = {dw0, dw0, dw1, dw1}, mv[4] = {dm0, dm0, dm1, dm1}, xv[4] = {x0, x1, x0, x1};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        acc[i][j][e] = __fmaf_rn(__fmul_rn(xv[e], wv[e]), (float)sa[i][j][e], acc[i][j][e]);
                        accm[i][j][e] = __fmaf_rn(__fmul_rn(-xv[e], mv[e]), (float)sm[i][j][e], accm[i][j][e]);
                        sa[i][j][e] = 0;
                        sm[i][j][e] = 0;
                    }
                }
            }
        }
    }
#pragma unroll
    for (int i = 0; i < IT; ++i)
#pragma unroll
        for (int j = 0; j < MT; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int n = n0 + wn * (16 * IT) + i * 16 + g + ((e >> 1) << 3);
                const int m = m0 + wm * (8 * MT) + j * 8 + 2 * t + (e & 1);
                if (n < N && m < M) {
                    float v = (WT == W_Q4_K) ? __fadd_rn(acc[i][j][e], accm[i][j][e]) : acc[i][j][e];
                    if (bias) v = __fadd_rn(v, bias[n]);
                    if (relu) v = (v > 0.0f) ? v : 0.0f;
                    if (use_qkv) qkv_store(qkv, m, n, v);
                    else y[(size_t)m * N + n] = v;
                }
            }
}

template <int WT, int MT, int WN = 4, int NSTG = 2, int IT = 2>
static void launch_mma(const DevW& W, const ActQ& a, int M, const float* bias, int relu, float* y, const QKVStore* qkv,
                       cudaStream_t st) {
    using C = Cfg<WT, MT, WN, NSTG, IT>;
    static PerDeviceOnce setup;   // the shared-memory limit, set once on each device that launches it
    if (!setup.ensure([](int, int*) {
            return cudaFuncSetAttribute(k_mm_mma<WT, MT, WN, NSTG, IT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        C::SMEM) == cudaSuccess;
        }))
        return;   // the launch below is skipped and the caller's launch check reports the failure
    dim3 grid((W.N + C::BN - 1) / C::BN, (M + C::BM - 1) / C::BM);
    QKVStore q{};
    if (qkv) q = *qkv;
    launch_k((k_mm_mma<WT, MT, WN, NSTG, IT>), grid, dim3(C::NT), C::SMEM, st, W, a, M, bias, relu, y, q, qkv ? 1 : 0);
}

bool matmul_mma(const DevW& W, const ActQ& a, int M, const float* bias, int relu, float* y, const QKVStore* qkv,
                cudaStream_t st) {
    if (W.K % (32 * KB)) return false;
    // 64-row activation tiles when they still give two CTAs per SM, else 32-row tiles
    const bool wide = (long)((W.N + 127) / 128) * ((M + 63) / 64) >= 2 * 148;
    switch (W.type) {
        case W_Q8_0: wide ? launch_mma<W_Q8_0, 4>(W, a, M, bias, relu, y, qkv, st) : launch_mma<W_Q8_0, 2>(W, a, M, bias, relu, y, qkv, st); return true;
        case W_Q4_0: wide ? launch_mma<W_Q4_0, 4>(W, a, M, bias, relu, y, qkv, st) : launch_mma<W_Q4_0, 2>(W, a, M, bias, relu, y, qkv, st); return true;
        case W_Q4_K: launch_mma<W_Q4_K, 2>(W, a, M, bias, relu, y, qkv, st); return true;
    }
    return false;
}

// Narrow tiles (32 weight rows x 16 activation rows, 2 warps per CTA) for few activation rows:
// the matmul spreads over N/32 CTAs along the weight rows and ceil(M/16) along the activation
// rows, and the activation tile is staged once per CTA in shared memory instead of being re-read
// per weight row.  16-row tiles also for 17-32 rows: the 512-wide projections then run on 32
// CTAs instead of 16 (32 sessions: 1.66 -> 1.44 ms per decode step).  With few CTAs per SM the
// K loop is latency-bound, so the ring keeps 5 stages (640 elements of K) in flight.
// 16 weight rows per narrow CTA (T2SX_NARROW_W32=1: 32, two m16 tiles per warp).
static bool narrow16() {
    static const bool v = [] {
        const char* e = getenv("T2SX_NARROW_W32");
        return !(e && e[0] == '1');
    }();
    return v;
}

// ---------------------------------------------------------------------------------------------
// Split-K tiles for few activation rows (8-32): a CTA computes 16 weight rows x 16 activation rows.
// Its NW warps each take a contiguous range of K blocks (a multiple of 4, so a Q4_K range is a
// whole half or whole super-block), stage that range for all 32 rows with cp.async into their own
// slice of shared memory -- every byte of the tile in flight at once, no CTA-wide barrier before
// the MMAs -- and store the exact per-block integer dots (one mma.sync.m16n8k32 per block and
// 8-row half).  After one barrier each thread folds its output over all blocks of K in increasing
// order, the canonical fold of the kernels above:
//   Q8_0 / Q4_0: acc = fma(dw_b * dx_b, (float)isum_b, acc)
//   Q4_K:        per super-block sa = sum_j sc_j isum_j, sm = sum_j mn_j bsum_j (integers), then
//                acc = fma(dx * d, (float)sa, acc), accm = fma(-dx * dmin, (float)sm, accm)
// The weight slices are requested before griddepcontrol.wait (they are constants), the
// activations after it.
// ---------------------------------------------------------------------------------------------
namespace sk {
constexpr int BN = 16, BM = 16;   // weight rows, activation rows per CTA
constexpr int OUT = BN * BM;      // outputs per CTA = ints per block in the dot array

struct Layout {
    int nb, nsb, wrow, xrow, srow;   // blocks, super-blocks; row strides (bytes, bytes, floats)
    int off_x, off_dw, off_dx, off_dd, off_scm, off_dx8, off_is, bytes;
};
// Shared-memory layout for a weight of type wt with K columns.  Row strides are padded so that
// the fragment loads of the 8 rows a warp reads at once fall into distinct banks.
__host__ __device__ inline Layout layout(int wt, int K) {
    Layout L{};
    L.nb = K / 32;
    L.nsb = K / 256;
    L.wrow = (wt == W_Q8_0 ? K : K / 2) + 16;
    L.xrow = K + 16;
    L.srow = L.nb + 4;
    int o = BN * L.wrow;
    L.off_x = o;   o += BM * L.xrow;
    L.off_dw = o;  o += (wt == W_Q4_K ? 0 : BN * L.srow * 4);
    L.off_dx = o;  o += BM * L.srow * 4;                           // Q4_K: the int sub-block sums
    L.off_dd = o;  o += (wt == W_Q4_K ? BN * (2 * L.nsb + 1) * 4 : 0);   // d, dmin [n][sb][2] (+1 pad)
    o = (o + 15) & ~15;
    L.off_scm = o; o += (wt == W_Q4_K ? BN * (L.nsb + 1) * 16 : 0);      // [n][sb][16]: scales, mins (+16 B pad)
    L.off_dx8 = o; o += (wt == W_Q4_K ? BM * (L.nsb + 1) * 4 : 0);       // Q8_K row scale [m][sb] (+1 pad)
    o = (o + 15) & ~15;
    L.off_is = o;  o += L.nb * OUT * 4;
    L.bytes = o;
    return L;
}
}  // namespace sk

template <int WT, int NW>
__global__ void __launch_bounds__(32 * NW) k_mm_sk(DevW W, ActQ A, int M, const float* __restrict__ bias, int relu,
                                                   float* __restrict__ y, QKVStore qkv, int use_qkv) {
    constexpr int NT = 32 * NW;
    constexpr int BW = (WT == W_Q8_0) ? 32 : 16;   // weight bytes per 32-element block
    extern __shared__ __align__(16) uint8_t smem[];
    const int N = W.N, K = W.K;
    const sk::Layout L = sk::layout(WT, K);
    const int nb = L.nb, nsb = L.nsb;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int n0 = blockIdx.x * sk::BN, m0 = blockIdx.y * sk::BM;
    const int chunk = nb / NW, b0 = warp * chunk;   // this warp's blocks [b0, b0 + chunk)
    uint8_t* sW = smem;
    uint8_t* sX = smem + L.off_x;
    float* sDw = reinterpret_cast<float*>(smem + L.off_dw);
    float* sDx = reinterpret_cast<float*>(smem + L.off_dx);
    int* sBs = reinterpret_cast<int*>(smem + L.off_dx);
    float* sDd = reinterpret_cast<float*>(smem + L.off_dd);
    uint8_t* sScm = smem + L.off_scm;
    float* sDx8 = reinterpret_cast<float*>(smem + L.off_dx8);
    int* sIs = reinterpret_cast<int*>(smem + L.off_is);

    // ---- weight slices of this warp's blocks (constants: before the wait) ----
    {
        const int cpr = chunk * BW / 16;   // 16-byte pieces per row
        const uint8_t* wsrc = (WT == W_Q8_0) ? reinterpret_cast<const uint8_t*>(W.q8) : W.q4;
        const int wrow_g = (WT == W_Q8_0) ? K : K / 2;
        for (int i = lane; i < sk::BN * cpr; i += 32) {
            const int r = i / cpr, c = i % cpr, n = n0 + r;
            const bool ok = n < N;
            cp_async16(sW + r * L.wrow + b0 * BW + c * 16, ok ? (const void*)(wsrc + (size_t)n * wrow_g + b0 * BW + c * 16) : (const void*)wsrc, ok);
        }
        if (WT != W_Q4_K) {
            const int spr = chunk / 4;
            for (int i = lane; i < sk::BN * spr; i += 32) {
                const int r = i / spr, c = i % spr, n = n0 + r;
                const bool ok = n < N;
                cp_async16(sDw + r * L.srow + b0 + c * 4, ok ? (const void*)(W.d + (size_t)n * nb + b0 + c * 4) : (const void*)W.d, ok);
            }
        } else {   // scales of the super-blocks whose first block is in this warp's range
            for (int sb = (b0 + 7) >> 3; sb * 8 < b0 + chunk; ++sb)
                for (int r = lane; r < sk::BN; r += 32) {
                    const int n = n0 + r;
                    const bool ok = n < N;
                    cp_async16(sScm + (r * (nsb + 1) + sb) * 16, ok ? (const void*)(W.scm + ((size_t)n * nsb + sb) * 16) : (const void*)W.scm, ok);
                    cp_async4(sDd + r * (2 * nsb + 1) + 2 * sb, ok ? (const void*)(W.d + (size_t)n * nsb + sb) : (const void*)W.d, ok);
                    cp_async4(sDd + r * (2 * nsb + 1) + 2 * sb + 1, ok ? (const void*)(W.dmin + (size_t)n * nsb + sb) : (const void*)W.dmin, ok);
                }
        }
    }
    // ---- cache destinations of this thread's K/V outputs (QKV projection): above layer 0 the rows'
    // positions, slots and pages were written two or more launches back, so they are read before
    // the wait; layer 0 follows the embedding that writes them, so it reads them just after ----
    static_assert(sk::OUT % NT == 0, "whole outputs per thread");
    constexpr int NO = sk::OUT / NT;   // outputs per thread
    int2 dst[NO];
    auto out_row = [&](int o) {
        const int je = o >> 5, l = o & 31, j = je >> 2, e = je & 3;
        return m0 + j * 8 + 2 * (l & 3) + (e & 1);
    };
    auto out_col = [&](int o) {
        const int je = o >> 5, l = o & 31, e = je & 3;
        return n0 + (l >> 2) + ((e >> 1) << 3);
    };
    auto dest_of = [&](int o) {
        const int m = out_row(o);
        return (m < M && out_col(o) >= kD) ? qkv_dest(qkv, qkv.rows.pos[m], qkv.rows.slot[m]) : make_int2(-1, 0);
    };
    const bool early_dst = use_qkv && qkv.layer > 0;
    if (early_dst) {
#pragma unroll
        for (int i = 0; i < NO; ++i) dst[i] = dest_of(tid + i * NT);
    }
    float bv[NO];   // the outputs' biases (constants)
#pragma unroll
    for (int i = 0; i < NO; ++i) {
        const int n = out_col(tid + i * NT);
        bv[i] = (bias && n < N) ? bias[n] : 0.0f;
    }
    pdl_wait();
    pdl_trigger();
    if (use_qkv && !early_dst) {
#pragma unroll
        for (int i = 0; i < NO; ++i) dst[i] = dest_of(tid + i * NT);
    }
    // ---- activation slices ----
    {
        const int cpr = chunk * 2;   // 32 int8 per block
        for (int i = lane; i < sk::BM * cpr; i += 32) {
            const int r = i / cpr, c = i % cpr, m = m0 + r;
            const bool ok = m < M;
            cp_async16(sX + r * L.xrow + b0 * 32 + c * 16, ok ? (const void*)(A.q + (size_t)m * K + b0 * 32 + c * 16) : (const void*)A.q, ok);
        }
        const int spr = chunk / 4;
        for (int i = lane; i < sk::BM * spr; i += 32) {
            const int r = i / spr, c = i % spr, m = m0 + r;
            const bool ok = m < M;
            if (WT == W_Q4_K)
                cp_async16(sBs + r * L.srow + b0 + c * 4, ok ? (const void*)(A.bs + (size_t)m * nb + b0 + c * 4) : (const void*)A.bs, ok);
            else
                cp_async16(sDx + r * L.srow + b0 + c * 4, ok ? (const void*)(A.d + (size_t)m * nb + b0 + c * 4) : (const void*)A.d, ok);
        }
        if (WT == W_Q4_K) {
            for (int sb = (b0 + 7) >> 3; sb * 8 < b0 + chunk; ++sb)
                for (int r = lane; r < sk::BM; r += 32) {
                    const int m = m0 + r;
                    const bool ok = m < M;
                    cp_async4(sDx8 + r * (nsb + 1) + sb, ok ? (const void*)(A.d + (size_t)m * nsb + sb) : (const void*)A.d, ok);
                }
        }
    }
    cp_commit();
    cp_wait<0>();
    __syncwarp();

    // ---- exact block dots of this warp's range ----
    for (int b = b0; b < b0 + chunk; ++b) {
        int af[4];
        const uint8_t* wr0 = sW + g * L.wrow;
        const uint8_t* wr1 = sW + (g + 8) * L.wrow;
        if (WT == W_Q8_0) {
            af[0] = lds32(wr0 + b * 32 + t * 4);
            af[1] = lds32(wr1 + b * 32 + t * 4);
            af[2] = lds32(wr0 + b * 32 + 16 + t * 4);
            af[3] = lds32(wr1 + b * 32 + 16 + t * 4);
        } else if (WT == W_Q4_0) {
            const int w0 = lds32(wr0 + b * 16 + t * 4);
            const int w1 = lds32(wr1 + b * 16 + t * 4);
            af[0] = __vsub4(w0 & 0x0F0F0F0F, 0x08080808);
            af[1] = __vsub4(w1 & 0x0F0F0F0F, 0x08080808);
            af[2] = __vsub4((w0 >> 4) & 0x0F0F0F0F, 0x08080808);
            af[3] = __vsub4((w1 >> 4) & 0x0F0F0F0F, 0x08080808);
        } else {
            // sub-block js of super-block sb: 32-byte chunk js >> 1 of the super-block's 128 bytes,
            // low nibbles for even js, high for odd
            const int sb = b >> 3, js = b & 7;
            const int off = sb * 128 + (js >> 1) * 32, sh = (js & 1) * 4;
            af[0] = (lds32(wr0 + off + t * 4) >> sh) & 0x0F0F0F0F;
            af[1] = (lds32(wr1 + off + t * 4) >> sh) & 0x0F0F0F0F;
            af[2] = (lds32(wr0 + off + 16 + t * 4) >> sh) & 0x0F0F0F0F;
            af[3] = (lds32(wr1 + off + 16 + t * 4) >> sh) & 0x0F0F0F0F;
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const uint8_t* xr = sX + (j * 8 + g) * L.xrow + b * 32;
            int is[4];
            mma_s8(is, af[0], af[1], af[2], af[3], lds32(xr + t * 4), lds32(xr + 16 + t * 4));
#pragma unroll
            for (int e = 0; e < 4; ++e) sIs[b * sk::OUT + (j * 4 + e) * 32 + lane] = is[e];
        }
    }
    __syncthreads();

    // ---- ordered fold, one output per thread (two with 4 warps) ----
#pragma unroll
    for (int i = 0; i < NO; ++i) {
        const int o = tid + i * NT;
        const int je = o >> 5, l = o & 31;
        const int j = je >> 2, e = je & 3;
        const int nl = (l >> 2) + ((e >> 1) << 3), ml = j * 8 + 2 * (l & 3) + (e & 1);
        const int n = n0 + nl, m = m0 + ml;
        float v;
        if (WT == W_Q4_K) {
            float acc = 0.0f, accm = 0.0f;
            const int4* scm = reinterpret_cast<const int4*>(sScm) + nl * (nsb + 1);
            const int* bs = sBs + ml * L.srow;
            for (int sb = 0; sb < nsb; ++sb) {
                const int4 sc4 = scm[sb];   // bytes 0-7: the sub-block scales, 8-15: the mins
                const uint32_t sw[4] = {(uint32_t)sc4.x, (uint32_t)sc4.y, (uint32_t)sc4.z, (uint32_t)sc4.w};
                int sa = 0, sm = 0;
#pragma unroll
                for (int js = 0; js < 8; ++js) {
                    sa += (int)((sw[js >> 2] >> (8 * (js & 3))) & 0xFFu) * sIs[(sb * 8 + js) * sk::OUT + o];
                    sm += (int)((sw[2 + (js >> 2)] >> (8 * (js & 3))) & 0xFFu) * bs[sb * 8 + js];
                }
                const float xv = sDx8[ml * (nsb + 1) + sb];
                const float wv = sDd[nl * (2 * nsb + 1) + 2 * sb], mv = sDd[nl * (2 * nsb + 1) + 2 * sb + 1];
                acc = __fmaf_rn(__fmul_rn(xv, wv), (float)sa, acc);
                accm = __fmaf_rn(__fmul_rn(-xv, mv), (float)sm, accm);
            }
            v = __fadd_rn(acc, accm);
        } else {
            float acc = 0.0f;
            const float* dw = sDw + nl * L.srow;
            const float* dx = sDx + ml * L.srow;
#pragma unroll 8
            for (int b = 0; b < nb; ++b) acc = __fmaf_rn(__fmul_rn(dw[b], dx[b]), i2f_small(sIs[b * sk::OUT + o]), acc);
            v = acc;
        }
        if (n < N && m < M) {
            if (bias) v = __fadd_rn(v, bv[i]);
            if (relu) v = (v > 0.0f) ? v : 0.0f;
            if (use_qkv) qkv_store_at(qkv, m, n, v, dst[i]);
            else y[(size_t)m * N + n] = v;
        }
    }
}

// ---------------------------------------------------------------------------------------------
// F16 weights (f16 activations), 8-256 rows: split-K tiles of 16 weight rows x 16 activation rows.
// The canonical F16 arithmetic -- per 32-element block an fma chain from 0 over the elements in
// order, the block sums added in order from 0 -- lets the blocks' chains run in parallel: each of
// the 8 warps stages its contiguous range of blocks for the 32 rows (weights before the
// programmatic wait, activations after it), runs the 32-term chains of its blocks on the packed f16
// pairs with the mixed-precision fma (the f16 operands convert exactly; one rounding per step, as
// the f32 chain on converted operands), and stores the block sums; after one barrier each thread
// adds its output's block sums in order.  A lane owns 4 weight rows x 2 activation rows.
// ---------------------------------------------------------------------------------------------
namespace fsk {
constexpr int BN = 16, BM = 16, NW = 8;
__host__ __device__ inline int row_h(int K) { return K + 8; }   // staged row: halves (16-byte pad)
__host__ __device__ inline int smem_bytes(int K) { return 32 * row_h(K) * 2 + (K / 32) * BN * BM * 4; }
}  // namespace fsk

__global__ void __launch_bounds__(32 * fsk::NW) k_mm_f16_sk(DevW W, ActQ A, int M, const float* __restrict__ bias, int relu,
                                                            float* __restrict__ y, QKVStore qkv, int use_qkv) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int N = W.N, K = W.K, nb = K / 32, rh = fsk::row_h(K);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int n0 = blockIdx.x * fsk::BN, m0 = blockIdx.y * fsk::BM;
    const int chunk = nb / fsk::NW, b0 = warp * chunk;   // this warp's blocks [b0, b0 + chunk)
    uint16_t* sW = reinterpret_cast<uint16_t*>(smem);
    uint16_t* sX = sW + fsk::BN * rh;
    float* sS = reinterpret_cast<float*>(smem + 32 * rh * 2);   // [nb][BN * BM] block sums
    const int cpr = chunk * 4;   // 16-byte pieces (8 halves) per row of the range
    for (int i = lane; i < fsk::BN * cpr; i += 32) {
        const int r = i / cpr, c = i % cpr, n = n0 + r;
        const bool ok = n < N;
        cp_async16(sW + r * rh + b0 * 32 + c * 8, ok ? (const void*)(W.h + (size_t)n * K + b0 * 32 + c * 8) : (const void*)W.h, ok);
    }
    const int n_out = n0 + tid / fsk::BM;
    const float b_out = (bias && n_out < N) ? bias[n_out] : 0.0f;   // this thread's output's bias (a constant)
    pdl_wait();
    pdl_trigger();
    for (int i = lane; i < fsk::BM * cpr; i += 32) {
        const int r = i / cpr, c = i % cpr, m = m0 + r;
        const bool ok = m < M;
        cp_async16(sX + r * rh + b0 * 32 + c * 8, ok ? (const void*)(A.h + (size_t)m * K + b0 * 32 + c * 8) : (const void*)A.h, ok);
    }
    cp_commit();
    cp_wait<0>();
    __syncwarp();
    const int nq = (lane & 3) * 4, mq = (lane >> 2) * 2;
    for (int b = b0; b < b0 + chunk; ++b) {
        uint4 xv[2][4];
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int c = 0; c < 4; ++c) xv[j][c] = *reinterpret_cast<const uint4*>(sX + (mq + j) * rh + b * 32 + c * 8);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            uint4 wv[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) wv[c] = *reinterpret_cast<const uint4*>(sW + (nq + i) * rh + b * 32 + c * 8);
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                float sblk = 0.0f;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    sblk = fma_h2(wv[c].x, xv[j][c].x, sblk);
                    sblk = fma_h2(wv[c].y, xv[j][c].y, sblk);
                    sblk = fma_h2(wv[c].z, xv[j][c].z, sblk);
                    sblk = fma_h2(wv[c].w, xv[j][c].w, sblk);
                }
                sS[b * (fsk::BN * fsk::BM) + (nq + i) * fsk::BM + mq + j] = sblk;
            }
        }
    }
    __syncthreads();
    const int nl = tid / fsk::BM, ml = tid % fsk::BM, n = n0 + nl, m = m0 + ml;
    float acc = 0.0f;
#pragma unroll 8
    for (int b = 0; b < nb; ++b) acc = __fadd_rn(acc, sS[b * (fsk::BN * fsk::BM) + tid]);
    if (n < N && m < M) {
        float v = bias ? __fadd_rn(acc, b_out) : acc;
        if (relu) v = (v > 0.0f) ? v : 0.0f;
        if (use_qkv) qkv_store(qkv, m, n, v);
        else y[(size_t)m * N + n] = v;
    }
}

bool matmul_f16_sk(const DevW& W, const ActQ& a, int M, const float* bias, int relu, float* y, const QKVStore* qkv,
                   cudaStream_t st) {
    if (W.type != W_F16 || M < 1 || M > 256 || W.K % 256 || W.K > 2048 || !a.h ||
        (((uintptr_t)a.h | (uintptr_t)W.h) & 15))
        return false;
    static PerDeviceOnce setup;   // the shared-memory limit for K = 2048, once per device
    if (!setup.ensure([](int, int*) {
            return cudaFuncSetAttribute(k_mm_f16_sk, cudaFuncAttributeMaxDynamicSharedMemorySize, fsk::smem_bytes(2048)) ==
                   cudaSuccess;
        }))
        return false;
    const dim3 grid((W.N + fsk::BN - 1) / fsk::BN, (M + fsk::BM - 1) / fsk::BM);
    QKVStore q{};
    if (qkv) q = *qkv;
    launch_k(k_mm_f16_sk, grid, dim3(32 * fsk::NW), (size_t)fsk::smem_bytes(W.K), st, W, a, M, bias, relu, y, q, qkv ? 1 : 0);
    return true;
}

// Split-K tiles for 8-32 rows (T2SX_SPLITK=0: the narrow ring kernel below instead).
static bool splitk_on() {
    static const bool v = [] {
        const char* e = getenv("T2SX_SPLITK");
        return !(e && e[0] == '0');
    }();
    return v;
}

// false: nothing launched (the shared-memory limit could not be set); the caller falls back
template <int WT, int NW>
static bool launch_sk(const DevW& W, const ActQ& a, int M, const float* bias, int relu, float* y, const QKVStore* qkv,
                      cudaStream_t st, int smem) {
    static PerDeviceOnce setup;   // the shared-memory limit for the largest K (2048: 140 KB), once per device
    if (!setup.ensure([](int, int*) {
            return cudaFuncSetAttribute(k_mm_sk<WT, NW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        sk::layout(WT, 2048).bytes) == cudaSuccess;
        }))
        return false;
    const dim3 grid((W.N + sk::BN - 1) / sk::BN, (M + sk::BM - 1) / sk::BM);
    QKVStore q{};
    if (qkv) q = *qkv;
    launch_k((k_mm_sk<WT, NW>), grid, dim3(32 * NW), (size_t)smem, st, W, a, M, bias, relu, y, q, qkv ? 1 : 0);
    return true;
}

static bool matmul_sk(const DevW& W, const ActQ& a, int M, const float* bias, int relu, float* y, const QKVStore* qkv,
                      cudaStream_t st) {
    const int nb = W.K / 32;
    if (W.K % 128 || W.K > 2048 || M > 256) return false;
    const int nw = (nb % 32 == 0) ? 8 : (nb % 16 == 0 ? 4 : 0);   // chunk = nb / nw, a multiple of 4
    if (!nw) return false;
    const int smem = sk::layout(W.type, W.K).bytes;
    switch (W.type) {
        case W_Q8_0: return nw == 8 ? launch_sk<W_Q8_0, 8>(W, a, M, bias, relu, y, qkv, st, smem) : launch_sk<W_Q8_0, 4>(W, a, M, bias, relu, y, qkv, st, smem);
        case W_Q4_0: return nw == 8 ? launch_sk<W_Q4_0, 8>(W, a, M, bias, relu, y, qkv, st, smem) : launch_sk<W_Q4_0, 4>(W, a, M, bias, relu, y, qkv, st, smem);
        case W_Q4_K: return nw == 8 ? launch_sk<W_Q4_K, 8>(W, a, M, bias, relu, y, qkv, st, smem) : launch_sk<W_Q4_K, 4>(W, a, M, bias, relu, y, qkv, st, smem);
    }
    return false;
}

// Rows up to which the split-K tiles also take Q8_0/Q4_0 (and Q4_K below the tcgen05 threshold)
// matmuls above 32 rows instead of the mma.sync ring kernel: 64 rows, 160 for K = 2048, or
// T2SX_SK_MAX_ROWS for every K (at most 256).  Isolated calls: K = 2048 at 40-64 rows 22.6 ->
// 12.3 us, at 130 rows 22.6 -> 16.4 us; K = 512 at 40-64 rows 12.3 -> 10.3 us; at 256 rows the
// ring kernel's 128-row weight tiles are as fast or faster.
static int sk_env_rows() {
    static const int v = [] {
        const char* e = getenv("T2SX_SK_MAX_ROWS");
        const int r = e ? atoi(e) : 0;
        return r <= 0 ? 0 : (r < 32 ? 32 : (r > 256 ? 256 : r));
    }();
    return v;
}

bool matmul_sk_mid(const DevW& W, const ActQ& a, int M, const float* bias, int relu, float* y, const QKVStore* qkv,
                   cudaStream_t st) {
    const int lim = sk_env_rows() ? sk_env_rows() : (W.K >= 2048 ? 160 : 64);
    return M > 32 && M <= lim && splitk_on() && matmul_sk(W, a, M, bias, relu, y, qkv, st);
}

bool matmul_mma_narrow(const DevW& W, const ActQ& a, int M, const float* bias, int relu, float* y, const QKVStore* qkv,
                       cudaStream_t st) {
    if (M <= 32 && splitk_on() && matmul_sk(W, a, M, bias, relu, y, qkv, st)) return true;
    if (W.K % (32 * KB) || M > 32) return false;
    switch (W.type) {
        case W_Q8_0: narrow16() ? launch_mma<W_Q8_0, 1, 1, 6, 1>(W, a, M, bias, relu, y, qkv, st) : launch_mma<W_Q8_0, 1, 1, 6>(W, a, M, bias, relu, y, qkv, st); return true;
        case W_Q4_0: narrow16() ? launch_mma<W_Q4_0, 1, 1, 6, 1>(W, a, M, bias, relu, y, qkv, st) : launch_mma<W_Q4_0, 1, 1, 6>(W, a, M, bias, relu, y, qkv, st); return true;
        case W_Q4_K: narrow16() ? launch_mma<W_Q4_K, 1, 1, 6, 1>(W, a, M, bias, relu, y, qkv, st) : launch_mma<W_Q4_K, 1, 1, 6>(W, a, M, bias, relu, y, qkv, st); return true;
    }
    return false;
}

}  // namespace t2sx
