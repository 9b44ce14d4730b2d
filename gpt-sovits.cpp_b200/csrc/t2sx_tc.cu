// tcgen05 (5th-generation tensor core) matmul for Q4_K weights and batched rows:
//     y[m][n] = bias[n] + W[n] . x[m]
// with the ggml-CPU arithmetic of the reference's mul_mat on Q4_K weights and Q8_K activations
// (src/t2s/block.cpp:539-634 call sites): per 256-element super-block,
//     sa = sum_j sc_j * (sum_{k in j} q_k x_k),   sm = sum_j mn_j * (sum_{k in j} x_k)   (integers)
//     acc  = fma(dx * d, (float)sa, acc),   accm = fma(-dx * dmin, (float)sm, accm)
// over the super-blocks in order, output acc + accm.
//
// The weights are repacked at load into three int8 planes (lo = (sc*q) & 127, hi = (sc*q) >> 7,
// mn), so both integer sums of a super-block come out of the tensor core exactly:
//     sa = S_lo + 128 * S_hi,  sm = S_m,  S_p = sum_k plane_p[n][k] * x[m][k]  (tcgen05.mma.kind::i8,
// accumulated in TMEM over the 8 K-steps of 32 of the super-block).  Each accumulator starts at
// the bit pattern 0x4B400000 instead of 0, so the column read back as a float is 12582912 + S_p
// exactly (|S_p| < 2^22) and float(S_p) is one subtraction.  The fold then runs once per
// super-block on the CUDA cores, two columns per f32x2 instruction:
// (float)sa = fma(float(S_hi), 128, float(S_lo)) (one rounding of the exact sum), (float)sm = float(S_m).
//
// Persistent CTAs (one per SM) walk 128-row x 64-row output tiles; 12 warps in 3 warpgroups:
//   warp 0     : TMA producer (cp.async.bulk.tensor, 128-byte swizzle), 3-stage ring of half
//                super-blocks (3 weight planes x 128 rows x 128 B + 64 activation rows x 128 B); the
//                first three stages' weight planes are requested before the programmatic wait;
//   warps 1-3  : one thread each issues one weight plane's MMAs (4 per stage) and its tcgen05.commit
//                arrivals (the barriers count the three issuers);
//   warps 4-11 : fold -- warp w owns TMEM lanes 32*(w%4).. (weight rows) and 32 of the 64 columns,
//                reads them in 8-column groups (next group's load in flight while folding), resets
//                them to the start pattern, and stages the finished tile in smem for coalesced stores.
// TMEM: 2 super-block buffers x [S_lo | S_hi | S_m] x 64 columns (384 of 512 allocated).
//
// Every mbarrier wait is bounded (about a second of clock); on expiry the CTA raises a shared
// abort flag, drains what it issued, frees its TMEM, writes NaN outputs and records the failure
// in the row error flag when it has one.
#include "t2sx_kernels.cuh"
#include "t2sx_math.cuh"
#include "t2sx_kv.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

namespace t2sx {

namespace tc {

constexpr int BM = 128;           // weight rows per tile (MMA M, TMEM lanes)
constexpr int BN = 64;            // activation rows per tile (MMA N)
constexpr int NS = 3;             // smem stages (half super-blocks: 128 elements of K)
constexpr int NBUF = 2;           // TMEM super-block buffers
constexpr int PLANES = 3;
constexpr int BUF_COLS = PLANES * BN;
constexpr int TMEM_COLS = 512;
constexpr int EPI_WARPS = 8;
constexpr int EPI_WARP0 = 4;                  // warpgroup 0 = control, warpgroups 1-2 = fold
constexpr int THREADS = 32 * (EPI_WARP0 + EPI_WARPS);
// Register split (setmaxnreg): launched at kLaunchRegs per thread (384 threads, one CTA per SM),
// the control warpgroup gives registers back and the fold warpgroups take them:
// 128 * kCtrlRegs + 256 * kEpiRegs must not exceed 384 * kLaunchRegs.
constexpr int kLaunchRegs = 168, kCtrlRegs = 88, kEpiRegs = 208;
static_assert(128 * kCtrlRegs + 256 * kEpiRegs <= 384 * kLaunchRegs, "register split exceeds the launch allocation");
constexpr int A_PLANE = BM * 128;             // one weight plane of a stage (16 KB)
constexpr int B_TILE = BN * 128;              // activation tile of a stage (8 KB)
constexpr int STAGE = PLANES * A_PLANE + B_TILE;
constexpr int DX_BYTES = EPI_WARPS * 32 * 4;  // per epilogue warp: its 32 columns' activation scale
constexpr int OUT_BYTES = BN * BM * 4;        // finished output tile, [BN activation rows][BM] f32
constexpr int KVB_BYTES = BN * 8;             // per activation row of the tile: its K/V cache base offset
// ring full/empty, TMEM full/empty, MMA done, and one barrier nothing arrives on (test stall)
constexpr int BAR_BYTES = 8 * (2 * NS + 2 * NBUF + 2) + 16;
constexpr int SMEM = 1024 + NS * STAGE + OUT_BYTES + DX_BYTES + KVB_BYTES + BAR_BYTES;
// TMEM accumulators start at this bit pattern: the MMA adds the integer dot S to it and the
// result, read as a float, is 12582912 + S exactly (|S| < 2^22), so float(S) is one subtraction.
constexpr int kMagic = 0x4B400000;
constexpr float kMagicF = 12582912.0f;
constexpr long long kSpinCycles = 2000000000LL;   // bound of one wait (~1 s at 1.9 GHz)
// Value the kernel stores into its error word when a CTA gave up waiting (the session's bounds
// checks store 1 into the same word).
constexpr int kErrTimeout = 3;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void bar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void bar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool bar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Wait for the phase of the given parity; false when the CTA aborted or the wait ran out after
// `limit` cycles (kSpinCycles unless a test shortened it).
__device__ __forceinline__ bool bar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, long long limit) {
    long long t0 = 0;
    for (uint32_t it = 0;; ++it) {
        if (bar_try(bar, parity)) return true;
        if ((it & 31) == 31) {
            if (*abort_flag) return false;
            const long long now = clock64();
            if (t0 == 0) t0 = now;
            else if (now - t0 > limit) { *abort_flag = 1; return false; }
        }
    }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n"
        ::"r"(dst), "l"((uint64_t)map), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

// barrier of the 8 epilogue warps only (named barrier 1)
// tensor store of one box from shared memory (x, y >= 0; x * element size a multiple of 16 bytes;
// the parts of the box outside the tensor are not written), tracked per thread
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, int x, int y, const void* ssrc) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];\n" ::"l"((uint64_t)map), "r"(x),
                 "r"(y), "r"(smem_u32(ssrc))
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;\n" ::: "memory"); }
// this thread's tensor stores have read their shared-memory source
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory"); }
// this thread's tensor stores have completed
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory"); }
// shared-memory writes of this thread become visible to the tensor-store (async) proxy
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, %0;\n" ::"n"(32 * EPI_WARPS) : "memory"); }
// the same barrier, returning the OR of v over the 8 warps (one decision for all of them)
__device__ __forceinline__ bool epi_sync_or(bool v) {
    uint32_t r;
    asm volatile("{\n.reg .pred p, q;\nsetp.ne.u32 q, %1, 0;\nbar.red.or.pred p, 1, %2, q;\nselp.u32 %0, 1, 0, p;\n}\n"
                 : "=r"(r)
                 : "r"((uint32_t)v), "n"(32 * EPI_WARPS)
                 : "memory");
    return r != 0;
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar) : "memory");
}
// D[tmem] (=|+=) A[smem] . B[smem]^T, s8 x s8 -> s32
__device__ __forceinline__ void tc_mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\ntcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n"
        ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, 8-row core groups 1024 B apart.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)1 << 16;             // leading byte offset (16 B; unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;   // stride byte offset
    d |= (uint64_t)1 << 46;             // descriptor version (sm_100)
    d |= (uint64_t)2 << 61;             // SWIZZLE_128B
    return d;
}

// Instruction descriptor: kind::i8, s8 x s8 -> s32, both K-major, M = BM, N = BN.
constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

// columns [c, c+8) of each of the three planes (BN columns apart) of this thread's lane (no wait)
__device__ __forceinline__ void tmem_ld3x8(uint32_t taddr, int (&v)[24]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%24];\n"
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%8,%9,%10,%11,%12,%13,%14,%15}, [%25];\n"
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%16,%17,%18,%19,%20,%21,%22,%23}, [%26];\n"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23])
        : "r"(taddr), "r"(taddr + (uint32_t)BN), "r"(taddr + (uint32_t)(2 * BN)));
}
// wait for this thread's TMEM loads, then pin the loaded registers after the wait (the compiler
// must not read them earlier)
template <int NR>
__device__ __forceinline__ void tmem_wait_ld_regs2(int (&v)[NR], int (&w)[NR]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
    for (int i = 0; i < NR; ++i) asm volatile("" : "+r"(v[i]), "+r"(w[i]));
}
// 32 consecutive TMEM columns of this thread's lane := c (four 8-column stores: the source of one
// store is 8 consecutive registers, so this keeps the constant's register footprint at 8)
__device__ __forceinline__ void tmem_st32_const(uint32_t taddr, int c) {
#pragma unroll
    for (int g = 0; g < 4; ++g)
        asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1};\n" ::"r"(taddr + 8 * g), "r"(c)
                     : "memory");
}
// columns [c, c+8) of each of the three planes := k
__device__ __forceinline__ void tmem_st3x8_const(uint32_t taddr, int k) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%3,%3,%3,%3,%3,%3,%3,%3};\n"
        "tcgen05.st.sync.aligned.32x32b.x8.b32 [%1], {%3,%3,%3,%3,%3,%3,%3,%3};\n"
        "tcgen05.st.sync.aligned.32x32b.x8.b32 [%2], {%3,%3,%3,%3,%3,%3,%3,%3};\n" ::"r"(taddr),
        "r"(taddr + (uint32_t)BN), "r"(taddr + (uint32_t)(2 * BN)), "r"(k)
        : "memory");
}
// packed pairs of IEEE f32 operations, each lane rounded to nearest even as the scalar op
__device__ __forceinline__ uint64_t f2u(float2 a) { return *reinterpret_cast<uint64_t*>(&a); }
__device__ __forceinline__ float2 u2f(uint64_t a) { return *reinterpret_cast<float2*>(&a); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;\n" : "=l"(r) : "l"(f2u(a)), "l"(f2u(b)));
    return u2f(r);
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;\n" : "=l"(r) : "l"(f2u(a)), "l"(f2u(b)));
    return u2f(r);
}
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;\n" : "=l"(r) : "l"(f2u(a)), "l"(f2u(b)), "l"(f2u(c)));
    return u2f(r);
}


__global__ void __launch_bounds__(THREADS, 1)
k_mm_tc_q4k(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
            const __grid_constant__ CUtensorMap tmY, DevW W, ActQ A, int M, const float* __restrict__ bias, int relu,
            float* __restrict__ y, QKVStore qkv, int use_qkv, int tstore, int32_t* err, long long spin, int test_stall) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    float* out_tile = (float*)(smem + NS * STAGE);
    float* dx_base = (float*)(smem + NS * STAGE + OUT_BYTES);
    long long* kvb = (long long*)(smem + NS * STAGE + OUT_BYTES + DX_BYTES);
    uint64_t* bars = (uint64_t*)(smem + NS * STAGE + OUT_BYTES + DX_BYTES + KVB_BYTES);
    uint32_t* tmem_holder = (uint32_t*)(bars + 2 * NS + 2 * NBUF + 2);
    volatile int* abort_flag = (volatile int*)(tmem_holder + 1);
    const uint32_t full0 = smem_u32(bars), empty0 = full0 + 8 * NS, tfull0 = empty0 + 8 * NS,
                   tempty0 = tfull0 + 8 * NBUF, done_bar = tempty0 + 8 * NBUF, stall_bar = done_bar + 8;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {   // the producer's first copies need both descriptors
        asm volatile("prefetch.tensormap [%0];\n" ::"l"((uint64_t)&tmW) : "memory");
        asm volatile("prefetch.tensormap [%0];\n" ::"l"((uint64_t)&tmX) : "memory");
    }
    const int N = W.N, K = W.K, nsb = K / 256;
    const int tiles_n = (N + BM - 1) / BM, tiles_m = (M + BN - 1) / BN;
    const int n_tiles = tiles_n * tiles_m;

    // The first tile's first stages: their weight planes are constants, so the producer thread
    // requests them here, before the programmatic wait; their activation tiles follow the wait.
    const int pre = (blockIdx.x < n_tiles) ? (2 * nsb < NS ? 2 * nsb : NS) : 0;
    const int n0_first = (blockIdx.x % tiles_n) * BM, m0_first = (blockIdx.x / tiles_n) * BN;
    if (tid == 0) {
        for (int i = 0; i < NS; ++i) { bar_init(full0 + 8 * i, 1); bar_init(empty0 + 8 * i, PLANES); }
        for (int i = 0; i < NBUF; ++i) { bar_init(tfull0 + 8 * i, PLANES); bar_init(tempty0 + 8 * i, EPI_WARPS); }
        bar_init(done_bar, PLANES);
        bar_init(stall_bar, 1);   // no thread ever arrives on it
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        for (int s = 0; s < pre; ++s) {
            const uint32_t fb = full0 + 8 * s;
            bar_expect_tx(fb, STAGE);   // the whole stage: these planes and, after the wait, the activations
            const uint32_t st = smem_u32(smem + s * STAGE);
#pragma unroll
            for (int p = 0; p < PLANES; ++p) tma_load_2d(st + p * A_PLANE, &tmW, s * 128, p * W.tc_npad + n0_first, fb);
        }
    }
    if (warp == 0) {
        __syncwarp();
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_holder)),
                     "r"(TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    if (warp >= EPI_WARP0) {
        // every accumulator column starts at the magic pattern (the epilogue restores it after each read)
        const uint32_t tl0 = tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)(((warp - EPI_WARP0) >> 2) * 32);
#pragma unroll
        for (int b = 0; b < NBUF; ++b)
#pragma unroll
            for (int p = 0; p < PLANES; ++p) tmem_st32_const(tl0 + (uint32_t)(b * BUF_COLS + p * BN), kMagic);
        asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    // the set-up above touches no data of earlier kernels; everything below may
    pdl_wait();
    pdl_trigger();
    bool aborted = false;
    if (warp < EPI_WARP0) {   // control warpgroup: warp 0 TMA, warps 1-3 MMA (one plane each)
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(kCtrlRegs));
        if (warp == 0) {
            // ---------------- TMA producer: stages of 128 K-elements, 2 per super-block ----------------
            if (lane == 0) {
                // the activation tiles of the stages whose planes went out before the wait (always
                // issued, so that those stages complete and the abort drain below ends)
                for (int s = 0; s < pre; ++s)
                    tma_load_2d(smem_u32(smem + s * STAGE) + PLANES * A_PLANE, &tmX, s * 128, m0_first, full0 + 8 * s);
                int stg = 0;
                for (int t = blockIdx.x; t < n_tiles && !aborted; t += gridDim.x) {
                    const int n0 = (t % tiles_n) * BM, m0 = (t / tiles_n) * BN;
                    for (int h = 0; h < 2 * nsb; ++h, ++stg) {
                        if (stg < pre) continue;   // issued above
                        const int ss = stg % NS;
                        if (!bar_wait(empty0 + 8 * ss, ((stg / NS) & 1) ^ 1, abort_flag, spin)) { aborted = true; break; }
                        const uint32_t fb = full0 + 8 * ss;
                        bar_expect_tx(fb, STAGE);
                        const uint32_t st = smem_u32(smem + ss * STAGE);
                        const int k0 = h * 128;
#pragma unroll
                        for (int p = 0; p < PLANES; ++p) tma_load_2d(st + p * A_PLANE, &tmW, k0, p * W.tc_npad + n0, fb);
                        tma_load_2d(st + PLANES * A_PLANE, &tmX, k0, m0, fb);
                    }
                }
                if (aborted) {
                    // let the copies already issued land before the CTA's smem is released
                    for (int s = stg - NS < 0 ? 0 : stg - NS; s < stg; ++s) {
                        const long long t0 = clock64();
                        while (!bar_try(full0 + 8 * (s % NS), (s / NS) & 1) && clock64() - t0 < kSpinCycles) {}
                    }
                }
            }
        } else {
            // ---------------- MMA issuers: warp 1 + p issues plane p's 8 MMAs of each super-block ----------------
            if (lane == 0) {
                const int p = warp - 1;
                int stg = 0, gsb = 0;
                const uint64_t d0 = sdesc(smem_u32(smem));
                for (int t = blockIdx.x; t < n_tiles && !aborted; t += gridDim.x) {
                    for (int sb = 0; sb < nsb && !aborted; ++sb, ++gsb) {
                        const int buf = gsb % NBUF;
                        if (!bar_wait(tempty0 + 8 * buf, ((gsb / NBUF) & 1) ^ 1, abort_flag, spin)) { aborted = true; break; }
                        tc_fence_after();
                        const uint32_t dcol = tmem + (uint32_t)(buf * BUF_COLS + p * BN);
                        for (int h = 0; h < 2; ++h, ++stg) {
                            const int ss = stg % NS;
                            if (!bar_wait(full0 + 8 * ss, (stg / NS) & 1, abort_flag, spin)) { aborted = true; break; }
                            tc_fence_after();
                            // descriptor start addresses advance in 16-byte units in the low bits
                            const uint64_t dst = d0 + (uint64_t)((ss * STAGE) >> 4);
#pragma unroll
                            for (int kk = 0; kk < 4; ++kk)
                                tc_mma_i8(dcol, dst + (uint64_t)((p * A_PLANE + kk * 32) >> 4),
                                          dst + (uint64_t)((PLANES * A_PLANE + kk * 32) >> 4), kIdesc, 1u);
                            tc_commit(empty0 + 8 * ss);
                        }
                        tc_commit(tfull0 + 8 * buf);
                    }
                }
                // every MMA this thread issued has completed once the barrier flips (all three issuers)
                tc_commit(done_bar);
                const long long t0 = clock64();
                while (!bar_try(done_bar, 0) && clock64() - t0 < kSpinCycles) {}
            }
        }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(kEpiRegs));
        // ---------------- fold (epilogue) warps ----------------
        const int e = warp - EPI_WARP0;
        const int quarter = warp & 3;          // TMEM lanes this warp may access
        const int cg = e >> 2;                 // column group: activation rows 32*cg .. of the tile
        float* dxs = dx_base + e * 32;
        const uint32_t tl = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(cg * 32);
        int gsb = 0;
        for (int t = blockIdx.x; t < n_tiles && !aborted; t += gridDim.x) {
            const int n0 = (t % tiles_n) * BM, m0 = (t / tiles_n) * BN;
            const int n = n0 + quarter * 32 + lane;
            const bool nok = n < N;
            const int mt = m0 + cg * 32 + lane;    // the activation row whose scale this lane stages
            const bool mok = mt < M;
            float2 acc[16], accm[16];   // columns (2i, 2i+1)
#pragma unroll
            for (int c = 0; c < 16; ++c) { acc[c] = make_float2(0.0f, 0.0f); accm[c] = make_float2(0.0f, 0.0f); }
            float wd = nok ? W.d[(size_t)n * nsb] : 0.0f, wm = nok ? W.dmin[(size_t)n * nsb] : 0.0f;
            float xd = mok ? A.d[(size_t)mt * nsb] : 0.0f;
            // for the epilogue, requested now so that the loads overlap the fold: this lane's bias
            // and (QKV projection) the K/V cache offset of (page, layer, K, head 0, pos, dim 0) of
            // tile row m0 + et, or -1
            const float bn = (bias && nok) ? bias[n] : 0.0f;
            const int et = tid - 32 * EPI_WARP0;   // 0..255
            long long kv_row = -1;
            if (use_qkv && et < BN && m0 + et < M) {
                const int m = m0 + et;
                const int pos = qkv.rows.pos[m], sl = qkv.rows.slot[m];
                const int pg = min(max(pos, 0) / kPage, qkv.kv.max_pages - 1);
                const int cap = qkv.rows.cap[sl];
                const int page = qkv.kv.ptab[(size_t)sl * qkv.kv.max_pages + pg];
                if (pos >= 0 && pos < cap) kv_row = (long long)kv_off(qkv.kv, page, qkv.layer, 0, 0, pos % kPage);
            }
            for (int sb = 0; sb < nsb; ++sb, ++gsb) {
                const float2 d2 = make_float2(wd, wd), ndm2 = make_float2(-wm, -wm);
                __syncwarp();
                dxs[lane] = xd;
                __syncwarp();
                if (sb + 1 < nsb) {
                    wd = nok ? W.d[(size_t)n * nsb + sb + 1] : 0.0f;
                    wm = nok ? W.dmin[(size_t)n * nsb + sb + 1] : 0.0f;
                    xd = mok ? A.d[(size_t)mt * nsb + sb + 1] : 0.0f;
                }
                const int buf = gsb % NBUF;
                // test_stall (test hook only): the first wait is on a barrier that nothing completes,
                // so it runs out after `spin` cycles and the abort path below is taken
                bool ok = !(test_stall && gsb == 0) || bar_wait(stall_bar, 0, abort_flag, spin);
                ok = ok && bar_wait(tfull0 + 8 * buf, (gsb / NBUF) & 1, abort_flag, spin);
                if (__any_sync(0xffffffffu, !ok)) { aborted = true; break; }   // also reconverges the warp
                tc_fence_after();
                const uint32_t tb = tl + (uint32_t)(buf * BUF_COLS);
                // fold 8 columns: v = [S_lo + magic | S_hi + magic | S_m + magic] as float bits
                auto fold8 = [&](const int (&v)[24], int q) {
                    const float2 mg = make_float2(-kMagicF, -kMagicF), k128 = make_float2(128.0f, 128.0f);
                    const float4 xa = reinterpret_cast<const float4*>(dxs + q * 8)[0];
                    const float4 xb = reinterpret_cast<const float4*>(dxs + q * 8)[1];
                    const float2 xs[4] = {make_float2(xa.x, xa.y), make_float2(xa.z, xa.w), make_float2(xb.x, xb.y),
                                          make_float2(xb.z, xb.w)};
#pragma unroll
                    for (int pr = 0; pr < 4; ++pr) {
                        const float2 lo = add2(make_float2(__int_as_float(v[2 * pr]), __int_as_float(v[2 * pr + 1])), mg);
                        const float2 hi = add2(make_float2(__int_as_float(v[8 + 2 * pr]), __int_as_float(v[8 + 2 * pr + 1])), mg);
                        const float2 mn = add2(make_float2(__int_as_float(v[16 + 2 * pr]), __int_as_float(v[16 + 2 * pr + 1])), mg);
                        const float2 fa = fma2(hi, k128, lo);   // (float)(S_lo + 128 S_hi), one rounding
                        const int c2 = q * 4 + pr;
                        acc[c2] = fma2(mul2(xs[pr], d2), fa, acc[c2]);
                        accm[c2] = fma2(mul2(xs[pr], ndm2), mn, accm[c2]);
                    }
                };
                auto ld24 = [&](int (&v)[24], int q) { tmem_ld3x8(tb + q * 8, v); };
                // each 8-column group is restored to the magic pattern as soon as it is in registers
                auto reset8 = [&](int q) { tmem_st3x8_const(tb + q * 8, kMagic); };
                // two 8-column groups per TMEM round trip; the second pair loads while the first folds
                int va[24], vb[24], vc[24], vd[24];
                ld24(va, 0); ld24(vb, 1); tmem_wait_ld_regs2(va, vb); reset8(0); reset8(1);
                ld24(vc, 2); ld24(vd, 3); fold8(va, 0); fold8(vb, 1); tmem_wait_ld_regs2(vc, vd); reset8(2); reset8(3);
                // this warp's columns are read and reset: hand the buffer back
                asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
                tc_fence_before();
                __syncwarp();
                if (lane == 0) bar_arrive(tempty0 + 8 * buf);
                fold8(vc, 2); fold8(vd, 3);
            }
            // ---------------- output: registers -> smem tile -> global ----------------
            // The tile is staged in shared memory (f16 for the QKV projection, else f32).  An f32
            // tile or a Q tile then leaves as one tensor store issued by one thread, so the fold
            // warps go on to the next tile while it drains (that thread waits until the store has
            // read the tile before the tile is written again); K/V tiles go to each row's page
            // slot with 16-byte stores.  Every epilogue warp takes the same abort decision at the
            // first barrier.
            if (tstore && et == 0) bulk_wait_read();
            aborted = epi_sync_or(aborted || *abort_flag);
            const float nan_v = __int_as_float(0x7FC00000);
            uint16_t* out_h = reinterpret_cast<uint16_t*>(out_tile);   // [BN][BM] f16 (QKV)
            {
                // acc + accm is never -0 (both chains start at +0), so adding a zero bias changes no value
                const int col = quarter * 32 + lane;
                const float2 bn2 = make_float2(bn, bn);
                float2 v2[16];
#pragma unroll
                for (int c2 = 0; c2 < 16; ++c2) {
                    v2[c2] = add2(add2(acc[c2], accm[c2]), bn2);
                    if (relu && !(v2[c2].x > 0.0f)) v2[c2].x = 0.0f;
                    if (relu && !(v2[c2].y > 0.0f)) v2[c2].y = 0.0f;
                    if (aborted) v2[c2] = make_float2(nan_v, nan_v);
                }
                if (use_qkv) {
#pragma unroll
                    for (int c2 = 0; c2 < 16; ++c2) {
                        out_h[(cg * 32 + 2 * c2) * BM + col] = f2h(v2[c2].x);
                        out_h[(cg * 32 + 2 * c2 + 1) * BM + col] = f2h(v2[c2].y);
                    }
                } else {
#pragma unroll
                    for (int c2 = 0; c2 < 16; ++c2) {
                        out_tile[(cg * 32 + 2 * c2) * BM + col] = v2[c2].x;
                        out_tile[(cg * 32 + 2 * c2 + 1) * BM + col] = v2[c2].y;
                    }
                }
            }
            if (use_qkv && et < BN) kvb[et] = kv_row;
            if (tstore) fence_proxy_async_smem();
            epi_sync();
            if (use_qkv && n0 >= kD) {
                // K or V tile: 4 heads of 32 values per row; (row, head) chunks of 64 B to the row's page slot
                const int ml = et >> 2, hh = et & 3;
                const int m = m0 + ml;
                const long long base = kvb[ml];
                if (m < M && base >= 0) {
                    const int j = n0 - kD + hh * kHeadDim, which = j / kD, head = (j % kD) / kHeadDim;
                    uint4* dst = reinterpret_cast<uint4*>(qkv.kv.pool + (size_t)base + (size_t)(which * kHeads + head) * kPage * kHeadDim);
                    const uint4* src = reinterpret_cast<const uint4*>(out_h + ml * BM + hh * kHeadDim);
#pragma unroll
                    for (int c = 0; c < 4; ++c) dst[c] = src[c];
                }
            } else if (tstore) {
                if (et == 0) {
                    tma_store_2d(&tmY, n0, m0, out_tile);   // Q rows (f16) or y rows (f32)
                    bulk_commit();
                }
            } else {
#pragma unroll 1
                for (int i = et; i < BN * BM; i += 32 * EPI_WARPS) {
                    const int ml = i / BM, nl = i % BM;
                    const int m = m0 + ml, nn = n0 + nl;
                    if (m >= M || nn >= N) continue;
                    y[(size_t)m * N + nn] = out_tile[i];
                }
            }
        }
        if (tstore && tid == 32 * EPI_WARP0) bulk_wait_all();   // the stores are complete before the CTA exits
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (*abort_flag && tid == 0 && err) atomicExch(err, kErrTimeout);
    if (warp == 0) {
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
    });
    return fn;
}

// row-major [rows][cols] of f32 or f16 (elem_bytes 4 or 2), boxes of BM columns x BN rows, no
// swizzle: the staged output tile of the kernel.
bool make_out_map(CUtensorMap* map, const void* base, int cols, int rows, int elem_bytes) {
    auto fn = encode_fn();
    if (!fn || ((uintptr_t)base & 15) || (((size_t)cols * elem_bytes) & 15)) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)cols * elem_bytes};
    cuuint32_t box[2] = {(cuuint32_t)BM, (cuuint32_t)BN};
    cuuint32_t es[2] = {1, 1};
    return fn(map, elem_bytes == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base),
              dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
              CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// int8 [rows][K] row-major, boxes of 128 bytes of K x box_rows rows, 128-byte swizzle.
bool make_map(CUtensorMap* map, const void* base, int K, int rows, int box_rows) {
    auto fn = encode_fn();
    if (!fn || ((uintptr_t)base & 15) || (K & 15)) return false;
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)K};
    cuuint32_t box[2] = {128, (cuuint32_t)box_rows};
    cuuint32_t es[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool launch_q4k(const DevW& W, const ActQ& a, int M, const float* bias, int relu, float* y, const QKVStore* qkv,
                cudaStream_t st) {
    // per device: the setmaxnreg split assumes exactly kLaunchRegs registers per thread at launch;
    // the shared-memory limit is set on that device; value = its SM count
    static PerDeviceOnce setup;
    int n_sm = 0;
    const bool usable = setup.ensure([](int dev, int* sms) {
        cudaFuncAttributes fa;
        if (cudaFuncGetAttributes(&fa, k_mm_tc_q4k) != cudaSuccess || fa.numRegs != kLaunchRegs) return false;
        if (cudaFuncSetAttribute(k_mm_tc_q4k, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM) != cudaSuccess) return false;
        return cudaDeviceGetAttribute(sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && *sms > 0;
    }, &n_sm);
    if (!usable) return false;
    CUtensorMap mw, mx;
    if (!make_map(&mw, W.tcw, W.K, PLANES * W.tc_npad, BM) || !make_map(&mx, a.q, W.K, M, BN)) return false;
    QKVStore q{};
    if (qkv) q = *qkv;
    const int tiles = ((W.N + BM - 1) / BM) * ((M + BN - 1) / BN);
    const int grid = tiles < n_sm ? tiles : n_sm;
    // tensor stores of the output tile: Q rows of the QKV projection (f16 [M][512]), else y (f32
    // [M][N]) when its rows are 16-byte aligned; otherwise the kernel stores element by element
    CUtensorMap my;
    std::memset(&my, 0, sizeof(my));
    const int tstore = qkv ? (make_out_map(&my, qkv->q16, kD, M, 2) ? 1 : 0) : (make_out_map(&my, y, W.N, M, 4) ? 1 : 0);
    if (qkv && !tstore) return false;
    // where a CTA that gives up waiting reports it: the error word of the entry point that
    // launched (or captured) this launch; the wait bound, unless a test shortened it
    int32_t* err = current_err_word();
    const long long test_spin = tc_test_wait_cycles();
    const long long spin = test_spin > 0 ? test_spin : kSpinCycles;
    const int stall = test_spin > 0 ? 1 : 0;
    // Programmatic dependent launch (T2SX_PDL_TC=0 turns it off): the set-up before the kernel's
    // griddepcontrol.wait (barriers, TMEM allocation and start pattern, descriptor prefetch) runs
    // while the preceding kernel drains.  A CTA of this kernel fills an SM, so it never shares
    // one with a CTA of another launch of it.  2048-row decode step: 8.03 -> 7.92 ms.
    static const bool pdl_tc = [] { const char* e = getenv("T2SX_PDL_TC"); return !(e && e[0] == '0'); }();
    if (pdl_tc) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(grid);
        cfg.blockDim = dim3(THREADS);
        cfg.dynamicSmemBytes = (size_t)SMEM;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        const int uq = qkv ? 1 : 0;
        cudaLaunchKernelEx(&cfg, k_mm_tc_q4k, mw, mx, my, W, a, M, bias, relu, y, q, uq, tstore, err, spin, stall);
    } else {
        launch_k(k_mm_tc_q4k, dim3(grid), dim3(THREADS), (size_t)SMEM, st, mw, mx, my, W, a, M, bias, relu, y, q, qkv ? 1 : 0,
                 tstore, err, spin, stall);
    }
    return true;
}

// ---------------------------------------------------------------------------------------------
// int8 tensor-core peak probe: each CTA (one per SM) issues tcgen05.mma.kind::i8 with M = 128,
// N = 256, K = 32 from zero-filled shared-memory operands (the same 128-byte-swizzled K-major
// layout as the matmul's stages), `issuers` threads per CTA into their own 256-column TMEM
// accumulators, then waits (bounded) for the last MMA and frees TMEM.  The operands' values do
// not change the instruction's cost.
// ---------------------------------------------------------------------------------------------
constexpr int PB_N = 256;
constexpr int PB_A = BM * 128;     // 16 KB: 128 rows x 128 B (four K-steps of 32)
constexpr int PB_B = PB_N * 128;   // 32 KB
// more shared memory than two CTAs can share, so each SM runs one probe CTA
constexpr int PB_SMEM = 120 * 1024;
constexpr uint32_t kIdescProbe =
    (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(PB_N >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

__global__ void __launch_bounds__(64, 1) k_probe_i8_mma(int iters, int issuers, int32_t* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* bar = (uint64_t*)(smem + PB_A + PB_B);
    uint32_t* holder = (uint32_t*)(bar + 1);
    const int tid = threadIdx.x, warp = tid >> 5;
    for (int i = tid; i < (PB_A + PB_B) / 16; i += blockDim.x) reinterpret_cast<int4*>(smem)[i] = make_int4(0, 0, 0, 0);
    if (tid == 0) {
        bar_init(smem_u32(bar), (uint32_t)issuers);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    if (warp == 0) {
        __syncwarp();
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(holder)),
                     "r"(TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
    }
    fence_proxy_async_smem();   // the zeroed operands are read by the tensor core (async proxy)
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *holder;
    if ((tid & 31) == 0 && warp < issuers) {
        const uint64_t a0 = sdesc(smem_u32(smem)), b0 = sdesc(smem_u32(smem + PB_A));
        const uint32_t d = tmem + (uint32_t)(warp * PB_N);
        for (int it = 0; it < iters; ++it)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
                tc_mma_i8(d, a0 + (uint64_t)((kk * 32) >> 4), b0 + (uint64_t)((kk * 32) >> 4), kIdescProbe,
                          (it | kk) ? 1u : 0u);
        tc_commit(smem_u32(bar));
        const long long t0 = clock64();
        bool done = false;
        while (!(done = bar_try(smem_u32(bar), 0)) && clock64() - t0 < kSpinCycles) {}
        if (!done && err) atomicExch(err, kErrTimeout);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
}

}  // namespace tc

// One launch of the probe on every SM of the current device; *ctas = CTAs launched.
bool probe_i8_mma(int iters, int issuers, int32_t* err, cudaStream_t st, int* ctas) {
    if (iters <= 0 || issuers < 1 || issuers > 2) return false;
    static PerDeviceOnce setup;
    int n_sm = 0;
    if (!setup.ensure([](int dev, int* sms) {
            if (cudaFuncSetAttribute(tc::k_probe_i8_mma, cudaFuncAttributeMaxDynamicSharedMemorySize, tc::PB_SMEM) != cudaSuccess)
                return false;
            return cudaDeviceGetAttribute(sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && *sms > 0;
        }, &n_sm))
        return false;
    tc::k_probe_i8_mma<<<n_sm, 64, tc::PB_SMEM, st>>>(iters, issuers, err);
    if (ctas) *ctas = n_sm;
    return cudaGetLastError() == cudaSuccess;
}

bool matmul_tc(const DevW& W, const ActQ& a, int M, const float* bias, int relu, float* y, const QKVStore* qkv,
               cudaStream_t st) {
    if (W.type != W_Q4_K || !W.tcw || !a.q || W.K % 256 != 0 || M <= 0) return false;
    return tc::launch_q4k(W, a, M, bias, relu, y, qkv, st);
}

}  // namespace t2sx
