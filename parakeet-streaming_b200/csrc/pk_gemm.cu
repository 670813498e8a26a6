// bf16 GEMM on the 5th-generation tensor cores with the encoder's epilogues.
//
//   C[m][n] = epilogue( sum_k A[m][k] * W[n][k] ),  A, W, C bf16, fp32 accumulation
//   epilogue: store | SiLU | R[m][n] + alpha * acc (optionally ReLU'd) | acc + bias[n]
//
// These are the Conformer layer's projections (parakeet/modules/feedforward.py:
// Linear -> SiLU -> Linear; attention.py qkv / linear_out; convolution.py
// pointwise convs), with the activation and the residual add of
// ConformerLayer.forward (encoder.py:60-81: x + 0.5 * ff, x + attn, x + conv)
// done on the accumulator instead of by separate elementwise launches.
//
// One CTA computes a 128 x BN tile (128 threads).  Lane 0 of warp 0 streams
// 64-wide K blocks of A and W into a ring of NS shared-memory stages with TMA
// (128B swizzle, the layout the tensor-core descriptors read); lane 0 of warp 1
// issues tcgen05.mma (M = 128, N = BN, K = 16, four per stage) into a TMEM
// accumulator of BN fp32 columns and releases each stage with tcgen05.commit;
// after the last commit all four warps read their 32 TMEM lanes (= tile rows)
// with tcgen05.ld, apply the epilogue and store.  The weights do not depend on
// the previous kernel, so their first stages are requested before the
// programmatic-dependent-launch wait.  Every wait is bounded (PK_DEV_TIMEOUT).
#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {
namespace {

constexpr int kBM = 128, kBK = 64, kThreads = 128;
constexpr int kABytes = kBM * kBK * 2;   // 16 KB per stage

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar,
                                            int32_t c0, int32_t c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}

// Shared-memory matrix descriptor of a K-major operand tile written by TMA
// with 128B swizzle (rows of 128 bytes, 8-row swizzle atoms of 1024 bytes):
// start address >> 4, leading byte offset 1 (unused for swizzled K-major),
// stride byte offset 1024 >> 4 between 8-row groups, descriptor version 1,
// layout type 2 = 128B swizzle.  The tile base is 1024-byte aligned, so the
// base offset is 0; a K step of 16 elements inside the atom advances the start
// address by 32 bytes.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) |
           ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor, kind::f16: D fp32 (bits 4-5 = 1), A and B bf16
// (bits 7-9, 10-12 = 1), both K-major (bits 15, 16 = 0), N >> 3 at bit 17,
// M >> 4 at bit 24.
constexpr uint32_t idesc_bf16(int m, int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) |
           ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mbar_arrive_cta(uint64_t *bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// arrive on `bar` when every tcgen05.mma issued so far by this thread is done
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t *dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
        "%28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Epilogue staging: each epilogue warp owns a 32-row tile of 64 bf16 columns
// in shared memory (rows padded to 144 bytes: a row-per-lane 16-byte access
// and a row-segment access are both free of bank conflicts).
constexpr int kStageRow = 144;
constexpr int kStageBytes = 32 * kStageRow;

// The epilogue of accumulator columns [col, col + 64) of the warp's tile rows
// row0 .. row0 + 31 (TMEM lane l of taddr = row row0 + l).  The arithmetic runs
// a row per lane, as the accumulator comes out of TMEM; the residual rows are
// read and the output rows written through the warp's staging tile as whole
// 128-byte row segments (four rows per warp access), where a row per lane would
// touch 32 rows per access.
constexpr bool is_residual(int epi) {
    return epi == PK_GEMM_RESIDUAL || epi == PK_GEMM_RESIDUAL_RELU;
}

// This lane's share of the residual rows of the same 64 columns, as row
// segments (piece i: row row0 + 4 i + lane / 8, bytes (lane % 8) * 16 ..):
// loaded ahead of the columns' epilogue so that the load latency overlaps work.
__device__ __forceinline__ void load_residual64(uint4 (&rv)[8], int row0, int M, int col,
                                                const __nv_bfloat16 *R, int64_t ldr) {
    const int lane = threadIdx.x & 31;
    const int sr = lane >> 3, sb = (lane & 7) * 16;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int r = i * 4 + sr;
        rv[i] = make_uint4(0u, 0u, 0u, 0u);
        if (row0 + r < M)
            rv[i] = *reinterpret_cast<const uint4 *>(
                reinterpret_cast<const char *>(R + (int64_t)(row0 + r) * ldr + col) + sb);
    }
}

template <int EPI>
__device__ __forceinline__ void epilogue_tile64(uint32_t taddr, int row0, int M, int col,
                                                __nv_bfloat16 *C, int64_t ldc,
                                                const uint4 (&rv)[8], const __nv_bfloat16 *bias,
                                                float alpha, uint8_t *stage) {
    constexpr bool kRes = is_residual(EPI);
    const int lane = threadIdx.x & 31;
    const int sr = lane >> 3, sb = (lane & 7) * 16;   // row-segment phase: row in 4, byte
    if (kRes) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
            *reinterpret_cast<uint4 *>(stage + (i * 4 + sr) * kStageRow + sb) = rv[i];
    }
    float v[64];
    tmem_ld32(taddr, *reinterpret_cast<float(*)[32]>(v));
    tmem_ld32(taddr + 32, *reinterpret_cast<float(*)[32]>(v + 32));
    __syncwarp();   // residual rows staged
    uint8_t *mine = stage + lane * kStageRow;
    if (EPI == PK_GEMM_SILU) {
#pragma unroll
        for (int i = 0; i < 64; ++i) v[i] = __fdividef(v[i], 1.f + __expf(-v[i]));
    } else if (kRes) {
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            float f[8];
            unpack16(*reinterpret_cast<const uint4 *>(mine + q * 16), f, bias);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float t = f[i] + alpha * v[q * 8 + i];
                v[q * 8 + i] = EPI == PK_GEMM_RESIDUAL_RELU ? fmaxf(t, 0.f) : t;
            }
        }
    } else if (EPI == PK_GEMM_BIAS) {
        const uint4 *bp = reinterpret_cast<const uint4 *>(bias + col);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            float f[8];
            unpack16(bp[q], f, bias);
#pragma unroll
            for (int i = 0; i < 8; ++i) v[q * 8 + i] += f[i];
        }
    }
    __syncwarp();   // every lane's residual row read
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        uint4 o;
        __nv_bfloat162 *h = reinterpret_cast<__nv_bfloat162 *>(&o);
#pragma unroll
        for (int i = 0; i < 4; ++i)
            h[i] = __floats2bfloat162_rn(v[q * 8 + 2 * i], v[q * 8 + 2 * i + 1]);
        *reinterpret_cast<uint4 *>(mine + q * 16) = o;
    }
    __syncwarp();   // output rows staged
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int r = i * 4 + sr;
        if (row0 + r < M)
            *reinterpret_cast<uint4 *>(reinterpret_cast<char *>(C + (int64_t)(row0 + r) * ldc + col) +
                                       sb) = *reinterpret_cast<const uint4 *>(stage + r * kStageRow + sb);
    }
    __syncwarp();   // staging tile free again
}

template <int BN, int NS, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_w,
                     int M, int K, __nv_bfloat16 *C, int64_t ldc, const __nv_bfloat16 *R,
                     int64_t ldr, const __nv_bfloat16 *bias, float alpha, int32_t *error) {
    constexpr int kBBytes = BN * kBK * 2;
    extern __shared__ uint8_t gemm_smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(gemm_smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem, *sB = smem + NS * kABytes;
    __shared__ __align__(8) uint64_t full[NS], empty[NS], done;
    __shared__ uint32_t tmem_base;
    __shared__ int failed;

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int m0 = blockIdx.y * kBM, n0 = blockIdx.x * BN;
    const int nk = K / kBK;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(&done, 1);
        failed = 0;
        fence_mbar_init();
        prefetch_tmap(&tm_a);
        prefetch_tmap(&tm_w);
    }
    if (warp == 0) {
        tmem_alloc(&tmem_base, BN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;

    if (warp == 0 && lane == 0) {
        // producer: the weights of the first stages before the wait on the
        // previous kernel (they are constants), then A, then the steady ring
        const int pre = nk < NS ? nk : NS;
        for (int kb = 0; kb < pre; ++kb) {
            mbar_arrive_expect_tx(&full[kb], kABytes + kBBytes);
            tma_load_2d(sB + kb * kBBytes, &tm_w, &full[kb], kb * kBK, n0);
        }
        grid_dep_wait();
        for (int kb = 0; kb < pre; ++kb)
            tma_load_2d(sA + kb * kABytes, &tm_a, &full[kb], kb * kBK, m0);
        for (int kb = NS; kb < nk; ++kb) {
            const int s = kb % NS;
            if (!mbar_wait_bounded(&empty[s], ((kb / NS) - 1) & 1, kWaitLimitNs)) {
                raise(error, PK_DEV_TIMEOUT);
                failed = 1;
                break;
            }
            mbar_arrive_expect_tx(&full[s], kABytes + kBBytes);
            tma_load_2d(sB + s * kBBytes, &tm_w, &full[s], kb * kBK, n0);
            tma_load_2d(sA + s * kABytes, &tm_a, &full[s], kb * kBK, m0);
        }
    } else if (warp == 1 && lane == 0) {
        // MMA issuer
        constexpr uint32_t idesc = idesc_bf16(kBM, BN);
        grid_dep_wait();
        for (int kb = 0; kb < nk; ++kb) {
            const int s = kb % NS;
            if (!mbar_wait_bounded(&full[s], (kb / NS) & 1, kWaitLimitNs)) {
                raise(error, PK_DEV_TIMEOUT);
                failed = 1;
                break;
            }
            tc_fence_after();
            const uint32_t a0 = smem_u32(sA + s * kABytes), b0 = smem_u32(sB + s * kBBytes);
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)
                umma_bf16(tmem, sw128_desc(a0 + kk * 32), sw128_desc(b0 + kk * 32), idesc,
                          (kb | kk) != 0);
            umma_commit(&empty[s]);
        }
        umma_commit(&done);
    } else {
        grid_dep_wait();   // the residual rows may come from the previous kernel
    }
    __syncwarp();

    // epilogue: warp w owns TMEM lanes (tile rows) 32w .. 32w + 31; the first
    // residual columns are requested while the MMAs still run
    uint4 rv[8], rn[8];
    if (is_residual(EPI)) load_residual64(rn, m0 + warp * 32, M, n0, R, ldr);
    const bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(&done, 0, kWaitLimitNs));
    if (!ok && lane == 0) raise(error, PK_DEV_TIMEOUT);
    tc_fence_after();
    grid_dep_launch();
    if (ok && !failed) {
        // the stage ring is idle now (every MMA is done): it holds the staging tiles
        uint8_t *stage = smem + warp * kStageBytes;
#pragma unroll 1
        for (int c = 0; c < BN / 64; ++c) {
#pragma unroll
            for (int i = 0; i < 8; ++i) rv[i] = rn[i];
            if (is_residual(EPI) && c + 1 < BN / 64)
                load_residual64(rn, m0 + warp * 32, M, n0 + (c + 1) * 64, R, ldr);
            epilogue_tile64<EPI>(tmem + ((uint32_t)(warp * 32) << 16) + c * 64, m0 + warp * 32, M,
                                 n0 + c * 64, C, ldc, rv, bias, alpha, stage);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, BN);
    }
}

// Persistent form for many tiles: one CTA per SM walks tiles t = blockIdx.x +
// k * gridDim.x (row tiles fastest, so the CTAs at work share a weight tile in
// L2).  Warp 0 lane 0 streams K blocks through the stage ring across tiles,
// warp 1 lane 0 issues the MMAs into one of two TMEM accumulators (2 x BN
// columns), and warps 2-5 drain the other accumulator through the epilogue, so
// a tile's epilogue runs under the next tile's mainloop.  tmem_full[a] (MMA ->
// epilogue, by tcgen05.commit) and tmem_empty[a] (4 epilogue warps -> MMA)
// hand the accumulators over.  Warp w of the epilogue reads TMEM lanes
// 32 * (w % 4) .. + 31.
constexpr int kPThreads = 192;

template <int BN, int NS, int EPI>
__global__ void __launch_bounds__(kPThreads, 1)
    gemm_bf16_persistent_kernel(const __grid_constant__ CUtensorMap tm_a,
                                const __grid_constant__ CUtensorMap tm_w, int M, int N, int K,
                                __nv_bfloat16 *C, int64_t ldc, const __nv_bfloat16 *R, int64_t ldr,
                                const __nv_bfloat16 *bias, float alpha, int32_t *error) {
    constexpr int kBBytes = BN * kBK * 2;
    extern __shared__ uint8_t gemm_smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(gemm_smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem, *sB = smem + NS * kABytes;
    __shared__ __align__(8) uint64_t full[NS], empty[NS], tmem_full[2], tmem_empty[2];
    __shared__ uint32_t tmem_base;
    __shared__ volatile int failed;

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    uint8_t *stage = sB + NS * kBBytes + (warp & 3) * kStageBytes;   // epilogue warps
    const int mtiles = (M + kBM - 1) / kBM, tiles = mtiles * (N / BN), nk = K / kBK;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tmem_full[a], 1);
            mbar_init(&tmem_empty[a], 4);
        }
        failed = 0;
        fence_mbar_init();
        prefetch_tmap(&tm_a);
        prefetch_tmap(&tm_w);
    }
    if (warp == 0) {
        tmem_alloc(&tmem_base, 2 * BN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            // producer: K blocks of every tile of this CTA through the ring
            grid_dep_wait();
            int g = 0;
            for (int tile = blockIdx.x; tile < tiles && !failed; tile += gridDim.x) {
                const int m0 = (tile % mtiles) * kBM, n0 = (tile / mtiles) * BN;
                for (int kb = 0; kb < nk; ++kb, ++g) {
                    const int s = g % NS, u = g / NS;
                    if (u >= 1 && !mbar_wait_bounded(&empty[s], (u - 1) & 1, kWaitLimitNs)) {
                        raise(error, PK_DEV_TIMEOUT);
                        failed = 1;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[s], kABytes + kBBytes);
                    tma_load_2d(sB + s * kBBytes, &tm_w, &full[s], kb * kBK, n0);
                    tma_load_2d(sA + s * kABytes, &tm_a, &full[s], kb * kBK, m0);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // MMA issuer: accumulator t & 1 for the CTA's t-th tile
            constexpr uint32_t idesc = idesc_bf16(kBM, BN);
            int g = 0, t = 0;
            for (int tile = blockIdx.x; tile < tiles && !failed; tile += gridDim.x, ++t) {
                const int acc = t & 1, use = t >> 1;
                if (use >= 1 && !mbar_wait_bounded(&tmem_empty[acc], (use - 1) & 1, kWaitLimitNs)) {
                    raise(error, PK_DEV_TIMEOUT);
                    failed = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + acc * BN;
                for (int kb = 0; kb < nk; ++kb, ++g) {
                    const int s = g % NS;
                    if (!mbar_wait_bounded(&full[s], (g / NS) & 1, kWaitLimitNs)) {
                        raise(error, PK_DEV_TIMEOUT);
                        failed = 1;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sA + s * kABytes), b0 = smem_u32(sB + s * kBBytes);
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk)
                        umma_bf16(d, sw128_desc(a0 + kk * 32), sw128_desc(b0 + kk * 32), idesc,
                                  (kb | kk) != 0);
                    umma_commit(&empty[s]);
                }
                umma_commit(&tmem_full[acc]);
            }
        }
    } else {
        // epilogue warps 2..5
        grid_dep_wait();   // the residual rows may come from the previous kernel
        const int q = warp & 3;
        int t = 0;
        uint4 rv[8], rn[8];
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++t) {
            const int acc = t & 1, use = t >> 1;
            const int m0 = (tile % mtiles) * kBM, n0 = (tile / mtiles) * BN;
            // the tile's first residual columns are requested while its MMAs run
            if (is_residual(EPI)) load_residual64(rn, m0 + q * 32, M, n0, R, ldr);
            const bool ok = __all_sync(0xffffffffu,
                                       mbar_wait_bounded(&tmem_full[acc], use & 1, kWaitLimitNs));
            if (!ok) {
                if (lane == 0) raise(error, PK_DEV_TIMEOUT);
                failed = 1;
                break;
            }
            tc_fence_after();
            if (tile + (int)gridDim.x >= tiles) grid_dep_launch();
#pragma unroll 1
            for (int c = 0; c < BN / 64; ++c) {
#pragma unroll
                for (int i = 0; i < 8; ++i) rv[i] = rn[i];
                if (is_residual(EPI) && c + 1 < BN / 64)
                    load_residual64(rn, m0 + q * 32, M, n0 + (c + 1) * 64, R, ldr);
                epilogue_tile64<EPI>(tmem + acc * BN + ((uint32_t)(q * 32) << 16) + c * 64,
                                     m0 + q * 32, M, n0 + c * 64, C, ldc, rv, bias, alpha, stage);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cta(&tmem_empty[acc]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 2 * BN);
    }
}

// ---------------------------------------------------------------------------
// CTA-pair form (tcgen05.mma.cta_group::2): a cluster of two CTAs on two SMs
// computes a 256 x BN tile with M = 256 MMAs.  CTA r of the pair loads rows
// m0 + 128 r .. + 127 of A and rows n0 + (BN/2) r .. of W into its own shared
// memory (plain TMA tile loads, no multicast); the MMA issued by the pair's
// even CTA reads A from each CTA's own stage and B from both, and writes rows
// 128 r .. of the tile to CTA r's TMEM.  Each SM thus streams 128 + BN/2
// operand rows per K block for a 128 x BN product, where a one-CTA tile streams
// 128 + BN.  Both CTAs' loads complete on the even CTA's full[s] barrier (the
// .cta_group::2 form of the TMA load may signal the peer's barrier); the MMA
// commits release stage s in both CTAs (commit multicast to both empty[s]) and
// hand each accumulator to both CTAs' epilogue warps (tmem_full[a]); all eight
// epilogue warps of the pair return an accumulator on the even CTA's
// tmem_empty[a].  Tiles are walked persistently, row tiles fastest.

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// shared::cluster address of the same shared-memory object in CTA `rank`
__device__ __forceinline__ uint32_t mapa_rank(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// arrive on an mbarrier of either CTA of the cluster (release at cluster scope)
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "n"(kSuspendNs)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster_bounded(uint64_t *bar, uint32_t parity,
                                                          uint64_t limit_ns) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait_cluster(bar, parity)) {
        if (globaltimer_ns() - t0 > limit_ns) return false;
    }
    return true;
}
// 2-D tile load into this CTA's shared memory, completion on an mbarrier of
// either CTA of the pair (bar: shared::cluster address)
__device__ __forceinline__ void tma_load_2d_pair(void *dst, const CUtensorMap *map, uint32_t bar,
                                                 int32_t c0, int32_t c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void umma_bf16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                               uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// arrive on `bar` (same offset) in both CTAs of the pair when the MMAs issued so
// far by this thread are done
__device__ __forceinline__ void umma_commit_pair(uint64_t *bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
        " [%0], %1;" ::"r"(smem_u32(bar)),
        "h"((uint16_t)0x3)
        : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t *dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

template <int BN, int NS, int EPI>
__global__ void __launch_bounds__(kPThreads, 1)
    gemm_bf16_pair_kernel(const __grid_constant__ CUtensorMap tm_a,
                          const __grid_constant__ CUtensorMap tm_w, int M, int N, int K,
                          __nv_bfloat16 *C, int64_t ldc, const __nv_bfloat16 *R, int64_t ldr,
                          const __nv_bfloat16 *bias, float alpha, int32_t *error) {
    constexpr int kHalfB = BN / 2;                  // W rows per CTA
    constexpr int kBBytes = kHalfB * kBK * 2;
    constexpr uint32_t kStageTx = 2 * (kABytes + kBBytes);   // both CTAs' loads
    extern __shared__ uint8_t gemm_smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(gemm_smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem, *sB = smem + NS * kABytes;
    __shared__ __align__(8) uint64_t full[NS], empty[NS], tmem_full[2], tmem_empty[2];
    __shared__ uint32_t tmem_base;
    __shared__ volatile int failed;

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    uint8_t *stage = sB + NS * kBBytes + (warp & 3) * kStageBytes;   // epilogue warps
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int pair = blockIdx.x / 2, npairs = gridDim.x / 2;
    const int mtiles = (M + 2 * kBM - 1) / (2 * kBM), tiles = mtiles * (N / BN), nk = K / kBK;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tmem_full[a], 1);
            mbar_init(&tmem_empty[a], 8);   // 4 epilogue warps in each CTA of the pair
        }
        failed = 0;
        fence_mbar_init();
        prefetch_tmap(&tm_a);
        prefetch_tmap(&tm_w);
    }
    if (warp == 0) {
        tmem_alloc_pair(&tmem_base, 2 * BN);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync_all();   // both CTAs' barriers initialised and TMEM allocated
    tc_fence_after();
    const uint32_t tmem = tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            // producer: this CTA's halves of every K block of the pair's tiles
            grid_dep_wait();
            int g = 0;
            for (int tile = pair; tile < tiles && !failed; tile += npairs) {
                const int m0 = (tile % mtiles) * 2 * kBM + (int)rank * kBM;
                const int n0 = (tile / mtiles) * BN + (int)rank * kHalfB;
                for (int kb = 0; kb < nk; ++kb, ++g) {
                    const int s = g % NS, u = g / NS;
                    if (u >= 1 && !mbar_wait_bounded(&empty[s], (u - 1) & 1, kWaitLimitNs)) {
                        raise(error, PK_DEV_TIMEOUT);
                        failed = 1;
                        break;
                    }
                    const uint32_t fb = mapa_rank(smem_u32(&full[s]), 0);
                    if (leader) mbar_arrive_expect_tx(&full[s], kStageTx);
                    tma_load_2d_pair(sB + s * kBBytes, &tm_w, fb, kb * kBK, n0);
                    tma_load_2d_pair(sA + s * kABytes, &tm_a, fb, kb * kBK, m0);
                }
            }
            if (leader) {   // leave none of the pair's loads in flight
                for (int s = 0; s < NS; ++s)
                    if (g > s) {
                        const int last = g - 1 - (g - 1 - s) % NS;
                        mbar_wait_bounded(&full[s], (last / NS) & 1, kWaitLimitNs);
                    }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            // MMA issuer of the pair: accumulator t & 1 for the pair's t-th tile
            constexpr uint32_t idesc = idesc_bf16(2 * kBM, BN);
            int g = 0, t = 0;
            for (int tile = pair; tile < tiles && !failed; tile += npairs, ++t) {
                const int acc = t & 1, use = t >> 1;
                if (use >= 1 &&
                    !mbar_wait_cluster_bounded(&tmem_empty[acc], (use - 1) & 1, kWaitLimitNs)) {
                    raise(error, PK_DEV_TIMEOUT);
                    failed = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + acc * BN;
                for (int kb = 0; kb < nk; ++kb, ++g) {
                    const int s = g % NS;
                    if (!mbar_wait_bounded(&full[s], (g / NS) & 1, kWaitLimitNs)) {
                        raise(error, PK_DEV_TIMEOUT);
                        failed = 1;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sA + s * kABytes), b0 = smem_u32(sB + s * kBBytes);
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk)
                        umma_bf16_pair(d, sw128_desc(a0 + kk * 32), sw128_desc(b0 + kk * 32), idesc,
                                       (kb | kk) != 0);
                    umma_commit_pair(&empty[s]);
                }
                if (failed) break;
                umma_commit_pair(&tmem_full[acc]);
            }
        }
    } else {
        // epilogue warps 2..5: TMEM lanes 32 (w % 4) .. = tile rows 128 rank + 32 (w % 4) ..
        grid_dep_wait();   // the residual rows may come from the previous kernel
        const int q = warp & 3;
        const uint32_t empty0 = mapa_rank(smem_u32(&tmem_empty[0]), 0),
                       empty1 = mapa_rank(smem_u32(&tmem_empty[1]), 0);
        int t = 0;
        uint4 rv[8], rn[8];
        for (int tile = pair; tile < tiles; tile += npairs, ++t) {
            const int acc = t & 1, use = t >> 1;
            const int m0 = (tile % mtiles) * 2 * kBM + (int)rank * kBM, n0 = (tile / mtiles) * BN;
            // the tile's first residual columns are requested while its MMAs run
            if (is_residual(EPI)) load_residual64(rn, m0 + q * 32, M, n0, R, ldr);
            const bool ok = __all_sync(0xffffffffu,
                                       mbar_wait_bounded(&tmem_full[acc], use & 1, kWaitLimitNs));
            if (!ok) {
                if (lane == 0) raise(error, PK_DEV_TIMEOUT);
                failed = 1;
                break;
            }
            tc_fence_after();
            if (tile + npairs >= tiles) grid_dep_launch();
#pragma unroll 1
            for (int c = 0; c < BN / 64; ++c) {
#pragma unroll
                for (int i = 0; i < 8; ++i) rv[i] = rn[i];
                if (is_residual(EPI) && c + 1 < BN / 64)
                    load_residual64(rn, m0 + q * 32, M, n0 + (c + 1) * 64, R, ldr);
                epilogue_tile64<EPI>(tmem + acc * BN + ((uint32_t)(q * 32) << 16) + c * 64,
                                     m0 + q * 32, M, n0 + c * 64, C, ldc, rv, bias, alpha, stage);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(acc ? empty1 : empty0);
        }
    }
    // every thread of both CTAs gets here: the pair's MMAs, loads and TMEM reads
    // are done before either CTA frees its TMEM columns or leaves
    tc_fence_before();
    __syncthreads();
    cluster_sync_all();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, 2 * BN);
    }
}

template <int BN, int NS, int EPI>
int launch_gemm_pair_t(const GemmArgs &g, const CUtensorMap &ta, const CUtensorMap &tw,
                       int num_sms, cudaStream_t s) {
    auto k = gemm_bf16_pair_kernel<BN, NS, EPI>;
    const size_t smem = (size_t)NS * (kABytes + (BN / 2) * kBK * 2) + 4 * kStageBytes + 1024;
    static bool attr = false;
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(gemm pair)");
        attr = true;
    }
    const int tiles = ((g.M + 2 * kBM - 1) / (2 * kBM)) * (g.N / BN);
    const int pairs = tiles < num_sms / 2 ? tiles : num_sms / 2;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pairs);
    cfg.blockDim = dim3(kPThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attrs[2];
    attrs[0].id = cudaLaunchAttributeClusterDimension;
    attrs[0].val.clusterDim.x = 2;
    attrs[0].val.clusterDim.y = 1;
    attrs[0].val.clusterDim.z = 1;
    attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attrs;
    cfg.numAttrs = 2;
    cudaError_t e = cudaLaunchKernelEx(&cfg, k, ta, tw, g.M, g.N, g.K,
                                       static_cast<__nv_bfloat16 *>(g.C), g.ldc,
                                       static_cast<const __nv_bfloat16 *>(g.R), g.ldr,
                                       static_cast<const __nv_bfloat16 *>(g.bias), g.alpha, g.error);
    return cuda_status(e, "gemm_bf16_pair_kernel");
}

template <int BN, int NS>
int launch_gemm_pair(const GemmArgs &g, const CUtensorMap &ta, const CUtensorMap &tw, int num_sms,
                     cudaStream_t s) {
    switch (g.epilogue) {
        case PK_GEMM_SILU: return launch_gemm_pair_t<BN, NS, PK_GEMM_SILU>(g, ta, tw, num_sms, s);
        case PK_GEMM_RESIDUAL:
            return launch_gemm_pair_t<BN, NS, PK_GEMM_RESIDUAL>(g, ta, tw, num_sms, s);
        case PK_GEMM_RESIDUAL_RELU:
            return launch_gemm_pair_t<BN, NS, PK_GEMM_RESIDUAL_RELU>(g, ta, tw, num_sms, s);
        case PK_GEMM_BIAS: return launch_gemm_pair_t<BN, NS, PK_GEMM_BIAS>(g, ta, tw, num_sms, s);
        default: return launch_gemm_pair_t<BN, NS, PK_GEMM_STORE>(g, ta, tw, num_sms, s);
    }
}

template <int BN, int NS, int EPI>
int launch_gemm_persistent_t(const GemmArgs &g, const CUtensorMap &ta, const CUtensorMap &tw,
                             int num_sms, cudaStream_t s) {
    auto k = gemm_bf16_persistent_kernel<BN, NS, EPI>;
    const size_t smem = (size_t)NS * (kABytes + BN * kBK * 2) + 4 * kStageBytes + 1024;
    static bool attr = false;
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(gemm persistent)");
        attr = true;
    }
    const int tiles = ((g.M + kBM - 1) / kBM) * (g.N / BN);
    const dim3 grid(tiles < num_sms ? tiles : num_sms);
    cudaError_t e = launch_pdl(k, grid, dim3(kPThreads), smem, s, ta, tw, g.M, g.N, g.K,
                               static_cast<__nv_bfloat16 *>(g.C), g.ldc,
                               static_cast<const __nv_bfloat16 *>(g.R), g.ldr,
                               static_cast<const __nv_bfloat16 *>(g.bias), g.alpha, g.error);
    return cuda_status(e, "gemm_bf16_persistent_kernel");
}

template <int BN, int NS>
int launch_gemm_persistent(const GemmArgs &g, const CUtensorMap &ta, const CUtensorMap &tw,
                           int num_sms, cudaStream_t s) {
    switch (g.epilogue) {
        case PK_GEMM_SILU:
            return launch_gemm_persistent_t<BN, NS, PK_GEMM_SILU>(g, ta, tw, num_sms, s);
        case PK_GEMM_RESIDUAL:
            return launch_gemm_persistent_t<BN, NS, PK_GEMM_RESIDUAL>(g, ta, tw, num_sms, s);
        case PK_GEMM_RESIDUAL_RELU:
            return launch_gemm_persistent_t<BN, NS, PK_GEMM_RESIDUAL_RELU>(g, ta, tw, num_sms, s);
        case PK_GEMM_BIAS:
            return launch_gemm_persistent_t<BN, NS, PK_GEMM_BIAS>(g, ta, tw, num_sms, s);
        default: return launch_gemm_persistent_t<BN, NS, PK_GEMM_STORE>(g, ta, tw, num_sms, s);
    }
}

template <int BN, int NS, int EPI>
int launch_gemm_t(const GemmArgs &g, const CUtensorMap &ta, const CUtensorMap &tw,
                  cudaStream_t s) {
    auto k = gemm_bf16_kernel<BN, NS, EPI>;
    const size_t smem = (size_t)NS * (kABytes + BN * kBK * 2) + 1024;
    static bool attr = false;
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(gemm)");
        attr = true;
    }
    const dim3 grid(g.N / BN, (g.M + kBM - 1) / kBM);
    cudaError_t e = launch_pdl(k, grid, dim3(kThreads), smem, s, ta, tw, g.M, g.K,
                               static_cast<__nv_bfloat16 *>(g.C), g.ldc,
                               static_cast<const __nv_bfloat16 *>(g.R), g.ldr,
                               static_cast<const __nv_bfloat16 *>(g.bias), g.alpha, g.error);
    return cuda_status(e, "gemm_bf16_kernel");
}

template <int BN, int NS>
int launch_gemm_epi(const GemmArgs &g, const CUtensorMap &ta, const CUtensorMap &tw,
                    cudaStream_t s) {
    switch (g.epilogue) {
        case PK_GEMM_SILU: return launch_gemm_t<BN, NS, PK_GEMM_SILU>(g, ta, tw, s);
        case PK_GEMM_RESIDUAL: return launch_gemm_t<BN, NS, PK_GEMM_RESIDUAL>(g, ta, tw, s);
        case PK_GEMM_RESIDUAL_RELU:
            return launch_gemm_t<BN, NS, PK_GEMM_RESIDUAL_RELU>(g, ta, tw, s);
        case PK_GEMM_BIAS: return launch_gemm_t<BN, NS, PK_GEMM_BIAS>(g, ta, tw, s);
        default: return launch_gemm_t<BN, NS, PK_GEMM_STORE>(g, ta, tw, s);
    }
}

}  // namespace

int launch_gemm(const GemmArgs &g, cudaStream_t s) {
    if (g.M == 0) return PK_OK;
    static int num_sms = 0;
    if (num_sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            num_sms = 148;
    }
    // N tile: narrow tiles when there are few row tiles (more CTAs for the
    // weight stream), wide ones otherwise; with more 256-wide tiles than two
    // waves the persistent kernel takes over
    const int mtiles = (g.M + kBM - 1) / kBM;
    int bn = mtiles * (g.N / 256) >= 148 && g.N % 256 == 0 ? 256
             : (mtiles * (g.N / 128) >= 148 && g.N % 128 == 0 ? 128 : 64);
    // persistent when the tiles make more than two waves: 256-wide, or 128-wide
    // when the 256-wide tiling is too short (an N = 1024 output)
    int pbn = 0;
    if (g.N % 256 == 0 && mtiles * (g.N / 256) >= 2 * num_sms) pbn = 256;
    else if (g.N % 128 == 0 && mtiles * (g.N / 128) >= 2 * num_sms) pbn = 128;
    if (pbn) bn = pbn;
    CUtensorMap ta, tw;
    const uint64_t adims[2] = {(uint64_t)g.K, (uint64_t)g.M}, astr[1] = {(uint64_t)g.lda * 2};
    const uint64_t wdims[2] = {(uint64_t)g.K, (uint64_t)g.N}, wstr[1] = {(uint64_t)g.ldw * 2};
    const uint32_t abox[2] = {kBK, kBM}, wbox[2] = {kBK, (uint32_t)bn};
    int st = encode_tmap(&ta, PK_DTYPE_BF16, g.A, 2, adims, astr, abox);
    if (st != PK_OK) return st;
    st = encode_tmap(&tw, PK_DTYPE_BF16, g.W, 2, wdims, wstr, wbox);
    if (st != PK_OK) return st;
    // CTA pairs (256 x 256 tiles on two SMs) when the pair tiles fill a wave of
    // pairs and either their waves are at least 80 % full or K is long (measured:
    // a 1.3- or 1.46-wave grid of short-K pair tiles is slower than one-CTA tiles)
    const int mt2 = (g.M + 2 * kBM - 1) / (2 * kBM), pairs = num_sms / 2;
    const int t2 = g.N % 256 == 0 ? mt2 * (g.N / 256) : 0;
    const bool full_waves = t2 >= pairs && 5 * t2 >= 4 * pairs * ((t2 + pairs - 1) / pairs);
    if (t2 >= pairs && (full_waves || g.K >= 2048)) {
        CUtensorMap tw2;
        const uint32_t wbox2[2] = {kBK, 128};
        st = encode_tmap(&tw2, PK_DTYPE_BF16, g.W, 2, wdims, wstr, wbox2);
        if (st != PK_OK) return st;
        return launch_gemm_pair<256, 6>(g, ta, tw2, num_sms, s);
    }
    if (pbn == 256) return launch_gemm_persistent<256, 4>(g, ta, tw, num_sms, s);
    if (pbn == 128) return launch_gemm_persistent<128, 6>(g, ta, tw, num_sms, s);
    // more tiles than SMs but not two waves of them: a shallower ring (96 KB of
    // stages) lets two CTAs share an SM, so the grid runs as one wave
    const int ctas = mtiles * (g.N / bn);
    if (ctas > num_sms && ctas <= 2 * num_sms) {
        switch (bn) {
            case 256: return launch_gemm_epi<256, 2>(g, ta, tw, s);
            case 128: return launch_gemm_epi<128, 3>(g, ta, tw, s);
            default: return launch_gemm_epi<64, 4>(g, ta, tw, s);
        }
    }
    switch (bn) {
        case 256: return launch_gemm_epi<256, 3>(g, ta, tw, s);
        case 128: return launch_gemm_epi<128, 4>(g, ta, tw, s);
        default: return launch_gemm_epi<64, 6>(g, ta, tw, s);
    }
}

}  // namespace pk
