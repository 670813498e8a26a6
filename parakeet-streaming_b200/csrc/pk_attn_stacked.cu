// Paged chunked rel-pos attention, bf16, for chunks where heads x chunk <= 16
// (the small streaming model: 8 heads x 2 frames): persistent CTAs, each item
// one (stream, layer) with all of its heads.
//
// Same computation as pk_attn.cu / pk_attn_bf16.cu (ConformerAttention.
// forward lines 99-122, parakeet/modules/attention.py; streaming mask of
// parakeet/modules/encoder.py:167-227).  With only T = 2 query rows per
// head, a per-head CTA spends most of its instructions on setup and on the
// padding rows of every m16 tile, and a per-(stream, layer) CTA that starts
// cold leaves DRAM idle while it resolves its window.  Here:
//
// * a producer warp walks the CTA's items and, per item, copies the window
//   descriptor into a double-buffered item slot and starts bulk async copies
//   (cp.async.bulk) of the item's query rows, new K/V rows and pos_bias_u/v
//   into it; then it streams 16 KB blocks through an NS-stage ring with
//   128B-swizzled TMA tile loads (cp.async.bulk.tensor, one box per head):
//   the K pages, the rel-pos rows in blocks of 16, the V pages - each page
//   box shifted so that rows outside the window are zero-filled without
//   being read.  The ring never drains between items;
// * consumer warp h owns head h: S = (q+u) K^T and BD = (q+v) P^T on tensor
//   cores (mma.sync m16n8k16, bf16 in, fp32 accumulate), stored in the
//   stacked [head * T + query] row order;
// * one dense softmax over all heads' rows (16 threads per row) with the
//   reference's -1e5 masked fill, probabilities kept as bf16 per page box;
// * O_h = P V_h on tensor cores, normalised by the row sums;
// * with new K/V rows given, each warp writes its head's rows into its page
//   in global memory and over the freshly landed box in shared memory: the
//   append costs no launch and no second read;
// * every mbarrier wait is bounded (1 s) and records PK_DEV_TIMEOUT.
#include <math.h>

#include <algorithm>

#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {
namespace {

constexpr int kH = 8;                    // heads = consumer warps
constexpr int kD = kH * 64;              // model width
constexpr int kTMax = 2;                 // chunk frames (kH * kTMax = 16 rows)
constexpr int kThreads = (kH + 1) * 32;  // + producer warp
constexpr int kBox = 2048;               // one head's 16 rows x 128 bytes
constexpr int kStage = kH * kBox;        // one block: every head's box
constexpr int kMaxBoxes = 8;             // pages per window handled
constexpr int kMaxPosBlocks = 8;         // rel-pos blocks of 16 rows (R <= 128)
constexpr int kPStride = 48;             // bytes per row of a 16x16 bf16 probability tile

// Per-item slot written by the producer (header by stores, rows by bulk copies)
struct ItemHdr {
    int ok, nb, w, nfirst, b, lrel, pad0, pad1;
    int start[kMaxBoxes];
    int page[kMaxBoxes];
    uint32_t mask[64];
};
constexpr uint32_t kSlotQ = 512;                     // [kTMax][kD] bf16
constexpr uint32_t kSlotK = kSlotQ + kTMax * kD * 2; // [kTMax][kD] bf16
constexpr uint32_t kSlotV = kSlotK + kTMax * kD * 2;
constexpr uint32_t kSlotU = kSlotV + kTMax * kD * 2; // [kD] bf16
constexpr uint32_t kSlotVB = kSlotU + kD * 2;
constexpr uint32_t kSlotBytes = ((kSlotVB + kD * 2) + 1023) / 1024 * 1024;
static_assert(sizeof(ItemHdr) <= kSlotQ, "item header too large");

struct SGeom {
    int num_layers, left, chunk, W, R, npb, max_boxes, items, batch;
    uint32_t off_slots, off_s, off_bd, off_p;
    int bd_stride;  // floats per stacked row of sBD
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void consumer_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kH * 32) : "memory");
}
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity) {
    return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity, kWaitLimitNs));
}

template <int NS>
__global__ void __launch_bounds__(kThreads, NS <= 4 ? 2 : 1)
    paged_attn_stacked_kernel(const __grid_constant__ CUtensorMap kv_map,
                              const __grid_constant__ CUtensorMap pos_map, const SGeom g,
                              const pk_paged_kv_desc d, const AttnArgs a) {
    using T = __nv_bfloat16;
    extern __shared__ char smem_raw[];
    char *smem = reinterpret_cast<char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                          ~uintptr_t(1023));
    __shared__ uint64_t full[NS], empty[NS], info_full[2], info_empty[2];
    __shared__ volatile int s_abort;
    __shared__ float s_rowsum[16];

    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    const int chunk = g.chunk, W = g.W, npb = g.npb;
    const bool has_kv = a.k_new != nullptr;
    char *slots = smem + g.off_slots;                           // [2][kSlotBytes]
    float *sS = reinterpret_cast<float *>(smem + g.off_s);      // [box][16 rows][16]
    float *sBD = reinterpret_cast<float *>(smem + g.off_bd);    // [16 rows][bd_stride]
    char *sP = smem + g.off_p;                                  // [box][16 rows][kPStride B]

    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kH);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&info_full[s], 1);
            mbar_init(&info_empty[s], kH);
        }
        s_abort = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kH) {
        // ============================ producer warp ============================
        if (lane == 0) {
            prefetch_tmap(&kv_map);
            prefetch_tmap(&pos_map);
        }
        int n = 0, k = 0;
        int last_n[NS];
#pragma unroll
        for (int s = 0; s < NS; ++s) last_n[s] = -1;
        int last_k[2] = {-1, -1};
        for (int item = blockIdx.x; item < g.items; item += gridDim.x, ++k) {
            const int slot = k & 1;
            if (k >= 2) {
                int got = 1;
                if (lane == 0) got = mbar_wait_bounded(&info_empty[slot], ((k >> 1) - 1) & 1, kWaitLimitNs);
                if (!__shfl_sync(0xffffffffu, got, 0)) {
                    if (lane == 0) {
                        raise(d.error, PK_DEV_TIMEOUT);
                        s_abort = 1;
                    }
                    break;
                }
            }
            const int b = item % g.batch, lrel = item / g.batch;
            const int layer = a.layer0 + lrel;
            char *sl = slots + slot * kSlotBytes;
            ItemHdr &hd = *reinterpret_cast<ItemHdr *>(sl);
            // window descriptor of this stream (written by pk_pages_begin_step)
            const int32_t *wd = d.window + (int64_t)b * PK_WIN_STRIDE;
            const int nb = wd[PK_WIN_NB];
            const int ok = wd[PK_WIN_OK] && nb <= g.max_boxes && nb <= kMaxBoxes;
            const int page = lane < kMaxBoxes ? wd[PK_WIN_PAGE + lane] : 0;
            const int start = lane < kMaxBoxes ? wd[PK_WIN_START + lane] : 0;
            hd.mask[lane] = (uint32_t)wd[PK_WIN_MASK + lane];
            hd.mask[32 + lane] = (uint32_t)wd[PK_WIN_MASK + 32 + lane];
            if (lane < kMaxBoxes) {
                hd.start[lane] = start;
                hd.page[lane] = page;
            }
            if (lane == 0) {
                hd.ok = ok;
                hd.nb = nb;
                hd.w = wd[PK_WIN_W];
                hd.nfirst = wd[PK_WIN_NFIRST];
                hd.b = b;
                hd.lrel = lrel;
            }
            __syncwarp();
            // rows of this item: query (+ new K, V) rows and the two position biases
            const uint32_t row_bytes = kD * 2;
            if (lane == 0) {
                const uint32_t bytes = ok ? (uint32_t)chunk * row_bytes * (has_kv ? 3 : 1) + 2 * row_bytes : 0;
                mbar_arrive_expect_tx(&info_full[slot], bytes);   // release: the header above
            }
            __syncwarp();
            if (ok) {
                const int64_t base = (int64_t)lrel * a.q_ls + (int64_t)b * a.q_bs;
                if (lane < chunk)
                    bulk_load(sl + kSlotQ + lane * row_bytes,
                              static_cast<const T *>(a.q) + base + (int64_t)lane * a.q_rs, row_bytes,
                              &info_full[slot]);
                if (has_kv && lane >= 8 && lane < 8 + chunk)
                    bulk_load(sl + kSlotK + (lane - 8) * row_bytes,
                              static_cast<const T *>(a.k_new) + base + (int64_t)(lane - 8) * a.q_rs,
                              row_bytes, &info_full[slot]);
                if (has_kv && lane >= 16 && lane < 16 + chunk)
                    bulk_load(sl + kSlotV + (lane - 16) * row_bytes,
                              static_cast<const T *>(a.v_new) + base + (int64_t)(lane - 16) * a.q_rs,
                              row_bytes, &info_full[slot]);
                if (lane == 30)
                    bulk_load(sl + kSlotU, static_cast<const T *>(a.bias_u) + (int64_t)lrel * a.bias_ls,
                              row_bytes, &info_full[slot]);
                if (lane == 31)
                    bulk_load(sl + kSlotVB, static_cast<const T *>(a.bias_v) + (int64_t)lrel * a.bias_ls,
                              row_bytes, &info_full[slot]);
            }
            last_k[slot] = k;
            if (!ok) continue;
            // blocks: K pages, rel-pos rows, V pages
            const int nblocks = 2 * nb + npb;
            bool stop = false;
            for (int q = 0; q < nblocks; ++q, ++n) {
                const int s = n % NS, u = n / NS;
                int got = 1;
                if (u >= 1 && lane == 0) got = mbar_wait_bounded(&empty[s], (u - 1) & 1, kWaitLimitNs);
                if (!__shfl_sync(0xffffffffu, got, 0)) {
                    if (lane == 0) {
                        raise(d.error, PK_DEV_TIMEOUT);
                        s_abort = 1;
                    }
                    stop = true;
                    break;
                }
                if (lane == 0) mbar_arrive_expect_tx(&full[s], kStage);
                __syncwarp();
                int kind, i;   // 0 = K page, 1 = rel-pos block, 2 = V page
                if (q < nb) {
                    kind = 0;
                    i = q;
                } else if (q < nb + npb) {
                    kind = 1;
                    i = q - nb;
                } else {
                    kind = 2;
                    i = q - nb - npb;
                }
                const int pg = __shfl_sync(0xffffffffu, page, i & 31);
                const int st = __shfl_sync(0xffffffffu, start, i & 31);
                if (lane < kH) {
                    char *dst = smem + s * kStage + lane * kBox;
                    if (kind == 1) {
                        tma_load_3d(dst, &pos_map, &full[s], lane * 64, i * 16, lrel);
                    } else {
                        const int plane = ((pg * d.num_layers + layer) * 2 + (kind == 2)) * kH + lane;
                        tma_load_3d(dst, &kv_map, &full[s], 0, st, plane);
                    }
                }
                last_n[s] = n;
            }
            if (stop) break;
        }
        if (lane == 0) {   // leave none of our copies in flight
#pragma unroll
            for (int s = 0; s < NS; ++s)
                if (last_n[s] >= 0) mbar_wait_bounded(&full[s], (last_n[s] / NS) & 1, kWaitLimitNs);
            for (int s = 0; s < 2; ++s)
                if (last_k[s] >= 0) mbar_wait_bounded(&info_full[s], (last_k[s] >> 1) & 1, kWaitLimitNs);
        }
        return;
    }

    // ============================ consumer warp h = head h ============================
    const int h = warp;
    const int gq = lane / 4, tq = lane % 4;
    const float scale = 0.125f;  // 1 / sqrt(64)
    const int bds = g.bd_stride;
    int n = 0, k = 0;
    for (int item = blockIdx.x; item < g.items; item += gridDim.x, ++k) {
        const int slot = k & 1;
        if (s_abort) break;
        if (!warp_wait(&info_full[slot], (k >> 1) & 1)) {
            if (lane == 0) {
                raise(d.error, PK_DEV_TIMEOUT);
                s_abort = 1;
            }
            break;
        }
        const char *sl = slots + slot * kSlotBytes;
        const ItemHdr &hd = *reinterpret_cast<const ItemHdr *>(sl);
        const int b = hd.b, lrel = hd.lrel, nb = hd.nb, w = hd.w, nfirst = hd.nfirst;
        const int layer = a.layer0 + lrel;
        T *out_base = static_cast<T *>(a.out) + (int64_t)lrel * a.o_ls + (int64_t)b * a.o_bs + h * 64;
        if (!hd.ok) {
            for (int idx = lane; idx < chunk * 64; idx += 32)
                out_base[(int64_t)(idx / 64) * a.o_rs + idx % 64] = __float2bfloat16_rn(0.f);
            __syncwarp();
            if (lane == 0) mbar_arrive(&info_empty[slot]);
            continue;
        }

        // A fragments: rows 0..chunk-1 of the m16 tile are this head's queries,
        // (q + u) and (q + v) rounded to bf16 as the reference's bf16 add is
        uint32_t fu[4][4], fv[4][4];
        {
            const T *qs = reinterpret_cast<const T *>(sl + kSlotQ) + h * 64;
            const T *us = reinterpret_cast<const T *>(sl + kSlotU) + h * 64;
            const T *vs = reinterpret_cast<const T *>(sl + kSlotVB) + h * 64;
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const int row = gq + (r & 1) * 8, col = ks * 16 + (r >> 1) * 8 + 2 * tq;
                    uint32_t pu = 0u, pv = 0u;
                    if (row < chunk) {
                        const float2 q = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(qs + row * kD + col));
                        const float2 u = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(us + col));
                        const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(vs + col));
                        __nv_bfloat162 xu = __floats2bfloat162_rn(q.x + u.x, q.y + u.y);
                        __nv_bfloat162 xv = __floats2bfloat162_rn(q.x + v.x, q.y + v.y);
                        pu = *reinterpret_cast<uint32_t *>(&xu);
                        pv = *reinterpret_cast<uint32_t *>(&xv);
                    }
                    fu[ks][r] = pu;
                    fv[ks][r] = pv;
                }
        }
        // write this step's rows of box i (K or V, head h) to the page and over the box
        auto append_rows = [&](uint32_t src_off, int kvi, int i, char *box) {
            for (int idx = lane; idx < chunk * 8; idx += 32) {
                const int t = idx / 8, c = idx % 8;
                const int av = w + t;
                if ((av >> 4) - nfirst != i) continue;
                const int pr = av & 15, r = pr - hd.start[i];
                const uint4 val = *reinterpret_cast<const uint4 *>(sl + src_off + (t * kD + h * 64 + c * 8) * 2);
                *reinterpret_cast<uint4 *>(box + sw128(r, c * 16)) = val;
                const int64_t plane = ((int64_t)(hd.page[i] * d.num_layers + layer) * 2 + kvi) * kH + h;
                *reinterpret_cast<uint4 *>(static_cast<T *>(d.kv) + (plane * 16 + pr) * 64 + c * 8) = val;
            }
            __syncwarp();
        };

        // ---- pass 1: K pages -> S rows, rel-pos blocks -> BD rows
        bool failed = false;
        for (int q = 0; q < nb + npb; ++q, ++n) {
            const int s = n % NS;
            if (!warp_wait(&full[s], (n / NS) & 1)) {
                if (lane == 0) {
                    raise(d.error, PK_DEV_TIMEOUT);
                    s_abort = 1;
                }
                failed = true;
                break;
            }
            char *box = smem + s * kStage + h * kBox;
            const uint32_t abox = smem_u32(box);
            const bool is_k = q < nb;
            if (is_k && has_kv) append_rows(kSlotK, 0, q, box);
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
                float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int kp = 0; kp < 4; kp += 2) {
                    uint32_t bb[4];
                    ldsm_x4(abox + sw128(nt * 8 + (lane % 8), (kp * 16 + (lane / 8) * 8) * 2), bb);
                    if (is_k) {
                        mma_bf16(c, fu[kp], bb[0], bb[1]);
                        mma_bf16(c, fu[kp + 1], bb[2], bb[3]);
                    } else {
                        mma_bf16(c, fv[kp], bb[0], bb[1]);
                        mma_bf16(c, fv[kp + 1], bb[2], bb[3]);
                    }
                }
                if (gq < chunk) {
                    float *dst = is_k ? sS + (q * 16 + h * chunk + gq) * 16 + nt * 8 + 2 * tq
                                      : sBD + (h * chunk + gq) * bds + (q - nb) * 16 + nt * 8 + 2 * tq;
                    *reinterpret_cast<float2 *>(dst) = make_float2(c[0], c[1]);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        consumer_sync();   // S and BD of every head complete (all warps reach this)
        if (s_abort || failed) break;

        // ---- dense softmax over the stacked rows: 16 threads per row
        {
            const int row = tid / 16, sub = tid % 16;
            const int rows = kH * chunk;
            const int iq = row % chunk;
            float sv[kMaxBoxes];
            float mx = -INFINITY;
#pragma unroll
            for (int i = 0; i < kMaxBoxes; ++i) {
                sv[i] = -INFINITY;
                if (i < nb && row < rows) {
                    const int pr = hd.start[i] + sub;
                    const int av = ((nfirst + i) << 4) + pr;
                    const int j = av - (w - g.left);
                    if (pr >= 0 && pr < 16 && av >= 0 && j >= 0 && j < W) {
                        const float c = sS[(i * 16 + row) * 16 + sub] * scale;
                        const bool allowed = (hd.mask[iq * 4 + (j >> 5)] >> (j & 31)) & 1u;
                        sv[i] = allowed ? c + sBD[row * bds + chunk - 1 - iq + j] * scale
                                        : c - 1e5f;   // masked_fill(-1e5), attention.py:115
                    }
                }
                mx = fmaxf(mx, sv[i]);
            }
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            float sum = 0.f;
#pragma unroll
            for (int i = 0; i < kMaxBoxes; ++i) {
                if (i < nb) {
                    const float p = sv[i] == -INFINITY ? 0.f : __expf(sv[i] - mx);
                    sum += p;
                    *reinterpret_cast<__nv_bfloat16 *>(sP + (i * 16 + row) * kPStride + sub * 2) =
                        __float2bfloat16_rn(p);
                }
            }
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
            if (sub == 0) s_rowsum[row] = sum;
        }
        consumer_sync();   // probabilities visible

        // ---- pass 2: O_h = P V_h over the V pages
        float o[4][2][4];
#pragma unroll
        for (int np = 0; np < 4; ++np)
#pragma unroll
            for (int kk = 0; kk < 2; ++kk)
#pragma unroll
                for (int e = 0; e < 4; ++e) o[np][kk][e] = 0.f;
        for (int i = 0; i < nb; ++i, ++n) {
            const int s = n % NS;
            if (!warp_wait(&full[s], (n / NS) & 1)) {
                if (lane == 0) {
                    raise(d.error, PK_DEV_TIMEOUT);
                    s_abort = 1;
                }
                failed = true;
                break;
            }
            char *box = smem + s * kStage + h * kBox;
            const uint32_t abox = smem_u32(box);
            if (has_kv) append_rows(kSlotV, 1, i, box);
            uint32_t pa[4];
            ldsm_x4(smem_u32(sP) + (i * 16 + lane % 16) * kPStride + (lane / 16) * 16, pa);
            const int key = (lane % 8) + ((lane / 8) & 1) * 8;
#pragma unroll
            for (int np = 0; np < 4; ++np) {
                uint32_t vb[4];
                ldsm_x4_t(abox + sw128(key, (np * 16 + (lane / 16) * 8) * 2), vb);
                mma_bf16(o[np][0], pa, vb[0], vb[1]);
                mma_bf16(o[np][1], pa, vb[2], vb[3]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        if (failed) break;

        // ---- this head's rows h*chunk + t of the stacked tile -> out
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const int srow = gq + half * 8;
            const int t = srow - h * chunk;
            if (t < 0 || t >= chunk) continue;
            const float inv = 1.f / s_rowsum[srow];
            T *orow = out_base + (int64_t)t * a.o_rs;
#pragma unroll
            for (int np = 0; np < 4; ++np)
#pragma unroll
                for (int kk = 0; kk < 2; ++kk)
                    *reinterpret_cast<__nv_bfloat162 *>(orow + np * 16 + kk * 8 + 2 * tq) =
                        __floats2bfloat162_rn(o[np][kk][2 * half] * inv, o[np][kk][2 * half + 1] * inv);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&info_empty[slot]);   // this warp is done with the slot
    }
}

}  // namespace

int launch_attention_stacked(const pk_paged_kv *kv, const CUtensorMap &pos_map16,
                             const AttnArgs &a, cudaStream_t s) {
    const pk_paged_kv_desc &d = kv->d;
    if (d.dtype != PK_DTYPE_BF16 || kv->head_dim != 64 || d.num_heads != kH ||
        d.chunk > kTMax || d.page_size != 16)
        return PK_ENOTSUP;
    // the slot's bulk copies need 16-byte aligned, 16-byte strided rows
    if ((reinterpret_cast<uintptr_t>(a.bias_u) | reinterpret_cast<uintptr_t>(a.bias_v)) & 15 ||
        (a.bias_ls * 2) % 16)
        return PK_ENOTSUP;
    constexpr int NS = 4;
    SGeom g;
    g.num_layers = d.num_layers;
    g.left = d.left;
    g.chunk = d.chunk;
    g.W = d.left + d.chunk;
    g.R = g.W + d.chunk - 1;
    g.npb = (g.R + 15) / 16;
    g.max_boxes = pk_pages_per_stream(d.left, d.chunk, d.page_size);
    g.items = a.batch * a.nlayers;
    g.batch = a.batch;
    if (g.max_boxes > kMaxBoxes || g.npb > kMaxPosBlocks) return PK_ENOTSUP;
    g.off_slots = NS * kStage;
    g.off_s = g.off_slots + 2 * kSlotBytes;
    g.off_bd = g.off_s + kMaxBoxes * 16 * 16 * 4;
    g.bd_stride = g.npb * 16;
    g.off_p = g.off_bd + 16 * g.bd_stride * 4;
    const size_t smem = g.off_p + kMaxBoxes * 16 * kPStride + 1024;
    auto kernel = paged_attn_stacked_kernel<NS>;
    static size_t limit = 48 * 1024;
    static int sms = 0;
    if (smem > limit) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(paged_attn_stacked)");
        limit = smem;
    }
    if (sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaError_t e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return cuda_status(e, "cudaDeviceGetAttribute");
    }
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, smem);
    if (e != cudaSuccess) return cuda_status(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
    if (per_sm < 1) return PK_ENOTSUP;
    const int grid = (int)std::min<long long>(g.items, (long long)sms * per_sm);
    kernel<<<grid, kThreads, smem, s>>>(kv->kv_map, pos_map16, g, d, a);
    return cuda_status(cudaGetLastError(), "paged_attn_stacked_kernel");
}

}  // namespace pk
