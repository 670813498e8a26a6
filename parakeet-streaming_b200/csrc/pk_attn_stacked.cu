// Paged chunked rel-pos attention, bf16, head_dim 64, for chunks of at most 4
// frames (the small streaming model: 8 heads x 2 frames): one CTA per (stream,
// layer, group of 4 heads), the group's queries stacked in one m16 tile.
//
// Same computation as pk_attn.cu / pk_attn_bf16.cu (ConformerAttention.
// forward lines 99-122, parakeet/modules/attention.py; streaming mask of
// parakeet/modules/encoder.py:167-227).  With only T = 2 query rows per
// head, a per-head CTA spends most of its instructions on setup and on the
// 14 padding rows of every m16 tile.  Here:
//
// * a producer warp streams 8 KB blocks (a 16-row slot per head: one page box
//   of 16 frames, or two of 8) through an NS-stage ring with 128B-swizzled TMA
//   tile loads (cp.async.bulk.tensor, L2 evict-first): the stream's K pages,
//   then its V pages - each page box shifted so that rows outside the window
//   are zero-filled without being read;
// * meanwhile consumer warp h computes its head's BD = (q+v) P^T from the
//   rel-pos rows P read straight from global memory (L2-resident: every
//   stream of the layer reads the same rows), so they take no turns of the
//   ring; then S = (q+u) K^T as the K pages arrive; both on tensor cores
//   (mma.sync m16n8k16, bf16 in, fp32 accumulate), written to shared memory
//   in the stacked [head * T + query] row order;
// * one dense softmax over the group's rows (16 threads per row) with the
//   reference's -1e5 masked fill, probabilities kept as bf16 per 16 window
//   columns (one 16-frame page box, or two 8-frame ones);
// * O_h = P V_h on tensor cores, normalised by the row sums;
// * optionally the step's new K/V rows are appended here as well: each
//   warp writes its head's rows to the page in global memory and over the
//   freshly loaded box in shared memory, so no separate append launch and
//   no second read of the new rows are needed;
// * every mbarrier wait is bounded (1 s) and records PK_DEV_TIMEOUT.
#include <math.h>

#include "pk_common.cuh"
#include "pk_internal.h"
#include "pk_relpos.cuh"

namespace pk {
namespace {

constexpr int kH = 4;                    // heads per CTA = consumer warps
constexpr int kThreads = (kH + 1) * 32;  // + producer warp
// Pages of PS = 16 or 8 rows: a head's page box is PS rows x 128 bytes (two or
// one 1 KB 128B-swizzle atoms); a window spans at most 8 boxes of 16 rows or
// 16 of 8.  S, the softmax and P V walk 16-row slots ("virtual boxes") of the
// window: one 16-row box, or two consecutive 8-row boxes.
template <int PS> constexpr int box_bytes() { return PS * 128; }
template <int PS> constexpr int max_boxes() { return PS == 16 ? 8 : 16; }
constexpr int kMaxBoxes = 16;            // descriptor entries read (either page size)
constexpr int kMaxPosBlocks = 8;         // rel-pos blocks of 16 rows (R <= 128)
constexpr int kPStride = 48;             // bytes per row of a 16x16 bf16 probability tile
// Four CTAs of 4 heads per SM, each with a 4-stage ring of 8 KB blocks (52 KB of
// shared memory), measured 2.5% faster than three CTAs of 8 heads with three
// 16 KB stages, and well ahead of two heads per CTA or deeper rings at fewer
// CTAs: half-size CTAs shorten the last, partly filled wave.
constexpr int kStages = 4;
constexpr int kCtasPerSm = 4;
// A ring stage holds one 16-row slot per head: one 16-frame page box, or two
// 8-frame ones back to back (two 1 KB swizzle atoms: the same bytes and
// swizzle as one 16-row box), so both page sizes run the same ring.
constexpr int kSlot = 2048;

struct SGeom {
    int num_layers, left, chunk, W, R, npb, max_boxes;
    uint32_t off_s, off_bd, off_p, stage_bytes;
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
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void consumer_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kH * 32) : "memory");
}

template <int NS, bool kRows16, int MB, int PS>
__global__ void __launch_bounds__(kThreads, kCtasPerSm)
    paged_attn_stacked_kernel(const __grid_constant__ CUtensorMap kv_map, const SGeom g,
                              const pk_paged_kv_desc d, const AttnArgs a) {
    using T = __nv_bfloat16;
    extern __shared__ char smem_raw[];
    char *smem = reinterpret_cast<char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                          ~uintptr_t(1023));
    __shared__ uint64_t full[NS], empty[NS];
    __shared__ int s_ok, s_w, s_nfirst, s_nb;
    __shared__ volatile int s_abort;
    __shared__ int s_page[kMaxBoxes], s_start[kMaxBoxes];
    // per page box: its first window column (jbase) and the box rows [lo, hi)
    // that hold window frames (inside the page, at or after frame 0, in the window)
    __shared__ int s_jbase[kMaxBoxes], s_lo[kMaxBoxes], s_hi[kMaxBoxes];
    __shared__ uint32_t s_mask[16 * 4];
    __shared__ float s_rowsum[16];

    const int b = blockIdx.x, lrel = blockIdx.y, hg0 = blockIdx.z * kH;   // first head of the group
    const int layer = a.layer0 + lrel;
    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    const int chunk = g.chunk, npb = g.npb;
    constexpr int kMB = max_boxes<PS>(), kVB = 16 / PS;   // page boxes per 16-row slot
    float *sS = reinterpret_cast<float *>(smem + g.off_s);    // [box][16 rows][PS]
    float *sBD = reinterpret_cast<float *>(smem + g.off_bd);  // [16 rows][bd_stride]
    char *sP = smem + g.off_p;                                // [virtual box][16 rows][kPStride B]

    if (warp == kH && lane == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kH);
        }
        fence_mbar_init();
        s_abort = 0;
    }
    grid_dep_wait();   // descriptors, pages and q may come from the previous kernel
    if (warp == kH) {
        // window descriptor of this stream (written by pk_pages_begin_step)
        const int32_t *wd = d.window + (int64_t)b * PK_WIN_STRIDE;
        if (lane < kMB) {
            s_page[lane] = wd[PK_WIN_PAGE + lane];
            s_start[lane] = wd[PK_WIN_START + lane];
        }
        s_mask[lane] = (uint32_t)wd[PK_WIN_MASK + lane];
        s_mask[32 + lane] = (uint32_t)wd[PK_WIN_MASK + 32 + lane];
        if (lane == 0) {
            const int nb = wd[PK_WIN_NB];
            s_ok = wd[PK_WIN_OK] && nb <= g.max_boxes && (PS == 16 ? nb : (nb + 1) / 2) <= MB;
            s_w = wd[PK_WIN_W];
            s_nfirst = wd[PK_WIN_NFIRST];
            s_nb = nb;
        }
        if (lane < kMB) {
            // row r of box `lane` is window column jbase + r when it is a real frame:
            // 0 <= start + r < PS (inside the page), abs frame >= 0, 0 <= column < W
            const int st = wd[PK_WIN_START + lane];
            const int abs0 = (wd[PK_WIN_NFIRST] + lane) * PS + st;
            const int jb = abs0 - (wd[PK_WIN_W] - g.left);
            s_jbase[lane] = jb;
            s_lo[lane] = max(max(-st, -abs0), -jb);
            s_hi[lane] = min(PS - st, g.W - jb);
        }
    }
    __syncthreads();
    const int nb = s_nb, w = s_w, nfirst = s_nfirst;
    const int nvb = (nb + kVB - 1) / kVB;   // 16-row slots ("virtual boxes") of the window
    const int nblocks = 2 * nvb;             // K slots, then V slots
    T *out_base = static_cast<T *>(a.out) + (int64_t)lrel * a.o_ls + (int64_t)b * a.o_bs + hg0 * 64;
    if (!s_ok) {
        for (int idx = tid; idx < chunk * kH * 64; idx += kThreads)
            out_base[(int64_t)(idx / (kH * 64)) * a.o_rs + idx % (kH * 64)] = __float2bfloat16_rn(0.f);
        return;
    }

    if (warp == kH) {
        // ======================= producer: K pages, then V pages =======================
        int last_n[NS];
#pragma unroll
        for (int s = 0; s < NS; ++s) last_n[s] = -1;
        for (int n = 0; n < nblocks; ++n) {
            const int s = n % NS, u = n / NS;
            int got = 1;
            if (u >= 1 && lane == 0) got = mbar_wait_bounded(&empty[s], (u - 1) & 1, kWaitLimitNs);
            got = __shfl_sync(0xffffffffu, got, 0);
            if (!got) {
                if (lane == 0) {
                    raise(d.error, PK_DEV_TIMEOUT);
                    s_abort = 1;
                }
                break;
            }
            if (lane == 0) mbar_arrive_expect_tx(&full[s], kH * kSlot);
            __syncwarp();
            if (lane < kH * kVB) {
                // lane: head lane % kH, half lane / kH of the slot; past the last
                // page box the half repeats the slot's first box (finite rows that
                // the softmax gives p = 0)
                const int hd = lane % kH, half = lane / kH;
                const int v = n < nvb ? n : n - nvb, kvi = n < nvb ? 0 : 1;
                const int i = v * kVB + half < nb ? v * kVB + half : v * kVB;
                char *dst = smem + s * g.stage_bytes + hd * kSlot + half * box_bytes<PS>();
                const int plane = ((s_page[i] * d.num_layers + layer) * 2 + kvi) * d.num_heads + hg0 + hd;
                tma_load_3d_hint(dst, &kv_map, &full[s], 0, s_start[i], plane, l2_evict_first());
            }
            last_n[s] = n;
        }
        if (lane == 0) {   // leave none of our loads in flight
#pragma unroll
            for (int s = 0; s < NS; ++s)
                if (last_n[s] >= 0) mbar_wait_bounded(&full[s], (last_n[s] / NS) & 1, kWaitLimitNs);
        }
        return;
    }

    // ============================ consumer warp h = head h ============================
    const int h = warp;
    const int gq = lane / 4, tq = lane % 4;
    const float scale = 0.125f;  // 1 / sqrt(64)
    const int bds = g.bd_stride;

    const int hh = hg0 + h;
    const T *qb = static_cast<const T *>(a.q) + (int64_t)lrel * a.q_ls + (int64_t)b * a.q_bs + hh * 64;

    // this step's new K/V rows of head h, 16 bytes per lane (chunk * 8 <= 16 lanes),
    // fetched now so that the append below does not wait on memory
    uint4 knew = make_uint4(0, 0, 0, 0), vnew = knew;
    const bool app_lane = a.k_new != nullptr && lane < chunk * 8;
    if (app_lane) {
        const int64_t off = (int64_t)lrel * a.q_ls + (int64_t)b * a.q_bs +
                            (int64_t)(lane / 8) * a.q_rs + (hg0 + h) * 64 + (lane % 8) * 8;
        knew = *reinterpret_cast<const uint4 *>(static_cast<const T *>(a.k_new) + off);
        vnew = *reinterpret_cast<const uint4 *>(static_cast<const T *>(a.v_new) + off);
    }
    // ---- BD rows of this CTA's heads: from the all-stream pre-pass when given
    // (a contiguous [head][query][bds] block), else computed here by warp h from
    // the rel-pos rows, while the producer's first K pages are in flight
    if (a.bd) {   // (its latency overlaps that of the first K pages)
        const float4 *src = reinterpret_cast<const float4 *>(
            a.bd + ((((int64_t)lrel * a.batch + b) * d.num_heads + hg0) * chunk) * bds);
        float4 *dst = reinterpret_cast<float4 *>(sBD);
        for (int i = tid; i < kH * chunk * bds / 4; i += kH * 32) dst[i] = src[i];
    } else {
        uint32_t xa[8], xb[8];   // query rows gq and gq + 8
        const __nv_bfloat162 *bv2 = reinterpret_cast<const __nv_bfloat162 *>(
            static_cast<const T *>(a.bias_v) + (int64_t)lrel * a.bias_ls + hh * 64 + 16 * tq);
        bd_a_words(gq < chunk ? qb + (int64_t)gq * a.q_rs + 16 * tq : nullptr, bv2, xa);
        bd_a_words(gq + 8 < chunk ? qb + (int64_t)(gq + 8) * a.q_rs + 16 * tq : nullptr, bv2, xb);
        const T *p_base = static_cast<const T *>(a.pos) + (int64_t)lrel * a.pos_ls + hh * 64 + 16 * tq;
        bd_tile<kBdBatch>(xa, xb, p_base, d.dim, a.pos_rows, 2 * npb, gq, [&](int nt, const float (&c)[4]) {
            if (gq < chunk)
                *reinterpret_cast<float2 *>(sBD + (h * chunk + gq) * bds + nt * 8 + 2 * tq) =
                    make_float2(c[0], c[1]);
        });
    }

    // A fragments of S: rows 0..chunk-1 of the m16 tile are this head's queries
    uint32_t fu[4][4];
    {
        const T *bu = static_cast<const T *>(a.bias_u) + (int64_t)lrel * a.bias_ls + hh * 64;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const int row = gq + (r & 1) * 8, col = ks * 16 + (r >> 1) * 8 + 2 * tq;
                uint32_t pu = 0u;
                if (row < chunk) {
                    const float2 q = __bfloat1622float2(
                        *reinterpret_cast<const __nv_bfloat162 *>(qb + (int64_t)row * a.q_rs + col));
                    const float2 u = __bfloat1622float2(__ldg(reinterpret_cast<const __nv_bfloat162 *>(bu + col)));
                    __nv_bfloat162 xu = __floats2bfloat162_rn(q.x + u.x, q.y + u.y);
                    pu = *reinterpret_cast<uint32_t *>(&xu);
                }
                fu[ks][r] = pu;
            }
    }

    // write those rows into box i (K or V) and into their page in global memory
    auto append_rows = [&](const uint4 &val, int kvi, int i, char *box) {
        if (app_lane) {
            const int t = lane / 8, c = lane % 8;
            const int av = w + t;
            if (av / PS - nfirst == i) {
                const int pr = av & (PS - 1), r = pr - s_start[i];
                *reinterpret_cast<uint4 *>(box + sw128(r, c * 16)) = val;
                T *pool = static_cast<T *>(d.kv);
                const int64_t plane =
                    ((int64_t)(s_page[i] * d.num_layers + layer) * 2 + kvi) * d.num_heads + hg0 + h;
                *reinterpret_cast<uint4 *>(pool + (plane * PS + pr) * 64 + c * 8) = val;
            }
        }
        __syncwarp();
    };

    // ---- pass 1: K slots -> S rows
    for (int v = 0; v < nvb; ++v) {
        const int s = v % NS;
        if (s_abort) break;
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&full[s], (v / NS) & 1, kWaitLimitNs))) {
            if (lane == 0) {
                raise(d.error, PK_DEV_TIMEOUT);
                s_abort = 1;
            }
            break;
        }
        char *slot = smem + s * g.stage_bytes + h * kSlot;
        const uint32_t aslot = smem_u32(slot);
        if (a.k_new) {
#pragma unroll
            for (int half = 0; half < kVB; ++half)
                if (v * kVB + half < nb) append_rows(knew, 0, v * kVB + half, slot + half * box_bytes<PS>());
        }
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {   // n-tiles of 8 keys: slot rows 8 nt ..
            float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int kp = 0; kp < 4; kp += 2) {
                uint32_t bb[4];
                ldsm_x4(aslot + sw128(nt * 8 + (lane % 8), (kp * 16 + (lane / 8) * 8) * 2), bb);
                mma_bf16(c, fu[kp], bb[0], bb[1]);
                mma_bf16(c, fu[kp + 1], bb[2], bb[3]);
            }
            // page box bi, its columns from cb
            const int bi = PS == 16 ? v : 2 * v + nt, cb = PS == 16 ? nt * 8 : 0;
            if (gq < chunk && bi < nb)
                *reinterpret_cast<float2 *>(sS + (bi * 16 + h * chunk + gq) * PS + cb + 2 * tq) =
                    make_float2(c[0], c[1]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    consumer_sync();   // S and BD of every head complete
    if (s_abort) return;

    // ---- dense softmax over the stacked rows: 16 threads per row
    // (a chunk of 3 or 4 frames stacks 12 or 16 rows: the 128 consumer threads
    // then take rows 8-15 in a second pass)
#pragma unroll
    for (int pass = 0; pass < (kRows16 ? 2 : 1); ++pass) {
        const int row = tid / 16 + pass * 8, sub = tid % 16;
        const int rows = kH * chunk;
        const int iq = row % chunk;
        // column sub of virtual box v: column cs of page box bi
        const int cs = PS == 16 ? sub : (sub & 7);
        float sv[MB];
        float mx = -INFINITY;
#pragma unroll
        for (int v = 0; v < MB; ++v) {
            const int bi = PS == 16 ? v : 2 * v + (sub >> 3);
            sv[v] = -INFINITY;
            if (bi < nb && row < rows) {
                if (cs >= s_lo[bi] && cs < s_hi[bi]) {
                    const int j = s_jbase[bi] + cs;
                    const float c = sS[(bi * 16 + row) * PS + cs] * scale;
                    const bool allowed = (s_mask[iq * 4 + (j >> 5)] >> (j & 31)) & 1u;
                    sv[v] = allowed ? c + sBD[row * bds + chunk - 1 - iq + j] * scale
                                    : c - 1e5f;   // masked_fill(-1e5), attention.py:115
                }
            }
            mx = fmaxf(mx, sv[v]);
        }
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float sum = 0.f;
#pragma unroll
        for (int v = 0; v < MB; ++v) {
            if (v < nvb) {   // (keys past the last box get p = 0, which P V needs)
                const float p = sv[v] == -INFINITY ? 0.f : __expf(sv[v] - mx);
                sum += p;
                *reinterpret_cast<__nv_bfloat16 *>(sP + (v * 16 + row) * kPStride + sub * 2) =
                    __float2bfloat16_rn(p);
            }
        }
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (sub == 0) s_rowsum[row] = sum;
    }
    consumer_sync();   // probabilities visible
    grid_dep_launch();   // the step's next kernel may be scheduled (it waits for us)

    // ---- pass 2: O_h = P V_h over the V pages
    float o[4][2][4];
#pragma unroll
    for (int np = 0; np < 4; ++np)
#pragma unroll
        for (int k = 0; k < 2; ++k)
#pragma unroll
            for (int e = 0; e < 4; ++e) o[np][k][e] = 0.f;
    for (int v = 0; v < nvb; ++v) {
        const int n = nvb + v, s = n % NS;   // V slot v
        if (s_abort) break;
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&full[s], (n / NS) & 1, kWaitLimitNs))) {
            if (lane == 0) {
                raise(d.error, PK_DEV_TIMEOUT);
                s_abort = 1;
            }
            break;
        }
        char *slot = smem + s * g.stage_bytes + h * kSlot;
        const uint32_t aslot = smem_u32(slot);
        if (a.v_new) {
#pragma unroll
            for (int half = 0; half < kVB; ++half)
                if (v * kVB + half < nb) append_rows(vnew, 1, v * kVB + half, slot + half * box_bytes<PS>());
        }
        uint32_t pa[4];
        ldsm_x4(smem_u32(sP) + (v * 16 + lane % 16) * kPStride + (lane / 16) * 16, pa);
        const int key = (lane % 8) + ((lane / 8) & 1) * 8;   // slot row = window key of the slot
#pragma unroll
        for (int np = 0; np < 4; ++np) {
            uint32_t vb[4];
            ldsm_x4_t(aslot + sw128(key, (np * 16 + (lane / 16) * 8) * 2), vb);
            mma_bf16(o[np][0], pa, vb[0], vb[1]);
            mma_bf16(o[np][1], pa, vb[2], vb[3]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (s_abort) return;

    // ---- this head's rows h*chunk + t of the stacked tile -> out
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        const int srow = gq + half * 8;                 // stacked row held in c[2*half..]
        const int t = srow - h * chunk;
        if (t < 0 || t >= chunk) continue;
        const float inv = 1.f / s_rowsum[srow];
        T *orow = out_base + (int64_t)t * a.o_rs + h * 64;
#pragma unroll
        for (int np = 0; np < 4; ++np)
#pragma unroll
            for (int k = 0; k < 2; ++k)
                *reinterpret_cast<__nv_bfloat162 *>(orow + np * 16 + k * 8 + 2 * tq) =
                    __floats2bfloat162_rn(o[np][k][2 * half] * inv, o[np][k][2 * half + 1] * inv);
    }
}

// grid (num_layers, num_heads, ceil(batch * chunk / 32)): one pre-pass tile per CTA
__global__ void __launch_bounds__(kRelposThreads, 5)   // 5 CTAs per SM: the small step in one wave
    relpos_bd_kernel(const pk_paged_kv_desc d, const AttnArgs a, int bds, float *bd) {
    grid_dep_wait();     // q may come from the previous kernel
    grid_dep_launch();   // the attention kernel waits for all of us
    relpos_tile(d, a, bds, bd, blockIdx.x, blockIdx.y, blockIdx.z);
}

bool stacked_shape(const pk_paged_kv *kv, SGeom *g) {
    const pk_paged_kv_desc &d = kv->d;
    if (d.dtype != PK_DTYPE_BF16 || kv->head_dim != 64 || d.num_heads % kH != 0 ||
        kH * d.chunk > 16 || (d.page_size != 16 && d.page_size != 8))
        return false;
    g->num_layers = d.num_layers;
    g->left = d.left;
    g->chunk = d.chunk;
    g->W = d.left + d.chunk;
    g->R = g->W + d.chunk - 1;
    g->npb = (g->R + 15) / 16;
    g->max_boxes = pk_pages_per_stream(d.left, d.chunk, d.page_size);
    return g->max_boxes <= (d.page_size == 16 ? max_boxes<16>() : max_boxes<8>()) &&
           g->npb <= kMaxPosBlocks;
}

}  // namespace

int relpos_bd_cols(const pk_paged_kv *kv) {
    SGeom g;   // a pre-pass warp holds half of the 2 * npb n-tiles in registers
    return stacked_shape(kv, &g) && g.npb <= kBdBatch ? g.npb * 16 : 0;
}

int launch_relpos_bd(const pk_paged_kv *kv, const AttnArgs &a, float *bd, cudaStream_t s) {
    SGeom g;
    if (!stacked_shape(kv, &g) || g.npb > kBdBatch) return PK_ENOTSUP;
    if (a.batch == 0 || a.nlayers == 0) return PK_OK;
    dim3 grid(a.nlayers, kv->d.num_heads, (a.batch * kv->d.chunk + kRelposRows - 1) / kRelposRows);
    return cuda_status(launch_pdl(relpos_bd_kernel, grid, dim3(kRelposThreads), 0, s, kv->d, a,
                                  g.npb * 16, bd),
                       "relpos_bd_kernel");
}

namespace {

template <int PS>
int launch_stacked_ps(const pk_paged_kv *kv, SGeom g, const AttnArgs &a, cudaStream_t s) {
    const pk_paged_kv_desc &d = kv->d;
    constexpr int NS = kStages;
    constexpr int kVirt = max_boxes<PS>() * PS / 16;   // 16-row slots of a window (8)
    g.stage_bytes = kH * kSlot;
    g.off_s = NS * g.stage_bytes;
    g.off_bd = g.off_s + max_boxes<PS>() * 16 * PS * 4;
    g.bd_stride = g.npb * 16;
    g.off_p = g.off_bd + 16 * g.bd_stride * 4;
    const size_t smem = g.off_p + kVirt * 16 * kPStride + 1024;
    // more than 8 stacked query rows (chunks of 3 or 4) take a second softmax pass
    // and the softmax loops run over at most MB virtual boxes (6 for the small model)
    const bool r16 = kH * d.chunk > 8, mb6 = (g.max_boxes * PS + 15) / 16 <= 6;
    auto kernel = r16 ? (mb6 ? paged_attn_stacked_kernel<NS, true, 6, PS>
                             : paged_attn_stacked_kernel<NS, true, kVirt, PS>)
                      : (mb6 ? paged_attn_stacked_kernel<NS, false, 6, PS>
                             : paged_attn_stacked_kernel<NS, false, kVirt, PS>);
    static size_t limit[4] = {48 * 1024, 48 * 1024, 48 * 1024, 48 * 1024};
    size_t &lim = limit[2 * r16 + mb6];
    if (smem > lim) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(paged_attn_stacked)");
        lim = smem;
    }
    dim3 grid(a.batch, a.nlayers, d.num_heads / kH);
    return cuda_status(launch_pdl(kernel, grid, dim3(kThreads), smem, s, kv->kv_map, g, d, a),
                       "paged_attn_stacked_kernel");
}

}  // namespace

int launch_attention_stacked(const pk_paged_kv *kv, const CUtensorMap &pos_map16,
                             const AttnArgs &a, cudaStream_t s) {
    (void)pos_map16;   // the rel-pos rows are read through a.pos (or a.bd)
    SGeom g;
    if (!stacked_shape(kv, &g)) return PK_ENOTSUP;
    return kv->d.page_size == 16 ? launch_stacked_ps<16>(kv, g, a, s)
                                 : launch_stacked_ps<8>(kv, g, a, s);
}

}  // namespace pk
