// Paged chunked rel-pos attention, bf16: persistent, warp-specialised,
// tensor-core kernel.
//
// Same computation as the fp32 kernel in pk_attn.cu (ConformerAttention.
// forward lines 99-122, parakeet/modules/attention.py, with the streaming
// mask of parakeet/modules/encoder.py:167-227), organised for throughput:
//
// * one CTA per SM slot, looping over work items (layer, stream, head);
// * a producer warp resolves each item's pages (slot counters -> page ring),
//   issues 128B-swizzled TMA tile loads (cp.async.bulk.tensor) of the K
//   window and the rel-pos rows on one mbarrier and of the V window on a
//   second, into a ring of NS shared-memory stages, and meanwhile builds the
//   item's bf16 (q + pos_bias_u) and (q + pos_bias_v) tiles, its row table
//   and its streaming mask as bit rows;
// * four consumer warps compute BD = (q+v) P^T, S = (q+u) K^T, the masked
//   softmax and O = P V with mma.sync m16n8k16 (bf16 in, fp32 accumulate;
//   the query chunk, T <= 16 frames, is one m16 tile, and when T <= 8 the
//   upper half of the tile is skipped), then release the stage through an
//   "empty" mbarrier;
// * every wait is bounded (1 s); a wait that gives up records
//   PK_DEV_TIMEOUT in the error word and the CTA leaves its loop.
#include <math.h>

#include <algorithm>

#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {
namespace {

constexpr int kCW = 4;                      // consumer warps
constexpr int kThreads = (kCW + 1) * 32;    // + one producer warp
constexpr int kMaxBoxes = 16;
constexpr int kMaxKeys = 128;               // window rows handled (16 * key steps)

struct StageInfo {
    int ok, lrel, b, h;
    int rowoff[kMaxKeys];   // byte offset of window row j's box, -1 = zero row
    int rowr[kMaxKeys];     // row inside that box
    uint32_t mask[16][4];   // bit j%32 of [i][j/32]: key j allowed for query i
};

struct PipeGeom {
    int num_layers, num_heads, left, chunk, page_size, ps_shift, ring, num_pages, num_slots;
    int W, R, max_boxes, items, batch;
    uint32_t box_bytes, pos_colbox_bytes;
    uint32_t st_k, st_v, st_pos, st_q, st_info, stage_bytes;  // offsets inside a stage
    uint32_t off_p, off_bd, off_red, off_zero;                 // consumer scratch
    uint32_t p_stride;
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
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void consumer_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kCW * 32) : "memory");
}

// Where window row j lives in a K or V region: its box base and row, or the
// zero row when j is outside the window.
struct RowRef {
    uint32_t base;
    uint32_t row;
    bool zero;
};
__device__ __forceinline__ RowRef row_ref(uint32_t region, uint32_t zero, const StageInfo &in,
                                          int j) {
    const int ro = in.rowoff[j];
    RowRef r;
    r.zero = ro < 0;
    r.base = r.zero ? zero : region + ro;
    r.row = r.zero ? 0u : (uint32_t)in.rowr[j];
    return r;
}
// 16-byte chunk `ch` (0..7) of column box `cb` of that row
__device__ __forceinline__ uint32_t row_addr(const RowRef &r, uint32_t box_bytes, int cb, int ch) {
    return r.zero ? r.base + ch * 16 : r.base + cb * box_bytes + sw128(r.row, ch * 16);
}

template <int DH, int NS, bool HI>
__global__ void __launch_bounds__(kThreads)
    paged_attn_pipe_kernel(const __grid_constant__ CUtensorMap kv_map,
                           const __grid_constant__ CUtensorMap pos_map, const PipeGeom g,
                           const int32_t *__restrict__ page_table,
                           const int32_t *__restrict__ meta, int32_t *error, const AttnArgs a) {
    constexpr int NCOL = DH / 64;       // 128-byte column boxes per head
    constexpr int KSTEPS = DH / 16;
    constexpr int MAXT = 4;             // key tiles of 8 per consumer warp (W <= 128)
    constexpr int NE = HI ? 4 : 2;      // fragment elements per tile that can be live rows
    using T = __nv_bfloat16;
    extern __shared__ char smem_raw[];
    char *smem = reinterpret_cast<char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                          ~uintptr_t(1023));
    __shared__ uint64_t full_k[NS], full_v[NS], empty[NS];
    __shared__ int s_abort;

    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    const int chunk = g.chunk, W = g.W;
    const int KS_P = (W + 15) / 16;
    const int NT_S = (W + 7) / 8;
    const int NT_P = (g.R + 7) / 8;
    const int RPAD = NT_P * 8;

    // query tiles: rows >= chunk stay zero for the whole kernel
    for (int s = 0; s < NS; ++s)
        for (int i = tid; i < 2 * NCOL * 2048 / 16; i += kThreads)
            reinterpret_cast<uint4 *>(smem + s * g.stage_bytes + g.st_q)[i] = make_uint4(0, 0, 0, 0);
    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full_k[s], 1);
            mbar_init(&full_v[s], 1);
            mbar_init(&empty[s], kCW);
        }
        s_abort = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kCW) {
        // ============================ producer warp ============================
        if (lane == 0) {
            prefetch_tmap(&kv_map);
            prefetch_tmap(&pos_map);
        }
        const int ps = g.page_size, psh = g.ps_shift;
        int it = 0;
        int last_it[NS];
#pragma unroll
        for (int s = 0; s < NS; ++s) last_it[s] = -1;
        for (int item = blockIdx.x; item < g.items; item += gridDim.x, ++it) {
            const int s = it % NS;
            if (it >= NS) {   // the consumers' release of this stage's previous use
                int got = 1;
                if (lane == 0) got = mbar_wait_bounded(&empty[s], ((it / NS) - 1) & 1, kWaitLimitNs);
                got = __shfl_sync(0xffffffffu, got, 0);
                if (!got) {
                    if (lane == 0) raise(error, PK_DEV_TIMEOUT);
                    break;
                }
            }
            char *st = smem + s * g.stage_bytes;
            StageInfo &in = *reinterpret_cast<StageInfo *>(st + g.st_info);
            const int h = item % g.num_heads;
            const int b = (item / g.num_heads) % g.batch;
            const int lrel = item / (g.num_heads * g.batch);
            const int layer = a.layer0 + lrel;
            // slot counters (lane 0), then one page-table entry per lane
            int slot = 0, w = 0, proc = 0, clen = 0, len = 0, ok = 1;
            if (lane == 0) {
                slot = a.slots[b];
                if (slot < 0 || slot >= g.num_slots) {
                    ok = 0;
                    raise(error, PK_DEV_BAD_SLOT);
                } else {
                    const int32_t *m = meta + (int64_t)slot * PK_META_STRIDE;
                    w = m[PK_META_WRITTEN];
                    proc = m[PK_META_PROCESSED];
                    clen = m[PK_META_CACHE_LEN];
                    len = a.lengths[b];
                }
            }
            slot = __shfl_sync(0xffffffffu, slot, 0);
            w = __shfl_sync(0xffffffffu, w, 0);
            proc = __shfl_sync(0xffffffffu, proc, 0);
            clen = __shfl_sync(0xffffffffu, clen, 0);
            len = __shfl_sync(0xffffffffu, len, 0);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            const int a_lo = max(w - g.left, 0), a_hi = w + chunk;
            const int nfirst = a_lo >> psh;
            const int nb = ((a_hi - 1) >> psh) - nfirst + 1;
            if (nb > g.max_boxes) ok = 0;
            int page = 0, start = 0;
            if (ok && lane < nb) {
                const int n = nfirst + lane;
                page = page_table[(int64_t)slot * g.ring + (n & (g.ring - 1))];
                const int lo = max(a_lo - (n << psh), 0), hi = min(a_hi - (n << psh), ps);
                start = lo > 0 ? lo : (hi < ps ? hi - ps : 0);
            }
            const bool bad = ok && lane < nb && (page < 0 || page >= g.num_pages);
            if (__any_sync(0xffffffffu, bad)) {
                if (lane == 0) raise(error, PK_DEV_BAD_PAGE);
                ok = 0;
            }
            if (lane == 0 && ok) {
                const uint32_t kvb = nb * NCOL * g.box_bytes;
                mbar_expect_tx(&full_k[s], kvb + NCOL * (uint32_t)g.R * 128u);
                mbar_expect_tx(&full_v[s], kvb);
            }
            __syncwarp();
            if (ok) {
                // lane i issues the loads of page i; lane 31 the rel-pos rows
                if (lane < nb) {
                    const int kplane = ((page * g.num_layers + layer) * 2) * g.num_heads + h;
                    const int vplane = kplane + g.num_heads;
#pragma unroll
                    for (int cb = 0; cb < NCOL; ++cb)
                        tma_load_3d(st + g.st_k + (lane * NCOL + cb) * g.box_bytes, &kv_map,
                                    &full_k[s], cb * 64, start, kplane);
#pragma unroll
                    for (int cb = 0; cb < NCOL; ++cb)
                        tma_load_3d(st + g.st_v + (lane * NCOL + cb) * g.box_bytes, &kv_map,
                                    &full_v[s], cb * 64, start, vplane);
                }
                if (lane == 31) {
#pragma unroll
                    for (int cb = 0; cb < NCOL; ++cb)
                        tma_load_3d(st + g.st_pos + cb * g.pos_colbox_bytes, &pos_map, &full_k[s],
                                    h * DH + cb * 64, 0, lrel);
                }
                // Qu = q + pos_bias_u, Qv = q + pos_bias_v in bf16 (the reference's bf16
                // add, attention.py:108-109): 8 columns per lane per pass
                const T *qb = static_cast<const T *>(a.q) + (int64_t)lrel * a.q_ls +
                              (int64_t)b * a.q_bs + h * DH;
                const T *bu = static_cast<const T *>(a.bias_u) + (int64_t)lrel * a.bias_ls + h * DH;
                const T *bv = static_cast<const T *>(a.bias_v) + (int64_t)lrel * a.bias_ls + h * DH;
                for (int idx = lane; idx < chunk * (DH / 8); idx += 32) {
                    const int t = idx / (DH / 8), c8 = (idx % (DH / 8)) * 8;
                    const uint4 q4 = *reinterpret_cast<const uint4 *>(qb + (int64_t)t * a.q_rs + c8);
                    const uint4 u4 = __ldg(reinterpret_cast<const uint4 *>(bu + c8));
                    const uint4 v4 = __ldg(reinterpret_cast<const uint4 *>(bv + c8));
                    const __nv_bfloat162 *q2 = reinterpret_cast<const __nv_bfloat162 *>(&q4);
                    const __nv_bfloat162 *u2 = reinterpret_cast<const __nv_bfloat162 *>(&u4);
                    const __nv_bfloat162 *v2 = reinterpret_cast<const __nv_bfloat162 *>(&v4);
                    uint4 ou, ov;
                    __nv_bfloat162 *pu = reinterpret_cast<__nv_bfloat162 *>(&ou);
                    __nv_bfloat162 *pv = reinterpret_cast<__nv_bfloat162 *>(&ov);
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const float2 fq = __bfloat1622float2(q2[k]);
                        const float2 fu = __bfloat1622float2(u2[k]);
                        const float2 fv = __bfloat1622float2(v2[k]);
                        pu[k] = __floats2bfloat162_rn(fq.x + fu.x, fq.y + fu.y);
                        pv[k] = __floats2bfloat162_rn(fq.x + fv.x, fq.y + fv.y);
                    }
                    const uint32_t off = (c8 >> 6) * 2048u + sw128(t, (c8 & 63) * 2);
                    *reinterpret_cast<uint4 *>(st + g.st_q + off) = ou;
                    *reinterpret_cast<uint4 *>(st + g.st_q + NCOL * 2048u + off) = ov;
                }
            }
            // row table: window row j -> (box, row in box); the zero row outside
            // the window.  Box i's start row lives in lane i.
            for (int j0 = 0; j0 < 16 * KS_P; j0 += 32) {
                const int j = j0 + lane;
                const int av = w - g.left + j;
                const bool live = ok && j < W && av >= 0;
                const int bi = live ? (av >> psh) - nfirst : 0;
                const int sbox = __shfl_sync(0xffffffffu, start, bi & 31);
                if (j < 16 * KS_P) {
                    in.rowoff[j] = live ? bi * NCOL * (int)g.box_bytes : -1;
                    in.rowr[j] = live ? (av & (ps - 1)) - sbox : 0;
                }
            }
            // streaming mask bits (encoder.py:167-227), one key per lane
            {
                const int key_start = max(proc - clen, 0), off = g.left - clen;
                const int left_chunks = g.left / chunk;
                for (int kb = 0; kb < (W + 31) / 32; ++kb) {
                    const int j = kb * 32 + lane;
                    bool key_ok = j < W && j >= off;
                    int kc = 0;
                    if (key_ok) {
                        const int rr = j - off;
                        key_ok = rr < clen || (rr - clen) < len;
                        kc = (key_start + rr) / chunk;
                    }
                    int qc = (key_start + clen) / chunk, qrem = (key_start + clen) % chunk;
                    for (int i = 0; i < chunk; ++i) {
                        const int dc = qc - kc;
                        const unsigned bits = __ballot_sync(
                            0xffffffffu, key_ok && i < len && dc >= 0 && dc <= left_chunks);
                        if (lane == 0) in.mask[i][kb] = bits;
                        if (++qrem == chunk) {
                            qrem = 0;
                            ++qc;
                        }
                    }
                }
            }
            if (lane == 0) {
                in.ok = ok;
                in.lrel = lrel;
                in.b = b;
                in.h = h;
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&full_k[s]);  // release: the tiles and info above are visible
                mbar_arrive(&full_v[s]);
            }
            last_it[s] = it;
        }
        // leave no load of ours in flight: wait (bounded) for the last use of each stage
        if (lane == 0) {
#pragma unroll
            for (int s = 0; s < NS; ++s) {
                if (last_it[s] < 0) continue;
                const uint32_t p = (last_it[s] / NS) & 1;
                mbar_wait_bounded(&full_k[s], p, kWaitLimitNs);
                mbar_wait_bounded(&full_v[s], p, kWaitLimitNs);
            }
        }
        return;
    }

    // ============================ consumer warps ============================
    const int gq = lane / 4, tq = lane % 4;
    char *sPr = smem + g.off_p;
    float *sBD = reinterpret_cast<float *>(smem + g.off_bd);
    float *sRed = reinterpret_cast<float *>(smem + g.off_red);
    char *sZero = smem + g.off_zero;
    if (tid < 32) reinterpret_cast<float *>(sZero)[tid] = 0.f;
    consumer_sync();
    const uint32_t aZ = smem_u32(sZero), aPr = smem_u32(sPr);
    const float scale = rsqrtf((float)DH);
    const int pad = 16 * KS_P - NT_S * 8;   // probability columns past the last key tile

    // Every consumer warp runs the same sequence of named barriers for every
    // item, whatever happens; a bounded wait that gives up sets s_abort, which
    // all consumer warps read after the next barrier and leave together.
    int it = 0;
    for (int item = blockIdx.x; item < g.items; item += gridDim.x, ++it) {
        const int s = it % NS;
        const uint32_t ph = (it / NS) & 1;
        const bool got_k = __all_sync(0xffffffffu, mbar_wait_bounded(&full_k[s], ph, kWaitLimitNs));
        if (!got_k && lane == 0) {
            raise(error, PK_DEV_TIMEOUT);
            s_abort = 1;
        }
        char *st = smem + s * g.stage_bytes;
        const StageInfo &in = *reinterpret_cast<const StageInfo *>(st + g.st_info);
        const bool run = got_k && in.ok;
        const int h = in.h, b = in.b, lrel = in.lrel;
        T *out_base = static_cast<T *>(a.out) + (int64_t)lrel * a.o_ls + (int64_t)b * a.o_bs + h * DH;
        if (got_k && !in.ok) {
            for (int idx = tid; idx < chunk * DH; idx += kCW * 32)
                out_base[(int64_t)(idx / DH) * a.o_rs + idx % DH] = __float2bfloat16_rn(0.f);
        }
        const uint32_t aK = smem_u32(st + g.st_k), aV = smem_u32(st + g.st_v);
        const uint32_t aP = smem_u32(st + g.st_pos), aQ = smem_u32(st + g.st_q);

        float sc[MAXT][4];
#pragma unroll
        for (int t = 0; t < MAXT; ++t)
#pragma unroll
            for (int e = 0; e < 4; ++e) sc[t][e] = 0.f;
        if (run) {
            // A fragments of Qu (tile 0) and Qv (tile 1), rows 0..15
            uint32_t fu[KSTEPS][4], fv[KSTEPS][4];
#pragma unroll
            for (int ks = 0; ks < KSTEPS; ++ks) {
                const int col = ks * 16 + (lane / 16) * 8;
                const uint32_t off = (col >> 6) * 2048u + sw128(lane % 16, (col & 63) * 2);
                ldsm_x4(aQ + off, fu[ks]);
                ldsm_x4(aQ + NCOL * 2048u + off, fv[ks]);
            }
            // BD = Qv . P^T (rel-pos tiles split over the consumer warps) -> sBD rows < chunk
            for (int nt = warp; nt < NT_P; nt += kCW) {
                float c[4] = {0.f, 0.f, 0.f, 0.f};
                const uint32_t prow = nt * 8 + (lane % 8);
#pragma unroll
                for (int kp = 0; kp < KSTEPS; kp += 2) {
                    const int col = kp * 16 + (lane / 8) * 8;
                    uint32_t bb[4];
                    ldsm_x4(aP + (col >> 6) * g.pos_colbox_bytes + sw128(prow, (col & 63) * 2), bb);
                    mma_bf16(c, fv[kp], bb[0], bb[1]);
                    mma_bf16(c, fv[kp + 1], bb[2], bb[3]);
                }
                const int p0 = nt * 8 + 2 * tq;
                if (gq < chunk) *reinterpret_cast<float2 *>(sBD + gq * RPAD + p0) = make_float2(c[0], c[1]);
                if (HI && gq + 8 < chunk)
                    *reinterpret_cast<float2 *>(sBD + (gq + 8) * RPAD + p0) = make_float2(c[2], c[3]);
            }
            // S = Qu . K^T (key tiles split over the consumer warps), in registers
#pragma unroll
            for (int t = 0; t < MAXT; ++t) {
                const int nt = warp + t * kCW;
                if (nt < NT_S) {
                    const RowRef rk = row_ref(aK, aZ, in, nt * 8 + (lane % 8));
#pragma unroll
                    for (int kp = 0; kp < KSTEPS; kp += 2) {
                        const int col = kp * 16 + (lane / 8) * 8;
                        uint32_t bb[4];
                        ldsm_x4(row_addr(rk, g.box_bytes, col >> 6, (col & 63) >> 3), bb);
                        mma_bf16(sc[t], fu[kp], bb[0], bb[1]);
                        mma_bf16(sc[t], fu[kp + 1], bb[2], bb[3]);
                    }
                }
            }
        }
        consumer_sync();  // sBD complete (barrier 1 of 3)
        if (s_abort) break;

        // scores with the mask; row max over this warp's tiles, then over warps
        float mx[2] = {-INFINITY, -INFINITY};
        if (run) {
            uint32_t mrow[2][4];
#pragma unroll
            for (int r = 0; r < 2; ++r)
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    mrow[r][k] = (gq + 8 * r < chunk) ? in.mask[gq + 8 * r][k] : 0u;
#pragma unroll
            for (int t = 0; t < MAXT; ++t) {
                const int nt = warp + t * kCW;
                if (nt >= NT_S) break;
#pragma unroll
                for (int e = 0; e < NE; ++e) {
                    const int i = gq + (e >> 1) * 8, j = nt * 8 + 2 * tq + (e & 1);
                    float sv;
                    if (j >= W) {
                        sv = -INFINITY;                                  // key padding
                    } else if (i >= chunk) {
                        sv = 0.f;                                        // query padding
                    } else if ((mrow[e >> 1][j >> 5] >> (j & 31)) & 1u) {
                        sv = (sc[t][e] + sBD[i * RPAD + chunk - 1 - i + j]) * scale;
                    } else {
                        sv = sc[t][e] * scale - 1e5f;                    // attention.py:115
                    }
                    sc[t][e] = sv;
                    mx[e >> 1] = fmaxf(mx[e >> 1], sv);
                }
            }
        }
#pragma unroll
        for (int r = 0; r < (HI ? 2 : 1); ++r) {
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
        }
        if (tq == 0) {
            sRed[warp * 16 + gq] = mx[0];
            if (HI) sRed[warp * 16 + gq + 8] = mx[1];
        }
        consumer_sync();  // barrier 2 of 3
#pragma unroll
        for (int r = 0; r < (HI ? 2 : 1); ++r) {
            float m = -INFINITY;
#pragma unroll
            for (int w2 = 0; w2 < kCW; ++w2) m = fmaxf(m, sRed[w2 * 16 + gq + r * 8]);
            mx[r] = m;
        }
        float sum[2] = {0.f, 0.f};
        if (run) {
#pragma unroll
            for (int t = 0; t < MAXT; ++t) {
                const int nt = warp + t * kCW;
                if (nt >= NT_S) break;
                float p[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int e = 0; e < NE; ++e) {
                    p[e] = __expf(sc[t][e] - mx[e >> 1]);
                    sum[e >> 1] += p[e];
                }
                const int j0 = nt * 8 + 2 * tq;
                *reinterpret_cast<__nv_bfloat162 *>(sPr + gq * g.p_stride + j0 * 2) =
                    __floats2bfloat162_rn(p[0], p[1]);
                *reinterpret_cast<__nv_bfloat162 *>(sPr + (gq + 8) * g.p_stride + j0 * 2) =
                    __floats2bfloat162_rn(p[2], p[3]);
            }
            for (int idx = tid; idx < 16 * pad; idx += kCW * 32) {
                const int r = idx / pad, j = NT_S * 8 + idx % pad;
                *reinterpret_cast<__nv_bfloat16 *>(sPr + r * g.p_stride + j * 2) = __float2bfloat16_rn(0.f);
            }
        }
#pragma unroll
        for (int r = 0; r < (HI ? 2 : 1); ++r) {
            sum[r] += __shfl_xor_sync(0xffffffffu, sum[r], 1);
            sum[r] += __shfl_xor_sync(0xffffffffu, sum[r], 2);
        }
        if (tq == 0) {
            sRed[kCW * 16 + warp * 16 + gq] = sum[0];
            if (HI) sRed[kCW * 16 + warp * 16 + gq + 8] = sum[1];
        }
        consumer_sync();  // probabilities and partial sums visible (barrier 3 of 3)
#pragma unroll
        for (int r = 0; r < (HI ? 2 : 1); ++r) {
            float t2 = 0.f;
#pragma unroll
            for (int w2 = 0; w2 < kCW; ++w2) t2 += sRed[kCW * 16 + w2 * 16 + gq + r * 8];
            sum[r] = t2;
        }

        const bool got_v = __all_sync(0xffffffffu, mbar_wait_bounded(&full_v[s], ph, kWaitLimitNs));
        if (!got_v && lane == 0) {
            raise(error, PK_DEV_TIMEOUT);
            s_abort = 1;
        }
        // O = P . V over this warp's pairs of 8-column output tiles
        if (run && got_v) {
            const float inv0 = 1.f / sum[0], inv1 = HI ? 1.f / sum[1] : 0.f;
            for (int np = warp; np < DH / 16; np += kCW) {
                float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
                const int col = np * 16 + (lane / 16) * 8;
                for (int ks = 0; ks < KS_P; ++ks) {
                    uint32_t pa[4];
                    ldsm_x4(aPr + (lane % 16) * g.p_stride + (ks * 16 + (lane / 16) * 8) * 2, pa);
                    const RowRef rv = row_ref(aV, aZ, in, ks * 16 + (lane % 8) + ((lane / 8) & 1) * 8);
                    uint32_t vb[4];
                    ldsm_x4_t(row_addr(rv, g.box_bytes, col >> 6, (col & 63) >> 3), vb);
                    mma_bf16(c0, pa, vb[0], vb[1]);
                    mma_bf16(c1, pa, vb[2], vb[3]);
                }
                const int d0 = np * 16 + 2 * tq;
                if (gq < chunk) {
                    T *o = out_base + (int64_t)gq * a.o_rs;
                    *reinterpret_cast<__nv_bfloat162 *>(o + d0) = __floats2bfloat162_rn(c0[0] * inv0, c0[1] * inv0);
                    *reinterpret_cast<__nv_bfloat162 *>(o + d0 + 8) = __floats2bfloat162_rn(c1[0] * inv0, c1[1] * inv0);
                }
                if (HI && gq + 8 < chunk) {
                    T *o = out_base + (int64_t)(gq + 8) * a.o_rs;
                    *reinterpret_cast<__nv_bfloat162 *>(o + d0) = __floats2bfloat162_rn(c0[2] * inv1, c0[3] * inv1);
                    *reinterpret_cast<__nv_bfloat162 *>(o + d0 + 8) = __floats2bfloat162_rn(c1[2] * inv1, c1[3] * inv1);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);  // this warp is done with stage s
    }
}

bool fill_pipe_geom(const pk_paged_kv *kv, const AttnArgs &a, int head_dim, int ns, PipeGeom &g,
                    size_t &smem) {
    const pk_paged_kv_desc &d = kv->d;
    const int ncol = head_dim / 64;
    g.num_layers = d.num_layers;
    g.num_heads = d.num_heads;
    g.left = d.left;
    g.chunk = d.chunk;
    g.page_size = d.page_size;
    g.ps_shift = 0;
    while ((1 << g.ps_shift) < d.page_size) ++g.ps_shift;
    if ((1 << g.ps_shift) != d.page_size) return false;
    g.ring = d.ring;
    g.num_pages = d.num_pages;
    g.num_slots = d.num_slots;
    g.W = d.left + d.chunk;
    g.R = g.W + d.chunk - 1;
    g.max_boxes = pk_pages_per_stream(d.left, d.chunk, d.page_size);
    g.batch = a.batch;
    g.items = a.nlayers * a.batch * d.num_heads;
    if (g.max_boxes > kMaxBoxes || g.max_boxes > 31 || d.chunk > 16) return false;
    const int ks_p = (g.W + 15) / 16;
    if (16 * ks_p > kMaxKeys) return false;
    g.box_bytes = d.page_size * 128u;
    const int rpad = (g.R + 7) / 8 * 8;
    g.pos_colbox_bytes = (rpad * 128u + 1023u) & ~1023u;
    g.st_k = 0;
    g.st_v = g.max_boxes * ncol * g.box_bytes;
    g.st_pos = 2 * g.st_v;
    g.st_q = g.st_pos + ncol * g.pos_colbox_bytes;
    g.st_info = g.st_q + 2 * ncol * 2048u;
    g.stage_bytes = (g.st_info + (uint32_t)sizeof(StageInfo) + 1023u) & ~1023u;
    g.p_stride = ks_p * 32 + 16;
    g.off_p = ns * g.stage_bytes;
    g.off_bd = g.off_p + 16 * g.p_stride;
    g.off_red = g.off_bd + ((d.chunk * rpad * 4 + 15) & ~15);
    g.off_zero = g.off_red + 2 * kCW * 16 * 4;
    smem = g.off_zero + 128 + 1024;
    return smem <= 227 * 1024;
}

template <int DH, int NS, bool HI>
int launch_pipe(const pk_paged_kv *kv, const CUtensorMap &pos_map, const AttnArgs &a,
                cudaStream_t s) {
    PipeGeom g;
    size_t smem;
    if (!fill_pipe_geom(kv, a, DH, NS, g, smem)) return PK_ENOTSUP;
    auto kernel = paged_attn_pipe_kernel<DH, NS, HI>;
    static size_t limit = 48 * 1024;
    static int sms = 0;
    if (smem > limit) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(paged_attn_pipe)");
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
    const int grid = (int)std::min<long long>((long long)g.items, (long long)sms * per_sm);
    kernel<<<grid, kThreads, smem, s>>>(kv->kv_map, pos_map, g, kv->d.page_table, kv->d.meta,
                                        kv->d.error, a);
    return cuda_status(cudaGetLastError(), "paged_attn_pipe_kernel");
}

}  // namespace

int launch_attention_bf16(const pk_paged_kv *kv, const CUtensorMap &pos_map, const AttnArgs &a,
                          cudaStream_t s) {
    const bool hi = kv->d.chunk > 8;
    switch (kv->head_dim) {
        case 64:
            return hi ? launch_pipe<64, 2, true>(kv, pos_map, a, s)
                      : launch_pipe<64, 2, false>(kv, pos_map, a, s);
        case 128:
            return hi ? launch_pipe<128, 2, true>(kv, pos_map, a, s)
                      : launch_pipe<128, 2, false>(kv, pos_map, a, s);
        default:
            return PK_ENOTSUP;
    }
}

}  // namespace pk
