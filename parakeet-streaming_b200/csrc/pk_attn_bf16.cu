// Paged chunked rel-pos attention, bf16, tensor cores: one CTA of four warps
// per (head, stream, layer).
//
// Same computation as the fp32 kernel in pk_attn.cu (ConformerAttention.
// forward lines 99-122, parakeet/modules/attention.py, with the streaming
// mask of parakeet/modules/encoder.py:167-227):
//
// * the stream's window descriptor (pages, box start rows, mask bit rows),
//   written once per step by pk_pages_begin_step, is read by warp 0, whose
//   lanes issue one 128B-swizzled TMA tile load (cp.async.bulk.tensor) per
//   page for K and for V plus one for the L2-resident rel-pos rows of the
//   head; K and rel-pos complete on one mbarrier, V on a second, so the V
//   load overlaps the score computation;
// * meanwhile warps 1-3 build the bf16 (q + pos_bias_u) and (q + pos_bias_v)
//   tiles (the reference's bf16 add, attention.py:108-109);
// * BD = (q+v) P^T, S = (q+u) K^T and O = P V run as mma.sync m16n8k16
//   (bf16 in, fp32 accumulate); the query chunk (T <= 16 frames) is one m16
//   tile and when T <= 8 the upper half of every fragment is skipped;
// * every mbarrier wait is bounded (1 s) and records PK_DEV_TIMEOUT.
#include <math.h>

#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {
namespace {


struct Geom {
    int num_layers, num_heads, left, chunk, page_size, ps_shift, W, R, max_boxes;
    uint32_t box_bytes, pos_colbox_bytes;
    uint32_t off_v, off_pos, off_q, off_p, off_bd, off_red, off_zero;
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

// Window row j of a K or V box region: box base and row inside the box, or
// the zero row when j is outside the window.
struct RowRef {
    uint32_t base, row;
    bool zero;
};
__device__ __forceinline__ RowRef row_ref(uint32_t region, uint32_t zero, const Geom &g, int w,
                                          int nfirst, const int *s_start, int ncol, int j) {
    const int av = w - g.left + j;
    RowRef r;
    r.zero = j >= g.W || av < 0;
    if (r.zero) {
        r.base = zero;
        r.row = 0;
    } else {
        const int bi = (av >> g.ps_shift) - nfirst;
        r.base = region + bi * ncol * g.box_bytes;
        r.row = (uint32_t)((av & (g.page_size - 1)) - s_start[bi]);
    }
    return r;
}
// 16-byte chunk `ch` (0..7) of column box `cb` of that row
__device__ __forceinline__ uint32_t row_addr(const RowRef &r, uint32_t box_bytes, int cb, int ch) {
    return r.zero ? r.base + ch * 16 : r.base + cb * box_bytes + sw128(r.row, ch * 16);
}

template <int DH, bool HI, int NW>
__global__ void __launch_bounds__(NW * 32)
    paged_attn_bf16_kernel(const __grid_constant__ CUtensorMap kv_map,
                           const __grid_constant__ CUtensorMap pos_map, const Geom g,
                           const int32_t *__restrict__ window, int32_t *error, const AttnArgs a) {
    constexpr int NCOL = DH / 64;       // 128-byte column boxes per head
    constexpr int KSTEPS = DH / 16;
    constexpr int kThreads = NW * 32;
    constexpr int kWarps = NW;
    constexpr int MAXT = (16 + NW - 1) / NW;   // key tiles of 8 per warp (W <= 128)
    constexpr int MAXP = (18 + NW - 1) / NW;   // rel-pos tiles of 8 per warp (R <= 143)
    constexpr int MAXKS = 8;                   // key steps of 16 for P.V (W <= 128)
    constexpr int NE = HI ? 4 : 2;      // fragment elements per tile that can be live rows
    using T = __nv_bfloat16;
    extern __shared__ char smem_raw[];
    char *smem = reinterpret_cast<char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                          ~uintptr_t(1023));
    __shared__ uint64_t bar_k, bar_v;
    __shared__ int s_ok, s_w, s_nfirst;
    __shared__ int s_start[PK_WIN_MAX_PAGES];
    __shared__ uint32_t s_mask[16 * 4];

    const int h = blockIdx.x, b = blockIdx.y, lrel = blockIdx.z;
    const int layer = a.layer0 + lrel;
    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    const int chunk = g.chunk, W = g.W;
    const int KS_P = (W + 15) / 16;
    const int NT_S = (W + 7) / 8;
    const int NT_P = (g.R + 7) / 8;
    const int RPAD = NT_P * 8;
    char *sK = smem, *sV = smem + g.off_v, *sP = smem + g.off_pos, *sQ = smem + g.off_q;
    char *sPr = smem + g.off_p;
    float *sBD = reinterpret_cast<float *>(smem + g.off_bd);
    float *sRed = reinterpret_cast<float *>(smem + g.off_red);
    char *sZero = smem + g.off_zero;
    grid_dep_wait();   // descriptors, pages and q may come from the previous kernel

    if (warp == 0) {
        // window descriptor -> TMA loads, one page per lane
        const int32_t *wd = window + (int64_t)b * PK_WIN_STRIDE;
        const int ok = wd[PK_WIN_OK];
        const int nb = wd[PK_WIN_NB];
        const int page = lane < PK_WIN_MAX_PAGES ? wd[PK_WIN_PAGE + lane] : -1;
        const int start = lane < PK_WIN_MAX_PAGES ? wd[PK_WIN_START + lane] : 0;
        const bool run = ok && nb <= g.max_boxes;
        if (lane == 0) {
            mbar_init(&bar_k, 1);
            mbar_init(&bar_v, 1);
            fence_mbar_init();
            if (run) {
                const uint32_t kvb = nb * NCOL * g.box_bytes;
                mbar_arrive_expect_tx(&bar_k, kvb + NCOL * (uint32_t)g.R * 128u);
                mbar_arrive_expect_tx(&bar_v, kvb);
            }
            s_ok = run;
            s_w = wd[PK_WIN_W];
            s_nfirst = wd[PK_WIN_NFIRST];
        }
        __syncwarp();
        if (run) {
            if (lane < nb) {
                const int kplane = ((page * g.num_layers + layer) * 2) * g.num_heads + h;
                const int vplane = kplane + g.num_heads;
                const uint64_t stream_once = l2_evict_first();
#pragma unroll
                for (int cb = 0; cb < NCOL; ++cb)
                    tma_load_3d_hint(sK + (lane * NCOL + cb) * g.box_bytes, &kv_map, &bar_k,
                                     cb * 64, start, kplane, stream_once);
#pragma unroll
                for (int cb = 0; cb < NCOL; ++cb)
                    tma_load_3d_hint(sV + (lane * NCOL + cb) * g.box_bytes, &kv_map, &bar_v,
                                     cb * 64, start, vplane, stream_once);
            }
            if (lane == 31) {
#pragma unroll
                for (int cb = 0; cb < NCOL; ++cb)
                    tma_load_3d(sP + cb * g.pos_colbox_bytes, &pos_map, &bar_k, h * DH + cb * 64, 0,
                                lrel);
            }
        }
        if (lane < PK_WIN_MAX_PAGES) s_start[lane] = start;
        s_mask[lane] = (uint32_t)wd[PK_WIN_MASK + lane];
        s_mask[32 + lane] = (uint32_t)wd[PK_WIN_MASK + 32 + lane];
        reinterpret_cast<float *>(sZero)[lane] = 0.f;
    } else {
        // (q + u) and (q + v) tiles, 8 columns per thread per pass; rows >= chunk zero
        const T *qb = static_cast<const T *>(a.q) + (int64_t)lrel * a.q_ls + (int64_t)b * a.q_bs + h * DH;
        const T *bu = static_cast<const T *>(a.bias_u) + (int64_t)lrel * a.bias_ls + h * DH;
        const T *bv = static_cast<const T *>(a.bias_v) + (int64_t)lrel * a.bias_ls + h * DH;
        for (int idx = tid - 32; idx < 16 * (DH / 8); idx += kThreads - 32) {
            const int t = idx / (DH / 8), c8 = (idx % (DH / 8)) * 8;
            uint4 ou = make_uint4(0, 0, 0, 0), ov = ou;
            if (t < chunk) {
                const uint4 q4 = *reinterpret_cast<const uint4 *>(qb + (int64_t)t * a.q_rs + c8);
                const uint4 u4 = __ldg(reinterpret_cast<const uint4 *>(bu + c8));
                const uint4 v4 = __ldg(reinterpret_cast<const uint4 *>(bv + c8));
                const __nv_bfloat162 *q2 = reinterpret_cast<const __nv_bfloat162 *>(&q4);
                const __nv_bfloat162 *u2 = reinterpret_cast<const __nv_bfloat162 *>(&u4);
                const __nv_bfloat162 *v2 = reinterpret_cast<const __nv_bfloat162 *>(&v4);
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
            }
            const uint32_t off = (c8 >> 6) * 2048u + sw128(t, (c8 & 63) * 2);
            *reinterpret_cast<uint4 *>(sQ + off) = ou;
            *reinterpret_cast<uint4 *>(sQ + NCOL * 2048u + off) = ov;
        }
    }
    __syncthreads();

    T *out_base = static_cast<T *>(a.out) + (int64_t)lrel * a.o_ls + (int64_t)b * a.o_bs + h * DH;
    if (!s_ok) {
        for (int idx = tid; idx < chunk * DH; idx += kThreads)
            out_base[(int64_t)(idx / DH) * a.o_rs + idx % DH] = __float2bfloat16_rn(0.f);
        return;
    }
    const int w = s_w, nfirst = s_nfirst;
    const uint32_t aK = smem_u32(sK), aV = smem_u32(sV), aP = smem_u32(sP), aQ = smem_u32(sQ);
    const uint32_t aZ = smem_u32(sZero), aPr = smem_u32(sPr);
    const int gq = lane / 4, tq = lane % 4;
    const float scale = rsqrtf((float)DH);

    // A fragments of Qu (tile 0) and Qv (tile 1), rows 0..15
    uint32_t fu[KSTEPS][4], fv[KSTEPS][4];
#pragma unroll
    for (int ks = 0; ks < KSTEPS; ++ks) {
        const int col = ks * 16 + (lane / 16) * 8;
        const uint32_t off = (col >> 6) * 2048u + sw128(lane % 16, (col & 63) * 2);
        ldsm_x4(aQ + off, fu[ks]);
        ldsm_x4(aQ + NCOL * 2048u + off, fv[ks]);
    }
    // one CTA-wide verdict on the K wait, so that no warp leaves alone
    if (!__syncthreads_and(mbar_wait_bounded(&bar_k, 0, kWaitLimitNs))) {
        if (tid == 0) {
            raise(error, PK_DEV_TIMEOUT);
            mbar_wait_bounded(&bar_v, 0, kWaitLimitNs);
        }
        return;
    }

    // BD = Qv . P^T over the rel-pos tiles of this warp -> sBD rows < chunk
    {
        float c[MAXP][4];
#pragma unroll
        for (int t = 0; t < MAXP; ++t)
#pragma unroll
            for (int e = 0; e < 4; ++e) c[t][e] = 0.f;
#pragma unroll
        for (int kp = 0; kp < KSTEPS; kp += 2) {
            const int col = kp * 16 + (lane / 8) * 8;
#pragma unroll
            for (int t = 0; t < MAXP; ++t) {
                const int nt = warp + t * kWarps;
                if (nt < NT_P) {
                    uint32_t bb[4];
                    ldsm_x4(aP + (col >> 6) * g.pos_colbox_bytes +
                                sw128(nt * 8 + (lane % 8), (col & 63) * 2), bb);
                    mma_bf16(c[t], fv[kp], bb[0], bb[1]);
                    mma_bf16(c[t], fv[kp + 1], bb[2], bb[3]);
                }
            }
        }
#pragma unroll
        for (int t = 0; t < MAXP; ++t) {
            const int nt = warp + t * kWarps;
            if (nt < NT_P) {
                const int p0 = nt * 8 + 2 * tq;
                if (gq < chunk)
                    *reinterpret_cast<float2 *>(sBD + gq * RPAD + p0) = make_float2(c[t][0], c[t][1]);
                if (HI && gq + 8 < chunk)
                    *reinterpret_cast<float2 *>(sBD + (gq + 8) * RPAD + p0) = make_float2(c[t][2], c[t][3]);
            }
        }
    }
    // S = Qu . K^T over the key tiles of this warp, in registers
    float sc[MAXT][4];
    RowRef rk[MAXT];
#pragma unroll
    for (int t = 0; t < MAXT; ++t) {
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[t][e] = 0.f;
        rk[t] = row_ref(aK, aZ, g, w, nfirst, s_start, NCOL, (warp + t * kWarps) * 8 + (lane % 8));
    }
#pragma unroll
    for (int kp = 0; kp < KSTEPS; kp += 2) {
        const int col = kp * 16 + (lane / 8) * 8;
#pragma unroll
        for (int t = 0; t < MAXT; ++t) {
            if (warp + t * kWarps < NT_S) {
                uint32_t bb[4];
                ldsm_x4(row_addr(rk[t], g.box_bytes, col >> 6, (col & 63) >> 3), bb);
                mma_bf16(sc[t], fu[kp], bb[0], bb[1]);
                mma_bf16(sc[t], fu[kp + 1], bb[2], bb[3]);
            }
        }
    }
    __syncthreads();  // sBD complete

    // scores with the mask; row max over this warp's tiles, then over warps
    float mx[2] = {-INFINITY, -INFINITY};
    {
        uint32_t mrow[2][4];
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int k = 0; k < 4; ++k) mrow[r][k] = s_mask[(gq + 8 * r) * 4 + k];
#pragma unroll
        for (int t = 0; t < MAXT; ++t) {
            const int nt = warp + t * kWarps;
            if (nt >= NT_S) break;
#pragma unroll
            for (int e = 0; e < NE; ++e) {
                const int i = gq + (e >> 1) * 8, j = nt * 8 + 2 * tq + (e & 1);
                float sv;
                if (j >= W) {
                    sv = -INFINITY;                                      // key padding
                } else if (i >= chunk) {
                    sv = 0.f;                                            // query padding
                } else if ((mrow[e >> 1][j >> 5] >> (j & 31)) & 1u) {
                    sv = (sc[t][e] + sBD[i * RPAD + chunk - 1 - i + j]) * scale;
                } else {
                    sv = sc[t][e] * scale - 1e5f;                        // attention.py:115
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
    __syncthreads();
#pragma unroll
    for (int r = 0; r < (HI ? 2 : 1); ++r) {
        float m = -INFINITY;
#pragma unroll
        for (int w2 = 0; w2 < kWarps; ++w2) m = fmaxf(m, sRed[w2 * 16 + gq + r * 8]);
        mx[r] = m;
    }
    float sum[2] = {0.f, 0.f};
#pragma unroll
    for (int t = 0; t < MAXT; ++t) {
        const int nt = warp + t * kWarps;
        if (nt >= NT_S) break;
        float p[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int e = 0; e < NE; ++e) {
            p[e] = __expf(sc[t][e] - mx[e >> 1]);
            sum[e >> 1] += p[e];
        }
        const int j0 = nt * 8 + 2 * tq;
        *reinterpret_cast<__nv_bfloat162 *>(sPr + gq * g.p_stride + j0 * 2) = __floats2bfloat162_rn(p[0], p[1]);
        *reinterpret_cast<__nv_bfloat162 *>(sPr + (gq + 8) * g.p_stride + j0 * 2) =
            __floats2bfloat162_rn(p[2], p[3]);
    }
    {   // probability columns past the last key tile
        const int pad = 16 * KS_P - NT_S * 8;
        for (int idx = tid; idx < 16 * pad; idx += kThreads) {
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
        sRed[kWarps * 16 + warp * 16 + gq] = sum[0];
        if (HI) sRed[kWarps * 16 + warp * 16 + gq + 8] = sum[1];
    }
    // probabilities and partial sums visible; one CTA-wide verdict on the V wait
    if (!__syncthreads_and(mbar_wait_bounded(&bar_v, 0, kWaitLimitNs))) {
        if (tid == 0) raise(error, PK_DEV_TIMEOUT);
        return;
    }
#pragma unroll
    for (int r = 0; r < (HI ? 2 : 1); ++r) {
        float t2 = 0.f;
#pragma unroll
        for (int w2 = 0; w2 < kWarps; ++w2) t2 += sRed[kWarps * 16 + w2 * 16 + gq + r * 8];
        sum[r] = t2;
    }

    // O = P . V over this warp's pairs of 8-column output tiles
    const float inv0 = 1.f / sum[0], inv1 = HI ? 1.f / sum[1] : 0.f;
    for (int np = warp; np < DH / 16; np += kWarps) {
        float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
        float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
        const int col = np * 16 + (lane / 16) * 8;
#pragma unroll
        for (int ks = 0; ks < MAXKS; ++ks) {
            if (ks < KS_P) {
                uint32_t pa[4];
                ldsm_x4(aPr + (lane % 16) * g.p_stride + (ks * 16 + (lane / 16) * 8) * 2, pa);
                const RowRef rv = row_ref(aV, aZ, g, w, nfirst, s_start, NCOL,
                                          ks * 16 + (lane % 8) + ((lane / 8) & 1) * 8);
                uint32_t vb[4];
                ldsm_x4_t(row_addr(rv, g.box_bytes, col >> 6, (col & 63) >> 3), vb);
                if (ks & 1) {
                    mma_bf16(d0, pa, vb[0], vb[1]);
                    mma_bf16(d1, pa, vb[2], vb[3]);
                } else {
                    mma_bf16(c0, pa, vb[0], vb[1]);
                    mma_bf16(c1, pa, vb[2], vb[3]);
                }
            }
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            c0[e] += d0[e];
            c1[e] += d1[e];
        }
        const int oc = np * 16 + 2 * tq;
        if (gq < chunk) {
            T *o = out_base + (int64_t)gq * a.o_rs;
            *reinterpret_cast<__nv_bfloat162 *>(o + oc) = __floats2bfloat162_rn(c0[0] * inv0, c0[1] * inv0);
            *reinterpret_cast<__nv_bfloat162 *>(o + oc + 8) = __floats2bfloat162_rn(c1[0] * inv0, c1[1] * inv0);
        }
        if (HI && gq + 8 < chunk) {
            T *o = out_base + (int64_t)(gq + 8) * a.o_rs;
            *reinterpret_cast<__nv_bfloat162 *>(o + oc) = __floats2bfloat162_rn(c0[2] * inv1, c0[3] * inv1);
            *reinterpret_cast<__nv_bfloat162 *>(o + oc + 8) = __floats2bfloat162_rn(c1[2] * inv1, c1[3] * inv1);
        }
    }
}

bool fill_geom(const pk_paged_kv *kv, int head_dim, int nw, Geom &g, size_t &smem) {
    const pk_paged_kv_desc &d = kv->d;
    const int ncol = head_dim / 64;
    g.num_layers = d.num_layers;
    g.num_heads = d.num_heads;
    g.left = d.left;
    g.chunk = d.chunk;
    g.page_size = d.page_size;
    g.ps_shift = 0;
    while ((1 << g.ps_shift) < d.page_size) ++g.ps_shift;
    if ((1 << g.ps_shift) != d.page_size || d.chunk > 16) return false;
    g.W = d.left + d.chunk;
    g.R = g.W + d.chunk - 1;
    g.max_boxes = pk_pages_per_stream(d.left, d.chunk, d.page_size);
    if (g.max_boxes > PK_WIN_MAX_PAGES || g.W > 128) return false;
    g.box_bytes = d.page_size * 128u;
    const int rpad = (g.R + 7) / 8 * 8;
    const int ks_p = (g.W + 15) / 16;
    g.pos_colbox_bytes = (rpad * 128u + 1023u) & ~1023u;
    g.off_v = g.max_boxes * ncol * g.box_bytes;
    g.off_pos = 2 * g.off_v;
    g.off_q = g.off_pos + ncol * g.pos_colbox_bytes;
    g.off_p = g.off_q + 2 * ncol * 2048u;
    g.p_stride = ks_p * 32 + 16;
    g.off_bd = g.off_p + 16 * g.p_stride;
    g.off_red = g.off_bd + ((d.chunk * rpad * 4 + 15) & ~15);
    g.off_zero = g.off_red + 2 * nw * 16 * 4;
    smem = g.off_zero + 128 + 1024;
    return smem <= 227 * 1024;
}

template <int DH, bool HI>
int launch_typed(const pk_paged_kv *kv, const CUtensorMap &pos_map, const AttnArgs &a,
                 cudaStream_t s) {
    constexpr int NW = DH == 128 ? 8 : 4;   // warps per CTA
    Geom g;
    size_t smem;
    if (!fill_geom(kv, DH, NW, g, smem)) return PK_ENOTSUP;
    auto kernel = paged_attn_bf16_kernel<DH, HI, NW>;
    static size_t limit = 48 * 1024;
    if (smem > limit) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(paged_attn_bf16)");
        limit = smem;
    }
    dim3 grid(kv->d.num_heads, a.batch, a.nlayers);
    return cuda_status(launch_pdl(kernel, grid, dim3(NW * 32), smem, s, kv->kv_map, pos_map, g,
                                  kv->d.window, kv->d.error, a),
                       "paged_attn_bf16_kernel");
}

}  // namespace

int launch_attention_bf16(const pk_paged_kv *kv, const CUtensorMap &pos_map, const AttnArgs &a,
                          cudaStream_t s) {
    const bool hi = kv->d.chunk > 8;
    switch (kv->head_dim) {
        case 64:
            return hi ? launch_typed<64, true>(kv, pos_map, a, s)
                      : launch_typed<64, false>(kv, pos_map, a, s);
        case 128:
            return hi ? launch_typed<128, true>(kv, pos_map, a, s)
                      : launch_typed<128, false>(kv, pos_map, a, s);
        default:
            return PK_ENOTSUP;
    }
}

}  // namespace pk
