// Paged chunked rel-pos attention, bf16, head_dim 128, for chunks of 8 to 16
// frames (the large streaming model: T = 14): one CTA per (stream, layer, group
// of 4 heads).
//
// Same computation as pk_attn.cu / pk_attn_bf16.cu (ConformerAttention.forward
// lines 99-122, parakeet/modules/attention.py; streaming mask of
// parakeet/modules/encoder.py:167-227).  Each head's T queries fill the rows of
// one m16 tile, so a warp per head keeps its scores, softmax and probabilities
// in registers:
//
// * a producer warp streams 16 KB blocks through an NS-stage ring with
//   128B-swizzled TMA tile loads (two 2 KB column boxes per head): the rel-pos
//   projection rows in blocks of 16 (L2-resident), then the stream's K pages,
//   then its V pages; page boxes are shifted so that rows outside the window
//   are zero-filled without being read;
// * consumer warp g owns head hg0 + g: BD = (q+v) P^T per projection block on
//   tensor cores (mma.sync m16n8k16, bf16 in, fp32 accumulate) into the warp's
//   rows of shared memory; S = (q+u) K^T per K page, scaled, plus the shifted
//   BD (rel_shift), with the reference's -1e5 masked fill, kept in registers;
//   softmax over the row in registers (the 4 lanes of a row hold its keys); the
//   probabilities are the A fragments of O = P V (the accumulator layout of one
//   mma is the operand layout of the next);
// * the step's new K/V rows are appended by pk_append_kv before this kernel;
// * every mbarrier wait is bounded (1 s) and records PK_DEV_TIMEOUT.
#include <math.h>

#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {
namespace {

constexpr int kDH = 128;                  // head_dim
constexpr int kHG = 4;                    // heads per CTA = consumer warps
constexpr int kThreads = (kHG + 1) * 32;  // + producer warp
constexpr int kHeadBox = 16 * kDH * 2;    // one head's 16 rows: 4 KB (two 2 KB column boxes)
constexpr int kBlock = kHG * kHeadBox;    // 16 KB
constexpr int kStages = 3;
constexpr int kMaxPosBlocks = 9;          // rel-pos blocks of 16 rows (R <= 143)
constexpr int kDescBar = 1;               // named barrier: window descriptor in smem

struct HGeom {
    int num_layers, left, chunk, W, R, npb, max_boxes;
    uint32_t off_bd;
    int bd_stride;  // floats per query row of a warp's BD rows
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
__device__ __forceinline__ void named_arrive(int id, int count) {
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ void named_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}
// byte offset of (row, dim byte) in a head's 4 KB box: two 128B-swizzled column boxes
__device__ __forceinline__ uint32_t head_off(int row, int byte) {
    return (byte >> 7) * 2048u + sw128(row, byte & 127);
}

// MB: pages per window at most (register arrays of the scores)
template <int MB>
__global__ void __launch_bounds__(kThreads, 3)
    paged_attn_heads_kernel(const __grid_constant__ CUtensorMap kv_map,
                            const __grid_constant__ CUtensorMap pos_map, const HGeom g,
                            const pk_paged_kv_desc d, const AttnArgs a) {
    using T = __nv_bfloat16;
    constexpr int NS = kStages;
    extern __shared__ char smem_raw[];
    char *smem = reinterpret_cast<char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                          ~uintptr_t(1023));
    __shared__ uint64_t full[NS], empty[NS];
    __shared__ int s_ok, s_w, s_nfirst, s_nb;
    __shared__ volatile int s_abort;
    __shared__ int s_page[PK_WIN_MAX_PAGES], s_start[PK_WIN_MAX_PAGES];
    __shared__ uint32_t s_mask[16 * 4];

    const int b = blockIdx.x, lrel = blockIdx.y, hg0 = blockIdx.z * kHG;
    const int layer = a.layer0 + lrel;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int chunk = g.chunk, W = g.W, npb = g.npb;

    if (warp == kHG && lane == 0) {
        prefetch_tmap(&kv_map);
        prefetch_tmap(&pos_map);
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kHG);
        }
        fence_mbar_init();
        s_abort = 0;
    }
    grid_dep_wait();   // descriptors, pages, q and the projection may come from the previous kernel

    if (warp == kHG) {
        // ====== producer: window descriptor, then projection blocks, K pages, V pages ======
        const int32_t *wd = d.window + (int64_t)b * PK_WIN_STRIDE;
        int page = -1, start = 0;
        if (lane < PK_WIN_MAX_PAGES) {
            page = wd[PK_WIN_PAGE + lane];
            start = wd[PK_WIN_START + lane];
            s_page[lane] = page;
            s_start[lane] = start;
        }
        s_mask[lane] = (uint32_t)wd[PK_WIN_MASK + lane];
        s_mask[32 + lane] = (uint32_t)wd[PK_WIN_MASK + 32 + lane];
        const int nb = wd[PK_WIN_NB];
        const int ok = wd[PK_WIN_OK] && nb <= g.max_boxes && nb <= MB;
        if (lane == 0) {
            s_ok = ok;
            s_w = wd[PK_WIN_W];
            s_nfirst = wd[PK_WIN_NFIRST];
            s_nb = nb;
        }
        named_arrive(kDescBar, kThreads);
        if (!ok) return;
        int last_n[NS];
#pragma unroll
        for (int s = 0; s < NS; ++s) last_n[s] = -1;
        const int hb = lane >> 1, cb = lane & 1;   // lanes 0..7: (head of the group, column box)
        for (int n = 0; n < npb + 2 * nb; ++n) {
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
            if (lane == 0) mbar_arrive_expect_tx(&full[s], kBlock);
            __syncwarp();
            const bool is_pos = n < npb;
            const int i = is_pos ? 0 : (n - npb) % nb, kvi = n < npb + nb ? 0 : 1;
            const int pg = __shfl_sync(0xffffffffu, page, i);
            const int st = __shfl_sync(0xffffffffu, start, i);
            if (lane < 2 * kHG) {
                char *dst = smem + s * kBlock + hb * kHeadBox + cb * 2048;
                if (is_pos) {
                    tma_load_3d_hint(dst, &pos_map, &full[s], (hg0 + hb) * kDH + cb * 64, n * 16,
                                     lrel, l2_evict_last());
                } else {
                    const int plane = ((pg * d.num_layers + layer) * 2 + kvi) * d.num_heads + hg0 + hb;
                    tma_load_3d_hint(dst, &kv_map, &full[s], cb * 64, st, plane, l2_evict_first());
                }
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

    // ============================ consumer warp: head h ============================
    const int h = hg0 + warp;
    const int gq = lane / 4, tq = lane % 4;   // mma fragment coordinates
    const float scale = 0.08838834764831845f;   // 1 / sqrt(128)
    const T *qb = static_cast<const T *>(a.q) + (int64_t)lrel * a.q_ls + (int64_t)b * a.q_bs + h * kDH;
    const T *bub = static_cast<const T *>(a.bias_u) + (int64_t)lrel * a.bias_ls + h * kDH;
    const T *bvb = static_cast<const T *>(a.bias_v) + (int64_t)lrel * a.bias_ls + h * kDH;

    // A fragments of q + bias: rows gq, gq + 8 are queries (rows >= chunk zero)
    auto q_frags = [&](const T *bias, uint32_t (&f)[8][4]) {
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const int row = gq + (r & 1) * 8, col = ks * 16 + (r >> 1) * 8 + 2 * tq;
                uint32_t v = 0u;
                if (row < chunk) {
                    const float2 q = __bfloat1622float2(
                        *reinterpret_cast<const __nv_bfloat162 *>(qb + (int64_t)row * a.q_rs + col));
                    const float2 u = __bfloat1622float2(
                        __ldg(reinterpret_cast<const __nv_bfloat162 *>(bias + col)));
                    v = pack_bf16(q.x + u.x, q.y + u.y);
                }
                f[ks][r] = v;
            }
    };

    named_sync(kDescBar, kThreads);   // window descriptor in shared memory
    const int nb = s_nb, w = s_w, nfirst = s_nfirst;
    T *out_base = static_cast<T *>(a.out) + (int64_t)lrel * a.o_ls + (int64_t)b * a.o_bs + h * kDH;
    if (!s_ok) {
        for (int idx = lane; idx < chunk * kDH; idx += 32)
            out_base[(int64_t)(idx / kDH) * a.o_rs + idx % kDH] = __float2bfloat16_rn(0.f);
        return;
    }
    auto wait_full = [&](int n) -> bool {
        if (s_abort) return false;
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&full[n % NS], (n / NS) & 1, kWaitLimitNs))) {
            if (lane == 0) {
                raise(d.error, PK_DEV_TIMEOUT);
                s_abort = 1;
            }
            return false;
        }
        return true;
    };
    auto release = [&](int n) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[n % NS]);
    };

    // ---- rel-pos blocks: bd[t][p] = (q_t + v) . P[p] for the warp's head
    float *bd = reinterpret_cast<float *>(smem + g.off_bd) + warp * chunk * g.bd_stride;
    bool alive = true;
    {
        uint32_t fv[8][4];
        q_frags(bvb, fv);
        for (int pb = 0; pb < npb; ++pb) {
            if (!wait_full(pb)) {
                alive = false;
                break;
            }
            const uint32_t box = smem_u32(smem + (pb % NS) * kBlock + warp * kHeadBox);
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
                float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int kp = 0; kp < 8; kp += 2) {
                    uint32_t bb[4];
                    ldsm_x4(box + head_off(nt * 8 + (lane % 8), (kp * 16 + (lane / 8) * 8) * 2), bb);
                    mma_bf16(c, fv[kp], bb[0], bb[1]);
                    mma_bf16(c, fv[kp + 1], bb[2], bb[3]);
                }
                const int p = pb * 16 + nt * 8 + 2 * tq;
                if (gq < chunk)
                    *reinterpret_cast<float2 *>(bd + gq * g.bd_stride + p) = make_float2(c[0], c[1]);
                if (gq + 8 < chunk)
                    *reinterpret_cast<float2 *>(bd + (gq + 8) * g.bd_stride + p) = make_float2(c[2], c[3]);
            }
            release(pb);
        }
    }
    __syncwarp();   // the warp's BD rows visible to all its lanes

    // ---- K pages: scores of rows gq (sc[i][nt][0..1]) and gq + 8 (sc[i][nt][2..3]) against
    // box rows nt * 8 + 2tq, +1; scale, + BD at the shifted position, masked fill
    float sc[MB][2][4];
    {
        uint32_t fu[8][4];
        q_frags(bub, fu);
        const int wl = w - g.left;
#pragma unroll
        for (int i = 0; i < MB; ++i) {
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) sc[i][nt][e] = -INFINITY;
            if (i >= nb || !alive) continue;
            const int n = npb + i;
            if (!wait_full(n)) {
                alive = false;
                continue;
            }
            const uint32_t box = smem_u32(smem + (n % NS) * kBlock + warp * kHeadBox);
            float c[2][4];
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
                for (int e = 0; e < 4; ++e) c[nt][e] = 0.f;
#pragma unroll
                for (int kp = 0; kp < 8; kp += 2) {
                    uint32_t bb[4];
                    ldsm_x4(box + head_off(nt * 8 + (lane % 8), (kp * 16 + (lane / 8) * 8) * 2), bb);
                    mma_bf16(c[nt], fu[kp], bb[0], bb[1]);
                    mma_bf16(c[nt], fu[kp + 1], bb[2], bb[3]);
                }
            }
            release(n);
            const int r0 = s_start[i], pbase = (nfirst + i) << 4;
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int t = gq + (e >> 1) * 8;                      // query row
                    const int pr = r0 + nt * 8 + 2 * tq + (e & 1);        // page row of the key
                    const int av = pbase + pr, j = av - wl;
                    if (t < chunk && pr >= 0 && pr < 16 && av >= 0 && j >= 0 && j < W) {
                        const float x = c[nt][e] * scale;
                        const bool allowed = (s_mask[t * 4 + (j >> 5)] >> (j & 31)) & 1u;
                        sc[i][nt][e] = allowed ? x + bd[t * g.bd_stride + chunk - 1 - t + j] * scale
                                               : x - 1e5f;   // masked_fill(-1e5), attention.py:115
                    }
                }
        }
    }
    if (!alive) return;

    // ---- softmax of rows gq and gq + 8: the 4 lanes of a row hold its keys
    float mx[2] = {-INFINITY, -INFINITY}, sum[2] = {0.f, 0.f};
#pragma unroll
    for (int i = 0; i < MB; ++i)
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) mx[e >> 1] = fmaxf(mx[e >> 1], sc[i][nt][e]);
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    uint32_t pa[MB][4];   // A fragments of P per page: rows gq, gq + 8
#pragma unroll
    for (int i = 0; i < MB; ++i) {
        float p[2][4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float v = sc[i][nt][e];
                p[nt][e] = v == -INFINITY ? 0.f : __expf(v - mx[e >> 1]);
                sum[e >> 1] += p[nt][e];
            }
        pa[i][0] = pack_bf16(p[0][0], p[0][1]);
        pa[i][1] = pack_bf16(p[0][2], p[0][3]);
        pa[i][2] = pack_bf16(p[1][0], p[1][1]);
        pa[i][3] = pack_bf16(p[1][2], p[1][3]);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        sum[r] += __shfl_xor_sync(0xffffffffu, sum[r], 1);
        sum[r] += __shfl_xor_sync(0xffffffffu, sum[r], 2);
    }
    grid_dep_launch();   // the step's next kernel may be scheduled (it waits for us)

    // ---- V pages: O = P V, 16 column tiles of 8
    float o[16][4];
#pragma unroll
    for (int n8 = 0; n8 < 16; ++n8)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[n8][e] = 0.f;
    const int key = (lane % 8) + ((lane / 8) & 1) * 8;
#pragma unroll
    for (int i = 0; i < MB; ++i) {
        if (i >= nb || !alive) continue;
        const int n = npb + nb + i;
        if (!wait_full(n)) {
            alive = false;
            continue;
        }
        const uint32_t box = smem_u32(smem + (n % NS) * kBlock + warp * kHeadBox);
#pragma unroll
        for (int np = 0; np < 8; ++np) {
            uint32_t vb[4];
            ldsm_x4_t(box + head_off(key, (np * 16 + (lane / 16) * 8) * 2), vb);
            mma_bf16(o[2 * np], pa[i], vb[0], vb[1]);
            mma_bf16(o[2 * np + 1], pa[i], vb[2], vb[3]);
        }
        release(n);
    }
    if (!alive) return;

    // ---- rows gq, gq + 8 of head h -> out
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int t = gq + r * 8;
        if (t >= chunk) continue;
        const float inv = 1.f / sum[r];
        T *orow = out_base + (int64_t)t * a.o_rs;
#pragma unroll
        for (int n8 = 0; n8 < 16; ++n8)
            *reinterpret_cast<__nv_bfloat162 *>(orow + n8 * 8 + 2 * tq) =
                __floats2bfloat162_rn(o[n8][2 * r] * inv, o[n8][2 * r + 1] * inv);
    }
}

}  // namespace

int launch_attention_heads(const pk_paged_kv *kv, const CUtensorMap &pos_map16,
                           const AttnArgs &a, cudaStream_t s) {
    const pk_paged_kv_desc &d = kv->d;
    if (d.dtype != PK_DTYPE_BF16 || kv->head_dim != kDH || d.num_heads % kHG != 0 ||
        d.chunk < 8 || d.chunk > 16 || d.page_size != 16 || a.k_new != nullptr)
        return PK_ENOTSUP;
    HGeom g;
    g.num_layers = d.num_layers;
    g.left = d.left;
    g.chunk = d.chunk;
    g.W = d.left + d.chunk;
    g.R = g.W + d.chunk - 1;
    g.npb = (g.R + 15) / 16;
    g.max_boxes = pk_pages_per_stream(d.left, d.chunk, d.page_size);
    if (g.max_boxes > 8 || g.npb > kMaxPosBlocks) return PK_ENOTSUP;
    g.bd_stride = g.npb * 16;
    g.off_bd = kStages * kBlock;
    const size_t smem = g.off_bd + (size_t)kHG * d.chunk * g.bd_stride * 4 + 1024;
    auto kernel = g.max_boxes <= 7 ? paged_attn_heads_kernel<7> : paged_attn_heads_kernel<8>;
    static size_t limit[2] = {48 * 1024, 48 * 1024};
    size_t &lim = limit[g.max_boxes <= 7 ? 0 : 1];
    if (smem > lim) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(paged_attn_heads)");
        lim = smem;
    }
    dim3 grid(a.batch, a.nlayers, d.num_heads / kHG);
    return cuda_status(launch_pdl(kernel, grid, dim3(kThreads), smem, s, kv->kv_map, pos_map16, g,
                                  d, a),
                       "paged_attn_heads_kernel");
}

}  // namespace pk
