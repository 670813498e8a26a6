// Paged chunked rel-pos multi-head self-attention, one CTA per
// (head, stream, layer).
//
// Restates ConformerAttention.forward lines 99-122
// (parakeet/modules/attention.py): content score (q + u) . k / sqrt(dh),
// position score (q + v) . P[rel_shift] / sqrt(dh) replaced by -1e5 where
// the streaming mask says so (attention.py:108-115), softmax and P.V
// (sdpa_attention_forward, attention.py:9-20).  The mask of
// ConformerEncoder._create_streaming_masks (parakeet/modules/encoder.py:
// 167-227) is evaluated per (query, key) from the slot's counters, and the
// K/V window is read straight from its pages instead of a dense copy.
//
// Data movement: one thread issues 128B-swizzled TMA tile loads
// (cp.async.bulk.tensor.3d).  The pool is head-major, so one page of one
// (layer, K|V, head) is a contiguous page_size x head_dim block and every
// box is a contiguous read; rows outside the window fall outside the box's
// row range and are zero-filled without being read.  K and the L2-resident
// rel-pos rows complete on one mbarrier, V on a second, so the V load
// overlaps the score computation.  All waits are bounded.
//
// Math: bf16 on tensor cores (mma.sync m16n8k16, fp32 accumulate; the
// query chunk, T <= 16 frames, is one m16 tile), fp32 on CUDA cores (the
// exact-parity path).
#include <math.h>

#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {
namespace {

constexpr int kMaxBoxes = 16;

struct AttnGeom {
    int num_layers, num_heads, left, chunk, page_size, ring, num_pages, num_slots;
    int W, R, max_boxes;
    uint32_t box_bytes;         // one page box: page_size rows x 128 bytes
    uint32_t pos_colbox_bytes;  // one column box of rel-pos rows (1024-aligned)
    uint32_t off_v, off_pos, off_q, off_s, off_rows, off_zero, off_red, off_mask;
    uint32_t p_stride;          // bytes per row of the bf16 probability tile
};

template <typename T, int DH>
struct Cfg {
    static constexpr int ES = sizeof(T);
    static constexpr int BC = 128 / ES;   // elements per 128-byte column box
    static constexpr int NCOL = DH / BC;  // column boxes per head
    static constexpr int EPC = 16 / ES;   // elements per 16-byte chunk
};

// Window bookkeeping shared by both kernels, written by thread 0.
struct WinShared {
    uint64_t bar_k, bar_v;
    int w, proc, clen, len, nfirst, nb, ok;
    int start[kMaxBoxes];
};

// Thread 0: read the slot's counters, resolve its pages, issue every load.
template <typename T, int DH>
__device__ __forceinline__ void issue_window_loads(const CUtensorMap *kv_map,
                                                   const CUtensorMap *pos_map, const AttnGeom &g,
                                                   const int32_t *page_table, const int32_t *meta,
                                                   int32_t *error, const AttnArgs &a, int h, int b,
                                                   int lrel, char *sK, char *sV, char *sP,
                                                   WinShared &ws) {
    using C = Cfg<T, DH>;
    const int ps = g.page_size, chunk = g.chunk;
    const int layer = a.layer0 + lrel;
    int ok = 1, w = 0, proc = 0, clen = 0, nfirst = 0, nb = 0;
    const int s = a.slots[b];
    if (s < 0 || s >= g.num_slots) {
        raise(error, PK_DEV_BAD_SLOT);
        ok = 0;
    } else {
        const int32_t *m = meta + (int64_t)s * PK_META_STRIDE;
        w = m[PK_META_WRITTEN];
        proc = m[PK_META_PROCESSED];
        clen = m[PK_META_CACHE_LEN];
        const int a_lo = max(w - g.left, 0), a_hi = w + chunk;
        nfirst = a_lo / ps;
        nb = (a_hi - 1) / ps - nfirst + 1;
        if (nb > g.max_boxes || nb > kMaxBoxes) {
            raise(error, PK_DEV_BAD_PAGE);
            ok = 0;
        }
        for (int i = 0; ok && i < nb; ++i) {
            const int n = nfirst + i;
            const int page = page_table[(int64_t)s * g.ring + (n & (g.ring - 1))];
            if (page < 0 || page >= g.num_pages) {
                raise(error, PK_DEV_BAD_PAGE);
                ok = 0;
                break;
            }
            // rows [lo, hi) of this page are in the window; the box starts at
            // `start`, so rows outside [0, page_size) of the box read as zero
            const int lo = max(a_lo - n * ps, 0), hi = min(a_hi - n * ps, ps);
            ws.start[i] = lo > 0 ? lo : (hi < ps ? hi - ps : 0);
        }
    }
    if (ok) {
        mbar_init(&ws.bar_k, 1);
        mbar_init(&ws.bar_v, 1);
        fence_mbar_init();
        const uint32_t kv_bytes = nb * C::NCOL * g.box_bytes;
        mbar_arrive_expect_tx(&ws.bar_k, kv_bytes + C::NCOL * (uint32_t)g.R * 128u);
        mbar_arrive_expect_tx(&ws.bar_v, kv_bytes);
        for (int i = 0; i < nb; ++i) {
            const int n = nfirst + i;
            const int page = page_table[(int64_t)s * g.ring + (n & (g.ring - 1))];
            const int plane = ((page * g.num_layers + layer) * 2) * g.num_heads + h;
#pragma unroll
            for (int cb = 0; cb < C::NCOL; ++cb) {
                const uint32_t off = (i * C::NCOL + cb) * g.box_bytes;
                tma_load_3d(sK + off, kv_map, &ws.bar_k, cb * C::BC, ws.start[i], plane);
            }
        }
#pragma unroll
        for (int cb = 0; cb < C::NCOL; ++cb)
            tma_load_3d(sP + cb * g.pos_colbox_bytes, pos_map, &ws.bar_k, h * DH + cb * C::BC, 0,
                        lrel);
        for (int i = 0; i < nb; ++i) {
            const int n = nfirst + i;
            const int page = page_table[(int64_t)s * g.ring + (n & (g.ring - 1))];
            const int plane = ((page * g.num_layers + layer) * 2 + 1) * g.num_heads + h;
#pragma unroll
            for (int cb = 0; cb < C::NCOL; ++cb) {
                const uint32_t off = (i * C::NCOL + cb) * g.box_bytes;
                tma_load_3d(sV + off, kv_map, &ws.bar_v, cb * C::BC, ws.start[i], plane);
            }
        }
    }
    ws.w = w;
    ws.proc = proc;
    ws.clen = clen;
    ws.len = ok ? a.lengths[b] : 0;
    ws.nfirst = nfirst;
    ws.nb = nb;
    ws.ok = ok;
}

// Streaming mask of encoder.py:167-227 for query row i, window row j.
struct MaskCtx {
    int clen, n, key_start, off, chunk, left_chunks;
    __device__ __forceinline__ bool masked(int i, int j) const {
        if (j < off) return true;
        const int rr = j - off;
        const bool valid_k = rr < clen || (rr - clen) < n;
        const bool valid_q = i < n;
        const int dchunk = (key_start + clen + i) / chunk - (key_start + rr) / chunk;
        return !(valid_k && valid_q && dchunk >= 0 && dchunk <= left_chunks);
    }
};

__device__ __forceinline__ MaskCtx make_mask(const WinShared &ws, const AttnGeom &g) {
    MaskCtx m;
    m.clen = ws.clen;
    m.n = ws.len;
    m.key_start = max(ws.proc - ws.clen, 0);
    m.off = g.left - ws.clen;
    m.chunk = g.chunk;
    m.left_chunks = g.left / g.chunk;
    return m;
}

// ------------------------------------------------------------------ fp32 path
template <typename T, int DH>
__device__ __forceinline__ float dot_row(const char *box_base, uint32_t colbox_stride, int r,
                                         const float *q) {
    using C = Cfg<T, DH>;
    float acc = 0.f;
#pragma unroll
    for (int cb = 0; cb < C::NCOL; ++cb) {
        const char *base = box_base + cb * colbox_stride;
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
            const uint4 u = *reinterpret_cast<const uint4 *>(base + sw128(r, ch * 16));
            float f[C::EPC];
            unpack16(u, f, static_cast<const T *>(nullptr));
            const float *qq = q + cb * C::BC + ch * C::EPC;
#pragma unroll
            for (int e = 0; e < C::EPC; ++e) acc = fmaf(f[e], qq[e], acc);
        }
    }
    return acc;
}

constexpr int kF32Threads = 128;

template <int DH>
__global__ void __launch_bounds__(kF32Threads)
    paged_attn_f32_kernel(const __grid_constant__ CUtensorMap kv_map,
                          const __grid_constant__ CUtensorMap pos_map, const AttnGeom g,
                          const int32_t *__restrict__ page_table,
                          const int32_t *__restrict__ meta, int32_t *error, const AttnArgs a) {
    using T = float;
    using C = Cfg<T, DH>;
    extern __shared__ char smem_raw[];
    char *smem = reinterpret_cast<char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                          ~uintptr_t(1023));
    __shared__ WinShared ws;
    const int h = blockIdx.x, b = blockIdx.y, lrel = blockIdx.z, tid = threadIdx.x;
    const int chunk = g.chunk, W = g.W, ps = g.page_size;
    char *sK = smem, *sV = smem + g.off_v, *sP = smem + g.off_pos;
    float *qu = reinterpret_cast<float *>(smem + g.off_q);
    float *qv = qu + chunk * DH;
    float *S = reinterpret_cast<float *>(smem + g.off_s);
    int *rowoff = reinterpret_cast<int *>(smem + g.off_rows);
    int *rowr = rowoff + W;

    if (tid == 0)
        issue_window_loads<T, DH>(&kv_map, &pos_map, g, page_table, meta, error, a, h, b, lrel,
                                  sK, sV, sP, ws);
    __syncthreads();
    T *out_base = static_cast<T *>(a.out) + (int64_t)lrel * a.o_ls + (int64_t)b * a.o_bs + h * DH;
    if (!ws.ok) {
        for (int idx = tid; idx < chunk * DH; idx += kF32Threads)
            out_base[(int64_t)(idx / DH) * a.o_rs + idx % DH] = 0.f;
        return;
    }
    {
        const T *qb = static_cast<const T *>(a.q) + (int64_t)lrel * a.q_ls + (int64_t)b * a.q_bs + h * DH;
        const T *bu = static_cast<const T *>(a.bias_u) + (int64_t)lrel * a.bias_ls + h * DH;
        const T *bv = static_cast<const T *>(a.bias_v) + (int64_t)lrel * a.bias_ls + h * DH;
        for (int idx = tid; idx < chunk * DH; idx += kF32Threads) {
            const int t = idx / DH, d = idx % DH;
            const float q = qb[(int64_t)t * a.q_rs + d];
            qu[idx] = q + bu[d];
            qv[idx] = q + bv[d];
        }
        for (int j = tid; j < W; j += kF32Threads) {
            const int av = ws.w - g.left + j;
            if (av < 0) {
                rowoff[j] = -1;
                rowr[j] = 0;
            } else {
                const int bi = av / ps - ws.nfirst;
                rowoff[j] = bi * C::NCOL * g.box_bytes;
                rowr[j] = av % ps - ws.start[bi];
            }
        }
    }
    __syncthreads();
    if (!mbar_wait_bounded(&ws.bar_k, 0, kWaitLimitNs)) {
        if (tid == 0) raise(error, PK_DEV_TIMEOUT);
        mbar_wait_bounded(&ws.bar_k, 0, kWaitLimitNs);
        mbar_wait_bounded(&ws.bar_v, 0, kWaitLimitNs);
        return;
    }
    const float scale = rsqrtf((float)DH);
    const MaskCtx mk = make_mask(ws, g);
    for (int idx = tid; idx < chunk * W; idx += kF32Threads) {
        const int i = idx / W, j = idx % W;
        const int ro = rowoff[j];
        const float content = ro < 0 ? 0.f : dot_row<T, DH>(sK + ro, g.box_bytes, rowr[j], qu + i * DH);
        float bias = -1e5f;
        if (!mk.masked(i, j))
            bias = dot_row<T, DH>(sP, g.pos_colbox_bytes, chunk - 1 - i + j, qv + i * DH) * scale;
        S[idx] = content * scale + bias;
    }
    __syncthreads();
    const int warp = tid / 32, lane = tid % 32;
    for (int i = warp; i < chunk; i += kF32Threads / 32) {
        float *row = S + i * W;
        float mx = -INFINITY;
        for (int j = lane; j < W; j += 32) mx = fmaxf(mx, row[j]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float sum = 0.f;
        for (int j = lane; j < W; j += 32) {
            const float e = expf(row[j] - mx);
            row[j] = e;
            sum += e;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        const float inv = 1.f / sum;
        for (int j = lane; j < W; j += 32) row[j] *= inv;
    }
    __syncthreads();
    if (!mbar_wait_bounded(&ws.bar_v, 0, kWaitLimitNs)) {
        if (tid == 0) raise(error, PK_DEV_TIMEOUT);
        mbar_wait_bounded(&ws.bar_v, 0, kWaitLimitNs);
        return;
    }
    for (int idx = tid; idx < chunk * (DH / 2); idx += kF32Threads) {
        const int i = idx / (DH / 2), d = 2 * (idx % (DH / 2));
        const int cb = d / C::BC;
        const uint32_t byte = (d % C::BC) * C::ES;
        const float *prow = S + i * W;
        float acc0 = 0.f, acc1 = 0.f;
        for (int j = 0; j < W; ++j) {
            const int ro = rowoff[j];
            if (ro < 0) continue;
            const float2 v = *reinterpret_cast<const float2 *>(sV + ro + cb * g.box_bytes +
                                                               sw128(rowr[j], byte));
            acc0 = fmaf(prow[j], v.x, acc0);
            acc1 = fmaf(prow[j], v.y, acc1);
        }
        *reinterpret_cast<float2 *>(out_base + (int64_t)i * a.o_rs + d) = make_float2(acc0, acc1);
    }
}

// ------------------------------------------------------------------ bf16 path
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

template <int DH, int NW>
struct MmaCfg {
    static constexpr int NCOL = DH / 64;   // 128-byte column boxes per head (bf16)
    static constexpr int KSTEPS = DH / 16;  // k-steps of the score MMAs
    static constexpr int THREADS = NW * 32;
    static constexpr int MAXT = (16 + NW - 1) / NW;  // 8-key tiles per warp: W <= 128
};

// shared-memory byte address of window row j, column `col` (a multiple of 8)
// of the K or V box region; rows outside the window map to the zero row
__device__ __forceinline__ uint32_t win_addr(uint32_t region, uint32_t zero, const int *rowoff,
                                             const int *rowr, uint32_t box_bytes, int j, int col) {
    const int ro = rowoff[j];
    if (ro < 0) return zero + ((col & 63) * 2);
    return region + ro + (col >> 6) * box_bytes + sw128(rowr[j], (col & 63) * 2);
}

template <int DH, int NW>
__global__ void __launch_bounds__(MmaCfg<DH, NW>::THREADS)
    paged_attn_bf16_kernel(const __grid_constant__ CUtensorMap kv_map,
                           const __grid_constant__ CUtensorMap pos_map, const AttnGeom g,
                           const int32_t *__restrict__ page_table,
                           const int32_t *__restrict__ meta, int32_t *error, const AttnArgs a) {
    using T = __nv_bfloat16;
    using M = MmaCfg<DH, NW>;
    extern __shared__ char smem_raw[];
    char *smem = reinterpret_cast<char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                          ~uintptr_t(1023));
    __shared__ WinShared ws;
    const int h = blockIdx.x, b = blockIdx.y, lrel = blockIdx.z;
    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    const int gq = lane / 4, tq = lane % 4;  // mma fragment row group / column pair
    const int chunk = g.chunk, W = g.W, ps = g.page_size;
    const int NT_S = (W + 7) / 8;            // key tiles of 8
    const int KS_P = (W + 15) / 16;          // key steps of 16 for P.V
    const int NT_P = (g.R + 7) / 8;          // rel-pos tiles of 8
    const int RPAD = NT_P * 8;

    char *sK = smem, *sV = smem + g.off_v, *sP = smem + g.off_pos;
    char *sQ = smem + g.off_q;                 // Qu then Qv: NCOL x (16 rows x 128 B) each
    char *sPr = smem + g.off_s;                // probabilities, bf16 [16][p_stride]
    float *sBD = reinterpret_cast<float *>(smem + g.off_s + 16 * g.p_stride);  // [chunk][RPAD]
    int *rowoff = reinterpret_cast<int *>(smem + g.off_rows);
    int *rowr = rowoff + 16 * KS_P;
    char *sZero = smem + g.off_zero;
    float *sRed = reinterpret_cast<float *>(smem + g.off_red);  // [2][NW][16]
    uint32_t *sMask = reinterpret_cast<uint32_t *>(smem + g.off_mask);  // [16][4] key bits

    if (tid == 0)
        issue_window_loads<T, DH>(&kv_map, &pos_map, g, page_table, meta, error, a, h, b, lrel,
                                  sK, sV, sP, ws);
    __syncthreads();
    T *out_base = static_cast<T *>(a.out) + (int64_t)lrel * a.o_ls + (int64_t)b * a.o_bs + h * DH;
    if (!ws.ok) {
        for (int idx = tid; idx < chunk * DH; idx += M::THREADS)
            out_base[(int64_t)(idx / DH) * a.o_rs + idx % DH] = __float2bfloat16_rn(0.f);
        return;
    }

    // Qu = q + pos_bias_u, Qv = q + pos_bias_v, rounded to bf16 as the reference's
    // bf16 (query + pos_bias_*) is (attention.py:108-109).  Rows >= chunk of the
    // m16 tile are left as they are: their scores are replaced by a constant
    // below and their outputs are never stored, and MMA rows are independent.
    {
        const T *qb = static_cast<const T *>(a.q) + (int64_t)lrel * a.q_ls + (int64_t)b * a.q_bs + h * DH;
        const T *bu = static_cast<const T *>(a.bias_u) + (int64_t)lrel * a.bias_ls + h * DH;
        const T *bv = static_cast<const T *>(a.bias_v) + (int64_t)lrel * a.bias_ls + h * DH;
        for (int idx = tid; idx < chunk * (DH / 2); idx += M::THREADS) {
            const int t = idx / (DH / 2), d = 2 * (idx % (DH / 2));
            const float2 q = __bfloat1622float2(
                *reinterpret_cast<const __nv_bfloat162 *>(qb + (int64_t)t * a.q_rs + d));
            const float2 fu = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(bu + d));
            const float2 fv = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(bv + d));
            const uint32_t off = (d >> 6) * 2048u + sw128(t, (d & 63) * 2);
            *reinterpret_cast<__nv_bfloat162 *>(sQ + off) = __floats2bfloat162_rn(q.x + fu.x, q.y + fu.y);
            *reinterpret_cast<__nv_bfloat162 *>(sQ + M::NCOL * 2048u + off) =
                __floats2bfloat162_rn(q.x + fv.x, q.y + fv.y);
        }
        // streaming mask as bits: sMask[i][kb] bit (j % 32) set = key j allowed for query i
        {
            const int clen = ws.clen, n = ws.len, key_start = max(ws.proc - clen, 0);
            const int off = g.left - clen, left_chunks = g.left / chunk;
            for (int kb = warp; kb < 4; kb += NW) {
                const int j = kb * 32 + lane;
                bool key_ok = j < W && j >= off;
                int kc = 0;
                if (key_ok) {
                    const int rr = j - off;
                    key_ok = rr < clen || (rr - clen) < n;
                    kc = (key_start + rr) / chunk;
                }
                for (int i = 0; i < chunk; ++i) {
                    const int dc = (key_start + clen + i) / chunk - kc;
                    const unsigned bits = __ballot_sync(0xffffffffu, key_ok && i < n && dc >= 0 &&
                                                                         dc <= left_chunks);
                    if (lane == 0) sMask[i * 4 + kb] = bits;
                }
            }
        }
        for (int j = tid; j < 16 * KS_P; j += M::THREADS) {
            const int av = ws.w - g.left + j;
            if (j >= W || av < 0) {
                rowoff[j] = -1;
                rowr[j] = 0;
            } else {
                const int bi = av / ps - ws.nfirst;
                rowoff[j] = bi * M::NCOL * g.box_bytes;
                rowr[j] = av % ps - ws.start[bi];
            }
        }
        for (int i = tid; i < 32; i += M::THREADS) reinterpret_cast<float *>(sZero)[i] = 0.f;
    }
    __syncthreads();

    const uint32_t aK = smem_u32(sK), aV = smem_u32(sV), aP = smem_u32(sP);
    const uint32_t aQ = smem_u32(sQ), aZ = smem_u32(sZero), aPr = smem_u32(sPr);

    // A fragments of Qu and Qv (rows 0..15, all k-steps)
    uint32_t fu[M::KSTEPS][4], fv[M::KSTEPS][4];
#pragma unroll
    for (int ks = 0; ks < M::KSTEPS; ++ks) {
        const int col = ks * 16 + (lane / 16) * 8;
        const uint32_t off = (col >> 6) * 2048u + sw128(lane % 16, (col & 63) * 2);
        ldsm_x4(aQ + off, fu[ks]);
        ldsm_x4(aQ + M::NCOL * 2048u + off, fv[ks]);
    }

    if (!mbar_wait_bounded(&ws.bar_k, 0, kWaitLimitNs)) {
        if (tid == 0) raise(error, PK_DEV_TIMEOUT);
        mbar_wait_bounded(&ws.bar_k, 0, kWaitLimitNs);
        mbar_wait_bounded(&ws.bar_v, 0, kWaitLimitNs);
        return;
    }

    // BD = Qv . P^T over rel-pos tiles; rows < chunk go to shared memory
    for (int nt = warp; nt < NT_P; nt += NW) {
        float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int kp = 0; kp < M::KSTEPS; kp += 2) {
            const int col = kp * 16 + (lane / 8) * 8;
            const int p = nt * 8 + (lane % 8);
            uint32_t bb[4];
            ldsm_x4(aP + (col >> 6) * g.pos_colbox_bytes + sw128(p, (col & 63) * 2), bb);
            mma_bf16(c, fv[kp], bb[0], bb[1]);
            mma_bf16(c, fv[kp + 1], bb[2], bb[3]);
        }
        const int p0 = nt * 8 + 2 * tq;
        if (gq < chunk) *reinterpret_cast<float2 *>(sBD + gq * RPAD + p0) = make_float2(c[0], c[1]);
        if (gq + 8 < chunk)
            *reinterpret_cast<float2 *>(sBD + (gq + 8) * RPAD + p0) = make_float2(c[2], c[3]);
    }

    // S = Qu . K^T over this warp's key tiles (kept in registers)
    constexpr int MAXT = M::MAXT;            // key tiles per warp held in registers
    float sc[MAXT][4];
#pragma unroll
    for (int t = 0; t < MAXT; ++t) {
        const int nt = warp + t * NW;
        float c[4] = {0.f, 0.f, 0.f, 0.f};
        if (nt < NT_S) {
            const int j = nt * 8 + (lane % 8);
#pragma unroll
            for (int kp = 0; kp < M::KSTEPS; kp += 2) {
                const int col = kp * 16 + (lane / 8) * 8;
                uint32_t bb[4];
                ldsm_x4(win_addr(aK, aZ, rowoff, rowr, g.box_bytes, j, col), bb);
                mma_bf16(c, fu[kp], bb[0], bb[1]);
                mma_bf16(c, fu[kp + 1], bb[2], bb[3]);
            }
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[t][e] = c[e];
    }
    __syncthreads();  // sBD complete

    // scores, mask, row max (rows gq and gq + 8 of the fragment)
    const float scale = rsqrtf((float)DH);
    float mx[2] = {-INFINITY, -INFINITY};
    {
        uint32_t mrow[2][4];
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int k = 0; k < 4; ++k)
                mrow[r][k] = (gq + 8 * r < chunk) ? sMask[(gq + 8 * r) * 4 + k] : 0u;
#pragma unroll
        for (int t = 0; t < MAXT; ++t) {
            const int nt = warp + t * NW;
            if (nt >= NT_S) break;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int i = gq + (e >> 1) * 8, j = nt * 8 + 2 * tq + (e & 1);
                float s;
                if (j >= W) {
                    s = -INFINITY;                        // key padding of the last tile
                } else if (i >= chunk) {
                    s = 0.f;                              // query padding of the m16 tile
                } else if ((mrow[e >> 1][j >> 5] >> (j & 31)) & 1u) {
                    s = sc[t][e] * scale + sBD[i * RPAD + chunk - 1 - i + j] * scale;
                } else {
                    s = sc[t][e] * scale - 1e5f;          // masked_fill(-1e5), attention.py:115
                }
                sc[t][e] = s;
                mx[e >> 1] = fmaxf(mx[e >> 1], s);
            }
        }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    if (NW > 1) {
        if (tq == 0) {
            sRed[warp * 16 + gq] = mx[0];
            sRed[warp * 16 + gq + 8] = mx[1];
        }
        __syncthreads();
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            float m = -INFINITY;
            for (int w2 = 0; w2 < NW; ++w2) m = fmaxf(m, sRed[w2 * 16 + gq + r * 8]);
            mx[r] = m;
        }
    }
    float sum[2] = {0.f, 0.f};
    {
#pragma unroll
        for (int t = 0; t < MAXT; ++t) {
            const int nt = warp + t * NW;
            if (nt >= NT_S) break;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float p = expf(sc[t][e] - mx[e >> 1]);
                sc[t][e] = p;
                sum[e >> 1] += p;
            }
            const int j0 = nt * 8 + 2 * tq;
            *reinterpret_cast<__nv_bfloat162 *>(sPr + gq * g.p_stride + j0 * 2) =
                __floats2bfloat162_rn(sc[t][0], sc[t][1]);
            *reinterpret_cast<__nv_bfloat162 *>(sPr + (gq + 8) * g.p_stride + j0 * 2) =
                __floats2bfloat162_rn(sc[t][2], sc[t][3]);
        }
    }
    // zero probability columns between the last key tile and the last P.V step
    for (int idx = tid; idx < 16 * (16 * KS_P - NT_S * 8); idx += M::THREADS) {
        const int r = idx / (16 * KS_P - NT_S * 8), j = NT_S * 8 + idx % (16 * KS_P - NT_S * 8);
        *reinterpret_cast<__nv_bfloat16 *>(sPr + r * g.p_stride + j * 2) = __float2bfloat16_rn(0.f);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        sum[r] += __shfl_xor_sync(0xffffffffu, sum[r], 1);
        sum[r] += __shfl_xor_sync(0xffffffffu, sum[r], 2);
    }
    if (NW > 1) {
        if (tq == 0) {
            sRed[NW * 16 + warp * 16 + gq] = sum[0];
            sRed[NW * 16 + warp * 16 + gq + 8] = sum[1];
        }
    }
    __syncthreads();  // probabilities and partial sums visible
    if (NW > 1) {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            float s = 0.f;
            for (int w2 = 0; w2 < NW; ++w2) s += sRed[NW * 16 + w2 * 16 + gq + r * 8];
            sum[r] = s;
        }
    }

    if (!mbar_wait_bounded(&ws.bar_v, 0, kWaitLimitNs)) {
        if (tid == 0) raise(error, PK_DEV_TIMEOUT);
        mbar_wait_bounded(&ws.bar_v, 0, kWaitLimitNs);
        return;
    }

    // O = P . V: this warp's pairs of 8-column output tiles
    const float inv0 = 1.f / sum[0], inv1 = 1.f / sum[1];
    for (int np = warp; np < DH / 16; np += NW) {
        float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
        for (int ks = 0; ks < KS_P; ++ks) {
            uint32_t pa[4];
            ldsm_x4(aPr + (lane % 16) * g.p_stride + (ks * 16 + (lane / 16) * 8) * 2, pa);
            const int j = ks * 16 + (lane % 8) + ((lane / 8) & 1) * 8;
            const int col = np * 16 + (lane / 16) * 8;
            uint32_t vb[4];
            ldsm_x4_t(win_addr(aV, aZ, rowoff, rowr, g.box_bytes, j, col), vb);
            mma_bf16(c0, pa, vb[0], vb[1]);
            mma_bf16(c1, pa, vb[2], vb[3]);
        }
        const int d0 = np * 16 + 2 * tq;
        if (gq < chunk) {
            T *o = out_base + (int64_t)gq * a.o_rs;
            *reinterpret_cast<__nv_bfloat162 *>(o + d0) = __floats2bfloat162_rn(c0[0] * inv0, c0[1] * inv0);
            *reinterpret_cast<__nv_bfloat162 *>(o + d0 + 8) = __floats2bfloat162_rn(c1[0] * inv0, c1[1] * inv0);
        }
        if (gq + 8 < chunk) {
            T *o = out_base + (int64_t)(gq + 8) * a.o_rs;
            *reinterpret_cast<__nv_bfloat162 *>(o + d0) = __floats2bfloat162_rn(c0[2] * inv1, c0[3] * inv1);
            *reinterpret_cast<__nv_bfloat162 *>(o + d0 + 8) = __floats2bfloat162_rn(c1[2] * inv1, c1[3] * inv1);
        }
    }
}

// ------------------------------------------------------------------ launch
template <typename T, int DH>
bool fill_geom(const pk_paged_kv *kv, AttnGeom &g, size_t &smem, bool mma) {
    using C = Cfg<T, DH>;
    const pk_paged_kv_desc &d = kv->d;
    g.num_layers = d.num_layers;
    g.num_heads = d.num_heads;
    g.left = d.left;
    g.chunk = d.chunk;
    g.page_size = d.page_size;
    g.ring = d.ring;
    g.num_pages = d.num_pages;
    g.num_slots = d.num_slots;
    g.W = d.left + d.chunk;
    g.R = g.W + d.chunk - 1;
    g.max_boxes = pk_pages_per_stream(d.left, d.chunk, d.page_size);
    if (g.max_boxes > kMaxBoxes) return false;
    g.box_bytes = d.page_size * 128u;
    const uint32_t region = g.max_boxes * C::NCOL * g.box_bytes;
    g.pos_colbox_bytes = (((g.R + 7) / 8 * 8) * 128u + 1023u) & ~1023u;
    g.off_v = region;
    g.off_pos = 2 * region;
    g.off_q = g.off_pos + C::NCOL * g.pos_colbox_bytes;
    const int KS_P = (g.W + 15) / 16;
    const int RPAD = (g.R + 7) / 8 * 8;
    if (mma) {
        g.off_s = g.off_q + 2 * C::NCOL * 2048u;
        g.p_stride = KS_P * 32 + 16;
        g.off_rows = g.off_s + 16 * g.p_stride + ((d.chunk * RPAD * 4 + 15) & ~15);
        g.off_zero = g.off_rows + 2 * 16 * KS_P * 4;
        g.off_red = g.off_zero + 128;
        g.off_mask = g.off_red + 2 * 8 * 16 * 4;
        smem = g.off_mask + 16 * 4 * 4 + 1024;
    } else {
        g.off_s = g.off_q + 2 * d.chunk * DH * 4;
        g.p_stride = 0;
        g.off_rows = g.off_s + ((d.chunk * g.W * 4 + 15) & ~15);
        g.off_zero = g.off_rows + 2 * g.W * 4;
        g.off_red = g.off_zero;
        g.off_mask = g.off_zero;
        smem = g.off_zero + 1024;
    }
    return smem <= 220 * 1024;
}

template <typename K>
int set_smem(K kernel, size_t smem, size_t &limit) {
    if (smem > limit) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(paged attention)");
        limit = smem;
    }
    return PK_OK;
}

template <int DH, int NW>
int launch_bf16(const pk_paged_kv *kv, const CUtensorMap &pos_map, const AttnArgs &a,
                cudaStream_t s) {
    AttnGeom g;
    size_t smem;
    if (kv->d.chunk > 16 || !fill_geom<__nv_bfloat16, DH>(kv, g, smem, true)) return PK_ENOTSUP;
    if ((g.W + 7) / 8 > MmaCfg<DH, NW>::MAXT * NW) return PK_ENOTSUP;  // tiles in registers
    static size_t limit = 48 * 1024;
    int st = set_smem(paged_attn_bf16_kernel<DH, NW>, smem, limit);
    if (st != PK_OK) return st;
    dim3 grid(kv->d.num_heads, a.batch, a.nlayers);
    paged_attn_bf16_kernel<DH, NW><<<grid, NW * 32, smem, s>>>(kv->kv_map, pos_map, g,
                                                               kv->d.page_table, kv->d.meta,
                                                               kv->d.error, a);
    return cuda_status(cudaGetLastError(), "paged_attn_bf16_kernel");
}

template <int DH>
int launch_f32(const pk_paged_kv *kv, const CUtensorMap &pos_map, const AttnArgs &a,
               cudaStream_t s) {
    AttnGeom g;
    size_t smem;
    if (!fill_geom<float, DH>(kv, g, smem, false)) return PK_ENOTSUP;
    static size_t limit = 48 * 1024;
    int st = set_smem(paged_attn_f32_kernel<DH>, smem, limit);
    if (st != PK_OK) return st;
    dim3 grid(kv->d.num_heads, a.batch, a.nlayers);
    paged_attn_f32_kernel<DH><<<grid, kF32Threads, smem, s>>>(kv->kv_map, pos_map, g,
                                                              kv->d.page_table, kv->d.meta,
                                                              kv->d.error, a);
    return cuda_status(cudaGetLastError(), "paged_attn_f32_kernel");
}

}  // namespace

int launch_attention(const pk_paged_kv *kv, const CUtensorMap &pos_map, const AttnArgs &a,
                     cudaStream_t s) {
    if (a.batch == 0 || a.nlayers == 0) return PK_OK;
    const bool bf16 = kv->d.dtype == PK_DTYPE_BF16;
    switch (kv->head_dim) {
        case 64:
            return bf16 ? launch_bf16<64, 4>(kv, pos_map, a, s) : launch_f32<64>(kv, pos_map, a, s);
        case 128:
            return bf16 ? launch_bf16<128, 4>(kv, pos_map, a, s) : launch_f32<128>(kv, pos_map, a, s);
        default:
            return PK_ENOTSUP;
    }
}

}  // namespace pk
