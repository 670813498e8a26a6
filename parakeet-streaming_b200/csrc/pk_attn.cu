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
// This file holds the fp32 path (CUDA cores, the exact-parity path) and the
// dispatch; the bf16 path is the persistent tensor-core kernel of
// pk_attn_bf16.cu.
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
    grid_dep_wait();   // pages, counters and q may come from the previous kernel

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
    return cuda_status(launch_pdl(paged_attn_f32_kernel<DH>, grid, dim3(kF32Threads), smem, s,
                                  kv->kv_map, pos_map, g,
                                  static_cast<const int32_t *>(kv->d.page_table),
                                  static_cast<const int32_t *>(kv->d.meta), kv->d.error, a),
                       "paged_attn_f32_kernel");
}

}  // namespace

int launch_attention(const pk_paged_kv *kv, const CUtensorMap &pos_map, const AttnArgs &a,
                     cudaStream_t s) {
    if (a.batch == 0 || a.nlayers == 0) return PK_OK;
    if (kv->d.dtype == PK_DTYPE_BF16) return launch_attention_bf16(kv, pos_map, a, s);
    switch (kv->head_dim) {
        case 64:
            return launch_f32<64>(kv, pos_map, a, s);
        case 128:
            return launch_f32<128>(kv, pos_map, a, s);
        default:
            return PK_ENOTSUP;
    }
}

}  // namespace pk
