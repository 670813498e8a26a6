// Paged chunked rel-pos multi-head self-attention (one CTA per
// (head, stream, layer)).
//
// Restates ConformerAttention.forward lines 99-122
// (parakeet/modules/attention.py): content score (q + u) . k / sqrt(dh),
// position score (q + v) . P[rel_shift] / sqrt(dh) with the streaming mask
// written as -1e5 (attention.py:108-115), softmax and P.V
// (sdpa_attention_forward, attention.py:9-20).  The mask of
// ConformerEncoder._create_streaming_masks (parakeet/modules/encoder.py:
// 167-227) is evaluated per (query, key) from the slot's counters, and the
// K/V window is read straight from its pages instead of a dense copy.
//
// Data movement: one thread issues 128B-swizzled TMA tile loads
// (cp.async.bulk.tensor.3d) of exactly the window's rows, one box per page
// (rows outside the window fall out of the box's range and are zero-filled
// without being read), plus the L2-resident rel-pos rows this head needs;
// completion is one mbarrier with a bounded wait.
#include <math.h>

#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {
namespace {

constexpr int kAttnThreads = 128;
constexpr int kMaxBoxes = 16;

struct AttnGeom {
    int num_layers, dim, left, chunk, page_size, ring, num_pages, num_slots;
    int W, R, max_boxes;
    uint32_t kv_region_bytes;   // bytes of the K (and of the V) box region
    uint32_t pos_colbox_bytes;  // bytes per column box of rel-pos rows
    uint32_t off_v, off_pos, off_q, off_s, off_rows;
};

template <typename T, int DH>
struct Cfg {
    static constexpr int ES = sizeof(T);
    static constexpr int BC = 128 / ES;   // elements per 128-byte column box
    static constexpr int NCOL = DH / BC;  // column boxes per head
    static constexpr int EPC = 16 / ES;   // elements per 16-byte chunk
};

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

template <typename T>
__device__ __forceinline__ float2 load2(const char *p) {
    if constexpr (sizeof(T) == 2) {
        return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(p));
    } else {
        return *reinterpret_cast<const float2 *>(p);
    }
}

template <typename T>
__device__ __forceinline__ void store2(T *p, float x, float y) {
    if constexpr (sizeof(T) == 2) {
        *reinterpret_cast<__nv_bfloat162 *>(p) = __floats2bfloat162_rn(x, y);
    } else {
        *reinterpret_cast<float2 *>(p) = make_float2(x, y);
    }
}

template <typename T, int DH>
__global__ void __launch_bounds__(kAttnThreads)
    paged_attn_kernel(const __grid_constant__ CUtensorMap kv_map,
                      const __grid_constant__ CUtensorMap pos_map, const AttnGeom g,
                      const int32_t *__restrict__ page_table, const int32_t *__restrict__ meta,
                      int32_t *error, const AttnArgs a) {
    using C = Cfg<T, DH>;
    extern __shared__ char smem_raw[];
    // dynamic smem is only 16-byte aligned by contract: align to 1024 here
    char *smem = reinterpret_cast<char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                          ~uintptr_t(1023));
    __shared__ uint64_t bar;
    __shared__ int s_w, s_proc, s_clen, s_len, s_nfirst, s_nb, s_ok;
    __shared__ int s_start[kMaxBoxes];

    const int h = blockIdx.x;
    const int b = blockIdx.y;
    const int lrel = blockIdx.z;
    const int layer = a.layer0 + lrel;
    const int tid = threadIdx.x;
    const int chunk = g.chunk, W = g.W, ps = g.page_size;
    const uint32_t box_bytes = ps * 128u;

    char *sK = smem;
    char *sV = smem + g.off_v;
    char *sP = smem + g.off_pos;
    float *qu = reinterpret_cast<float *>(smem + g.off_q);
    float *qv = qu + chunk * DH;
    float *S = reinterpret_cast<float *>(smem + g.off_s);
    int *rowoff = reinterpret_cast<int *>(smem + g.off_rows);  // per window row: box*NCOL*box_bytes, -1 = zero row
    int *rowr = rowoff + W;                                    // per window row: row inside box

    if (tid == 0) {
        int ok = 1;
        const int s = a.slots[b];
        int w = 0, proc = 0, clen = 0, nfirst = 0, nb = 0;
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
            if (nb > g.max_boxes) {
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
                const int lo = max(a_lo - n * ps, 0), hi = min(a_hi - n * ps, ps);
                s_start[i] = lo > 0 ? lo : (hi < ps ? hi - ps : 0);
            }
            if (ok) {
                mbar_init(&bar, 1);
                fence_mbar_init();
            }
            // issue all loads: K and V boxes of every page, then rel-pos rows
            if (ok) {
                const uint32_t bytes =
                    2u * nb * C::NCOL * box_bytes + C::NCOL * (uint32_t)g.R * 128u;
                mbar_arrive_expect_tx(&bar, bytes);
                for (int i = 0; i < nb; ++i) {
                    const int n = nfirst + i;
                    const int page = page_table[(int64_t)s * g.ring + (n & (g.ring - 1))];
                    const int plane = (page * g.num_layers + layer) * 2;
                    for (int cb = 0; cb < C::NCOL; ++cb) {
                        const int x = h * DH + cb * C::BC;
                        char *dk = sK + (i * C::NCOL + cb) * box_bytes;
                        tma_load_3d(dk, &kv_map, &bar, x, s_start[i], plane);
                        tma_load_3d(sV + (dk - sK), &kv_map, &bar, x, s_start[i], plane + 1);
                    }
                }
                for (int cb = 0; cb < C::NCOL; ++cb)
                    tma_load_3d(sP + cb * g.pos_colbox_bytes, &pos_map, &bar, h * DH + cb * C::BC,
                                0, lrel);
            }
        }
        s_w = w;
        s_proc = proc;
        s_clen = clen;
        s_len = ok ? a.lengths[b] : 0;
        s_nfirst = nfirst;
        s_nb = nb;
        s_ok = ok;
    }
    __syncthreads();

    T *out_base = static_cast<T *>(a.out) + (int64_t)lrel * a.o_ls + (int64_t)b * a.o_bs + h * DH;
    if (!s_ok) {
        for (int idx = tid; idx < chunk * DH; idx += kAttnThreads)
            out_base[(int64_t)(idx / DH) * a.o_rs + idx % DH] = Elem<T>::from_f(0.f);
        return;
    }

    // queries with the two position biases, rounded to the model dtype as the
    // reference's (query + pos_bias_u/v) is (attention.py:108-109)
    {
        const T *qb = static_cast<const T *>(a.q) + (int64_t)lrel * a.q_ls + (int64_t)b * a.q_bs +
                      h * DH;
        const T *bu = static_cast<const T *>(a.bias_u) + (int64_t)lrel * a.bias_ls + h * DH;
        const T *bv = static_cast<const T *>(a.bias_v) + (int64_t)lrel * a.bias_ls + h * DH;
        for (int idx = tid; idx < chunk * DH; idx += kAttnThreads) {
            const int t = idx / DH, d = idx % DH;
            const float q = Elem<T>::to_f(qb[(int64_t)t * a.q_rs + d]);
            qu[idx] = Elem<T>::to_f(Elem<T>::from_f(q + Elem<T>::to_f(bu[d])));
            qv[idx] = Elem<T>::to_f(Elem<T>::from_f(q + Elem<T>::to_f(bv[d])));
        }
        const int w = s_w;
        for (int j = tid; j < W; j += kAttnThreads) {
            const int av = w - g.left + j;
            if (av < 0) {
                rowoff[j] = -1;
                rowr[j] = 0;
            } else {
                const int bi = av / ps - s_nfirst;
                rowoff[j] = bi * C::NCOL * box_bytes;
                rowr[j] = av % ps - s_start[bi];
            }
        }
    }
    __syncthreads();

    if (!mbar_wait_bounded(&bar, 0, kWaitLimitNs)) {
        if (tid == 0) raise(error, PK_DEV_TIMEOUT);
        mbar_wait_bounded(&bar, 0, kWaitLimitNs);
        return;
    }

    // scores
    const float scale = rsqrtf((float)DH);
    const int clen = s_clen, n = s_len, proc = s_proc;
    const int key_start = max(proc - clen, 0);
    const int off = g.left - clen;
    const int left_chunks = g.left / chunk;
    for (int idx = tid; idx < chunk * W; idx += kAttnThreads) {
        const int i = idx / W, j = idx % W;
        const int ro = rowoff[j];
        const float content =
            ro < 0 ? 0.f : dot_row<T, DH>(sK + ro, box_bytes, rowr[j], qu + i * DH);
        bool masked = j < off;
        if (!masked) {
            const int rr = j - off;
            const bool valid_k = rr < clen || (rr - clen) < n;
            const bool valid_q = i < n;
            const int dchunk = (key_start + clen + i) / chunk - (key_start + rr) / chunk;
            masked = !(valid_k && valid_q && dchunk >= 0 && dchunk <= left_chunks);
        }
        float bias = -1e5f;
        if (!masked) {
            const int p = chunk - 1 - i + j;  // rel_shift: column j of row i
            bias = dot_row<T, DH>(sP, g.pos_colbox_bytes, p, qv + i * DH) * scale;
        }
        S[idx] = content * scale + bias;
    }
    __syncthreads();

    // softmax over keys, one warp per query row
    const int warp = tid / 32, lane = tid % 32;
    for (int i = warp; i < chunk; i += kAttnThreads / 32) {
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

    // P . V, two output columns per thread
    for (int idx = tid; idx < chunk * (DH / 2); idx += kAttnThreads) {
        const int i = idx / (DH / 2), d = 2 * (idx % (DH / 2));
        const int cb = d / C::BC;
        const uint32_t byte = (d % C::BC) * C::ES;
        const float *prow = S + i * W;
        float acc0 = 0.f, acc1 = 0.f;
        for (int j = 0; j < W; ++j) {
            const int ro = rowoff[j];
            if (ro < 0) continue;
            const float2 v = load2<T>(sV + ro + cb * box_bytes + sw128(rowr[j], byte));
            const float p = prow[j];
            acc0 = fmaf(p, v.x, acc0);
            acc1 = fmaf(p, v.y, acc1);
        }
        store2<T>(out_base + (int64_t)i * a.o_rs + d, acc0, acc1);
    }
}

template <typename T, int DH>
int launch_typed(const pk_paged_kv *kv, const CUtensorMap &pos_map, const AttnArgs &a,
                 cudaStream_t s) {
    using C = Cfg<T, DH>;
    const pk_paged_kv_desc &d = kv->d;
    AttnGeom g;
    g.num_layers = d.num_layers;
    g.dim = d.dim;
    g.left = d.left;
    g.chunk = d.chunk;
    g.page_size = d.page_size;
    g.ring = d.ring;
    g.num_pages = d.num_pages;
    g.num_slots = d.num_slots;
    g.W = d.left + d.chunk;
    g.R = g.W + d.chunk - 1;
    g.max_boxes = pk_pages_per_stream(d.left, d.chunk, d.page_size);
    if (g.max_boxes > kMaxBoxes) return PK_ENOTSUP;
    const uint32_t box_bytes = d.page_size * 128u;
    g.kv_region_bytes = g.max_boxes * C::NCOL * box_bytes;
    g.pos_colbox_bytes = (g.R * 128u + 1023u) & ~1023u;
    g.off_v = g.kv_region_bytes;
    g.off_pos = 2 * g.kv_region_bytes;
    g.off_q = g.off_pos + C::NCOL * g.pos_colbox_bytes;
    g.off_s = g.off_q + 2 * d.chunk * DH * 4;
    g.off_rows = g.off_s + ((d.chunk * g.W * 4 + 15) & ~15);
    const size_t smem = g.off_rows + 2 * g.W * 4 + 1024;  // + alignment slack
    if (smem > 220 * 1024) return PK_ENOTSUP;
    // raise the kernel's dynamic shared memory limit once per size increase
    static size_t smem_limit = 48 * 1024;
    if (smem > smem_limit) {
        cudaError_t e = cudaFuncSetAttribute(paged_attn_kernel<T, DH>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(paged_attn)");
        smem_limit = smem;
    }
    dim3 grid(d.num_heads, a.batch, a.nlayers);
    paged_attn_kernel<T, DH><<<grid, kAttnThreads, smem, s>>>(kv->kv_map, pos_map, g, d.page_table,
                                                              d.meta, d.error, a);
    return cuda_status(cudaGetLastError(), "paged_attn_kernel");
}

}  // namespace

int launch_attention(const pk_paged_kv *kv, const CUtensorMap &pos_map, const AttnArgs &a,
                     cudaStream_t s) {
    if (a.batch == 0 || a.nlayers == 0) return PK_OK;
    const bool bf16 = kv->d.dtype == PK_DTYPE_BF16;
    switch (kv->head_dim) {
        case 64:
            return bf16 ? launch_typed<__nv_bfloat16, 64>(kv, pos_map, a, s)
                        : launch_typed<float, 64>(kv, pos_map, a, s);
        case 128:
            return bf16 ? launch_typed<__nv_bfloat16, 128>(kv, pos_map, a, s)
                        : launch_typed<float, 128>(kv, pos_map, a, s);
        default:
            return PK_ENOTSUP;
    }
}

}  // namespace pk
