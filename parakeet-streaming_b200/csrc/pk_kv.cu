// Paged K/V append and window gather: pure data movement with 128-bit
// loads and stores.
//
// append  replaces the shift-by-copy of ModelCache.update_attn_cache
//         (parakeet/modules/cache.py:36-45): only the chunk's new rows move.
// gather  materialises the dense window the reference returns from that
//         call (cache.py:45) and that pack_states copies out of the pool
//         (parakeet/engine/scheduler.py:150-161).
#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {
namespace {

// A stream's step context in shared memory: its slot, rows written so far
// (meta) and its page-table ring, read once per CTA.  Loads that do not depend
// on it are issued before it (they overlap its two dependent round trips).
struct SlotCtx {
    int ok, w;
    int ring[PK_WIN_MAX_PAGES];
};

__device__ __forceinline__ void load_slot_ctx(const pk_paged_kv_desc &d, const int32_t *slots,
                                              int b, SlotCtx &c) {
    if (threadIdx.x < 32) {
        const int s = slots[b];
        const bool ok = s >= 0 && s < d.num_slots;
        if (threadIdx.x < d.ring)
            c.ring[threadIdx.x] = ok ? d.page_table[(int64_t)s * d.ring + threadIdx.x] : -1;
        if (threadIdx.x == 0) {
            c.ok = ok;
            c.w = ok ? d.meta[(int64_t)s * PK_META_STRIDE + PK_META_WRITTEN] : 0;
            if (!ok) raise(d.error, PK_DEV_BAD_SLOT);
        }
    }
    __syncthreads();
}

// grid (batch, num_layers), 2 * (16-byte vectors per row) threads: thread
// (K|V, v) moves vector v of the chunk's TM >= T new rows of one (stream,
// layer).  The rows are loaded first; the slot context is read meanwhile.
template <int TM>
__global__ void __launch_bounds__(512)
    append_kernel(pk_paged_kv_desc d, int esize, int layer0, const char *key, const char *value,
                  int64_t ls, int64_t bs, int64_t rs, const int32_t *slots) {
    __shared__ SlotCtx ctx;
    const int b = blockIdx.x, lrel = blockIdx.y, l = layer0 + lrel;
    const int vpr = d.dim * esize / 16;   // 16-byte vectors per row
    const int vph = vpr / d.num_heads;    // per head row
    const int kvi = threadIdx.x / vpr, v = threadIdx.x - kvi * vpr;
    const int h = v / vph, vin = v - h * vph;
    const uint4 *src = reinterpret_cast<const uint4 *>((kvi ? value : key) +
                                                       ((int64_t)lrel * ls + (int64_t)b * bs) * esize) + v;
    const int64_t rs16 = rs * esize / 16;
    grid_dep_wait();     // the new rows may come from the previous kernel
    grid_dep_launch();   // one wave: the next kernel may be scheduled (it waits for us)
    uint4 val[TM];
#pragma unroll
    for (int t = 0; t < TM; ++t)
        if (t < d.chunk) val[t] = __ldcs(src + t * rs16);   // read once: evict first
    load_slot_ctx(d, slots, b, ctx);
    if (!ctx.ok) return;
    const int ps_shift = __ffs(d.page_size) - 1;
    char *pool = static_cast<char *>(d.kv);
    const int dh_bytes = vph * 16;
#pragma unroll
    for (int t = 0; t < TM; ++t) {
        if (t >= d.chunk) break;
        const int a = ctx.w + t;
        const int page = ctx.ring[(a >> ps_shift) & (d.ring - 1)];
        if (page < 0 || page >= d.num_pages) {
            raise(d.error, PK_DEV_BAD_PAGE);
            continue;
        }
        const int64_t plane = (((int64_t)page * d.num_layers + l) * 2 + kvi) * d.num_heads + h;
        char *dst = pool + ((plane << ps_shift) + (a & (d.page_size - 1))) * dh_bytes + vin * 16;
        *reinterpret_cast<uint4 *>(dst) = val[t];
    }
}

constexpr int kGatherThreads = 256;
constexpr int kGatherBatch = 8;

// grid (batch, 2 * num_layers, splits): CTA (b, (l, K|V), z) writes window rows
// [z * rows, (z + 1) * rows) of out[l][b][W][dim].  A warp reads four 128-byte head
// rows and writes 512 contiguous bytes.
__global__ void __launch_bounds__(kGatherThreads)
    gather_kernel(pk_paged_kv_desc d, int esize, int layer0, const int32_t *slots, char *k_out,
                  char *v_out, int64_t out_ls, int rows) {
    __shared__ SlotCtx ctx;
    const int b = blockIdx.x, lrel = blockIdx.y >> 1, kvi = blockIdx.y & 1, l = layer0 + lrel;
    const int W = d.left + d.chunk;
    const int j0 = blockIdx.z * rows;
    const int nrows = min(rows, W - j0);
    grid_dep_wait();     // pages and counters may come from the previous kernel
    grid_dep_launch();   // one wave: the next kernel may be scheduled (it waits for us)
    if (nrows <= 0) return;
    load_slot_ctx(d, slots, b, ctx);
    const int vpr = d.dim * esize / 16, vph = vpr / d.num_heads, dh_bytes = vph * 16;
    const int items = nrows * vpr;
    char *out = (kvi ? v_out : k_out) + ((int64_t)lrel * out_ls + ((int64_t)b * W + j0) * d.dim) * esize;
    const char *pool = static_cast<const char *>(d.kv);
    for (int base = 0; base < items; base += kGatherBatch * kGatherThreads) {
        uint4 val[kGatherBatch];
#pragma unroll
        for (int k = 0; k < kGatherBatch; ++k) {
            const int it = base + threadIdx.x + k * kGatherThreads;
            val[k] = make_uint4(0, 0, 0, 0);
            if (it >= items) continue;
            const int r = it / vpr, v = it % vpr;
            const int a = ctx.w - d.left + j0 + r;   // frame slot; < 0 reads as zero
            if (!ctx.ok || a < 0) continue;
            const int page = ctx.ring[(a / d.page_size) & (d.ring - 1)];
            if (page < 0 || page >= d.num_pages) {
                raise(d.error, PK_DEV_BAD_PAGE);
                continue;
            }
            const int h = v / vph;
            const int64_t plane = (((int64_t)page * d.num_layers + l) * 2 + kvi) * d.num_heads + h;
            val[k] = __ldcs(reinterpret_cast<const uint4 *>(   // read once: evict first
                pool + (plane * d.page_size + a % d.page_size) * dh_bytes + (v % vph) * 16));
        }
#pragma unroll
        for (int k = 0; k < kGatherBatch; ++k) {
            const int it = base + threadIdx.x + k * kGatherThreads;
            if (it < items) reinterpret_cast<uint4 *>(out)[it] = val[k];
        }
    }
}

}  // namespace

int launch_append(const pk_paged_kv *kv, int layer0, int nlayers, const void *key,
                  const void *value, int64_t ls, int64_t bs, int64_t rs, const int32_t *slots,
                  int batch, cudaStream_t s) {
    if (batch == 0 || nlayers == 0) return PK_OK;
    if (kv->d.ring > PK_WIN_MAX_PAGES) return PK_ENOTSUP;
    const int threads = 2 * kv->d.dim * kv->esize / 16;
    if (threads > 512 || kv->d.chunk > 16) return PK_ENOTSUP;
    dim3 grid(batch, nlayers);
    const char *k = static_cast<const char *>(key), *v = static_cast<const char *>(value);
    const int c = kv->d.chunk;
    auto kernel = c <= 2 ? append_kernel<2> : c <= 4 ? append_kernel<4>
                : c <= 8 ? append_kernel<8> : append_kernel<16>;
    return cuda_status(launch_pdl(kernel, grid, dim3(threads), 0, s, kv->d, kv->esize, layer0, k,
                                  v, ls, bs, rs, slots),
                       "append_kernel");
}

int launch_gather(const pk_paged_kv *kv, int layer0, int nlayers, const int32_t *slots, int batch,
                  void *k_out, void *v_out, int64_t out_ls, cudaStream_t s) {
    if (batch == 0 || nlayers == 0) return PK_OK;
    if (kv->d.ring > PK_WIN_MAX_PAGES) return PK_ENOTSUP;
    const int W = kv->d.left + kv->d.chunk;
    // about kGatherBatch vectors per thread per CTA
    const int vpr = kv->d.dim * kv->esize / 16;
    int rows = (kGatherBatch * kGatherThreads) / vpr;
    if (rows < 1) rows = 1;
    if (rows > W) rows = W;
    dim3 grid(batch, 2 * nlayers, (W + rows - 1) / rows);
    return cuda_status(launch_pdl(gather_kernel, grid, dim3(kGatherThreads), 0, s, kv->d,
                                  kv->esize, layer0, slots, static_cast<char *>(k_out),
                                  static_cast<char *>(v_out), out_ls, rows),
                       "gather_kernel");
}

}  // namespace pk
