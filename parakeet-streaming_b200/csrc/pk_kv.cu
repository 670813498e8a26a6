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

// Element offset of (page, layer, K|V, row, model column) in the head-major
// pool [pages][layers][2][heads][page_size][head_dim].
__device__ __forceinline__ int64_t pool_offset(const pk_paged_kv_desc &d, int page, int layer,
                                               int kvi, int row, int col) {
    const int dh = d.dim / d.num_heads;
    const int h = col / dh;
    return (((((int64_t)page * d.num_layers + layer) * 2 + kvi) * d.num_heads + h) * d.page_size +
            row) * dh + (col - h * dh);
}

// grid (batch, num_layers); every CTA moves T rows of K and of V of one
// (stream, layer).  `esize` bytes per element, 16-byte vectors.
__global__ void __launch_bounds__(128)
    append_kernel(pk_paged_kv_desc d, int esize, int layer0, const char *key, const char *value,
                  int64_t ls, int64_t bs, int64_t rs, const int32_t *slots) {
    const int b = blockIdx.x;
    const int l = layer0 + blockIdx.y;
    const int s = slots[b];
    if (s < 0 || s >= d.num_slots) {
        if (threadIdx.x == 0) raise(d.error, PK_DEV_BAD_SLOT);
        return;
    }
    const int w = d.meta[(int64_t)s * PK_META_STRIDE + PK_META_WRITTEN];
    const int vpr = d.dim * esize / 16;  // 16-byte vectors per row
    const int items = 2 * d.chunk * vpr;
    char *pool = static_cast<char *>(d.kv);
    for (int it = threadIdx.x; it < items; it += blockDim.x) {
        const int v = it % vpr;
        const int t = (it / vpr) % d.chunk;
        const int kvi = it / (vpr * d.chunk);
        const int a = w + t;
        const int page = d.page_table[(int64_t)s * d.ring + ((a / d.page_size) & (d.ring - 1))];
        if (page < 0 || page >= d.num_pages) {
            raise(d.error, PK_DEV_BAD_PAGE);
            continue;
        }
        const char *src = (kvi ? value : key) +
                          ((int64_t)blockIdx.y * ls + (int64_t)b * bs + (int64_t)t * rs) * esize;
        const uint4 val = __ldg(reinterpret_cast<const uint4 *>(src) + v);
        const int col = v * (16 / esize);
        char *dst = pool + pool_offset(d, page, l, kvi, a % d.page_size, col) * esize;
        *reinterpret_cast<uint4 *>(dst) = val;
    }
}

// grid (batch, 2, ceil(W / kRows)); out [batch][W][dim] for K (y=0) and V (y=1).
constexpr int kGatherRows = 8;
__global__ void __launch_bounds__(256)
    gather_kernel(pk_paged_kv_desc d, int esize, int layer, const int32_t *slots, char *k_out,
                  char *v_out) {
    const int b = blockIdx.x;
    const int kvi = blockIdx.y;
    const int W = d.left + d.chunk;
    const int s = slots[b];
    const bool slot_ok = s >= 0 && s < d.num_slots;
    if (!slot_ok && threadIdx.x == 0) raise(d.error, PK_DEV_BAD_SLOT);
    const int w = slot_ok ? d.meta[(int64_t)s * PK_META_STRIDE + PK_META_WRITTEN] : 0;
    const int vpr = d.dim * esize / 16;
    const int j0 = blockIdx.z * kGatherRows;
    const int rows = min(kGatherRows, W - j0);
    char *out = (kvi ? v_out : k_out) + ((int64_t)b * W + j0) * d.dim * esize;
    const char *pool = static_cast<const char *>(d.kv);
    for (int it = threadIdx.x; it < rows * vpr; it += blockDim.x) {
        const int r = it / vpr, v = it % vpr;
        const int a = w - d.left + j0 + r;
        uint4 val = make_uint4(0, 0, 0, 0);
        if (slot_ok && a >= 0) {
            const int page =
                d.page_table[(int64_t)s * d.ring + ((a / d.page_size) & (d.ring - 1))];
            if (page >= 0 && page < d.num_pages) {
                const int col = v * (16 / esize);
                const char *src = pool + pool_offset(d, page, layer, kvi, a % d.page_size, col) * esize;
                val = __ldg(reinterpret_cast<const uint4 *>(src));
            } else {
                raise(d.error, PK_DEV_BAD_PAGE);
            }
        }
        reinterpret_cast<uint4 *>(out + (int64_t)r * d.dim * esize)[v] = val;
    }
}

}  // namespace

int launch_append(const pk_paged_kv *kv, int layer0, int nlayers, const void *key,
                  const void *value, int64_t ls, int64_t bs, int64_t rs, const int32_t *slots,
                  int batch, cudaStream_t s) {
    if (batch == 0 || nlayers == 0) return PK_OK;
    dim3 grid(batch, nlayers);
    append_kernel<<<grid, 128, 0, s>>>(kv->d, kv->esize, layer0, static_cast<const char *>(key),
                                       static_cast<const char *>(value), ls, bs, rs, slots);
    return cuda_status(cudaGetLastError(), "append_kernel");
}

int launch_gather(const pk_paged_kv *kv, int layer, const int32_t *slots, int batch, void *k_out,
                  void *v_out, cudaStream_t s) {
    if (batch == 0) return PK_OK;
    const int W = kv->d.left + kv->d.chunk;
    dim3 grid(batch, 2, (W + kGatherRows - 1) / kGatherRows);
    gather_kernel<<<grid, 256, 0, s>>>(kv->d, kv->esize, layer, slots,
                                       static_cast<char *>(k_out), static_cast<char *>(v_out));
    return cuda_status(cudaGetLastError(), "gather_kernel");
}

}  // namespace pk
