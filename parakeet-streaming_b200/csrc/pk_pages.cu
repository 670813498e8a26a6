// Device page allocator for the paged K/V window.
//
// The reference keeps one dense window per slot (parakeet/modules/cache.py:24-29)
// and hands out slots from a FIFO deque (parakeet/engine/scheduler.py:84,93-104).
// Here every slot owns a ring of page-table entries and pages come from one
// FIFO free ring.  A single CTA runs each step's releases, frees and
// allocations in batch order with block-wide scans, so the page-id sequence
// is deterministic and equals the CPU model op for op.
#include <cub/block/block_scan.cuh>

#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {
namespace {

constexpr int kAllocThreads = 1024;
using Scan = cub::BlockScan<int, kAllocThreads>;

__global__ void pages_reset_kernel(pk_paged_kv_desc d, const int32_t *init_order) {
    const int tid = blockIdx.x * blockDim.x + threadIdx.x;
    const int n = gridDim.x * blockDim.x;
    for (int i = tid; i < d.num_pages; i += n) d.free_ring[i] = init_order ? init_order[i] : i;
    for (int i = tid; i < d.num_slots * d.ring; i += n) d.page_table[i] = -1;
    for (int i = tid; i < d.num_slots * PK_META_STRIDE; i += n) d.meta[i] = 0;
    if (tid == 0) {
        d.ring_ctr[0] = 0;            // head: next entry to pop
        d.ring_ctr[1] = d.num_pages;  // tail: next entry to push
        *d.error = 0;
    }
}

__device__ __forceinline__ int64_t ring_idx(int64_t ctr, int n) { return ctr % n; }

__global__ void __launch_bounds__(kAllocThreads)
    pages_begin_kernel(pk_paged_kv_desc d, const int32_t *slots, int batch,
                       const int32_t *released, int num_released) {
    __shared__ typename Scan::TempStorage scan_tmp;
    __shared__ int64_t s_head, s_tail;
    __shared__ int s_total;
    __shared__ int s_fail;
    const int tid = threadIdx.x;
    const int N = d.num_pages;

    if (tid == 0) {
        s_head = d.ring_ctr[0];
        s_tail = d.ring_ctr[1];
        s_fail = 0;
        // 0. releases, in release order (serial: a handful of pages each)
        for (int r = 0; r < num_released; ++r) {
            const int s = released[r];
            if (s < 0 || s >= d.num_slots) {
                raise(d.error, PK_DEV_BAD_SLOT);
                continue;
            }
            int32_t *m = d.meta + (int64_t)s * PK_META_STRIDE;
            for (int pg = m[PK_META_FIRST]; pg < m[PK_META_NEXT]; ++pg) {
                int32_t *e = d.page_table + (int64_t)s * d.ring + (pg & (d.ring - 1));
                d.free_ring[ring_idx(s_tail++, N)] = *e;
                *e = -1;
            }
            for (int f = 0; f < PK_META_STRIDE; ++f) m[f] = 0;
        }
    }
    __syncthreads();

    // 1. frees: pages n with (n + 1) * page_size <= written - left, batch order
    for (int base = 0; base < batch; base += kAllocThreads) {
        const int b = base + tid;
        int s = -1, first = 0, nfree = 0;
        if (b < batch) {
            s = slots[b];
            if (s >= 0 && s < d.num_slots) {
                const int32_t *m = d.meta + (int64_t)s * PK_META_STRIDE;
                first = m[PK_META_FIRST];
                const int next = m[PK_META_NEXT];
                const int lim = m[PK_META_WRITTEN] - d.left;
                while (first + nfree < next && (first + nfree + 1) * d.page_size <= lim) ++nfree;
            } else {
                raise(d.error, PK_DEV_BAD_SLOT);
                s = -1;
            }
        }
        int off, total;
        Scan(scan_tmp).ExclusiveSum(nfree, off, total);
        if (s >= 0 && nfree > 0) {
            int32_t *row = d.page_table + (int64_t)s * d.ring;
            for (int k = 0; k < nfree; ++k) {
                int32_t *e = row + ((first + k) & (d.ring - 1));
                d.free_ring[ring_idx(s_tail + off + k, N)] = *e;
                *e = -1;
            }
            d.meta[(int64_t)s * PK_META_STRIDE + PK_META_FIRST] = first + nfree;
        }
        __syncthreads();
        if (tid == 0) s_tail += total;
        __syncthreads();
    }

    // 2a. total demand of the batch; all-or-nothing like the CPU model
    int demand = 0;
    for (int base = 0; base < batch; base += kAllocThreads) {
        const int b = base + tid;
        int need = 0;
        if (b < batch) {
            const int s = slots[b];
            if (s >= 0 && s < d.num_slots) {
                const int32_t *m = d.meta + (int64_t)s * PK_META_STRIDE;
                const int last = (m[PK_META_WRITTEN] + d.chunk - 1) / d.page_size;
                need = max(0, last - m[PK_META_NEXT] + 1);
            }
        }
        int off, total;
        Scan(scan_tmp).ExclusiveSum(need, off, total);
        demand += total;
        __syncthreads();
    }
    if (tid == 0) {
        s_total = demand;
        if ((int64_t)demand > s_tail - s_head) {
            s_fail = 1;
            raise(d.error, PK_DEV_POOL_EXHAUSTED);
        }
    }
    __syncthreads();

    // 2b. allocations from the head, batch order
    if (!s_fail) {
        for (int base = 0; base < batch; base += kAllocThreads) {
            const int b = base + tid;
            int s = -1, next = 0, need = 0;
            if (b < batch) {
                s = slots[b];
                if (s >= 0 && s < d.num_slots) {
                    const int32_t *m = d.meta + (int64_t)s * PK_META_STRIDE;
                    next = m[PK_META_NEXT];
                    const int last = (m[PK_META_WRITTEN] + d.chunk - 1) / d.page_size;
                    need = max(0, last - next + 1);
                } else {
                    s = -1;
                }
            }
            int off, total;
            Scan(scan_tmp).ExclusiveSum(need, off, total);
            if (s >= 0 && need > 0) {
                int32_t *row = d.page_table + (int64_t)s * d.ring;
                for (int k = 0; k < need; ++k)
                    row[(next + k) & (d.ring - 1)] = d.free_ring[ring_idx(s_head + off + k, N)];
                d.meta[(int64_t)s * PK_META_STRIDE + PK_META_NEXT] = next + need;
            }
            __syncthreads();
            if (tid == 0) s_head += total;
            __syncthreads();
        }
    }
    if (tid == 0) {
        d.ring_ctr[0] = s_head;
        d.ring_ctr[1] = s_tail;
    }
}

__global__ void pages_end_kernel(pk_paged_kv_desc d, const int32_t *slots, const int32_t *lengths,
                                 int batch) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= batch) return;
    const int s = slots[b];
    if (s < 0 || s >= d.num_slots) {
        raise(d.error, PK_DEV_BAD_SLOT);
        return;
    }
    int32_t *m = d.meta + (int64_t)s * PK_META_STRIDE;
    const int n = lengths[b];
    m[PK_META_WRITTEN] += d.chunk;
    m[PK_META_PROCESSED] += n;
    m[PK_META_CACHE_LEN] = min(m[PK_META_CACHE_LEN] + n, d.left);
}

}  // namespace

int launch_pages_reset(const pk_paged_kv *kv, const int32_t *init_order, cudaStream_t s) {
    pages_reset_kernel<<<148, 256, 0, s>>>(kv->d, init_order);
    return cuda_status(cudaGetLastError(), "pages_reset_kernel");
}

int launch_pages_begin(const pk_paged_kv *kv, const int32_t *slots, int batch,
                       const int32_t *released, int num_released, cudaStream_t s) {
    pages_begin_kernel<<<1, kAllocThreads, 0, s>>>(kv->d, slots, batch, released, num_released);
    return cuda_status(cudaGetLastError(), "pages_begin_kernel");
}

int launch_pages_end(const pk_paged_kv *kv, const int32_t *slots, const int32_t *lengths,
                     int batch, cudaStream_t s) {
    if (batch == 0) return PK_OK;
    pages_end_kernel<<<(batch + 255) / 256, 256, 0, s>>>(kv->d, slots, lengths, batch);
    return cuda_status(cudaGetLastError(), "pages_end_kernel");
}

}  // namespace pk
