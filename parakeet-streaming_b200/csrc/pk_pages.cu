// Device page allocator for the paged K/V window, and the step's window
// descriptors.
//
// The reference keeps one dense window per slot (parakeet/modules/cache.py:24-29)
// and hands out slots from a FIFO deque (parakeet/engine/scheduler.py:84,93-104).
// Here every slot owns a ring of page-table entries and pages come from one
// FIFO free ring.  One CTA runs each step's releases, frees and allocations in
// batch order with block-wide scans, so the page-id sequence is deterministic
// and equals the CPU model op for op; the same CTA then writes, one warp per
// batch row, the row's window descriptor: its pages, the first row of each
// page's TMA box, and the streaming mask of ConformerEncoder.
// _create_streaming_masks (parakeet/modules/encoder.py:167-227) as bit rows.
#include <cub/block/block_scan.cuh>

#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {
namespace {

constexpr int kAllocThreads = 1024;
constexpr int kRowsPerThread = 4;   // batch <= 4096
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

// Window descriptor of batch row b (one warp): pages of rows [w - left, w + chunk),
// each page's box start row, and the mask bit rows.
__device__ void build_window(const pk_paged_kv_desc &d, const int32_t *slots,
                             const int32_t *lengths, int b, int lane) {
    const int chunk = d.chunk, W = d.left + d.chunk, ps = d.page_size;
    int32_t *out = d.window + (int64_t)b * PK_WIN_STRIDE;
    int ok = 1, w = 0, proc = 0, clen = 0, len = chunk;
    const int slot = slots[b];
    if (slot < 0 || slot >= d.num_slots) {
        ok = 0;
    } else {
        const int32_t *m = d.meta + (int64_t)slot * PK_META_STRIDE;
        w = m[PK_META_WRITTEN];
        proc = m[PK_META_PROCESSED];
        clen = m[PK_META_CACHE_LEN];
        if (lengths) len = lengths[b];
    }
    const int a_lo = max(w - d.left, 0), a_hi = w + chunk;
    const int nfirst = a_lo / ps;
    const int nb = (a_hi - 1) / ps - nfirst + 1;
    if (nb > PK_WIN_MAX_PAGES) ok = 0;
    int page = -1, start = 0;
    if (ok && lane < nb) {
        const int n = nfirst + lane;
        page = d.page_table[(int64_t)slot * d.ring + (n & (d.ring - 1))];
        const int lo = max(a_lo - n * ps, 0), hi = min(a_hi - n * ps, ps);
        start = lo > 0 ? lo : (hi < ps ? hi - ps : 0);
    }
    if (__any_sync(0xffffffffu, ok && lane < nb && (page < 0 || page >= d.num_pages))) {
        if (lane == 0) raise(d.error, PK_DEV_BAD_PAGE);
        ok = 0;
    }
    if (lane < PK_WIN_MAX_PAGES) {
        out[PK_WIN_PAGE + lane] = lane < nb ? page : -1;
        out[PK_WIN_START + lane] = start;
    }
    // mask rows < chunk; rows >= chunk stay zero
    const int key_start = max(proc - clen, 0), off = d.left - clen;
    const int left_chunks = d.left / chunk;
    for (int kb = 0; kb < 4; ++kb) {
        const int j = kb * 32 + lane;
        bool key_ok = ok && j < W && j >= off;
        int kc = 0;
        if (key_ok) {
            const int rr = j - off;
            key_ok = rr < clen || (rr - clen) < len;
            kc = (key_start + rr) / chunk;
        }
        int qc = (key_start + clen) / chunk, qrem = (key_start + clen) % chunk;
        for (int i = 0; i < chunk; ++i) {
            const int dc = qc - kc;
            const unsigned bits =
                __ballot_sync(0xffffffffu, key_ok && i < len && dc >= 0 && dc <= left_chunks);
            if (lane == 0) out[PK_WIN_MASK + i * 4 + kb] = (int32_t)bits;
            if (++qrem == chunk) {
                qrem = 0;
                ++qc;
            }
        }
    }
    for (int idx = chunk * 4 + lane; idx < 64; idx += 32) out[PK_WIN_MASK + idx] = 0;
    if (lane == 0) {
        out[PK_WIN_OK] = ok;
        out[PK_WIN_W] = w;
        out[PK_WIN_PROC] = proc;
        out[PK_WIN_CLEN] = clen;
        out[PK_WIN_LEN] = len;
        out[PK_WIN_NB] = nb;
        out[PK_WIN_NFIRST] = nfirst;
        out[PK_WIN_SLOT] = slot;
    }
}

__global__ void __launch_bounds__(kAllocThreads)
    pages_begin_kernel(pk_paged_kv_desc d, const int32_t *slots, const int32_t *lengths,
                       int batch, const int32_t *released, int num_released) {
    __shared__ typename Scan::TempStorage scan_tmp;
    __shared__ int64_t s_head, s_tail;
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

    // this thread's batch rows b = tid + k * 1024 and their counters, read once
    int slot[kRowsPerThread], first[kRowsPerThread], next[kRowsPerThread], wr[kRowsPerThread];
#pragma unroll
    for (int k = 0; k < kRowsPerThread; ++k) {
        const int b = tid + k * kAllocThreads;
        slot[k] = -1;
        first[k] = next[k] = wr[k] = 0;
        if (b < batch) {
            const int s = slots[b];
            if (s >= 0 && s < d.num_slots) {
                const int32_t *m = d.meta + (int64_t)s * PK_META_STRIDE;
                slot[k] = s;
                first[k] = m[PK_META_FIRST];
                next[k] = m[PK_META_NEXT];
                wr[k] = m[PK_META_WRITTEN];
            } else {
                raise(d.error, PK_DEV_BAD_SLOT);
            }
        }
    }

    // 1. frees: pages n with (n + 1) * page_size <= written - left, batch order
#pragma unroll
    for (int k = 0; k < kRowsPerThread; ++k) {
        if (k * kAllocThreads >= batch) break;
        int nfree = 0;
        if (slot[k] >= 0) {
            const int lim = wr[k] - d.left;
            while (first[k] + nfree < next[k] && (first[k] + nfree + 1) * d.page_size <= lim) ++nfree;
        }
        int off, total;
        Scan(scan_tmp).ExclusiveSum(nfree, off, total);
        if (nfree > 0) {
            int32_t *row = d.page_table + (int64_t)slot[k] * d.ring;
            for (int j = 0; j < nfree; ++j) {
                int32_t *e = row + ((first[k] + j) & (d.ring - 1));
                d.free_ring[ring_idx(s_tail + off + j, N)] = *e;
                *e = -1;
            }
            first[k] += nfree;
            d.meta[(int64_t)slot[k] * PK_META_STRIDE + PK_META_FIRST] = first[k];
        }
        __syncthreads();
        if (tid == 0) s_tail += total;
        __syncthreads();
    }

    // 2. allocations from the head, batch order; all-or-nothing like the CPU model
    int need[kRowsPerThread];
    int demand = 0;
#pragma unroll
    for (int k = 0; k < kRowsPerThread; ++k) {
        need[k] = 0;
        if (slot[k] >= 0) need[k] = max(0, (wr[k] + d.chunk - 1) / d.page_size - next[k] + 1);
        demand += need[k];
    }
    int demand_off, total_demand;
    Scan(scan_tmp).ExclusiveSum(demand, demand_off, total_demand);
    __syncthreads();
    if (tid == 0 && (int64_t)total_demand > s_tail - s_head) {
        s_fail = 1;
        raise(d.error, PK_DEV_POOL_EXHAUSTED);
    }
    __syncthreads();
    if (!s_fail) {
#pragma unroll
        for (int k = 0; k < kRowsPerThread; ++k) {
            if (k * kAllocThreads >= batch) break;
            int off, total;
            Scan(scan_tmp).ExclusiveSum(need[k], off, total);
            if (need[k] > 0) {
                int32_t *row = d.page_table + (int64_t)slot[k] * d.ring;
                for (int j = 0; j < need[k]; ++j)
                    row[(next[k] + j) & (d.ring - 1)] = d.free_ring[ring_idx(s_head + off + j, N)];
                d.meta[(int64_t)slot[k] * PK_META_STRIDE + PK_META_NEXT] = next[k] + need[k];
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
    __syncthreads();   // page table of this step visible to every warp of the block

    // 3. window descriptors, one warp per batch row
    const int warp = tid / 32, lane = tid % 32;
    for (int b = warp; b < batch; b += kAllocThreads / 32) build_window(d, slots, lengths, b, lane);
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

int launch_pages_begin(const pk_paged_kv *kv, const int32_t *slots, const int32_t *lengths,
                       int batch, const int32_t *released, int num_released, cudaStream_t s) {
    if (batch > kAllocThreads * kRowsPerThread) return PK_ENOTSUP;
    pages_begin_kernel<<<1, kAllocThreads, 0, s>>>(kv->d, slots, lengths, batch, released,
                                                   num_released);
    return cuda_status(cudaGetLastError(), "pages_begin_kernel");
}

int launch_pages_end(const pk_paged_kv *kv, const int32_t *slots, const int32_t *lengths,
                     int batch, cudaStream_t s) {
    if (batch == 0) return PK_OK;
    pages_end_kernel<<<(batch + 255) / 256, 256, 0, s>>>(kv->d, slots, lengths, batch);
    return cuda_status(cudaGetLastError(), "pages_end_kernel");
}

}  // namespace pk
