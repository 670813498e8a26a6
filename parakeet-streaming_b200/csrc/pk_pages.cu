// Device page allocator for the paged K/V window, and the step's window
// descriptors.
//
// The reference keeps one dense window per slot (parakeet/modules/cache.py:24-29)
// and hands out slots from a FIFO deque (parakeet/engine/scheduler.py:84,93-104).
// Here every slot owns a ring of page-table entries and pages come from one
// FIFO free ring.  One CTA, one thread per batch row, runs each step's
// releases, frees and allocations in batch order with block-wide scans, so the
// page-id sequence is deterministic and equals the CPU model op for op; each
// row's thread then writes the row's window descriptor: its pages, the first
// row of each page's TMA box, and the streaming mask of ConformerEncoder.
// _create_streaming_masks (parakeet/modules/encoder.py:167-227) as bit rows.
#include "pk_common.cuh"
#include "pk_internal.h"
#include "pk_relpos.cuh"

namespace pk {
namespace {

constexpr int kAllocThreads = 1024;            // most threads of the step-start CTA
// Rows of one step: up to 2048 the rows keep a copy of their page-table rings in
// shared memory (96 bytes a row); up to 6144 the rings stay in global memory
// (32 bytes of shared memory a row).  Both fit the CTA's 192 KB.
constexpr int kMaxBatchShared = 2 * kAllocThreads;
constexpr int kMaxBatch = 6 * kAllocThreads;
static_assert(kMaxBatch == PK_MAX_BATCH, "step rows");
constexpr int kMaxBatchRelpos = 256;           // step start fused with the rel-pos pre-pass

// Exclusive prefix sum of v over the CTA (blockDim.x a multiple of 32), in batch
// order of the threads; `total` gets the CTA's sum.  s_warp: 33 ints of scratch.
__device__ int block_exclusive_sum(int v, int &total, int *s_warp) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) s_warp[wid] = x;
    __syncthreads();
    if (wid == 0) {
        int t = lane < nw ? s_warp[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, t, o);
            if (lane >= o) t += y;
        }
        if (lane < nw) s_warp[lane] = t;   // inclusive over warps
        if (lane == 31) s_warp[32] = t;
    }
    __syncthreads();
    total = s_warp[32];
    const int res = (wid > 0 ? s_warp[wid - 1] : 0) + x - v;
    __syncthreads();   // scratch free for the next scan
    return res;
}

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

// Per-row state of one step, in shared memory: the row's slot and counters,
// and a copy of its page-table ring (ring <= PK_WIN_MAX_PAGES entries).
struct RowState {
    int slot, len, first, next, w, proc, clen, valid;
};

__device__ __forceinline__ unsigned range_bits(int lo, int hi, int base) {
    const int a = max(lo, base), b = min(hi, base + 32);
    if (a >= b) return 0u;
    const unsigned n = (unsigned)(b - a);
    return (n == 32u ? 0xffffffffu : ((1u << n) - 1u)) << (a - base);
}

// Window descriptor of one batch row, written by the thread that owns the row:
// pages of rows [w - left, w + chunk), each page's box start row, and the mask
// bit rows.  Key j of query row i is visible when ConformerEncoder's mask allows
// it (parakeet/modules/encoder.py:167-227): the key holds a real frame,
// j - off < clen + len, and its chunk index is 0..left/chunk chunks behind the
// query's.  Both conditions are intervals in j, so each bit row is one range.
__device__ void write_window(const pk_paged_kv_desc &d, const RowState &r, const int *ring,
                             int b) {
    const int chunk = d.chunk, W = d.left + chunk, ps = d.page_size, rmask = d.ring - 1;
    int4 *out = reinterpret_cast<int4 *>(d.window + (int64_t)b * PK_WIN_STRIDE);
    int ok = r.valid;
    const int a_lo = max(r.w - d.left, 0), a_hi = r.w + chunk;
    const int nfirst = a_lo / ps;
    const int nb = (a_hi - 1) / ps - nfirst + 1;
    if (nb > PK_WIN_MAX_PAGES) ok = 0;
    bool bad = false;
#pragma unroll
    for (int g = 0; g < PK_WIN_MAX_PAGES / 4; ++g) {
        int pv[4], sv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int l = g * 4 + e;
            pv[e] = -1;
            sv[e] = 0;
            if (ok && l < nb) {
                const int n = nfirst + l;
                pv[e] = ring[n & rmask];
                bad |= pv[e] < 0 || pv[e] >= d.num_pages;
                const int lo = max(a_lo - n * ps, 0), hi = min(a_hi - n * ps, ps);
                sv[e] = lo > 0 ? lo : (hi < ps ? hi - ps : 0);
            }
        }
        out[PK_WIN_PAGE / 4 + g] = make_int4(pv[0], pv[1], pv[2], pv[3]);
        out[PK_WIN_START / 4 + g] = make_int4(sv[0], sv[1], sv[2], sv[3]);
    }
    if (bad) {
        raise(d.error, PK_DEV_BAD_PAGE);
        ok = 0;
    }
    const int key_start = max(r.proc - r.clen, 0), off = d.left - r.clen;
    const int lc = d.left / chunk;
    for (int i = 0; i < 16; ++i) {
        int4 m = make_int4(0, 0, 0, 0);
        if (ok && i < chunk && i < r.len) {
            const int qc = (key_start + r.clen + i) / chunk;
            const int lo = off + max(0, (qc - lc) * chunk - key_start);
            const int hi = min(W, off + min(r.clen + r.len, (qc + 1) * chunk - key_start));
            m = make_int4((int)range_bits(lo, hi, 0), (int)range_bits(lo, hi, 32),
                          (int)range_bits(lo, hi, 64), (int)range_bits(lo, hi, 96));
        }
        out[PK_WIN_MASK / 4 + i] = m;
    }
    out[0] = make_int4(ok, r.w, r.proc, r.clen);
    out[1] = make_int4(r.len, nb, nfirst, r.slot);
}

// One CTA, one thread per batch row (several for batches above the CTA's
// threads).  Every row keeps its owner thread through all phases, so only the
// scans cross threads.  kSharedRings: each row's page-table ring is copied to
// shared memory and written to both copies; otherwise the owner thread reads
// and writes the slot's ring in global memory.
template <bool kSharedRings>
__device__ __forceinline__ void pages_begin_body(const pk_paged_kv_desc &d, const int32_t *slots,
                                                 const int32_t *lengths, int batch,
                                                 const int32_t *released, int num_released) {
    extern __shared__ __align__(16) int s_dyn[];
    __shared__ int scan_tmp[33];
    __shared__ int64_t s_ctr[2];
    RowState *rows = reinterpret_cast<RowState *>(s_dyn);
    int *rings = s_dyn + batch * (int)(sizeof(RowState) / sizeof(int));   // kSharedRings only
    // ring of row b (slot s): shared copy or the page table itself
    auto ring_of = [&](int b, int s) -> int32_t * {
        return kSharedRings ? rings + b * PK_WIN_MAX_PAGES : d.page_table + (int64_t)s * d.ring;
    };
    const int tid = threadIdx.x;
    const int N = d.num_pages, rmask = d.ring - 1;
    const int nthreads = blockDim.x;
    const int nk = (batch + nthreads - 1) / nthreads;
    grid_dep_wait();     // the previous step's counters and this step's inputs
    grid_dep_launch();   // the step's attention may be scheduled (it waits for us)

    // inputs first: they do not depend on the releases below
    for (int k = 0; k < nk; ++k) {
        const int b = tid + k * nthreads;
        if (b < batch) {
            rows[b].slot = slots[b];
            rows[b].len = lengths ? lengths[b] : d.chunk;
        }
    }
    if (tid == 0) {
        int64_t tail = d.ring_ctr[1];
        s_ctr[0] = d.ring_ctr[0];
        // 0. releases, in release order (serial: a handful of pages each)
        for (int r = 0; r < num_released; ++r) {
            const int s = released[r];
            if (s < 0 || s >= d.num_slots) {
                raise(d.error, PK_DEV_BAD_SLOT);
                continue;
            }
            int32_t *m = d.meta + (int64_t)s * PK_META_STRIDE;
            for (int pg = m[PK_META_FIRST]; pg < m[PK_META_NEXT]; ++pg) {
                int32_t *e = d.page_table + (int64_t)s * d.ring + (pg & rmask);
                d.free_ring[tail++ % N] = *e;
                *e = -1;
            }
            for (int f = 0; f < PK_META_STRIDE; ++f) m[f] = 0;
        }
        s_ctr[1] = tail;
    }
    __syncthreads();

    // counters and page-table ring of each row (after the releases reset theirs)
    for (int k = 0; k < nk; ++k) {
        const int b = tid + k * nthreads;
        if (b >= batch) continue;
        RowState &r = rows[b];
        const int s = r.slot;
        r.valid = s >= 0 && s < d.num_slots;
        r.first = r.next = r.w = r.proc = r.clen = 0;
        if (r.valid) {
            const int32_t *m = d.meta + (int64_t)s * PK_META_STRIDE;
            const int32_t *pt = d.page_table + (int64_t)s * d.ring;
            r.first = m[PK_META_FIRST];
            r.next = m[PK_META_NEXT];
            r.w = m[PK_META_WRITTEN];
            r.proc = m[PK_META_PROCESSED];
            r.clen = m[PK_META_CACHE_LEN];
            if (kSharedRings) {
#pragma unroll
                for (int p = 0; p < PK_WIN_MAX_PAGES; ++p)
                    if (p <= rmask) rings[b * PK_WIN_MAX_PAGES + p] = pt[p];
            }
        } else {
            r.len = d.chunk;
            raise(d.error, PK_DEV_BAD_SLOT);
        }
    }
    int64_t head = s_ctr[0], tail = s_ctr[1];

    // 1. frees: pages n < (written - left) / page_size still held, batch order
    for (int k = 0; k < nk; ++k) {
        const int b = tid + k * nthreads;
        int nfree = 0;
        if (b < batch && rows[b].valid) {
            const int lim = rows[b].w - d.left;   // C division: <= 0 pages for lim < page_size
            nfree = max(0, min(rows[b].next, lim / d.page_size) - rows[b].first);
        }
        int total;
        const int off = block_exclusive_sum(nfree, total, scan_tmp);
        if (nfree > 0) {
            RowState &r = rows[b];
            int32_t *pt = d.page_table + (int64_t)r.slot * d.ring;
            int32_t *rg = ring_of(b, r.slot);
            for (int j = 0; j < nfree; ++j) {
                const int pos = (r.first + j) & rmask;
                d.free_ring[(tail + off + j) % N] = rg[pos];
                rg[pos] = -1;
                if (kSharedRings) pt[pos] = -1;
            }
            r.first += nfree;
            d.meta[(int64_t)r.slot * PK_META_STRIDE + PK_META_FIRST] = r.first;
        }
        tail += total;
        __syncthreads();   // scan storage reuse; pushed entries visible to the pops
    }

    // 2. allocations from the head, batch order; all-or-nothing like the CPU model
    int demand = 0;
    for (int k = 0; k < nk; ++k) {
        const int b = tid + k * nthreads;
        if (b < batch && rows[b].valid)
            demand += max(0, (rows[b].w + d.chunk - 1) / d.page_size - rows[b].next + 1);
    }
    int total_demand;
    block_exclusive_sum(demand, total_demand, scan_tmp);
    if ((int64_t)total_demand > tail - head) {   // block-uniform
        if (tid == 0) raise(d.error, PK_DEV_POOL_EXHAUSTED);
    } else {
        for (int k = 0; k < nk; ++k) {
            const int b = tid + k * nthreads;
            int need = 0;
            if (b < batch && rows[b].valid)
                need = max(0, (rows[b].w + d.chunk - 1) / d.page_size - rows[b].next + 1);
            int total;
            const int off = block_exclusive_sum(need, total, scan_tmp);
            if (need > 0) {
                RowState &r = rows[b];
                int32_t *pt = d.page_table + (int64_t)r.slot * d.ring;
                int32_t *rg = ring_of(b, r.slot);
                for (int j = 0; j < need; ++j) {
                    const int pos = (r.next + j) & rmask;
                    const int page = d.free_ring[(head + off + j) % N];
                    rg[pos] = page;
                    if (kSharedRings) pt[pos] = page;
                }
                r.next += need;
                d.meta[(int64_t)r.slot * PK_META_STRIDE + PK_META_NEXT] = r.next;
            }
            head += total;
            __syncthreads();
        }
    }
    if (tid == 0) {
        d.ring_ctr[0] = head;
        d.ring_ctr[1] = tail;
    }

    // 3. window descriptors: each thread its own rows
    for (int k = 0; k < nk; ++k) {
        const int b = tid + k * nthreads;
        if (b < batch) write_window(d, rows[b], ring_of(b, rows[b].slot), b);
    }
}

template <bool kSharedRings>
__global__ void __launch_bounds__(kAllocThreads)
    pages_begin_kernel(pk_paged_kv_desc d, const int32_t *slots, const int32_t *lengths,
                       int batch, const int32_t *released, int num_released) {
    pages_begin_body<kSharedRings>(d, slots, lengths, batch, released, num_released);
}

// The step start and the all-stream rel-pos pre-pass in one launch: CTA 0 runs
// the allocator and window descriptors, CTAs 1.. one pre-pass tile each.  They
// touch disjoint memory, so the allocator's serial chain and the tiles overlap
// instead of being two links of the step's launch chain.
__global__ void __launch_bounds__(kRelposThreads, 5)
    pages_begin_relpos_kernel(pk_paged_kv_desc d, const int32_t *slots, const int32_t *lengths,
                              int batch, const int32_t *released, int num_released,
                              const AttnArgs a, int bds, float *bd, int tiles_z) {
    if (blockIdx.x == 0) {
        pages_begin_body<true>(d, slots, lengths, batch, released, num_released);
        return;
    }
    grid_dep_wait();     // q may come from the previous kernel
    grid_dep_launch();
    const int t = blockIdx.x - 1, z = t % tiles_z, lh = t / tiles_z;
    relpos_tile(d, a, bds, bd, lh / d.num_heads, lh % d.num_heads, z);
}

__global__ void pages_end_kernel(pk_paged_kv_desc d, const int32_t *slots, const int32_t *lengths,
                                 int batch) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    grid_dep_wait();
    grid_dep_launch();
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
    if (batch > kMaxBatch || kv->d.ring > PK_WIN_MAX_PAGES) return PK_ENOTSUP;
    const bool shared_rings = batch <= kMaxBatchShared;
    const size_t row_bytes = sizeof(RowState) + (shared_rings ? PK_WIN_MAX_PAGES * sizeof(int) : 0);
    const size_t smem = (size_t)batch * row_bytes;
    auto kernel = shared_rings ? pages_begin_kernel<true> : pages_begin_kernel<false>;
    static size_t limit[2] = {48 * 1024, 48 * 1024};
    size_t &lim = limit[shared_rings];
    if (smem > lim) {
        const size_t most = shared_rings
                                ? kMaxBatchShared * (sizeof(RowState) + PK_WIN_MAX_PAGES * sizeof(int))
                                : kMaxBatch * sizeof(RowState);
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)most);
        if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(pages_begin)");
        lim = most;
    }
    // one thread per row up to 1024 rows: small batches scan over a few warps only
    int threads = batch >= kAllocThreads ? kAllocThreads : (batch + 31) / 32 * 32;
    if (threads == 0) threads = 32;
    return cuda_status(launch_pdl(kernel, dim3(1), dim3(threads), smem, s, kv->d, slots, lengths,
                                  batch, released, num_released),
                       "pages_begin_kernel");
}

int launch_pages_begin_relpos(const pk_paged_kv *kv, const int32_t *slots,
                              const int32_t *lengths, int batch, const int32_t *released,
                              int num_released, const AttnArgs &a, float *bd, cudaStream_t s) {
    const int bds = relpos_bd_cols(kv);
    // the allocator runs in a pre-pass-sized CTA here, and every tile CTA gets
    // the allocator's shared memory: small batches only
    if (bds == 0 || batch > kMaxBatchRelpos || kv->d.ring > PK_WIN_MAX_PAGES) return PK_ENOTSUP;
    const size_t smem = (size_t)batch * (sizeof(RowState) + PK_WIN_MAX_PAGES * sizeof(int));
    const int tiles_z = (a.batch * kv->d.chunk + kRelposRows - 1) / kRelposRows;
    const int grid = 1 + (a.batch > 0 ? a.nlayers * kv->d.num_heads * tiles_z : 0);
    return cuda_status(launch_pdl(pages_begin_relpos_kernel, dim3(grid), dim3(kRelposThreads), smem,
                                  s, kv->d, slots, lengths, batch, released, num_released, a, bds,
                                  bd, tiles_z),
                       "pages_begin_relpos_kernel");
}

int launch_pages_end(const pk_paged_kv *kv, const int32_t *slots, const int32_t *lengths,
                     int batch, cudaStream_t s) {
    if (batch == 0) return PK_OK;
    return cuda_status(launch_pdl(pages_end_kernel, dim3((batch + 255) / 256), dim3(256), 0, s,
                                  kv->d, slots, lengths, batch),
                       "pages_end_kernel");
}

}  // namespace pk
