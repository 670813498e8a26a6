// Per-step window descriptors: one warp per batch row.
//
// Everything the attention kernels need to find a stream's window that does
// not depend on the layer or the head is resolved here once per step instead
// of once per (layer, head): the slot's counters, the pages that hold rows
// [w - left, w + chunk), the row each page's TMA box starts at, and the
// streaming mask of ConformerEncoder._create_streaming_masks
// (parakeet/modules/encoder.py:167-227) as bit rows, bit (j % 32) of word
// [i][j / 32] set when key j is allowed for query i.
#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {
namespace {

__global__ void __launch_bounds__(32)
    window_desc_kernel(pk_paged_kv_desc d, const int32_t *slots, const int32_t *lengths) {
    const int b = blockIdx.x, lane = threadIdx.x;
    const int chunk = d.chunk, W = d.left + d.chunk, ps = d.page_size;
    int32_t *out = d.window + (int64_t)b * PK_WIN_STRIDE;
    int ok = 1, w = 0, proc = 0, clen = 0, len = chunk, slot = slots[b];
    if (slot < 0 || slot >= d.num_slots) {
        ok = 0;
        if (lane == 0) raise(d.error, PK_DEV_BAD_SLOT);
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
    // mask rows; rows >= chunk and words past the window are zero
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
        for (int i = 0; i < 16; ++i) {
            const int dc = (key_start + clen + i) / chunk - kc;
            const unsigned bits =
                __ballot_sync(0xffffffffu, key_ok && i < chunk && i < len && dc >= 0 &&
                                               dc <= left_chunks);
            if (lane == 0) out[PK_WIN_MASK + i * 4 + kb] = (int32_t)bits;
        }
    }
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

}  // namespace

int launch_window_desc(const pk_paged_kv *kv, const int32_t *slots, const int32_t *lengths,
                       int batch, cudaStream_t s) {
    if (batch == 0) return PK_OK;
    window_desc_kernel<<<batch, 32, 0, s>>>(kv->d, slots, lengths);
    return cuda_status(cudaGetLastError(), "window_desc_kernel");
}

}  // namespace pk
