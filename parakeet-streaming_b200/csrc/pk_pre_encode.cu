// Mel-frame cache of the streaming pre-encoder, batched over streams.
//
// Restates the cache handling of ModelRunner._run_pre_encode (parakeet/engine/
// model_runner.py:197-233): a chunk's features are prefixed with the frames
// cached from the stream's previous chunks (feats_in = cat(cache, feats)), and
// the cache becomes the last C frames of feats_in, or all of feats_in when it
// is shorter (a first chunk of fewer than C frames, :225-230).  Here the caches
// of all slots live in one pool [slots][feat_in][C], valid frames
// right-aligned, and one launch builds feats_in for a whole batch and advances
// every row's cache.
#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {
namespace {

constexpr int kWarps = 8;

// one warp per (row, feature bin): the old cache row is read into registers
// and exchanged by shuffles before the new one is written, so the in-place
// update needs no second launch
template <typename T>
__global__ void __launch_bounds__(kWarps * 32)
    pre_encode_window_kernel(T *cache, const T *feats, const int32_t *slots, int batch, int feat_in,
                             int frames, int csize, int prefix, T *out, int32_t *error,
                             int num_slots) {
    const int row = blockIdx.x * kWarps + threadIdx.x / 32, lane = threadIdx.x % 32;
    if (row >= batch * feat_in) return;
    const int b = row / feat_in, m = row - b * feat_in;
    const int s = slots[b];
    if (s < 0 || s >= num_slots) {
        if (lane == 0 && m == 0) raise(error, PK_DEV_BAD_SLOT);
        return;
    }
    T *crow = cache + ((int64_t)s * feat_in + m) * csize;
    const T *frow = feats + ((int64_t)b * feat_in + m) * frames;
    const int total = prefix + frames;
    T *orow = out + ((int64_t)b * feat_in + m) * total;
    const float old = lane < csize ? Elem<T>::to_f(crow[lane]) : 0.f;
    // window frame j < prefix is cache frame csize - prefix + j
    const float pre = __shfl_sync(0xffffffffu, old, min(csize - prefix + lane, 31));
    // new cache frame j is window frame total - csize + j: cache frame frames + j
    // when that is still inside the old prefix
    const float kept = __shfl_sync(0xffffffffu, old, min(frames + lane, 31));
    for (int j = lane; j < total; j += 32)
        orow[j] = j < prefix ? Elem<T>::from_f(pre) : frow[j - prefix];
    if (lane < csize) {
        const int p = total - csize + lane;
        crow[lane] = p < 0 ? Elem<T>::from_f(0.f)
                           : (p < prefix ? Elem<T>::from_f(kept) : frow[p - prefix]);
    }
}

}  // namespace

int launch_pre_encode_window(void *cache, const void *feats, const int32_t *slots, int batch,
                             int feat_in, int frames, int csize, int prefix, void *out,
                             int dtype, int32_t *error, int num_slots, cudaStream_t s) {
    const int64_t rows = (int64_t)batch * feat_in;
    if (rows == 0) return PK_OK;
    const dim3 grid((unsigned)((rows + kWarps - 1) / kWarps));
    if (dtype == PK_DTYPE_BF16)
        pre_encode_window_kernel<<<grid, kWarps * 32, 0, s>>>(
            static_cast<__nv_bfloat16 *>(cache), static_cast<const __nv_bfloat16 *>(feats), slots,
            batch, feat_in, frames, csize, prefix, static_cast<__nv_bfloat16 *>(out), error,
            num_slots);
    else
        pre_encode_window_kernel<<<grid, kWarps * 32, 0, s>>>(
            static_cast<float *>(cache), static_cast<const float *>(feats), slots, batch, feat_in,
            frames, csize, prefix, static_cast<float *>(out), error, num_slots);
    return cuda_status(cudaGetLastError(), "pre_encode_window_kernel");
}

}  // namespace pk
