// Greedy RNNT decode step kernels: the per-symbol bookkeeping of a batched
// greedy decode kept on the device, so a chunk's whole decode loop runs without
// a host round trip (and can be captured in one CUDA graph).
//
// rnnt_pick   restates model_runner.py:423-430 (parakeet/engine): argmax over
//             the joint's classes, the blank mask, the emitted token lists;
//             plus the per-frame row bookkeeping the reference does on the host
//             (rows stop at their first blank of a frame, at most max_symbols
//             per frame, frames beyond a stream's chunk length are skipped,
//             model_runner.py:370-376).
// lstm_cell   restates one LSTM step of Predictor.forward (parakeet/modules/
//             decoder.py:44-50, PyTorch gate order i, f, g, o) fused with the
//             torch.where that keeps the state of rows that emitted blank
//             (model_runner.py:433-445).
#include <math.h>

#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {
namespace {

constexpr int kPickWarps = 8;

// one warp per batch row
template <typename T>
__global__ void __launch_bounds__(kPickWarps * 32)
    rnnt_pick_kernel(const T *logits, int64_t ld, int batch, int nclass, int blank,
                     const int32_t *lengths, int frame, int symbol, int max_symbols, int frames,
                     int32_t *done, int32_t *emit, int64_t *ids, int32_t *tokens, int32_t *counts) {
    const int b = blockIdx.x * kPickWarps + threadIdx.x / 32, lane = threadIdx.x % 32;
    if (b >= batch) return;
    const T *row = logits + (int64_t)b * ld;
    float best = -INFINITY;
    int arg = 0x7fffffff;
    for (int k = lane; k < nclass; k += 32) {
        const float v = Elem<T>::to_f(row[k]);
        if (v > best || (v == best && k < arg)) {   // first maximum, like torch.argmax
            best = v;
            arg = k;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oa = __shfl_xor_sync(0xffffffffu, arg, o);
        if (ov > best || (ov == best && oa < arg)) {
            best = ov;
            arg = oa;
        }
    }
    if (lane == 0) {
        const int finished = symbol == 0 ? 0 : done[b];
        const bool live = !finished && frame < lengths[b];
        const bool e = live && arg != blank;
        emit[b] = e;
        ids[b] = e ? arg : blank;
        tokens[((int64_t)b * frames + frame) * max_symbols + symbol] = e ? arg : -1;
        int32_t *cnt = counts + (int64_t)b * frames + frame;
        *cnt = (symbol == 0 ? 0 : *cnt) + (e ? 1 : 0);
        done[b] = !e;
    }
}

__device__ __forceinline__ float sigmoidf(float x) { return 1.f / (1.f + expf(-x)); }

// one thread per (row, hidden unit); rows that did not emit keep their state.
// xtab (optional): a per-token addend row of the gates, xtab[ids[b]] (the
// embedding already multiplied by W_ih, plus both biases)
template <typename T>
__global__ void __launch_bounds__(256)
    lstm_cell_kernel(const T *gates, int64_t gld, const T *xtab, int64_t xld, const int64_t *ids,
                     T *h, T *c, int64_t sld, const int32_t *emit, int batch, int hidden) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)batch * hidden) return;
    const int b = (int)(idx / hidden), j = (int)(idx - (int64_t)b * hidden);
    if (!emit[b]) return;
    const T *g = gates + (int64_t)b * gld;
    float gi = Elem<T>::to_f(g[j]), gf = Elem<T>::to_f(g[hidden + j]);
    float gg = Elem<T>::to_f(g[2 * hidden + j]), go = Elem<T>::to_f(g[3 * hidden + j]);
    if (xtab) {
        const T *x = xtab + ids[b] * xld;
        gi += Elem<T>::to_f(x[j]);
        gf += Elem<T>::to_f(x[hidden + j]);
        gg += Elem<T>::to_f(x[2 * hidden + j]);
        go += Elem<T>::to_f(x[3 * hidden + j]);
    }
    T *cp = c + (int64_t)b * sld + j;
    const float cn = sigmoidf(gf) * Elem<T>::to_f(*cp) + sigmoidf(gi) * tanhf(gg);
    const T cq = Elem<T>::from_f(cn);
    *cp = cq;
    h[(int64_t)b * sld + j] = Elem<T>::from_f(sigmoidf(go) * tanhf(cn));
}

}  // namespace

int launch_rnnt_pick(const void *logits, int64_t ld, int dtype, int batch, int nclass, int blank,
                     const int32_t *lengths, int frame, int symbol, int max_symbols, int frames,
                     int32_t *done, int32_t *emit, int64_t *ids, int32_t *tokens, int32_t *counts,
                     cudaStream_t s) {
    if (batch == 0) return PK_OK;
    const dim3 grid((batch + kPickWarps - 1) / kPickWarps);
    if (dtype == PK_DTYPE_BF16)
        rnnt_pick_kernel<<<grid, kPickWarps * 32, 0, s>>>(
            static_cast<const __nv_bfloat16 *>(logits), ld, batch, nclass, blank, lengths, frame,
            symbol, max_symbols, frames, done, emit, ids, tokens, counts);
    else
        rnnt_pick_kernel<<<grid, kPickWarps * 32, 0, s>>>(
            static_cast<const float *>(logits), ld, batch, nclass, blank, lengths, frame, symbol,
            max_symbols, frames, done, emit, ids, tokens, counts);
    return cuda_status(cudaGetLastError(), "rnnt_pick_kernel");
}

int launch_lstm_cell(const void *gates, int64_t gld, const void *xtab, int64_t xld,
                     const int64_t *ids, void *h, void *c, int64_t sld, const int32_t *emit,
                     int batch, int hidden, int dtype, cudaStream_t s) {
    const int64_t n = (int64_t)batch * hidden;
    if (n == 0) return PK_OK;
    const dim3 grid((unsigned)((n + 255) / 256));
    if (dtype == PK_DTYPE_BF16)
        lstm_cell_kernel<<<grid, 256, 0, s>>>(
            static_cast<const __nv_bfloat16 *>(gates), gld,
            static_cast<const __nv_bfloat16 *>(xtab), xld, ids, static_cast<__nv_bfloat16 *>(h),
            static_cast<__nv_bfloat16 *>(c), sld, emit, batch, hidden);
    else
        lstm_cell_kernel<<<grid, 256, 0, s>>>(static_cast<const float *>(gates), gld,
                                              static_cast<const float *>(xtab), xld, ids,
                                              static_cast<float *>(h), static_cast<float *>(c),
                                              sld, emit, batch, hidden);
    return cuda_status(cudaGetLastError(), "lstm_cell_kernel");
}

}  // namespace pk
