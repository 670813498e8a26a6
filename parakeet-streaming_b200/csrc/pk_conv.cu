// Depthwise causal conv with its time cache, fused with GLU, the pad mask,
// LayerNorm and SiLU.  One CTA per stream.  A layer's call moves about 1.8 MB
// for 80 streams, so the kernel is latency-bound: the loads that do not depend
// on the slot go out before the slot's cache, and the LayerNorm runs one warp
// per frame over the conv outputs kept in shared memory.
//
// Restates ConformerConvolution.forward (parakeet/modules/convolution.py:
// 150-162) from the GLU to the SiLU, with CausalConv1d.update_cache/forward
// (convolution.py:37-52): new_x = cat(cache, x), y = depthwise conv
// (kernel K, no bias), next cache = last K-1 columns of new_x.  The cache
// stays in the reference's [slot][layer][dim][K-1] layout (ModelCache.conv,
// parakeet/modules/cache.py:30-34) and is updated in place by slot id, so
// there is no gather/scatter (scheduler.py:162-168,196-201) around it.
#include <math.h>

#include <type_traits>

#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {
namespace {

constexpr int kTMax = 16;  // frames per chunk handled by one thread's registers

__device__ __forceinline__ float round_to(float v, const __nv_bfloat16 *) {
    return __bfloat162float(__float2bfloat16_rn(v));
}
__device__ __forceinline__ float round_to(float v, const float *) { return v; }

template <typename T>
__device__ __forceinline__ void load2(const T *p, float *f) {
    if constexpr (sizeof(T) == 2) {
        const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(p));
        f[0] = a.x, f[1] = a.y;
    } else {
        const float2 u = *reinterpret_cast<const float2 *>(p);
        f[0] = u.x, f[1] = u.y;
    }
}
template <typename T>
__device__ __forceinline__ void store2(T *p, const float *f) {
    if constexpr (sizeof(T) == 2)
        *reinterpret_cast<__nv_bfloat162 *>(p) = __floats2bfloat162_rn(f[0], f[1]);
    else
        *reinterpret_cast<float2 *>(p) = make_float2(f[0], f[1]);
}
// a channel's K-1 = 8 cached frames: 16 bytes in bf16
template <typename T, int KC>
__device__ __forceinline__ void load_cache(const T *p, float *h) {
    if constexpr (sizeof(T) == 2 && KC == 8) {
        const uint4 u = *reinterpret_cast<const uint4 *>(p);
        unpack16(u, h, static_cast<const __nv_bfloat16 *>(nullptr));
    } else {
#pragma unroll
        for (int k = 0; k < KC; ++k) h[k] = Elem<T>::to_f(p[k]);
    }
}
template <typename T, int KC>
__device__ __forceinline__ void store_cache(T *p, const float *h) {
    if constexpr (sizeof(T) == 2 && KC == 8) {
        uint4 u;
        uint32_t *w = reinterpret_cast<uint32_t *>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            __nv_bfloat162 v = __floats2bfloat162_rn(h[2 * i], h[2 * i + 1]);
            w[i] = *reinterpret_cast<uint32_t *>(&v);
        }
        *reinterpret_cast<uint4 *>(p) = u;
    } else {
#pragma unroll
        for (int k = 0; k < KC; ++k) p[k] = Elem<T>::from_f(h[k]);
    }
}
__device__ __forceinline__ float sigmoid(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }

constexpr int kCpt = 2;   // channels per thread in the conv phase

// One CTA per stream, D / 2 threads.  The stream's GLU input rows [chunk][2D]
// are staged in shared memory with 16-byte loads (the loads do not depend on
// the slot, the cache load follows the slot id); each thread then takes its two
// channels one at a time: GLU, pad mask, depthwise conv over cat(cache, x) with
// TM >= chunk frames of history in registers, the next cache; the conv outputs
// go to shared memory in the element type (the reference's conv output is a
// tensor of the model dtype), and one warp per frame takes the exact two-pass
// LayerNorm statistics and writes the frame's SiLU output with coalesced stores.
// Keeping the inputs out of registers holds a thread to a few dozen registers,
// so two CTAs of 512 threads share an SM at the large model's width.
template <typename T, int K, int TM>
__global__ void __launch_bounds__(512) conv_step_kernel(const ConvArgs a) {
    constexpr int KC = K - 1;
    extern __shared__ __align__(16) char conv_smem[];
    const int b = blockIdx.x;
    const int D = a.dim, chunk = a.chunk;
    T *xs = reinterpret_cast<T *>(conv_smem);            // [chunk][2D] GLU inputs
    T *ys = xs + (size_t)chunk * 2 * D;                  // [chunk][D] conv outputs
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, nw = blockDim.x / 32;

    grid_dep_wait();     // x and the cache may come from the previous kernel
    grid_dep_launch();   // the next kernel may be scheduled (it waits for us)
    const int s = a.slots[b];
    const int n = a.lengths[b];
    {
        const T *xb = static_cast<const T *>(a.x) + (int64_t)b * a.x_bs;
        constexpr int kVec = 16 / sizeof(T);
        const int per_row = 2 * D / kVec;
        if (a.x_vec) {
            for (int i = threadIdx.x; i < chunk * per_row; i += blockDim.x) {
                const int t = i / per_row, j = i - t * per_row;
                *reinterpret_cast<uint4 *>(xs + (size_t)t * 2 * D + j * kVec) =
                    *reinterpret_cast<const uint4 *>(xb + (int64_t)t * a.x_rs + j * kVec);
            }
        } else {
            for (int i = threadIdx.x; i < chunk * 2 * D; i += blockDim.x) {
                const int t = i / (2 * D), j = i - t * 2 * D;
                xs[i] = xb[(int64_t)t * a.x_rs + j];
            }
        }
    }
    const bool slot_ok = s >= 0 && s < a.num_slots;   // block-uniform
    if (!slot_ok) {
        if (threadIdx.x == 0) raise(a.error, PK_DEV_BAD_SLOT);
        return;
    }
    __syncthreads();

    const int c0 = threadIdx.x * kCpt;
    T *yb = static_cast<T *>(a.y) + (int64_t)b * chunk * D;
    if (c0 < D) {
        T *cache = static_cast<T *>(a.state) + (((int64_t)s * a.num_layers + a.layer) * D + c0) * KC;
        const T *wt = static_cast<const T *>(a.w) + (int64_t)c0 * K;
#pragma unroll 1
        for (int ch = 0; ch < kCpt; ++ch) {
            const int c = c0 + ch;
            float wk[K], hist[KC + TM];
#pragma unroll
            for (int k = 0; k < K; ++k) wk[k] = Elem<T>::to_f(wt[ch * K + k]);
            load_cache<T, KC>(cache + ch * KC, hist);
#pragma unroll
            for (int t = 0; t < TM; ++t) {
                if (t >= chunk) break;
                // F.glu then masked_fill(pad_mask, 0) (convolution.py:153-155)
                const float va = Elem<T>::to_f(xs[(size_t)t * 2 * D + c]);
                const float vg = Elem<T>::to_f(xs[(size_t)t * 2 * D + D + c]);
                const float v = round_to(va * sigmoid(vg), static_cast<const T *>(nullptr));
                hist[KC + t] = t < n ? v : 0.f;
            }
#pragma unroll
            for (int t = 0; t < TM; ++t) {
                if (t >= chunk) break;
                float acc = 0.f;
#pragma unroll
                for (int k = 0; k < K; ++k) acc = fmaf(wk[k], hist[t + k], acc);
                if (a.ln_w)
                    ys[(size_t)t * D + c] = Elem<T>::from_f(acc);
                else
                    yb[(int64_t)t * D + c] = Elem<T>::from_f(acc);
            }
            // next cache: the last K-1 entries of cat(cache, x)
            float nc[KC];
#pragma unroll
            for (int k = 0; k < KC; ++k) {
                float v = 0.f;
#pragma unroll
                for (int t = 0; t <= TM; ++t)
                    if (t == chunk) v = hist[t + k];
                nc[k] = v;
            }
            store_cache<T, KC>(cache + ch * KC, nc);
        }
    }
    if (!a.ln_w) return;
    __syncthreads();

    // LayerNorm over channels (the module's "batch_norm", convolution.py:138,157), then SiLU
    const T *lw = static_cast<const T *>(a.ln_w), *lb = static_cast<const T *>(a.ln_b);
    for (int t = warp; t < chunk; t += nw) {
        const T *row = ys + (size_t)t * D;
        float sum = 0.f;
        for (int c = 2 * lane; c < D; c += 64) {
            float v[2];
            load2<T>(row + c, v);
            sum += v[0] + v[1];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        const float mean = sum / D;
        float sq = 0.f;
        for (int c = 2 * lane; c < D; c += 64) {
            float v[2];
            load2<T>(row + c, v);
            sq += (v[0] - mean) * (v[0] - mean) + (v[1] - mean) * (v[1] - mean);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
        const float inv = rsqrtf(sq / D + a.eps);
        for (int c = 2 * lane; c < D; c += 64) {
            float v[2], gw[2], gb[2];
            load2<T>(row + c, v);
            load2<T>(lw + c, gw);
            load2<T>(lb + c, gb);
            const float z0 = (v[0] - mean) * inv * gw[0] + gb[0];
            const float z1 = (v[1] - mean) * inv * gw[1] + gb[1];
            const float o[2] = {z0 * sigmoid(z0), z1 * sigmoid(z1)};
            store2<T>(yb + (int64_t)t * D + c, o);
        }
    }
}

// Short chunks (the small model's 2 frames): everything in registers, no shared
// memory but the LayerNorm's cross-warp partial sums.  Thread i owns channels
// 2i and 2i + 1 of one stream (NT = D / 2 threads per CTA); the chunk length
// and the width are compile-time constants, so every loop below is unrolled
// and the next cache is plain register moves.  The two channels' weights (18
// contiguous values, loaded as 9 words) and LayerNorm parameters are read
// before the wait on the previous kernel (no kernel of the stream writes
// them); then the slot and the GLU inputs; then both 8-frame caches at once
// (16 bytes each in bf16).  The frames' LayerNorm statistics are block
// reductions (exact two passes: the mean, then the sum of squared
// deviations): each warp's partial sums meet in shared memory and are summed
// by the lanes of every warp with shuffles, so each thread normalises its own
// channels.
template <typename T, int CH, int NT>
__global__ void __launch_bounds__(NT) conv_step_reg_kernel(const ConvArgs a) {
    constexpr int K = 9, KC = K - 1, D = 2 * NT, NW = NT / 32;
    static_assert(NW <= 32, "one lane per warp in the cross-warp sums");
    __shared__ float red[2][NW][CH];   // per-warp partial sums
    const int b = blockIdx.x;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int c0 = 2 * threadIdx.x;
    const bool ln = a.ln_w != nullptr;
    float wk[2][K], gw[2] = {0.f, 0.f}, gb[2] = {0.f, 0.f};
    {
        const T *wt = static_cast<const T *>(a.w) + c0 * K;   // 2K values, 4-byte aligned
        if constexpr (sizeof(T) == 2) {
            const uint32_t *w32 = reinterpret_cast<const uint32_t *>(wt);
#pragma unroll
            for (int i = 0; i < K; ++i) {
                const uint32_t u = __ldg(w32 + i);
                const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&u));
                wk[(2 * i) / K][(2 * i) % K] = f.x;
                wk[(2 * i + 1) / K][(2 * i + 1) % K] = f.y;
            }
        } else {
            const float2 *w2 = reinterpret_cast<const float2 *>(wt);
#pragma unroll
            for (int i = 0; i < K; ++i) {
                const float2 f = __ldg(w2 + i);
                wk[(2 * i) / K][(2 * i) % K] = f.x;
                wk[(2 * i + 1) / K][(2 * i + 1) % K] = f.y;
            }
        }
        if (ln) {
            load2<T>(static_cast<const T *>(a.ln_w) + c0, gw);
            load2<T>(static_cast<const T *>(a.ln_b) + c0, gb);
        }
    }
    grid_dep_wait();     // x and the cache may come from the previous kernel
    grid_dep_launch();   // the next kernel may be scheduled (it waits for us)
    const int s = a.slots[b];
    const int n = a.lengths[b];
    float xa[CH][2], xg[CH][2];
    {
        const T *xb = static_cast<const T *>(a.x) + (int64_t)b * a.x_bs + c0;
#pragma unroll
        for (int t = 0; t < CH; ++t) {
            load2<T>(xb + (int64_t)t * a.x_rs, xa[t]);
            load2<T>(xb + (int64_t)t * a.x_rs + D, xg[t]);
        }
    }
    if (s < 0 || s >= a.num_slots) {   // block-uniform
        if (threadIdx.x == 0) raise(a.error, PK_DEV_BAD_SLOT);
        return;
    }
    T *cache = static_cast<T *>(a.state) + (((int64_t)s * a.num_layers + a.layer) * D + c0) * KC;
    float hist[2][KC + CH];
    load_cache<T, KC>(cache, hist[0]);
    load_cache<T, KC>(cache + KC, hist[1]);
    float y[CH][2];
#pragma unroll
    for (int ch = 0; ch < 2; ++ch) {
#pragma unroll
        for (int t = 0; t < CH; ++t) {
            // F.glu then masked_fill(pad_mask, 0) (convolution.py:153-155)
            const float v = round_to(xa[t][ch] * sigmoid(xg[t][ch]), static_cast<const T *>(nullptr));
            hist[ch][KC + t] = t < n ? v : 0.f;
        }
#pragma unroll
        for (int t = 0; t < CH; ++t) {
            float acc = 0.f;
#pragma unroll
            for (int k = 0; k < K; ++k) acc = fmaf(wk[ch][k], hist[ch][t + k], acc);
            y[t][ch] = round_to(acc, static_cast<const T *>(nullptr));   // the conv output's dtype
        }
    }
    // next cache: the last K-1 entries of cat(cache, x)
    store_cache<T, KC>(cache, hist[0] + CH);
    store_cache<T, KC>(cache + KC, hist[1] + CH);
    T *yb = static_cast<T *>(a.y) + (int64_t)b * CH * D + c0;
    if (!ln) {
#pragma unroll
        for (int t = 0; t < CH; ++t) store2<T>(yb + t * D, y[t]);
        return;
    }
    // LayerNorm over channels (the module's "batch_norm", convolution.py:138,157), then SiLU
    auto block_sum = [&](float (&v)[CH], int which) {
#pragma unroll
        for (int t = 0; t < CH; ++t)
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v[t] += __shfl_xor_sync(0xffffffffu, v[t], o);
        if (lane == 0)
#pragma unroll
            for (int t = 0; t < CH; ++t) red[which][warp][t] = v[t];
        __syncthreads();
#pragma unroll
        for (int t = 0; t < CH; ++t) {
            float u = lane < NW ? red[which][lane][t] : 0.f;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) u += __shfl_xor_sync(0xffffffffu, u, o);
            v[t] = u;
        }
    };
    float part[CH], mean[CH];
#pragma unroll
    for (int t = 0; t < CH; ++t) part[t] = y[t][0] + y[t][1];
    block_sum(part, 0);
#pragma unroll
    for (int t = 0; t < CH; ++t) {
        mean[t] = part[t] / D;
        const float d0 = y[t][0] - mean[t], d1 = y[t][1] - mean[t];
        part[t] = d0 * d0 + d1 * d1;
    }
    block_sum(part, 1);
#pragma unroll
    for (int t = 0; t < CH; ++t) {
        const float inv = rsqrtf(part[t] / D + a.eps);
        const float z0 = (y[t][0] - mean[t]) * inv * gw[0] + gb[0];
        const float z1 = (y[t][1] - mean[t]) * inv * gw[1] + gb[1];
        const float o[2] = {z0 * sigmoid(z0), z1 * sigmoid(z1)};
        store2<T>(yb + t * D, o);
    }
}

}  // namespace

int launch_conv(const ConvArgs &a, cudaStream_t s) {
    if (a.batch == 0) return PK_OK;
    if (a.kernel != 9 || a.chunk > kTMax || a.dim % kCpt != 0 || a.dim > 512 * kCpt)
        return PK_ENOTSUP;
    const int threads = ((a.dim / kCpt + 31) / 32) * 32;
    const int tm = a.chunk <= 2 ? 2 : a.chunk <= 4 ? 4 : a.chunk <= 8 ? 8 : 16;
    // chunks of 1 to 4 frames at widths 512 and 1024: the register form (no
    // staging, one load round after the slot)
    if (a.chunk <= 4 && (a.dim == 512 || a.dim == 1024)) {
        auto pick = [&](auto tag) {
            using T = decltype(tag);
            auto by_chunk = [&](auto nt) {
                constexpr int NT = decltype(nt)::value;
                void (*k)(const ConvArgs) = a.chunk == 1   ? conv_step_reg_kernel<T, 1, NT>
                                          : a.chunk == 2 ? conv_step_reg_kernel<T, 2, NT>
                                          : a.chunk == 3 ? conv_step_reg_kernel<T, 3, NT>
                                                         : conv_step_reg_kernel<T, 4, NT>;
                return launch_pdl(k, dim3(a.batch), dim3(NT), 0, s, a);
            };
            return a.dim == 512 ? by_chunk(std::integral_constant<int, 256>())
                                : by_chunk(std::integral_constant<int, 512>());
        };
        const cudaError_t e = a.dtype == PK_DTYPE_BF16 ? pick(__nv_bfloat16()) : pick(float());
        return cuda_status(e, "conv_step_reg_kernel");
    }
    auto pick = [&](auto tag) {
        using T = decltype(tag);
        auto kernel = tm == 2 ? conv_step_kernel<T, 9, 2> : tm == 4 ? conv_step_kernel<T, 9, 4>
                    : tm == 8 ? conv_step_kernel<T, 9, 8> : conv_step_kernel<T, 9, 16>;
        // GLU inputs [chunk][2D] and conv outputs [chunk][D] in the element type
        const size_t smem = (size_t)a.chunk * 3 * a.dim * sizeof(T);
        if (smem > 48 * 1024) {   // at most 96 KB in bf16: chunk <= 16, dim <= 1024
            const cudaError_t e = cudaFuncSetAttribute(
                kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return e;
        }
        return launch_pdl(kernel, dim3(a.batch), dim3(threads), smem, s, a);
    };
    const cudaError_t e = a.dtype == PK_DTYPE_BF16 ? pick(__nv_bfloat16()) : pick(float());
    return cuda_status(e, "conv_step_kernel");
}

}  // namespace pk
