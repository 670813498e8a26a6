// Depthwise causal conv with its time cache, fused with GLU, the pad mask,
// LayerNorm and SiLU.  One CTA per stream, four channels per thread.
//
// Restates ConformerConvolution.forward (parakeet/modules/convolution.py:
// 150-162) from the GLU to the SiLU, with CausalConv1d.update_cache/forward
// (convolution.py:37-52): new_x = cat(cache, x), y = depthwise conv
// (kernel K, no bias), next cache = last K-1 columns of new_x.  The cache
// stays in the reference's [slot][layer][dim][K-1] layout (ModelCache.conv,
// parakeet/modules/cache.py:30-34) and is updated in place by slot id, so
// there is no gather/scatter (scheduler.py:162-168,196-201) around it.
#include <math.h>

#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {
namespace {

constexpr int kTMax = 16;  // frames per chunk handled by one thread's registers

template <typename T>
__device__ __forceinline__ void load4(const T *p, float *f) {
    if constexpr (sizeof(T) == 2) {
        const uint2 u = *reinterpret_cast<const uint2 *>(p);
        const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&u.x));
        const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&u.y));
        f[0] = a.x, f[1] = a.y, f[2] = b.x, f[3] = b.y;
    } else {
        const float4 u = *reinterpret_cast<const float4 *>(p);
        f[0] = u.x, f[1] = u.y, f[2] = u.z, f[3] = u.w;
    }
}

template <typename T>
__device__ __forceinline__ void store4(T *p, const float *f) {
    if constexpr (sizeof(T) == 2) {
        __nv_bfloat162 a = __floats2bfloat162_rn(f[0], f[1]);
        __nv_bfloat162 b = __floats2bfloat162_rn(f[2], f[3]);
        uint2 u;
        u.x = *reinterpret_cast<uint32_t *>(&a);
        u.y = *reinterpret_cast<uint32_t *>(&b);
        *reinterpret_cast<uint2 *>(p) = u;
    } else {
        *reinterpret_cast<float4 *>(p) = make_float4(f[0], f[1], f[2], f[3]);
    }
}

__device__ __forceinline__ float round_to(float v, const __nv_bfloat16 *) {
    return __bfloat162float(__float2bfloat16_rn(v));
}
__device__ __forceinline__ float round_to(float v, const float *) { return v; }

// Sum of v over the CTA for every frame t < chunk; all threads get the sums.
__device__ __forceinline__ void block_sum(float (&v)[kTMax], int chunk, float (*red)[8]) {
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, nw = blockDim.x / 32;
#pragma unroll
    for (int t = 0; t < kTMax; ++t) {
        if (t >= chunk) break;
        float x = v[t];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
        if (lane == 0) red[t][warp] = x;
    }
    __syncthreads();
#pragma unroll
    for (int t = 0; t < kTMax; ++t) {
        if (t >= chunk) break;
        float x = 0.f;
        for (int k = 0; k < nw; ++k) x += red[t][k];
        v[t] = x;
    }
    __syncthreads();
}

template <typename T, int K>
__global__ void __launch_bounds__(256) conv_step_kernel(const ConvArgs a) {
    constexpr int KC = K - 1;
    __shared__ float red[kTMax][8];
    const int b = blockIdx.x;
    const int s = a.slots[b];
    if (s < 0 || s >= a.num_slots) {
        if (threadIdx.x == 0) raise(a.error, PK_DEV_BAD_SLOT);
        return;
    }
    const int D = a.dim, chunk = a.chunk;
    const int n = a.lengths[b];
    const int c0 = threadIdx.x * 4;
    const bool active = c0 < D;

    float hist[4][KC + kTMax];
    float y[4][kTMax];
    T *cache = static_cast<T *>(a.state) + (((int64_t)s * a.num_layers + a.layer) * D + c0) * KC;
    if (active) {
#pragma unroll
        for (int ch = 0; ch < 4; ++ch)
#pragma unroll
            for (int k = 0; k < KC; ++k) hist[ch][k] = Elem<T>::to_f(cache[ch * KC + k]);
        const T *xb = static_cast<const T *>(a.x) + (int64_t)b * a.x_bs;
#pragma unroll
        for (int t = 0; t < kTMax; ++t) {
            if (t >= chunk) break;
            float va[4], vg[4];
            load4<T>(xb + (int64_t)t * a.x_rs + c0, va);
            load4<T>(xb + (int64_t)t * a.x_rs + D + c0, vg);
#pragma unroll
            for (int ch = 0; ch < 4; ++ch) {
                // F.glu then masked_fill(pad_mask, 0) (convolution.py:153-155)
                const float v = round_to(va[ch] / (1.f + expf(-vg[ch])), static_cast<const T *>(nullptr));
                hist[ch][KC + t] = t < n ? v : 0.f;
            }
        }
        const T *wt = static_cast<const T *>(a.w) + (int64_t)c0 * K;
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {
            float wk[K];
#pragma unroll
            for (int k = 0; k < K; ++k) wk[k] = Elem<T>::to_f(wt[ch * K + k]);
#pragma unroll
            for (int t = 0; t < kTMax; ++t) {
                if (t >= chunk) break;
                float acc = 0.f;
#pragma unroll
                for (int k = 0; k < K; ++k) acc = fmaf(wk[k], hist[ch][t + k], acc);
                y[ch][t] = acc;
            }
            // next cache: the last K-1 entries of cat(cache, x)
#pragma unroll
            for (int k = 0; k < KC; ++k) {
                float v = 0.f;
#pragma unroll
                for (int t = 0; t <= kTMax; ++t)
                    if (t == chunk) v = hist[ch][t + k];
                cache[ch * KC + k] = Elem<T>::from_f(v);
            }
        }
    } else {
#pragma unroll
        for (int ch = 0; ch < 4; ++ch)
#pragma unroll
            for (int t = 0; t < kTMax; ++t) y[ch][t] = 0.f;
    }

    T *yb = static_cast<T *>(a.y) + (int64_t)b * chunk * D;
    if (a.ln_w) {
        // LayerNorm over channels (the module's "batch_norm", convolution.py:138,157), then SiLU
        float m[kTMax], v[kTMax];
#pragma unroll
        for (int t = 0; t < kTMax; ++t) m[t] = active ? y[0][t] + y[1][t] + y[2][t] + y[3][t] : 0.f;
        block_sum(m, chunk, red);
#pragma unroll
        for (int t = 0; t < kTMax; ++t) {
            m[t] *= 1.f / D;
            float q = 0.f;
            if (active)
#pragma unroll
                for (int ch = 0; ch < 4; ++ch) q += (y[ch][t] - m[t]) * (y[ch][t] - m[t]);
            v[t] = q;
        }
        block_sum(v, chunk, red);
        if (active) {
            float g[4], be[4];
            load4<T>(static_cast<const T *>(a.ln_w) + c0, g);
            load4<T>(static_cast<const T *>(a.ln_b) + c0, be);
#pragma unroll
            for (int t = 0; t < kTMax; ++t) {
                if (t >= chunk) break;
                const float inv = rsqrtf(v[t] * (1.f / D) + a.eps);
                float o[4];
#pragma unroll
                for (int ch = 0; ch < 4; ++ch) {
                    const float z = (y[ch][t] - m[t]) * inv * g[ch] + be[ch];
                    o[ch] = z / (1.f + expf(-z));
                }
                store4<T>(yb + (int64_t)t * D + c0, o);
            }
        }
    } else if (active) {
#pragma unroll
        for (int t = 0; t < kTMax; ++t) {
            if (t >= chunk) break;
            float o[4] = {y[0][t], y[1][t], y[2][t], y[3][t]};
            store4<T>(yb + (int64_t)t * D + c0, o);
        }
    }
}

}  // namespace

int launch_conv(const ConvArgs &a, cudaStream_t s) {
    if (a.batch == 0) return PK_OK;
    if (a.kernel != 9 || a.chunk > kTMax || a.dim % 4 != 0 || a.dim > 1024) return PK_ENOTSUP;
    const int threads = ((a.dim / 4 + 31) / 32) * 32;
    if (a.dtype == PK_DTYPE_BF16)
        conv_step_kernel<__nv_bfloat16, 9><<<a.batch, threads, 0, s>>>(a);
    else
        conv_step_kernel<float, 9><<<a.batch, threads, 0, s>>>(a);
    return cuda_status(cudaGetLastError(), "conv_step_kernel");
}

}  // namespace pk
