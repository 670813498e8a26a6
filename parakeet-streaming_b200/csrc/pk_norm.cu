// Row LayerNorm for the encoder layers, optionally two in a row.
//
// nn.LayerNorm over the model width (parakeet/modules/encoder.py:50-81: the
// five LayerNorms of a ConformerLayer).  One warp per row: the row is loaded
// once into registers (16-byte vectors), the mean and then the variance of the
// deviations are reduced with warp shuffles (exact two-pass, fp32), and the
// normalised row is written with 16-byte stores.  With a second (gamma2, beta2)
// the kernel also normalises its own output, rounded to the element type as a
// separate LayerNorm would see it: a layer's norm_out followed by the next
// layer's norm_feed_forward1 is one launch that writes both rows.
#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {
namespace {

constexpr int kWarps = 8;

template <typename T> struct Vec;
template <> struct Vec<float> {
    static constexpr int kN = 4;
    static __device__ __forceinline__ void load(const float *p, float *v) {
        const float4 q = *reinterpret_cast<const float4 *>(p);
        v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
    }
    static __device__ __forceinline__ void store(float *p, const float *v) {
        *reinterpret_cast<float4 *>(p) = make_float4(v[0], v[1], v[2], v[3]);
    }
};
template <> struct Vec<__nv_bfloat16> {
    static constexpr int kN = 8;
    static __device__ __forceinline__ void load(const __nv_bfloat16 *p, float *v) {
        const uint4 q = *reinterpret_cast<const uint4 *>(p);
        const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&q);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(h[i]);
            v[2 * i] = f.x;
            v[2 * i + 1] = f.y;
        }
    }
    static __device__ __forceinline__ void store(__nv_bfloat16 *p, const float *v) {
        uint4 q;
        __nv_bfloat162 *h = reinterpret_cast<__nv_bfloat162 *>(&q);
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
        *reinterpret_cast<uint4 *>(p) = q;
    }
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// normalise the row held in v[] (lane's vectors j at columns (j*32 + lane)*kN)
template <typename T, int NV>
__device__ __forceinline__ void normalize(float (&v)[NV][Vec<T>::kN], int dim, const T *g,
                                          const T *b, float eps, int lane) {
    constexpr int kN = Vec<T>::kN;
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j)
#pragma unroll
        for (int e = 0; e < kN; ++e) s += v[j][e];
    const float mean = warp_sum(s) / dim;
    float q = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j)
#pragma unroll
        for (int e = 0; e < kN; ++e) {
            const float d = v[j][e] - mean;
            q += d * d;
        }
    const float rstd = rsqrtf(warp_sum(q) / dim + eps);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
        float gv[kN], bv[kN];
        const int c = (j * 32 + lane) * kN;
        Vec<T>::load(g + c, gv);
        Vec<T>::load(b + c, bv);
#pragma unroll
        for (int e = 0; e < kN; ++e) v[j][e] = (v[j][e] - mean) * rstd * gv[e] + bv[e];
    }
}

template <typename T, int NV>
__global__ void __launch_bounds__(kWarps * 32)
    layer_norm_kernel(const T *x, int64_t x_ld, int rows, int dim, const T *g1, const T *b1,
                      float eps1, T *y1, int64_t y1_ld, const T *g2, const T *b2, float eps2,
                      T *y2, int64_t y2_ld) {
    constexpr int kN = Vec<T>::kN;
    grid_dep_wait();
    grid_dep_launch();
    const int row = blockIdx.x * kWarps + threadIdx.x / 32, lane = threadIdx.x % 32;
    if (row >= rows) return;
    float v[NV][kN];
    const T *xr = x + (int64_t)row * x_ld;
#pragma unroll
    for (int j = 0; j < NV; ++j) Vec<T>::load(xr + (j * 32 + lane) * kN, v[j]);
    normalize<T, NV>(v, dim, g1, b1, eps1, lane);
    T *o1 = y1 + (int64_t)row * y1_ld;
#pragma unroll
    for (int j = 0; j < NV; ++j) Vec<T>::store(o1 + (j * 32 + lane) * kN, v[j]);
    if (!g2) return;
    // the second LayerNorm sees the first one's output as stored
#pragma unroll
    for (int j = 0; j < NV; ++j)
#pragma unroll
        for (int e = 0; e < kN; ++e) v[j][e] = Elem<T>::to_f(Elem<T>::from_f(v[j][e]));
    normalize<T, NV>(v, dim, g2, b2, eps2, lane);
    T *o2 = y2 + (int64_t)row * y2_ld;
#pragma unroll
    for (int j = 0; j < NV; ++j) Vec<T>::store(o2 + (j * 32 + lane) * kN, v[j]);
}

template <typename T>
int launch_ln_t(const LnArgs &a, cudaStream_t s) {
    constexpr int kN = Vec<T>::kN;
    const int nv = a.dim / (32 * kN);
    const dim3 grid((a.rows + kWarps - 1) / kWarps), block(kWarps * 32);
    const T *x = static_cast<const T *>(a.x);
    const T *g1 = static_cast<const T *>(a.g1), *b1 = static_cast<const T *>(a.b1);
    const T *g2 = static_cast<const T *>(a.g2), *b2 = static_cast<const T *>(a.b2);
    T *y1 = static_cast<T *>(a.y1), *y2 = static_cast<T *>(a.y2);
    cudaError_t e;
    switch (nv) {
#define PK_LN_CASE(N)                                                                         \
    case N:                                                                                   \
        e = launch_pdl(layer_norm_kernel<T, N>, grid, block, 0, s, x, a.x_ld, a.rows, a.dim, \
                       g1, b1, a.eps1, y1, a.y1_ld, g2, b2, a.eps2, y2, a.y2_ld);            \
        break;
        PK_LN_CASE(1)
        PK_LN_CASE(2)
        PK_LN_CASE(4)
        PK_LN_CASE(8)
#undef PK_LN_CASE
        default:
            set_error("layer norm width %d not handled", a.dim);
            return PK_ENOTSUP;
    }
    return cuda_status(e, "layer_norm_kernel");
}

}  // namespace

int launch_layer_norm(const LnArgs &a, cudaStream_t s) {
    if (a.rows == 0) return PK_OK;
    return a.dtype == PK_DTYPE_BF16 ? launch_ln_t<__nv_bfloat16>(a, s) : launch_ln_t<float>(a, s);
}

}  // namespace pk
