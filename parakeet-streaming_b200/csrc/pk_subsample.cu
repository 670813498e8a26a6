// The strided convolutions of the streaming pre-encoder, fused per channel.
//
// ConvSubsampling (parakeet/modules/subsample.py:61-179, dw_striding, 8x):
//   conv1  Conv2d(1 -> C, 3x3, stride 2) + bias -> ReLU
//   conv2  depthwise Conv2d(C, 3x3, stride 2, groups C) + bias -> pointwise 1x1 + bias -> ReLU
//   conv3  depthwise Conv2d(C, 3x3, stride 2, groups C) + bias -> pointwise 1x1 + bias -> ReLU
//   out    Linear(C * F3 -> hidden) over (channel, frequency) per output frame
// Every conv is causal (CausalConv2D, convolution.py:55-104): 2 zero rows and
// columns before the input, 1 after, so output (o, p) reads input rows
// 2o-2 .. 2o and columns 2p-2 .. 2p.
//
// conv1 and the depthwise conv2 touch one channel at a time, so
// `subsample_stage12_kernel` computes both for a block of channels and output
// rows without writing conv1's activation (C x T/2 x 65 per stream, the largest
// tensor of the pre-encoder) anywhere but shared memory; its output is
// channels-last [B][rows][F2][C], the layout the pointwise conv reads as a GEMM
// operand.  `subsample_dw_kernel` is the depthwise conv3 over channels-last
// rows.  Rows before `first` output rows are never computed: the streaming
// pre-encode drops its first outputs, and an output depends only on its own
// receptive field.
#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {
namespace {

constexpr int kCB = 16;        // channels per CTA (stage 1 + 2)
constexpr int kThreads = 256;

__host__ __device__ constexpr int conv_out(int n) { return n / 2 + 1; }   // (n + 3 - 3) / 2 + 1

template <typename T>
__global__ void __launch_bounds__(kThreads)
    subsample_stage12_kernel(const T *x, int64_t xb, int64_t xf, int64_t xt, int frames, int feat,
                             const T *w1, const T *b1, const T *w2, const T *b2, int C,
                             int first2, int rows_per_cta, T *y) {
    extern __shared__ float s12_smem[];
    const int t1n = conv_out(frames), f1n = conv_out(feat);
    const int t2n = conv_out(t1n), f2n = conv_out(f1n);
    const int b = blockIdx.z, c0 = blockIdx.x * kCB;
    const int o0 = first2 + blockIdx.y * rows_per_cta;
    const int o1 = min(t2n, o0 + rows_per_cta);
    if (o0 >= o1) return;
    // stage-1 rows r_lo .. r_lo + nr1 - 1, input rows t_lo .. t_lo + nin - 1
    const int r_lo = 2 * o0 - 2, nr1 = 2 * (o1 - o0) + 1;
    const int t_lo = 2 * r_lo - 2, nin = 2 * nr1 + 1;
    const int fpad = feat + 3;                        // input columns -2 .. feat
    float *xs = s12_smem;                             // [nin][fpad]
    float *s1 = xs + nin * fpad;                      // [kCB][nr1][f1n + 3]
    const int s1w = f1n + 3;                          // stage-1 columns -2 .. f1n
    grid_dep_wait();
    const T *xrow = x + (int64_t)b * xb;
    for (int i = threadIdx.x; i < nin * fpad; i += kThreads) {
        const int r = i / fpad, f = i - r * fpad - 2;
        const int t = t_lo + r;
        float v = 0.f;
        if (t >= 0 && t < frames && f >= 0 && f < feat)
            v = Elem<T>::to_f(xrow[(int64_t)f * xf + (int64_t)t * xt]);
        xs[i] = v;
    }
    __syncthreads();
    // conv1 + bias + ReLU, zero outside the stage-1 grid (the next conv's padding)
    for (int i = threadIdx.x; i < kCB * nr1 * s1w; i += kThreads) {
        const int c = i / (nr1 * s1w), rem = i - c * nr1 * s1w;
        const int r = rem / s1w, q = rem - r * s1w - 2;
        const int ra = r_lo + r;
        float v = 0.f;
        if (ra >= 0 && ra < t1n && q >= 0 && q < f1n) {
            const T *w = w1 + (c0 + c) * 9;
            const float *xa = xs + (2 * ra - 2 - t_lo) * fpad + (2 * q - 2 + 2);
            float acc = Elem<T>::to_f(b1[c0 + c]);
#pragma unroll
            for (int di = 0; di < 3; ++di)
#pragma unroll
                for (int dj = 0; dj < 3; ++dj)
                    acc = fmaf(Elem<T>::to_f(w[di * 3 + dj]), xa[di * fpad + dj], acc);
            v = fmaxf(acc, 0.f);
        }
        s1[i] = v;
    }
    __syncthreads();
    grid_dep_launch();
    // depthwise conv2 + bias, channels-last output rows o0 .. o1-1
    const int no = o1 - o0;
    for (int i = threadIdx.x; i < no * f2n * kCB; i += kThreads) {
        const int c = i % kCB, op = i / kCB;
        const int o = op / f2n, p = op - o * f2n;
        const T *w = w2 + (c0 + c) * 9;
        const float *sa = s1 + (c * nr1 + 2 * o) * s1w + 2 * p;   // rows 2o..2o+2 (local), cols 2p-2..
        float acc = Elem<T>::to_f(b2[c0 + c]);
#pragma unroll
        for (int di = 0; di < 3; ++di)
#pragma unroll
            for (int dj = 0; dj < 3; ++dj)
                acc = fmaf(Elem<T>::to_f(w[di * 3 + dj]), sa[di * s1w + dj], acc);
        y[(((int64_t)b * (t2n - first2) + (o0 + o - first2)) * f2n + p) * C + c0 + c] =
            Elem<T>::from_f(acc);
    }
}

// depthwise 3x3 stride-2 causal conv + bias over channels-last rows:
// x [B][tin - first_in][fin][C] holds input rows first_in .. tin-1,
// y [B][tout - first_out][fout][C] gets output rows first_out .. tout-1
template <typename T>
__global__ void __launch_bounds__(kThreads)
    subsample_dw_kernel(const T *x, int batch, int tin, int first_in, int fin, const T *w,
                        const T *bias, int C, int first_out, T *y) {
    const int tout = conv_out(tin), fout = conv_out(fin);
    const int64_t n = (int64_t)batch * (tout - first_out) * fout * C;
    grid_dep_wait();
    grid_dep_launch();
    for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * kThreads) {
        const int c = (int)(i % C);
        int64_t r = i / C;
        const int p = (int)(r % fout);
        r /= fout;
        const int o = first_out + (int)(r % (tout - first_out));
        const int b = (int)(r / (tout - first_out));
        float acc = Elem<T>::to_f(bias[c]);
        const T *wc = w + c * 9;
#pragma unroll
        for (int di = 0; di < 3; ++di) {
            const int t = 2 * o - 2 + di;
            if (t < first_in || t >= tin) continue;   // rows before first_in are not read
#pragma unroll
            for (int dj = 0; dj < 3; ++dj) {
                const int f = 2 * p - 2 + dj;
                if (f < 0 || f >= fin) continue;
                acc = fmaf(Elem<T>::to_f(wc[di * 3 + dj]),
                           Elem<T>::to_f(x[(((int64_t)b * (tin - first_in) + (t - first_in)) * fin + f) * C + c]),
                           acc);
            }
        }
        y[i] = Elem<T>::from_f(acc);
    }
}

template <typename T>
int launch_stage12_t(const SubsampleArgs &a, cudaStream_t s) {
    const int t1n = conv_out(a.frames), f1n = conv_out(a.feat);
    const int t2n = conv_out(t1n);
    const int rows = t2n - a.first;
    if (rows <= 0) return PK_OK;
    const int per = rows <= 8 ? rows : 8;
    const int nr1 = 2 * per + 1, nin = 2 * nr1 + 1;
    const size_t smem = sizeof(float) * ((size_t)nin * (a.feat + 3) + (size_t)kCB * nr1 * (f1n + 3));
    auto k = subsample_stage12_kernel<T>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(subsample)");
    }
    const dim3 grid(a.channels / kCB, (rows + per - 1) / per, a.batch);
    cudaError_t e = launch_pdl(k, grid, dim3(kThreads), smem, s, static_cast<const T *>(a.x), a.xb,
                               a.xf, a.xt, a.frames, a.feat, static_cast<const T *>(a.w1),
                               static_cast<const T *>(a.b1), static_cast<const T *>(a.w2),
                               static_cast<const T *>(a.b2), a.channels, a.first, per,
                               static_cast<T *>(a.y));
    return cuda_status(e, "subsample_stage12_kernel");
}

template <typename T>
int launch_dw_t(const SubsampleArgs &a, cudaStream_t s) {
    const int tout = conv_out(a.frames), fout = conv_out(a.feat);
    const int64_t n = (int64_t)a.batch * (tout - a.first_out) * fout * a.channels;
    if (n <= 0) return PK_OK;
    const int64_t blocks = (n + kThreads - 1) / kThreads;
    const dim3 grid((unsigned)(blocks < 148 * 16 ? blocks : 148 * 16));
    cudaError_t e = launch_pdl(subsample_dw_kernel<T>, grid, dim3(kThreads), 0, s,
                               static_cast<const T *>(a.x), a.batch, a.frames, a.first, a.feat,
                               static_cast<const T *>(a.w2), static_cast<const T *>(a.b2),
                               a.channels, a.first_out, static_cast<T *>(a.y));
    return cuda_status(e, "subsample_dw_kernel");
}

}  // namespace

int launch_subsample_stage12(const SubsampleArgs &a, cudaStream_t s) {
    if (a.batch == 0) return PK_OK;
    return a.dtype == PK_DTYPE_BF16 ? launch_stage12_t<__nv_bfloat16>(a, s)
                                    : launch_stage12_t<float>(a, s);
}

int launch_subsample_dw(const SubsampleArgs &a, cudaStream_t s) {
    if (a.batch == 0) return PK_OK;
    return a.dtype == PK_DTYPE_BF16 ? launch_dw_t<__nv_bfloat16>(a, s) : launch_dw_t<float>(a, s);
}

}  // namespace pk
