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
    // time fastest: the window is stored frames-contiguous per feature bin
    for (int i = threadIdx.x; i < nin * fpad; i += kThreads) {
        const int j = i / nin, r = i - j * nin;
        const int t = t_lo + r, f = j - 2;
        float v = 0.f;
        if (t >= 0 && t < frames && f >= 0 && f < feat)
            v = Elem<T>::to_f(xrow[(int64_t)f * xf + (int64_t)t * xt]);
        xs[r * fpad + j] = v;
    }
    __syncthreads();
    // thread = (channel c of the block, position lane l of kLanes): the
    // channel's taps stay in registers, positions are walked without divisions
    constexpr int kLanes = kThreads / kCB;
    const int c = threadIdx.x % kCB, l = threadIdx.x / kCB;
    float wa[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) wa[i] = Elem<T>::to_f(w1[(c0 + c) * 9 + i]);
    const float ba = Elem<T>::to_f(b1[c0 + c]);
    // conv1 + bias + ReLU, zero outside the stage-1 grid (the next conv's padding)
    float *s1c = s1 + c * nr1 * s1w;
    for (int r = 0; r < nr1; ++r) {
        const int ra = r_lo + r;
        const bool row_ok = ra >= 0 && ra < t1n;
        const float *xr = xs + (2 * ra - 2 - t_lo) * fpad;
        for (int col = l; col < s1w; col += kLanes) {
            const int q = col - 2;
            float v = 0.f;
            if (row_ok && q >= 0 && q < f1n) {
                const float *xa = xr + 2 * q;              // input columns 2q-2 .. 2q
                float acc = ba;
#pragma unroll
                for (int di = 0; di < 3; ++di)
#pragma unroll
                    for (int dj = 0; dj < 3; ++dj)
                        acc = fmaf(wa[di * 3 + dj], xa[di * fpad + dj], acc);
                v = fmaxf(acc, 0.f);
            }
            s1c[r * s1w + col] = v;
        }
    }
#pragma unroll
    for (int i = 0; i < 9; ++i) wa[i] = Elem<T>::to_f(w2[(c0 + c) * 9 + i]);
    const float bb = Elem<T>::to_f(b2[c0 + c]);
    __syncthreads();
    grid_dep_launch();
    // depthwise conv2 + bias, channels-last output rows o0 .. o1-1
    const int no = o1 - o0;
    T *yb = y + ((int64_t)b * (t2n - first2) + (o0 - first2)) * f2n * C + c0 + c;
    for (int o = 0; o < no; ++o) {
        const float *sr = s1c + 2 * o * s1w;            // stage-1 rows 2o .. 2o+2 (local)
        for (int p = l; p < f2n; p += kLanes) {
            const float *sa = sr + 2 * p;               // stage-1 columns 2p-2 .. 2p
            float acc = bb;
#pragma unroll
            for (int di = 0; di < 3; ++di)
#pragma unroll
                for (int dj = 0; dj < 3; ++dj)
                    acc = fmaf(wa[di * 3 + dj], sa[di * s1w + dj], acc);
            yb[((int64_t)o * f2n + p) * C] = Elem<T>::from_f(acc);
        }
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
