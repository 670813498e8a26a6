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

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// conv1 of a bf16 model on the tensor cores: an im2col product per block of 16
// stage-1 positions (rows of A: positions (r, q) in row-major order; columns:
// the 9 taps, padded to 16 with zeros) and the block's 16 channels (two n8
// tiles of B = the taps of each channel).  Inputs and taps are bf16 values, so
// the products are exact and only the fp32 accumulation order differs from a
// direct convolution.  Writes ReLU(acc + bias) for positions inside the
// stage-1 grid and 0 elsewhere (rows outside it, the padding columns).
__device__ __forceinline__ void conv1_tensor_core(const float *xs, int fpad,
                                                  const __nv_bfloat16 *w1, const __nv_bfloat16 *b1,
                                                  int t_lo, int r_lo, int nr1, int t1n, int f1n,
                                                  float *s1, int s1w) {
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int gq = lane / 4, tq = lane % 4;
    // B: (tap k, channel n) = w1[n][k]; b0 holds taps 2tq, 2tq+1, b1 taps 2tq+8, 2tq+9
    auto tap = [&](int n, int k) { return k < 9 ? __bfloat162float(w1[n * 9 + k]) : 0.f; };
    uint32_t bw[2][2];
    float bias[2][2];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
        const int n = nt * 8 + gq;
        bw[nt][0] = pack_bf16(tap(n, 2 * tq), tap(n, 2 * tq + 1));
        bw[nt][1] = pack_bf16(tap(n, 2 * tq + 8), tap(n, 2 * tq + 9));
        bias[nt][0] = __bfloat162float(b1[nt * 8 + 2 * tq]);
        bias[nt][1] = __bfloat162float(b1[nt * 8 + 2 * tq + 1]);
    }
    const int npos = nr1 * f1n, ntiles = (npos + 15) / 16;
    for (int mt = warp; mt < ntiles; mt += kThreads / 32) {
        uint32_t a[4];
        int pr[2], pq[2];
        bool ok[2];
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const int p = mt * 16 + gq + 8 * half;
            const int pp = p < npos ? p : 0;
            const int r = pp / f1n, q = pp - r * f1n;
            const int ra = r_lo + r;
            pr[half] = r;
            pq[half] = q;
            ok[half] = p < npos && ra >= 0 && ra < t1n;
            const float *xb = xs + (2 * ra - 2 - t_lo) * fpad + 2 * q;   // input columns 2q-2 ..
            auto x = [&](int k) { return k < 9 ? xb[(k / 3) * fpad + k % 3] : 0.f; };
            a[half] = pack_bf16(x(2 * tq), x(2 * tq + 1));
            a[2 + half] = pack_bf16(x(2 * tq + 8), x(2 * tq + 9));
        }
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
            float c[4] = {0.f, 0.f, 0.f, 0.f};
            mma16816(c, a, bw[nt][0], bw[nt][1]);
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                if (mt * 16 + gq + 8 * half >= npos) continue;
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int ch = nt * 8 + 2 * tq + e;
                    const float v = ok[half] ? fmaxf(c[2 * half + e] + bias[nt][e], 0.f) : 0.f;
                    s1[(ch * nr1 + pr[half]) * s1w + pq[half] + 2] = v;
                }
            }
        }
    }
    // the padding columns q = -2, -1 and f1n of every row and channel
    for (int i = threadIdx.x; i < kCB * nr1 * 3; i += kThreads) {
        const int rc = i / 3, k = i - rc * 3;
        s1[rc * s1w + (k < 2 ? k : s1w - 1)] = 0.f;
    }
}

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
    float *s1c = s1 + c * nr1 * s1w;
    if constexpr (sizeof(T) == 2) {
        conv1_tensor_core(xs, fpad, w1 + c0 * 9, b1 + c0, t_lo, r_lo, nr1, t1n, f1n, s1, s1w);
    } else {
#pragma unroll
    for (int i = 0; i < 9; ++i) wa[i] = Elem<T>::to_f(w1[(c0 + c) * 9 + i]);
    const float ba = Elem<T>::to_f(b1[c0 + c]);
    // conv1 + bias + ReLU, zero outside the stage-1 grid (the next conv's padding)
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

// bf16 models: one CTA per (stream, block of stage-2 rows) for ALL channels.
// conv1's im2col A fragments (16 stage-1 positions x 9 taps, padded to 16) do
// not depend on the channel, so each warp builds those of its MT position
// tiles once, in registers, and the CTA then walks the channels in blocks of
// 16: conv1 on the tensor cores (two n8 tiles of taps) -> ReLU(acc + bias)
// rounded to bf16 (what the reference's conv of a bf16 model leaves) into a
// shared tile [stage-1 row][column parity][column / 2][16 channels] (double
// buffered: one barrier per block; even and odd columns apart, so that the
// stride-2 reads of conv2 by neighbouring positions hit distinct banks) -> the
// depthwise conv2 + bias, a thread per (channel pair, output position) item
// with bf16x2 reads of the tile -> channels-last output rows.  The input
// window is read once per CTA instead of once per channel block.
template <int MT>
__global__ void __launch_bounds__(kThreads)
    subsample_stage12_allc_kernel(const __nv_bfloat16 *x, int64_t xb, int64_t xf, int64_t xt,
                                  int frames, int feat, const __nv_bfloat16 *w1,
                                  const __nv_bfloat16 *b1, const __nv_bfloat16 *w2,
                                  const __nv_bfloat16 *b2, int C, int first2, int rows_per_cta,
                                  __nv_bfloat16 *y) {
    using T = __nv_bfloat16;
    extern __shared__ __align__(16) char s12c_smem[];
    const int t1n = conv_out(frames), f1n = conv_out(feat);
    const int t2n = conv_out(t1n), f2n = conv_out(f1n);
    const int b = blockIdx.y;
    const int o0 = first2 + blockIdx.x * rows_per_cta;
    const int o1 = min(t2n, o0 + rows_per_cta);
    if (o0 >= o1) return;
    const int r_lo = 2 * o0 - 2, nr1 = 2 * (o1 - o0) + 1;
    const int t_lo = 2 * r_lo - 2, nin = 2 * nr1 + 1;
    const int fpad = feat + 3;
    const int half_w = (f1n + 3 + 1) / 2;              // columns -2 .. f1n, per parity
    const int row_el = 2 * half_w * kCB;               // one stage-1 row of the tile
    const int plane = nr1 * row_el;                    // one tile, elements
    T *xs = reinterpret_cast<T *>(s12c_smem);          // [nin][fpad]
    T *s1 = xs + ((nin * fpad + 7) & ~7);               // [2][nr1][2][half_w][kCB], 16-byte aligned
    // element offset of stage-1 column index cc (= q + 2, 0 .. f1n + 2) within a row
    auto col_off = [&](int cc) { return ((cc & 1) * half_w + (cc >> 1)) * kCB; };
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int gq = lane / 4, tq = lane % 4;
    const T zero = __float2bfloat16_rn(0.f);
    grid_dep_wait();
    const T *xrow = x + (int64_t)b * xb;
    for (int i = threadIdx.x; i < nin * fpad; i += kThreads) {
        const int j = i / nin, r = i - j * nin;
        const int t = t_lo + r, f = j - 2;
        xs[r * fpad + j] = (t >= 0 && t < frames && f >= 0 && f < feat)
                               ? xrow[(int64_t)f * xf + (int64_t)t * xt] : zero;
    }
    // the padding columns q = -2, -1, f1n of both tiles stay zero for every block
    for (int i = threadIdx.x; i < 2 * nr1 * 3 * (kCB / 2); i += kThreads) {
        const int cp = i % (kCB / 2), rest = i / (kCB / 2);
        const int k = rest % 3, rb = rest / 3;               // rb = buffer * nr1 + row
        const int cc = k < 2 ? k : f1n + 2;
        reinterpret_cast<uint32_t *>(s1 + (size_t)(rb / nr1) * plane + (rb % nr1) * row_el +
                                     col_off(cc))[cp] = 0u;
    }
    __syncthreads();
    // A fragments of this warp's position tiles, and where each row of them goes
    const int npos = nr1 * f1n, ntiles = (npos + 15) / 16;
    uint32_t af[MT][4];
    int dst[MT][2];           // element offset of the position in a tile, -1: none
    uint32_t inside = 0;      // bit 2i + half: a stage-1 position inside the grid (else 0)
#pragma unroll
    for (int i = 0; i < MT; ++i) {
        const int mt = warp + i * (kThreads / 32);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const int p = mt * 16 + gq + 8 * half;
            const int pp = p < npos ? p : 0;
            const int r = pp / f1n, q = pp - r * f1n;
            const int ra = r_lo + r;
            dst[i][half] = (mt < ntiles && p < npos) ? r * row_el + col_off(q + 2) : -1;
            if (ra >= 0 && ra < t1n) inside |= 1u << (2 * i + half);
            const T *xp = xs + (2 * ra - 2 - t_lo) * fpad + 2 * q;   // input columns 2q-2 ..
            auto xv = [&](int k) {
                return (k < 9 && mt < ntiles) ? __bfloat162float(xp[(k / 3) * fpad + k % 3]) : 0.f;
            };
            af[i][half] = pack_bf16(xv(2 * tq), xv(2 * tq + 1));
            af[i][2 + half] = pack_bf16(xv(2 * tq + 8), xv(2 * tq + 9));
        }
    }
    // conv2 items: (output position idx = o * f2n + p, channel pair cp)
    const int cp = threadIdx.x % (kCB / 2), i0 = threadIdx.x / (kCB / 2);
    constexpr int kStride = kThreads / (kCB / 2);
    const int no = o1 - o0, nitems = no * f2n;
    T *yb = y + ((int64_t)b * (t2n - first2) + (o0 - first2)) * f2n * C + 2 * cp;
    for (int cb = 0; cb < C / kCB; ++cb) {
        T *tile = s1 + (size_t)(cb & 1) * plane;
        // ---- conv1 of channels [16 cb, 16 cb + 16)
        uint32_t bw[2][2];
        float bias[2][2];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
            const T *wn = w1 + (cb * kCB + nt * 8 + gq) * 9;
            auto tap = [&](int k) { return k < 9 ? __bfloat162float(wn[k]) : 0.f; };
            bw[nt][0] = pack_bf16(tap(2 * tq), tap(2 * tq + 1));
            bw[nt][1] = pack_bf16(tap(2 * tq + 8), tap(2 * tq + 9));
            bias[nt][0] = __bfloat162float(b1[cb * kCB + nt * 8 + 2 * tq]);
            bias[nt][1] = __bfloat162float(b1[cb * kCB + nt * 8 + 2 * tq + 1]);
        }
#pragma unroll
        for (int i = 0; i < MT; ++i) {
            if (warp + i * (kThreads / 32) >= ntiles) break;
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
                float c[4] = {0.f, 0.f, 0.f, 0.f};
                mma16816(c, af[i], bw[nt][0], bw[nt][1]);
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    if (dst[i][half] < 0) continue;
                    const bool in = (inside >> (2 * i + half)) & 1u;
                    const float v0 = in ? fmaxf(c[2 * half] + bias[nt][0], 0.f) : 0.f;
                    const float v1 = in ? fmaxf(c[2 * half + 1] + bias[nt][1], 0.f) : 0.f;
                    *reinterpret_cast<uint32_t *>(tile + dst[i][half] + nt * 8 + 2 * tq) =
                        pack_bf16(v0, v1);
                }
            }
        }
        __syncthreads();   // the block's stage-1 tile is complete
        if (cb == 0) grid_dep_launch();
        // ---- depthwise conv2 + bias of channels 16 cb + 2 cp, + 1
        float wa[2][9];
        const T *wc = w2 + (cb * kCB + 2 * cp) * 9;
#pragma unroll
        for (int k = 0; k < 18; ++k) wa[k / 9][k % 9] = __bfloat162float(wc[k]);
        const float bb0 = __bfloat162float(b2[cb * kCB + 2 * cp]);
        const float bb1 = __bfloat162float(b2[cb * kCB + 2 * cp + 1]);
        for (int idx = i0; idx < nitems; idx += kStride) {
            const int o = idx / f2n, p = idx - o * f2n;
            // stage-1 rows 2o .. 2o+2 (local), columns 2p-2 .. 2p (column index 2p + dj)
            const T *sr = tile + 2 * o * row_el + 2 * cp;
            float a0 = bb0, a1 = bb1;
#pragma unroll
            for (int di = 0; di < 3; ++di)
#pragma unroll
                for (int dj = 0; dj < 3; ++dj) {
                    const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(
                        sr + di * row_el + col_off(2 * p + dj)));
                    a0 = fmaf(wa[0][di * 3 + dj], v.x, a0);
                    a1 = fmaf(wa[1][di * 3 + dj], v.y, a1);
                }
            *reinterpret_cast<uint32_t *>(yb + (int64_t)idx * C + cb * kCB) = pack_bf16(a0, a1);
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

// bf16, channel counts that are a power of two in [32, 512]: the depthwise conv3
// with one CTA per output row of one stream and a thread per (channel pair,
// every (256 / (C / 2))-th output column): the pair's 18 taps and 2 biases in
// registers, bf16x2 reads of the channels-last input rows (a warp reads 128
// contiguous bytes), no per-output index divisions.
__global__ void __launch_bounds__(kThreads)
    subsample_dw_pairs_kernel(const __nv_bfloat16 *x, int tin, int first_in, int fin,
                              const __nv_bfloat16 *w, const __nv_bfloat16 *bias, int C,
                              int first_out, __nv_bfloat16 *y) {
    const int tout = conv_out(tin), fout = conv_out(fin);
    const int rows_out = tout - first_out;
    const int b = blockIdx.x / rows_out, o = first_out + (blockIdx.x - b * rows_out);
    const int half_c = C / 2, cp = threadIdx.x % half_c, pl = threadIdx.x / half_c;
    const int p_stride = kThreads / half_c;
    float wa[2][9];
    const __nv_bfloat16 *wc = w + 2 * cp * 9;
#pragma unroll
    for (int k = 0; k < 18; ++k) wa[k / 9][k % 9] = __bfloat162float(wc[k]);
    const float b0 = __bfloat162float(bias[2 * cp]), b1 = __bfloat162float(bias[2 * cp + 1]);
    grid_dep_wait();
    grid_dep_launch();
    const __nv_bfloat16 *xb = x + (int64_t)b * (tin - first_in) * fin * C + 2 * cp;
    __nv_bfloat16 *yb = y + ((int64_t)b * rows_out + (o - first_out)) * fout * C + 2 * cp;
    for (int p = pl; p < fout; p += p_stride) {
        float a0 = b0, a1 = b1;
#pragma unroll
        for (int di = 0; di < 3; ++di) {
            const int t = 2 * o - 2 + di;
            if (t < first_in || t >= tin) continue;   // rows before first_in are not read
#pragma unroll
            for (int dj = 0; dj < 3; ++dj) {
                const int f = 2 * p - 2 + dj;
                if (f < 0 || f >= fin) continue;
                const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(
                    xb + ((int64_t)(t - first_in) * fin + f) * C));
                a0 = fmaf(wa[0][di * 3 + dj], v.x, a0);
                a1 = fmaf(wa[1][di * 3 + dj], v.y, a1);
            }
        }
        *reinterpret_cast<uint32_t *>(yb + (int64_t)p * C) = pack_bf16(a0, a1);
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
    if constexpr (sizeof(T) == 2) {
        // every channel per CTA while the position tiles fit the warps' registers
        // (6 tiles per warp: the later chunks of the small model; else up to 9)
        const int ntiles = (nr1 * f1n + 15) / 16;
        if (ntiles <= 9 * (kThreads / 32)) {
            const int half_w = (f1n + 3 + 1) / 2;
            const size_t smem = 2 * (((size_t)nin * (a.feat + 3) + 7) / 8 * 8 +
                                     2 * (size_t)nr1 * 2 * half_w * kCB);
            auto k = ntiles <= 6 * (kThreads / 32) ? subsample_stage12_allc_kernel<6>
                                                   : subsample_stage12_allc_kernel<9>;
            if (smem > 48 * 1024) {
                cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                     (int)smem);
                if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(subsample)");
            }
            const dim3 grid((rows + per - 1) / per, a.batch);
            cudaError_t e = launch_pdl(k, grid, dim3(kThreads), smem, s, static_cast<const T *>(a.x),
                                       a.xb, a.xf, a.xt, a.frames, a.feat,
                                       static_cast<const T *>(a.w1), static_cast<const T *>(a.b1),
                                       static_cast<const T *>(a.w2), static_cast<const T *>(a.b2),
                                       a.channels, a.first, per, static_cast<T *>(a.y));
            return cuda_status(e, "subsample_stage12_allc_kernel");
        }
    }
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
    const int C = a.channels;
    if constexpr (sizeof(T) == 2) {
        if (C >= 32 && C <= 512 && (C & (C - 1)) == 0 &&
            (int64_t)a.batch * (tout - a.first_out) < (1ll << 31) &&
            reinterpret_cast<uintptr_t>(a.x) % 4 == 0 && reinterpret_cast<uintptr_t>(a.y) % 4 == 0 &&
            reinterpret_cast<uintptr_t>(a.w2) % 4 == 0) {
            cudaError_t e = launch_pdl(subsample_dw_pairs_kernel,
                                       dim3((unsigned)(a.batch * (tout - a.first_out))),
                                       dim3(kThreads), 0, s, static_cast<const T *>(a.x), a.frames,
                                       a.first, a.feat, static_cast<const T *>(a.w2),
                                       static_cast<const T *>(a.b2), C, a.first_out,
                                       static_cast<T *>(a.y));
            return cuda_status(e, "subsample_dw_pairs_kernel");
        }
    }
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
