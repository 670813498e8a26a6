// Streaming log-mel features, batched over streams.
//
// Restates FeatureExtractor._compute_features and push (parakeet/modules/
// feature_extractor.py:63-133) for a whole batch of streams in one launch.
// The reference keeps each stream's recent samples in a host buffer and, at
// every push, recomputes the STFT of the whole buffer to slice out the new
// frames.  A frame depends only on n_fft samples around its centre, so here
// each slot keeps its last PK_FE_HIST samples and its two counters (samples
// seen, frames emitted) on the device, and a push computes exactly the frames
// it emits:
//
//   x  = samples (+ dither), zero before the stream and after its last sample
//   y  = x[t] - preemph * x[t-1]                      (y = 0 past the end)
//   z  = window * y over [f*hop - n_fft/2, f*hop + n_fft/2)
//   P  = |rfft(z)| ** mag_power                       (n_fft/2 + 1 bins)
//   out[m][f] = log(sum_k fb[m][k] * P[k] + guard)
//
// Grid: (frame groups, batch rows).  A CTA stages the samples of its frames in
// shared memory once (windows overlap by n_fft - hop), then each warp takes a
// frame: the 512-point real FFT is a 256-point complex FFT of the even/odd
// sample pairs (radix-4 Stockham, four stages through two shared-memory
// buffers) and the split of its result into the real transform; the mel
// filters are applied over their nonzero runs only (about 2 per FFT bin
// instead of n_mels).  The CTAs of a row count themselves out on a ticket in
// the slot's meta; the last one advances the slot's history and counters, so
// the push stays one launch without any CTA waiting on another.
#include <math.h>

#include <algorithm>
#include <vector>

#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {

// ------------------------------------------------------------ host tables
namespace {

// Slaney's mel scale (librosa hz_to_mel / mel_to_hz with htk=False): linear,
// 3 mels per 200 Hz, below 1 kHz; logarithmic, 27 mels per factor 6.4, above.
constexpr double kMelFsp = 200.0 / 3.0, kMelMinLogHz = 1000.0;
double hz_to_mel(double f) {
    const double min_log_mel = kMelMinLogHz / kMelFsp, logstep = log(6.4) / 27.0;
    return f >= kMelMinLogHz ? min_log_mel + log(f / kMelMinLogHz) / logstep : f / kMelFsp;
}
double mel_to_hz(double m) {
    const double min_log_mel = kMelMinLogHz / kMelFsp, logstep = log(6.4) / 27.0;
    return m >= min_log_mel ? kMelMinLogHz * exp(logstep * (m - min_log_mel)) : kMelFsp * m;
}

}  // namespace

// librosa.filters.mel's published algorithm: n_mels + 2 points evenly spaced
// in mels between fmin and fmax (numpy linspace: start + i * step, the last
// one exactly fmax), filter i the triangle through points i, i+1, i+2 sampled
// at the FFT bin frequencies k / (n_fft / sr), rounded to float32, then (slaney
// norm) scaled by 2 / (hz[i+2] - hz[i]) and rounded again.
int build_feature_tables(int sr, int n_fft, int win, int n_mels, double f_lo, double f_hi,
                         int norm, int32_t *words, int64_t *nwords, int32_t *nnz_out) {
    const int nbins = n_fft / 2 + 1;
    std::vector<double> mel_f(n_mels + 2);
    const double m0 = hz_to_mel(f_lo), m1 = hz_to_mel(f_hi);
    const double step = (m1 - m0) / (n_mels + 1);
    for (int i = 0; i < n_mels + 2; ++i) mel_f[i] = mel_to_hz(i == n_mels + 1 ? m1 : m0 + i * step);
    std::vector<float> fb((size_t)n_mels * nbins);
    std::vector<int32_t> lo(n_mels), cnt(n_mels), off(n_mels);
    const double bin_hz = 1.0 / (n_fft * (1.0 / sr));   // numpy rfftfreq's spacing
    int nnz = 0;
    for (int i = 0; i < n_mels; ++i) {
        const double enorm = 2.0 / (mel_f[i + 2] - mel_f[i]);
        int first = -1, last = -2;
        for (int k = 0; k < nbins; ++k) {
            const double fk = (double)k * bin_hz;
            const double lower = -(mel_f[i] - fk) / (mel_f[i + 1] - mel_f[i]);
            const double upper = (mel_f[i + 2] - fk) / (mel_f[i + 2] - mel_f[i + 1]);
            float w = (float)std::max(0.0, std::min(lower, upper));
            if (norm == 1) w = (float)((double)w * enorm);
            fb[(size_t)i * nbins + k] = w;
            if (w != 0.f) {
                if (first < 0) first = k;
                last = k;
            }
        }
        lo[i] = first < 0 ? 0 : first;
        cnt[i] = last - first + 1 > 0 && first >= 0 ? last - first + 1 : 0;
        off[i] = nnz;
        nnz += cnt[i];
    }
    const int64_t total = kFeHeader + 3LL * n_fft + 3LL * n_mels + nnz;
    *nwords = total;
    *nnz_out = nnz;
    if (!words) return PK_OK;
    for (int i = 0; i < kFeHeader; ++i) words[i] = 0;
    words[kFeMagic] = kFeMagicValue;
    words[kFeNfft] = n_fft;
    words[kFeNmels] = n_mels;
    words[kFeNnz] = nnz;
    words[kFeWin] = win;
    words[kFeRate] = sr;
    float *tw = reinterpret_cast<float *>(words + kFeHeader);
    for (int u = 0; u < n_fft; ++u) {
        const double a = 2.0 * M_PI * u / n_fft;
        tw[2 * u] = (float)cos(a);
        tw[2 * u + 1] = (float)-sin(a);
    }
    float *wnd = tw + 2 * n_fft;
    const int left = (n_fft - win) / 2;   // torch.stft centres a shorter window
    for (int n = 0; n < n_fft; ++n) {
        const int i = n - left;
        double v = 0.0;
        if (i >= 0 && i < win) v = win == 1 ? 1.0 : 0.5 - 0.5 * cos(2.0 * M_PI * i / (win - 1));
        wnd[n] = (float)v;
    }
    int32_t *tl = reinterpret_cast<int32_t *>(wnd + n_fft);
    for (int i = 0; i < n_mels; ++i) {
        tl[i] = lo[i];
        tl[n_mels + i] = cnt[i];
        tl[2 * n_mels + i] = off[i];
    }
    float *tw8 = reinterpret_cast<float *>(tl + 3 * n_mels);
    for (int i = 0; i < n_mels; ++i)
        for (int j = 0; j < cnt[i]; ++j) tw8[off[i] + j] = fb[(size_t)i * nbins + lo[i] + j];
    return PK_OK;
}

// ------------------------------------------------------------ device
namespace {

constexpr int kN = 512, kH = kN / 2, kWarps = 8, kThreads = kWarps * 32;

struct RowHead {
    long long T0, E0;
    int nf, slot, n, epoch, bad, last;
};

__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
    return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}

// Philox-4x32-10 (Salmon, Moraes, Dror and Shaw, "Parallel random numbers: as
// easy as 1, 2, 3", SC 2011): a counter-based generator, so the dither of a
// sample depends only on (seed, slot, stream epoch, sample index), never on
// which CTA computes it.
__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint2 k) {
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        const uint32_t hi0 = __umulhi(0xD2511F53u, c.x), lo0 = 0xD2511F53u * c.x;
        const uint32_t hi1 = __umulhi(0xCD9E8D57u, c.z), lo1 = 0xCD9E8D57u * c.z;
        c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
        k.x += 0x9E3779B9u;
        k.y += 0xBB67AE85u;
    }
    return c;
}

// standard normal for sample s: Box-Muller on one Philox draw per sample pair
__device__ __forceinline__ float gauss(uint32_t seed_lo, uint32_t seed_hi, int slot, int epoch,
                                       long long s) {
    const unsigned long long pair = (unsigned long long)s >> 1;
    const uint4 r = philox4x32_10(make_uint4((uint32_t)pair, (uint32_t)(pair >> 32),
                                             (uint32_t)slot, (uint32_t)epoch),
                                  make_uint2(seed_lo, seed_hi));
    const float u1 = (float)((r.x >> 8) + 1u) * (1.0f / 16777216.0f);   // (0, 1]
    const float u2 = (float)(r.y >> 8) * (1.0f / 16777216.0f);          // [0, 1)
    const float rad = sqrtf(-2.0f * logf(u1));
    float sn, cs;
    sincospif(2.0f * u2, &sn, &cs);
    return (s & 1) ? rad * sn : rad * cs;
}

// 256-point complex DFT of a[] by one warp, radix-4 Stockham (self-sorting):
// stage p = 1, 4, 16, 64 reads a[j + r*64] (r = 0..3), twiddles them by
// w^r with w = exp(-2 pi i (j mod p) / 4p), and writes the 4-point DFT to
// (j - j mod p) * 4 + j mod p + r*p.  The result ends in a[]; b[] is scratch.
// tw[u] = exp(-2 pi i u / 512).
__device__ __forceinline__ void fft256(float2 *a, float2 *b, const float2 *tw, int lane) {
    float2 *src = a, *dst = b;
#pragma unroll
    for (int st = 0; st < 4; ++st) {
        const int p = 1 << (2 * st);
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
            const int j = lane + 32 * jj;
            const int k = j & (p - 1);
            float2 x0 = src[j], x1 = src[j + 64], x2 = src[j + 128], x3 = src[j + 192];
            if (st > 0) {
                const int u = (128 >> (2 * st)) * k;   // w = tw[2 * 64k/p]
                x1 = cmul(x1, tw[u]);
                x2 = cmul(x2, tw[2 * u]);
                x3 = cmul(x3, tw[3 * u]);
            }
            const float2 s02 = make_float2(x0.x + x2.x, x0.y + x2.y);
            const float2 d02 = make_float2(x0.x - x2.x, x0.y - x2.y);
            const float2 s13 = make_float2(x1.x + x3.x, x1.y + x3.y);
            const float2 d13 = make_float2(x1.x - x3.x, x1.y - x3.y);
            const int o = (j - k) * 4 + k;
            dst[o] = make_float2(s02.x + s13.x, s02.y + s13.y);
            dst[o + p] = make_float2(d02.x + d13.y, d02.y - d13.x);       // d02 - i d13
            dst[o + 2 * p] = make_float2(s02.x - s13.x, s02.y - s13.y);
            dst[o + 3 * p] = make_float2(d02.x - d13.y, d02.y + d13.x);   // d02 + i d13
        }
        __syncwarp();
        float2 *t = src;
        src = dst;
        dst = t;
    }
}

__host__ __device__ constexpr int round4(int n) { return (n + 3) & ~3; }

template <typename TO>
__global__ void __launch_bounds__(kThreads)
    features_push_kernel(const FeArgs a, const int fpc, const int span_max) {
    extern __shared__ float4 fe_smem[];
    float *sm = reinterpret_cast<float *>(fe_smem);
    const int tab_words = 3 * kN + 3 * a.n_mels + a.nnz;
    const float2 *tw = reinterpret_cast<const float2 *>(sm);           // [kN]
    const float *win = sm + 2 * kN;                                    // [kN]
    const int *mlo = reinterpret_cast<const int *>(win + kN);          // [n_mels]
    const int *mcnt = mlo + a.n_mels, *moff = mcnt + a.n_mels;
    const float *mw = reinterpret_cast<const float *>(moff + a.n_mels);   // [nnz]
    float2 *fftbuf = reinterpret_cast<float2 *>(sm + round4(tab_words));  // [kWarps][2][kH]
    float *span = reinterpret_cast<float *>(fftbuf + kWarps * 2 * kH);    // [span_max]
    float *stage = span + span_max;                                       // [n_mels][fpc]
    __shared__ RowHead hd;

    const int row = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // the tables are constant: stage them before waiting on the previous kernel
    for (int i = tid; i < tab_words; i += kThreads)
        reinterpret_cast<int32_t *>(sm)[i] = __ldg(a.tables + kFeHeader + i);
    grid_dep_wait();
    grid_dep_launch();
    if (tid == 0) {
        RowHead h;
        h.bad = 0;
        h.last = 0;
        h.nf = 0;
        h.slot = a.slots[row];
        h.n = a.nsamp[row];
        const int fl = a.flags[row];
        if (h.slot < 0 || h.slot >= a.num_slots) {
            if (blockIdx.x == 0) raise(a.error, PK_DEV_BAD_SLOT);
            h.bad = 1;
        } else if (h.n < 0 || (long long)h.n > a.ld) {
            if (blockIdx.x == 0) raise(a.error, PK_DEV_BAD_COUNT);
            h.bad = 1;
        }
        if (!h.bad) {
            const int64_t *m = a.meta + (long long)h.slot * PK_FE_META_STRIDE;
            const bool first = fl & PK_FE_FIRST;
            h.T0 = first ? 0 : m[0];
            h.E0 = first ? 0 : m[1];
            h.epoch = (int)(m[2] + (first ? 1 : 0));
            const long long T1 = h.T0 + h.n;
            long long last;   // last frame this push emits (feature_extractor.py:111-125)
            if (h.n == 0)
                last = h.E0 - 1;
            else if (fl & PK_FE_FINAL)
                last = T1 / a.hop;
            else
                last = T1 <= kH ? h.E0 - 1 : (T1 - kH) / a.hop;
            const long long nf = last >= h.E0 ? last - h.E0 + 1 : 0;
            if (nf > a.max_frames && blockIdx.x == 0) raise(a.error, PK_DEV_BAD_COUNT);
            h.nf = (int)(nf < 0x7fffffffLL ? nf : 0x7fffffffLL);
        }
        if (blockIdx.x == 0) a.nframes[row] = h.bad ? 0 : min(h.nf, a.max_frames);
        hd = h;
    }
    __syncthreads();
    const int fr0 = blockIdx.x * fpc;
    const int ncols = min(fpc, a.max_frames - fr0);
    TO *orow = static_cast<TO *>(a.out) + (long long)row * a.n_mels * a.max_frames + fr0;
    if (hd.bad) {
        for (int i = tid; i < a.n_mels * ncols; i += kThreads) {
            const int m = i / ncols, j = i - m * ncols;
            orow[(long long)m * a.max_frames + j] = Elem<TO>::from_f(a.pad);
        }
        return;   // every CTA of the row takes this branch: no ticket to settle
    }
    const long long T0 = hd.T0, T1 = hd.T0 + hd.n;
    const int nloc = max(0, min(fpc, min(hd.nf, a.max_frames) - fr0));
    const float *xs = a.samples + (long long)row * a.ld;
    float *hx = a.hist + (long long)hd.slot * PK_FE_HIST;

    // x over [S0, S0 + len): one sample before the first window (pre-emphasis)
    const long long S0 = (hd.E0 + fr0) * (long long)a.hop - kH - 1;
    const int len = nloc > 0 ? (nloc - 1) * a.hop + kN + 1 : 0;
    for (int i = tid; i < len; i += kThreads) {
        const long long s = S0 + i;
        float v = 0.f;
        if (s >= 0 && s < T1) {
            if (s >= T0)
                v = xs[s - T0];
            else if (s >= T0 - PK_FE_HIST)
                v = hx[s - (T0 - PK_FE_HIST)];
            else
                raise(a.error, PK_DEV_BAD_COUNT);   // the history covers every frame a push emits
            if (a.dither != 0.f)
                v += a.dither * gauss(a.seed_lo, a.seed_hi, hd.slot, hd.epoch, s);
        }
        span[i] = v;
    }
    __syncthreads();

    float2 *A = fftbuf + warp * 2 * kH, *B = A + kH;
    for (int lf = warp; lf < nloc; lf += kWarps) {
        const float *xf = span + lf * a.hop + 1;   // xf[n]: sample at p0 + n; xf[-1] exists
        const long long p0 = (hd.E0 + fr0 + lf) * (long long)a.hop - kH;
        for (int m = lane; m < kH; m += 32) {
            const int n = 2 * m;
            const float xm = xf[n - 1], x0 = xf[n], x1 = xf[n + 1];
            const float z0 = p0 + n < T1 ? win[n] * (x0 - a.preemph * xm) : 0.f;
            const float z1 = p0 + n + 1 < T1 ? win[n + 1] * (x1 - a.preemph * x0) : 0.f;
            A[m] = make_float2(z0, z1);
        }
        __syncwarp();
        fft256(A, B, tw, lane);
        // split the half-length transform Z into the real one:
        // X[k] = (Z[k] + conj Z[-k]) / 2 + tw[k] (Z[k] - conj Z[-k]) / 2i
        float *P = reinterpret_cast<float *>(B);
        for (int k = lane; k <= kH; k += 32) {
            const float2 zk = A[k & (kH - 1)], zn = A[(kH - k) & (kH - 1)];
            const float2 e = make_float2(0.5f * (zk.x + zn.x), 0.5f * (zk.y - zn.y));
            const float2 o = make_float2(0.5f * (zk.y + zn.y), -0.5f * (zk.x - zn.x));
            const float2 t = cmul(tw[k], o);
            const float re = e.x + t.x, im = e.y + t.y;
            const float mag = sqrtf(re * re + im * im);
            P[k] = a.mag_power == 2.f ? mag * mag
                                      : (a.mag_power == 1.f ? mag : powf(mag, a.mag_power));
        }
        __syncwarp();
        for (int m = lane; m < a.n_mels; m += 32) {
            const int lo = mlo[m], c = mcnt[m];
            const float *w = mw + moff[m];
            float acc = 0.f;
            for (int j = 0; j < c; ++j) acc = fmaf(w[j], P[lo + j], acc);
            stage[m * fpc + lf] = logf(acc + a.guard);
        }
        __syncwarp();
    }
    __syncthreads();
    for (int i = tid; i < a.n_mels * ncols; i += kThreads) {
        const int m = i / ncols, j = i - m * ncols;
        orow[(long long)m * a.max_frames + j] = Elem<TO>::from_f(j < nloc ? stage[m * fpc + j] : a.pad);
    }

    // the last CTA of the row (all others have finished reading the history)
    // moves the slot on: history = samples [T1 - HIST, T1), counters
    if (tid == 0) {
        __threadfence();
        unsigned long long *ticket = reinterpret_cast<unsigned long long *>(
            a.meta + (long long)hd.slot * PK_FE_META_STRIDE + 3);
        const unsigned long long t = atomicAdd(ticket, 1ull);
        hd.last = t == (unsigned long long)(gridDim.x - 1);
        if (hd.last) atomicExch(ticket, 0ull);
    }
    __syncthreads();
    if (!hd.last) return;
    __threadfence();
    constexpr int kPer = PK_FE_HIST / kThreads;
    float nh[kPer];
#pragma unroll
    for (int r = 0; r < kPer; ++r) {
        const long long s = T1 - PK_FE_HIST + tid + r * kThreads;
        nh[r] = s < 0 ? 0.f : (s >= T0 ? xs[s - T0] : hx[s - (T0 - PK_FE_HIST)]);
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < kPer; ++r) hx[tid + r * kThreads] = nh[r];
    if (tid == 0) {
        int64_t *m = a.meta + (long long)hd.slot * PK_FE_META_STRIDE;
        m[0] = T1;
        m[1] = hd.E0 + hd.nf;
        m[2] = hd.epoch;
    }
}

int g_num_sms = 0;

}  // namespace

static_assert(PK_FE_HIST % kThreads == 0, "history update splits evenly over the CTA");

int launch_features(const FeArgs &a, cudaStream_t s) {
    if (a.batch == 0) return PK_OK;
    if (g_num_sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            g_num_sms = 148;
    }
    // 1..4 frames per warp: enough CTAs for two per SM, the tables staged once per CTA
    int fpc = kWarps;
    while (fpc < 4 * kWarps &&
           (long long)a.batch * ((a.max_frames + 2 * fpc - 1) / (2 * fpc)) >= 2LL * g_num_sms)
        fpc *= 2;
    const int span_max = round4((fpc - 1) * a.hop + kN + 1);
    const int tab_words = 3 * kN + 3 * a.n_mels + a.nnz;
    const size_t smem = sizeof(float) * ((size_t)round4(tab_words) + span_max +
                                         (size_t)a.n_mels * fpc) +
                        sizeof(float2) * kWarps * 2 * kH;
    if (smem > 227 * 1024) {
        set_error("features: %zu bytes of shared memory needed", smem);
        return PK_ENOTSUP;
    }
    const int gx = a.max_frames > 0 ? (a.max_frames + fpc - 1) / fpc : 1;
    const dim3 grid(gx, a.batch);
    cudaError_t e;
    if (a.out_dtype == PK_DTYPE_BF16) {
        auto k = features_push_kernel<__nv_bfloat16>;
        static size_t lim = 48 * 1024;
        if (smem > lim) {
            e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(features)");
            lim = smem;
        }
        e = launch_pdl(k, grid, dim3(kThreads), smem, s, a, fpc, span_max);
    } else {
        auto k = features_push_kernel<float>;
        static size_t lim = 48 * 1024;
        if (smem > lim) {
            e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(features)");
            lim = smem;
        }
        e = launch_pdl(k, grid, dim3(kThreads), smem, s, a, fpc, span_max);
    }
    return cuda_status(e, "features_push_kernel");
}

}  // namespace pk
