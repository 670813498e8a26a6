// Internal interfaces between the C-ABI layer (pk_api.cu) and the kernel
// translation units.  Nothing here is exported.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "pk.h"

struct pk_paged_kv {
    pk_paged_kv_desc d;
    CUtensorMap kv_map;  // 3-D view {dim, page_size, pages*layers*2}, 128B-swizzled boxes
    int head_dim;
    int esize;
};

namespace pk {

void set_error(const char *fmt, ...);
int cuda_status(cudaError_t e, const char *what);
// pk_selftest.cu: one CTA waits on an mbarrier with the shared bounded wait
int launch_selftest_wait(int32_t *error, int32_t arrive, uint64_t limit_ns, int64_t *waited_ns,
                         cudaStream_t stream);
// Encode a tiled TMA descriptor (driver entry point fetched once via cudart).
int encode_tmap(CUtensorMap *map, int dtype, const void *base, int rank, const uint64_t *dims,
                const uint64_t *strides_bytes, const uint32_t *box);
int encode_tmap_3d(CUtensorMap *map, int dtype, const void *base, uint64_t d0, uint64_t d1,
                   uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box0,
                   uint32_t box1, uint32_t box2);

// Launch with programmatic stream serialization: the kernel may be scheduled
// while the previous kernel of the stream finishes, and must call
// grid_dep_wait() before it reads anything that kernel could have written.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t s, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args &&>(args)...);
}

// pk_pages.cu
int launch_pages_reset(const pk_paged_kv *kv, const int32_t *init_order, cudaStream_t s);
int launch_pages_begin(const pk_paged_kv *kv, const int32_t *slots, const int32_t *lengths,
                       int batch, const int32_t *released, int num_released, cudaStream_t s);
int launch_pages_end(const pk_paged_kv *kv, const int32_t *slots, const int32_t *lengths,
                     int batch, cudaStream_t s);


// pk_kv.cu
int launch_append(const pk_paged_kv *kv, int layer0, int nlayers, const void *key,
                  const void *value, int64_t ls, int64_t bs, int64_t rs, const int32_t *slots,
                  int batch, cudaStream_t s);
int launch_gather(const pk_paged_kv *kv, int layer0, int nlayers, const int32_t *slots, int batch,
                  void *k_out, void *v_out, int64_t out_layer_stride, cudaStream_t s);

// pk_attn.cu
struct AttnArgs {
    const void *q;
    int64_t q_ls, q_bs, q_rs;
    const void *k_new, *v_new;   // optional: this step's K/V rows (q's strides) to append
    const void *bias_u, *bias_v;
    int64_t bias_ls;
    const void *pos;             // pos_proj rows (l, p, c) at l * pos_ls + p * dim + c
    int64_t pos_ls;
    int pos_rows;                // 2 * (left + chunk) - 1
    const float *bd;             // optional: rel-pos term from launch_relpos_bd (replaces pos)
    const int32_t *slots, *lengths;
    int batch;
    void *out;
    int64_t o_ls, o_bs, o_rs;
    int layer0, nlayers;
};
int launch_attention(const pk_paged_kv *kv, const CUtensorMap &pos_map, const AttnArgs &a,
                     cudaStream_t s);
// pk_attn_bf16.cu
int launch_attention_bf16(const pk_paged_kv *kv, const CUtensorMap &pos_map, const AttnArgs &a,
                          cudaStream_t s);
// pk_attn_stacked.cu: all heads of a (stream, layer) per CTA, when heads * chunk <= 16;
// returns PK_ENOTSUP for other shapes.  pos_map16 has 16-row boxes.
int launch_attention_stacked(const pk_paged_kv *kv, const CUtensorMap &pos_map16,
                             const AttnArgs &a, cudaStream_t s);
// pk_attn_stacked.cu: the rel-pos term of every (layer, stream, head, query) of a
// step, bd[l][b][h][t][relpos_bd_cols], for the shapes launch_attention_stacked
// handles (PK_ENOTSUP otherwise); reads a.q, a.bias_v, a.pos.
int relpos_bd_cols(const pk_paged_kv *kv);
int launch_relpos_bd(const pk_paged_kv *kv, const AttnArgs &a, float *bd, cudaStream_t s);
// pk_pages.cu: launch_pages_begin and launch_relpos_bd in one launch (batch <= 256,
// shapes with the pre-pass; PK_ENOTSUP otherwise)
int launch_pages_begin_relpos(const pk_paged_kv *kv, const int32_t *slots,
                              const int32_t *lengths, int batch, const int32_t *released,
                              int num_released, const AttnArgs &a, float *bd, cudaStream_t s);
// pk_attn_heads.cu: head_dim 128, chunks of 8..16 frames, K/V appended before;
// returns PK_ENOTSUP for other shapes.  pos_map16 has 16-row boxes of 64 columns.
int launch_attention_heads(const pk_paged_kv *kv, const CUtensorMap &pos_map16,
                           const AttnArgs &a, cudaStream_t s);

// pk_conv.cu
struct ConvArgs {
    void *state;
    int num_slots, num_layers, layer, dim, kernel, chunk, dtype;
    const void *x;
    int64_t x_bs, x_rs;
    const void *w, *ln_w, *ln_b;
    float eps;
    const int32_t *slots, *lengths;
    int batch;
    void *y;
    int32_t *error;
    int x_vec;   // x rows 16-byte aligned (base, row and batch strides): vector staging
};
int launch_conv(const ConvArgs &a, cudaStream_t s);

// pk_pre_encode.cu
int launch_pre_encode_window(void *cache, const void *feats, const int32_t *slots, int batch,
                             int feat_in, int frames, int csize, int prefix, void *out,
                             int dtype, int32_t *error, int num_slots, cudaStream_t s);

// pk_rnnt.cu
int launch_rnnt_pick(const void *logits, int64_t ld, int dtype, int batch, int nclass, int blank,
                     const int32_t *lengths, int frame, int symbol, int max_symbols, int frames,
                     int32_t *done, int32_t *emit, int64_t *ids, int32_t *tokens, int32_t *counts,
                     cudaStream_t s);
int launch_lstm_cell(const void *gates, int64_t gld, const void *xtab, int64_t xld,
                     const int64_t *ids, void *h, void *c, int64_t sld, const int32_t *emit,
                     int batch, int hidden, int dtype, cudaStream_t s);

// pk_norm.cu
struct LnArgs {
    const void *x;
    int64_t x_ld;
    int rows, dim, dtype;
    const void *g1, *b1;
    float eps1;
    void *y1;
    int64_t y1_ld;
    const void *g2, *b2;   // optional second LayerNorm of y1 (g2 == nullptr: none)
    float eps2;
    void *y2;
    int64_t y2_ld;
};
int launch_layer_norm(const LnArgs &a, cudaStream_t s);

// pk_gemm.cu
struct GemmArgs {
    const void *A, *W;
    int64_t lda, ldw;
    int M, N, K, epilogue;
    void *C;
    int64_t ldc;
    const void *R;
    int64_t ldr;
    const void *bias;
    float alpha;
    int32_t *error;
};
int launch_gemm(const GemmArgs &g, cudaStream_t s);

// pk_subsample.cu
struct SubsampleArgs {
    const void *x;
    int64_t xb, xf, xt;      // stage12: x[b][f][t] strides (elements)
    int batch, frames, feat, channels, dtype;
    const void *w1, *b1, *w2, *b2;   // dw: w2 / b2 are the depthwise conv's
    int first, first_out;
    void *y;
};
int launch_subsample_stage12(const SubsampleArgs &a, cudaStream_t s);
int launch_subsample_dw(const SubsampleArgs &a, cudaStream_t s);

// pk_features.cu.  Table block: int32 header[kFeHeader], then float2
// twiddle[n_fft] (exp(-2 pi i u / n_fft)), float window[n_fft], int32 lo[n_mels],
// cnt[n_mels], off[n_mels] (first bin, length and offset of each filter's
// nonzero run), float weight[nnz].
constexpr int kFeHeader = 16;
enum FeHeaderField { kFeMagic = 0, kFeNfft, kFeNmels, kFeNnz, kFeWin, kFeRate };
constexpr int32_t kFeMagicValue = 0x45464b50;  // "PKFE"
int build_feature_tables(int sample_rate, int n_fft, int win_length, int n_mels, double fmin,
                         double fmax, int norm, int32_t *words, int64_t *nwords, int32_t *nnz);
struct FeArgs {
    const int32_t *tables;
    float *hist;
    int64_t *meta;
    int32_t *error;
    int num_slots, hop, n_mels, nnz;
    float preemph, dither, mag_power, guard, pad;
    uint32_t seed_lo, seed_hi;
    const float *samples;
    int64_t ld;
    const int32_t *nsamp, *flags, *slots;
    int batch;
    void *out;
    int out_dtype, max_frames;
    int32_t *nframes;
};
int launch_features(const FeArgs &a, cudaStream_t s);

}  // namespace pk
