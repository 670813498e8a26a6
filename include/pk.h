/*
 * pk.h - C ABI of libpk.so, the B200 (sm_100a) kernels for the streaming
 * FastConformer hot path of odunola499/parakeet-streaming:
 *
 *   paged K/V append, page-table window gather, paged chunked rel-pos
 *   self-attention, depthwise-conv time-cache step, and the device page
 *   allocator that replaces the reference's dense per-slot pool.
 *
 * Every device buffer is allocated and owned by the caller; the library
 * allocates no device memory.  Pointers are raw device addresses, strides
 * are in elements, `stream` is a cudaStream_t (NULL = legacy default
 * stream).  Every entry point returns PK_OK or a PK_E* status; argument
 * errors are detected on the host before anything is launched.  Faults
 * that only the device can see (pool exhausted, a page id out of range, a
 * bounded wait that gave up) set bits in the caller's `error` word instead
 * of trapping; read it with any device-to-host copy.
 *
 * Citations name the reference interface each entry point stands in for
 * (paths inside the reference source tree).
 */
#ifndef PK_H
#define PK_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define PK_OK 0
#define PK_EINVAL 1   /* bad argument: shape, alignment, null pointer      */
#define PK_ECUDA 2    /* a CUDA runtime call failed (see pk_last_error)    */
#define PK_ENOTSUP 3  /* configuration this build does not handle          */

/* element types */
#define PK_DTYPE_F32 0
#define PK_DTYPE_BF16 1

/* bits of the device error word */
#define PK_DEV_POOL_EXHAUSTED 1  /* a step asked for more pages than free  */
#define PK_DEV_BAD_PAGE 2        /* a page-table entry outside the pool    */
#define PK_DEV_TIMEOUT 4         /* a bounded wait on a TMA barrier ran out */
#define PK_DEV_BAD_SLOT 8        /* a slot id outside [0, num_slots)       */

/* per-slot counters, int32 [num_slots][PK_META_STRIDE] */
#define PK_META_FIRST 0      /* oldest logical page held                   */
#define PK_META_NEXT 1       /* next logical page to allocate              */
#define PK_META_WRITTEN 2    /* rows written so far (chunk per step)       */
#define PK_META_PROCESSED 3  /* StreamingState.processed_frames            */
#define PK_META_CACHE_LEN 4  /* StreamingState.cache_lengths (<= left)     */
#define PK_META_STRIDE 8

/* per-batch-row window descriptor of the current step, int32
 * [num_slots][PK_WIN_STRIDE], written by pk_pages_begin_step: the pages
 * that hold the stream's window, the first row of each page's box, and the
 * streaming mask as bit rows (bit j%32 of word [i*4 + j/32]: key j allowed
 * for query i) */
#define PK_WIN_OK 0
#define PK_WIN_W 1
#define PK_WIN_PROC 2
#define PK_WIN_CLEN 3
#define PK_WIN_LEN 4
#define PK_WIN_NB 5
#define PK_WIN_NFIRST 6
#define PK_WIN_SLOT 7
#define PK_WIN_PAGE 8
#define PK_WIN_START 24
#define PK_WIN_MASK 40
#define PK_WIN_MAX_PAGES 16
#define PK_WIN_STRIDE 128
/* most batch rows of one step (pk_pages_begin_step) */
#define PK_MAX_BATCH 6144

/*
 * Paged K/V window of every stream slot.  Replaces ModelCache.attn_k /
 * attn_v (parakeet/modules/cache.py:24-29) and the slot pool's state
 * tensors (parakeet/engine/scheduler.py:68-84).
 */
typedef struct pk_paged_kv_desc {
    void *kv;             /* [num_pages][num_layers][2][num_heads][page_size][head_dim] */
    int32_t *page_table;  /* [num_slots][ring], -1 = no page                 */
    int32_t *free_ring;   /* [num_pages] FIFO of free page ids               */
    int64_t *ring_ctr;    /* [2] monotonic head (pop) and tail (push)        */
    int32_t *meta;        /* [num_slots][PK_META_STRIDE]                     */
    int32_t *error;       /* [1] device error word (PK_DEV_* bits)           */
    int32_t *window;      /* [num_slots][PK_WIN_STRIDE] step window descriptors,
                             16-byte aligned */
    int32_t num_pages;
    int32_t num_slots;
    int32_t num_layers;
    int32_t dim;          /* model width D                                   */
    int32_t num_heads;    /* H, head_dim = dim / num_heads (64 or 128)       */
    int32_t left;         /* left attention context (70)                     */
    int32_t chunk;        /* frames per step T = right context + 1           */
    int32_t page_size;    /* frames per page (16)                            */
    int32_t ring;         /* page-table entries per slot (power of two,
                             pk_pages_per_stream() <= ring <= PK_WIN_MAX_PAGES) */
    int32_t dtype;        /* PK_DTYPE_*                                       */
} pk_paged_kv_desc;

typedef struct pk_paged_kv pk_paged_kv; /* opaque: desc + TMA descriptors */

/* Validate `desc`, encode the pool's TMA descriptor, return a host handle.
 * Replaces Scheduler.init_state_pool (parakeet/engine/scheduler.py:68-84). */
int pk_paged_kv_create(const pk_paged_kv_desc *desc, pk_paged_kv **out);
int pk_paged_kv_destroy(pk_paged_kv *kv);

/* Page-table entries a stream needs at most / the ring size to give it. */
int32_t pk_pages_per_stream(int32_t left, int32_t chunk, int32_t page_size);
int32_t pk_ring_size(int32_t left, int32_t chunk, int32_t page_size);

/* Reset the pool: every page free in `init_order` (device int32
 * [num_pages], a permutation) or 0..num_pages-1 when NULL; every slot
 * empty; error word cleared.  The free_ring order is the allocation order,
 * like deque(range(pool)) in scheduler.py:84. */
int pk_pages_reset(pk_paged_kv *kv, const int32_t *init_order, void *stream);

/* Start of one batched step (one CTA, deterministic order;
 * batch <= PK_MAX_BATCH):
 *  0. return every page of the `released` slots (finished streams,
 *     parakeet/engine/scheduler.py:101-104) and zero their counters;
 *  1. per batch row, in order: free pages wholly left of the window;
 *  2. per batch row, in order: allocate pages for rows [w, w + chunk);
 *  3. write each batch row's window descriptor (`lengths` NULL = full
 *     chunks), read by the attention kernels of every layer of the step.
 * Replaces the pool half of Scheduler.pack_states (scheduler.py:128-170):
 * nothing is gathered, the kernels read the pages in place. */
int pk_pages_begin_step(pk_paged_kv *kv, const int32_t *slots, const int32_t *lengths,
                        int32_t batch, const int32_t *released, int32_t num_released,
                        void *stream);

/* End of the step: written += chunk, processed += length,
 * cache_len = min(cache_len + length, left) per batch row
 * (parakeet/modules/encoder.py:257-260; unpack_states, scheduler.py:172-201,
 * has nothing left to scatter). */
int pk_pages_end_step(pk_paged_kv *kv, const int32_t *slots,
                      const int32_t *lengths, int32_t batch, void *stream);

/* Write this step's `chunk` new K and V rows of layers
 * [layer0, layer0 + num_layers) into the pages.  key/value element
 * (l, b, t, c) is at l*layer_stride + b*batch_stride + t*row_stride + c,
 * e.g. the K and V thirds of the fused qkv GEMM output.
 * Replaces ModelCache.update_attn_cache (parakeet/modules/cache.py:36-45). */
int pk_append_kv(pk_paged_kv *kv, int32_t layer0, int32_t num_layers,
                 const void *key, const void *value, int64_t layer_stride,
                 int64_t batch_stride, int64_t row_stride,
                 const int32_t *slots, int32_t batch, void *stream);

/* Materialise the [batch][left + chunk][dim] K and V windows of one layer
 * exactly as the reference's dense cache holds them (rows before a
 * stream's first frame are zero).  Call after pk_append_kv of the step.
 * Replaces the (K, V) return value of ModelCache.update_attn_cache
 * (cache.py:45) and the index_select gather (scheduler.py:150-161). */
int pk_gather_window(pk_paged_kv *kv, int32_t layer, const int32_t *slots,
                     int32_t batch, void *k_out, void *v_out, void *stream);

/* pk_gather_window for layers [layer0, layer0 + num_layers) in one launch:
 * layer l's windows at k_out / v_out + (l - layer0) * out_layer_stride
 * elements (>= batch * (left + chunk) * dim, 16-byte multiple).  Same
 * replaced calls, for callers that materialise every layer of a step. */
int pk_gather_windows(pk_paged_kv *kv, int32_t layer0, int32_t num_layers,
                      const int32_t *slots, int32_t batch, void *k_out, void *v_out,
                      int64_t out_layer_stride, void *stream);

/* Chunked rel-pos multi-head self-attention over the paged window, for
 * layers [layer0, layer0 + num_layers).
 *   query  (l, b, t, c)  at l*q_layer_stride + b*q_batch_stride + t*q_row_stride + c
 *   key/value            NULL, or this step's new K/V rows with the query's
 *                        strides (e.g. the K and V thirds of the fused qkv GEMM
 *                        output): they are appended to the pages as part of
 *                        the call, so pk_append_kv is not needed.  With NULL,
 *                        pk_append_kv must have run for this step.
 *   pos_proj (l, p, c)   at l*pos_layer_stride + p*dim + c, p < 2*(left+chunk)-1:
 *                        linear_pos(pos_emb) of that layer (attention.py:102-106)
 *   bias_u/v (l, h, d)   at l*bias_layer_stride + h*head_dim + d (pos_bias_u/v)
 *   out    (l, b, t, c)  at l*out_layer_stride + b*out_batch_stride + t*out_row_stride + c
 * The streaming mask (parakeet/modules/encoder.py:167-227) comes from the
 * step's window descriptors, so pk_pages_begin_step must have run for the
 * same `slots` and `lengths`.  Output is the heads concatenated, before
 * linear_out.
 * Replaces ModelCache.update_attn_cache (cache.py:36-45, when key/value are
 * given) and ConformerAttention.forward lines 99-122
 * (parakeet/modules/attention.py), i.e. rel_shift + bias + SDPA. */
int pk_paged_attention(pk_paged_kv *kv, int32_t layer0, int32_t num_layers,
                       const void *query, int64_t q_layer_stride,
                       int64_t q_batch_stride, int64_t q_row_stride,
                       const void *key, const void *value,
                       const void *pos_proj, int64_t pos_layer_stride,
                       const void *bias_u, const void *bias_v,
                       int64_t bias_layer_stride, const int32_t *slots,
                       const int32_t *lengths, int32_t batch, void *out,
                       int64_t out_layer_stride, int64_t out_batch_stride,
                       int64_t out_row_stride, void *stream);

/* Row length (floats) of the rel-pos term pk_relpos_bd writes for this pool:
 * 16 * ceil((left + 2 * chunk - 1) / 16); 0 when the pool's shape has no
 * pre-pass (it needs bf16, head_dim 64, heads a multiple of 4, 4 * chunk <= 16
 * and 16-frame pages; pk_paged_attention covers every shape). */
int32_t pk_relpos_bd_cols(const pk_paged_kv *kv);

/* The rel-pos term of the attention logits for every (layer, stream, head,
 * query row) of a step, before its 1/sqrt(head_dim) scale:
 *   bd[l][b][h][t][r] = sum_d bf16(q[l][b][t][h*dh + d] + bias_v[l][h][d])
 *                             * pos_proj[l][r][h*dh + d]      (fp32)
 * for r < pk_relpos_bd_cols(kv) (rows >= 2*(left+chunk)-1 read as zero);
 * query / pos_proj / bias_v as in pk_paged_attention, bd 16-byte aligned with
 * num_layers * batch * heads * chunk * cols floats.  Every stream of a layer
 * uses the same pos_proj rows, so this pass reads them once per (layer, head)
 * instead of once per stream.  It is the (q + pos_bias_v) pos^T product of
 * ConformerAttention.forward lines 108-110 (parakeet/modules/attention.py),
 * before rel_shift. */
int pk_relpos_bd(pk_paged_kv *kv, int32_t layer0, int32_t num_layers,
                 const void *query, int64_t q_layer_stride, int64_t q_batch_stride,
                 int64_t q_row_stride, const void *pos_proj, int64_t pos_layer_stride,
                 const void *bias_v, int64_t bias_layer_stride, int32_t batch,
                 float *bd, void *stream);

/* pk_pages_begin_step and pk_relpos_bd for the same step in one launch (its
 * first CTA runs the page allocator and window descriptors, the others the
 * pre-pass tiles): the same outputs as the two calls, with one link fewer in
 * the step's launch chain.  Arguments are those of the two calls (the
 * pre-pass's batch is the step's batch).  Batches above 256 rows run as the
 * two launches.  Replaces, as those two do, Scheduler.pack_states +
 * _create_streaming_masks (parakeet/engine/scheduler.py:106-170,
 * parakeet/modules/encoder.py:167-227) and the (q + pos_bias_v) pos^T product
 * of ConformerAttention.forward lines 108-110 (parakeet/modules/attention.py). */
int pk_pages_begin_step_relpos(pk_paged_kv *kv, const int32_t *slots,
                               const int32_t *lengths, int32_t batch,
                               const int32_t *released, int32_t num_released,
                               int32_t layer0, int32_t num_layers, const void *query,
                               int64_t q_layer_stride, int64_t q_batch_stride,
                               int64_t q_row_stride, const void *pos_proj,
                               int64_t pos_layer_stride, const void *bias_v,
                               int64_t bias_layer_stride, float *bd, void *stream);

/* pk_paged_attention with the rel-pos term taken from pk_relpos_bd's output
 * for the same query, layers and batch (in place of pos_proj and bias_v).
 * Same outputs, same replaced calls; for the shapes pk_relpos_bd_cols
 * accepts. */
int pk_paged_attention_bd(pk_paged_kv *kv, int32_t layer0, int32_t num_layers,
                          const void *query, int64_t q_layer_stride,
                          int64_t q_batch_stride, int64_t q_row_stride,
                          const void *key, const void *value, const float *bd,
                          const void *bias_u, int64_t bias_layer_stride,
                          const int32_t *slots, const int32_t *lengths, int32_t batch,
                          void *out, int64_t out_layer_stride, int64_t out_batch_stride,
                          int64_t out_row_stride, void *stream);

/* Size of the one static device array pk_paged_attention_noalloc works in. */
#define PK_NOALLOC_SCRATCH_BYTES (32 * 1024 * 1024)

/* pk_paged_attention (same arguments, same output) for callers that cannot
 * allocate device memory: hosts whose device memory is all reserved up front
 * and owned by another allocator (a framework's caching pool, a fixed memory
 * cap per process), and latency-bound serving loops that must not call
 * cudaMalloc / cudaFree, which can block and synchronise the device.  The
 * rel-pos term that pk_relpos_bd would write into a caller buffer goes into a
 * static device array of PK_NOALLOC_SCRATCH_BYTES (32 MiB) that every GPU
 * loading this library holds until the process exits; the call allocates
 * nothing, with no allocating library routine either.  It has no counterpart
 * in the reference.
 *   - limit: PK_EINVAL before any launch when num_layers * batch * heads *
 *     chunk * pk_relpos_bd_cols * 4 bytes exceeds PK_NOALLOC_SCRATCH_BYTES
 *     (split the call by layers or streams);
 *   - the first call on a device, and the first after a pool is created on
 *     that device, looks up the array's device address (cudaGetSymbolAddress,
 *     with that device current): make those calls before any stream capture;
 *     the pool must be on the current device.  A device reset
 *     (cudaDeviceReset) loads the array anew at another address; the pools
 *     made after the reset (the old ones lost their memory) renew it;
 *   - every call uses the same array: calls whose work overlaps on the GPU
 *     (other streams, other threads) race; order them on one stream.  Each
 *     call writes every element it reads, so no clearing is needed;
 *   - shapes without the pre-pass (pk_relpos_bd_cols == 0) run
 *     pk_paged_attention, which needs no scratch. */
int pk_paged_attention_noalloc(pk_paged_kv *kv, int32_t layer0, int32_t num_layers,
                               const void *query, int64_t q_layer_stride,
                               int64_t q_batch_stride, int64_t q_row_stride,
                               const void *key, const void *value,
                               const void *pos_proj, int64_t pos_layer_stride,
                               const void *bias_u, const void *bias_v,
                               int64_t bias_layer_stride, const int32_t *slots,
                               const int32_t *lengths, int32_t batch, void *out,
                               int64_t out_layer_stride, int64_t out_batch_stride,
                               int64_t out_row_stride, void *stream);

/* Depthwise causal conv step with its time cache, one layer:
 *   GLU over the pw-conv1 output x (l=0: [batch][chunk][2*dim] with
 *   x_batch_stride / x_row_stride) -> zero rows t >= length -> depthwise conv
 *   over cat(cache, x) with weight [dim][kernel] -> cache = last kernel-1
 *   frames -> if ln_weight: LayerNorm(eps) then SiLU -> y [batch][chunk][dim].
 * conv_state is [num_slots][num_layers][dim][kernel-1] in the reference's
 * own layout (ModelCache.conv, cache.py:30-34), updated in place by slot.
 * Replaces ConformerConvolution.forward lines 153-159 with
 * CausalConv1d.update_cache (parakeet/modules/convolution.py:37-52,150-162)
 * and ModelCache.get/update_conv_cache (cache.py:47-53). */
int pk_conv_step(void *conv_state, int32_t num_slots, int32_t num_layers,
                 int32_t layer, int32_t dim, int32_t kernel, int32_t chunk,
                 int32_t dtype, const void *x, int64_t x_batch_stride,
                 int64_t x_row_stride, const void *weight,
                 const void *ln_weight, const void *ln_bias, float ln_eps,
                 const int32_t *slots, const int32_t *lengths, int32_t batch,
                 void *y, int32_t *error, void *stream);

/* Streaming pre-encoder input of a batch: out[b] = cat(the last prefix_frames
 * cached frames of slot slots[b], feats[b]) along time ([batch][feat_in]
 * [prefix_frames + frames]; prefix_frames = 0 for a stream's first chunk),
 * then cache[slots[b]] = the last min(csize, prefix_frames + frames) frames of
 * out[b], right-aligned.  cache [num_slots][feat_in][csize], feats [batch]
 * [feat_in][frames], `dtype` PK_DTYPE_*; prefix_frames must not exceed the
 * frames the slot's cache holds (csize, or a shorter first window); bad slot
 * ids set PK_DEV_BAD_SLOT in *error.  Replaces the per-stream cache copies of
 * ModelRunner._run_pre_encode (parakeet/engine/model_runner.py:197-233). */
int pk_pre_encode_window(void *cache, int32_t num_slots, const void *feats,
                         const int32_t *slots, int32_t batch, int32_t feat_in, int32_t frames,
                         int32_t csize, int32_t prefix_frames, void *out, int32_t dtype,
                         int32_t *error, void *stream);

/* The strided convs of ConvSubsampling (parakeet/modules/subsample.py:
 * 61-179, dw_striding; every conv causal: CausalConv2D, convolution.py:55-104,
 * output (o, p) reads input rows 2o-2 .. 2o and columns 2p-2 .. 2p, zero
 * outside).  pk_subsample_stage12: conv1 (1 -> C, 3x3 stride 2, bias, ReLU)
 * and the depthwise conv2 (3x3 stride 2, bias) in one launch, conv1's
 * activation kept in shared memory; x[b][f][t] at b*x_batch_stride +
 * f*x_feat_stride + t*x_time_stride (the pre-encode window, frames x feat
 * per row); y channels-last [batch][T2 - first_row][F2][C] with T2, F2 the
 * conv2 output sizes, holding conv2 rows first_row .. T2-1.  C a multiple of
 * 16.  w1, w2 are [C][1][3][3], b1, b2 [C]. */
int pk_subsample_stage12(const void *x, int64_t x_batch_stride, int64_t x_feat_stride,
                         int64_t x_time_stride, int32_t batch, int32_t frames, int32_t feat,
                         const void *w1, const void *b1, const void *w2, const void *b2,
                         int32_t channels, int32_t first_row, void *y, int32_t dtype,
                         void *stream);

/* Depthwise 3x3 stride-2 causal conv + bias over channels-last rows: x
 * [batch][rows_in - first_in][cols_in][C] holds input rows first_in ..
 * rows_in-1 (earlier rows are never read: first_in <= max(0, 2*first_out - 2));
 * y [batch][R - first_out][Cout][C] gets output rows first_out .. R-1 (R =
 * rows_in / 2 + 1, Cout = cols_in / 2 + 1).  w [C][1][3][3], b [C]. */
int pk_subsample_dw(const void *x, int32_t batch, int32_t rows_in, int32_t first_in,
                    int32_t cols_in, const void *w, const void *b, int32_t channels,
                    int32_t first_out, void *y, int32_t dtype, void *stream);

/* ---------------- batched greedy RNNT decode (device-side bookkeeping) ----
 * A chunk's decode runs, for every frame f < frames and symbol s <
 * max_symbols, joint -> pk_rnnt_pick -> prediction step -> pk_lstm_cell, all
 * on one stream with no host round trip.  Replaces the per-symbol host work of
 * ModelRunner._decode_frame_batch (parakeet/engine/model_runner.py:415-447):
 * logits.argmax, the blank mask, `bool(blank_mask.all())`, `ids.tolist()` and
 * the torch.where state selects. */

/* Argmax (first maximum) of each row's `num_classes` logits (row stride
 * `logits_ld` elements, `dtype` PK_DTYPE_*).  Row b emits when it has not
 * stopped in this frame (done[b], reset when symbol == 0), frame < lengths[b]
 * and the argmax is not `blank`: emit[b] = 1, ids[b] = token, tokens[b][frame]
 * [symbol] = token, counts[b][frame] += 1; otherwise emit[b] = 0, ids[b] =
 * blank, tokens[...] = -1 and the row stops for the frame.  tokens is int32
 * [batch][frames][max_symbols], counts int32 [batch][frames]. */
int pk_rnnt_pick(const void *logits, int64_t logits_ld, int32_t dtype, int32_t batch,
                 int32_t num_classes, int32_t blank, const int32_t *lengths, int32_t frame,
                 int32_t symbol, int32_t max_symbols, int32_t frames, int32_t *done,
                 int32_t *emit, int64_t *ids, int32_t *tokens, int32_t *counts, void *stream);

/* One LSTM cell step from precomputed gates [batch][4 * hidden] (x W_ih^T +
 * h W_hh^T + biases, PyTorch order i, f, g, o; row stride `gates_ld`), plus,
 * when xtab != NULL, the row xtab[ids[b]] (row stride xtab_ld: a per-token
 * table of the embedding times W_ih plus the biases), into the state rows
 * h, c (row stride `state_ld`), only for rows with emit[b] != 0; other rows
 * keep their state.  Replaces the embedding and nn.LSTM step of
 * Predictor.forward (parakeet/modules/decoder.py:44-50) and the torch.where
 * of model_runner.py:433-445. */
int pk_lstm_cell(const void *gates, int64_t gates_ld, const void *xtab, int64_t xtab_ld,
                 const int64_t *ids, void *h, void *c, int64_t state_ld, const int32_t *emit,
                 int32_t batch, int32_t hidden, int32_t dtype, void *stream);

/* bf16 GEMM on the tcgen05 tensor cores (fp32 accumulation in tensor
 * memory) with the encoder's epilogues:
 *   C[m][n] = epi(acc[m][n]),  acc = sum_k A[m][k] * W[n][k]
 *   PK_GEMM_STORE: acc;  PK_GEMM_SILU: acc * sigmoid(acc);
 *   PK_GEMM_RESIDUAL: R[m][n] + alpha * acc (R may be C);
 *   PK_GEMM_RESIDUAL_RELU: max(R[m][n] + alpha * acc, 0);
 *   PK_GEMM_BIAS: acc + bias[n].
 * A [M][K] (row stride lda), W [N][K] (ldw, an nn.Linear weight), C and R
 * [M][N] (ldc, ldr), bias [N], all bf16, 16-byte aligned, strides multiples
 * of 8; K a multiple of 64, N a multiple of 64.  Replaces the Linear -> SiLU
 * -> Linear of ConformerFeedForward (parakeet/modules/feedforward.py), the
 * residual adds of ConformerLayer.forward (parakeet/modules/encoder.py:
 * 60-81) and the joint network's enc + pred -> ReLU -> Linear
 * (parakeet/modules/decoder.py:82-86). */
#define PK_GEMM_STORE 0
#define PK_GEMM_SILU 1
#define PK_GEMM_RESIDUAL 2
#define PK_GEMM_RESIDUAL_RELU 3
#define PK_GEMM_BIAS 4
int pk_gemm_bf16(const void *A, int64_t lda, const void *W, int64_t ldw, int32_t M, int32_t N,
                 int32_t K, void *C, int64_t ldc, int32_t epilogue, const void *R, int64_t ldr,
                 const void *bias, float alpha, int32_t *error, void *stream);

/* LayerNorm over the last dimension of `rows` rows (row strides x_ld, y_ld
 * elements): y = (x - mean) / sqrt(var + eps) * gamma + beta, fp32 statistics
 * (exact two-pass).  With gamma2 != NULL the same launch also writes
 * y2 = LayerNorm(y as stored; gamma2, beta2, eps2): a ConformerLayer's
 * norm_out followed by the next layer's norm_feed_forward1.  dim = 1, 2, 4
 * or 8 x 256 (bf16) / x 128 (f32); buffers 16-byte aligned.  Replaces the
 * nn.LayerNorm calls of ConformerLayer.forward (parakeet/modules/encoder.py:
 * 60-81). */
int pk_layer_norm(const void *x, int64_t x_ld, int32_t rows, int32_t dim, const void *gamma,
                  const void *beta, float eps, void *y, int64_t y_ld, const void *gamma2,
                  const void *beta2, float eps2, void *y2, int64_t y2_ld, int32_t dtype,
                  void *stream);

/* ---------------- streaming log-mel features ------------------------------
 * The feature extractor of every stream in one launch per push.  Replaces
 * FeatureExtractor.push / _compute_features / _trim_samples
 * (parakeet/modules/feature_extractor.py:63-151), which recompute an STFT
 * over each stream's retained samples on the host at every push: here each
 * slot keeps its last PK_FE_HIST samples and two counters on the device, and
 * a push computes only the frames it emits.  Frame f of a stream covers
 * samples [f*hop - n_fft/2, f*hop + n_fft/2) after pre-emphasis (y[0] = x[0]),
 * zero outside [0, samples seen); a push emits the frames the reference's
 * push emits (every frame whose window ends inside the samples seen, or up to
 * samples_seen / hop on a final push; none on an empty push). */
#define PK_FE_HIST 512        /* samples of history kept per slot             */
#define PK_FE_META_STRIDE 4   /* int64 per slot: samples seen, frames emitted,
                                 stream epoch, CTA ticket (zero when idle)     */
#define PK_FE_FIRST 1         /* push flag: a fresh stream (counters restart)  */
#define PK_FE_FINAL 2         /* push flag: the stream's last samples (frames
                                 up to samples_seen / hop, zero-padded)        */
#define PK_DEV_BAD_COUNT 16   /* device error bit: a row's sample count outside
                                 [0, samples_ld] or more frames than max_frames */

typedef struct pk_features_desc {
    const void *tables;   /* device copy of pk_features_tables' output        */
    float *history;       /* [num_slots][PK_FE_HIST] last samples of each slot */
    int64_t *meta;        /* [num_slots][PK_FE_META_STRIDE], zeroed once       */
    int32_t *error;       /* [1] device error word (PK_DEV_* bits)            */
    int32_t num_slots;
    int32_t n_fft;        /* 512 (the only size this build handles)           */
    int32_t hop;          /* window_stride * sample_rate (160), <= n_fft      */
    int32_t n_mels;       /* <= 256                                           */
    int32_t mel_nnz;      /* nonzero filter weights, from pk_features_tables  */
    float preemph;        /* 0.97                                             */
    float dither;         /* std of the Gaussian dither added to the samples  */
    float mag_power;      /* spectrum = |X| ** mag_power (2.0)                */
    float log_guard;      /* log(mel + log_guard) (2 ** -24)                  */
    float pad_value;      /* output columns past a row's frame count          */
    uint64_t seed;        /* dither: Philox-4x32-10 key                       */
} pk_features_desc;

/* Constant tables of an extractor configuration, written to the host buffer
 * `host_out` (NULL: only report the size): the n_fft-point twiddles, the
 * symmetric Hann window of win_length samples centred in n_fft
 * (torch.hann_window(periodic=False), as torch.stft pads it), and the mel
 * filters of librosa.filters.mel(sr, n_fft, n_mels, fmin, fmax, norm) with
 * norm 1 = "slaney", 0 = none, stored by their nonzero runs.  *bytes is the
 * size, *mel_nnz the nonzero weights (the desc's mel_nnz).  Replaces the
 * constructor's tables (feature_extractor.py:46-57). */
int pk_features_tables(int32_t sample_rate, int32_t n_fft, int32_t win_length, int32_t n_mels,
                       double fmin, double fmax, int32_t mel_norm, void *host_out,
                       int64_t *bytes, int32_t *mel_nnz);

/* One push for `batch` streams: row b appends num_samples[b] float samples
 * (samples + b * samples_ld) to slot slots[b] (flags[b]: PK_FE_FIRST,
 * PK_FE_FINAL) and writes the log-mel frames it emits to out[b] ([n_mels]
 * [max_frames], `out_dtype` PK_DTYPE_*, columns past the row's count =
 * pad_value) and their count to num_frames[b].  A row with more frames than
 * max_frames keeps the first max_frames and sets PK_DEV_BAD_COUNT.  Each slot
 * appears at most once per call. */
int pk_features_push(const pk_features_desc *fe, const float *samples, int64_t samples_ld,
                     const int32_t *num_samples, const int32_t *flags, const int32_t *slots,
                     int32_t batch, void *out, int32_t out_dtype, int32_t max_frames,
                     int32_t *num_frames, void *stream);

/* Self-test of the failure path of every TMA pipeline here: the bounded
 * mbarrier wait that gives up after a time limit and records PK_DEV_TIMEOUT in
 * *error (instead of hanging the GPU), leaving the context usable.  One CTA
 * waits on an mbarrier's first phase for at most limit_ns (0 < limit_ns <=
 * 10 s); with arrive != 0 it arrives first (the wait returns at once, no error
 * bit), with arrive == 0 nothing arrives and no copy is issued, so the wait
 * runs out.  *waited_ns receives the time the wait took.  Asynchronous on
 * `stream`.  No counterpart in the reference, which has no device waits. */
int pk_selftest_bounded_wait(int32_t *error, int32_t arrive, int64_t limit_ns, int64_t *waited_ns,
                             void *stream);

/* Text of the last PK_ECUDA / PK_EINVAL cause seen by this thread. */
const char *pk_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* PK_H */
