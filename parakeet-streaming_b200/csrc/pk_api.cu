// C-ABI entry points of libpk.so (declared in include/pk.h): argument
// checks on the host, TMA descriptor encoding, kernel dispatch.
#include <cudaTypedefs.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>

#include "pk_internal.h"

namespace pk {

static thread_local char g_err[512];

void set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

int cuda_status(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return PK_OK;
    set_error("%s: %s", what, cudaGetErrorString(e));
    return PK_ECUDA;
}

static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000,
                                             cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

int encode_tmap(CUtensorMap *map, int dtype, const void *base, int rank, const uint64_t *dims,
                const uint64_t *strides_bytes, const uint32_t *box) {
    auto fn = get_encode_fn();
    if (!fn) {
        set_error("cuTensorMapEncodeTiled unavailable from the driver");
        return PK_ECUDA;
    }
    cuuint64_t d[5], st[4];
    cuuint32_t bx[5], estr[5];
    for (int i = 0; i < rank; ++i) {
        d[i] = dims[i];
        bx[i] = box[i];
        estr[i] = 1;
        if (i + 1 < rank) st[i] = strides_bytes[i];
    }
    CUresult r = fn(map, dtype == PK_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                    rank, const_cast<void *>(base), d, st, bx, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed (%d)", (int)r);
        return PK_ECUDA;
    }
    return PK_OK;
}

int encode_tmap_3d(CUtensorMap *map, int dtype, const void *base, uint64_t d0, uint64_t d1,
                   uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box0,
                   uint32_t box1, uint32_t box2) {
    const uint64_t dims[3] = {d0, d1, d2};
    const uint64_t strides[2] = {stride1_bytes, stride2_bytes};
    const uint32_t box[3] = {box0, box1, box2};
    return encode_tmap(map, dtype, base, 3, dims, strides, box);
}

}  // namespace pk

using namespace pk;

#define PK_CHECK(cond, ...)          \
    do {                             \
        if (!(cond)) {               \
            pk::set_error(__VA_ARGS__); \
            return PK_EINVAL;        \
        }                            \
    } while (0)

static bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

extern "C" {

const char *pk_last_error(void) { return pk::g_err; }

int32_t pk_pages_per_stream(int32_t left, int32_t chunk, int32_t page_size) {
    if (left < 0 || chunk <= 0 || page_size <= 0) return -1;
    const int span = left + chunk - 1;
    return (span + page_size - 1) / page_size + 1;
}

int32_t pk_ring_size(int32_t left, int32_t chunk, int32_t page_size) {
    const int n = pk_pages_per_stream(left, chunk, page_size);
    if (n <= 0) return -1;
    int r = 1;
    while (r < n) r *= 2;
    return r;
}

// Device addresses of the no-allocation entry point's static scratch array
// (g_noalloc_scratch, below), one per device, looked up on first use.
namespace {
constexpr int kNoallocMaxDevices = 64;
float *g_noalloc_ptrs[kNoallocMaxDevices] = {};
std::mutex g_noalloc_mu;

// A pool created on a device makes the next no-allocation call on that device
// look the scratch address up again.  After a device reset (cudaDeviceReset)
// the library's device code is loaded anew, at a new address, and the pools
// made before it are gone with their memory: the pools made after it renew
// the address.
void noalloc_forget(const void *dev_ptr) {
    cudaPointerAttributes attr{};
    if (cudaPointerGetAttributes(&attr, dev_ptr) != cudaSuccess) {
        (void)cudaGetLastError();
        return;
    }
    if (attr.type == cudaMemoryTypeDevice && attr.device >= 0 && attr.device < kNoallocMaxDevices) {
        std::lock_guard<std::mutex> lock(g_noalloc_mu);
        g_noalloc_ptrs[attr.device] = nullptr;
    }
}
}  // namespace

int pk_paged_kv_create(const pk_paged_kv_desc *desc, pk_paged_kv **out) {
    PK_CHECK(desc && out, "null argument");
    const pk_paged_kv_desc &d = *desc;
    PK_CHECK(d.kv && d.page_table && d.free_ring && d.ring_ctr && d.meta && d.error && d.window,
             "null device buffer in descriptor");
    PK_CHECK(d.dtype == PK_DTYPE_F32 || d.dtype == PK_DTYPE_BF16, "bad dtype %d", d.dtype);
    PK_CHECK(d.num_pages > 0 && d.num_slots > 0 && d.num_layers > 0, "empty pool");
    PK_CHECK(d.num_heads > 0 && d.dim % d.num_heads == 0, "dim %% heads != 0");
    PK_CHECK(d.left >= 0 && d.chunk > 0, "bad left/chunk");
    PK_CHECK(d.page_size >= 8 && d.page_size <= 256 && (d.page_size & (d.page_size - 1)) == 0,
             "page_size must be a power of two in [8, 256]");
    PK_CHECK(d.ring >= pk_pages_per_stream(d.left, d.chunk, d.page_size) &&
                 d.ring <= PK_WIN_MAX_PAGES && (d.ring & (d.ring - 1)) == 0,
             "ring must be a power of two in [pk_pages_per_stream(), PK_WIN_MAX_PAGES]");
    PK_CHECK(aligned16(d.window), "window descriptors not 16-byte aligned");
    PK_CHECK(aligned16(d.kv), "kv pool not 16-byte aligned");
    const int esize = d.dtype == PK_DTYPE_BF16 ? 2 : 4;
    PK_CHECK(((d.dim / d.num_heads) * esize) % 128 == 0,
             "head_dim * element size must be a multiple of 128 bytes");
    PK_CHECK(d.chunk <= 16 && d.left + d.chunk <= 128,
             "chunk must be <= 16 frames and left + chunk <= 128");
    PK_CHECK(pk_pages_per_stream(d.left, d.chunk, d.page_size) <= PK_WIN_MAX_PAGES,
             "window spans more than PK_WIN_MAX_PAGES pages");
    pk_paged_kv *kv = static_cast<pk_paged_kv *>(calloc(1, sizeof(pk_paged_kv)));
    if (!kv) return PK_EINVAL;
    kv->d = d;
    kv->esize = esize;
    kv->head_dim = d.dim / d.num_heads;
    // head-major planes: one (page, layer, K|V, head) is page_size x head_dim contiguous
    const uint64_t row = (uint64_t)kv->head_dim * esize;
    int st = encode_tmap_3d(&kv->kv_map, d.dtype, d.kv, kv->head_dim, d.page_size,
                            (uint64_t)d.num_pages * d.num_layers * 2 * d.num_heads, row,
                            row * d.page_size, 128 / esize, d.page_size, 1);
    if (st != PK_OK) {
        free(kv);
        return st;
    }
    noalloc_forget(d.kv);
    *out = kv;
    return PK_OK;
}

int pk_paged_kv_destroy(pk_paged_kv *kv) {
    free(kv);
    return PK_OK;
}

int pk_pages_reset(pk_paged_kv *kv, const int32_t *init_order, void *stream) {
    PK_CHECK(kv, "null pool");
    return launch_pages_reset(kv, init_order, static_cast<cudaStream_t>(stream));
}

int pk_pages_begin_step(pk_paged_kv *kv, const int32_t *slots, const int32_t *lengths,
                        int32_t batch, const int32_t *released, int32_t num_released,
                        void *stream) {
    PK_CHECK(kv, "null pool");
    PK_CHECK(batch >= 0 && num_released >= 0, "negative count");
    PK_CHECK(batch <= kv->d.num_slots, "batch larger than the pool's slots");
    PK_CHECK(batch == 0 || slots, "null slots");
    PK_CHECK(num_released == 0 || released, "null released");
    PK_CHECK(batch <= PK_MAX_BATCH, "batch above PK_MAX_BATCH rows");
    return launch_pages_begin(kv, slots, lengths, batch, released, num_released,
                              static_cast<cudaStream_t>(stream));
}

int pk_pages_end_step(pk_paged_kv *kv, const int32_t *slots, const int32_t *lengths,
                      int32_t batch, void *stream) {
    PK_CHECK(kv, "null pool");
    PK_CHECK(batch >= 0, "negative batch");
    PK_CHECK(batch == 0 || (slots && lengths), "null slots/lengths");
    return launch_pages_end(kv, slots, lengths, batch, static_cast<cudaStream_t>(stream));
}

int pk_append_kv(pk_paged_kv *kv, int32_t layer0, int32_t num_layers, const void *key,
                 const void *value, int64_t layer_stride, int64_t batch_stride,
                 int64_t row_stride, const int32_t *slots, int32_t batch, void *stream) {
    PK_CHECK(kv, "null pool");
    PK_CHECK(batch >= 0 && num_layers >= 0 && layer0 >= 0 &&
                 layer0 + num_layers <= kv->d.num_layers,
             "layer range [%d, %d) outside [0, %d)", layer0, layer0 + num_layers,
             kv->d.num_layers);
    if (batch == 0 || num_layers == 0) return PK_OK;
    PK_CHECK(key && value && slots, "null pointer");
    PK_CHECK(aligned16(key) && aligned16(value), "key/value not 16-byte aligned");
    const int es = kv->esize;
    PK_CHECK((layer_stride * es) % 16 == 0 && (batch_stride * es) % 16 == 0 &&
                 (row_stride * es) % 16 == 0,
             "strides must be multiples of 16 bytes");
    return launch_append(kv, layer0, num_layers, key, value, layer_stride, batch_stride,
                         row_stride, slots, batch, static_cast<cudaStream_t>(stream));
}

int pk_gather_window(pk_paged_kv *kv, int32_t layer, const int32_t *slots, int32_t batch,
                     void *k_out, void *v_out, void *stream) {
    PK_CHECK(kv, "null pool");
    PK_CHECK(layer >= 0 && layer < kv->d.num_layers, "layer out of range");
    PK_CHECK(batch >= 0, "negative batch");
    if (batch == 0) return PK_OK;
    PK_CHECK(slots && k_out && v_out, "null pointer");
    PK_CHECK(aligned16(k_out) && aligned16(v_out), "outputs not 16-byte aligned");
    return launch_gather(kv, layer, 1, slots, batch, k_out, v_out, 0,
                         static_cast<cudaStream_t>(stream));
}

int pk_gather_windows(pk_paged_kv *kv, int32_t layer0, int32_t num_layers, const int32_t *slots,
                      int32_t batch, void *k_out, void *v_out, int64_t out_layer_stride,
                      void *stream) {
    PK_CHECK(kv, "null pool");
    PK_CHECK(batch >= 0 && num_layers >= 0 && layer0 >= 0 &&
                 layer0 + num_layers <= kv->d.num_layers,
             "layer range [%d, %d) outside [0, %d)", layer0, layer0 + num_layers,
             kv->d.num_layers);
    if (batch == 0 || num_layers == 0) return PK_OK;
    PK_CHECK(slots && k_out && v_out, "null pointer");
    PK_CHECK(aligned16(k_out) && aligned16(v_out), "outputs not 16-byte aligned");
    const int64_t W = kv->d.left + kv->d.chunk;
    PK_CHECK(num_layers == 1 || out_layer_stride >= (int64_t)batch * W * kv->d.dim,
             "out_layer_stride below batch * window * dim");
    PK_CHECK((out_layer_stride * kv->esize) % 16 == 0, "out_layer_stride not 16-byte aligned");
    return launch_gather(kv, layer0, num_layers, slots, batch, k_out, v_out, out_layer_stride,
                         static_cast<cudaStream_t>(stream));
}

int pk_paged_attention(pk_paged_kv *kv, int32_t layer0, int32_t num_layers, const void *query,
                       int64_t q_layer_stride, int64_t q_batch_stride, int64_t q_row_stride,
                       const void *key, const void *value, const void *pos_proj,
                       int64_t pos_layer_stride, const void *bias_u, const void *bias_v,
                       int64_t bias_layer_stride, const int32_t *slots, const int32_t *lengths,
                       int32_t batch, void *out, int64_t out_layer_stride,
                       int64_t out_batch_stride, int64_t out_row_stride, void *stream) {
    PK_CHECK(kv, "null pool");
    PK_CHECK(batch >= 0 && num_layers >= 0 && layer0 >= 0 &&
                 layer0 + num_layers <= kv->d.num_layers,
             "layer range outside the pool");
    if (batch == 0 || num_layers == 0) return PK_OK;
    PK_CHECK(query && pos_proj && bias_u && bias_v && slots && lengths && out, "null pointer");
    PK_CHECK((key == nullptr) == (value == nullptr), "key and value go together");
    PK_CHECK(aligned16(pos_proj), "pos_proj not 16-byte aligned");
    PK_CHECK(kv->head_dim == 64 || kv->head_dim == 128, "head_dim %d not handled", kv->head_dim);
    PK_CHECK(out_row_stride % 2 == 0 && out_batch_stride % 2 == 0 && out_layer_stride % 2 == 0 &&
                 (reinterpret_cast<uintptr_t>(out) % (2 * kv->esize)) == 0,
             "out must allow 2-element stores");
    const int es = kv->esize;
    PK_CHECK(aligned16(query) && (q_row_stride * es) % 16 == 0 &&
                 (q_batch_stride * es) % 16 == 0 && (q_layer_stride * es) % 16 == 0,
             "query must be 16-byte aligned with 16-byte strides");
    PK_CHECK(!key || (aligned16(key) && aligned16(value)), "key/value not 16-byte aligned");
    const int P = 2 * (kv->d.left + kv->d.chunk) - 1;
    const int R = kv->d.left + 2 * kv->d.chunk - 1;
    const uint64_t row = (uint64_t)kv->d.dim * es;
    uint64_t lstride = (uint64_t)pos_layer_stride * es;
    if (num_layers == 1) lstride = row * P;
    PK_CHECK(lstride % 16 == 0 && lstride >= row * P, "bad pos_layer_stride");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    AttnArgs a;
    a.q = query;
    a.q_ls = q_layer_stride;
    a.q_bs = q_batch_stride;
    a.q_rs = q_row_stride;
    a.k_new = key;
    a.v_new = value;
    a.bias_u = bias_u;
    a.bias_v = bias_v;
    a.bias_ls = bias_layer_stride;
    a.pos = pos_proj;
    a.pos_ls = (int64_t)(lstride / es);
    a.pos_rows = P;
    a.bd = nullptr;
    a.slots = slots;
    a.lengths = lengths;
    a.batch = batch;
    a.out = out;
    a.o_ls = out_layer_stride;
    a.o_bs = out_batch_stride;
    a.o_rs = out_row_stride;
    a.layer0 = layer0;
    a.nlayers = num_layers;
    int st;
    CUtensorMap pos16;
    if (kv->d.dtype == PK_DTYPE_BF16) {
        // all heads of a (stream, layer) per CTA when they fill one m16 tile
        st = encode_tmap_3d(&pos16, kv->d.dtype, pos_proj, kv->d.dim, P, num_layers, row, lstride,
                            128 / es, 16, 1);
        if (st != PK_OK) return st;
        st = launch_attention_stacked(kv, pos16, a, s);
        if (st != PK_ENOTSUP) return st;
    }
    if (key) {   // the other kernels read the new rows from the pages: append first
        st = launch_append(kv, layer0, num_layers, key, value, q_layer_stride, q_batch_stride,
                           q_row_stride, slots, batch, s);
        if (st != PK_OK) return st;
        a.k_new = a.v_new = nullptr;
    }
    if (kv->d.dtype == PK_DTYPE_BF16) {
        // a group of heads per CTA when each head's chunk fills an m16 tile
        st = launch_attention_heads(kv, pos16, a, s);
        if (st != PK_ENOTSUP) return st;
    }
    CUtensorMap pos_map;
    st = encode_tmap_3d(&pos_map, kv->d.dtype, pos_proj, kv->d.dim, P, num_layers, row, lstride,
                        128 / es, R, 1);
    if (st != PK_OK) return st;
    st = launch_attention(kv, pos_map, a, s);
    if (st == PK_ENOTSUP) pk::set_error("attention configuration not handled (smem or boxes)");
    return st;
}

int32_t pk_relpos_bd_cols(const pk_paged_kv *kv) {
    return kv ? relpos_bd_cols(kv) : 0;
}

// argument checks of the rel-pos pre-pass; fills a (nothing launched)
static int relpos_args(pk_paged_kv *kv, int32_t layer0, int32_t num_layers, const void *query,
                       int64_t q_layer_stride, int64_t q_batch_stride, int64_t q_row_stride,
                       const void *pos_proj, int64_t pos_layer_stride, const void *bias_v,
                       int64_t bias_layer_stride, int32_t batch, float *bd, AttnArgs *out) {
    PK_CHECK(kv, "null pool");
    PK_CHECK(batch >= 0 && num_layers >= 0 && layer0 >= 0 &&
                 layer0 + num_layers <= kv->d.num_layers,
             "layer range outside the pool");
    PK_CHECK(relpos_bd_cols(kv) > 0, "no all-stream rel-pos pre-pass for this pool's shape");
    if (batch == 0 || num_layers == 0) return PK_OK;
    PK_CHECK(query && pos_proj && bias_v && bd, "null pointer");
    const int es = kv->esize;
    PK_CHECK(aligned16(query) && (q_row_stride * es) % 16 == 0 &&
                 (q_batch_stride * es) % 16 == 0 && (q_layer_stride * es) % 16 == 0,
             "query must be 16-byte aligned with 16-byte strides");
    PK_CHECK(aligned16(pos_proj) && aligned16(bd), "pos_proj / bd not 16-byte aligned");
    PK_CHECK((reinterpret_cast<uintptr_t>(bias_v) & 3u) == 0, "bias_v not 4-byte aligned");
    const int P = 2 * (kv->d.left + kv->d.chunk) - 1;
    const uint64_t row = (uint64_t)kv->d.dim * es;
    uint64_t lstride = (uint64_t)pos_layer_stride * es;
    if (num_layers == 1) lstride = row * P;
    PK_CHECK(lstride % 16 == 0 && lstride >= row * P, "bad pos_layer_stride");
    AttnArgs a{};
    a.q = query;
    a.q_ls = q_layer_stride;
    a.q_bs = q_batch_stride;
    a.q_rs = q_row_stride;
    a.bias_v = bias_v;
    a.bias_ls = bias_layer_stride;
    a.pos = pos_proj;
    a.pos_ls = (int64_t)(lstride / es);
    a.pos_rows = P;
    a.batch = batch;
    a.layer0 = layer0;
    a.nlayers = num_layers;
    *out = a;
    return PK_OK;
}

int pk_relpos_bd(pk_paged_kv *kv, int32_t layer0, int32_t num_layers, const void *query,
                 int64_t q_layer_stride, int64_t q_batch_stride, int64_t q_row_stride,
                 const void *pos_proj, int64_t pos_layer_stride, const void *bias_v,
                 int64_t bias_layer_stride, int32_t batch, float *bd, void *stream) {
    AttnArgs a{};
    const int st = relpos_args(kv, layer0, num_layers, query, q_layer_stride, q_batch_stride,
                               q_row_stride, pos_proj, pos_layer_stride, bias_v,
                               bias_layer_stride, batch, bd, &a);
    if (st != PK_OK || batch == 0 || num_layers == 0) return st;
    return launch_relpos_bd(kv, a, bd, static_cast<cudaStream_t>(stream));
}

int pk_pages_begin_step_relpos(pk_paged_kv *kv, const int32_t *slots, const int32_t *lengths,
                               int32_t batch, const int32_t *released, int32_t num_released,
                               int32_t layer0, int32_t num_layers, const void *query,
                               int64_t q_layer_stride, int64_t q_batch_stride,
                               int64_t q_row_stride, const void *pos_proj,
                               int64_t pos_layer_stride, const void *bias_v,
                               int64_t bias_layer_stride, float *bd, void *stream) {
    PK_CHECK(kv, "null pool");
    PK_CHECK(batch >= 0 && num_released >= 0, "negative count");
    PK_CHECK(batch <= kv->d.num_slots, "batch larger than the pool's slots");
    PK_CHECK(batch == 0 || slots, "null slots");
    PK_CHECK(num_released == 0 || released, "null released");
    PK_CHECK(batch <= PK_MAX_BATCH, "batch above PK_MAX_BATCH rows");
    AttnArgs a{};
    int st = relpos_args(kv, layer0, num_layers, query, q_layer_stride, q_batch_stride,
                         q_row_stride, pos_proj, pos_layer_stride, bias_v, bias_layer_stride,
                         batch, bd, &a);
    if (st != PK_OK) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (batch > 0 && num_layers > 0) {
        st = launch_pages_begin_relpos(kv, slots, lengths, batch, released, num_released, a, bd, s);
        if (st != PK_ENOTSUP) return st;
        // a batch too large for the one launch: the same work as two launches
        st = launch_relpos_bd(kv, a, bd, s);
        if (st != PK_OK) return st;
    }
    return launch_pages_begin(kv, slots, lengths, batch, released, num_released, s);
}

int pk_paged_attention_bd(pk_paged_kv *kv, int32_t layer0, int32_t num_layers, const void *query,
                          int64_t q_layer_stride, int64_t q_batch_stride, int64_t q_row_stride,
                          const void *key, const void *value, const float *bd,
                          const void *bias_u, int64_t bias_layer_stride, const int32_t *slots,
                          const int32_t *lengths, int32_t batch, void *out,
                          int64_t out_layer_stride, int64_t out_batch_stride,
                          int64_t out_row_stride, void *stream) {
    PK_CHECK(kv, "null pool");
    PK_CHECK(batch >= 0 && num_layers >= 0 && layer0 >= 0 &&
                 layer0 + num_layers <= kv->d.num_layers,
             "layer range outside the pool");
    PK_CHECK(relpos_bd_cols(kv) > 0, "no attention over a precomputed rel-pos term for this pool's shape");
    if (batch == 0 || num_layers == 0) return PK_OK;
    PK_CHECK(query && bd && bias_u && slots && lengths && out, "null pointer");
    PK_CHECK((key == nullptr) == (value == nullptr), "key and value go together");
    PK_CHECK(aligned16(bd), "bd not 16-byte aligned");
    PK_CHECK(out_row_stride % 2 == 0 && out_batch_stride % 2 == 0 && out_layer_stride % 2 == 0 &&
                 (reinterpret_cast<uintptr_t>(out) % (2 * kv->esize)) == 0,
             "out must allow 2-element stores");
    const int es = kv->esize;
    PK_CHECK(aligned16(query) && (q_row_stride * es) % 16 == 0 &&
                 (q_batch_stride * es) % 16 == 0 && (q_layer_stride * es) % 16 == 0,
             "query must be 16-byte aligned with 16-byte strides");
    PK_CHECK(!key || (aligned16(key) && aligned16(value)), "key/value not 16-byte aligned");
    AttnArgs a{};
    a.q = query;
    a.q_ls = q_layer_stride;
    a.q_bs = q_batch_stride;
    a.q_rs = q_row_stride;
    a.k_new = key;
    a.v_new = value;
    a.bias_u = bias_u;
    a.bias_ls = bias_layer_stride;
    a.bd = bd;
    a.slots = slots;
    a.lengths = lengths;
    a.batch = batch;
    a.out = out;
    a.o_ls = out_layer_stride;
    a.o_bs = out_batch_stride;
    a.o_rs = out_row_stride;
    a.layer0 = layer0;
    a.nlayers = num_layers;
    CUtensorMap unused{};
    return launch_attention_stacked(kv, unused, a, static_cast<cudaStream_t>(stream));
}

// Scratch of pk_paged_attention_noalloc, for callers that must not allocate
// device memory.  A file-scope device array of PK_NOALLOC_SCRATCH_BYTES:
// every GPU on which this library's code is loaded holds it until the process
// exits.  In host code its name is only a stand-in for the device copy, so
// the device address is looked up with cudaGetSymbolAddress, once per device,
// with that device current, and that address is what the kernels receive.
static __device__ __align__(256) float g_noalloc_scratch[PK_NOALLOC_SCRATCH_BYTES / sizeof(float)];

static int noalloc_scratch(float **out) {
    int dev = -1;
    int st = cuda_status(cudaGetDevice(&dev), "cudaGetDevice");
    if (st != PK_OK) return st;
    if (dev < 0 || dev >= kNoallocMaxDevices) {
        set_error("device %d above the %d the scratch table holds", dev, kNoallocMaxDevices);
        return PK_ENOTSUP;
    }
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptrs[dev]) {   // first call on this device since a pool was made: the set-up
        void *p = nullptr;
        st = cuda_status(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress");
        if (st != PK_OK) return st;
        g_noalloc_ptrs[dev] = static_cast<float *>(p);
    }
    *out = g_noalloc_ptrs[dev];
    return PK_OK;
}

int pk_paged_attention_noalloc(pk_paged_kv *kv, int32_t layer0, int32_t num_layers,
                               const void *query, int64_t q_layer_stride, int64_t q_batch_stride,
                               int64_t q_row_stride, const void *key, const void *value,
                               const void *pos_proj, int64_t pos_layer_stride, const void *bias_u,
                               const void *bias_v, int64_t bias_layer_stride,
                               const int32_t *slots, const int32_t *lengths, int32_t batch,
                               void *out, int64_t out_layer_stride, int64_t out_batch_stride,
                               int64_t out_row_stride, void *stream) {
    PK_CHECK(kv, "null pool");
    const int cols = relpos_bd_cols(kv);
    if (cols == 0 || batch <= 0 || num_layers <= 0)   // the in-kernel rel-pos term needs no scratch
        return pk_paged_attention(kv, layer0, num_layers, query, q_layer_stride, q_batch_stride,
                                  q_row_stride, key, value, pos_proj, pos_layer_stride, bias_u,
                                  bias_v, bias_layer_stride, slots, lengths, batch, out,
                                  out_layer_stride, out_batch_stride, out_row_stride, stream);
    const uint64_t need = (uint64_t)num_layers * batch * kv->d.num_heads * kv->d.chunk * cols *
                          sizeof(float);
    PK_CHECK(need <= (uint64_t)PK_NOALLOC_SCRATCH_BYTES,
             "rel-pos term of %d layers x %d streams needs %llu bytes; the static scratch "
             "holds %llu (PK_NOALLOC_SCRATCH_BYTES): split the call by layers or streams",
             num_layers, batch, (unsigned long long)need,
             (unsigned long long)PK_NOALLOC_SCRATCH_BYTES);
    // the scratch address belongs to the current device: the pool must be on it
    int dev = -1;
    cudaPointerAttributes attr{};
    int st = cuda_status(cudaGetDevice(&dev), "cudaGetDevice");
    if (st != PK_OK) return st;
    st = cuda_status(cudaPointerGetAttributes(&attr, kv->d.kv), "cudaPointerGetAttributes");
    if (st != PK_OK) return st;
    PK_CHECK(attr.type == cudaMemoryTypeDevice && attr.device == dev,
             "the pool is not on the current device (%d): make its device current first", dev);
    float *scratch = nullptr;
    st = noalloc_scratch(&scratch);
    if (st != PK_OK) return st;
    // every element the attention kernel reads is written by the pre-pass of
    // the same call, so nothing of the previous call's contents is used
    st = pk_relpos_bd(kv, layer0, num_layers, query, q_layer_stride, q_batch_stride, q_row_stride,
                      pos_proj, pos_layer_stride, bias_v, bias_layer_stride, batch, scratch, stream);
    if (st != PK_OK) return st;
    return pk_paged_attention_bd(kv, layer0, num_layers, query, q_layer_stride, q_batch_stride,
                                 q_row_stride, key, value, scratch, bias_u, bias_layer_stride,
                                 slots, lengths, batch, out, out_layer_stride, out_batch_stride,
                                 out_row_stride, stream);
}

int pk_conv_step(void *conv_state, int32_t num_slots, int32_t num_layers, int32_t layer,
                 int32_t dim, int32_t kernel, int32_t chunk, int32_t dtype, const void *x,
                 int64_t x_batch_stride, int64_t x_row_stride, const void *weight,
                 const void *ln_weight, const void *ln_bias, float ln_eps,
                 const int32_t *slots, const int32_t *lengths, int32_t batch, void *y,
                 int32_t *error, void *stream) {
    PK_CHECK(dtype == PK_DTYPE_F32 || dtype == PK_DTYPE_BF16, "bad dtype");
    PK_CHECK(layer >= 0 && layer < num_layers && num_slots > 0, "layer/slots out of range");
    PK_CHECK(batch >= 0, "negative batch");
    if (batch == 0) return PK_OK;
    PK_CHECK(conv_state && x && weight && slots && lengths && y, "null pointer");
    PK_CHECK((ln_weight == nullptr) == (ln_bias == nullptr), "ln_weight and ln_bias go together");
    const int es = dtype == PK_DTYPE_BF16 ? 2 : 4;
    PK_CHECK(dim % 4 == 0 && (reinterpret_cast<uintptr_t>(x) % (4 * es)) == 0 &&
                 (x_batch_stride % 4) == 0 && (x_row_stride % 4) == 0 &&
                 (reinterpret_cast<uintptr_t>(y) % (4 * es)) == 0,
             "x/y must allow 4-element vector access");
    ConvArgs a;
    a.state = conv_state;
    a.num_slots = num_slots;
    a.num_layers = num_layers;
    a.layer = layer;
    a.dim = dim;
    a.kernel = kernel;
    a.chunk = chunk;
    a.dtype = dtype;
    a.x = x;
    a.x_bs = x_batch_stride;
    a.x_rs = x_row_stride;
    a.w = weight;
    a.ln_w = ln_weight;
    a.ln_b = ln_bias;
    a.eps = ln_eps;
    a.slots = slots;
    a.lengths = lengths;
    a.batch = batch;
    a.y = y;
    a.error = error;
    const int vec = 16 / es;   // elements per 16-byte vector
    a.x_vec = aligned16(x) && x_batch_stride % vec == 0 && x_row_stride % vec == 0 &&
              (2 * dim) % vec == 0;
    int st = launch_conv(a, static_cast<cudaStream_t>(stream));
    if (st == PK_ENOTSUP) pk::set_error("conv configuration not handled (kernel 9, chunk <= 16)");
    return st;
}


int pk_pre_encode_window(void *cache, int32_t num_slots, const void *feats,
                         const int32_t *slots, int32_t batch, int32_t feat_in, int32_t frames,
                         int32_t csize, int32_t prefix_frames, void *out, int32_t dtype,
                         int32_t *error, void *stream) {
    PK_CHECK(dtype == PK_DTYPE_F32 || dtype == PK_DTYPE_BF16, "bad dtype %d", dtype);
    PK_CHECK(batch >= 0, "negative batch");
    if (batch == 0) return PK_OK;
    PK_CHECK(cache && feats && slots && out && num_slots > 0, "null pointer or empty pool");
    PK_CHECK(feat_in > 0 && csize > 0 && csize <= 32, "cache of 1..32 frames");
    PK_CHECK(frames > 0, "empty chunk");
    PK_CHECK(prefix_frames >= 0 && prefix_frames <= csize, "prefix_frames %d outside [0, %d]",
             prefix_frames, csize);
    return launch_pre_encode_window(cache, feats, slots, batch, feat_in, frames, csize,
                                    prefix_frames, out, dtype, error, num_slots,
                                    static_cast<cudaStream_t>(stream));
}

int pk_subsample_stage12(const void *x, int64_t x_batch_stride, int64_t x_feat_stride,
                         int64_t x_time_stride, int32_t batch, int32_t frames, int32_t feat,
                         const void *w1, const void *b1, const void *w2, const void *b2,
                         int32_t channels, int32_t first_row, void *y, int32_t dtype,
                         void *stream) {
    PK_CHECK(dtype == PK_DTYPE_F32 || dtype == PK_DTYPE_BF16, "bad dtype %d", dtype);
    PK_CHECK(batch >= 0, "negative batch");
    if (batch == 0) return PK_OK;
    PK_CHECK(x && w1 && b1 && w2 && b2 && y, "null pointer");
    PK_CHECK(frames > 0 && feat > 0 && feat <= 1024, "bad window %d x %d", frames, feat);
    PK_CHECK(channels > 0 && channels % 16 == 0, "channels %d: a multiple of 16", channels);
    const int t2 = (frames / 2 + 1) / 2 + 1;
    PK_CHECK(first_row >= 0 && first_row < t2, "first_row %d outside [0, %d)", first_row, t2);
    PK_CHECK(frames <= 4096 && batch <= 65535, "window or batch too large");
    SubsampleArgs a = {};
    a.x = x;
    a.xb = x_batch_stride;
    a.xf = x_feat_stride;
    a.xt = x_time_stride;
    a.batch = batch;
    a.frames = frames;
    a.feat = feat;
    a.channels = channels;
    a.dtype = dtype;
    a.w1 = w1;
    a.b1 = b1;
    a.w2 = w2;
    a.b2 = b2;
    a.first = first_row;
    a.y = y;
    return launch_subsample_stage12(a, static_cast<cudaStream_t>(stream));
}

int pk_subsample_dw(const void *x, int32_t batch, int32_t rows_in, int32_t first_in,
                    int32_t cols_in, const void *w, const void *b, int32_t channels,
                    int32_t first_out, void *y, int32_t dtype, void *stream) {
    PK_CHECK(dtype == PK_DTYPE_F32 || dtype == PK_DTYPE_BF16, "bad dtype %d", dtype);
    PK_CHECK(batch >= 0, "negative batch");
    if (batch == 0) return PK_OK;
    PK_CHECK(x && w && b && y, "null pointer");
    PK_CHECK(rows_in > 0 && cols_in > 0 && channels > 0, "bad shape");
    const int rows_out = rows_in / 2 + 1;
    PK_CHECK(first_out >= 0 && first_out < rows_out, "first_out %d outside [0, %d)", first_out,
             rows_out);
    const int need = 2 * first_out - 2 > 0 ? 2 * first_out - 2 : 0;
    PK_CHECK(first_in >= 0 && first_in <= need && first_in < rows_in,
             "first_in %d: rows the outputs read must be present (<= %d)", first_in, need);
    SubsampleArgs a = {};
    a.x = x;
    a.batch = batch;
    a.frames = rows_in;
    a.first = first_in;
    a.feat = cols_in;
    a.w2 = w;
    a.b2 = b;
    a.channels = channels;
    a.first_out = first_out;
    a.dtype = dtype;
    a.y = y;
    return launch_subsample_dw(a, static_cast<cudaStream_t>(stream));
}

int pk_rnnt_pick(const void *logits, int64_t logits_ld, int32_t dtype, int32_t batch,
                 int32_t num_classes, int32_t blank, const int32_t *lengths, int32_t frame,
                 int32_t symbol, int32_t max_symbols, int32_t frames, int32_t *done,
                 int32_t *emit, int64_t *ids, int32_t *tokens, int32_t *counts, void *stream) {
    PK_CHECK(dtype == PK_DTYPE_F32 || dtype == PK_DTYPE_BF16, "bad dtype %d", dtype);
    PK_CHECK(batch >= 0, "negative batch");
    if (batch == 0) return PK_OK;
    PK_CHECK(logits && lengths && done && emit && ids && tokens && counts, "null pointer");
    PK_CHECK(num_classes > 0 && logits_ld >= num_classes, "bad logits shape");
    PK_CHECK(blank >= 0 && blank < num_classes, "blank outside the classes");
    PK_CHECK(frames > 0 && frame >= 0 && frame < frames, "frame outside [0, frames)");
    PK_CHECK(max_symbols > 0 && symbol >= 0 && symbol < max_symbols,
             "symbol outside [0, max_symbols)");
    return launch_rnnt_pick(logits, logits_ld, dtype, batch, num_classes, blank, lengths, frame,
                            symbol, max_symbols, frames, done, emit, ids, tokens, counts,
                            static_cast<cudaStream_t>(stream));
}

int pk_lstm_cell(const void *gates, int64_t gates_ld, const void *xtab, int64_t xtab_ld,
                 const int64_t *ids, void *h, void *c, int64_t state_ld, const int32_t *emit,
                 int32_t batch, int32_t hidden, int32_t dtype, void *stream) {
    PK_CHECK(dtype == PK_DTYPE_F32 || dtype == PK_DTYPE_BF16, "bad dtype %d", dtype);
    PK_CHECK(batch >= 0 && hidden >= 0, "negative shape");
    if (batch == 0 || hidden == 0) return PK_OK;
    PK_CHECK(gates && h && c && emit, "null pointer");
    PK_CHECK(gates_ld >= 4 * (int64_t)hidden && state_ld >= hidden, "bad strides");
    PK_CHECK(!xtab || (ids && xtab_ld >= 4 * (int64_t)hidden), "xtab needs ids and a row stride");
    return launch_lstm_cell(gates, gates_ld, xtab, xtab_ld, ids, h, c, state_ld, emit, batch,
                            hidden, dtype, static_cast<cudaStream_t>(stream));
}

int pk_gemm_bf16(const void *A, int64_t lda, const void *W, int64_t ldw, int32_t M, int32_t N,
                 int32_t K, void *C, int64_t ldc, int32_t epilogue, const void *R, int64_t ldr,
                 const void *bias, float alpha, int32_t *error, void *stream) {
    PK_CHECK(M >= 0 && N > 0 && K > 0, "bad shape %d x %d x %d", M, N, K);
    if (M == 0) return PK_OK;
    PK_CHECK(K % 64 == 0 && N % 64 == 0, "K (%d) and N (%d) must be multiples of 64", K, N);
    PK_CHECK(epilogue >= PK_GEMM_STORE && epilogue <= PK_GEMM_BIAS, "bad epilogue %d", epilogue);
    PK_CHECK(A && W && C && error, "null pointer");
    PK_CHECK(aligned16(A) && aligned16(W) && aligned16(C), "operands must be 16-byte aligned");
    PK_CHECK(lda >= K && ldw >= K && ldc >= N && lda % 8 == 0 && ldw % 8 == 0 && ldc % 8 == 0,
             "row strides must cover the rows and be multiples of 8 elements");
    if (epilogue == PK_GEMM_RESIDUAL || epilogue == PK_GEMM_RESIDUAL_RELU)
        PK_CHECK(R && aligned16(R) && ldr >= N && ldr % 8 == 0, "bad residual operand");
    if (epilogue == PK_GEMM_BIAS) PK_CHECK(bias && aligned16(bias), "bad bias operand");
    PK_CHECK(M <= 65535 * 128, "M too large");
    GemmArgs g;
    g.A = A;
    g.W = W;
    g.lda = lda;
    g.ldw = ldw;
    g.M = M;
    g.N = N;
    g.K = K;
    g.epilogue = epilogue;
    g.C = C;
    g.ldc = ldc;
    g.R = R;
    g.ldr = ldr;
    g.bias = bias;
    g.alpha = alpha;
    g.error = error;
    return launch_gemm(g, static_cast<cudaStream_t>(stream));
}

int pk_layer_norm(const void *x, int64_t x_ld, int32_t rows, int32_t dim, const void *gamma,
                  const void *beta, float eps, void *y, int64_t y_ld, const void *gamma2,
                  const void *beta2, float eps2, void *y2, int64_t y2_ld, int32_t dtype,
                  void *stream) {
    PK_CHECK(dtype == PK_DTYPE_F32 || dtype == PK_DTYPE_BF16, "bad dtype %d", dtype);
    PK_CHECK(rows >= 0, "negative rows");
    if (rows == 0) return PK_OK;
    const int vec = dtype == PK_DTYPE_BF16 ? 8 : 4;
    const int nv = dim / (32 * vec);
    PK_CHECK(dim > 0 && dim % (32 * vec) == 0 && (nv == 1 || nv == 2 || nv == 4 || nv == 8),
             "dim %d: 1, 2, 4 or 8 x %d", dim, 32 * vec);
    PK_CHECK(x && gamma && beta && y, "null pointer");
    PK_CHECK(x_ld >= dim && y_ld >= dim && x_ld % vec == 0 && y_ld % vec == 0,
             "row strides must be >= dim and multiples of 16 bytes");
    PK_CHECK(aligned16(x) && aligned16(y) && aligned16(gamma) && aligned16(beta),
             "buffers must be 16-byte aligned");
    if (gamma2) {
        PK_CHECK(beta2 && y2 && aligned16(gamma2) && aligned16(beta2) && aligned16(y2),
                 "second LayerNorm: null or unaligned buffer");
        PK_CHECK(y2_ld >= dim && y2_ld % vec == 0, "bad y2 row stride");
    }
    LnArgs a;
    a.x = x;
    a.x_ld = x_ld;
    a.rows = rows;
    a.dim = dim;
    a.dtype = dtype;
    a.g1 = gamma;
    a.b1 = beta;
    a.eps1 = eps;
    a.y1 = y;
    a.y1_ld = y_ld;
    a.g2 = gamma2;
    a.b2 = beta2;
    a.eps2 = eps2;
    a.y2 = y2;
    a.y2_ld = y2_ld;
    return launch_layer_norm(a, static_cast<cudaStream_t>(stream));
}

int pk_features_tables(int32_t sample_rate, int32_t n_fft, int32_t win_length, int32_t n_mels,
                       double fmin, double fmax, int32_t mel_norm, void *host_out,
                       int64_t *bytes, int32_t *mel_nnz) {
    PK_CHECK(bytes && mel_nnz, "null pointer");
    PK_CHECK(sample_rate > 0, "sample rate %d", sample_rate);
    PK_CHECK(n_fft >= 2 && (n_fft & (n_fft - 1)) == 0 && n_fft <= 65536,
             "n_fft %d is not a power of two", n_fft);
    PK_CHECK(win_length >= 1 && win_length <= n_fft, "win_length %d outside [1, n_fft]",
             win_length);
    PK_CHECK(n_mels >= 1 && n_mels <= 256, "n_mels %d outside [1, 256]", n_mels);
    PK_CHECK(fmin >= 0.0 && fmax > fmin && fmax <= sample_rate / 2.0,
             "mel range [%g, %g] outside [0, sample_rate / 2]", fmin, fmax);
    PK_CHECK(mel_norm == 0 || mel_norm == 1, "mel_norm %d (0 none, 1 slaney)", mel_norm);
    int64_t words = 0;
    build_feature_tables(sample_rate, n_fft, win_length, n_mels, fmin, fmax, mel_norm, nullptr,
                         &words, mel_nnz);
    *bytes = words * (int64_t)sizeof(int32_t);
    if (!host_out) return PK_OK;
    return build_feature_tables(sample_rate, n_fft, win_length, n_mels, fmin, fmax, mel_norm,
                                static_cast<int32_t *>(host_out), &words, mel_nnz);
}

int pk_features_push(const pk_features_desc *fe, const float *samples, int64_t samples_ld,
                     const int32_t *num_samples, const int32_t *flags, const int32_t *slots,
                     int32_t batch, void *out, int32_t out_dtype, int32_t max_frames,
                     int32_t *num_frames, void *stream) {
    PK_CHECK(fe, "null descriptor");
    PK_CHECK(out_dtype == PK_DTYPE_F32 || out_dtype == PK_DTYPE_BF16, "bad dtype %d", out_dtype);
    PK_CHECK(batch >= 0 && batch <= 65535, "batch %d outside [0, 65535]", batch);
    if (batch == 0) return PK_OK;
    PK_CHECK(fe->tables && fe->history && fe->meta && fe->error && fe->num_slots > 0,
             "descriptor has a null buffer or no slots");
    if (fe->n_fft != 512) {
        set_error("n_fft %d: this build computes 512-point frames", fe->n_fft);
        return PK_ENOTSUP;
    }
    PK_CHECK(fe->hop >= 1 && fe->hop <= fe->n_fft, "hop %d outside [1, n_fft]", fe->hop);
    PK_CHECK(fe->n_mels >= 1 && fe->n_mels <= 256, "n_mels %d outside [1, 256]", fe->n_mels);
    PK_CHECK(fe->mel_nnz >= 0 && fe->mel_nnz <= fe->n_mels * (fe->n_fft / 2 + 1),
             "mel_nnz %d", fe->mel_nnz);
    PK_CHECK(num_samples && flags && slots && num_frames, "null pointer");
    PK_CHECK(samples || samples_ld == 0, "null samples with samples_ld > 0");
    PK_CHECK(samples_ld >= 0, "negative samples_ld");
    PK_CHECK(max_frames >= 0, "negative max_frames");
    PK_CHECK(max_frames == 0 || out, "null output");
    FeArgs a;
    a.tables = static_cast<const int32_t *>(fe->tables);
    a.hist = fe->history;
    a.meta = fe->meta;
    a.error = fe->error;
    a.num_slots = fe->num_slots;
    a.hop = fe->hop;
    a.n_mels = fe->n_mels;
    a.nnz = fe->mel_nnz;
    a.preemph = fe->preemph;
    a.dither = fe->dither;
    a.mag_power = fe->mag_power;
    a.guard = fe->log_guard;
    a.pad = fe->pad_value;
    a.seed_lo = (uint32_t)fe->seed;
    a.seed_hi = (uint32_t)(fe->seed >> 32);
    a.samples = samples;
    a.ld = samples_ld;
    a.nsamp = num_samples;
    a.flags = flags;
    a.slots = slots;
    a.batch = batch;
    a.out = out;
    a.out_dtype = out_dtype;
    a.max_frames = max_frames;
    a.nframes = num_frames;
    return launch_features(a, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

int pk_selftest_bounded_wait(int32_t *error, int32_t arrive, int64_t limit_ns, int64_t *waited_ns,
                             void *stream) {
    PK_CHECK(error && waited_ns, "null argument");
    PK_CHECK(limit_ns > 0 && limit_ns <= 10ll * 1000 * 1000 * 1000, "limit_ns must be in (0, 10 s]");
    return pk::launch_selftest_wait(error, arrive, static_cast<uint64_t>(limit_ns), waited_ns,
                                    static_cast<cudaStream_t>(stream));
}
