// The rel-pos term of the attention logits, BD = bf16(q + pos_bias_v) P^T
// (ConformerAttention.forward lines 108-110, parakeet/modules/attention.py,
// before rel_shift), on tensor cores with P (the layer's linear_pos rows) read
// straight from global memory.  Shared by the stacked attention kernel (the term
// of its own CTA) and by the all-stream pre-pass, which runs either alone
// (pk_relpos_bd) or in the step-start launch (pk_pages_begin_step_relpos), so
// that every form gives the same values bit for bit.
#pragma once

#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {
namespace {

__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// ---- rel-pos term BD = bf16(q + v) P^T on tensor cores, P (the layer's
// linear_pos rows) read straight from global memory.  The MMA's k index is
// permuted alike in both operands (a sum over k does not depend on its order)
// so that each lane's A and B fragments are the 32 contiguous bytes
// [16 tq, 16 tq + 16) of a row: logical k = 16 ks + 2 tq + 8 half + e sits in
// column 16 tq + 4 ks + 2 half + e.  The attention kernel and the all-stream
// pre-pass both use these two helpers, so their BD values are identical.

// One query row's A-fragment words: bf16(q + v) at columns [16 tq, 16 tq + 16)
// (q_row and bias_v2 already offset by the head and by 16 tq); zeros without q_row.
__device__ __forceinline__ void bd_a_words(const __nv_bfloat16 *q_row,
                                           const __nv_bfloat162 *bias_v2, uint32_t (&x)[8]) {
    uint4 q0 = make_uint4(0, 0, 0, 0), q1 = q0;
    if (q_row) {
        q0 = reinterpret_cast<const uint4 *>(q_row)[0];
        q1 = reinterpret_cast<const uint4 *>(q_row)[1];
    }
    const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        uint32_t xv = 0u;
        if (q_row) {
            const float2 q = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&qw[j]));
            const float2 v = __bfloat1622float2(__ldg(bias_v2 + j));
            __nv_bfloat162 t2 = __floats2bfloat162_rn(q.x + v.x, q.y + v.y);
            xv = *reinterpret_cast<uint32_t *>(&t2);
        }
        x[j] = xv;
    }
}

// n-tiles (8 rel-pos rows) whose B fragments one batch of loads brings in
// (5: half of the small config's 10, within the attention kernel's registers;
// the pre-pass gives each warp half of the n-tiles)
constexpr int kBdBatch = 5;

// BD of the m16 tile's rows gq (xa) and gq + 8 (xb) against rel-pos rows
// [0, 8 * ntiles) (rows >= pos_rows read as zero); p_base = the layer's P at
// row 0, offset by the head and by 16 tq, rows dim elements apart.
// store(nt, c) receives n-tile nt's accumulators (row gq: c[0..1], row gq + 8:
// c[2..3], columns nt * 8 + 2 tq + {0, 1}).
// B fragments of n-tiles [nt0, nt0 + NB) (those < ntiles) into pw
template <int NB>
__device__ __forceinline__ void bd_load_p(uint4 (&pw)[NB][2], const __nv_bfloat16 *p_base, int dim,
                                          int pos_rows, int nt0, int ntiles, int gq) {
#pragma unroll
    for (int i = 0; i < NB; ++i) {
        const int r = (nt0 + i) * 8 + gq;
        pw[i][0] = pw[i][1] = make_uint4(0, 0, 0, 0);
        if (nt0 + i < ntiles && r < pos_rows) {
            const uint4 *src = reinterpret_cast<const uint4 *>(p_base + (int64_t)r * dim);
            pw[i][0] = __ldg(src);
            pw[i][1] = __ldg(src + 1);
        }
    }
}

// the MMAs of those n-tiles, k-steps in order, each n-tile's result to store
template <int NB, class Store>
__device__ __forceinline__ void bd_mma_p(const uint4 (&pw)[NB][2], const uint32_t (&xa)[8],
                                         const uint32_t (&xb)[8], int nt0, int ntiles, Store store) {
#pragma unroll
    for (int i = 0; i < NB; ++i) {
        if (nt0 + i >= ntiles) break;
        const uint32_t pv[8] = {pw[i][0].x, pw[i][0].y, pw[i][0].z, pw[i][0].w,
                                pw[i][1].x, pw[i][1].y, pw[i][1].z, pw[i][1].w};
        float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
            const uint32_t af[4] = {xa[2 * ks], xb[2 * ks], xa[2 * ks + 1], xb[2 * ks + 1]};
            mma_bf16(c, af, pv[2 * ks], pv[2 * ks + 1]);
        }
        store(nt0 + i, c);
    }
}

template <int NB, class Store>
__device__ __forceinline__ void bd_tile(const uint32_t (&xa)[8], const uint32_t (&xb)[8],
                                        const __nv_bfloat16 *p_base, int dim, int pos_rows,
                                        int ntiles, int gq, Store store) {
    for (int nt0 = 0; nt0 < ntiles; nt0 += NB) {
        uint4 pw[NB][2];
        bd_load_p<NB>(pw, p_base, dim, pos_rows, nt0, ntiles, gq);
        bd_mma_p<NB>(pw, xa, xb, nt0, ntiles, store);
    }
}


// rows per pre-pass tile: 4 warps, two per 16-row m16 tile (each half of the n-tiles)
constexpr int kRelposThreads = 128;
constexpr int kRelposRows = 32;

// One pre-pass tile: BD of the (stream, query) rows [32 z + 16 (w / 2), +16) of
// layer lrel, head hh, for warp w against the first (w even) or second half of
// the rel-pos n-tiles; out [layer][batch][heads][chunk][bds].  Every stream of a
// layer uses the same rel-pos rows, which a tile reads once for 16 rows instead
// of once per (stream, head group) as the attention kernel would.
__device__ __forceinline__ void relpos_tile(const pk_paged_kv_desc &d, const AttnArgs &a, int bds,
                                            float *bd, int lrel, int hh, int z) {
    using T = __nv_bfloat16;
    const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
    if (warp >= kRelposThreads / 32) return;
    const int gq = lane / 4, tq = lane % 4;
    const int chunk = d.chunk, rows = a.batch * chunk;
    const int m0 = z * kRelposRows + (warp >> 1) * 16;
    const int nt_all = bds / 8, nt_half = (nt_all + 1) / 2;
    const int nt_begin = (warp & 1) ? nt_half : 0;
    const int nt_count = (warp & 1) ? nt_all - nt_half : nt_half;   // <= kBdBatch (launch check)
    if (m0 >= rows) return;
    // the rel-pos rows first: their loads do not wait for the query arithmetic
    const T *p_base = static_cast<const T *>(a.pos) + (int64_t)lrel * a.pos_ls +
                      (int64_t)nt_begin * 8 * d.dim + hh * 64 + 16 * tq;
    const int p_rows = a.pos_rows - nt_begin * 8;
    uint4 pw[kBdBatch][2];
    bd_load_p<kBdBatch>(pw, p_base, d.dim, p_rows, 0, nt_count, gq);
    const __nv_bfloat162 *bv2 = reinterpret_cast<const __nv_bfloat162 *>(
        static_cast<const T *>(a.bias_v) + (int64_t)lrel * a.bias_ls + hh * 64 + 16 * tq);
    // rows gq and gq + 8 of the tile: their query rows and their BD output rows
    const T *qr[2] = {nullptr, nullptr};
    float *orow[2] = {nullptr, nullptr};
#pragma unroll
    for (int rh = 0; rh < 2; ++rh) {
        const int m = m0 + gq + 8 * rh;
        if (m < rows) {
            const int b = m / chunk, t = m - b * chunk;
            qr[rh] = static_cast<const T *>(a.q) + (int64_t)lrel * a.q_ls + (int64_t)b * a.q_bs +
                     (int64_t)t * a.q_rs + hh * 64 + 16 * tq;
            orow[rh] = bd + (((int64_t)lrel * a.batch + b) * d.num_heads + hh) * chunk * bds +
                       (int64_t)t * bds + nt_begin * 8 + 2 * tq;
        }
    }
    uint32_t xa[8], xb[8];
    bd_a_words(qr[0], bv2, xa);
    bd_a_words(qr[1], bv2, xb);
    bd_mma_p<kBdBatch>(pw, xa, xb, 0, nt_count, [&](int nt, const float (&c)[4]) {
        if (orow[0]) *reinterpret_cast<float2 *>(orow[0] + nt * 8) = make_float2(c[0], c[1]);
        if (orow[1]) *reinterpret_cast<float2 *>(orow[1] + nt * 8) = make_float2(c[2], c[3]);
    });
}

}  // namespace
}  // namespace pk
