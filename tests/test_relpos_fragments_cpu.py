"""Index math of the rel-pos term's tensor-core fragments (csrc/pk_relpos.cuh),
checked on the CPU.  The kernels permute the k index of mma.m16n8k16 alike in
both operands so that lane (gq, tq) loads columns [16 tq, 16 tq + 16) of its
rows as 32 contiguous bytes: logical k = 16 ks + 2 tq + 8 half + e sits in
column 16 tq + 4 ks + 2 half + e.  Rebuilding the logical A (16 x 16) and B
(16 x 8) tiles of each k-step from what every lane holds, in the PTX fragment
layout, must give X P^T over the 64 columns: every column used once."""
import numpy as np


def _tiles(X, P):
    """Logical A_ks [16, 16] and B_ks [16, 8] of the four k-steps, from the
    registers each lane holds (words 2 ks and 2 ks + 1 of its 32 bytes)."""
    A = np.full((4, 16, 16), np.nan)
    B = np.full((4, 16, 8), np.nan)
    for lane in range(32):
        gq, tq = lane // 4, lane % 4
        for ks in range(4):
            for half in range(2):
                for e in range(2):
                    col = 16 * tq + 4 * ks + 2 * half + e   # column the lane loaded
                    k = 2 * tq + 8 * half + e                 # its place in the k-step
                    # a0/a2 (row gq), a1/a3 (row gq + 8); b0/b1 (n = gq)
                    A[ks, gq, k] = X[gq, col]
                    A[ks, gq + 8, k] = X[gq + 8, col]
                    B[ks, k, gq] = P[gq, col]
    return A, B


def test_permuted_fragments_give_the_plain_product():
    rng = np.random.default_rng(0)
    X, P = rng.standard_normal((16, 64)), rng.standard_normal((8, 64))
    A, B = _tiles(X, P)
    assert not np.isnan(A).any() and not np.isnan(B).any()   # every fragment slot filled
    C = sum(A[ks] @ B[ks] for ks in range(4))
    np.testing.assert_allclose(C, X @ P.T, rtol=1e-12, atol=1e-12)


def test_each_lane_reads_one_contiguous_32_byte_run():
    for lane in range(32):
        tq = lane % 4
        cols = sorted(16 * tq + 4 * ks + 2 * half + e
                      for ks in range(4) for half in range(2) for e in range(2))
        assert cols == list(range(16 * tq, 16 * tq + 16))   # 16 bf16 = 32 bytes, 16-byte aligned
