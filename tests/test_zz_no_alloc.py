"""pk_paged_attention_noalloc (C ABI): the rel-pos pre-pass into the
library's static device scratch, then attention over it.  Over two calls
(two steps of the same streams) it gives the output of the existing entry
point pk_paged_attention bit for bit, with no change in free device memory,
and it refuses a step whose rel-pos term exceeds the static scratch."""
import numpy as np
import pytest
import torch

from oracle import pages
from parakeet_b200 import _lib
from parakeet_b200.ops import PagedKVPool

pytestmark = pytest.mark.gpu
DEV = "cuda"
ATT, D, H, L = (70, 1), 512, 8, 17


def _inputs(rng, nl, B, T, P):
    to = lambda a: torch.tensor(np.asarray(a), dtype=torch.bfloat16, device=DEV)  # noqa: E731
    pos = to(rng.standard_normal((nl, P, D)) / 8)
    bu = to(rng.standard_normal((nl, H, D // H)) / 8)
    bv = to(rng.standard_normal((nl, H, D // H)) / 8)
    return to, pos, bu, bv


def test_noalloc_equals_paged_attention_over_two_calls():
    left, T = ATT[0], ATT[1] + 1
    P, n_slots = 2 * (left + T) - 1, 6
    rng = np.random.default_rng(5)
    order = rng.permutation(n_slots * pages.pages_per_stream(left, T, 16))
    ref, new = (PagedKVPool(L, D, H, ATT, n_slots, dtype=torch.bfloat16, device=DEV, page_order=order)
                for _ in range(2))
    assert new.relpos_bd_cols > 0   # the pre-pass (scratch) path runs, not the fallback
    to, pos, bu, bv = _inputs(rng, L, n_slots, T, P)
    slots = torch.tensor([3, 0, 5, 1], dtype=torch.int32, device=DEV)
    B = slots.numel()
    ln = torch.full((B,), T, dtype=torch.int32, device=DEV)
    out_ref = torch.empty(L, B, T, D, dtype=torch.bfloat16, device=DEV)
    out_new = torch.empty_like(out_ref)
    qkvs = [to(rng.standard_normal((L, B, T, 3 * D)) / 8) for _ in range(3)]

    def call(pool, qkv, out, noalloc):
        pool.begin_step(slots, ln)
        pool.attention(0, qkv[..., :D], pos, bu, bv, slots, ln, out, key=qkv[..., D:2 * D],
                       value=qkv[..., 2 * D:], noalloc=noalloc)
        pool.end_step(slots, ln)

    call(ref, qkvs[0], out_ref, False)   # first call: loads the scratch's module
    call(new, qkvs[0], out_new, True)
    torch.cuda.synchronize()
    assert torch.equal(out_ref, out_new)
    free0 = torch.cuda.mem_get_info()[0]
    for qkv in qkvs[1:]:                 # two more calls each, compared call by call
        call(ref, qkv, out_ref, False)
        call(new, qkv, out_new, True)
        torch.cuda.synchronize()
        assert torch.equal(out_ref, out_new)
    assert torch.cuda.mem_get_info()[0] == free0
    assert ref.read_error() == 0 and new.read_error() == 0


def test_noalloc_refuses_a_term_above_the_static_scratch():
    left, T = ATT[0], ATT[1] + 1
    P = 2 * (left + T) - 1
    limit = int(_lib.lib().pk_relpos_scratch_bytes())
    pool = PagedKVPool(L, D, H, ATT, 1, num_pages=8, dtype=torch.bfloat16, device=DEV)
    per_stream = L * H * T * pool.relpos_bd_cols * 4
    B = limit // per_stream + 1          # one stream more than the scratch holds
    rng = np.random.default_rng(6)
    _, pos, bu, bv = _inputs(rng, L, B, T, P)
    q = torch.zeros(L, B, T, D, dtype=torch.bfloat16, device=DEV)
    slots = torch.zeros(B, dtype=torch.int32, device=DEV)
    ln = torch.full((B,), T, dtype=torch.int32, device=DEV)
    with pytest.raises(_lib.PKError, match="static scratch"):
        pool.attention(0, q, pos, bu, bv, slots, ln, noalloc=True)
    torch.cuda.synchronize()
    assert pool.read_error() == 0


@pytest.mark.parametrize("dtype,att,dim", [(torch.float32, (70, 1), 512),
                                           (torch.bfloat16, (70, 13), 1024)])
def test_shapes_without_prepass(dtype, att, dim):
    """fp32 pools and the large shape have no pre-pass: relpos_bd_cols is 0,
    relpos_bd raises, and the no-allocation entry point runs pk_paged_attention
    itself (identical output on identical pools)."""
    left, T = att[0], att[1] + 1
    P, n_slots, nl = 2 * (left + T) - 1, 3, 2
    rng = np.random.default_rng(8)
    order = rng.permutation(n_slots * pages.pages_per_stream(left, T, 16))
    a, b = (PagedKVPool(nl, dim, H, att, n_slots, dtype=dtype, device=DEV, page_order=order)
            for _ in range(2))
    assert a.relpos_bd_cols == 0
    to = lambda x: torch.tensor(np.asarray(x), dtype=dtype, device=DEV)  # noqa: E731
    pos = to(rng.standard_normal((nl, P, dim)) / 8)
    bu, bv = to(rng.standard_normal((nl, H, dim // H)) / 8), to(rng.standard_normal((nl, H, dim // H)) / 8)
    slots = torch.tensor([2, 0], dtype=torch.int32, device=DEV)
    ln = torch.full((2,), T, dtype=torch.int32, device=DEV)
    qkv = to(rng.standard_normal((nl, 2, T, 3 * dim)) / 8)
    q, k, v = qkv[..., :dim], qkv[..., dim:2 * dim], qkv[..., 2 * dim:]
    with pytest.raises(_lib.PKError):
        a.relpos_bd(0, q, pos, bv)
    outs = []
    for pool, noalloc in ((a, False), (b, True)):
        pool.begin_step(slots, ln)
        outs.append(pool.attention(0, q, pos, bu, bv, slots, ln, key=k, value=v, noalloc=noalloc))
        pool.end_step(slots, ln)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])
    assert a.read_error() == 0 and b.read_error() == 0
