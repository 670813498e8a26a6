"""The attention entry point that allocates no device memory.

Some callers of this library cannot allocate: a host whose device memory is
all reserved up front by another allocator (a framework's caching pool, a
per-process memory cap), or a serving loop that must not call cudaMalloc /
cudaFree because they can block and synchronise the device.  For them
pk_paged_attention_noalloc runs the rel-pos pre-pass into the library's one
static device array instead of a caller buffer.  These tests call it through
the C ABI and check, on calls in a row over the same streams, that its output
matches the existing entry point pk_paged_attention within the bf16 tolerance
of the other attention tests (it is in fact identical), that torch's allocator
sees nothing allocated by the call, and that a step too large for the static
array is refused with a clear error.  This file is collected last."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import pages
from parakeet_b200 import _lib
from parakeet_b200.ops import PagedKVPool, _stream
from replay import rel_l2

pytestmark = pytest.mark.gpu
DEV = "cuda"
ATT, D, H, L = (70, 1), 512, 8, 17
TOL_BF16 = 1e-2


def _inputs(rng, nl, B, T, P):
    to = lambda a: torch.tensor(np.asarray(a), dtype=torch.bfloat16, device=DEV)  # noqa: E731
    pos = to(rng.standard_normal((nl, P, D)) / 8)
    bu = to(rng.standard_normal((nl, H, D // H)) / 8)
    bv = to(rng.standard_normal((nl, H, D // H)) / 8)
    return to, pos, bu, bv


def _noalloc(pool, q, k, v, pos, bu, bv, slots, ln, out):
    """pk_paged_attention_noalloc straight through ctypes (all layers of q)."""
    nl, B = q.shape[:2]
    return _lib.lib().pk_paged_attention_noalloc(
        pool._h, 0, nl, q.data_ptr(), q.stride(0), q.stride(1), q.stride(2),
        k.data_ptr(), v.data_ptr(), pos.data_ptr(), pos.stride(0), bu.data_ptr(), bv.data_ptr(),
        bu.stride(0), slots.data_ptr(), ln.data_ptr(), B, out.data_ptr(), out.stride(0),
        out.stride(1), out.stride(2), ctypes.c_void_p(_stream(pool.device)))


def test_noalloc_matches_paged_attention_on_calls_in_a_row():
    left, T = ATT[0], ATT[1] + 1
    P, n_slots = 2 * (left + T) - 1, 6
    rng = np.random.default_rng(5)
    order = rng.permutation(n_slots * pages.pages_per_stream(left, T, 16))
    ref, new = (PagedKVPool(L, D, H, ATT, n_slots, dtype=torch.bfloat16, device=DEV, page_order=order)
                for _ in range(2))
    assert new.relpos_bd_cols > 0   # the static-scratch path runs, not the fallback
    to, pos, bu, bv = _inputs(rng, L, n_slots, T, P)
    slots = torch.tensor([3, 0, 5, 1], dtype=torch.int32, device=DEV)
    B = slots.numel()
    ln = torch.full((B,), T, dtype=torch.int32, device=DEV)
    out_ref = torch.empty(L, B, T, D, dtype=torch.bfloat16, device=DEV)
    out_new = torch.empty_like(out_ref)
    for call in range(3):   # the first call on the device also looks up the array's address
        qkv = to(rng.standard_normal((L, B, T, 3 * D)) / 8)
        q, k, v = qkv[..., :D], qkv[..., D:2 * D], qkv[..., 2 * D:]
        ref.begin_step(slots, ln)
        ref.attention(0, q, pos, bu, bv, slots, ln, out_ref, key=k, value=v)
        ref.end_step(slots, ln)
        new.begin_step(slots, ln)
        torch.cuda.synchronize()
        before = (torch.cuda.memory_allocated(), torch.cuda.memory_reserved())
        _lib.check(_noalloc(new, q, k, v, pos, bu, bv, slots, ln, out_new),
                   "pk_paged_attention_noalloc")
        assert (torch.cuda.memory_allocated(), torch.cuda.memory_reserved()) == before
        new.end_step(slots, ln)
        torch.cuda.synchronize()
        got, want = out_new.float().cpu().numpy(), out_ref.float().cpu().numpy()
        assert rel_l2(got, want) <= TOL_BF16, call
        assert torch.equal(out_new, out_ref), call
    assert ref.read_error() == 0 and new.read_error() == 0


def test_noalloc_refuses_a_term_above_the_static_scratch():
    left, T = ATT[0], ATT[1] + 1
    P = 2 * (left + T) - 1
    pool = PagedKVPool(L, D, H, ATT, 1, num_pages=8, dtype=torch.bfloat16, device=DEV)
    per_stream = L * H * T * pool.relpos_bd_cols * 4
    B = _lib.PK_NOALLOC_SCRATCH_BYTES // per_stream + 1   # one stream more than the array holds
    rng = np.random.default_rng(6)
    _, pos, bu, bv = _inputs(rng, L, B, T, P)
    q = torch.zeros(L, B, T, D, dtype=torch.bfloat16, device=DEV)
    out = torch.empty_like(q)
    slots = torch.zeros(B, dtype=torch.int32, device=DEV)
    ln = torch.full((B,), T, dtype=torch.int32, device=DEV)
    st = _noalloc(pool, q, q, q, pos, bu, bv, slots, ln, out)
    assert st == _lib.PK_EINVAL
    assert "static scratch" in _lib.lib().pk_last_error().decode()
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
    outs = [torch.empty(nl, 2, T, dim, dtype=dtype, device=DEV) for _ in range(2)]
    with pytest.raises(ValueError):       # allocating nothing: the caller passes `out`
        b.attention(0, q, pos, bu, bv, slots, ln, key=k, value=v, noalloc=True)
    for pool, noalloc, out in ((a, False, outs[0]), (b, True, outs[1])):
        pool.begin_step(slots, ln)
        pool.attention(0, q, pos, bu, bv, slots, ln, key=k, value=v, noalloc=noalloc, out=out)
        pool.end_step(slots, ln)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])
    assert a.read_error() == 0 and b.read_error() == 0
