"""Parity of the libpk kernels (called through the C ABI) with the CPU oracle.

Page allocator: op-for-op equal to oracle.pages.PagePoolModel (page table,
free ring order, counters).  Append + gather: bit-exact against the oracle's
dense window, which equals the reference's (test_oracle_golden).  Attention
and conv step: rel-L2 against the float64 oracle on valid rows, <= 1e-5 in
fp32 and <= 1e-2 in bf16."""
import numpy as np
import pytest
import torch

from oracle import pages, streaming
from parakeet_b200 import _lib
from parakeet_b200.engine.scheduler import SlotAllocator
from parakeet_b200.ops import PagedKVPool
from replay import rel_l2

pytestmark = pytest.mark.gpu

DEV = "cuda"
TOL = {torch.float32: 1e-5, torch.bfloat16: 1e-2}
SHAPES = {"small": dict(att=(70, 1), dim=512, heads=8), "large": dict(att=(70, 13), dim=1024, heads=8),
          # head_dim 64 with chunks of 3 and 4 frames: 12 and 16 stacked query rows of
          # the 4-head CTA (the small model stacks 8)
          "small_t3": dict(att=(70, 2), dim=512, heads=8), "small_t4": dict(att=(70, 3), dim=512, heads=8),
          # the conv-cache step's register form at the large width, and a 1-frame chunk
          "wide_t2": dict(att=(70, 1), dim=1024, heads=8), "small_t1": dict(att=(70, 0), dim=512, heads=8),
          # pages of 8 frames (10 boxes per window; odd box counts at some alignments)
          "small_p8": dict(att=(70, 1), dim=512, heads=8, page=8),
          "small_t3_p8": dict(att=(70, 2), dim=512, heads=8, page=8),
          # the large model over 8-frame pages (the general bf16 kernel)
          "large_p8": dict(att=(70, 13), dim=1024, heads=8, page=8)}


def pool_state(pool):
    torch.cuda.synchronize()
    head, tail = pool.ring_ctr.tolist()
    ring = pool.free_ring.cpu().numpy()
    free = [int(ring[i % pool.num_pages]) for i in range(head, tail)]
    return pool.page_table.cpu().numpy(), pool.meta.cpu().numpy(), free


def assert_pool_equals_model(pool, model):
    table, meta, free = pool_state(pool)
    assert np.array_equal(table, model.table)
    assert np.array_equal(meta[:, _lib.META_FIRST], model.first)
    assert np.array_equal(meta[:, _lib.META_NEXT], model.next)
    assert np.array_equal(meta[:, _lib.META_WRITTEN], model.written)
    assert np.array_equal(meta[:, _lib.META_PROCESSED], model.processed)
    assert np.array_equal(meta[:, _lib.META_CACHE_LEN], model.cache_len)
    assert free == list(model.free)


@pytest.mark.parametrize("att,cap,n_slots,arrivals,steps", [((70, 1), 0.6, 24, 4, 160),
                                                            ((70, 13), 0.6, 24, 4, 160),
                                                            ((70, 1), 1.0, 24, 4, 160),
                                                            ((70, 1), 0.8, 1100, 120, 160),
                                                            ((70, 1), 1.0, 6144, 1200, 64)])
def test_page_allocator_matches_cpu_model(att, cap, n_slots, arrivals, steps):
    """Device allocator vs the CPU model, op for op; the 1100-slot case runs
    batches above 1024 rows (two rows per thread of the step-start CTA), the
    6144-slot case batches above 2048 rows (page-table rings read in place, up
    to six rows per thread)."""
    rng = np.random.default_rng(7)
    left, T, ps = att[0], att[1] + 1, 16
    per = pages.pages_per_stream(left, T, ps)
    n_pages = int(cap * n_slots * per)
    order = np.random.default_rng(1).permutation(n_pages)
    pool = PagedKVPool(1, 128, 2, att, n_slots, num_pages=n_pages, dtype=torch.float32,
                       device=DEV, page_order=order)
    model = pages.PagePoolModel(n_pages, n_slots, left, T, ps, init_order=order)
    alloc = SlotAllocator(n_slots, per, n_pages)
    live = []
    for step in range(steps):
        for _ in range(int(rng.integers(0, 3))):
            if live and rng.random() < 0.3:
                s = live.pop(int(rng.integers(len(live))))
                alloc.release(s)
                pool.release_slot(s)
                model.release_slot(s)
        for _ in range(int(rng.integers(0, arrivals))):
            s = alloc.acquire()
            if s is not None:
                live.append(s)
        batch = [s for s in live if rng.random() < 0.85]
        lengths = [T if rng.random() < 0.9 else int(rng.integers(1, T + 1)) for _ in batch]
        sl = torch.tensor(batch, dtype=torch.int32, device=DEV)
        ln = torch.tensor(lengths, dtype=torch.int32, device=DEV)
        assert model.begin_step(batch)
        pool.begin_step(sl, ln)
        model.end_step(batch, lengths)
        pool.end_step(sl, ln)
        if step % 8 == 0 or step > steps - 10:
            assert_pool_equals_model(pool, model)
    assert pool.read_error() == 0
    assert_pool_equals_model(pool, model)


def test_append_gather_above_2048_rows_matches_model():
    """Steps of 2600 rows (the step-start CTA's global-ring form): the window
    descriptors it writes drive the append and gather, bit-exact against the
    CPU page model's pool contents."""
    att, n_slots, D, steps = (70, 1), 2600, 128, 48
    left, T, ps = att[0], att[1] + 1, 16
    rng = np.random.default_rng(11)
    n_pages = n_slots * pages.pages_per_stream(left, T, ps)
    order = rng.permutation(n_pages)
    pool = PagedKVPool(1, D, 2, att, n_slots, num_pages=n_pages, dtype=torch.float32,
                       device=DEV, page_order=order)
    model = pages.PagedKVModel(pages.PagePoolModel(n_pages, n_slots, left, T, ps, init_order=order),
                               1, D, dtype=np.float32)
    start = np.where(np.arange(n_slots) < 2200, 0, rng.integers(1, 8, n_slots))
    for step in range(steps):
        batch = [int(s) for s in rng.permutation(n_slots) if start[s] <= step]
        sl = torch.tensor(batch, dtype=torch.int32, device=DEV)
        ln = torch.full((len(batch),), T, dtype=torch.int32, device=DEV)
        k = rng.standard_normal((len(batch), T, D)).astype(np.float32)
        v = rng.standard_normal((len(batch), T, D)).astype(np.float32)
        assert model.pool.begin_step(batch)
        pool.begin_step(sl, ln)
        model.append(0, batch, k, v)
        pool.append(0, torch.from_numpy(k).to(DEV), torch.from_numpy(v).to(DEV), sl)
        if step % 12 == 11 or step == steps - 1:
            kw, vw = pool.gather(0, sl)
            km, vm = model.gather(0, batch)
            assert np.array_equal(kw.cpu().numpy(), km), step
            assert np.array_equal(vw.cpu().numpy(), vm), step
        model.pool.end_step(batch, [T] * len(batch))
        pool.end_step(sl, ln)
    assert pool.read_error() == 0
    assert_pool_equals_model(pool, model.pool)


def test_pool_exhaustion_sets_error_bit_and_allocates_nothing():
    pool = PagedKVPool(1, 128, 2, (70, 1), 4, num_pages=2, dtype=torch.float32, device=DEV)
    sl = torch.tensor([0, 1, 2], dtype=torch.int32, device=DEV)
    pool.begin_step(sl)
    torch.cuda.synchronize()
    assert pool.read_error() & _lib.PK_DEV_POOL_EXHAUSTED
    assert (pool.page_table == -1).all()
    assert pool.ring_ctr.tolist() == [0, 2]


def run_stream_steps(shape, dtype, steps, n_slots, seed, check_every=1, short_last=True,
                     fused=False, prepass=False):
    """Staggered streams through append + gather + attention, against the
    oracle's dense slot pool (pack -> update_attn_cache -> unpack) and masks.
    prepass: the rel-pos term comes from the all-stream pre-pass (relpos_bd)."""
    cfg = SHAPES[shape]
    att, D, H = cfg["att"], cfg["dim"], cfg["heads"]
    left, T = att[0], att[1] + 1
    W, P, L = left + T, 2 * (left + T) - 1, 2
    ps = cfg.get("page", 16)
    rng = np.random.default_rng(seed)
    order = rng.permutation(n_slots * pages.pages_per_stream(left, T, ps))
    pool = PagedKVPool(L, D, H, att, n_slots, page_size=ps, dtype=dtype, device=DEV,
                       page_order=order)
    dense = streaming.SlotSchedulerModel(L, att, D, 9, n_slots)
    start = {s: int(rng.integers(0, steps // 2)) if s else 0 for s in range(n_slots)}
    pos = [rng.standard_normal((P, D)) / 8 for _ in range(L)]
    bu = [rng.standard_normal((H, D // H)) / 8 for _ in range(L)]
    bv = [rng.standard_normal((H, D // H)) / 8 for _ in range(L)]
    to = lambda a: torch.tensor(np.asarray(a), dtype=dtype, device=DEV)  # noqa: E731
    rd = lambda t: t.float().cpu().numpy().astype(np.float64)  # noqa: E731
    pos_t, bu_t, bv_t = [to(p) for p in pos], [to(b) for b in bu], [to(b) for b in bv]
    pos_r, bu_r, bv_r = [rd(t) for t in pos_t], [rd(t) for t in bu_t], [rd(t) for t in bv_t]
    worst = 0.0
    for step in range(steps):
        batch = [s for s in range(n_slots) if start[s] <= step]
        lengths = [T] * len(batch)
        if short_last and step == steps - 1:
            lengths[-1] = max(1, T // 2)
        sl = torch.tensor(batch, dtype=torch.int32, device=DEV)
        ln = torch.tensor(lengths, dtype=torch.int32, device=DEV)
        pool.begin_step(sl, ln)
        st, idx = dense.pack_states(batch)
        _, mask = streaming.streaming_masks(T, st.cache_lengths, st.processed_frames, lengths, att)
        for l in range(L):
            qkv = to(rng.standard_normal((len(batch), T, 3 * D)) / 8)
            q, k, v = qkv[..., :D], qkv[..., D:2 * D], qkv[..., 2 * D:]
            kw_ref, vw_ref = st.cache.update_attn_cache(l, rd(k), rd(v))
            if prepass:
                bd = pool.relpos_bd(l, q, pos_t[l], bv_t[l])
                out = pool.attention(l, q, None, bu_t[l], None, sl, ln, key=k, value=v, bd=bd)
            elif fused:   # the append happens inside the attention call
                out = pool.attention(l, q, pos_t[l], bu_t[l], bv_t[l], sl, ln, key=k, value=v)
            else:
                pool.append(l, k, v, sl)
                out = pool.attention(l, q, pos_t[l], bu_t[l], bv_t[l], sl, ln)
            if step % check_every == 0 or step == steps - 1:
                kw, vw = pool.gather(l, sl)
                assert np.array_equal(rd(kw), kw_ref), (step, l)
                assert np.array_equal(rd(vw), vw_ref), (step, l)
                ref = streaming.relpos_attention_core(rd(q), kw_ref, vw_ref, pos_r[l], bu_r[l],
                                                      bv_r[l], mask, H)
                got = rd(out)
                rows = [(b, t) for b in range(len(batch)) for t in range(lengths[b])]
                e = rel_l2(np.stack([got[b, t] for b, t in rows]), np.stack([ref[b, t] for b, t in rows]))
                worst = max(worst, e)
                assert e <= TOL[dtype], (step, l, e)
        if step % check_every == 0 or step == steps - 1:
            # every layer in one launch == the per-layer gathers, bit for bit
            kl, vl = pool.gather_layers(0, L, sl)
            for l in range(L):
                kw, vw = pool.gather(l, sl)
                assert torch.equal(kl[l], kw) and torch.equal(vl[l], vw), (step, l)
        st.processed_frames += np.asarray(lengths)
        st.cache_lengths = np.minimum(st.cache_lengths + np.asarray(lengths), left)
        dense.unpack_states(st, idx)
        pool.end_step(sl, ln)
    assert pool.read_error() == 0
    return worst


@pytest.mark.parametrize("fused", [False, True])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_append_gather_attention_small(dtype, fused):
    run_stream_steps("small", dtype, steps=44, n_slots=5, seed=3, check_every=5, fused=fused)


@pytest.mark.parametrize("fused", [False, True])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_append_gather_attention_large(dtype, fused):
    run_stream_steps("large", dtype, steps=9, n_slots=3, seed=4, fused=fused)


@pytest.mark.parametrize("fused", [False, True])
def test_append_gather_attention_large_8_frame_pages(fused):
    run_stream_steps("large_p8", torch.bfloat16, steps=9, n_slots=3, seed=9, fused=fused)


@pytest.mark.parametrize("shape", ["small_t3", "small_t4"])
@pytest.mark.parametrize("fused", [False, True])
def test_append_gather_attention_stacked_rows_above_8(shape, fused):
    run_stream_steps(shape, torch.bfloat16, steps=30, n_slots=4, seed=5, check_every=3, fused=fused)


def test_append_gather_attention_small_relpos_prepass():
    run_stream_steps("small", torch.bfloat16, steps=44, n_slots=5, seed=3, check_every=5,
                     prepass=True)


@pytest.mark.parametrize("shape", ["small_p8", "small_t3_p8"])
@pytest.mark.parametrize("fused,prepass", [(False, False), (True, False), (False, True)])
def test_append_gather_attention_8_frame_pages(shape, fused, prepass):
    """The stacked kernel over pages of 8 frames (two page boxes per 16 keys of
    P V), with the append fused or not and the rel-pos term from the pre-pass."""
    run_stream_steps(shape, torch.bfloat16, steps=44, n_slots=5, seed=8, check_every=3,
                     fused=fused, prepass=prepass)


def test_relpos_prepass_matches_in_kernel_term():
    """All layers in one call: relpos_bd + attention(bd=) gives the attention
    output of the in-kernel rel-pos term bit for bit (both run the same
    fragment code), and the pre-pass term itself matches float64 on the
    bf16-rounded operands."""
    cfg = SHAPES["small"]
    att, D, H = cfg["att"], cfg["dim"], cfg["heads"]
    left, T = att[0], att[1] + 1
    L, n_slots, dh = 3, 7, D // H
    P = 2 * (left + T) - 1
    rng = np.random.default_rng(21)
    order = rng.permutation(n_slots * pages.pages_per_stream(left, T, 16))
    pa, pb = (PagedKVPool(L, D, H, att, n_slots, dtype=torch.bfloat16, device=DEV, page_order=order)
              for _ in range(2))
    assert pa.relpos_bd_cols == 80
    to = lambda a: torch.tensor(np.asarray(a), dtype=torch.bfloat16, device=DEV)  # noqa: E731
    pos = to(rng.standard_normal((L, P, D)) / 8)
    bu, bv = to(rng.standard_normal((L, H, dh)) / 8), to(rng.standard_normal((L, H, dh)) / 8)
    slots = torch.tensor([4, 0, 6, 2, 5], dtype=torch.int32, device=DEV)
    B = slots.numel()
    ln = torch.full((B,), T, dtype=torch.int32, device=DEV)
    for step in range(7):
        qkv = to(rng.standard_normal((L, B, T, 3 * D)) / 8)
        q, k, v = qkv[..., :D], qkv[..., D:2 * D], qkv[..., 2 * D:]
        pa.begin_step(slots, ln)
        pb.begin_step(slots, ln)
        oa = pa.attention(0, q, pos, bu, bv, slots, ln, key=k, value=v)
        bd = pb.relpos_bd(0, q, pos, bv)
        ob = pb.attention(0, q, None, bu, None, slots, ln, key=k, value=v, bd=bd)
        pa.end_step(slots, ln)
        pb.end_step(slots, ln)
        assert torch.equal(oa, ob), step
        x = (q.double() + bv.double()[:, None, None].reshape(L, 1, 1, D)).to(torch.bfloat16).double()
        ref = torch.einsum("lbthd,lrhd->lbhtr", x.reshape(L, B, T, H, dh),
                           pos.double()[:, :80].reshape(L, 80, H, dh))
        assert rel_l2(bd.double().cpu().numpy(), ref.cpu().numpy()) <= 1e-5, step
    assert pa.read_error() == 0 and pb.read_error() == 0


@pytest.mark.parametrize("n_slots,batch,nl", [(9, 6, 3), (320, 300, 1)])
def test_step_start_with_relpos_equals_two_launches(n_slots, batch, nl):
    """pk_pages_begin_step_relpos (step start and rel-pos pre-pass in one launch;
    above 256 rows as two launches) against pk_relpos_bd + pk_pages_begin_step:
    the same page tables, counters, free ring and window descriptors, the same
    term and the same attention output, over steps with a released slot."""
    cfg = SHAPES["small"]
    att, D, H = cfg["att"], cfg["dim"], cfg["heads"]
    left, T = att[0], att[1] + 1
    P, dh = 2 * (left + T) - 1, D // H
    rng = np.random.default_rng(31)
    order = rng.permutation(n_slots * pages.pages_per_stream(left, T, 16))
    pa, pb = (PagedKVPool(nl, D, H, att, n_slots, dtype=torch.bfloat16, device=DEV, page_order=order)
              for _ in range(2))
    to = lambda a: torch.tensor(np.asarray(a), dtype=torch.bfloat16, device=DEV)  # noqa: E731
    pos = to(rng.standard_normal((nl, P, D)) / 8)
    bu, bv = to(rng.standard_normal((nl, H, dh)) / 8), to(rng.standard_normal((nl, H, dh)) / 8)
    slot_list = rng.permutation(n_slots)[:batch].tolist()
    for step in range(5):
        if step == 3:   # a stream ends; a new one takes its slot
            for p_ in (pa, pb):
                p_.release_slot(slot_list[0])
        slots = torch.tensor(slot_list, dtype=torch.int32, device=DEV)
        ln = torch.full((batch,), T, dtype=torch.int32, device=DEV)
        qkv = to(rng.standard_normal((nl, batch, T, 3 * D)) / 8)
        q, k, v = qkv[..., :D], qkv[..., D:2 * D], qkv[..., 2 * D:]
        bd_a = pa.relpos_bd(0, q, pos, bv)
        pa.begin_step(slots, ln)
        bd_b = pb.begin_step(slots, ln, relpos=(0, q, pos, bv, None))
        oa = pa.attention(0, q, None, bu, None, slots, ln, key=k, value=v, bd=bd_a)
        ob = pb.attention(0, q, None, bu, None, slots, ln, key=k, value=v, bd=bd_b)
        torch.cuda.synchronize()
        assert torch.equal(bd_a, bd_b), step
        assert torch.equal(oa, ob), step
        for name in ("page_table", "meta", "free_ring", "ring_ctr", "win_desc"):
            assert torch.equal(getattr(pa, name), getattr(pb, name)), (step, name)
        pa.end_step(slots, ln)
        pb.end_step(slots, ln)
    assert pa.read_error() == 0 and pb.read_error() == 0


def conv_oracle(x2d, cache, w, lengths, g, b, eps=1e-5):
    """GLU -> pad mask -> cached depthwise conv -> LayerNorm -> SiLU
    (convolution.py:153-159) on float64."""
    x = np.asarray(x2d, np.float64).transpose(0, 2, 1)          # [B, 2D, T]
    y = streaming.glu_channels(x)
    T = y.shape[-1]
    pad = np.arange(T)[None, :] >= np.asarray(lengths)[:, None]
    y = np.where(pad[:, None, :], 0.0, y)
    y, nxt = streaming.causal_depthwise_conv(y, cache, w)
    z = streaming.silu(streaming.layer_norm(y.transpose(0, 2, 1), g, b, eps))
    return z, y.transpose(0, 2, 1), nxt


@pytest.mark.parametrize("shape", ["small", "large", "small_t1", "small_t3", "small_t4", "wide_t2"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_conv_step_matches_oracle(shape, dtype):
    cfg = SHAPES[shape]
    D, T = cfg["dim"], cfg["att"][1] + 1
    rng = np.random.default_rng(5)
    n_slots, L, layer = 6, 3, 1
    pool = PagedKVPool(L, D, cfg["heads"], cfg["att"], n_slots, dtype=dtype, device=DEV)
    to = lambda a: torch.tensor(np.asarray(a), dtype=dtype, device=DEV)  # noqa: E731
    rd = lambda t: t.float().cpu().numpy().astype(np.float64)  # noqa: E731
    pool.conv.copy_(to(rng.standard_normal(pool.conv.shape)))
    w = to(rng.standard_normal((D, 1, 9)) / 3)
    g, b = to(1 + 0.1 * rng.standard_normal(D)), to(0.1 * rng.standard_normal(D))
    for it in range(3):
        batch = [4, 1, 3] if it != 1 else [0, 5]
        lengths = [T] * len(batch)
        lengths[0] = max(1, T - 1)
        sl = torch.tensor(batch, dtype=torch.int32, device=DEV)
        ln = torch.tensor(lengths, dtype=torch.int32, device=DEV)
        x = to(rng.standard_normal((len(batch), T, 2 * D)))
        others = [s for s in range(n_slots) if s not in batch]
        untouched = pool.conv[others].clone()
        cache_before = rd(pool.conv[sl.long(), layer])
        ref_z, ref_y, ref_next = conv_oracle(rd(x), cache_before, rd(w), lengths, rd(g), rd(b))
        raw = pool.conv_step(layer, x, w, sl, ln)                     # no LayerNorm
        pool.conv[sl.long(), layer] = to(cache_before)                # rewind the cache
        z = pool.conv_step(layer, x, w, sl, ln, g, b, 1e-5)
        tol = TOL[dtype]
        assert rel_l2(rd(raw), ref_y) <= tol
        assert rel_l2(rd(z), ref_z) <= tol
        got_next = rd(pool.conv[sl.long(), layer])
        if dtype == torch.float32:
            assert rel_l2(got_next, ref_next) <= tol
        else:   # cache holds dtype-rounded GLU outputs: equal up to one rounding step
            assert np.allclose(got_next, ref_next, rtol=1e-2, atol=1e-2)
        assert torch.equal(pool.conv[others], untouched)
    assert pool.read_error() == 0
