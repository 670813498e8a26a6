"""Host-side checks that need no GPU: the C-ABI library loads and exports
every declared entry point, argument errors come back as statuses, and the
slot allocator keeps the reference's FIFO order."""
import ctypes

import numpy as np
import pytest

from oracle import pages
from parakeet_b200 import _lib
from parakeet_b200.engine.scheduler import SlotAllocator
from replay import load


def test_library_exports_every_declared_symbol():
    names = _lib.declared_functions()
    assert len(names) >= 12
    lib = _lib.lib()
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing
    assert set(_lib.SIGNATURES) == set(names)


def test_ctypes_signatures_match_header_declarations():
    """Every entry point's ctypes argument list matches its declaration in
    include/pk.h parameter by parameter: the same count, pointers as pointers,
    and the same integer or float width (an int32 passed where int64 is
    declared leaves garbage in the upper half; an argument added on one side
    only shifts every later one)."""
    import ctypes
    import re
    text = re.sub(r"/\*.*?\*/", "", open(_lib.HEADER).read(), flags=re.S)
    decls = dict(re.findall(r"\b(pk_[a-z_0-9]+)\s*\(([^;{]*?)\)\s*;", text, flags=re.S))
    scalar = {"int32_t": ctypes.c_int32, "int64_t": ctypes.c_int64, "float": ctypes.c_float,
              "double": ctypes.c_double, "int": ctypes.c_int}
    checked = 0
    for name, args in _lib.SIGNATURES.items():
        params = decls[name].strip()
        plist = [] if params in ("", "void") else [p.strip() for p in params.split(",")]
        assert len(args) == len(plist), (name, len(args), len(plist))
        for i, (c_param, ct) in enumerate(zip(plist, args)):
            if "*" in c_param:
                assert ct is ctypes.c_void_p or ct is ctypes.c_char_p or \
                    issubclass(ct, ctypes._Pointer), (name, i, c_param, ct)
            else:
                ctype = c_param.replace("const ", "").split()[0]
                assert ct is scalar[ctype], (name, i, c_param, ct)
        checked += 1
    assert checked == len(_lib.declared_functions())


@pytest.mark.parametrize("left,chunk,ps", [(70, 2, 16), (70, 14, 16), (70, 2, 8), (33, 5, 16)])
def test_page_geometry_matches_model(left, chunk, ps):
    lib = _lib.lib()
    assert lib.pk_pages_per_stream(left, chunk, ps) == pages.pages_per_stream(left, chunk, ps)
    assert lib.pk_ring_size(left, chunk, ps) == pages.ring_size(left, chunk, ps)
    # the bound is tight: some window start touches exactly that many pages
    worst = max((w + chunk - 1) // ps - max(w - left, 0) // ps + 1 for w in range(0, 4 * ps, chunk))
    assert worst <= pages.pages_per_stream(left, chunk, ps)


def test_create_rejects_bad_descriptors_without_a_gpu():
    lib = _lib.lib()
    d = _lib.PagedKVDesc(num_pages=4, num_slots=2, num_layers=1, dim=512, num_heads=8, left=70,
                         chunk=2, page_size=16, ring=8, dtype=_lib.PK_DTYPE_BF16)
    h = ctypes.c_void_p()
    assert lib.pk_paged_kv_create(ctypes.byref(d), ctypes.byref(h)) == _lib.PK_EINVAL
    assert b"null" in lib.pk_last_error()
    fake = 1 << 20  # never dereferenced: validation fails first
    for k in ("kv", "page_table", "free_ring", "ring_ctr", "meta", "error", "window"):
        setattr(d, k, fake)
    d.ring = 4   # smaller than pages_per_stream(70, 2, 16) = 6
    assert lib.pk_paged_kv_create(ctypes.byref(d), ctypes.byref(h)) == _lib.PK_EINVAL
    d.ring, d.page_size = 8, 12
    assert lib.pk_paged_kv_create(ctypes.byref(d), ctypes.byref(h)) == _lib.PK_EINVAL
    assert lib.pk_conv_step(None, 1, 1, 0, 512, 9, 2, 5, None, 0, 0, None, None, None, 1e-5,
                            None, None, 1, None, None, None) == _lib.PK_EINVAL
    assert lib.pk_pages_begin_step(None, None, None, 1, None, 0, None) == _lib.PK_EINVAL


def test_slot_allocator_matches_reference_sequence():
    ops = load("scheduler_slots.npz")["ops"]
    a = SlotAllocator(8)
    for kind, slot in ops:
        if kind == 0:
            got = a.acquire()
            assert (-1 if got is None else got) == slot
        else:
            a.release(int(slot))


def test_slot_allocator_page_cap_admission():
    per = pages.pages_per_stream(70, 2, 16)
    a = SlotAllocator(10, per, num_pages=int(0.6 * 10 * per))
    got = [a.acquire() for _ in range(10)]
    assert got[:6] == list(range(6)) and got[6:] == [None] * 4
    a.release(2)
    assert a.acquire() == 6          # FIFO: released slot goes to the back
    with pytest.raises(ValueError):
        a.release(2)


def test_page_model_churn_conserves_pages():
    rng = np.random.default_rng(4)
    n_slots, per = 9, pages.pages_per_stream(70, 2, 16)
    pool = pages.PagePoolModel(int(0.6 * n_slots * per), n_slots, 70, 2, 16,
                               init_order=rng.permutation(int(0.6 * n_slots * per)))
    alloc = SlotAllocator(n_slots, per, pool.num_pages)
    live = []
    for _ in range(400):
        if live and rng.random() < 0.05:
            s = live.pop(int(rng.integers(len(live))))
            alloc.release(s)
            pool.release_slot(s)
        if rng.random() < 0.3:
            s = alloc.acquire()
            if s is not None:
                live.append(s)
        batch = [s for s in live if rng.random() < 0.9]
        assert pool.begin_step(batch)
        pool.end_step(batch, [2] * len(batch))
        held = int((pool.next - pool.first).sum())
        assert held + len(pool.free) == pool.num_pages
        assert set(pool.free).isdisjoint(set(pool.table[pool.table >= 0].tolist()))


def test_admission_queue_matches_reference_scheduler():
    """The drop-in Scheduler's add / admit_ready / release against the
    reference's (golden ``admission.npz`` from tests/golden/make_golden.py):
    the same sequences admitted per call, the same running order, and every
    status written with the caller's own enum."""
    import enum
    import json
    from types import SimpleNamespace

    from parakeet_b200.engine.scheduler import Scheduler

    class CallerStatus(enum.Enum):      # stands in for the reference's SequenceStatus
        WAITING = enum.auto()
        RUNNING = enum.auto()
        FINISHED = enum.auto()

    calls = json.loads(str(load("admission.npz")["calls"]))
    sched = Scheduler(max_active=3)
    seqs = []
    for c in calls:
        admitted = []
        if c["call"] == "add":
            seqs.append(SimpleNamespace(status=CallerStatus.WAITING, name=c["arg"]))
            sched.add(seqs[-1])
        elif c["call"] == "admit":
            admitted = [q.name for q in sched.admit_ready()]
        else:
            sched.release(seqs[c["arg"]])
        assert admitted == c["admitted"]
        assert [q.name for q in sched.active_sequences()] == c["active"]
        assert all(type(q.status) is CallerStatus for q in seqs)
        assert [q.status.name for q in seqs] == c["status"]
    assert any(c["admitted"] for c in calls) and sched.num_waiting >= 0


def test_python_constants_equal_header_defines():
    """Every integer #define of include/pk.h that _lib mirrors (same name, or
    without the PK_ prefix) has the same value."""
    import re
    text = open(_lib.HEADER).read()
    checked = 0
    for name, value in re.findall(r"^#define (PK_\w+) (\d+)\b", text, re.M):
        for py in (name, name[3:]):
            if hasattr(_lib, py):
                assert getattr(_lib, py) == int(value), (name, getattr(_lib, py), value)
                checked += 1
                break
    assert checked >= 20
    assert _lib.PK_NOALLOC_SCRATCH_BYTES == 32 * 1024 * 1024
