"""The failure path of the device pipelines, without a fault: every
TMA/mbarrier wait in this library is bounded and, when it runs out, records
PK_DEV_TIMEOUT in the caller's error word and returns, so that the context
stays usable (no trap, no hang).  pk_selftest_bounded_wait runs that same wait
(pk_common.cuh, mbar_wait_bounded) on an mbarrier that nothing arrives on; the
host reads the error word, and the next launches on the same context work."""
import ctypes

import pytest
import torch

from parakeet_b200 import _lib

pytestmark = pytest.mark.gpu


def _wait(err, arrive, limit_ns, waited):
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(_lib.lib().pk_selftest_bounded_wait(err.data_ptr(), arrive, limit_ns,
                                                    waited.data_ptr(), ctypes.c_void_p(stream)),
               "pk_selftest_bounded_wait")
    torch.cuda.synchronize()


def test_bounded_wait_runs_out_and_reports_timeout():
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    waited = torch.zeros(1, dtype=torch.int64, device="cuda")
    limit = 20_000_000                                   # 20 ms
    _wait(err, 0, limit, waited)                         # nothing arrives: the wait gives up
    assert int(err.item()) == _lib.PK_DEV_TIMEOUT
    assert limit <= int(waited.item()) < 1_000_000_000  # it waited its limit, then returned
    err.zero_()
    _wait(err, 1, limit, waited)                         # the phase completes: no error
    assert int(err.item()) == 0 and int(waited.item()) < limit
    x = torch.arange(1 << 20, device="cuda", dtype=torch.float32)
    assert float(x.sum().item()) == float((1 << 20) * ((1 << 20) - 1) // 2)  # context usable


def test_bounded_wait_rejects_bad_arguments():
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    waited = torch.zeros(1, dtype=torch.int64, device="cuda")
    for limit in (0, -5, 11_000_000_000):
        st = _lib.lib().pk_selftest_bounded_wait(err.data_ptr(), 0, limit, waited.data_ptr(), None)
        assert st == _lib.PK_EINVAL
    assert _lib.lib().pk_selftest_bounded_wait(None, 0, 1000, waited.data_ptr(), None) == _lib.PK_EINVAL
