"""A bounded device wait that runs out: the kernel waits on a counter that nothing ever
increments, with a 50 ms limit. It must return on its own, leave kErrTimeoutFlag in the
device's status word, surface as KernelError(timeout) on the host, and the worker must map
that to PoolError TIMEOUT (the router's re-dispatch signal). The context stays usable.
Nothing faults or hangs: the flag is ordinary device memory of this process."""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_wait_that_runs_out_reports_timeout_and_the_worker_maps_it(cuda_dev):
    from lake_b200.ops import core
    from lake_b200.ops._ext import native
    from lake_b200.pool.types import PoolErrorCode
    from lake_b200.runtime.worker_engine import _step_error_code

    core.check_status(cuda_dev)  # start from a clean status word
    cnt = torch.zeros(2, dtype=torch.int64, device=cuda_dev)  # never incremented
    status = core.status_word(cuda_dev)
    t0 = time.perf_counter()
    native().wait_counters(cnt.data_ptr(), 2, 1, status, limit_ns=50_000_000)
    torch.cuda.synchronize(cuda_dev)
    elapsed = time.perf_counter() - t0
    assert 0.04 < elapsed < 5.0, elapsed  # it waited about the limit, then returned
    with pytest.raises(core.KernelError) as e:
        core.check_status(cuda_dev)
    assert e.value.code == 2 and e.value.timeout
    assert _step_error_code(e.value) == PoolErrorCode.TIMEOUT
    core.check_status(cuda_dev)  # the word was cleared
    # a counter that has reached its target passes at once
    cnt.fill_(1)
    native().wait_counters(cnt.data_ptr(), 2, 1, status, limit_ns=50_000_000)
    torch.cuda.synchronize(cuda_dev)
    core.check_status(cuda_dev)
    x = torch.arange(16, device=cuda_dev, dtype=torch.float32)
    assert x.sum().item() == 120.0


def test_after_a_wait_ran_out_the_later_waits_of_the_step_fail_at_once(cuda_dev):
    """A lost peer costs one time bound per step: once the status word holds the time-out, a
    wait that would take 2 s returns at once; after the host has reported (and cleared) the word,
    waits behave normally again."""
    from lake_b200.ops import core
    from lake_b200.ops._ext import native

    core.check_status(cuda_dev)
    cnt = torch.zeros(1, dtype=torch.int64, device=cuda_dev)  # never incremented
    status = core.status_word(cuda_dev)
    native().wait_counters(cnt.data_ptr(), 1, 1, status, limit_ns=50_000_000)
    torch.cuda.synchronize(cuda_dev)
    t0 = time.perf_counter()
    native().wait_counters(cnt.data_ptr(), 1, 1, status, limit_ns=2_000_000_000)
    torch.cuda.synchronize(cuda_dev)
    assert time.perf_counter() - t0 < 1.0  # it did not wait its 2 s
    with pytest.raises(core.KernelError) as e:
        core.check_status(cuda_dev)
    assert e.value.code == 2
    t0 = time.perf_counter()
    native().wait_counters(cnt.data_ptr(), 1, 1, status, limit_ns=50_000_000)  # a fresh step waits again
    torch.cuda.synchronize(cuda_dev)
    assert time.perf_counter() - t0 > 0.04
    with pytest.raises(core.KernelError):
        core.check_status(cuda_dev)
    core.check_status(cuda_dev)
