"""Device-side failure detection without a GPU fault.

Every wait inside this library's kernels is bounded: when a phase does not
complete in time the waiting thread records DK_ERR_DEVICE_TIMEOUT in the
device status word and the kernel returns through its normal exit, so the CUDA
context stays usable.  dk_test_bounded_wait runs that same wait loop with a
short limit on a barrier whose producer can be told to skip its arrival.
"""
import time

import pytest



def _run(dev, skip_arrive, limit_ns):
    import torch

    from detkernels_b200 import _lib
    lib = _lib.load()
    _lib.device_status(dev.index, clear=True)
    rc = lib.dk_test_bounded_wait(int(skip_arrive), int(limit_ns), _lib.stream_ptr(dev))
    _lib.check(rc, "dk_test_bounded_wait")
    torch.cuda.synchronize(dev)
    return _lib.device_status(dev.index, clear=True)


@pytest.mark.gpu
def test_bounded_wait_completes_when_the_producer_arrives(dev):
    from detkernels_b200 import _lib
    code, detail = _run(dev, skip_arrive=False, limit_ns=50_000_000)
    assert (code, detail) == (_lib.DK_OK, 0)


@pytest.mark.gpu
def test_bounded_wait_runs_out_reports_and_returns(dev):
    import torch

    from detkernels_b200 import _lib
    from detkernels_b200.kernels.rmsnorm import rmsnorm_batch_invariant
    t0 = time.perf_counter()
    code, detail = _run(dev, skip_arrive=True, limit_ns=2_000_000)
    elapsed = time.perf_counter() - t0
    assert code == _lib.DK_ERR_DEVICE_TIMEOUT and detail == 0x7E57
    assert elapsed < 5.0
    # the context is still usable: a library kernel runs and the status stays clean
    x = torch.randn(4, 256, device=dev)
    w = torch.ones(256, device=dev)
    y = rmsnorm_batch_invariant(x, w)
    torch.cuda.synchronize(dev)
    assert torch.isfinite(y).all()
    assert _lib.device_status(dev.index, clear=True) == (_lib.DK_OK, 0)


def test_bounded_wait_rejects_unbounded_limits():
    import os

    from detkernels_b200 import _lib
    from detkernels_b200 import build
    if not os.path.exists(_lib.library_path()):
        build.build()
    lib = _lib.load()
    assert lib.dk_test_bounded_wait(1, 0, None) == _lib.DK_ERR_INVALID_ARGUMENT
    assert lib.dk_test_bounded_wait(1, 10 ** 10, None) == _lib.DK_ERR_INVALID_ARGUMENT
