"""Bounded device waits: an expired wait is recorded, reported and cleared.

Every spin-wait in the library's kernels has a time limit. This test makes one
run out on purpose without faulting or hanging the GPU: a one-thread kernel
waits, with a 1 ms limit, on a shared-memory barrier that nothing arrives at
(no copy or MMA is in flight). It then checks that the kernel returned, that
the status word and its host copy hold the kernel's code, that the next entry
point refuses to launch with H3B200_ERR_DEVICE instead of returning results
computed after the failure, and that clearing the status restores normal,
bit-exact operation.
"""

import numpy as np
import pytest
import torch

import h3b200
import oracle as O
from h3b200 import _lib

pytestmark = pytest.mark.gpu


def _bits(t):
    return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def test_expired_wait_is_reported_and_blocks_later_calls_until_cleared():
    lib = _lib.load()
    dev = torch.cuda.current_device()
    assert h3b200.device_status(dev) == 0
    x = torch.randn(64, 256, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16).cuda()
    h3b200.quantize_int8_rowwise(x)   # first call on the device: sets up the host copy of the status
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream().cuda_stream
    try:
        assert lib.h3b200_selftest_expire_wait(1_000_000, stream) == _lib.OK, lib.h3b200_last_error()
        torch.cuda.synchronize()          # the kernel returns after its 1 ms limit
        assert _lib.device_status_nowait(dev) == _lib.STATUS_SELFTEST
        with pytest.raises(RuntimeError, match="bounded device wait"):
            h3b200.quantize_int8_rowwise(x)
        with pytest.raises(RuntimeError, match="bounded device wait"):
            _lib.check_device(dev, "after the expired wait")
        assert h3b200.device_status(dev) == _lib.STATUS_SELFTEST   # synchronising read agrees
    finally:
        h3b200.device_status(dev, clear=True)
    assert h3b200.device_status(dev) == 0
    assert _lib.device_status_nowait(dev) == 0
    q, s = h3b200.quantize_int8_rowwise(x)
    qo, so = O.quantize_int8_rowwise(_bits(x))
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.reshape(-1).cpu().numpy(), so.reshape(-1))


def test_selftest_rejects_out_of_range_limits():
    lib = _lib.load()
    assert lib.h3b200_selftest_expire_wait(10, None) == _lib.ERR_INVALID
    assert lib.h3b200_selftest_expire_wait(5_000_000_000, None) == _lib.ERR_INVALID
