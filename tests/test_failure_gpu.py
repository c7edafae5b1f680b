"""Failure detection on the GPU without faulting it: a kernel wait that runs
out (an mbarrier nothing arrives on) ends with an error status the host reads,
and the CUDA context stays usable afterwards."""

from __future__ import annotations

import pytest
import torch

from semblend_b200 import _lib

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives():
    dev = torch.device("cuda", 0)
    lib = _lib.load()
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    _lib.check(lib.sb_selftest_wait_timeout(status.data_ptr(), 20_000_000, _lib.stream_ptr(dev)), "selftest")
    torch.cuda.synchronize(dev)
    assert int(status.item()) == 7
    x = torch.arange(10, device=dev)
    assert int(x.sum().item()) == 45  # context still healthy


def test_invalid_arguments_are_rejected_before_launch():
    lib = _lib.load()
    assert lib.sb_selftest_wait_timeout(None, 10, None) == _lib.SB_ERR_INVALID_ARGUMENT
    assert lib.sb_inject(None, 1, None, None, None) == _lib.SB_ERR_INVALID_ARGUMENT
