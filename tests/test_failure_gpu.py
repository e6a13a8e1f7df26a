"""Failure detection on the GPU without a fault: a kernel waits, through the
bounded-wait helper every kernel uses, on an mbarrier nothing completes. The
wait gives up after a short limit, the kernel records WX_DEVERR_TIMEOUT in the
device error word and returns, and the context stays usable for the next
launch. (The reference injects failures on the host only:
serve/npu_stt_server.py:128-129.)
"""
import time

import numpy as np
import pytest
import torch

import rowops_ref as O
from wxb200 import _lib as L
from wxb200 import ops

pytestmark = pytest.mark.gpu


def test_wait_runs_out_and_is_reported(cuda):
    assert L.device_error() == 0
    t0 = time.perf_counter()
    L.check(L.lib().wx_selftest_wait_timeout(50_000_000, None))   # 50 ms limit
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    assert 0.04 < dt < 5.0, dt                 # it waited about the limit, then returned
    assert L.device_error() == L.WX_DEVERR_TIMEOUT
    assert L.device_error() == 0               # reading cleared it


def test_context_usable_after_timeout(cuda):
    L.check(L.lib().wx_selftest_wait_timeout(10_000_000, None))
    torch.cuda.synchronize()
    assert L.device_error() == L.WX_DEVERR_TIMEOUT
    rng = np.random.default_rng(3)
    x = O.rbf(rng.normal(0, 2, (64, 512)).astype(np.float32), O.RNE)
    got = ops.gelu_poly4(torch.from_numpy(x).to(torch.bfloat16).cuda(), rounding=L.WX_ROUND_RNE)
    ref = O.gelu_poly4(x, O.RNE)
    assert np.array_equal(got.float().cpu().numpy().view(np.uint32), ref.view(np.uint32))
    assert L.device_error() == 0


def test_selftest_rejects_bad_limits(cuda):
    with pytest.raises(ValueError):
        L.check(L.lib().wx_selftest_wait_timeout(0, None))
    with pytest.raises(ValueError):
        L.check(L.lib().wx_selftest_wait_timeout(3_000_000_000, None))
