"""Failure detection on the GPU without a GPU fault: every device wait of the
library is bounded (a %globaltimer deadline) and reports through the device
status word.  The self-test makes one wait run out (an mbarrier that nothing
completes) and checks that the kernel returns, the status bit is set and then
cleared by the read, and the context still runs a convolution correctly."""
import numpy as np
import pytest
import torch

from oracle.oracle import rel_l2

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives(oracle):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from fufft_b200 import ops
    from fufft_b200._lib import check, lib
    ops.init()
    assert ops.device_status() == 0
    check(lib().fufft_selftest_wait_timeout(1000, torch.cuda.current_stream().cuda_stream),
          "fufft_selftest_wait_timeout")
    torch.cuda.synchronize()
    assert ops.device_status() == 1          # STATUS_TMA_TIMEOUT, read and cleared
    assert ops.device_status() == 0
    n, batch = 4096, 3
    a, b = oracle.gen_test(n, 1, batch)
    got = ops.conv(torch.from_numpy(a).cuda(), torch.from_numpy(oracle.permute_dr(b, n, 16)).cuda(), n,
                   ops.LAYOUT_R16).cpu().numpy()
    assert rel_l2(got, oracle.conv(a, oracle.permute_dr(b, n, 16), n, 16)) <= 2e-6
    assert ops.device_status() == 0


def test_selftest_rejects_bad_limits():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from fufft_b200._lib import lib
    assert lib().fufft_selftest_wait_timeout(0, None) != 0
    assert lib().fufft_selftest_wait_timeout(2000000, None) != 0
