"""Argument validation of the C ABI: every entry point returns a status code
(never exits or faults) for sizes, batches, layouts, enums, strides,
alignment and null pointers the library does not take.  The size, batch and
enum checks come before any device call, so they run without a GPU; the
pointer checks need the device context and run on a GPU."""
import ctypes as ct

import pytest

OK, SIZE, BATCH, MISALIGNED, CUDA, TIMEOUT, PEER, ARG, UNSUP = range(9)
P = 1 << 20        # a fake, 16-byte aligned address: never dereferenced by these calls


def _L():
    from fufft_b200._lib import lib
    return lib()


def test_sizes_batches_enums_rejected_before_device():
    L = _L()
    conv = L.fufft_conv_c2c_f32
    assert conv(P, P, P, 3000, 1, 3, 1, 3000, None) == SIZE          # not a power of two
    assert conv(P, P, P, 1 << 17, 1, 3, 1, 1 << 17, None) == SIZE    # beyond the one-kernel range
    assert conv(P, P, P, 4, 1, 3, 1, 4, None) == SIZE                # below the radix
    assert conv(P, P, P, 4096, -1, 3, 1, 4096, None) == BATCH
    assert conv(P, P, P, 4096, 1, 9, 1, 4096, None) == ARG           # unknown layout
    assert conv(P, P, P, 4096, 0, 3, 1, 4096, None) == OK            # empty batch: nothing to do
    assert L.fufft_conv_c2c_bfp(P, P, P, P, P, P, 4096, -5, 2, 1, 4096, None) == BATCH
    assert L.fufft_c2c_f32(P, P, 4096, 1, 0, None) == ARG            # sign must be -1 or +1
    assert L.fufft_c2c_f32(P, P, 4, 1, -1, None) == SIZE
    assert L.fufft_c2c_f32(P, P, 16384, 1, -1, None) == SIZE
    assert L.fufft_apply_grid_f32(P, -1, P, 4, P, 4096, 3, 1, None) == BATCH
    assert L.fufft_apply_grid_f32(P, 0, P, 4, P, 4096, 3, 1, None) == OK
    assert L.fufft_conv2d_f32(P, P, P, 100, 100, 1, 3, 1, 0, None) == SIZE
    assert L.fufft_conv_large_f32(P, P, 32768, 1, 16, 3000, 2, 1, None) == SIZE   # mid not a power of two
    assert L.fufft_conv_large_f32(P, P, 32768, 1, 4, 2048, 2, 1, None) == ARG     # outer radix 8 or 16
    assert L.fufft_conv_c2c_f32_host(P, P, P, 4096, 8, 3, 1, 100, P, 1 << 30, None) == ARG   # stride n or 0
    assert L.fufft_selftest_wait_timeout(0, None) == ARG
    assert L.fufft_dist_pass(P, 3, 1024, 0, 1 << 20, -1, None) != OK       # world 2, 4 or 8
    r, m = ct.c_int(), ct.c_int()
    assert L.fufft_large_plan(1000, 2, ct.byref(r), ct.byref(m)) == SIZE


@pytest.mark.gpu
def test_pointer_checks_on_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from fufft_b200 import ops
    ops.init()
    L = _L()
    x = torch.zeros(2 * 4096 + 8, dtype=torch.float32, device="cuda")
    b = torch.zeros(2 * 4096, dtype=torch.float32, device="cuda")
    a, bb = x.data_ptr(), b.data_ptr()
    conv = L.fufft_conv_c2c_f32
    assert conv(a + 4, bb, a, 4096, 1, 3, 1, 4096, None) == MISALIGNED     # signal not 8-byte aligned
    assert conv(a, bb + 8, a, 4096, 1, 3, 1, 4096, None) == MISALIGNED     # filter not 16-byte aligned
    assert conv(None, bb, a, 4096, 1, 3, 1, 4096, None) == ARG
    assert conv(a, None, a, 4096, 1, 3, 1, 4096, None) == ARG              # multiply needs a filter
    assert conv(a, None, a, 4096, 1, 3, 0, 4096, None) == OK               # mid-op none does not
    assert conv(a, bb, a, 4096, 1, 3, 7, 4096, None) == ARG                # unknown mid-op
    assert conv(a, bb, a, 4096, 1, 3, 1, -4096, None) == ARG               # negative filter stride
    torch.cuda.synchronize()
    assert ops.device_status() == 0
