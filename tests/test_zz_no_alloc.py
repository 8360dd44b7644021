"""The allocation-free BFP four-step entry point (fufft_conv_large_bfp_noalloc).

It serves callers that cannot allocate device memory when they call the
library -- a host whose device memory is all held by its own pool allocator,
or a latency-critical loop that must not risk an allocation's device-wide
synchronisation -- by using a fixed scratch area the library reserves on each
GPU instead of a caller workspace.  Called through the C ABI (ctypes), twice
in a row with different inputs, it must give the same result as the existing
entry point with a caller-provided workspace, within the BFP tolerance of the
other tests.  This file is collected last so a stopping run has already run
every other test; it also passes alone in a fresh process."""
import ctypes as ct

import numpy as np
import pytest
import torch

from oracle.oracle import rel_l2

pytestmark = pytest.mark.gpu
BFP_TOL = 6e-5


def _case(n, batch, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    a = torch.randn(n * batch, dtype=torch.complex64, device="cuda", generator=g)
    b = torch.randn(n * batch, dtype=torch.complex64, device="cuda", generator=g) / n
    return a, b


def test_noalloc_matches_workspace_entry_point_twice(oracle):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from fufft_b200 import ops
    from fufft_b200._lib import lib
    ops.init()
    L = lib()
    n = 32768
    r_out, mid = ops.large_plan(n, ops.LAYOUT_R16)
    stream = torch.cuda.current_stream().cuda_stream
    for call, (batch, seed) in enumerate([(4, 11), (8, 12)]):       # two calls in a row
        a, b = _case(n, batch, seed)
        aq, as_ = ops.bfp_pack(a, n)
        bq, bs = ops.bfp_pack(b, n)
        want_q, want_s = ops.conv_large_bfp(aq, as_, bq, bs, n, ops.LAYOUT_R16, r_out=r_out, mid_size=mid)
        oq = torch.empty_like(aq)
        os_ = torch.empty(batch, dtype=torch.float32, device="cuda")
        rc = L.fufft_conv_large_bfp_noalloc(aq.data_ptr(), as_.data_ptr(), bq.data_ptr(), bs.data_ptr(),
                                            oq.data_ptr(), os_.data_ptr(), n, batch, r_out, mid,
                                            ops.LAYOUT_R16, ops.MID_MULTIPLY, stream)
        assert rc == 0, f"call {call}: status {rc}"
        torch.cuda.synchronize()
        got = oracle.bfp_dequantize(oq.cpu().numpy(), os_.cpu().numpy(), n)
        want = oracle.bfp_dequantize(want_q.cpu().numpy(), want_s.cpu().numpy(), n)
        assert rel_l2(got, want) <= BFP_TOL, f"call {call}"


def test_noalloc_rejects_requests_beyond_its_scratch():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from fufft_b200._lib import lib
    n, batch = 1 << 21, 2                                  # needs 32 MiB of scratch: over the 16 MiB limit
    rc = lib().fufft_conv_large_bfp_noalloc(None, None, None, None, None, None, n, batch, 16, 2048, 2, 1,
                                            ct.c_void_p(0))
    assert rc == 1                                         # FUFFT_ERR_INVALID_SIZE
