"""The allocation-free BFP four-step entry point (fufft_conv_large_bfp_noalloc).

It serves callers that cannot allocate device memory when they call the
library -- a host whose device memory is all held by its own pool allocator,
or a latency-critical loop that must not risk an allocation's device-wide
synchronisation -- by using a fixed scratch area the library reserves on each
GPU instead of a caller workspace.  Called through the C ABI (ctypes) several
times in a row with different inputs and sizes, it must give the same result
as the existing entry point with a caller-provided workspace, within the BFP
tolerance of the other tests, and agree with the oracle.

The cases are chosen so the scratch area is really used: n = 262144 with the
radix-16 plan (16, 1024) has two outer levels and n = 32768 with a radix-8
middle runs the multi-kernel path, and both keep the fp32 intermediate in the
workspace.  (A one-outer-level radix-16 plan runs as one cluster kernel and
never touches it.)  This file is collected last so a stopping run has already
run every other test; it also passes alone in a fresh process."""
import ctypes as ct

import numpy as np
import pytest
import torch

from oracle.oracle import rel_l2

pytestmark = pytest.mark.gpu
BFP_TOL = 6e-5


@pytest.fixture(scope="module")
def env():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from fufft_b200 import ops
    from fufft_b200._lib import lib
    ops.init()
    return ops, lib()


# (n, batch, layout name, middle radix): two outer levels at 8 MiB and at the
# full 16 MiB, then a different n through the radix-8 middle (one outer level,
# multi-kernel path), then the first case again over the previous contents
CALLS = [(262144, 4, "R16", 16), (262144, 8, "R16", 16), (32768, 8, "R8", 8), (262144, 2, "R16", 16)]


def test_noalloc_matches_workspace_entry_point_in_a_row(env, oracle):
    ops, L = env
    stream = torch.cuda.current_stream().cuda_stream
    for call, (n, batch, lname, mr) in enumerate(CALLS):
        layout = getattr(ops, "LAYOUT_" + lname)
        r_out, mid = ops.large_plan(n, layout)
        lout, q = 0, n // mid
        while q > 1:
            q //= r_out
            lout += 1
        assert lout >= 2 or mr == 8, "the case must reach the multi-kernel path (scratch in use)"
        assert 8 * n * batch <= (16 << 20)
        rng = np.random.default_rng(1000 + call)
        a = (rng.standard_normal(n * batch) + 1j * rng.standard_normal(n * batch)).astype(np.complex64)
        taps = rng.uniform(-1, 1, n * batch) + 1j * rng.uniform(-1, 1, n * batch)
        spec = (np.fft.fft(taps.reshape(batch, n), axis=1) / n).astype(np.complex64)
        rev = oracle.rev_table(oracle.foursteps_chain(n, r_out, mid, mr), n)
        b_dr = np.ascontiguousarray(spec[:, rev]).ravel()
        aq, as_ = oracle.bfp_quantize(a, n)
        bq, bs = oracle.bfp_quantize(b_dr, n)
        daq, das, dbq, dbs = (torch.from_numpy(np.ascontiguousarray(x)).cuda() for x in (aq, as_, bq, bs))

        # the existing entry point, caller workspace
        want_q, want_s = ops.conv_large_bfp(daq, das, dbq, dbs, n, layout, r_out=r_out, mid_size=mid)
        # the allocation-free one, output buffers pre-filled with garbage
        oq = torch.full_like(daq, 12345)
        os_ = torch.full((batch,), 7.0, dtype=torch.float32, device="cuda")
        rc = L.fufft_conv_large_bfp_noalloc(daq.data_ptr(), das.data_ptr(), dbq.data_ptr(), dbs.data_ptr(),
                                            oq.data_ptr(), os_.data_ptr(), n, batch, r_out, mid, layout,
                                            ops.MID_MULTIPLY, stream)
        assert rc == 0, f"call {call}: status {rc}"
        torch.cuda.synchronize()
        got = oracle.bfp_dequantize(oq.cpu().numpy(), os_.cpu().numpy(), n)
        want = oracle.bfp_dequantize(want_q.cpu().numpy(), want_s.cpu().numpy(), n)
        assert rel_l2(got, want) <= BFP_TOL, f"call {call}: differs from the workspace entry point"
        # and against the oracle: dequantise, fp32 four-step, requantise
        want_f = oracle.conv_foursteps(oracle.bfp_dequantize(aq, as_, n), oracle.bfp_dequantize(bq, bs, n),
                                       n, r_out, mid, mr)
        wq, ws = oracle.bfp_quantize(want_f, n)
        assert rel_l2(got, oracle.bfp_dequantize(wq, ws, n)) <= BFP_TOL, f"call {call}: differs from the oracle"
    assert ops.device_status() == 0


def test_noalloc_status_codes(env):
    ops, L = env
    z = ct.c_void_p(0)
    # beyond the scratch: a valid plan, 2^21 points x 2 transforms, needs 32 MiB;
    # real buffers of the right size, so only the scratch limit can reject it
    n, batch = 1 << 21, 2
    q = [torch.zeros(n * batch, 2, dtype=torch.int16, device="cuda") for _ in range(3)]
    s = [torch.ones(batch, dtype=torch.float32, device="cuda") for _ in range(3)]
    rc = L.fufft_conv_large_bfp_noalloc(q[0].data_ptr(), s[0].data_ptr(), q[1].data_ptr(), s[1].data_ptr(),
                                        q[2].data_ptr(), s[2].data_ptr(), n, batch, 16, 8192, ops.LAYOUT_R16,
                                        ops.MID_MULTIPLY, z)
    assert rc == 1                                          # FUFFT_ERR_INVALID_SIZE
    # null pointers are reported before the size limit, as the workspace entry point reports them
    assert L.fufft_conv_large_bfp_noalloc(None, None, None, None, None, None, n, batch, 16, 8192, 2, 1, z) == 7
    # a bad plan is reported as the workspace entry point reports it, before the size limit
    for args in [((1 << 21) + 1, 2, 16, 2048, 2), (1 << 21, 2, 12, 2048, 2), (1 << 21, 2, 16, 2048, 9)]:
        n, batch, r_out, mid, layout = args
        want = L.fufft_conv_large_bfp(None, None, None, None, None, None, n, batch, r_out, mid, layout, 1,
                                      None, 0, z)
        got = L.fufft_conv_large_bfp_noalloc(None, None, None, None, None, None, n, batch, r_out, mid, layout, 1, z)
        assert got == want != 0, args
    # batch 0: nothing to do, whatever the pointers
    assert L.fufft_conv_large_bfp_noalloc(None, None, None, None, None, None, 262144, 0, 16, 1024, 2, 1, z) == 0
