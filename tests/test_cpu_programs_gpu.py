"""GPU parity against the reference's three CPU programs on the same inputs
(fixtures: tests/golden/cpu_programs.npz, made by make_cpu_programs.py from
the programs compiled out of the reference's sources, and pinned to them by
tests/test_oracle_golden.py):

  * cpu_fufft.cpp (Stockham radix 8, natural order; cpu_fufft.cpp:212-236):
    its filter spectrum / N, permuted by the library into the R16 and R8
    layouts, through the fused convolution, against the program's fp64 and
    fp32 convolutions; and the natural-order forward transform (fufft_c2c_f32)
    against its forward transform;
  * cpu_inplace.cpp (radix-8 DIF / DIT; cpu_inplace.cpp:173-193): its
    digit-reversed filter spectrum fed as is as the R8 layout (and in the
    register-boundary order as R8_BPERM), against its fp64 and fp32 results;
  * cpu_mixed.cpp (mixed radix, V = 8 and 16; cpu_mixed.cpp:238-252): its
    chain-order filter spectrum fed as is as the R8 (V = 8) or R16 (V = 16)
    layout, against its fp64 result.

Tolerance: rel L2 <= 2e-6 (fp32 outputs).
"""
import os

import numpy as np
import pytest
import torch

from oracle.oracle import rel_l2

pytestmark = pytest.mark.gpu
F32_TOL = 2e-6
G = np.load(os.path.join(os.path.dirname(__file__), "golden", "cpu_programs.npz"))


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from fufft_b200 import ops as o
    o.init()
    return o


def _dev(x):
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.complex64)).cuda()


def _bperm(x, n, v):
    """register-boundary order: dst[L + k*T] = src[v*L + k]"""
    return np.ascontiguousarray(np.asarray(x).reshape(n // v, v).T.ravel())


@pytest.mark.parametrize("n", [8, 64, 512, 4096])
def test_cpu_fufft_convolution_and_forward(ops, n):
    key = f"cpu_fufft/{n}"
    a, bspec = G[key + "/a"], G[key + "/bspec64"].astype(np.complex128) / n
    for layout in (ops.LAYOUT_R16_BPERM, ops.LAYOUT_R16, ops.LAYOUT_R8):
        if n < (16 if layout in (ops.LAYOUT_R16, ops.LAYOUT_R16_BPERM) else 8):
            continue
        filt = ops.filter_permute(_dev(bspec), n, layout)
        got = ops.conv(_dev(a), filt, n, layout).cpu().numpy()
        assert rel_l2(got, G[key + "/conv64"]) <= F32_TOL, (n, layout)
        assert rel_l2(got, G[key + "/conv32"]) <= F32_TOL, (n, layout)
    fwd = ops.c2c(_dev(a), n, -1).cpu().numpy()
    assert rel_l2(fwd, G[key + "/fwd64"]) <= F32_TOL
    assert rel_l2(fwd, G[key + "/fwd32"]) <= F32_TOL


@pytest.mark.parametrize("n", [8, 64, 512, 4096])
def test_cpu_inplace_digit_reversed_filter(ops, n):
    key = f"cpu_inplace/{n}"
    a = G[key + "/a"]
    for bs_key, out_key in (("bs64", "out64"), ("bs32", "out32")):
        bs = G[f"{key}/{bs_key}"]
        got = ops.conv(_dev(a), _dev(bs), n, ops.LAYOUT_R8).cpu().numpy()
        assert rel_l2(got, G[f"{key}/{out_key}"]) <= F32_TOL, (n, bs_key)
        if n >= 8:
            got = ops.conv(_dev(a), _dev(_bperm(bs, n, 8)), n, ops.LAYOUT_R8_BPERM).cpu().numpy()
            assert rel_l2(got, G[f"{key}/{out_key}"]) <= F32_TOL, (n, bs_key, "bperm")


@pytest.mark.parametrize("v", [8, 16])
@pytest.mark.parametrize("n", [16, 32, 64, 128, 256, 512, 1024, 2048, 4096])
def test_cpu_mixed_chain_order_filter(ops, v, n):
    if n < v:
        pytest.skip("a lane holds at least one butterfly")
    key = f"cpu_mixed/{v}/{n}"
    a, bs = G[key + "/a"], G[key + "/bs64"]
    layout = ops.LAYOUT_R8 if v == 8 else ops.LAYOUT_R16
    got = ops.conv(_dev(a), _dev(bs), n, layout).cpu().numpy()
    assert rel_l2(got, G[key + "/out64"]) <= F32_TOL, (n, v)
    lay_bp = ops.LAYOUT_R8_BPERM if v == 8 else ops.LAYOUT_R16_BPERM
    got = ops.conv(_dev(a), _dev(_bperm(bs, n, v)), n, lay_bp).cpu().numpy()
    assert rel_l2(got, G[key + "/out64"]) <= F32_TOL, (n, v, "bperm")
    torch.cuda.synchronize()
    assert ops.device_status() == 0
