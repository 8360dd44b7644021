"""GPU parity of the cluster-fused convolutions (fufft_cluster.cuh): 1-D
n = 16384 / 32768 / 65536 on the radix-16 chain, and 2-D images beyond one
CTA up to 256x256, against the oracle and fp64.
(The four-step with one outer level, e.g. the reference's N=32768 recipe,
runs on the same kernel: tests/test_large_gpu.py.)"""
import numpy as np
import pytest
import torch

from oracle.oracle import MID_CONJ, MID_MULTIPLY, MID_NONE, rel_l2

pytestmark = pytest.mark.gpu
F32_TOL = 2e-6


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from fufft_b200 import ops as o
    o.init()
    return o


def _dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def _block_bperm(x, n, blk, v=16):
    """register-boundary order inside each block of blk points"""
    T = blk // v
    i = np.arange(n)
    off, ii = (i // blk) * blk, i % blk
    src = off + v * (ii % T) + ii // T
    return np.ascontiguousarray(x.reshape(-1, n)[:, src].ravel())


@pytest.mark.parametrize("n,C", [(16384, 4), (32768, 8), (65536, 16)])
def test_cluster_conv1d(ops, oracle, n, C):
    batch = 3
    rng = np.random.default_rng(n)
    a = (rng.standard_normal(n * batch) + 1j * rng.standard_normal(n * batch)).astype(np.complex64)
    b = ((rng.uniform(-1, 1, n * batch) + 1j * rng.uniform(-1, 1, n * batch)) / n).astype(np.complex64)
    b16 = oracle.permute_dr(b, n, 16)
    bp = _block_bperm(b16, n, n // C)
    assert np.array_equal(ops.filter_permute_host(b, n, ops.LAYOUT_R16_BPERM), bp)
    for mid in (MID_MULTIPLY, MID_CONJ, MID_NONE):
        want = oracle.conv(a, b16, n, 16, mid)
        got = ops.conv(_dev(a), _dev(b16) if mid != MID_NONE else None, n, ops.LAYOUT_R16, mid).cpu().numpy()
        assert rel_l2(got, want) <= F32_TOL, (n, mid)
        if mid != MID_NONE:
            got = ops.conv(_dev(a), _dev(bp), n, ops.LAYOUT_R16_BPERM, mid).cpu().numpy()
            assert rel_l2(got, want) <= F32_TOL, (n, mid, "bperm")
    conv = ops.conv(_dev(a), _dev(b16), n, ops.LAYOUT_R16).cpu().numpy()
    assert rel_l2(conv[:n], oracle.conv_f64(a[:n], b[:n], n)) < 3e-6
    da = _dev(a)
    out = ops.conv(da, _dev(bp), n, ops.LAYOUT_R16_BPERM, out=da)          # in place
    assert rel_l2(out.cpu().numpy(), oracle.conv(a, b16, n, 16)) <= F32_TOL


@pytest.mark.parametrize("h,w", [(128, 128), (256, 128), (128, 256), (256, 256), (128, 512)])
def test_cluster_conv2d(ops, oracle, h, w):
    batch = 2
    n = h * w
    rng = np.random.default_rng(h + 3 * w)
    a = rng.uniform(0, 1, n * batch).astype(np.complex64)
    b = ((rng.standard_normal(n) + 1j * rng.standard_normal(n)) / n).astype(np.complex64)   # one shared filter
    b2 = oracle.permute2d(b, h, w, 16)
    want = oracle.conv2d(a, b2, h, w, 16, MID_MULTIPLY, filter_stride=0)
    got = ops.conv2d(_dev(a), _dev(b2), h, w, ops.LAYOUT_R16, filter_stride=0).cpu().numpy()
    assert rel_l2(got, want) <= F32_TOL
    assert rel_l2(got, oracle.conv2d_f64(a, np.tile(b, batch), h, w)) < 3e-6
    C = 16 if h == 256 else 8
    bp = _block_bperm(b2, n, n // C)
    dev_bp = ops.filter_permute2d(_dev(b), h, w, ops.LAYOUT_R16_BPERM)
    assert np.array_equal(dev_bp.cpu().numpy(), bp)
    got = ops.conv2d(_dev(a), dev_bp, h, w, ops.LAYOUT_R16_BPERM, filter_stride=0).cpu().numpy()
    assert rel_l2(got, want) <= F32_TOL
    got = ops.conv2d(_dev(a), _dev(b2), h, w, ops.LAYOUT_R16, MID_CONJ, filter_stride=0).cpu().numpy()
    assert rel_l2(got, oracle.conv2d(a, b2, h, w, 16, MID_CONJ, filter_stride=0)) <= F32_TOL
