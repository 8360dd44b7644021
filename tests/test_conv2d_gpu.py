"""GPU parity of the fused 2-D convolution (fufft_conv2d_f32) against the
oracle.  Radix 8 on power-of-8 sides is the reference's fufft_conv2d (pinned
bit-exact to its transcription in tests/test_oracle_golden.py); other shapes
and the radix-16 chains are checked against the oracle's generalisation and
against the fp64 row/column reference (verify_kernel.cpp:753-786)."""
import numpy as np
import pytest
import torch

from oracle.oracle import MID_CONJ, MID_MULTIPLY, rel_l2

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


def _bperm(x, n, v):
    T = n // v
    i = np.arange(n)
    src = v * (i % T) + i // T
    return np.ascontiguousarray(x.reshape(-1, n)[:, src].ravel())


@pytest.mark.parametrize("h,w,batch", [(64, 64, 3), (8, 512, 2), (512, 8, 2)])
def test_conv2d_reference_cases(ops, oracle, h, w, batch):
    a, b = oracle.gen_2d(h, w, batch)
    b2 = oracle.permute2d(b, h, w, 8)
    want = oracle.conv2d_pow8(a, b2, h, w)
    got = ops.conv2d(_dev(a), _dev(b2), h, w, ops.LAYOUT_R8).cpu().numpy()
    assert rel_l2(got, want) <= F32_TOL
    assert rel_l2(got, oracle.conv2d_f64(a, b, h, w)) < 3e-6
    got = ops.conv2d(_dev(a), _dev(_bperm(b2, h * w, 8)), h, w, ops.LAYOUT_R8_BPERM).cpu().numpy()
    assert rel_l2(got, want) <= F32_TOL


SHAPES16 = [(8, 16), (16, 16), (8, 64), (64, 64), (128, 64), (64, 128), (16, 512), (512, 16), (32, 256)]
SHAPES8 = [(8, 8), (16, 8), (16, 32), (32, 32), (64, 32), (8, 256), (256, 16)]


@pytest.mark.parametrize("radix,h,w", [(16, h, w) for h, w in SHAPES16] + [(8, h, w) for h, w in SHAPES8])
def test_conv2d_shapes(ops, oracle, radix, h, w):
    batch = 7
    rng = np.random.default_rng(h * 7 + w)
    a = (rng.uniform(0, 1, h * w * batch)).astype(np.complex64)         # config 4: real image
    b = (rng.standard_normal(h * w * batch) + 1j * rng.standard_normal(h * w * batch)).astype(np.complex64) / (h * w)
    b2 = oracle.permute2d(b, h, w, radix)
    for mid in (MID_MULTIPLY, MID_CONJ):
        want = oracle.conv2d(a, b2, h, w, radix, mid)
        lay, lay_b = (ops.LAYOUT_R16, ops.LAYOUT_R16_BPERM) if radix == 16 else (ops.LAYOUT_R8, ops.LAYOUT_R8_BPERM)
        got = ops.conv2d(_dev(a), _dev(b2), h, w, lay, mid).cpu().numpy()
        assert rel_l2(got, want) <= F32_TOL, (h, w, mid)
        got = ops.conv2d(_dev(a), _dev(_bperm(b2, h * w, radix)), h, w, lay_b, mid).cpu().numpy()
        assert rel_l2(got, want) <= F32_TOL, (h, w, mid, "bperm")
    assert rel_l2(ops.conv2d(_dev(a), _dev(b2), h, w, lay).cpu().numpy(), oracle.conv2d_f64(a, b, h, w)) < 3e-6


def test_conv2d_broadcast_filter_and_device_permute(ops, oracle):
    h, w, batch = 64, 128, 9
    rng = np.random.default_rng(5)
    a = rng.uniform(0, 1, h * w * batch).astype(np.complex64)
    b = (rng.standard_normal(h * w) + 1j * rng.standard_normal(h * w)).astype(np.complex64) / (h * w)
    b2 = oracle.permute2d(b, h, w, 16)
    dev_b2 = ops.filter_permute2d(_dev(b), h, w, ops.LAYOUT_R16_BPERM)
    assert np.array_equal(dev_b2.cpu().numpy(), _bperm(b2, h * w, 16))
    want = oracle.conv2d(a, b2, h, w, 16, MID_MULTIPLY, filter_stride=0)
    got = ops.conv2d(_dev(a), dev_b2, h, w, ops.LAYOUT_R16_BPERM, filter_stride=0).cpu().numpy()
    assert rel_l2(got, want) <= F32_TOL


@pytest.mark.parametrize("h,w", [(64, 64), (8, 512), (32, 16)])
def test_conv2d_reference_layout_shared_filter(ops, oracle, h, w):
    """the reference's 2-D filter order (radix 8 per dimension) with one filter
    for every image, in both orders: on the radix-16 engine through the bit
    permutation (rows of 16 or more)"""
    batch = 5
    rng = np.random.default_rng(h + 3 * w)
    a = rng.uniform(0, 1, h * w * batch).astype(np.complex64)
    b = (rng.standard_normal(h * w) + 1j * rng.standard_normal(h * w)).astype(np.complex64) / (h * w)
    b2 = oracle.permute2d(b, h, w, 8)
    for mid in (MID_MULTIPLY, MID_CONJ):
        want = oracle.conv2d(a, b2, h, w, 8, mid, filter_stride=0)
        got = ops.conv2d(_dev(a), _dev(b2), h, w, ops.LAYOUT_R8, mid, filter_stride=0).cpu().numpy()
        assert rel_l2(got, want) <= F32_TOL, mid
        got = ops.conv2d(_dev(a), _dev(_bperm(b2, h * w, 8)), h, w, ops.LAYOUT_R8_BPERM, mid,
                         filter_stride=0).cpu().numpy()
        assert rel_l2(got, want) <= F32_TOL, (mid, "bperm")


def test_conv2d_rejects_unsupported_shape(ops):
    from fufft_b200 import FufftError
    a = torch.zeros(256 * 256, dtype=torch.complex64, device="cuda")
    with pytest.raises(FufftError, match="INVALID_SIZE"):
        ops.conv2d(a, a, 256, 256, ops.LAYOUT_R8)
