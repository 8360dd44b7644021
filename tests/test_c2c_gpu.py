"""GPU parity of the natural-order transform fufft_c2c_f32 (the reference's
Mode A fufft_c2c, fufft.cuh:878-904) against the oracle's restatement, the
reference's own kernel_c2c (verify_kernel.cpp:1183-1201, powers of 8) and
float64.  Tolerance: fp32 rel L2 <= 2e-6."""
import numpy as np
import pytest
import torch

from oracle.oracle import rel_l2

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


@pytest.mark.parametrize("n", [8, 16, 32, 64, 128, 256, 512, 1024, 2048, 4096, 8192])
def test_c2c_forward_inverse(ops, oracle, n):
    batch = 37 if n <= 1024 else 5          # not a multiple of the transforms per CTA
    rng = np.random.default_rng(n)
    a = (rng.standard_normal(batch * n) + 1j * rng.standard_normal(batch * n)).astype(np.complex64)
    radix = 16 if n >= 16 else 8
    got = ops.c2c(_dev(a), n, -1).cpu().numpy()
    assert rel_l2(got, oracle.c2c(a, n, -1, radix)) <= F32_TOL
    f64 = np.fft.fft(a.astype(np.complex128).reshape(batch, n), axis=1).ravel()
    assert rel_l2(got, f64) <= F32_TOL
    inv = ops.c2c(_dev(got), n, +1).cpu().numpy()
    assert rel_l2(inv, oracle.c2c(got, n, +1, radix)) <= F32_TOL
    assert rel_l2(inv / n, a) <= F32_TOL
    # in place
    t = _dev(a)
    ops.c2c(t, n, -1, out=t)
    assert np.array_equal(t.cpu().numpy(), got)


@pytest.mark.parametrize("n", [8, 64, 512, 4096])
def test_c2c_matches_reference_kernel(ops, oracle, n):
    """the reference's own forward c2c on its seeded input (mt19937(N*131+CPB))"""
    from oracle.oracle import Reference
    try:
        ref = Reference()
    except OSError:
        pytest.skip("oracle/_ref not present")
    a, _ = oracle.gen_test(n, 1, 3)
    got = ops.c2c(_dev(a), n, -1).cpu().numpy()
    assert rel_l2(got, ref.c2c(a, n)) <= F32_TOL


def test_c2c_rejects_bad_arguments(ops):
    from fufft_b200._lib import FufftError
    x = torch.zeros(16384, dtype=torch.complex64, device="cuda")
    for n, sign in [(16, 0), (4, -1), (16384, -1), (24, -1)]:
        with pytest.raises(FufftError):
            ops.c2c(x[: (n if n > 0 else 16) * 2] if n != 24 else x[:48], n, sign)
