"""GPU parity of the one-signal-many-filters shape:
two-for-one packed forward transforms (fufft_fwd_r2_f32) and the grid apply
(fufft_apply_grid_f32 / _r2_f32: every spectrum against every filter in one
launch), against the oracle's split fwd / apply (the reference's
kernel_pipeline_fwd / kernel_pipeline_apply, verify_kernel.cpp:794-836) and,
for the real-pair form, against a float64 convolution / correlation.
Tolerance: fp32 rel L2 <= 2e-6 against the oracle."""
import numpy as np
import pytest
import torch

from oracle.oracle import MID_CONJ, MID_MULTIPLY, MID_NONE, rel_l2

pytestmark = pytest.mark.gpu

F32_TOL = 2e-6
# (layout id, radix, register-boundary width)
LAYOUTS = {"R8": (0, 8, 1), "R8_BPERM": (1, 8, 8), "R16": (2, 16, 1), "R16_BPERM": (3, 16, 16)}


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from fufft_b200 import ops as o
    o.init()
    return o


def _dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def _host(t):
    return t.cpu().numpy()


def _real_filters(rng, n, nf):
    """spectra (1/n folded in) of real taps iid U[-1,1), natural order"""
    taps = rng.uniform(-1.0, 1.0, (nf, n))
    return (np.fft.fft(taps, axis=1) / n).astype(np.complex64), taps


def _layout_filters(oracle, b_nat, n, radix, v):
    rows = [oracle.permute_dr(b_nat[f], n, radix) for f in range(b_nat.shape[0])]
    if v > 1:
        rows = [oracle.bperm(r, n, v) for r in rows]
    return np.concatenate(rows)


@pytest.mark.parametrize("lname", list(LAYOUTS))
@pytest.mark.parametrize("n", [256, 1024, 4096])
def test_fwd_r2_matches_packed_fwd(ops, oracle, lname, n):
    layout, radix, v = LAYOUTS[lname]
    if n > ops.max_n(layout):
        pytest.skip("size beyond the one-kernel range of the layout")
    rng = np.random.default_rng(n + 7)
    batch = 5
    xr = rng.standard_normal(batch * n).astype(np.float32)
    yr = rng.standard_normal(batch * n).astype(np.float32)
    got = _host(ops.fwd_r2(_dev(xr), _dev(yr), n, layout))
    want = oracle.fwd((xr + 1j * yr).astype(np.complex64), n, radix)
    if v > 1:     # register-boundary layouts keep spectra in the bperm order too
        want = oracle.bperm(want, n, v)
    assert rel_l2(got, want) <= F32_TOL


@pytest.mark.parametrize("lname", list(LAYOUTS))
@pytest.mark.parametrize("mid", [MID_MULTIPLY, MID_CONJ])
@pytest.mark.parametrize("n,ns,nf", [(512, 3, 5), (4096, 2, 7)])
def test_apply_grid_complex(ops, oracle, lname, mid, n, ns, nf):
    layout, radix, v = LAYOUTS[lname]
    if n > ops.max_n(layout):
        pytest.skip("size beyond the one-kernel range of the layout")
    rng = np.random.default_rng(1000 * ns + nf + n)
    a = (rng.standard_normal(ns * n) + 1j * rng.standard_normal(ns * n)).astype(np.complex64)
    b_nat = ((rng.uniform(-1, 1, (nf, n)) + 1j * rng.uniform(-1, 1, (nf, n))) / n).astype(np.complex64)
    spec = ops.fwd(_dev(a), n, layout)
    want_spec = oracle.fwd(a, n, radix)
    b_dr = np.concatenate([oracle.permute_dr(b_nat[f], n, radix) for f in range(nf)])
    want = oracle.apply_grid(want_spec, b_dr, n, radix, mid)
    got = _host(ops.apply_grid(spec, _dev(_layout_filters(oracle, b_nat, n, radix, v)), n, layout, mid))
    assert got.shape == want.shape
    assert rel_l2(got, want) <= F32_TOL


@pytest.mark.parametrize("lname", ["R16_BPERM", "R16", "R8"])
@pytest.mark.parametrize("mid", [MID_MULTIPLY, MID_CONJ])
def test_apply_grid_real_pairs_config3_shape(ops, oracle, lname, mid):
    """config 3 at reduced counts: 6 real signals (3 packed pairs) x 4 real
    filters at N=4096; each output row against the oracle and float64"""
    layout, radix, v = LAYOUTS[lname]
    n, npair, nf = 4096, 3, 4
    rng = np.random.default_rng(33 + mid)
    x = rng.standard_normal((2 * npair, n)).astype(np.float32)
    b_nat, taps = _real_filters(rng, n, nf)
    spec = ops.fwd_r2(_dev(x[0::2].reshape(-1)), _dev(x[1::2].reshape(-1)), n, layout)
    want_spec = oracle.fwd((x[0::2] + 1j * x[1::2]).astype(np.complex64).reshape(-1), n, radix)
    b_dr = np.concatenate([oracle.permute_dr(b_nat[f], n, radix) for f in range(nf)])
    want = oracle.apply_grid_r2(want_spec, b_dr, n, radix, mid)
    got = _host(ops.apply_grid_r2(spec, _dev(_layout_filters(oracle, b_nat, n, radix, v)), n, layout, mid))
    assert rel_l2(got, want) <= F32_TOL
    # row i*nf + f is signal i filtered by (or correlated with) filter f
    got = got.reshape(2 * npair, nf, n)
    X = np.fft.fft(x.astype(np.float64), axis=1)
    for i in range(2 * npair):
        for f in range(nf):
            H = np.fft.fft(taps[f])
            ref = np.fft.ifft(X[i] * (np.conj(H) if mid == MID_CONJ else H)).real
            assert rel_l2(got[i, f], ref) <= 2e-5, (i, f)


def test_apply_grid_edges(ops):
    from fufft_b200._lib import FufftError
    n = 1024
    spec = torch.zeros(2 * n, dtype=torch.complex64, device="cuda")
    b = torch.zeros(3 * n, dtype=torch.complex64, device="cuda")
    # an empty grid launches nothing
    out = ops.apply_grid(spec[:0], b, n, ops.LAYOUT_R16)
    assert out.numel() == 0
    # the grid apply needs a filter mid-op
    with pytest.raises(FufftError):
        ops.apply_grid(spec, b, n, ops.LAYOUT_R16, MID_NONE)
    # sizes the one-kernel chain cannot take
    m = 768
    with pytest.raises(FufftError):
        ops.apply_grid(torch.zeros(2 * m, dtype=torch.complex64, device="cuda"),
                       torch.zeros(3 * m, dtype=torch.complex64, device="cuda"), m, ops.LAYOUT_R16)
