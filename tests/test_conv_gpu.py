"""GPU parity of the fused kernels against the oracle (oracle/fufft_oracle.c).

Every call goes through the C ABI (libfufft_b200.so) via fufft_b200.ops.  The
oracle runs the reference's algorithm on the same seeded inputs; the oracle is
itself pinned bit-exact to the reference (tests/test_oracle_golden.py).
Tolerances: fp32 outputs rel L2 <= 2e-6,
int16-BFP outputs rel L2 <= 6e-5; index maps and the BFP quantiser bit-exact.
"""
import numpy as np
import pytest
import torch

from oracle.oracle import MID_CONJ, MID_MULTIPLY, MID_NONE, rel_l2

pytestmark = pytest.mark.gpu

F32_TOL = 2e-6
BFP_TOL = 6e-5


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


LAYOUTS = {  # layout -> (radix, register-boundary width)
    "R8": (0, 8, 1), "R8_BPERM": (1, 8, 8), "R16": (2, 16, 1), "R16_BPERM": (3, 16, 16),
}
MIDS = {"none": MID_NONE, "mul": MID_MULTIPLY, "conj": MID_CONJ}


def _filter(oracle, b_nat, n, radix, v):
    b = oracle.permute_dr(b_nat, n, radix)
    return oracle.bperm(b, n, v) if v > 1 else b


def _bperm_elems(x, n, v):
    """register-boundary order of any element type: dst[L + k*T] = src[v*L + k]"""
    T = n // v
    i = np.arange(n)
    src = v * (i % T) + i // T
    return np.ascontiguousarray(x.reshape(-1, n, *x.shape[1:])[:, src].reshape(x.shape))


def _sizes(radix):
    return [n for n in (8, 16, 32, 64, 128, 256, 512, 1024, 2048, 4096, 8192)
            if n >= radix and n <= (4096 if radix == 8 else 8192)]


@pytest.mark.parametrize("lname", list(LAYOUTS))
@pytest.mark.parametrize("mname", list(MIDS))
def test_conv_f32_all_sizes(ops, oracle, lname, mname):
    layout, radix, v = LAYOUTS[lname]
    mid = MIDS[mname]
    for n in _sizes(radix):
        batch = 5 if n >= 1024 else 37          # not a multiple of the transforms per CTA
        a, b = oracle.gen_test(n, 1, batch)
        bk = _filter(oracle, b, n, radix, v)
        want = oracle.conv(a, oracle.permute_dr(b, n, radix), n, radix, mid)
        got = _host(ops.conv(_dev(a), _dev(bk) if mid != MID_NONE else None, n, layout, mid))
        e = rel_l2(got, want)
        assert e <= F32_TOL, (n, lname, mname, e)


@pytest.mark.parametrize("n,cpb,batch", [(512, 1, 2), (1024, 1, 4), (2048, 1, 2), (4096, 1, 2), (256, 4, 8)])
def test_conv_matches_reference_golden(ops, oracle, n, cpb, batch):
    """the reference's own seeded cases, against its own outputs"""
    import json, os, hashlib
    a, b = oracle.gen_test(n, cpb, batch)
    with open(os.path.join(os.path.dirname(__file__), "golden", "reference_digests.json")) as f:
        rec = json.load(f)[f"conv/{n}/{cpb}/{batch}"]
    for radix, layout, key in [(8, 0, "ip"), (16, 2, "v16")]:
        want = oracle.conv(a, oracle.permute_dr(b, n, radix), n, radix)
        assert hashlib.sha256(want.tobytes()).hexdigest() == rec[key]   # oracle == reference
        got = _host(ops.conv(_dev(a), _dev(oracle.permute_dr(b, n, radix)), n, layout))
        assert rel_l2(got, want) <= F32_TOL
        # fp64 ground truth, as the reference's own test does (verify_kernel.cpp:1395)
        assert rel_l2(got, oracle.conv_f64(a, b, n)) < 3e-6


def test_conv_broadcast_filter_and_inplace(ops, oracle):
    n, batch = 4096, 6
    a, b = oracle.gen_test(n, 1, batch)
    b1 = b[:n]
    want = oracle.conv(a, oracle.permute_dr(b1, n, 16), n, 16, MID_MULTIPLY, filter_stride=0)
    da = _dev(a)
    out = ops.conv(da, _dev(oracle.bperm(oracle.permute_dr(b1, n, 16), n, 16)), n, ops.LAYOUT_R16_BPERM,
                   filter_stride=0, out=da)                # in place
    assert rel_l2(_host(out), want) <= F32_TOL
    assert out.data_ptr() == da.data_ptr()


@pytest.mark.parametrize("n", [512, 1024, 2048, 4096])
@pytest.mark.parametrize("lname", ["R8", "R8_BPERM"])
def test_conv_r8_filter_paths(ops, oracle, n, lname):
    """radix-8 layouts: the register-boundary filter read from global memory
    (R8_BPERM, 512 and 1024), the radix-16 engine with the filter staged through
    a bit permutation (R8 1024-4096, R8_BPERM 2048 and 4096), the radix-8
    chain-order filter staged per warp (R8, 512): shared and per-transform
    filters, both mid-ops, an odd batch (a partly filled CTA below 2048)"""
    layout, radix, v = LAYOUTS[lname]
    batch = 7
    a, b = oracle.gen_test(n, 1, batch)
    for mid in (MID_MULTIPLY, MID_CONJ):
        for fs in (n, 0):
            bb = b if fs else b[:n]
            want = oracle.conv(a, oracle.permute_dr(bb, n, radix), n, radix, mid, filter_stride=fs)
            got = _host(ops.conv(_dev(a), _dev(_filter(oracle, bb, n, radix, v)), n, layout, mid, filter_stride=fs))
            assert rel_l2(got, want) <= F32_TOL, (mid, fs)


@pytest.mark.parametrize("n", [1024, 4096])
def test_conv_8_byte_aligned_signal(ops, oracle, n):
    """signal and output 8 bytes off a 16-byte boundary (the filter must be
    16-byte aligned: the C ABI answers FUFFT_ERR_MISALIGNED otherwise)"""
    batch = 3
    a, b = oracle.gen_test(n, 1, batch)
    for lname, (layout, radix, v) in LAYOUTS.items():
        want = oracle.conv(a, oracle.permute_dr(b, n, radix), n, radix)
        da = torch.zeros(batch * n + 1, dtype=torch.complex64, device="cuda")
        do = torch.zeros(batch * n + 1, dtype=torch.complex64, device="cuda")
        da[1:] = _dev(a)
        bk = _dev(_filter(oracle, b, n, radix, v))
        got = _host(ops.conv(da[1:], bk, n, layout, out=do[1:]))
        assert rel_l2(got, want) <= F32_TOL, lname
        assert do[0].item() == 0
        db = torch.zeros(batch * n + 1, dtype=torch.complex64, device="cuda")
        db[1:] = bk
        with pytest.raises(RuntimeError, match="MISALIGNED"):
            ops.conv(da[1:], db[1:], n, layout, out=do[1:])


def test_device_filter_permute_bit_exact(ops, oracle):
    rng = np.random.default_rng(1)
    for n in (64, 512, 2048, 4096, 8192):      # shared-memory staged gather (8192: 64 KB)
        b = (rng.standard_normal(3 * n) + 1j * rng.standard_normal(3 * n)).astype(np.complex64)
        for lname, (layout, radix, v) in LAYOUTS.items():
            if n > (4096 if radix == 8 else 8192):
                continue
            got = _host(ops.filter_permute(_dev(b), n, layout))
            assert np.array_equal(got, _filter(oracle, b, n, radix, v)), (n, lname)


@pytest.mark.parametrize("n", [256, 512, 1024, 2048, 4096])
def test_split_fwd_apply(ops, oracle, n):
    batch = 9
    a, b = oracle.gen_test(n, 1, batch)
    for radix, layout, lay_b in [(8, 0, 1), (16, 2, 3)]:
        spec = ops.fwd(_dev(a), n, layout)
        want_spec = oracle.fwd(a, n, radix)
        assert rel_l2(_host(spec), want_spec) <= F32_TOL
        bdr = oracle.permute_dr(b, n, radix)
        for mid in (MID_MULTIPLY, MID_CONJ):
            want = oracle.apply(want_spec, bdr, n, radix, mid)
            got = _host(ops.apply(spec, _dev(bdr), n, layout, mid))
            assert rel_l2(got, want) <= F32_TOL
            # register-boundary layouts: spectrum and filter both in bperm order
            spec_b = ops.fwd(_dev(a), n, lay_b)
            assert rel_l2(_host(spec_b), oracle.bperm(want_spec, n, radix)) <= F32_TOL
            bp = _dev(oracle.bperm(bdr, n, radix))
            got = _host(ops.apply(spec_b, bp, n, lay_b, mid))
            assert rel_l2(got, want) <= F32_TOL
        # one spectrum, many filters (spec_stride = 0)
        want = oracle.apply(np.tile(want_spec[:n], batch), bdr, n, radix)
        got = _host(ops.apply(spec[:n], _dev(bdr), n, layout, batch=batch, spec_stride=0))
        assert rel_l2(got, want) <= F32_TOL


@pytest.mark.parametrize("key", ["r2/512/1/4", "r2/512/8/8", "r2/256/1/4"])
def test_r2_two_for_one(ops, oracle, key):
    import os
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "reference_cases.npz"))
    xr, yr, b_dr = g[key + "/xr"], g[key + "/yr"], g[key + "/b_dr"]
    n = int(key.split("/")[1])
    want_u, want_v = g[key + "/ur"], g[key + "/vr"]           # the reference's own output
    ur, vr = ops.conv_r2(_dev(xr), _dev(yr), _dev(b_dr), n, ops.LAYOUT_R8)
    assert rel_l2(_host(ur), want_u) <= F32_TOL and rel_l2(_host(vr), want_v) <= F32_TOL
    # the same real filter through the radix-16 chain (b_dr rows are one spectrum)
    nat = np.empty(n, np.complex64)
    rev = oracle.rev_table(oracle.chain(n, 8), n)
    nat[rev] = b_dr[:n]
    b16 = np.tile(oracle.bperm(oracle.permute_dr(nat, n, 16), n, 16), xr.size // n)
    ur, vr = ops.conv_r2(_dev(xr), _dev(yr), _dev(b16), n, ops.LAYOUT_R16_BPERM)
    assert rel_l2(_host(ur), want_u) <= F32_TOL and rel_l2(_host(vr), want_v) <= F32_TOL


@pytest.mark.parametrize("n", [512, 1024, 2048, 4096])
@pytest.mark.parametrize("lname", list(LAYOUTS))
def test_r2_every_layout_and_filter_path(ops, oracle, n, lname):
    """two-for-one real convolution in every filter layout: the radix-8 layouts
    on the radix-16 engine (bit-permutation staging, n >= 1024 / 2048), the
    radix-16 chain order staged per warp, the register-boundary order read
    directly; both mid-ops, per-transform and shared filters"""
    layout, radix, v = LAYOUTS[lname]
    batch = 5
    rng = np.random.default_rng(n + radix + v)
    xr = rng.standard_normal(batch * n).astype(np.float32)
    yr = rng.standard_normal(batch * n).astype(np.float32)
    _, b = oracle.gen_test(n, 1, batch)
    for mid in (MID_MULTIPLY, MID_CONJ):
        for fs in (n, 0):
            bb = b if fs else b[:n]
            b_dr = oracle.permute_dr(bb, n, radix)
            want_u, want_v = oracle.conv_r2(xr, yr, b_dr, n, radix, filter_stride=fs)
            bk = oracle.bperm(b_dr, n, radix) if v > 1 else b_dr
            ur, vr = ops.conv_r2(_dev(xr), _dev(yr), _dev(bk), n, layout, mid, filter_stride=fs)
            if mid == MID_CONJ:   # the oracle's two-for-one applies the multiply; conj through the complex form
                a = (xr + 1j * yr).astype(np.complex64)
                w = oracle.conv(a, b_dr, n, radix, MID_CONJ, filter_stride=fs)
                want_u, want_v = w.real.astype(np.float32), w.imag.astype(np.float32)
            assert rel_l2(_host(ur), want_u) <= F32_TOL and rel_l2(_host(vr), want_v) <= F32_TOL, (mid, fs)


# one-pass kernel: even n <= 8192 (powers of two and not); two passes: odd n, n > 8192
@pytest.mark.parametrize("n", [2, 16, 256, 512, 1024, 2048, 3000, 4096, 8192, 999, 16384])
def test_bfp_pack_bit_exact_and_unpack(ops, oracle, n):
    rng = np.random.default_rng(n)
    x = (rng.standard_normal(7 * n) + 1j * rng.standard_normal(7 * n)).astype(np.complex64)
    x[3 * n:4 * n] = 0                                          # an all-zero transform (1e-30 floor)
    q, s = ops.bfp_pack(_dev(x), n)
    wq, ws = oracle.bfp_quantize(x, n)
    assert np.array_equal(_host(q), wq)
    assert np.array_equal(_host(s).view(np.uint32), ws.view(np.uint32))
    back = _host(ops.bfp_unpack(q, s, n))
    assert np.array_equal(back.view(np.uint32), oracle.bfp_dequantize(wq, ws, n).view(np.uint32))


@pytest.mark.parametrize("key", ["bfp/512/0", "bfp/512/1", "bfp/4096/0", "bfp/4096/1"])
def test_bfp_conv_reference_cases(ops, oracle, key):
    _, n, seed = key.split("/")
    n, seed = int(n), int(seed)
    a, b = oracle.gen_bfp(n, seed)
    aq, as_ = oracle.bfp_quantize(a, n)
    bq, bs = oracle.bfp_quantize(oracle.permute_dr(b, n, 16), n)
    wq, ws = oracle.conv_bfp(aq, as_, bq, bs, n, 16)
    oq, os_ = ops.conv_bfp(_dev(aq), _dev(as_), _dev(bq), _dev(bs), n, ops.LAYOUT_R16)
    got = oracle.bfp_dequantize(_host(oq), _host(os_), n)
    want = oracle.bfp_dequantize(wq, ws, n)
    assert rel_l2(got, want) <= BFP_TOL
    dq = np.abs(_host(oq).astype(np.int32) - wq.astype(np.int32))
    assert dq.max() <= 2                         # LSBs; rounding of fp32 values that differ by ~1e-7
    # whole pipeline vs unquantised fp64 (verify_kernel.cpp:1176)
    rel = rel_l2(got, oracle.conv_f64(a, b, n))
    assert rel < 3e-4 and -np.log2(rel) >= 12.0


@pytest.mark.parametrize("lname", list(LAYOUTS))
@pytest.mark.parametrize("mid", [MID_MULTIPLY, MID_CONJ, MID_NONE])
def test_bfp_conv_all_sizes(ops, oracle, lname, mid):
    layout, radix, v = LAYOUTS[lname]
    for n in _sizes(radix):
        batch = 5 if n >= 1024 else 37
        a, b = oracle.gen_test(n, 1, batch)
        aq, as_ = oracle.bfp_quantize(a, n)
        bdr = oracle.permute_dr(b, n, radix)
        bq, bs = oracle.bfp_quantize(bdr, n)
        wq, ws = oracle.conv_bfp(aq, as_, bq, bs, n, radix, mid)
        bk = _bperm_elems(bq, n, v) if v > 1 else bq
        oq, os_ = ops.conv_bfp(_dev(aq), _dev(as_), _dev(np.ascontiguousarray(bk)), _dev(bs), n, layout, mid)
        got = oracle.bfp_dequantize(_host(oq), _host(os_), n)
        assert rel_l2(got, oracle.bfp_dequantize(wq, ws, n)) <= BFP_TOL, (n, lname, mid)


def test_errors_and_status(ops):
    from fufft_b200 import FufftError
    a = torch.zeros(3 * 1000, dtype=torch.complex64, device="cuda")
    with pytest.raises(FufftError, match="INVALID_SIZE"):
        ops.conv(a, a, 1000, ops.LAYOUT_R16)
    a = torch.zeros(8192, dtype=torch.complex64, device="cuda")
    with pytest.raises(FufftError, match="INVALID_SIZE"):
        ops.conv(a, a, 8192, ops.LAYOUT_R8)           # beyond the radix-8 one-kernel limit
    a = torch.zeros(4096, dtype=torch.complex64, device="cuda")
    with pytest.raises(FufftError, match="MISALIGNED"):
        ops.conv(a, torch.view_as_complex(torch.view_as_real(a).view(-1)[2:-6].view(-1, 2)), 1024, ops.LAYOUT_R16)
    with pytest.raises(FufftError, match="INVALID_ARG"):
        ops.conv(a, None, 1024, ops.LAYOUT_R16, ops.MID_MULTIPLY)
    empty = torch.zeros(0, dtype=torch.complex64, device="cuda")
    ops.conv(empty, empty, 1024, ops.LAYOUT_R16)       # batch 0: nothing to do
    torch.cuda.synchronize()
    assert ops.device_status() == 0


@pytest.mark.parametrize("n,batch,fs", [(4096, 37, "per"), (1024, 9000, "per"), (512, 30000, "shared"),
                                        (32768, 5, "per")])
def test_conv_host_pipeline(ops, oracle, n, batch, fs):
    """fufft_conv_c2c_f32_host: host buffers through the chunked upload /
    convolve / download pipeline equal the device-resident call bit for bit,
    over several chunks and a ragged last chunk; a shared filter is uploaded once"""
    rng = np.random.default_rng(n + batch)
    a = (rng.standard_normal(batch * n) + 1j * rng.standard_normal(batch * n)).astype(np.complex64)
    nb = batch if fs == "per" else 1
    b = ((rng.uniform(-1, 1, nb * n) + 1j * rng.uniform(-1, 1, nb * n)) / n).astype(np.complex64)
    stride = n if fs == "per" else 0
    want = _host(ops.conv(_dev(a), _dev(b), n, ops.LAYOUT_R16_BPERM, MID_MULTIPLY, filter_stride=stride))
    ha = torch.from_numpy(a).pin_memory()
    hb = torch.from_numpy(b).pin_memory()
    ho = torch.empty_like(ha).pin_memory()
    ws = ops.conv_host_workspace(n, batch, stride)
    for _ in range(2):       # the workspace is reused by consecutive calls on one stream
        ho.zero_()
        ops.conv_host(ha, hb, ho, n, ops.LAYOUT_R16_BPERM, MID_MULTIPLY, filter_stride=stride, workspace=ws)
        torch.cuda.current_stream().synchronize()
        assert np.array_equal(ho.numpy(), want)
    # mid-op none needs no filter
    ho.zero_()
    ops.conv_host(ha, None, ho, n, ops.LAYOUT_R16_BPERM, MID_NONE, workspace=ws)
    torch.cuda.current_stream().synchronize()
    assert rel_l2(ho.numpy() / n, a) <= F32_TOL
    from fufft_b200._lib import FufftError
    with pytest.raises(FufftError):      # too small a workspace
        ops.conv_host(ha, hb, ho, n, ops.LAYOUT_R16_BPERM, MID_MULTIPLY, filter_stride=stride, workspace=ws[:64])


@pytest.mark.parametrize("lname", list(LAYOUTS))
@pytest.mark.parametrize("n", [8, 64, 512, 4096, 8192])
def test_filter_from_taps(ops, oracle, lname, n):
    """taps -> spectrum x 1/n in the kernel layout on the device, against the
    oracle's permutation of a float64 spectrum; then used by a convolution"""
    layout, radix, v = LAYOUTS[lname]
    if n < radix or n > ops.max_n(layout) or (n > 4096 and radix == 8):
        pytest.skip("size outside the layout's one-kernel range")
    batch = 3
    rng = np.random.default_rng(n + layout)
    taps = (rng.uniform(-1, 1, batch * n) + 1j * rng.uniform(-1, 1, batch * n)).astype(np.complex64)
    spec = (np.fft.fft(taps.astype(np.complex128).reshape(batch, n), axis=1) / n).astype(np.complex64).ravel()
    want = _filter(oracle, spec, n, radix, v)
    got = _host(ops.filter_from_taps(_dev(taps), n, layout))
    assert rel_l2(got, want) <= F32_TOL
    a = (rng.standard_normal(batch * n) + 1j * rng.standard_normal(batch * n)).astype(np.complex64)
    conv = _host(ops.conv(_dev(a), _dev(got), n, layout))
    assert rel_l2(conv, oracle.conv_f64(a, spec, n)) <= 3e-6
