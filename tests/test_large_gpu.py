"""GPU parity of the four-step large-N convolution (fufft_conv_large_f32 /
_bfp) against the oracle on the reference's own cases
(verify_kernel.cpp:1455-1460 test_large_cfg, pinned bit-exact by
tests/test_oracle_golden.py), plus full-size
properties."""
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


def _chunk_bperm(x, mid, v):
    T = mid // v
    i = np.arange(mid)
    src = v * (i % T) + i // T
    return np.ascontiguousarray(x.reshape(-1, mid)[:, src].ravel())


CASES = [(32768, 2, 8, 4096, False), (32768, 2, 8, 4096, True), (32768, 2, 16, 2048, True),
         (131072, 1, 16, 8192, True), (524288, 1, 16, 2048, True)]


@pytest.mark.parametrize("n,batch,r_out,mid,v16", CASES)
def test_large_reference_cases(ops, oracle, n, batch, r_out, mid, v16):
    mr = 16 if v16 else 8
    a, b = oracle.gen_large_cfg(n, batch, r_out, mid)
    rev = oracle.rev_table(oracle.foursteps_chain(n, r_out, mid, mr), n)
    b_dr = np.ascontiguousarray(b.reshape(batch, n)[:, rev]).ravel()
    want = oracle.conv_foursteps(a, b_dr, n, r_out, mid, mr)
    lay, lay_b = (ops.LAYOUT_R16, ops.LAYOUT_R16_BPERM) if v16 else (ops.LAYOUT_R8, ops.LAYOUT_R8_BPERM)
    got = ops.conv_large(_dev(a), _dev(b_dr), n, lay, r_out=r_out, mid_size=mid).cpu().numpy()
    assert rel_l2(got, want) <= F32_TOL
    assert rel_l2(got[:n], oracle.conv_f64(a[:n], b[:n], n)) < 5e-6   # verify_kernel.cpp:524
    got = ops.conv_large(_dev(a), _dev(_chunk_bperm(b_dr, mid, mr)), n, lay_b, r_out=r_out, mid_size=mid)
    assert rel_l2(got.cpu().numpy(), want) <= F32_TOL


def test_large_plan_matches_reference_recipes(ops):
    assert ops.large_plan(32768, ops.LAYOUT_R16) == (16, 2048)        # bench_fufft.cu:520
    assert ops.large_plan(262144, ops.LAYOUT_R16) == (16, 1024)       # bench_fufft.cu:521
    assert ops.large_plan(1 << 26, ops.LAYOUT_R16) == (16, 1024)


@pytest.mark.parametrize("n,batch", [(32768, 3), (262144, 1)])
def test_large_bfp(ops, oracle, n, batch):
    r_out, mid = ops.large_plan(n, ops.LAYOUT_R16)
    rng = np.random.default_rng(n)
    a = (rng.standard_normal(n * batch) + 1j * rng.standard_normal(n * batch)).astype(np.complex64)
    taps = (rng.uniform(-1, 1, n * batch) + 1j * rng.uniform(-1, 1, n * batch))
    spec = (np.fft.fft(taps.reshape(batch, n), axis=1) / n).astype(np.complex64).ravel()
    rev = oracle.rev_table(oracle.foursteps_chain(n, r_out, mid, 16), n)
    b_dr = np.ascontiguousarray(spec.reshape(batch, n)[:, rev]).ravel()
    aq, as_ = oracle.bfp_quantize(a, n)
    bq, bs = oracle.bfp_quantize(b_dr, n)
    # oracle: dequantise, fp32 four-step, requantise (the same steps the library runs)
    want_f = oracle.conv_foursteps(oracle.bfp_dequantize(aq, as_, n), oracle.bfp_dequantize(bq, bs, n),
                                   n, r_out, mid, 16)
    wq, ws = oracle.bfp_quantize(want_f, n)
    oq, os_ = ops.conv_large_bfp(_dev(aq), _dev(as_), _dev(bq), _dev(bs), n, ops.LAYOUT_R16)
    got = oracle.bfp_dequantize(oq.cpu().numpy(), os_.cpu().numpy(), n)
    assert rel_l2(got, oracle.bfp_dequantize(wq, ws, n)) <= BFP_TOL
    # whole pipeline against the unquantised fp64 convolution
    rel = rel_l2(got[:n], oracle.conv_f64(a[:n], spec[:n], n))
    assert rel < 3e-4


@pytest.mark.parametrize("r_out,mid", [(16, 2048), (8, 4096)])
@pytest.mark.parametrize("lname", ["R16", "R16_BPERM"])
@pytest.mark.parametrize("midop", [MID_MULTIPLY, MID_CONJ, MID_NONE])
def test_large_bfp_cluster(ops, oracle, r_out, mid, lname, midop):
    """N=32768 with one outer level: the BFP four-step runs as one cluster
    kernel (int16 in, filter and out; cluster-wide abs-max for the scale)"""
    import ctypes as ct
    from fufft_b200._lib import lib
    n, batch = 32768, 3
    layout = getattr(ops, "LAYOUT_" + lname)
    rng = np.random.default_rng(n + r_out + midop)
    a = (rng.standard_normal(n * batch) + 1j * rng.standard_normal(n * batch)).astype(np.complex64)
    taps = (rng.uniform(-1, 1, n * batch) + 1j * rng.uniform(-1, 1, n * batch))
    spec = (np.fft.fft(taps.reshape(batch, n), axis=1) / n).astype(np.complex64)
    rev = oracle.rev_table(oracle.foursteps_chain(n, r_out, mid, 16), n)
    b_dr = np.ascontiguousarray(spec[:, rev]).ravel()
    aq, as_ = oracle.bfp_quantize(a, n)
    bq, bs = oracle.bfp_quantize(b_dr, n)
    # register-boundary layout: the int16 pairs of each mid-point chunk in bperm order
    bk = bq if lname == "R16" else _chunk_bperm(bq.view(np.int32).ravel(), mid, 16).view(np.int16).reshape(-1, 2)
    oq, os_ = ops.conv_large_bfp(_dev(aq), _dev(as_), _dev(bk), _dev(bs), n, layout, midop, r_out=r_out,
                                 mid_size=mid)
    got = oracle.bfp_dequantize(oq.cpu().numpy(), os_.cpu().numpy(), n)
    ad = oracle.bfp_dequantize(aq, as_, n).astype(np.complex128).reshape(batch, n)
    bd = oracle.bfp_dequantize(bq, bs, n).astype(np.complex128).reshape(batch, n)
    bnat = np.empty_like(bd)
    bnat[:, rev] = bd
    A = np.fft.fft(ad, axis=1)
    if midop == MID_MULTIPLY:
        want_f = oracle.conv_foursteps(oracle.bfp_dequantize(aq, as_, n), oracle.bfp_dequantize(bq, bs, n),
                                       n, r_out, mid, 16)
        wq, ws = oracle.bfp_quantize(want_f, n)
        assert rel_l2(got, oracle.bfp_dequantize(wq, ws, n)) <= BFP_TOL
        ref = np.fft.ifft(A * bnat, axis=1) * n
    elif midop == MID_CONJ:
        ref = np.fft.ifft(A * np.conj(bnat), axis=1) * n
    else:
        ref = ad * n
    assert rel_l2(got, ref.ravel()) < 1e-4
    # in place: the result may overwrite the signal
    if midop == MID_MULTIPLY:
        buf = _dev(aq)
        os2 = torch.empty(batch, dtype=torch.float32, device="cuda")
        ws_ = torch.empty(int(lib().fufft_conv_large_bfp_workspace(n, batch)), dtype=torch.uint8, device="cuda")
        bkd, asd, bsd = _dev(bk), _dev(as_), _dev(bs)
        rc = lib().fufft_conv_large_bfp(buf.data_ptr(), asd.data_ptr(), bkd.data_ptr(), bsd.data_ptr(),
                                        buf.data_ptr(), os2.data_ptr(), n, batch, r_out, mid, layout, midop,
                                        ws_.data_ptr(), ws_.numel(), None)
        assert rc == 0
        assert torch.equal(buf.cpu(), oq.cpu()) and torch.equal(os2.cpu(), os_.cpu())
    torch.cuda.synchronize()
    assert ops.device_status() == 0


def test_large_full_size_properties(ops):
    """config 5 (N=32768, batch 2048): identity filter and round trip, checked
    on the whole batch (size-independent properties)"""
    n, batch = 32768, 2048
    g = torch.Generator(device="cuda")
    g.manual_seed(5032768)
    a = torch.randn(n * batch, dtype=torch.complex64, device="cuda", generator=g)
    ident = torch.full((n * batch,), 1.0 / n, dtype=torch.complex64, device="cuda")   # DFT of a delta / n
    out = ops.conv_large(a.clone(), ident, n, ops.LAYOUT_R16)
    assert float((out - a).abs().pow(2).sum() / a.abs().pow(2).sum()) ** 0.5 < 2e-6
    rt = ops.conv_large(a.clone(), None, n, ops.LAYOUT_R16, MID_NONE)
    assert float((rt / n - a).abs().pow(2).sum() / a.abs().pow(2).sum()) ** 0.5 < 2e-6
    torch.cuda.synchronize()
    assert ops.device_status() == 0


@pytest.mark.parametrize("n,r_out,mid,lname", [(262144, 16, 1024, "R16"), (262144, 8, 4096, "R8"),
                                               (1 << 21, 16, 512, "R16_BPERM"), (1 << 21, 8, 4096, "R8")])
def test_large_multi_level_plans(ops, oracle, n, r_out, mid, lname):
    """two and three outer levels (radix 16 and 8): pairs of levels run as one
    fused pass, an odd level alone; fp32 and int16-BFP against the oracle's
    four-step on the same chain"""
    layout = getattr(ops, "LAYOUT_" + lname)
    mr = 16 if lname.startswith("R16") else 8
    batch = 2 if n <= 262144 else 1
    rng = np.random.default_rng(n + r_out)
    a = (rng.standard_normal(n * batch) + 1j * rng.standard_normal(n * batch)).astype(np.complex64)
    taps = rng.uniform(-1, 1, n * batch) + 1j * rng.uniform(-1, 1, n * batch)
    spec = (np.fft.fft(taps.reshape(batch, n), axis=1) / n).astype(np.complex64)
    rev = oracle.rev_table(oracle.foursteps_chain(n, r_out, mid, mr), n)
    b_dr = np.ascontiguousarray(spec[:, rev]).ravel()
    bk = _chunk_bperm(b_dr, mid, mr) if lname.endswith("BPERM") else b_dr
    want = oracle.conv_foursteps(a, b_dr, n, r_out, mid, mr)
    got = ops.conv_large(_dev(a), _dev(bk), n, layout, r_out=r_out, mid_size=mid).cpu().numpy()
    assert rel_l2(got, want) <= F32_TOL
    assert rel_l2(got[:n], oracle.conv_f64(a[:n], spec[0], n)) < 5e-6
    # int16-BFP on the same plan
    aq, as_ = oracle.bfp_quantize(a, n)
    bq, bs = oracle.bfp_quantize(b_dr, n)
    bqk = bq if not lname.endswith("BPERM") else \
        _chunk_bperm(bq.view(np.int32).ravel(), mid, mr).view(np.int16).reshape(-1, 2)
    want_f = oracle.conv_foursteps(oracle.bfp_dequantize(aq, as_, n), oracle.bfp_dequantize(bq, bs, n),
                                   n, r_out, mid, mr)
    wq, ws = oracle.bfp_quantize(want_f, n)
    oq, os_ = ops.conv_large_bfp(_dev(aq), _dev(as_), _dev(bqk), _dev(bs), n, layout, r_out=r_out, mid_size=mid)
    got = oracle.bfp_dequantize(oq.cpu().numpy(), os_.cpu().numpy(), n)
    assert rel_l2(got, oracle.bfp_dequantize(wq, ws, n)) <= BFP_TOL
    torch.cuda.synchronize()
    assert ops.device_status() == 0
