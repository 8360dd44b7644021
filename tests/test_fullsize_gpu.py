"""Parity at the benchmarked configurations themselves (
N = 512 .. 4096 with the signal filling 1 GiB, batch = 2^27 / N).

Each test builds the inputs exactly as bench.py does (bench.make_inputs: the
same seeds, the library's own forward transform for the filter spectra), runs
the same launch the bench times over the WHOLE batch (so the L2 prefetch one
wave ahead and the many waves of the direct-filter kernel are exercised),
then checks the first, the last and 256 seeded-random transforms:

  * fp32, register-boundary filter (the headline launch): against the
    reference's own transcription kernel_pipeline_v16f (oracle/_ref,
    verify_kernel.cpp:1012) when it is built, and always against the oracle
    port (pinned bit-exact to it); rel L2 <= 2e-6; and against float64
    (< 3e-6, the reference's own bound, verify_kernel.cpp:1395);
  * int16-BFP, linear filter (the bfp leg of the bench): device pack
    bit-exact against bfp_quantize; output against the reference's BFP
    pipeline (bfp_quantize + kernel_v16_bfp, verify_kernel.cpp:1092, :1109)
    at rel L2 <= 6e-5, and the mantissa / scale statistics the BFP parity
    contract asks to report: max |dq| in LSBs and the fraction of mantissas and
    scales that differ (printed; run with -s to see them).
"""
import numpy as np
import pytest
import torch

from oracle.oracle import MID_MULTIPLY, rel_l2

pytestmark = pytest.mark.gpu
F32_TOL = 2e-6
BFP_TOL = 6e-5
POINTS = 1 << 27


@pytest.fixture(scope="module")
def env():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import bench
    from fufft_b200 import ops
    ops.init()
    try:
        from oracle.oracle import Reference
        ref = Reference()
    except (FileNotFoundError, OSError):
        ref = None
    return ops, bench, ref


def _rows(batch, seed, k=256):
    rng = np.random.default_rng(seed)
    return np.unique(np.concatenate([[0, batch - 1], rng.choice(batch, k, replace=False)]))


def _take(t, idx, n, per=1):
    """rows idx of a device tensor holding transforms of n points (per values each)"""
    ii = torch.from_numpy(idx).to(t.device)
    return t.view(-1, n * per)[ii].reshape(-1).cpu().numpy()


def _unbperm(bp, n, v=16):
    """register-boundary order -> chain order: chain[v*L + k] = bperm[L + k*T]"""
    return np.ascontiguousarray(bp.reshape(-1, v, n // v).transpose(0, 2, 1).reshape(-1))


@pytest.mark.parametrize("n", [512, 1024, 2048, 4096])
def test_fullsize_fp32_headline_launch(env, oracle, n):
    ops, bench, ref = env
    batch = POINTS // n
    dev = torch.device("cuda", torch.cuda.current_device())
    a, spec, bperm = bench.make_inputs(ops, torch, n, batch, 1000 * 2 + n, dev)
    out = torch.empty_like(a)
    for _ in range(2):                       # two launches back to back, as the bench's loop
        ops.conv(a, bperm, n, ops.LAYOUT_R16_BPERM, ops.MID_MULTIPLY, out=out)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    idx = _rows(batch, n)
    ar, bpr, got = _take(a, idx, n), _take(bperm, idx, n), _take(out, idx, n)
    chain = _unbperm(bpr, n)
    assert np.array_equal(chain, _take(spec, idx, n))
    want = oracle.conv(ar, chain, n, 16, MID_MULTIPLY)
    e = rel_l2(got, want)
    assert e <= F32_TOL, (n, e)
    if ref is not None:
        e_ref = rel_l2(got, ref.pipeline_v16f(ar, bpr, n))
        assert e_ref <= F32_TOL, (n, e_ref)
    # float64 ground truth on the natural-order spectrum
    nat = np.empty_like(chain).reshape(-1, n)
    nat[:, ops.chain_rev_table(ops.chain(n, 16)).numpy()] = chain.reshape(-1, n)
    e64 = rel_l2(got, oracle.conv_f64(ar, nat.ravel(), n))
    assert e64 < 3e-6, (n, e64)
    print(f"\nfull-size fp32 N={n} batch={batch}: {idx.size} transforms checked, rel L2 vs oracle {e:.3g}"
          + (f", vs reference {e_ref:.3g}" if ref is not None else "") + f", vs fp64 {e64:.3g}")


@pytest.mark.parametrize("n", [512, 1024, 2048, 4096])
def test_fullsize_bfp_bench_launch(env, oracle, n):
    ops, bench, ref = env
    batch = POINTS // n
    dev = torch.device("cuda", torch.cuda.current_device())
    a, spec, bperm = bench.make_inputs(ops, torch, n, batch, 1000 * 2 + n, dev)
    del bperm
    aq, as_ = ops.bfp_pack(a, n)
    bq, bs = ops.bfp_pack(spec, n)
    oq, os_ = ops.conv_bfp(aq, as_, bq, bs, n, ops.LAYOUT_R16, ops.MID_MULTIPLY)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    idx = _rows(batch, n + 1)
    ar, sr = _take(a, idx, n), _take(spec, idx, n)
    aqr, bqr, oqr = (_take(t, idx, n, 2).reshape(-1, 2) for t in (aq, bq, oq))
    asr, bsr, osr = (t[torch.from_numpy(idx).to(t.device)].cpu().numpy() for t in (as_, bs, os_))
    # the device pack is bit-exact against the reference's quantiser
    wq, ws = oracle.bfp_quantize(ar, n)
    assert np.array_equal(aqr, wq) and np.array_equal(asr.view(np.uint32), ws.view(np.uint32))
    wq, ws = oracle.bfp_quantize(sr, n)
    assert np.array_equal(bqr, wq) and np.array_equal(bsr.view(np.uint32), ws.view(np.uint32))
    # output against the reference's BFP pipeline on the same quantised inputs
    wq, ws = oracle.conv_bfp(aqr, asr, bqr, bsr, n, 16, MID_MULTIPLY)
    if ref is not None:      # the reference's own code, one transform at a time
        for i in range(idx.size):
            rq, rs = ref.v16_bfp(aqr[i * n:(i + 1) * n], asr[i], bqr[i * n:(i + 1) * n], bsr[i], n)
            assert np.array_equal(rq, wq[i * n:(i + 1) * n]) and rs == ws[i]   # port == reference
    got = oracle.bfp_dequantize(oqr, osr, n)
    e = rel_l2(got, oracle.bfp_dequantize(wq, ws, n))
    assert e <= BFP_TOL, (n, e)
    dq = np.abs(oqr.astype(np.int32) - wq.astype(np.int32))
    mism = float(np.count_nonzero(dq)) / dq.size
    scale_mism = float(np.count_nonzero(osr.view(np.uint32) != ws.view(np.uint32))) / osr.size
    scale_rel = float(np.max(np.abs(osr.astype(np.float64) / ws - 1.0)))
    assert dq.max() <= 2, dq.max()
    print(f"\nfull-size int16-BFP N={n} batch={batch}: {idx.size} transforms checked, rel L2 vs reference "
          f"pipeline {e:.3g}, max |dq| {int(dq.max())} LSB, mantissas differing {mism:.4%}, scales differing "
          f"{scale_mism:.2%} (max rel {scale_rel:.2g})")
