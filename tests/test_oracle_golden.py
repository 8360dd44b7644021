"""Pins the oracle (oracle/fufft_oracle.c) to the reference's own transcription.

Every case below is one of the reference's seeded tests (verify_kernel.cpp).
The fixtures in tests/golden/ were produced by the reference code itself
(tests/golden/make_golden.py over oracle/_ref); here the oracle regenerates
each input from the same seed and recomputes each output, and both must
match the recorded SHA-256 digests bit for bit.
"""
import hashlib
import json
import os
import sys

import numpy as np
import pytest

from oracle.oracle import MID_MULTIPLY, rel_l2

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
with open(os.path.join(GOLD, "reference_digests.json")) as f:
    DIG = json.load(f)


def _d(x):
    return hashlib.sha256(np.ascontiguousarray(x).tobytes()).hexdigest()


def _cases(prefix):
    return [k for k in DIG if k.startswith(prefix + "/")]


def test_reference_suite_passed_when_fixtures_were_made():
    assert DIG["suite_all_pass"] is True


@pytest.mark.parametrize("key", _cases("conv"))
def test_conv_family_bit_exact(oracle, key):
    _, n, cpb, batch = key.split("/")
    n, cpb, batch = int(n), int(cpb), int(batch)
    rec = DIG[key]
    a, b = oracle.gen_test(n, cpb, batch)
    assert _d(a) == rec["a"] and _d(b) == rec["b"], "seeded generator drifted"
    b8 = oracle.permute_dr(b, n, 8)
    ip = oracle.conv(a, b8, n, 8)
    assert _d(ip) == rec["ip"]
    assert _d(ip) == rec["fused"]          # register boundary == in-place, bit for bit
    spec = oracle.fwd(a, n, 8)
    assert _d(spec) == rec["fwd"]
    assert _d(oracle.apply(spec, b8, n, 8)) == rec["apply"]
    assert rec["apply"] == rec["ip"]       # split fwd/apply == fused
    if "v16" in rec:
        v16 = oracle.conv(a, oracle.permute_dr(b, n, 16), n, 16)
        assert _d(v16) == rec["v16"] == rec["v16f"]
    ref64 = oracle.conv_f64(a, b, n)
    assert rel_l2(ip, ref64) < 3e-6       # verify_kernel.cpp:1395


@pytest.mark.parametrize("key", _cases("bfp"))
def test_bfp_bit_exact(oracle, key):
    _, n, seed = key.split("/")
    n, seed = int(n), int(seed)
    rec = DIG[key]
    a, b = oracle.gen_bfp(n, seed)
    assert _d(a) == rec["a"] and _d(b) == rec["b"]
    aq, as_ = oracle.bfp_quantize(a, n)
    bq, bs = oracle.bfp_quantize(oracle.permute_dr(b, n, 16), n)
    assert _d(aq) == rec["aq"] and _d(as_) == rec["a_scale"]
    assert _d(bq) == rec["bq"] and _d(bs) == rec["b_scale"]
    oq, os_ = oracle.conv_bfp(aq, as_, bq, bs, n, 16)
    assert _d(oq) == rec["oq"] and _d(os_) == rec["o_scale"]
    got = oracle.bfp_dequantize(oq, os_, n)
    rel = rel_l2(got, oracle.conv_f64(a, b, n))
    assert rel < 3e-4 and -np.log2(rel) >= 12.0      # verify_kernel.cpp:1176


@pytest.mark.parametrize("key", _cases("r2"))
def test_r2_bit_exact(oracle, key):
    _, n, cpb, batch = key.split("/")
    n, batch = int(n), int(batch)
    rec = DIG[key]
    xr, yr, h = oracle.gen_r2_signals(n, batch)
    assert _d(xr) == rec["xr"] and _d(yr) == rec["yr"] and _d(h) == rec["h"]
    g = np.load(os.path.join(GOLD, "reference_cases.npz"))
    b_dr = g[key + "/b_dr"]                 # fp64 spectrum rounded by the reference
    assert _d(b_dr) == rec["b_dr"]
    ur, vr = oracle.conv_r2(xr, yr, b_dr, n, 8)
    assert _d(ur) == rec["ur"] and _d(vr) == rec["vr"]


@pytest.mark.parametrize("key", _cases("conv2d"))
def test_conv2d_bit_exact(oracle, key):
    _, h, w, batch = key.split("/")
    h, w, batch = int(h), int(w), int(batch)
    rec = DIG[key]
    a, b = oracle.gen_2d(h, w, batch)
    assert _d(a) == rec["a"] and _d(b) == rec["b"]
    rows = oracle.rev_table(oracle.chain(h, 8), h)
    cols = oracle.rev_table(oracle.chain(w, 8), w)
    b2 = np.ascontiguousarray(b.reshape(batch, h, w)[:, rows][:, :, cols]).ravel()
    assert _d(b2) == rec["b_dr"]
    out = oracle.conv2d_pow8(a, b2, h, w)
    assert _d(out) == rec["out"]
    assert rel_l2(out, oracle.conv2d_f64(a, b, h, w)) < 3e-6     # verify_kernel.cpp:786


@pytest.mark.parametrize("key", _cases("large"))
def test_foursteps_bit_exact(oracle, key):
    _, n, batch, r_out, mid, v16 = key.split("/")
    n, batch, r_out, mid, v16 = int(n), int(batch), int(r_out), int(mid), int(v16)
    rec = DIG[key]
    a, b = oracle.gen_large_cfg(n, batch, r_out, mid)
    assert _d(a) == rec["a"] and _d(b) == rec["b"]
    chain = oracle.foursteps_chain(n, r_out, mid, 16 if v16 else 8)
    b_dr = np.ascontiguousarray(b.reshape(batch, n)[:, oracle.rev_table(chain, n)]).ravel()
    assert _d(b_dr) == rec["b_dr"]
    mr = 16 if v16 else 8
    assert _d(oracle.conv_foursteps(a, b_dr, n, r_out, mid, mr)) == rec["four"]
    assert _d(oracle.conv_monolithic(a, b_dr, n, r_out, mid, mr)) == rec["mono"]


def test_small_case_arrays_match_digests():
    g = np.load(os.path.join(GOLD, "reference_cases.npz"))
    for k in g.files:
        case, name = k.rsplit("/", 1)
        assert _d(g[k]) == DIG[case][name], k


@pytest.mark.parametrize("radix", [8, 16])
@pytest.mark.parametrize("mid", [1, 2])
def test_oracle_apply_grid_r2_is_real_conv(oracle, radix, mid):
    """the grid checker for packed real pairs: fwd of xr + i*yr, then apply
    against each real filter, gives each real signal's cyclic convolution
    (mid 1) or correlation (mid 2) with each filter (float64 numpy)"""
    n, npair, nf = 512, 2, 3
    rng = np.random.default_rng(91 + radix + mid)
    x = rng.standard_normal((2 * npair, n)).astype(np.float32)
    taps = rng.uniform(-1.0, 1.0, (nf, n))
    b_nat = (np.fft.fft(taps, axis=1) / n).astype(np.complex64)
    spec = oracle.fwd((x[0::2] + 1j * x[1::2]).astype(np.complex64).reshape(-1), n, radix)
    b_dr = np.concatenate([oracle.permute_dr(b_nat[f], n, radix) for f in range(nf)])
    got = oracle.apply_grid_r2(spec, b_dr, n, radix, mid).reshape(2 * npair, nf, n)
    X = np.fft.fft(x.astype(np.float64), axis=1)
    for i in range(2 * npair):
        for f in range(nf):
            H = np.fft.fft(taps[f])
            ref = np.fft.ifft(X[i] * (np.conj(H) if mid == 2 else H)).real
            assert np.linalg.norm(got[i, f] - ref) / np.linalg.norm(ref) <= 2e-5


@pytest.mark.parametrize("n", [8, 64, 512, 4096])
def test_oracle_c2c_pinned_to_reference(oracle, n):
    """natural-order c2c: the oracle's restatement (its own DIF chain +
    chain_rev unscramble) against the reference's own kernel_c2c (radix-8
    Stockham, verify_kernel.cpp:1183-1201) from oracle/_ref, on the
    reference's seeded input (mt19937(N*131+CPB), verify_kernel.cpp:1277),
    and against float64; the inverse undoes the forward"""
    from oracle.oracle import Reference
    try:
        ref = Reference()
    except OSError:
        pytest.skip("oracle/_ref not built (the reference sources are absent)")
    batch = 3
    a, _ = oracle.gen_test(n, 1, batch)
    want = ref.c2c(a, n)
    for radix in (8, 16):
        if n < radix:
            continue
        got = oracle.c2c(a, n, -1, radix)
        assert rel_l2(got, want) <= 1e-6, radix
        back = oracle.c2c(got, n, +1, radix) / n
        assert rel_l2(back, a) <= 2e-6
    f64 = np.fft.fft(a.astype(np.complex128).reshape(batch, n), axis=1).ravel()
    assert rel_l2(want, f64) <= 2e-6


# ---- the reference's three CPU programs (cpu_fufft.cpp, cpu_inplace.cpp, cpu_mixed.cpp) ----
def _cpu_programs():
    from oracle.oracle import CpuPrograms
    try:
        return CpuPrograms()
    except (FileNotFoundError, OSError):
        pytest.skip("oracle/_ref/libfufft_cpuref.so not built (needs the reference tree)")


def test_cpu_program_fixtures_are_the_programs_outputs():
    """tests/golden/cpu_programs.npz holds what the compiled programs produce:
    the digests of their fp64 outputs on the recorded inputs match"""
    import hashlib
    import json
    import os
    sys_path = os.path.join(os.path.dirname(__file__), "golden")
    sys.path.insert(0, sys_path)
    try:
        import make_cpu_programs as mk
    finally:
        sys.path.remove(sys_path)
    p = _cpu_programs()
    with open(os.path.join(sys_path, "cpu_programs_digests.json")) as f:
        dig = json.load(f)
    assert all(rc == 0 for rc in dig["programs"].values())
    g = np.load(os.path.join(sys_path, "cpu_programs.npz"))
    for key, rec in mk.cases(p):
        for k, v in rec.items():
            if k in dig[key]:
                assert hashlib.sha256(np.ascontiguousarray(v).tobytes()).hexdigest() == dig[key][k], (key, k)
            assert np.array_equal(g[f"{key}/{k}"], v.astype(np.complex64)), (key, k)   # the stored arrays


def test_cpu_program_index_maps_bit_exact():
    """the digit reversal of cpu_inplace and the mixed-radix reversal and
    factorisation of cpu_mixed equal the library's chain and chain_rev for every
    index (the filter layouts R8 / R16)"""
    from fufft_b200 import ops
    p = _cpu_programs()
    for n in (8, 64, 512, 4096):
        s = {8: 1, 64: 2, 512: 3, 4096: 4}[n]
        want = np.array([p.digitrev8(i, s) for i in range(n)])
        assert np.array_equal(ops.chain_rev_table(ops.chain(n, 8)).numpy(), want), n
    for v in (8, 16):
        for n in (16, 32, 64, 128, 256, 512, 1024, 2048, 4096):
            if n < v:
                continue
            rad = p.mixed_factorise(n, v)
            assert rad == ops.chain(n, v), (n, v)
            want = np.array([p.mixed_rev(i, rad) for i in range(n)])
            assert np.array_equal(ops.chain_rev_table(rad).numpy(), want), (n, v)


def test_cpu_program_outputs_agree_with_fp64():
    """sanity of the fixtures: the programs' convolutions equal a float64
    numpy convolution of the same inputs"""
    import os
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "cpu_programs.npz"))
    keys = sorted({k.rsplit("/", 1)[0] for k in g.files})
    for key in keys:
        a, b = g[key + "/a"].astype(np.complex128), g[key + "/b"].astype(np.complex128)
        want = np.fft.ifft(np.fft.fft(a) * np.fft.fft(b))
        for out in ("conv64", "out64", "conv32", "out32"):
            if f"{key}/{out}" in g.files:
                assert rel_l2(g[f"{key}/{out}"], want) < (1e-6 if out.endswith("32") else 1e-7), (key, out)
