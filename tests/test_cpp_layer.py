"""The C++ policy-struct layer (include/fufft_b200.hpp) compiles against the
C ABI, and on a GPU a reference-style C++ caller reproduces the oracle."""
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "cpp", "reference_style_caller.cu")


def _build(tmp_path):
    exe = str(tmp_path / "caller")
    lib_dir = os.path.join(ROOT, "fufft_b200")
    r = subprocess.run(["nvcc", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-I",
                        os.path.join(ROOT, "include"), SRC, "-o", exe, "-L", lib_dir, "-lfufft_b200",
                        f"-Xlinker=-rpath={lib_dir}"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]
    return exe


def test_cpp_layer_compiles_and_links(tmp_path):
    assert os.path.exists(_build(tmp_path))


@pytest.mark.gpu
def test_cpp_layer_matches_oracle(tmp_path, oracle):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from oracle.oracle import MID_CONJ, rel_l2
    exe = _build(tmp_path)
    n, batch = 4096, 3
    a, b = oracle.gen_test(n, 1, batch)
    b8, b16 = oracle.permute_dr(b, n, 8), oracle.permute_dr(b, n, 16)
    for name, arr in [("a", a), ("b8", b8), ("b16", b16), ("bp16", oracle.bperm(b16, n, 16))]:
        arr.astype(np.complex64).tofile(tmp_path / f"{name}.bin")
    r = subprocess.run([exe, str(tmp_path)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    out = lambda k: np.fromfile(tmp_path / f"out_{k}.bin", dtype=np.complex64)   # noqa: E731
    assert rel_l2(out("ip"), oracle.conv(a, b8, n, 8)) <= 2e-6
    assert rel_l2(out("ip_conj"), oracle.conv(a, b8, n, 8, MID_CONJ)) <= 2e-6
    want16 = oracle.conv(a, b16, n, 16)
    assert rel_l2(out("v16"), want16) <= 2e-6 and rel_l2(out("v16f"), want16) <= 2e-6
    assert rel_l2(out("c2c"), oracle.c2c(a, n, -1, 16)) <= 2e-6
