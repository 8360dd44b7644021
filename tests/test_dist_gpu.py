"""The distributed single-signal convolution on 2, 4 and 8 GPUs, with the
all-to-alls through NCCL and fused into the outer passes as NVLink stores /
loads (p2p), against the host simulation of the same scheme
(oracle.conv_dist) and fp64.  Each world size is skipped when fewer GPUs are
visible."""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch

from oracle.oracle import rel_l2

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("mode", ["nccl", "p2p"])
@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("n", [1 << 16, 1 << 20])
def test_distributed_conv(oracle, tmp_path, n, world, mode):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    out = str(tmp_path / "y.npy")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           os.path.join(HERE, "dist_gpu_worker.py"), str(n), out, mode]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stderr[-3000:]
    got = np.load(out)
    info = np.load(out + ".plan.npy")
    chain = [int(v) for v in info[3:]]
    rng = np.random.default_rng(n + world)
    a = (rng.standard_normal(n) + 1j * rng.standard_normal(n)).astype(np.complex64)
    spec = (np.fft.fft(rng.uniform(-1, 1, n) + 1j * rng.uniform(-1, 1, n)) / n).astype(np.complex64)
    rev = oracle.rev_table(chain, n)
    one_kernel, r_out, mid = bool(info[0]), int(info[1]), int(info[2])
    want = oracle.conv_dist(a, spec[rev], n, world, r_out if not one_kernel else 16, mid)
    assert rel_l2(got, want) <= 2e-6
    assert rel_l2(got, oracle.conv_f64(a, spec, n)) < 5e-6
