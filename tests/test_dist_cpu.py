"""Host-side logic of the distributed single-signal convolution
(fufft_b200.distributed) on CPU ranks over gloo: partition of the signal into
[world][cols] slices, the two all-to-alls, filter blocks and the plan.  The
local compute steps run through the oracle (same arithmetic as
oracle.conv_dist, the host simulation of the whole scheme), so the gathered
result must equal the simulation bit for bit and the fp64 convolution to
5e-6."""
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


class OracleBackend:
    def __init__(self):
        from fufft_b200 import ops
        from fufft_b200.distributed import make_plan
        from oracle.oracle import Oracle
        self.o, self.ops, self.make_plan = Oracle(), ops, make_plan

    def plan(self, n, world):
        # the library's own host-side planners (no GPU needed)
        return self.make_plan(n, world, 8192, lambda m: self.ops.large_plan(m, self.ops.LAYOUT_R16), self.ops.chain)

    def dist_pass(self, x, world, cols, col0, n, sign):
        x.copy_(torch.from_numpy(self.o.dist_pass(x.numpy(), world, cols, col0, n, sign)))

    def conv_block(self, block, b_block, plan):
        if plan.one_kernel:
            r = self.o.conv(block.numpy(), b_block.numpy(), plan.n_blk, 16)
        else:
            r = self.o.conv_foursteps(block.numpy(), b_block.numpy(), plan.n_blk, plan.r_out, plan.mid, 16)
        block.copy_(torch.from_numpy(r))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _inputs(n, seed):
    rng = np.random.default_rng(seed)
    a = (rng.standard_normal(n) + 1j * rng.standard_normal(n)).astype(np.complex64)
    taps = rng.uniform(-1, 1, n) + 1j * rng.uniform(-1, 1, n)
    spec = (np.fft.fft(taps) / n).astype(np.complex64)
    return a, spec


def _worker(rank, world, port, n, out_path):
    import datetime
    from fufft_b200.distributed import conv_distributed, filter_block, scatter_signal
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        be = OracleBackend()
        plan = be.plan(n, world)
        a, spec = _inputs(n, n + world)
        rev = be.o.rev_table(plan.chain, n)
        b_chain = torch.from_numpy(np.ascontiguousarray(spec[rev]))
        x = scatter_signal(torch.from_numpy(a), n, world, rank)
        y = conv_distributed(x, filter_block(b_chain, n, world, rank), n, backend=be, plan=plan)
        parts = [torch.empty_like(torch.view_as_real(y)) for _ in range(world)]
        dist.all_gather(parts, torch.view_as_real(y))
        if rank == 0:
            from fufft_b200.distributed import gather_signal
            full = gather_signal([torch.view_as_complex(p) for p in parts], n)
            np.save(out_path, full.numpy())
            np.save(out_path + ".plan.npy", np.array([plan.one_kernel, plan.r_out, plan.mid, *plan.chain]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n", [(2, 4096), (4, 16384), (2, 65536)])
def test_distributed_conv_on_cpu_ranks(oracle, world, n):
    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "y.npy")
        mp.spawn(_worker, args=(world, _free_port(), n, out), nprocs=world, join=True)
        got = np.load(out)
        info = np.load(out + ".plan.npy")
    from oracle.oracle import rel_l2
    a, spec = _inputs(n, n + world)
    chain = [int(v) for v in info[3:]]
    rev = oracle.rev_table(chain, n)
    one_kernel, r_out, mid = bool(info[0]), int(info[1]), int(info[2])
    want = oracle.conv_dist(a, spec[rev], n, world, r_out if not one_kernel else 16, mid)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert rel_l2(got, oracle.conv_f64(a, spec, n)) < 5e-6


def test_plan_and_partition_helpers():
    from fufft_b200 import ops
    from fufft_b200.distributed import gather_signal, make_plan, scatter_signal
    p = make_plan(1 << 26, 8, 8192, lambda m: ops.large_plan(m, ops.LAYOUT_R16), ops.chain)
    assert (p.n_blk, p.cols, p.one_kernel) == (1 << 23, 1 << 20, False)
    assert p.chain[0] == 8 and np.prod(p.chain) == 1 << 26
    x = torch.arange(4096, dtype=torch.float32)
    parts = [scatter_signal(x, 4096, 4, r) for r in range(4)]
    assert torch.equal(gather_signal(parts, 4096), x)
    with pytest.raises(ValueError):
        make_plan(1 << 20, 3, 8192, None, ops.chain)
