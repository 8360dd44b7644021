"""fufft_conv_multi_gpu on the GPU, through the C ABI.  Batch shards must give
the same bits as one single-GPU call over the whole batch (the same kernel
runs on every transform).  The single-signal mode must match the host
simulation of the same scheme (oracle.conv_dist) and fp64.  Shards go on
distinct GPUs when enough are visible, else they share cuda:0 (the phases are
ordered by events between streams, so that is a valid configuration too)."""
import numpy as np
import pytest
import torch

from oracle.oracle import rel_l2

pytestmark = pytest.mark.gpu


def _devices(k):
    cnt = torch.cuda.device_count()
    return [i if cnt >= k else 0 for i in range(k)]


def _data(n, batch, seed, device="cuda"):
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    a = torch.randn(batch * n, dtype=torch.complex64, generator=g)
    b = torch.randn(batch * n, dtype=torch.complex64, generator=g) / n
    return a.to(device), b.to(device)


@pytest.mark.parametrize("n,layout", [(4096, 3), (1024, 2), (32768, 2)])
def test_batch_shards_equal_one_call(n, layout):
    from fufft_b200 import ops
    from fufft_b200.multi_gpu import MG_BATCH, Shard, run
    ops.init()
    batch, k = 24, 3
    a, b = _data(n, batch, 11)
    want = ops.conv(a, b, n, layout)
    devs = _devices(k)
    per = batch // k
    streams = [torch.cuda.Stream(device=d) for d in devs]
    parts_a = [a[i * per * n:(i + 1) * per * n].to(f"cuda:{d}") for i, d in enumerate(devs)]
    parts_b = [b[i * per * n:(i + 1) * per * n].to(f"cuda:{d}") for i, d in enumerate(devs)]
    outs = [torch.empty_like(p) for p in parts_a]
    for d in set(devs):
        torch.cuda.synchronize(d)
    for _ in range(2):
        shards = [Shard(d, s.cuda_stream, pa.data_ptr(), pb.data_ptr(), o.data_ptr(), per, None, 0)
                  for d, s, pa, pb, o in zip(devs, streams, parts_a, parts_b, outs)]
        run(MG_BATCH, shards, n, layout, ops.MID_MULTIPLY, n)
        for d in set(devs):
            torch.cuda.synchronize(d)
        got = torch.cat([o.to("cuda:0") for o in outs])
        assert torch.equal(got, want)
    assert torch.cuda.current_device() == 0


def test_batch_host_equals_device_call():
    from fufft_b200 import ops
    from fufft_b200.multi_gpu import conv_batch_host
    ops.init()
    n, batch = 4096, 40
    a, b = _data(n, batch, 12, "cpu")
    a, b = a.pin_memory(), b.pin_memory()
    out = torch.empty_like(a).pin_memory()
    want = ops.conv(a.cuda(), b.cuda(), n, ops.LAYOUT_R16_BPERM).cpu()
    devs = _devices(2)
    ws = conv_batch_host(a, b, out, n, devs, ops.LAYOUT_R16_BPERM)
    for d in set(devs):
        torch.cuda.synchronize(d)
    assert torch.equal(out, want)
    shared = b[:n].clone().pin_memory()       # one filter for every transform
    want = ops.conv(a.cuda(), shared.cuda(), n, ops.LAYOUT_R16_BPERM, filter_stride=0).cpu()
    ws = conv_batch_host(a, shared, out, n, devs, ops.LAYOUT_R16_BPERM, filter_stride=0)
    for d in set(devs):
        torch.cuda.synchronize(d)
    assert torch.equal(out, want)
    del ws


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("n", [1 << 16, 1 << 20])
def test_single_signal(oracle, n, world):
    from fufft_b200 import ops
    from fufft_b200.distributed import filter_block, gather_signal, scatter_signal
    from fufft_b200.multi_gpu import conv_single_signal, mg_chain
    ops.init()
    chain = mg_chain(n, world)
    rng = np.random.default_rng(n + world)
    a = (rng.standard_normal(n) + 1j * rng.standard_normal(n)).astype(np.complex64)
    spec = (np.fft.fft(rng.uniform(-1, 1, n) + 1j * rng.uniform(-1, 1, n)) / n).astype(np.complex64)
    b_chain = torch.from_numpy(np.ascontiguousarray(spec[oracle.rev_table(chain, n)]))
    devs = _devices(world)
    blocks_f = [filter_block(b_chain, n, world, r).to(f"cuda:{d}") for r, d in enumerate(devs)]
    blocks = None
    for _ in range(2):     # the work buffers are reused by consecutive calls
        slices = [scatter_signal(torch.from_numpy(a), n, world, r).to(f"cuda:{d}") for r, d in enumerate(devs)]
        blocks = conv_single_signal(slices, blocks_f, n, blocks)
        for d in set(devs):
            torch.cuda.synchronize(d)
        assert ops.device_status() == 0
        got = gather_signal([s.cpu() for s in slices], n).numpy()
        n_blk = n // world
        one_kernel = n_blk <= ops.max_n(ops.LAYOUT_R16)
        r_out, mid = (16, n_blk) if one_kernel else ops.large_plan(n_blk, ops.LAYOUT_R16)
        want = oracle.conv_dist(a, spec[oracle.rev_table(chain, n)], n, world, r_out, mid)
        assert rel_l2(got, want) <= 2e-6
        assert rel_l2(got, oracle.conv_f64(a, spec, n)) < 5e-6
