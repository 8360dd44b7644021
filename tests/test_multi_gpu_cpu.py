"""fufft_conv_multi_gpu / fufft_mg_chain on the host side: the single-signal
radix chain agrees with the torch.distributed driver's plan, and every
argument the call does not take is rejected with a status code before any
device call (so these run without a GPU)."""
import ctypes as ct

import pytest

OK, SIZE, BATCH, MISALIGNED, CUDA, TIMEOUT, PEER, ARG, UNSUP = range(9)
P = 1 << 20        # a fake, 16-byte aligned address: never dereferenced by these calls


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("log_n", [16, 18, 20, 23, 26])
def test_chain_matches_distributed_plan(world, log_n):
    from fufft_b200 import ops
    from fufft_b200.distributed import make_plan
    from fufft_b200.multi_gpu import mg_chain
    n = 1 << log_n
    plan = make_plan(n, world, ops.max_n(ops.LAYOUT_R16), lambda m: ops.large_plan(m, ops.LAYOUT_R16), ops.chain)
    assert mg_chain(n, world) == plan.chain
    prod = 1
    for r in plan.chain:
        prod *= r
    assert prod == n


def test_chain_rejects_unsupported_shapes():
    from fufft_b200._lib import lib
    buf = (ct.c_int * 32)()
    assert lib().fufft_mg_chain(1 << 20, 3, buf) == -1
    assert lib().fufft_mg_chain((1 << 20) + 1, 2, buf) == -1
    assert lib().fufft_mg_chain(512, 2, buf) == -1          # below world^2 * 256
    assert lib().fufft_mg_chain(1 << 20, 2, None) == -1


def _call(mode, shards, n, layout=3, mid=1, fs=0, desc_shards=None, n_shards=None):
    from fufft_b200._lib import lib
    from fufft_b200.multi_gpu import Desc, Shard
    arr = (Shard * max(len(shards), 1))(*shards)
    d = Desc(mode, len(shards) if n_shards is None else n_shards,
             ct.cast(arr, ct.POINTER(Shard)) if desc_shards is None else desc_shards, n, layout, mid, fs)
    return lib().fufft_conv_multi_gpu(ct.byref(d))


def test_rejected_before_device():
    from fufft_b200._lib import lib
    from fufft_b200.multi_gpu import MG_BATCH, MG_BATCH_HOST, MG_SINGLE_SIGNAL, Shard
    assert lib().fufft_conv_multi_gpu(None) == ARG
    one = [Shard(0, None, P, P, P, 4, None, 0)]
    assert _call(MG_BATCH, one, 4096, n_shards=0) == ARG
    assert _call(MG_BATCH, one, 4096, n_shards=65) == ARG
    assert _call(7, one, 4096) == ARG                                     # unknown mode
    assert _call(MG_BATCH, one, 4096, mid=5) == ARG
    assert _call(MG_BATCH, [Shard(-1, None, P, P, P, 4, None, 0)], 4096) == ARG
    assert _call(MG_BATCH, one, 4096, layout=9) == ARG
    assert _call(MG_BATCH, one, 3000) == SIZE
    assert _call(MG_BATCH_HOST, one, 1 << 17) == SIZE
    assert _call(MG_BATCH, [Shard(0, None, P, P, P, -1, None, 0)], 4096) == BATCH
    n, world = 1 << 20, 2
    ws = (n // world) * 8
    ranks = [Shard(0, None, None, P, P, 0, P, ws) for _ in range(world)]
    assert _call(MG_SINGLE_SIGNAL, ranks + [ranks[0]], n) == UNSUP       # 3 ranks
    assert _call(MG_SINGLE_SIGNAL, ranks, n + 1) == SIZE
    assert _call(MG_SINGLE_SIGNAL, ranks, 512) == SIZE
    assert _call(MG_SINGLE_SIGNAL, [Shard(0, None, P + 64, P, P, 0, P, ws), ranks[1]], n) == ARG   # a != out
    assert _call(MG_SINGLE_SIGNAL, [Shard(0, None, None, P, P, 0, P, ws - 8), ranks[1]], n) == ARG
    assert _call(MG_SINGLE_SIGNAL, [Shard(0, None, None, None, P, 0, P, ws), ranks[1]], n) == ARG  # no filter
    assert _call(MG_SINGLE_SIGNAL, [Shard(0, None, None, P, P + 8, 0, P, ws), ranks[1]], n) == MISALIGNED
    assert _call(MG_SINGLE_SIGNAL, [Shard(0, None, None, P, P, 0, None, ws), ranks[1]], n) == ARG
