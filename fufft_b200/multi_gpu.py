"""Several GPUs from one process: ctypes front end of fufft_conv_multi_gpu.

The library enqueues every shard's work on a stream of that shard's GPU and
returns without waiting; these helpers use torch's current stream of each
device, so a torch.cuda.synchronize(device) per device (or a later op on those
streams) sees the results.

* conv_batch / conv_batch_host: independent transforms split over GPUs (device
  tensors already on each GPU, or pinned host tensors cut into per-GPU slices
  that each GPU's own PCIe link carries).
* conv_single_signal: one n-point signal over 2, 4 or 8 shards, the all-to-alls
  done as NVLink peer stores and loads inside the outer passes.  Shards may
  share a GPU (the phases are ordered by events between the streams).

The one-process-per-GPU form of the single-signal case, over
torch.distributed, is fufft_b200.distributed.
"""
from __future__ import annotations

import ctypes as ct

import torch

from ._lib import LAYOUT_R16_BPERM, MID_MULTIPLY, check, lib
from .ops import _batch, _complex, _hptr, _ptr, conv_host_workspace

MG_BATCH, MG_BATCH_HOST, MG_SINGLE_SIGNAL = 0, 1, 2


class Shard(ct.Structure):
    _fields_ = [("device", ct.c_int), ("stream", ct.c_void_p), ("a", ct.c_void_p), ("b", ct.c_void_p),
                ("out", ct.c_void_p), ("batch", ct.c_int64), ("workspace", ct.c_void_p),
                ("workspace_bytes", ct.c_size_t)]


class Desc(ct.Structure):
    _fields_ = [("mode", ct.c_int), ("n_shards", ct.c_int), ("shards", ct.POINTER(Shard)), ("n", ct.c_int64),
                ("layout", ct.c_int), ("mid", ct.c_int), ("filter_stride", ct.c_int64)]


def run(mode: int, shards: list[Shard], n: int, layout: int = LAYOUT_R16_BPERM, mid: int = MID_MULTIPLY,
        filter_stride: int = 0) -> None:
    """fufft_conv_multi_gpu on prepared shard records"""
    arr = (Shard * len(shards))(*shards)
    desc = Desc(mode, len(shards), ct.cast(arr, ct.POINTER(Shard)), n, layout, mid, filter_stride)
    check(lib().fufft_conv_multi_gpu(ct.byref(desc)), "fufft_conv_multi_gpu")


def _stream_of(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def mg_chain(n: int, world: int) -> list[int]:
    """radix chain of the single-signal transform ([world] ++ the block's chain)"""
    buf = (ct.c_int * 32)()
    k = lib().fufft_mg_chain(n, world, buf)
    if k < 0:
        raise ValueError(f"no single-signal plan for n={n} over {world} ranks")
    return list(buf[:k])


def conv_batch(a: list[torch.Tensor], b: list[torch.Tensor | None], out: list[torch.Tensor], n: int,
               layout: int = LAYOUT_R16_BPERM, mid: int = MID_MULTIPLY, filter_stride: int | None = None) -> None:
    """shard i: out[i] = conv(a[i], b[i]) on a[i]'s GPU (independent transforms)"""
    shards = []
    for ai, bi, oi in zip(a, b, out, strict=True):
        ai, oi = _complex(ai), _complex(oi)
        bt = None if bi is None else _complex(bi)
        shards.append(Shard(ai.device.index, _stream_of(ai.device), _ptr(ai), _ptr(bt), _ptr(oi), _batch(ai, n),
                            None, 0))
    run(MG_BATCH, shards, n, layout, mid, n if filter_stride is None else filter_stride)


def conv_batch_host(a: torch.Tensor, b: torch.Tensor | None, out: torch.Tensor, n: int, devices: list[int],
                    layout: int = LAYOUT_R16_BPERM, mid: int = MID_MULTIPLY, filter_stride: int | None = None,
                    workspaces: list[torch.Tensor] | None = None) -> list[torch.Tensor]:
    """pinned host batch split into len(devices) contiguous slices, each
    through its GPU's upload / convolve / download pipeline; returns the
    per-GPU workspaces (keep them alive until the streams are done)"""
    a, out = _complex(a), _complex(out)
    bt = None if b is None else _complex(b)
    batch = _batch(a, n)
    fs = (n if bt is None or bt.numel() > n else 0) if filter_stride is None else filter_stride
    per = -(-batch // len(devices))
    shards, ws = [], []
    for i, d in enumerate(devices):
        t0, t1 = min(i * per, batch), min((i + 1) * per, batch)
        cnt = t1 - t0
        w = workspaces[i] if workspaces else conv_host_workspace(n, max(cnt, 1), fs, torch.device("cuda", d))
        ws.append(w)
        bi = None if bt is None else (bt[t0 * n:t1 * n] if fs == n else bt)
        shards.append(Shard(d, _stream_of(torch.device("cuda", d)), _hptr(a[t0 * n:t1 * n]), _hptr(bi),
                            _hptr(out[t0 * n:t1 * n]), cnt, _ptr(w), w.numel()))
    run(MG_BATCH_HOST, shards, n, layout, mid, fs)
    return ws


def conv_single_signal(slices: list[torch.Tensor], b_blocks: list[torch.Tensor | None], n: int,
                       blocks: list[torch.Tensor] | None = None, mid: int = MID_MULTIPLY) -> list[torch.Tensor]:
    """one n-point convolution: slices[r] is rank r's [world][n/world^2] slice
    (convolved in place), b_blocks[r] block r of the filter in the order of
    mg_chain(n, world).  blocks: per-rank n/world-point work buffers on the
    slices' GPUs (allocated when None).  Returns the blocks (keep them alive
    until the streams are done)."""
    world = len(slices)
    blocks = blocks or [torch.empty(n // world, dtype=torch.complex64, device=s.device) for s in slices]
    shards = []
    for s, bb, blk in zip(slices, b_blocks, blocks, strict=True):
        s, blk = _complex(s), _complex(blk)
        bt = None if bb is None else _complex(bb)
        shards.append(Shard(s.device.index, _stream_of(s.device), None, _ptr(bt), _ptr(s), 0, _ptr(blk),
                            blk.numel() * 8))
    run(MG_SINGLE_SIGNAL, shards, n, LAYOUT_R16_BPERM, mid, 0)
    return blocks
