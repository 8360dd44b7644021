"""Multi-GPU drivers over torch.distributed (one process per GPU, NCCL).

Batch sharding needs no code here: transforms are independent, so each rank
calls the single-GPU entry points on its own slice of the batch (bench.py
--gpus N).  This module holds the one case that does communicate: a SINGLE
n-point convolution spread over W = 2, 4 or 8 ranks (
n = 2^26 over 8 GPUs).  The reference is single-GPU (README.md:112); the
scheme follows its four-step decomposition with the first outer level split
across ranks:

  view x as [W][n/W]; rank g owns columns g*cols .. (g+1)*cols-1 of every
  row (cols = n/W^2), stored row by row ([W][cols])
  1. fufft_dist_pass(-1): this rank's share of the radix-W DIF pass at stride
     n/W (one butterfly group per column: no communication)
  2. all_to_all: row k of every rank -> rank k, which now holds block k
     (n/W points, columns in order)
  3. block k is an independent n/W-point transform: fused one-kernel or
     four-step convolution with block k of the chain-ordered filter
  4. all_to_all back, 5. fufft_dist_pass(+1): the radix-W DIT pass

The chain of the whole transform is [W] ++ (chain of the n/W block), and
block k of a filter in that chain order is exactly the block's own
chain-ordered filter, so each rank needs only its n/W filter slice.

Compute goes through a backend object (GPU: this library; the CPU tests plug
in the oracle), so the partition and exchange logic is tested under gloo.

conv_distributed_p2p is the same scheme with the all-to-alls fused into the
outer passes over NVLink peer memory: every rank's n/W block buffer is mapped
into all ranks (CUDA IPC, PeerBlocks); step 1+2 become one kernel that stores
row k's results straight into rank k's block (fufft_dist_pass_push), step 4+5
one kernel that loads them back from the blocks (fufft_dist_pass_pull).  The
ranks only synchronise (a one-element all-reduce on the stream) between the
phases; no signal data goes through NCCL.
"""
from __future__ import annotations

import ctypes as ct
from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass
class DistPlan:
    n: int
    world: int
    n_blk: int           # points per block (n / world)
    cols: int            # columns per rank (n / world^2)
    one_kernel: bool     # block fits the fused one-kernel convolution
    r_out: int           # four-step outer radix of the block (if not one_kernel)
    mid: int             # four-step middle of the block
    chain: list[int]     # radix chain of the whole transform (filter order)


def make_plan(n: int, world: int, max_one_kernel: int = 8192, large_plan=None, chain_of=None) -> DistPlan:
    if world not in (2, 4, 8):
        raise ValueError("the distributed convolution runs on 2, 4 or 8 ranks")
    if n & (n - 1) or n < world * world * 256:
        raise ValueError(f"n={n} must be a power of two >= {world * world * 256}")
    n_blk = n // world
    if n_blk <= max_one_kernel:
        blk_chain = chain_of(n_blk, 16)
        return DistPlan(n, world, n_blk, n_blk // world, True, 0, n_blk, [world] + blk_chain)
    r_out, mid = large_plan(n_blk)
    lout, q = 0, n_blk // mid
    while q > 1:
        q //= r_out
        lout += 1
    return DistPlan(n, world, n_blk, n_blk // world, False, r_out, mid, [world] + [r_out] * lout + chain_of(mid, 16))


class GpuBackend:
    """compute on this rank's GPU through libfufft_b200"""

    def __init__(self):
        from . import ops
        from ._lib import check, lib
        self.ops, self.check, self.lib = ops, check, lib

    def plan(self, n: int, world: int) -> DistPlan:
        return make_plan(n, world, self.ops.max_n(self.ops.LAYOUT_R16),
                         lambda m: self.ops.large_plan(m, self.ops.LAYOUT_R16), self.ops.chain)

    def dist_pass(self, x: torch.Tensor, world: int, cols: int, col0: int, n: int, sign: int) -> None:
        self.check(self.lib().fufft_dist_pass(x.data_ptr(), world, cols, col0, n, sign,
                                              torch.cuda.current_stream().cuda_stream), "fufft_dist_pass")

    def conv_block(self, block: torch.Tensor, b_block: torch.Tensor, plan: DistPlan) -> None:
        if plan.one_kernel:
            self.ops.conv(block, b_block, plan.n_blk, self.ops.LAYOUT_R16, out=block)
        else:
            self.ops.conv_large(block, b_block, plan.n_blk, self.ops.LAYOUT_R16, r_out=plan.r_out,
                                mid_size=plan.mid)


class _DeviceArray:
    """a device float32 array at a raw address, for torch.as_tensor"""

    def __init__(self, ptr: int, count: int):
        self.__cuda_array_interface__ = {"shape": (count,), "typestr": "<f4", "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerBlocks:
    """This rank's block buffer (n_blk complex points) and the mapping of every
    rank's one into this process; `block` is this rank's buffer as a complex64
    tensor, `addresses` the host array of the world block addresses."""

    def __init__(self, n_blk: int, group=None):
        from ._lib import check, lib
        self.L, self.check = lib(), check
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        own, handle = ct.c_void_p(), (ct.c_char * 64)()
        check(self.L.fufft_peer_alloc(n_blk * 8, ct.byref(own), handle), "fufft_peer_alloc")
        self.own = own.value
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.mapped, ptrs = [], []
        for k, h in enumerate(handles):
            if k == self.rank:
                ptrs.append(self.own)
                continue
            p = ct.c_void_p()
            check(self.L.fufft_peer_open(h, ct.byref(p)), "fufft_peer_open")
            self.mapped.append(p.value)
            ptrs.append(p.value)
        self.addresses = (ct.c_uint64 * self.world)(*ptrs)
        flat = torch.as_tensor(_DeviceArray(self.own, 2 * n_blk), device="cuda")
        self.block = torch.view_as_complex(flat.view(-1, 2))

    def close(self, group=None):
        """unmap the peers' buffers; once every rank has, free this rank's own
        (a collective call: every rank of the group makes it)"""
        torch.cuda.current_stream().synchronize()
        for p in self.mapped:
            self.check(self.L.fufft_peer_close(p), "fufft_peer_close")
        self.mapped = []
        dist.barrier(group=group)
        if self.own:
            self.block = None
            self.check(self.L.fufft_peer_free(self.own), "fufft_peer_free")
            self.own = 0


def _stream_barrier(group, flag: torch.Tensor) -> None:
    """every rank's earlier work on the current stream is done before its later work starts"""
    dist.all_reduce(flag, group=group)


def conv_distributed_p2p(x_local: torch.Tensor, b_block: torch.Tensor, n: int, peers: PeerBlocks,
                         backend=None, group=None, plan: DistPlan | None = None) -> torch.Tensor:
    """conv_distributed with the all-to-alls fused into the outer passes as
    NVLink stores / loads; same arguments plus the mapped block buffers"""
    backend = backend or GpuBackend()
    world, rank = peers.world, peers.rank
    plan = plan or backend.plan(n, world)
    if x_local.numel() != world * plan.cols or b_block.numel() != plan.n_blk or peers.block.numel() != plan.n_blk:
        raise ValueError("slice sizes do not match the plan")
    flag = torch.zeros(1, device=x_local.device)
    st = torch.cuda.current_stream().cuda_stream
    xp = torch.view_as_real(x_local).data_ptr() if x_local.is_complex() else x_local.data_ptr()
    backend.check(backend.lib().fufft_dist_pass_push(xp, peers.addresses, world, rank, plan.cols, n, st),
                  "fufft_dist_pass_push")
    _stream_barrier(group, flag)
    backend.conv_block(peers.block, b_block, plan)
    _stream_barrier(group, flag)
    backend.check(backend.lib().fufft_dist_pass_pull(xp, peers.addresses, world, rank, plan.cols, n, st),
                  "fufft_dist_pass_pull")
    _stream_barrier(group, flag)   # the peers are done reading this rank's block
    return x_local


def scatter_signal(x: torch.Tensor, n: int, world: int, rank: int) -> torch.Tensor:
    """this rank's [world][cols] slice of a global n-point signal"""
    cols = n // (world * world)
    return x.view(world, n // world)[:, rank * cols:(rank + 1) * cols].contiguous().view(-1)


def gather_signal(parts: list[torch.Tensor], n: int) -> torch.Tensor:
    """inverse of scatter_signal over all ranks' slices"""
    world = len(parts)
    return torch.cat([p.view(world, -1) for p in parts], dim=1).contiguous().view(-1)


def filter_block(b_chain: torch.Tensor, n: int, world: int, rank: int) -> torch.Tensor:
    """block `rank` of a filter in the whole transform's chain order"""
    blk = n // world
    return b_chain[rank * blk:(rank + 1) * blk].contiguous()


def _as_real(t: torch.Tensor) -> torch.Tensor:
    return torch.view_as_real(t).view(-1) if t.is_complex() else t


def conv_distributed(x_local: torch.Tensor, b_block: torch.Tensor, n: int, backend=None, group=None,
                     plan: DistPlan | None = None) -> torch.Tensor:
    """Cyclic convolution of one n-point signal held as [world][cols] slices on
    every rank of `group`; returns this rank's slice of the result (in place)."""
    backend = backend or GpuBackend()
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    plan = plan or backend.plan(n, world)
    if x_local.numel() != world * plan.cols or b_block.numel() != plan.n_blk:
        raise ValueError("slice sizes do not match the plan")
    col0 = rank * plan.cols
    backend.dist_pass(x_local, world, plan.cols, col0, n, -1)
    block = torch.empty_like(x_local)
    dist.all_to_all_single(_as_real(block), _as_real(x_local), group=group)
    backend.conv_block(block, b_block, plan)
    dist.all_to_all_single(_as_real(x_local), _as_real(block), group=group)
    backend.dist_pass(x_local, world, plan.cols, col0, n, +1)
    return x_local
