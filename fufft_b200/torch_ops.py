"""torch.ops registration of the library's main entry points.

``import fufft_b200.torch_ops`` registers, under the ``fufft`` namespace:

  torch.ops.fufft.conv(a, b, n, layout, mid, filter_stride) -> Tensor
  torch.ops.fufft.conv2d(a, b, h, w, layout, mid, filter_stride) -> Tensor
  torch.ops.fufft.c2c(a, n, sign) -> Tensor
  torch.ops.fufft.filter_from_taps(taps, n, layout) -> Tensor

Tensors are complex64 CUDA tensors (flat or any shape whose element count is
a whole number of transforms); every op returns a new tensor of a's shape and
launches exactly the kernels of the matching fufft_b200.ops call on the
current stream.  Each op has a fake (shape-only) implementation, so the ops
trace under torch.compile / torch.export and show up as single graph nodes;
they have no autograd formula.
"""
from __future__ import annotations

import torch

from . import ops

_NS = "fufft"


@torch.library.custom_op(f"{_NS}::conv", mutates_args=())
def conv(a: torch.Tensor, b: torch.Tensor | None, n: int, layout: int, mid: int, filter_stride: int) -> torch.Tensor:
    return ops.conv(a.contiguous().view(-1), None if b is None else b.contiguous().view(-1), n, layout, mid,
                    filter_stride=filter_stride).view(a.shape)


@conv.register_fake
def _(a, b, n, layout, mid, filter_stride):
    return torch.empty_like(a)


@torch.library.custom_op(f"{_NS}::conv2d", mutates_args=())
def conv2d(a: torch.Tensor, b: torch.Tensor | None, h: int, w: int, layout: int, mid: int,
           filter_stride: int) -> torch.Tensor:
    return ops.conv2d(a.contiguous().view(-1), None if b is None else b.contiguous().view(-1), h, w, layout, mid,
                      filter_stride=filter_stride).view(a.shape)


@conv2d.register_fake
def _(a, b, h, w, layout, mid, filter_stride):
    return torch.empty_like(a)


@torch.library.custom_op(f"{_NS}::c2c", mutates_args=())
def c2c(a: torch.Tensor, n: int, sign: int) -> torch.Tensor:
    return ops.c2c(a.contiguous().view(-1), n, sign).view(a.shape)


@c2c.register_fake
def _(a, n, sign):
    return torch.empty_like(a)


@torch.library.custom_op(f"{_NS}::filter_from_taps", mutates_args=())
def filter_from_taps(taps: torch.Tensor, n: int, layout: int) -> torch.Tensor:
    return ops.filter_from_taps(taps.contiguous().view(-1), n, layout).view(taps.shape)


@filter_from_taps.register_fake
def _(taps, n, layout):
    return torch.empty_like(taps)
