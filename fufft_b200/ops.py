"""Python mirror of the reference's entry points over the C ABI.

The reference (weiwang217/FuFFT, fufft.cuh) exposes kernel templates that the
caller launches with a mid-op policy struct; here each becomes a function over
CUDA tensors that calls the corresponding C entry point on the current torch
stream.  Names follow the reference:

    pipeline_ip(a, b_dr)        fufft_pipeline_ip   (radix-8 chain, any mid-op)
    pipeline_fused(a, bperm)    fufft_pipeline_fused (radix-8 register boundary)
    pipeline_v16(a, b16)        fufft_pipeline_v16  (radix-16 chain)
    pipeline_v16f(a, bperm16)   fufft_pipeline_v16f (radix-16 register boundary)
    pipeline_r16(a, b16)        fufft_pipeline_r16  (same math as v16)
    pipeline_fwd / pipeline_apply   split forward / apply
    conv_r2                     fufft_conv_r2 (two-for-one real)
    pipeline_v16_bfp            fufft_pipeline_v16_bfp (int16 BFP)

Complex data: torch.complex64 (or float32 with a trailing dim of 2), one
transform per row of n points.  int16 BFP data: torch.int16 with a trailing
dim of 2 (re, im) plus one float32 scale per transform.
"""
from __future__ import annotations

import ctypes as ct

import torch

from ._lib import (LAYOUT_NATURAL, LAYOUT_R8, LAYOUT_R8_BPERM, LAYOUT_R16, LAYOUT_R16_BPERM,
                   MID_CONJ_MULTIPLY, MID_MULTIPLY, MID_NONE, FufftError, check, lib)

__all__ = [
    "MID_NONE", "MID_MULTIPLY", "MID_CONJ_MULTIPLY",
    "LAYOUT_R8", "LAYOUT_R8_BPERM", "LAYOUT_R16", "LAYOUT_R16_BPERM", "LAYOUT_NATURAL",
    "FufftError", "chain", "chain_rev", "chain_rev_table", "filter_permute", "filter_permute_host", "filter_permute2d", "conv",
    "conv2d", "fwd", "apply",
    "conv_r2", "bfp_pack", "bfp_unpack", "conv_bfp", "pipeline_ip", "pipeline_fused", "pipeline_v16",
    "pipeline_v16f", "pipeline_r16", "pipeline_fwd", "pipeline_apply", "pipeline_v16_bfp", "init",
    "device_status", "launch_count", "max_n", "large_plan", "conv_large", "conv_large_bfp",
]


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _hptr(t: torch.Tensor | None):
    """address of a contiguous HOST tensor"""
    if t is None:
        return None
    if t.is_cuda or not t.is_contiguous():
        raise ValueError("expected a contiguous host tensor")
    return t.data_ptr()


def _ptr(t: torch.Tensor | None):
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("fufft_b200 operates on CUDA tensors")
    if not t.is_contiguous():
        raise ValueError("tensor must be contiguous")
    return t.data_ptr()


def _complex(t: torch.Tensor) -> torch.Tensor:
    if t.dtype == torch.complex64:
        return t
    if t.dtype == torch.float32 and t.shape[-1] == 2:
        return torch.view_as_complex(t)
    raise TypeError("complex data must be complex64 (or float32 [..., 2])")


def _batch(t: torch.Tensor, n: int, per_point: int = 1) -> int:
    total = t.numel() // per_point
    if total % n:
        raise ValueError(f"{total} points is not a whole number of transforms of {n}")
    return total // n


# ---- library / index maps ---------------------------------------------------
def init() -> None:
    check(lib().fufft_init(), "fufft_init")


def max_n(layout: int) -> int:
    return lib().fufft_max_n(layout)


def launch_count() -> int:
    return int(lib().fufft_launch_count())


def device_status() -> int:
    v = ct.c_uint32()
    check(lib().fufft_device_status(ct.byref(v), _stream()), "fufft_device_status")
    return v.value


def chain(n: int, radix: int) -> list[int]:
    buf = (ct.c_int * 32)()
    p = lib().fufft_chain(n, radix, buf)
    if p < 0:
        raise ValueError(f"n={n} radix={radix}")
    return list(buf[:p])


def chain_rev(idx: int, radices) -> int:
    arr = (ct.c_int * len(radices))(*radices)
    return int(lib().fufft_chain_rev(idx, arr, len(radices)))


def chain_rev_table(radices, device=None) -> torch.Tensor:
    """natural (frequency) index of every chain position of the radix chain
    `radices` (pass 0 first), as an int64 tensor: the digits of p, pass 0 most
    significant, written back in reverse order -- fufft_chain_rev for all p at
    once (verify_kernel.cpp:460-477 chain_rev)"""
    n = 1
    for r in radices:
        n *= int(r)
    p = torch.arange(n, dtype=torch.int64, device=device)
    out = torch.zeros_like(p)
    rest, op = n, 1          # weight of the current digit in p; in the output
    for r in radices:
        rest //= int(r)
        out += ((p // rest) % int(r)) * op
        op *= int(r)
    return out


def filter_permute(spec_natural: torch.Tensor, n: int, layout: int) -> torch.Tensor:
    """natural-order spectrum (device) -> kernel layout, per transform"""
    s = _complex(spec_natural).contiguous()
    out = torch.empty_like(s)
    check(lib().fufft_filter_permute(_ptr(s), _ptr(out), n, _batch(s, n), layout, _stream()),
          "fufft_filter_permute")
    return out


def filter_permute_host(spec_natural, n: int, layout: int):
    """numpy complex64 natural-order spectrum -> kernel layout (host)"""
    import numpy as np
    s = np.ascontiguousarray(spec_natural, dtype=np.complex64)
    out = np.empty_like(s)
    check(lib().fufft_filter_permute_host(s.ctypes.data, out.ctypes.data, n, s.size // n, layout),
          "fufft_filter_permute_host")
    return out


# ---- fused convolutions -------------------------------------------------------
def conv(a: torch.Tensor, b: torch.Tensor | None, n: int, layout: int = LAYOUT_R16_BPERM,
         mid: int = MID_MULTIPLY, filter_stride: int | None = None,
         out: torch.Tensor | None = None) -> torch.Tensor:
    a = _complex(a)
    bt = None if b is None else _complex(b)
    out = torch.empty_like(a) if out is None else _complex(out)
    fs = n if filter_stride is None else filter_stride
    check(lib().fufft_conv_c2c_f32(_ptr(a), _ptr(bt), _ptr(out), n, _batch(a, n), layout, mid, fs, _stream()),
          "fufft_conv_c2c_f32")
    return out


def filter_permute2d(spec_natural: torch.Tensor, h: int, w: int, layout: int) -> torch.Tensor:
    """natural-order 2-D spectrum (device, row-major) -> 2-D kernel layout"""
    s = _complex(spec_natural).contiguous()
    out = torch.empty_like(s)
    check(lib().fufft_filter_permute2d(_ptr(s), _ptr(out), h, w, _batch(s, h * w), layout, 0, _stream()),
          "fufft_filter_permute2d")
    return out


def conv2d(a: torch.Tensor, b: torch.Tensor | None, h: int, w: int, layout: int = LAYOUT_R16_BPERM,
           mid: int = MID_MULTIPLY, filter_stride: int | None = None,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """fufft_conv2d<H, W, CPB>: fused 2-D cyclic convolution of row-major h x w images"""
    a = _complex(a)
    bt = None if b is None else _complex(b)
    out = torch.empty_like(a) if out is None else _complex(out)
    fs = h * w if filter_stride is None else filter_stride
    check(lib().fufft_conv2d_f32(_ptr(a), _ptr(bt), _ptr(out), h, w, _batch(a, h * w), layout, mid, fs, _stream()),
          "fufft_conv2d_f32")
    return out


def conv_host_workspace(n: int, batch: int, filter_stride: int, device=None) -> torch.Tensor:
    """device workspace for conv_host (allocate once, reuse across calls)"""
    need = int(lib().fufft_conv_host_workspace(n, batch, filter_stride))
    return torch.empty(max(need, 1), dtype=torch.uint8, device=device or "cuda")


def conv_host(a: torch.Tensor, b: torch.Tensor | None, out: torch.Tensor, n: int, layout: int = LAYOUT_R16_BPERM,
              mid: int = MID_MULTIPLY, filter_stride: int | None = None,
              workspace: torch.Tensor | None = None) -> torch.Tensor:
    """fused convolution of HOST tensors (pinned for overlap): chunked upload /
    convolve / download pipeline on the current device, asynchronous on the
    current stream"""
    a, out = _complex(a), _complex(out)
    if a.is_cuda or out.is_cuda or (b is not None and b.is_cuda):
        raise ValueError("conv_host takes host tensors")
    bt = None if b is None else _complex(b)
    batch = _batch(a, n)
    if out.numel() < a.numel():
        raise ValueError("out is smaller than a")
    fs = (n if bt is None or bt.numel() > n else 0) if filter_stride is None else filter_stride
    if workspace is None:
        workspace = conv_host_workspace(n, batch, fs)
    check(lib().fufft_conv_c2c_f32_host(_hptr(a), _hptr(bt), _hptr(out), n, batch, layout, mid, fs, _ptr(workspace),
                                        workspace.numel(), _stream()), "fufft_conv_c2c_f32_host")
    return out


def filter_from_taps(taps: torch.Tensor, n: int, layout: int = LAYOUT_R16_BPERM) -> torch.Tensor:
    """complex filter taps (natural order) -> filter spectrum x 1/n in `layout`, on the device"""
    taps = _complex(taps)
    out = torch.empty_like(taps)
    check(lib().fufft_filter_from_taps_f32(_ptr(taps), _ptr(out), n, _batch(taps, n), layout, _stream()),
          "fufft_filter_from_taps_f32")
    return out


def c2c(a: torch.Tensor, n: int, sign: int = -1, out: torch.Tensor | None = None) -> torch.Tensor:
    """natural-order DFT of each n-point transform (sign -1), or the unnormalised inverse (+1)"""
    a = _complex(a)
    out = torch.empty_like(a) if out is None else _complex(out)
    check(lib().fufft_c2c_f32(_ptr(a), _ptr(out), n, _batch(a, n), sign, _stream()), "fufft_c2c_f32")
    return out


def fwd(a: torch.Tensor, n: int, layout: int = LAYOUT_R8) -> torch.Tensor:
    a = _complex(a)
    spec = torch.empty_like(a)
    check(lib().fufft_fwd_f32(_ptr(a), _ptr(spec), n, _batch(a, n), layout, _stream()), "fufft_fwd_f32")
    return spec


def apply(spec: torch.Tensor, b: torch.Tensor | None, n: int, layout: int = LAYOUT_R8,
          mid: int = MID_MULTIPLY, batch: int | None = None, spec_stride: int | None = None,
          filter_stride: int | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    spec = _complex(spec)
    bt = None if b is None else _complex(b)
    batch = _batch(spec, n) if batch is None else batch
    ss = n if spec_stride is None else spec_stride
    fs = n if filter_stride is None else filter_stride
    if out is None:
        out = torch.empty(batch * n, dtype=torch.complex64, device=spec.device)
    check(lib().fufft_apply_f32(_ptr(spec), _ptr(bt), _ptr(out), n, batch, layout, mid, ss, fs, _stream()),
          "fufft_apply_f32")
    return out


def fwd_r2(xr: torch.Tensor, yr: torch.Tensor, n: int, layout: int = LAYOUT_R16) -> torch.Tensor:
    """chain-order spectra of the packed pairs xr + i*yr (two real signals per transform)"""
    if xr.shape != yr.shape:
        raise ValueError("xr and yr must have the same shape")
    spec = torch.empty(xr.numel(), dtype=torch.complex64, device=xr.device)
    check(lib().fufft_fwd_r2_f32(_ptr(xr), _ptr(yr), _ptr(spec), n, _batch(xr, n), layout, _stream()),
          "fufft_fwd_r2_f32")
    return spec


def apply_grid(spec: torch.Tensor, b: torch.Tensor, n: int, layout: int = LAYOUT_R16, mid: int = MID_MULTIPLY,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """every spectrum against every filter in one launch: out[s][f] = IDFT(spec_s (x) b_f), complex"""
    spec, bt = _complex(spec), _complex(b)
    ns, nf = _batch(spec, n), _batch(bt, n)
    if out is None:
        out = torch.empty(ns * nf * n, dtype=torch.complex64, device=spec.device)
    else:
        out = _complex(out)
        if out.numel() < ns * nf * n:
            raise ValueError("out must hold n_spec * n_filt * n complex points")
    check(lib().fufft_apply_grid_f32(_ptr(spec), ns, _ptr(bt), nf, _ptr(out), n, layout, mid, _stream()),
          "fufft_apply_grid_f32")
    return out


def apply_grid_r2(spec: torch.Tensor, b: torch.Tensor, n: int, layout: int = LAYOUT_R16, mid: int = MID_MULTIPLY,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """packed real pairs x real filters: out[2s + j][f][0..n) real (j = 0: xr of pair s, 1: yr)"""
    spec, bt = _complex(spec), _complex(b)
    ns, nf = _batch(spec, n), _batch(bt, n)
    if out is None:
        out = torch.empty(2 * ns * nf * n, dtype=torch.float32, device=spec.device)
    elif out.dtype != torch.float32 or out.numel() < 2 * ns * nf * n:
        raise ValueError("out must be float32 with 2 * n_pairs * n_filt * n elements")
    check(lib().fufft_apply_grid_r2_f32(_ptr(spec), ns, _ptr(bt), nf, _ptr(out), n, layout, mid, _stream()),
          "fufft_apply_grid_r2_f32")
    return out


def conv_r2(xr: torch.Tensor, yr: torch.Tensor, b: torch.Tensor, n: int, layout: int = LAYOUT_R8,
            mid: int = MID_MULTIPLY, filter_stride: int | None = None):
    bt = _complex(b)
    ur, vr = torch.empty_like(xr), torch.empty_like(yr)
    fs = n if filter_stride is None else filter_stride
    check(lib().fufft_conv_r2_f32(_ptr(xr), _ptr(yr), _ptr(bt), _ptr(ur), _ptr(vr), n, _batch(xr, n),
                                  layout, mid, fs, _stream()), "fufft_conv_r2_f32")
    return ur, vr


# ---- four-step large N ------------------------------------------------------------
def large_plan(n: int, layout: int = LAYOUT_R16) -> tuple[int, int]:
    r, m = ct.c_int(), ct.c_int()
    check(lib().fufft_large_plan(n, layout, ct.byref(r), ct.byref(m)), "fufft_large_plan")
    return r.value, m.value


def conv_large(buf: torch.Tensor, b: torch.Tensor | None, n: int, layout: int = LAYOUT_R16,
               mid: int = MID_MULTIPLY, r_out: int | None = None, mid_size: int | None = None) -> torch.Tensor:
    """run_large: in-place four-step convolution of transforms of n points"""
    buf = _complex(buf)
    if r_out is None or mid_size is None:
        r_out, mid_size = large_plan(n, layout)
    bt = None if b is None else _complex(b)
    check(lib().fufft_conv_large_f32(_ptr(buf), _ptr(bt), n, _batch(buf, n), r_out, mid_size, layout, mid,
                                     _stream()), "fufft_conv_large_f32")
    return buf


def conv_large_bfp(aq, a_scale, bq, b_scale, n: int, layout: int = LAYOUT_R16, mid: int = MID_MULTIPLY,
                   r_out: int | None = None, mid_size: int | None = None, workspace: torch.Tensor | None = None):
    if r_out is None or mid_size is None:
        r_out, mid_size = large_plan(n, layout)
    batch = _batch(aq, n, 2)
    need = int(lib().fufft_conv_large_bfp_workspace(n, batch))
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=aq.device)
    oq = torch.empty_like(aq)
    os_ = torch.empty(batch, dtype=torch.float32, device=aq.device)
    check(lib().fufft_conv_large_bfp(_ptr(aq), _ptr(a_scale), _ptr(bq), _ptr(b_scale), _ptr(oq), _ptr(os_), n, batch,
                                     r_out, mid_size, layout, mid, _ptr(workspace), workspace.numel(), _stream()),
          "fufft_conv_large_bfp")
    return oq, os_


# ---- int16 block floating point -------------------------------------------------
def bfp_pack(x: torch.Tensor, n: int):
    x = _complex(x)
    batch = _batch(x, n)
    q = torch.empty(x.numel(), 2, dtype=torch.int16, device=x.device)
    s = torch.empty(batch, dtype=torch.float32, device=x.device)
    check(lib().fufft_bfp_pack(_ptr(x), _ptr(q), _ptr(s), n, batch, _stream()), "fufft_bfp_pack")
    return q, s


def bfp_unpack(q: torch.Tensor, s: torch.Tensor, n: int) -> torch.Tensor:
    batch = _batch(q, n, 2)
    x = torch.empty(batch * n, dtype=torch.complex64, device=q.device)
    check(lib().fufft_bfp_unpack(_ptr(q), _ptr(s), _ptr(x), n, batch, _stream()), "fufft_bfp_unpack")
    return x


def conv_bfp(aq: torch.Tensor, a_scale: torch.Tensor, bq: torch.Tensor | None, b_scale: torch.Tensor | None,
             n: int, layout: int = LAYOUT_R16, mid: int = MID_MULTIPLY, filter_stride: int | None = None,
             out: tuple[torch.Tensor, torch.Tensor] | None = None):
    """int16-BFP fused convolution; out = (oq, o_scale) to reuse output buffers"""
    batch = _batch(aq, n, 2)
    oq, os_ = out if out is not None else (torch.empty_like(aq),
                                           torch.empty(batch, dtype=torch.float32, device=aq.device))
    fs = n if filter_stride is None else filter_stride
    check(lib().fufft_conv_c2c_bfp(_ptr(aq), _ptr(a_scale), _ptr(bq), _ptr(b_scale), _ptr(oq), _ptr(os_), n,
                                   batch, layout, mid, fs, _stream()), "fufft_conv_c2c_bfp")
    return oq, os_


# ---- the reference's entry-point names ----------------------------------------------
def pipeline_ip(a, b_dr, n, mid=MID_MULTIPLY):
    """fufft_pipeline_ip<N, LEAD, NR8, CPB, Mid>: radix-8 chain, filter in mixedrev order"""
    return conv(a, b_dr, n, LAYOUT_R8, mid)


def pipeline_fused(a, bperm, n):
    """fufft_pipeline_fused: radix-8 chain, filter in the register-boundary layout"""
    return conv(a, bperm, n, LAYOUT_R8_BPERM, MID_MULTIPLY)


def pipeline_v16(a, b16, n, mid=MID_MULTIPLY):
    """fufft_pipeline_v16: radix-16 chain, filter in mixedrev16 order"""
    return conv(a, b16, n, LAYOUT_R16, mid)


def pipeline_v16f(a, bperm16, n):
    """fufft_pipeline_v16f: radix-16 chain, filter in the register-boundary layout"""
    return conv(a, bperm16, n, LAYOUT_R16_BPERM, MID_MULTIPLY)


def pipeline_r16(a, b16, n, mid=MID_MULTIPLY):
    """fufft_pipeline_r16: same transform and filter order as pipeline_v16"""
    return conv(a, b16, n, LAYOUT_R16, mid)


def pipeline_fwd(a, n):
    """fufft_pipeline_fwd: radix-8 chain-order spectrum"""
    return fwd(a, n, LAYOUT_R8)


def pipeline_apply(spec, b_dr, n, mid=MID_MULTIPLY):
    """fufft_pipeline_apply: spectrum x filter, inverse (radix-8 chain)"""
    return apply(spec, b_dr, n, LAYOUT_R8, mid)


def pipeline_v16_bfp(aq, a_scale, bq, b_scale, n):
    """fufft_pipeline_v16_bfp: int16 BFP in and out, radix-16 chain"""
    return conv_bfp(aq, a_scale, bq, b_scale, n, LAYOUT_R16, MID_MULTIPLY)
