"""TEST INFRASTRUCTURE ONLY: numpy front end of the CPU checkers.

``Oracle`` wraps liboracle.so (the C restatement in fufft_oracle.c);
``Reference`` wraps _ref/libfufft_ref.so (the reference's own transcription,
compiled from its sources by the Makefile here); ``CpuPrograms`` wraps
_ref/libfufft_cpuref.so (its three CPU programs, the same way).  Only tests/,
``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg import this module;
the product library never does.

Complex data are numpy complex64 arrays (interleaved re/im float32), int16
block-floating-point data are int16 arrays of shape (..., 2).
"""
from __future__ import annotations

import ctypes as ct
import os
import subprocess
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libfufft_ref.so")

MID_NONE, MID_MULTIPLY, MID_CONJ = 0, 1, 2

_P = ct.c_void_p
_build_lock = threading.Lock()


def build(ref: bool = True) -> None:
    """Compile the checkers (gcc/g++ only); the reference part needs its tree."""
    with _build_lock:
        subprocess.run(["make", "-s", "-C", HERE] + ([] if ref else ["liboracle.so"]),
                       check=True, stdout=subprocess.DEVNULL)


def _ptr(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "checker arrays must be contiguous"
    return a.ctypes.data_as(_P)


def _c64(x) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=np.complex64)


def _f32(x) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=np.float32)


class Oracle:
    """The C restatement of the reference algorithm (bit-exact to it)."""

    def __init__(self) -> None:
        if not os.path.exists(ORACLE_SO):
            build(ref=False)
        L = ct.CDLL(ORACLE_SO)
        i, ll = ct.c_int, ct.c_longlong
        sig = {
            "orc_factorise": (i, [i, i, ct.POINTER(i), ct.POINTER(i)]),
            "orc_chain_rev": (ll, [ll, _P, i]),
            "orc_permute_dr": (i, [_P, _P, i, i, i]),
            "orc_bperm": (i, [_P, _P, i, i, i]),
            "orc_conv": (i, [i, i, i, _P, _P, _P, i, ll]),
            "orc_fwd": (i, [i, i, _P, _P, i]),
            "orc_c2c": (i, [i, i, i, _P, _P, i]),
            "orc_apply": (i, [i, i, i, _P, _P, _P, i, ll]),
            "orc_conv_r2": (i, [i, i, _P, _P, _P, _P, _P, i, ll]),
            "orc_conv2d_pow8": (i, [i, i, _P, _P, _P, i, ll]),
            "orc_conv2d": (i, [i, i, i, i, _P, _P, _P, i, ll]),
            "orc_bfp_quantize_batch": (None, [_P, i, i, _P, _P]),
            "orc_bfp_dequantize_batch": (None, [_P, _P, i, i, _P]),
            "orc_conv_bfp": (i, [i, i, i, _P, _P, _P, _P, _P, _P, i, ll]),
            "orc_foursteps_chain": (i, [ll, i, i, i, _P]),
            "orc_conv_foursteps": (i, [ll, i, i, i, i, _P, _P]),
            "orc_conv_monolithic": (i, [ll, i, i, i, i, _P, _P]),
            "orc_fft2_f64": (None, [_P, i, i]),
            "orc_conv_f64": (None, [_P, _P, _P, i, i, ll]),
            "orc_conv2d_f64": (None, [_P, _P, _P, i, i, i, ll]),
            "orc_ref_dft": (None, [_P, _P, i, i]),
            "orc_uniform_stream": (None, [ct.c_uint32, ll, _P]),
            "orc_dist_pass": (None, [_P, i, ll, ll, ll, i]),
            "orc_conv_dist": (i, [ll, i, i, i, _P, _P]),
        }
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype, f.argtypes = res, args
        self.L = L

    # ---- index maps -------------------------------------------------------
    def factorise(self, n: int, radix: int) -> tuple[int, int]:
        lead, nr = ct.c_int(), ct.c_int()
        if self.L.orc_factorise(n, radix, ct.byref(lead), ct.byref(nr)):
            raise ValueError(f"n={n} is not a power of two")
        return lead.value, nr.value

    def chain(self, n: int, radix: int) -> list[int]:
        lead, nr = self.factorise(n, radix)
        return ([lead] if lead > 1 else []) + [radix] * nr

    def chain_rev(self, idx: int, radices) -> int:
        r = np.ascontiguousarray(radices, dtype=np.int32)
        return int(self.L.orc_chain_rev(idx, _ptr(r), len(r)))

    def rev_table(self, radices, n: int) -> np.ndarray:
        return np.array([self.chain_rev(i, radices) for i in range(n)], dtype=np.int64)

    def permute_dr(self, b: np.ndarray, n: int, radix: int) -> np.ndarray:
        b = _c64(b)
        out = np.empty_like(b)
        if self.L.orc_permute_dr(_ptr(b), _ptr(out), n, b.size // n, radix):
            raise ValueError("bad size")
        return out

    def bperm(self, b_dr: np.ndarray, n: int, v: int) -> np.ndarray:
        b_dr = _c64(b_dr)
        out = np.empty_like(b_dr)
        if self.L.orc_bperm(_ptr(b_dr), _ptr(out), n, b_dr.size // n, v):
            raise ValueError("bad size")
        return out

    # ---- pipelines --------------------------------------------------------
    def conv(self, a, b_dr, n: int, radix: int = 16, mid: int = MID_MULTIPLY,
             filter_stride: int | None = None) -> np.ndarray:
        a, b_dr = _c64(a), _c64(b_dr)
        out = np.empty_like(a)
        fs = n if filter_stride is None else filter_stride
        rc = self.L.orc_conv(n, radix, mid, _ptr(a), _ptr(b_dr), _ptr(out), a.size // n, fs)
        assert rc == 0
        return out

    def fwd(self, a, n: int, radix: int = 8) -> np.ndarray:
        a = _c64(a)
        out = np.empty_like(a)
        assert self.L.orc_fwd(n, radix, _ptr(a), _ptr(out), a.size // n) == 0
        return out

    def c2c(self, a, n: int, sign: int = -1, radix: int = 16) -> np.ndarray:
        """natural-order transform (sign -1 forward, +1 unnormalised inverse)"""
        a = _c64(a)
        out = np.empty_like(a)
        assert self.L.orc_c2c(n, radix, sign, _ptr(a), _ptr(out), a.size // n) == 0
        return out

    def apply(self, spec, b_dr, n: int, radix: int = 8, mid: int = MID_MULTIPLY,
              filter_stride: int | None = None) -> np.ndarray:
        spec, b_dr = _c64(spec), _c64(b_dr)
        out = np.empty_like(spec)
        fs = n if filter_stride is None else filter_stride
        assert self.L.orc_apply(n, radix, mid, _ptr(spec), _ptr(b_dr), _ptr(out), spec.size // n, fs) == 0
        return out

    def apply_grid(self, spec, b_dr, n: int, radix: int = 8, mid: int = MID_MULTIPLY) -> np.ndarray:
        """every spectrum against every filter: out[s][f] = apply(spec_s, b_f), each
        cell the reference's split apply (kernel_pipeline_apply,
        verify_kernel.cpp:815-836) of one spectrum with one filter"""
        spec, b_dr = _c64(spec), _c64(b_dr)
        ns, nf = spec.size // n, b_dr.size // n
        rows = [self.apply(np.tile(spec[s * n:(s + 1) * n], nf), b_dr, n, radix, mid) for s in range(ns)]
        return np.concatenate(rows) if rows else np.empty(0, np.complex64)

    def apply_grid_r2(self, spec, b_dr, n: int, radix: int = 8, mid: int = MID_MULTIPLY) -> np.ndarray:
        """packed real pairs: real rows [2s + j][f] = re (j = 0) / im (j = 1) of apply_grid's [s][f]"""
        g = self.apply_grid(spec, b_dr, n, radix, mid)
        ns, nf = spec.size // n, b_dr.size // n
        g = g.reshape(ns, nf, n)
        return np.stack([g.real, g.imag], axis=1).astype(np.float32).reshape(-1)

    def conv_r2(self, xr, yr, b_dr, n: int, radix: int = 8, filter_stride: int | None = None):
        xr, yr, b_dr = _f32(xr), _f32(yr), _c64(b_dr)
        ur, vr = np.empty_like(xr), np.empty_like(yr)
        fs = n if filter_stride is None else filter_stride
        assert self.L.orc_conv_r2(n, radix, _ptr(xr), _ptr(yr), _ptr(b_dr), _ptr(ur), _ptr(vr),
                                  xr.size // n, fs) == 0
        return ur, vr

    def conv2d_pow8(self, a, b2d, h: int, w: int, filter_stride: int | None = None) -> np.ndarray:
        a, b2d = _c64(a), _c64(b2d)
        out = np.empty_like(a)
        fs = h * w if filter_stride is None else filter_stride
        assert self.L.orc_conv2d_pow8(h, w, _ptr(a), _ptr(b2d), _ptr(out), a.size // (h * w), fs) == 0
        return out

    def conv2d(self, a, b2d, h: int, w: int, radix: int = 8, mid: int = MID_MULTIPLY,
               filter_stride: int | None = None) -> np.ndarray:
        a, b2d = _c64(a), _c64(b2d)
        out = np.empty_like(a)
        fs = h * w if filter_stride is None else filter_stride
        assert self.L.orc_conv2d(h, w, radix, mid, _ptr(a), _ptr(b2d), _ptr(out), a.size // (h * w), fs) == 0
        return out

    def permute2d(self, b, h: int, w: int, radix: int) -> np.ndarray:
        """natural 2-D spectrum -> chain order: slot (r, c) = spectrum(rev_H(r), rev_W(c))"""
        rows = self.rev_table(self.chain(h, radix), h) if h > 1 else np.zeros(1, np.int64)
        cols = self.rev_table(self.chain(w, radix), w)
        bb = _c64(b).reshape(-1, h, w)
        return np.ascontiguousarray(bb[:, rows][:, :, cols]).ravel()

    def bfp_quantize(self, x, n: int):
        x = _c64(x)
        batch = x.size // n
        q = np.empty((x.size, 2), dtype=np.int16)
        s = np.empty(batch, dtype=np.float32)
        self.L.orc_bfp_quantize_batch(_ptr(x), n, batch, _ptr(q), _ptr(s))
        return q, s

    def bfp_dequantize(self, q, s, n: int) -> np.ndarray:
        q, s = np.ascontiguousarray(q, dtype=np.int16), _f32(s)
        out = np.empty(q.shape[0], dtype=np.complex64)
        self.L.orc_bfp_dequantize_batch(_ptr(q), _ptr(s), n, s.size, _ptr(out))
        return out

    def conv_bfp(self, aq, as_, bq, bs, n: int, radix: int = 16, mid: int = MID_MULTIPLY,
                 filter_stride: int | None = None):
        aq, bq = np.ascontiguousarray(aq, np.int16), np.ascontiguousarray(bq, np.int16)
        as_, bs = _f32(as_), _f32(bs)
        batch = as_.size
        oq = np.empty_like(aq)
        os_ = np.empty(batch, dtype=np.float32)
        fs = n if filter_stride is None else filter_stride
        assert self.L.orc_conv_bfp(n, radix, mid, _ptr(aq), _ptr(as_), _ptr(bq), _ptr(bs), _ptr(oq),
                                   _ptr(os_), batch, fs) == 0
        return oq, os_

    def foursteps_chain(self, n: int, r_out: int, mid: int, mid_radix: int = 16) -> list[int]:
        rad = np.zeros(64, dtype=np.int32)
        p = self.L.orc_foursteps_chain(n, r_out, mid, mid_radix, _ptr(rad))
        return [int(x) for x in rad[:p]]

    def conv_foursteps(self, a, b_dr, n: int, r_out: int, mid: int, mid_radix: int = 16) -> np.ndarray:
        A = _c64(a).copy()
        b_dr = _c64(b_dr)
        assert self.L.orc_conv_foursteps(n, A.size // n, r_out, mid, mid_radix, _ptr(A), _ptr(b_dr)) == 0
        return A

    def conv_monolithic(self, a, b_dr, n: int, r_out: int, mid: int, mid_radix: int = 16) -> np.ndarray:
        A = _c64(a).copy()
        b_dr = _c64(b_dr)
        assert self.L.orc_conv_monolithic(n, A.size // n, r_out, mid, mid_radix, _ptr(A), _ptr(b_dr)) == 0
        return A

    # ---- seeded inputs of the reference's tests ----------------------------
    def uniform_stream(self, seed: int, count: int) -> np.ndarray:
        """std::uniform_real_distribution<float>(-1,1) over std::mt19937(seed)."""
        out = np.empty(count, np.float32)
        self.L.orc_uniform_stream(seed & 0xFFFFFFFF, count, _ptr(out))
        return out

    @staticmethod
    def _pair(re, im) -> np.ndarray:
        z = np.empty(re.shape, np.complex64)
        z.real, z.imag = re, im
        return z

    def _signal_filter(self, seed: int, count: int, n_norm: int):
        # a = cf(d, d), b = cf(d * invN, d * invN) per point, with the second
        # constructor argument drawn first (GCC's evaluation order, pinned
        # against the compiled reference)
        s = self.uniform_stream(seed, 4 * count).reshape(-1, 4)
        inv = np.float32(1.0) / np.float32(n_norm)
        return self._pair(s[:, 1], s[:, 0]), self._pair(s[:, 3] * inv, s[:, 2] * inv)

    def gen_test(self, n: int, cpb: int, batch: int):
        """test(): verify_kernel.cpp:1277-1286"""
        return self._signal_filter(n * 131 + cpb, n * batch, n)

    def gen_bfp(self, n: int, seed: int):
        """test_bfp(): verify_kernel.cpp:1142-1149"""
        return self._signal_filter(seed * 991 + n, n, n)

    def gen_2d(self, h: int, w: int, batch: int):
        """test_2d(): verify_kernel.cpp:727-737"""
        return self._signal_filter(h * 131 + w, h * w * batch, h * w)

    def gen_large_cfg(self, n: int, batch: int, r_out: int, mid: int):
        """test_large_cfg(): verify_kernel.cpp:487-496"""
        return self._signal_filter(n ^ (r_out * 7919) ^ (mid * 104729), n * batch, n)

    def gen_r2_signals(self, n: int, batch: int):
        """test_r2(): verify_kernel.cpp:620-629 -- xr, yr, then the real taps"""
        s = self.uniform_stream(n * 77 + 5, 2 * n * batch + n)
        xy = s[: 2 * n * batch].reshape(-1, 2)
        return xy[:, 0].copy(), xy[:, 1].copy(), s[2 * n * batch:].copy()

    # ---- distributed single-signal convolution ---------------------------
    def dist_pass(self, x_local, W: int, cols: int, col0: int, n: int, sign: int) -> np.ndarray:
        A = _c64(x_local).copy()
        self.L.orc_dist_pass(_ptr(A), W, cols, col0, n, sign)
        return A

    def conv_dist(self, a, b_dr, n: int, W: int, r_out: int, mid: int) -> np.ndarray:
        A = _c64(a).copy()
        assert self.L.orc_conv_dist(n, W, r_out, mid, _ptr(A), _ptr(_c64(b_dr))) == 0
        return A

    # ---- fp64 ground truth ------------------------------------------------
    def conv_f64(self, a, bnat, n: int, filter_stride: int | None = None) -> np.ndarray:
        a, bnat = _c64(a), _c64(bnat)
        out = np.empty(a.size, dtype=np.complex128)
        fs = n if filter_stride is None else filter_stride
        self.L.orc_conv_f64(_ptr(a), _ptr(bnat), _ptr(out), n, a.size // n, fs)
        return out

    def conv2d_f64(self, a, bnat, h: int, w: int, filter_stride: int | None = None) -> np.ndarray:
        a, bnat = _c64(a), _c64(bnat)
        out = np.empty(a.size, dtype=np.complex128)
        fs = h * w if filter_stride is None else filter_stride
        self.L.orc_conv2d_f64(_ptr(a), _ptr(bnat), _ptr(out), h, w, a.size // (h * w), fs)
        return out

    def fft2_f64(self, x, sign: int) -> np.ndarray:
        y = np.ascontiguousarray(x, dtype=np.complex128).copy()
        self.L.orc_fft2_f64(_ptr(y), y.size, sign)
        return y


class Reference:
    """The reference's own transcription, compiled from its sources (oracle/_ref)."""

    def __init__(self) -> None:
        if not os.path.exists(REF_SO):
            raise FileNotFoundError(REF_SO)
        L = ct.CDLL(REF_SO)
        i = ct.c_int
        sig = {
            "ref_run_suite": (i, []),
            "ref_mixedrev": (i, [i, i, i]),
            "ref_mixedrev16": (i, [i, i, i]),
            "ref_chain_rev": (i, [i, _P, i]),
            "ref_pipeline_ip": (None, [i, i, _P, _P, _P, i]),
            "ref_pipeline_fused": (None, [i, i, _P, _P, _P, i]),
            "ref_pipeline_v16": (None, [i, i, _P, _P, _P, i]),
            "ref_pipeline_v16f": (None, [i, i, _P, _P, _P, i]),
            "ref_pipeline_r16": (None, [i, i, _P, _P, _P, i]),
            "ref_pipeline_fwd": (None, [i, i, _P, _P, i]),
            "ref_c2c": (None, [i, i, _P, _P, i]),
            "ref_pipeline_apply": (None, [i, i, _P, _P, _P, i]),
            "ref_conv_r2": (None, [i, i, _P, _P, _P, _P, _P, i]),
            "ref_conv2d": (None, [i, i, _P, _P, _P, i]),
            "ref_bfp_quantize": (None, [_P, i, _P, _P]),
            "ref_v16_bfp": (None, [i, _P, ct.c_float, _P, ct.c_float, _P, _P]),
            "ref_foursteps_cfg": (None, [i, i, i, i, i, _P, _P]),
            "ref_monolithic_cfg": (None, [i, i, i, i, i, _P, _P]),
            "ref_fft2_f64": (None, [_P, i, i]),
            "ref_gen_test": (None, [i, i, i, _P, _P]),
            "ref_gen_bfp": (None, [i, i, _P, _P]),
            "ref_gen_r2": (None, [i, i, _P, _P, _P, _P]),
            "ref_gen_2d": (None, [i, i, i, _P, _P]),
            "ref_gen_large_cfg": (None, [i, i, i, i, _P, _P]),
        }
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype, f.argtypes = res, args
        self.L = L

    def _run(self, fname: str, n: int, cpb: int, *arrays) -> np.ndarray:
        ins = [_c64(x) for x in arrays]
        out = np.empty_like(ins[0])
        getattr(self.L, fname)(n, cpb, *[_ptr(x) for x in ins], _ptr(out), ins[0].size // n)
        return out

    def pipeline_ip(self, a, b_dr, n, cpb=1):
        return self._run("ref_pipeline_ip", n, cpb, a, b_dr)

    def pipeline_fused(self, a, bperm, n, cpb=1):
        return self._run("ref_pipeline_fused", n, cpb, a, bperm)

    def pipeline_v16(self, a, b16, n, cpb=1):
        return self._run("ref_pipeline_v16", n, cpb, a, b16)

    def pipeline_v16f(self, a, bp16, n, cpb=1):
        return self._run("ref_pipeline_v16f", n, cpb, a, bp16)

    def pipeline_r16(self, a, b16, n, cpb=1):
        return self._run("ref_pipeline_r16", n, cpb, a, b16)

    def pipeline_fwd(self, a, n, cpb=1):
        return self._run("ref_pipeline_fwd", n, cpb, a)

    def c2c(self, a, n, cpb=1):
        """the reference's natural-order forward c2c (kernel_c2c, N a power of 8)"""
        return self._run("ref_c2c", n, cpb, a)

    def pipeline_apply(self, spec, b_dr, n, cpb=1):
        return self._run("ref_pipeline_apply", n, cpb, spec, b_dr)

    def conv_r2(self, xr, yr, b_dr, n, cpb=1):
        xr, yr, b_dr = _f32(xr), _f32(yr), _c64(b_dr)
        ur, vr = np.empty_like(xr), np.empty_like(yr)
        self.L.ref_conv_r2(n, cpb, _ptr(xr), _ptr(yr), _ptr(b_dr), _ptr(ur), _ptr(vr), xr.size // n)
        return ur, vr

    def conv2d(self, a, b_dr, h, w):
        a, b_dr = _c64(a), _c64(b_dr)
        out = np.empty_like(a)
        self.L.ref_conv2d(h, w, _ptr(a), _ptr(b_dr), _ptr(out), a.size // (h * w))
        return out

    def bfp_quantize(self, x):
        x = _c64(x)
        q = np.empty((x.size, 2), dtype=np.int16)
        s = ct.c_float()
        self.L.ref_bfp_quantize(_ptr(x), x.size, _ptr(q), ct.byref(s))
        return q, np.float32(s.value)

    def v16_bfp(self, aq, as_, bq, bs, n):
        aq, bq = np.ascontiguousarray(aq, np.int16), np.ascontiguousarray(bq, np.int16)
        oq = np.empty_like(aq)
        os_ = ct.c_float()
        self.L.ref_v16_bfp(n, _ptr(aq), float(as_), _ptr(bq), float(bs), _ptr(oq), ct.byref(os_))
        return oq, np.float32(os_.value)

    def foursteps_cfg(self, a, b_dr, n, r_out, mid, v16_mid=True):
        A = _c64(a).copy()
        self.L.ref_foursteps_cfg(n, A.size // n, r_out, mid, int(v16_mid), _ptr(A), _ptr(_c64(b_dr)))
        return A

    def monolithic_cfg(self, a, b_dr, n, r_out, mid, v16_mid=True):
        A = _c64(a).copy()
        self.L.ref_monolithic_cfg(n, A.size // n, r_out, mid, int(v16_mid), _ptr(A), _ptr(_c64(b_dr)))
        return A

    # seeded inputs of the reference's own tests
    def gen_test(self, n, cpb, batch):
        a = np.empty(n * batch, np.complex64)
        b = np.empty(n * batch, np.complex64)
        self.L.ref_gen_test(n, cpb, batch, _ptr(a), _ptr(b))
        return a, b

    def gen_bfp(self, n, seed):
        a = np.empty(n, np.complex64)
        b = np.empty(n, np.complex64)
        self.L.ref_gen_bfp(n, seed, _ptr(a), _ptr(b))
        return a, b

    def gen_r2(self, n, batch):
        xr = np.empty(n * batch, np.float32)
        yr = np.empty(n * batch, np.float32)
        h = np.empty(n, np.float32)
        b_dr = np.empty(n * batch, np.complex64)
        self.L.ref_gen_r2(n, batch, _ptr(xr), _ptr(yr), _ptr(h), _ptr(b_dr))
        return xr, yr, h, b_dr

    def gen_2d(self, h, w, batch):
        a = np.empty(h * w * batch, np.complex64)
        b = np.empty(h * w * batch, np.complex64)
        self.L.ref_gen_2d(h, w, batch, _ptr(a), _ptr(b))
        return a, b

    def gen_large_cfg(self, n, batch, r_out, mid):
        a = np.empty(n * batch, np.complex64)
        b = np.empty(n * batch, np.complex64)
        self.L.ref_gen_large_cfg(n, batch, r_out, mid, _ptr(a), _ptr(b))
        return a, b


class CpuPrograms:
    """The reference's three CPU programs (cpu_fufft.cpp, cpu_inplace.cpp,
    cpu_mixed.cpp), compiled from its sources through cpuref/ into
    _ref/libfufft_cpuref.so.  Complex arrays in and out are complex128."""

    SO = os.path.join(HERE, "_ref", "libfufft_cpuref.so")

    def __init__(self) -> None:
        if not os.path.exists(self.SO):
            raise FileNotFoundError(self.SO)
        L = ct.CDLL(self.SO)
        i = ct.c_int
        sig = {
            "ref_cpufufft_main": (i, []), "ref_inplace_main": (i, []), "ref_mixed_main": (i, []),
            "ref_cpufufft_gen_conv": (None, [i, _P, _P]),
            "ref_cpufufft_conv": (None, [i, i, _P, _P, _P]),
            "ref_cpufufft_forward": (None, [i, i, _P, _P]),
            "ref_inplace_digitrev8": (i, [i, i]),
            "ref_inplace_conv": (None, [i, i, _P, _P, _P, _P]),
            "ref_mixed_factorise": (i, [i, i, _P]),
            "ref_mixed_rev": (i, [i, _P, i]),
            "ref_mixed_conv": (i, [i, i, _P, _P, _P, _P]),
        }
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype, f.argtypes = res, args
        self.L = L

    @staticmethod
    def _c128(x) -> np.ndarray:
        return np.ascontiguousarray(x, dtype=np.complex128)

    def fufft_gen_conv(self, n: int):
        """check_convolution(n)'s seeded inputs (cpu_fufft.cpp:214-218)"""
        a, b = np.empty(n, np.complex128), np.empty(n, np.complex128)
        self.L.ref_cpufufft_gen_conv(n, _ptr(a), _ptr(b))
        return a, b

    def fufft_conv(self, a, b, n: int, fp32: bool = False) -> np.ndarray:
        a, b = self._c128(a), self._c128(b)
        out = np.empty(n, np.complex128)
        self.L.ref_cpufufft_conv(n, int(fp32), _ptr(a), _ptr(b), _ptr(out))
        return out

    def fufft_forward(self, x, n: int, fp32: bool = False) -> np.ndarray:
        x = self._c128(x)
        out = np.empty(n, np.complex128)
        self.L.ref_cpufufft_forward(n, int(fp32), _ptr(x), _ptr(out))
        return out

    def inplace_conv(self, a, b, n: int, fp32: bool = False):
        """(digit-reversed filter spectrum / n, convolution)"""
        a, b = self._c128(a), self._c128(b)
        bs, out = np.empty(n, np.complex128), np.empty(n, np.complex128)
        self.L.ref_inplace_conv(n, int(fp32), _ptr(a), _ptr(b), _ptr(bs), _ptr(out))
        return bs, out

    def digitrev8(self, i: int, s: int) -> int:
        return int(self.L.ref_inplace_digitrev8(i, s))

    def mixed_factorise(self, n: int, v: int) -> list[int]:
        r = np.zeros(16, np.int32)
        p = self.L.ref_mixed_factorise(n, v, _ptr(r))
        return [int(x) for x in r[:p]]

    def mixed_rev(self, i: int, radices) -> int:
        r = np.ascontiguousarray(radices, dtype=np.int32)
        return int(self.L.ref_mixed_rev(i, _ptr(r), len(r)))

    def mixed_conv(self, a, b, n: int, v: int):
        """(chain-order filter spectrum / n, convolution)"""
        a, b = self._c128(a), self._c128(b)
        bs, out = np.empty(n, np.complex128), np.empty(n, np.complex128)
        assert self.L.ref_mixed_conv(n, v, _ptr(a), _ptr(b), _ptr(bs), _ptr(out)) > 0
        return bs, out


def rel_l2(x, y) -> float:
    """sqrt(sum|x-y|^2 / sum|y|^2) in fp64 (bench_fufft.cu:51-61)."""
    x = np.asarray(x).astype(np.complex128).ravel()
    y = np.asarray(y).astype(np.complex128).ravel()
    return float(np.sqrt(np.sum(np.abs(x - y) ** 2) / np.sum(np.abs(y) ** 2)))
