"""ctypes binding of libfufft_b200.so (the C ABI in include/fufft_b200.h).

The shared library is the product: every entry point here is a thin call into
it.  There is no CPU or PyTorch fallback: if the library is missing this
module raises at import time.
"""
from __future__ import annotations

import ctypes as ct
import os

HERE = os.path.dirname(os.path.abspath(__file__))
# FUFFT_B200_LIB points at another build of the same library (A/B runs)
LIB_PATH = os.environ.get("FUFFT_B200_LIB") or os.path.join(HERE, "libfufft_b200.so")

# enums of include/fufft_b200.h
OK = 0
STATUS_NAMES = {0: "OK", 1: "INVALID_SIZE", 2: "INVALID_BATCH", 3: "MISALIGNED", 4: "CUDA",
                5: "TIMEOUT", 6: "PEER_UNAVAILABLE", 7: "INVALID_ARG", 8: "UNSUPPORTED"}
MID_NONE, MID_MULTIPLY, MID_CONJ_MULTIPLY = 0, 1, 2
LAYOUT_R8, LAYOUT_R8_BPERM, LAYOUT_R16, LAYOUT_R16_BPERM, LAYOUT_NATURAL = 0, 1, 2, 3, 4

# every symbol the header declares, with its C signature
_P, _I, _I64, _U32 = ct.c_void_p, ct.c_int, ct.c_int64, ct.c_uint32
SIGNATURES = {
    "fufft_status_string": (ct.c_char_p, [_I]),
    "fufft_last_cuda_error": (ct.c_char_p, []),
    "fufft_max_n": (_I, [_I]),
    "fufft_init": (_I, []),
    "fufft_device_status": (_I, [ct.POINTER(_U32), _P]),
    "fufft_launch_count": (ct.c_uint64, []),
    "fufft_selftest_wait_timeout": (_I, [_U32, _P]),
    "fufft_chain": (_I, [_I, _I, ct.POINTER(_I)]),
    "fufft_chain_rev": (_I64, [_I64, ct.POINTER(_I), _I]),
    "fufft_filter_permute_host": (_I, [_P, _P, _I, _I, _I]),
    "fufft_filter_permute": (_I, [_P, _P, _I, _I, _I, _P]),
    "fufft_conv_c2c_f32": (_I, [_P, _P, _P, _I, _I64, _I, _I, _I64, _P]),
    "fufft_filter_permute2d": (_I, [_P, _P, _I, _I, _I, _I, _I, _P]),
    "fufft_conv2d_f32": (_I, [_P, _P, _P, _I, _I, _I64, _I, _I, _I64, _P]),
    "fufft_fwd_f32": (_I, [_P, _P, _I, _I64, _I, _P]),
    "fufft_apply_f32": (_I, [_P, _P, _P, _I, _I64, _I, _I, _I64, _I64, _P]),
    "fufft_fwd_r2_f32": (_I, [_P, _P, _P, _I, _I64, _I, _P]),
    "fufft_c2c_f32": (_I, [_P, _P, _I, _I64, _I, _P]),
    "fufft_filter_from_taps_f32": (_I, [_P, _P, _I, _I64, _I, _P]),
    "fufft_conv_host_workspace": (ct.c_size_t, [_I, _I64, _I64]),
    "fufft_conv_c2c_f32_host": (_I, [_P, _P, _P, _I, _I64, _I, _I, _I64, _P, ct.c_size_t, _P]),
    "fufft_apply_grid_f32": (_I, [_P, _I64, _P, _I64, _P, _I, _I, _I, _P]),
    "fufft_apply_grid_r2_f32": (_I, [_P, _I64, _P, _I64, _P, _I, _I, _I, _P]),
    "fufft_conv_r2_f32": (_I, [_P, _P, _P, _P, _P, _I, _I64, _I, _I, _I64, _P]),
    "fufft_bfp_pack": (_I, [_P, _P, _P, _I, _I64, _P]),
    "fufft_bfp_unpack": (_I, [_P, _P, _P, _I, _I64, _P]),
    "fufft_conv_c2c_bfp": (_I, [_P, _P, _P, _P, _P, _P, _I, _I64, _I, _I, _I64, _P]),
    "fufft_large_plan": (_I, [_I64, _I, ct.POINTER(_I), ct.POINTER(_I)]),
    "fufft_conv_large_f32": (_I, [_P, _P, _I64, _I64, _I, _I, _I, _I, _P]),
    "fufft_conv_large_bfp_workspace": (ct.c_size_t, [_I64, _I64]),
    "fufft_conv_large_bfp": (_I, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I, _I, _I, _I, _P, ct.c_size_t, _P]),
    "fufft_conv_large_bfp_noalloc": (_I, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I, _I, _I, _I, _P]),
    "fufft_dist_pass": (_I, [_P, _I, _I64, _I64, _I64, _I, _P]),
    "fufft_dist_pass_push": (_I, [_P, _P, _I, _I, _I64, _I64, _P]),
    "fufft_dist_pass_pull": (_I, [_P, _P, _I, _I, _I64, _I64, _P]),
    "fufft_peer_alloc": (_I, [ct.c_size_t, ct.POINTER(_P), _P]),
    "fufft_peer_open": (_I, [_P, ct.POINTER(_P)]),
    "fufft_peer_close": (_I, [_P]),
    "fufft_peer_free": (_I, [_P]),
    "fufft_conv_multi_gpu": (_I, [_P]),
    "fufft_mg_chain": (_I, [_I64, _I, ct.POINTER(_I)]),
}


class FufftError(RuntimeError):
    def __init__(self, status: int, what: str):
        self.status = status
        msg = f"{what}: {STATUS_NAMES.get(status, status)}"
        if status == 4:
            err = lib().fufft_last_cuda_error()
            msg += f" ({err.decode() if err else ''})"
        super().__init__(msg)


_LIB = None


def lib() -> ct.CDLL:
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m fufft_b200.build` "
                              "(nvcc, sm_100a); fufft_b200 has no fallback path")
        L = ct.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype, f.argtypes = res, args
        _LIB = L
    return _LIB


def check(status: int, what: str) -> None:
    if status != OK:
        raise FufftError(status, what)
