"""Fixtures from the reference's three CPU programs (cpu_fufft.cpp,
cpu_inplace.cpp, cpu_mixed.cpp), compiled from its sources into
oracle/_ref/libfufft_cpuref.so.  Run here, where the reference tree exists:

    make -C oracle REF_DIR=<reference tree> && python tests/golden/make_cpu_programs.py

Records, per case, the inputs (complex64: exactly the values the GPU kernels
get; the programs are fed the same values, widened to fp64) and the
programs' own outputs:
  * cpu_fufft (Stockham radix 8, natural order, N = 8 .. 4096 powers of 8):
    check_convolution's seeded inputs (cpu_fufft.cpp:214-218), the fp64 and the
    fp32 convolution, the fp64 spectrum of the filter taps, the fp64 and fp32
    forward transforms of the signal;
  * cpu_inplace (in-place radix-8 DIF/DIT, N = 8 .. 4096): the digit-reversed
    filter spectrum / N and the convolution, fp64 and fp32;
  * cpu_mixed (mixed radix, V = 8 and 16, N = 16 .. 4096): the chain-order
    filter spectrum / N and the fp64 convolution.
into cpu_programs.npz (outputs stored as complex64) and the SHA-256 digests
of the fp64 outputs into cpu_programs_digests.json, which
tests/test_oracle_golden.py checks against the compiled programs.
"""
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle.oracle import CpuPrograms  # noqa: E402

FUFFT_SIZES = [8, 64, 512, 4096]
INPLACE_SIZES = [8, 64, 512, 4096]
MIXED_SIZES = [16, 32, 64, 128, 256, 512, 1024, 2048, 4096]


def digest(x: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(x).tobytes()).hexdigest()


def seeded(n: int, seed: int):
    """signal and taps iid U[-1,1) complex, rounded to complex64"""
    rng = np.random.default_rng(seed)
    a = (rng.uniform(-1, 1, n) + 1j * rng.uniform(-1, 1, n)).astype(np.complex64)
    b = (rng.uniform(-1, 1, n) + 1j * rng.uniform(-1, 1, n)).astype(np.complex64)
    return a, b


def cases(p: CpuPrograms):
    """(key, arrays): the digested fp64 outputs are the keys ending in 64"""
    for n in FUFFT_SIZES:
        a64, b64 = p.fufft_gen_conv(n)
        a, b = a64.astype(np.complex64), b64.astype(np.complex64)
        yield f"cpu_fufft/{n}", dict(a=a, b=b, conv64=p.fufft_conv(a, b, n), conv32=p.fufft_conv(a, b, n, True),
                                      bspec64=p.fufft_forward(b, n), fwd64=p.fufft_forward(a, n),
                                      fwd32=p.fufft_forward(a, n, True))
    for n in INPLACE_SIZES:
        a, b = seeded(n, 7000 + n)
        bs64, out64 = p.inplace_conv(a, b, n)
        bs32, out32 = p.inplace_conv(a, b, n, True)
        yield f"cpu_inplace/{n}", dict(a=a, b=b, bs64=bs64, out64=out64, bs32=bs32, out32=out32)
    for v in (8, 16):
        for n in MIXED_SIZES:
            if n < v:
                continue
            a, b = seeded(n, 9000 + 3 * n + v)
            bs64, out64 = p.mixed_conv(a, b, n, v)
            yield f"cpu_mixed/{v}/{n}", dict(a=a, b=b, bs64=bs64, out64=out64)


def main() -> None:
    p = CpuPrograms()
    verdict = {"cpu_fufft_main_rc": p.L.ref_cpufufft_main(), "cpu_inplace_main_rc": p.L.ref_inplace_main(),
               "cpu_mixed_main_rc": p.L.ref_mixed_main()}
    arrays, dig = {}, {"programs": verdict}
    for key, rec in cases(p):
        dig[key] = {k: digest(v) for k, v in rec.items() if k.endswith("64") or k in ("a", "b")}
        for k, v in rec.items():
            arrays[f"{key}/{k}"] = v.astype(np.complex64)
    np.savez_compressed(os.path.join(HERE, "cpu_programs.npz"), **arrays)
    with open(os.path.join(HERE, "cpu_programs_digests.json"), "w") as f:
        json.dump(dig, f, indent=1, sort_keys=True)
    print(f"{len(arrays)} arrays, {len(dig) - 1} cases; program exit codes {verdict}")


if __name__ == "__main__":
    main()
