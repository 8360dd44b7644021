"""The C-ABI library loads and exports every entry point include/*.h declares
(CPU only: no compute call)."""
import ctypes
import glob
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names |= set(re.findall(r"\b(fufft_[a-z0-9_]+)\s*\(", src))
    return names


def test_library_exports_every_declared_symbol():
    from fufft_b200 import _lib
    L = _lib.lib()
    declared = _declared()
    assert declared, "no declarations found"
    missing = [n for n in sorted(declared) if not hasattr(L, n)]
    assert not missing, missing
    assert declared == set(_lib.SIGNATURES), declared ^ set(_lib.SIGNATURES)


def test_host_side_calls_without_gpu():
    from fufft_b200 import ops
    assert ops.chain(4096, 16) == [16, 16, 16]
    assert ops.chain(2048, 8) == [4, 8, 8, 8]
    assert ops.max_n(ops.LAYOUT_R16) == 65536 and ops.max_n(ops.LAYOUT_R8) == 4096
    assert ctypes.string_at(ops.lib().fufft_status_string(1)).startswith(b"invalid size")


def test_host_permutation_matches_oracle(oracle):
    import numpy as np
    from fufft_b200 import ops
    rng = np.random.default_rng(0)
    for n in (16, 128, 512, 1024, 2048, 4096, 8192):
        b = (rng.standard_normal(2 * n) + 1j * rng.standard_normal(2 * n)).astype(np.complex64)
        for layout, radix, v in [(0, 8, 1), (1, 8, 8), (2, 16, 1), (3, 16, 16)]:
            want = oracle.permute_dr(b, n, radix)
            if v > 1:
                want = oracle.bperm(want, n, v)
            assert np.array_equal(ops.filter_permute_host(b, n, layout), want)
            for i in range(0, n, max(1, n // 64)):
                assert ops.chain_rev(i, ops.chain(n, radix)) == oracle.chain_rev(i, oracle.chain(n, radix))


def test_chain_rev_table_matches_oracle(oracle):
    """the vectorised digit-reversal table equals the oracle's chain_rev for
    one-kernel chains, four-step chains and the distributed chain"""
    import numpy as np
    from fufft_b200 import ops
    chains = [ops.chain(n, r) for n, r in [(512, 16), (2048, 8), (4096, 16), (8192, 16)]]
    chains += [oracle.foursteps_chain(32768, 16, 2048, 16), [8, 16, 16, 16]]
    for ch in chains:
        n = int(np.prod(ch))
        got = ops.chain_rev_table(ch).numpy()
        assert np.array_equal(got, oracle.rev_table(ch, n)), ch
