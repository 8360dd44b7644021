"""The radix-16 engine reads filters and spectra in the reference's radix-8
layouts through compile-time staging tables (R8Perm in fufft_conv.cuh).  This
CPU test compiles those tables on the host, replays the per-warp staging that
the kernels do with them, and checks that every lane ends up holding, for each
of its 16 chain positions, the value at the layout index that the oracle's own
digit-reversal tables give for the same frequency -- for every 1-D size and
2-D image shape the library sends down this path, in both radix-8 orders.  It
also checks that no two values of a warp land in the same exchange slot, and
that the direct read of the register-boundary order (lane part plus a
constant per register) addresses the same indices in whole 32-byte sectors."""
import json
import os
import shutil
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SHAPES_1D = [512, 1024, 2048, 4096]
SHAPES_2D = [(8, 64), (8, 128), (8, 512), (16, 32), (16, 64), (16, 256), (32, 16), (32, 32), (32, 128),
             (64, 16), (64, 64), (128, 32), (256, 16)]

PROG = r"""
#include "fufft_b200/csrc/fufft_conv.cuh"
#include <cstdio>
template<class C, bool BP> void emit(int h, int w, bool& first)
{
   using PM = fufft::R8Perm<C, BP>;
   constexpr auto T = PM::tables();
   printf("%s{\"h\":%d,\"w\":%d,\"bp\":%d,\"b0\":%d,\"lane\":[", first ? "" : ",", h, w, BP ? 1 : 0, T.b0);
   first = false;
   for(int t = 0; t < 5; ++t) printf("%s%d", t ? "," : "", T.lane[t]);
   printf("],\"sig_lane\":[");
   for(int t = 0; t < 5; ++t) printf("%s%d", t ? "," : "", T.sig_lane[t]);
   printf("],\"sig_w\":[");
   for(int t = 0; t < PM::LB - 9; ++t) printf("%s%d", t ? "," : "", T.sig_w[t]);
   printf("],\"qh\":[");
   for(int i = 0; i < 8; ++i) printf("%s%d", i ? "," : "", T.qh[i]);
   printf("],\"s0\":[");
   for(int i = 0; i < 8; ++i) printf("%s%d", i ? "," : "", T.s0[i]);
   printf("],\"s1\":[");
   for(int i = 0; i < 8; ++i) printf("%s%d", i ? "," : "", T.s1[i]);
   printf("],\"sig\":[");
   for(int b = 0; b < PM::LB; ++b) printf("%s%d", b ? "," : "", T.sig[b]);
   printf("],\"mapk\":[");
   for(int k = 0; k < 16; ++k) printf("%s%d", k ? "," : "", T.mapk[k]);
   printf("],\"cover\":%d}", PM::lanes_cover_q01() ? 1 : 0);
}
#define BOTH(H, W) emit<fufft::Chain2<H, W, 16>, false>(H, W, first); emit<fufft::Chain2<H, W, 16>, true>(H, W, first);
int main()
{
   bool first = true;
   printf("[");
   BOTH(1, 512) BOTH(1, 1024) BOTH(1, 2048) BOTH(1, 4096)
   BOTH(8, 64) BOTH(8, 128) BOTH(8, 512) BOTH(16, 32) BOTH(16, 64) BOTH(16, 256) BOTH(32, 16)
   BOTH(32, 32) BOTH(32, 128) BOTH(64, 16) BOTH(64, 64) BOTH(128, 32) BOTH(256, 16)
   printf("]\n");
   return 0;
}
"""


def _nvcc():
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    return None


@pytest.fixture(scope="module")
def tables(tmp_path_factory):
    nvcc = _nvcc()
    if nvcc is None:
        pytest.skip("nvcc not available")
    d = tmp_path_factory.mktemp("r8perm")
    src, exe = d / "tables.cu", d / "tables"
    src.write_text(PROG)
    subprocess.run([nvcc, "-std=c++17", "--expt-relaxed-constexpr", "-gencode", "arch=compute_100a,code=sm_100a",
                    "-I", os.path.join(ROOT, "include"), "-I", ROOT, "-o", str(exe), str(src)],
                   check=True, capture_output=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    return {(t["h"], t["w"], t["bp"]): t for t in json.loads(out)}


def _layout_index(oracle, h, w, bp):
    """radix-16 engine position p -> index of the same frequency in the radix-8 layout, from the oracle's
    digit-reversal tables (slot p of a chain order holds frequency rev[p])"""
    def dim(n, radix):
        return oracle.rev_table(oracle.chain(n, radix), n) if n > 1 else np.zeros(1, np.int64)
    r16h, r16w, r8h, r8w = dim(h, 16), dim(w, 16), dim(h, 8), dim(w, 8)
    inv8h, inv8w = np.empty_like(r8h), np.empty_like(r8w)
    inv8h[r8h] = np.arange(h)
    inv8w[r8w] = np.arange(w)
    p = np.arange(h * w)
    q = inv8h[r16h[p // w]] * w + inv8w[r16w[p % w]]
    if bp:
        n = h * w
        q = q // 8 + (q % 8) * (n // 8)
    return q


def _slot(p):
    return 2 * ((p >> 1) ^ ((p >> 4) & 7)) + (p & 1)


@pytest.mark.parametrize("shape", [(1, n) for n in SHAPES_1D] + SHAPES_2D)
@pytest.mark.parametrize("bp", [0, 1])
def test_staging_tables_match_oracle_layouts(tables, oracle, shape, bp):
    h, w = shape
    n = h * w
    tb = tables[(h, w, bp)]
    want = _layout_index(oracle, h, w, bp)
    lb = n.bit_length() - 1
    for warp in range(n // 16 // 32):
        slots = [None] * 512
        for l in range(32):
            pl = sum(((l >> t) & 1) << tb["lane"][t] for t in range(5))
            ql = sum(((l >> t) & 1) << tb["sig_lane"][t] for t in range(5))
            ql |= sum(((warp >> t) & 1) << tb["sig_w"][t] for t in range(lb - 9))
            sl = _slot(pl)
            for i in range(8):
                q = ql | tb["qh"][i]
                assert q % 2 == 0 and q + 1 < n
                for s, val in ((sl ^ tb["s0"][i], q), (sl ^ tb["s1"][i], q + 1)):
                    assert slots[s] is None, (warp, l, i)      # each exchange slot written once
                    slots[s] = val
        for l in range(32):
            lane = 32 * warp + l
            for i in range(8):
                row = (8 * l + i) ^ (((8 * l + i) >> 3) & 7)
                for half in (0, 1):
                    assert slots[2 * row + half] == want[16 * lane + 2 * i + half], (warp, l, i, half)


@pytest.mark.parametrize("shape", [(1, n) for n in SHAPES_1D] + SHAPES_2D)
def test_direct_register_boundary_read(tables, oracle, shape):
    """Flt::R8BP_DIRECT: register k of `lane` reads index ql(lane) + map(k), and
    each warp-wide load covers whole 32-byte sectors (four consecutive elements)"""
    h, w = shape
    n = h * w
    tb = tables[(h, w, 1)]
    if not tb["cover"]:
        pytest.skip("this shape stages the register-boundary order instead")
    want = _layout_index(oracle, h, w, 1)
    lb = n.bit_length() - 1
    sig = tb["sig"]
    for lane in range(n // 16):
        ql = sum(((lane >> t) & 1) << sig[4 + t] for t in range(lb - 4))
        for k in range(16):
            assert tb["mapk"][k] == sum(1 << sig[b] for b in range(4) if (k >> b) & 1)
            assert ql + tb["mapk"][k] == want[16 * lane + k], (lane, k)
    for warp in range(n // 16 // 32):
        for k in range(16):
            idx = [int(want[16 * (32 * warp + l) + k]) for l in range(32)]
            sectors = {}
            for q in idx:
                sectors.setdefault(q // 4, set()).add(q % 4)
            assert all(v == {0, 1, 2, 3} for v in sectors.values()), (warp, k)
