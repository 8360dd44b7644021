"""bench.py's reference arm on the host cores: one JSON line with the same
metric and config as the library's arm, marked impl=reference, with a
cpu_baseline that describes the run and an e2e block that moves no bytes
(the reference's path is CPU code)."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_json_line():
    if not os.path.exists(os.path.join(ROOT, "oracle", "_ref", "libfufft_ref.so")) and \
            not os.path.exists(os.path.join(ROOT, "oracle", "liboracle.so")):
        pytest.skip("CPU checkers not built")
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3"],
                       cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    if "unavailable" in d:
        pytest.skip(d["unavailable"])
    assert d["unit"] == "Gpoints/s" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["config"]["n"] == 4096 and d["config"]["layout"] == "R16_BPERM"
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["e2e"]["value"] == d["value"]
