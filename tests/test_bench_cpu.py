"""CPU: the benchmark's reference arm runs the reference's own code only.

The reference arm (`bench.py --impl reference`) must time the reference's
ct_attn_forward from oracle/_ref without this repository's library in the
process: its workload (lengths, seeds) is derived in pure Python."""
import os
import subprocess
import sys
from pathlib import Path

import pytest

import oracle

ROOT = Path(__file__).resolve().parent.parent

PROBE = r"""
import sys, numpy as np
sys.path.insert(0, sys.argv[1])
import bench
lens, desc, seed = bench.workload("sharded")
assert len(lens) == 1024 and lens.min() >= 512 and lens.max() <= 65536
rate, tok, el = bench.cpu_sample(lens, seed, 0.05, 2)
assert rate > 0 and tok > 0
maps = open("/proc/self/maps").read()
print("MODULE" if "cautreo_b200" in sys.modules else "no-module")
print("SO" if "libcautreo_b200" in maps else "no-so")
print("REF" if "libctref" in maps else "no-ref")
"""


@pytest.mark.skipif(not oracle.ref_available(), reason="reference objects not built")
def test_reference_arm_does_not_load_the_library():
    r = subprocess.run([sys.executable, "-c", PROBE, str(ROOT)], capture_output=True, text=True, timeout=300,
                       cwd=str(ROOT), env=dict(os.environ))
    assert r.returncode == 0, r.stderr
    out = r.stdout.split()
    assert out == ["no-module", "no-so", "REF"], r.stdout


def test_workload_lengths_match_the_oracle_generator():
    sys.path.insert(0, str(ROOT))
    import bench
    for seed, n, lo, hi in ((4, 1024, 512, 65536), (3, 256, 512, 32768)):
        got = bench.lengths_loguniform(n, lo, hi, seed)
        want = oracle.lengths_loguniform(oracle.key(seed, 0), n, lo, hi)
        assert got.tolist() == want.tolist()
