"""GPU: the reference's own unit-test programs for kv_cache, attention and
quant (tests/unit/*_test.c of the reference), compiled against this
repository's library instead of the reference objects (oracle/Makefile,
target ours-tests) -- the drop-in check that the reference interfaces keep
their results.  The programs are built where the reference sources are; here
they only run."""
import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
TESTS = ["kv_cache_test", "attention_test", "quant_test"]


@pytest.mark.parametrize("name", TESTS)
def test_reference_unit_test_passes_against_library(name, tmp_path):
    exe = ROOT / "oracle" / "_ref" / f"ours_{name}"
    if not exe.exists():
        pytest.skip("reference unit tests not built (make -C oracle ours-tests where the reference sources are)")
    (tmp_path / "build").mkdir()                 # kv_cache_test saves a checkpoint under build/
    r = subprocess.run([str(exe)], cwd=tmp_path, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "FAIL" not in r.stdout
