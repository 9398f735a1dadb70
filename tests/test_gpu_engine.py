"""GPU: the reference engine's own decode loop on the library's KV cache.

oracle/Makefile compiles the reference's transformer.c, model.c and gguf.c
unmodified (from the reference tree, where it is present) with a small driver,
once against the reference's kv_cache.c and once against this library.  The
transformer's per-layer loop (transformer.c:158-214) appends every token's
K/V with ct_kv_append and reads the cache back with ct_kv_get for each head
and position, so the library's device-resident cache is exercised exactly as
the engine uses it.  A tiny GQA llama model (2 layers, 8 query / 2 KV heads,
GGUF written by tests/engine_gguf.py) runs 40 steps; the logits of every step
must equal the reference's bit for bit (the KV rows round-trip exactly)."""
import subprocess
from pathlib import Path

import numpy as np
import pytest

from engine_gguf import write_tiny_llama

pytestmark = pytest.mark.gpu
REF = Path(__file__).resolve().parent.parent / "oracle" / "_ref"


@pytest.mark.skipif(not (REF / "engine_ours").exists() or not (REF / "engine_ref").exists(),
                    reason="engine programs not built (they need the reference sources at build time)")
def test_reference_transformer_loop_on_library_kv_cache(tmp_path):
    cfg = write_tiny_llama(tmp_path / "tiny.gguf")
    n = 40
    outs = {}
    for name in ("engine_ref", "engine_ours"):
        out = tmp_path / f"{name}.bin"
        r = subprocess.run([str(REF / name), str(tmp_path / "tiny.gguf"), str(n), str(out)], capture_output=True,
                           text=True, timeout=300)
        assert r.returncode == 0, r.stdout + r.stderr
        assert f"kv_len {n}" in r.stdout
        outs[name] = np.fromfile(out, np.float32).reshape(n, cfg["n_vocab"])
    assert np.isfinite(outs["engine_ref"]).all()
    assert np.array_equal(outs["engine_ours"].view(np.uint32), outs["engine_ref"].view(np.uint32))
