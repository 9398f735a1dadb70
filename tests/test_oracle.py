"""CPU: pin the oracle restatement against the reference's own code and the
committed golden fixtures (tests/golden/, made by make_golden.py)."""
import ctypes as C
import subprocess
from pathlib import Path

import numpy as np
import pytest

import oracle
from helpers import MLA_DV, MLA_E, MLA_SCALE, PAGE, mla_case, plain_inputs

GOLD = Path(__file__).resolve().parent / "golden"
O = oracle.port()
needs_ref = pytest.mark.skipif(not oracle.ref_available(), reason="reference objects not built here")


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


# ---- reference unit tests (kv_cache_test.c, attention_test.c, quant_test.c) --

@pytest.mark.skipif(not (oracle.HERE / "_ref" / "quant_test").exists(), reason="reference tests not built")
@pytest.mark.parametrize("name", ["kv_cache_test", "attention_test", "quant_test"])
def test_reference_unit_tests_pass(name, tmp_path):
    (tmp_path / "build").mkdir()
    r = subprocess.run([str(oracle.HERE / "_ref" / name)], cwd=tmp_path, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout


# ---- fp16 / bf16 / e4m3 ------------------------------------------------------

def test_fp16_decode_matches_golden_exhaustive():
    g = np.load(GOLD / "quant_ref.npz")
    mine = np.array([O.orc_ct_fp16_to_f32(h) for h in range(65536)], np.float32)
    assert np.array_equal(bits(mine), bits(g["fp16_to_f32"]))


def test_fp16_encode_matches_golden():
    g = np.load(GOLD / "quant_ref.npz")
    mine = np.array([O.orc_ct_f32_to_fp16(float(v)) for v in g["f32"]], np.uint16)
    assert np.array_equal(mine, g["f32_to_fp16"])


@needs_ref
def test_fp16_encode_matches_reference_random_bits():
    R = oracle.ref()
    rng = np.random.default_rng(0)
    u = rng.integers(0, 2 ** 32, 200000, dtype=np.uint64).astype(np.uint32)
    f = u.view(np.float32)
    for v in f[:20000]:
        assert O.orc_ct_f32_to_fp16(float(v)) == R.ct_quant_f32_to_fp16(float(v))


def test_fp16_quirks():
    # |x| < 2^-15 encodes as Inf (unsigned exponent wrap); exponent 112 is a subnormal
    assert O.orc_ct_f32_to_fp16(1e-5) == 0x7C00
    assert O.orc_ct_f32_to_fp16(-1e-5) == 0xFC00
    assert O.orc_ct_f32_to_fp16(2.0 ** -15) == 0x0200
    # truncation, not rounding
    assert O.orc_ct_f32_to_fp16(1.0 + 2 ** -11 + 2 ** -12) == 0x3C00
    # decode halves subnormals
    assert O.orc_ct_fp16_to_f32(1) == 2.0 ** -25


def test_bf16_rne():
    for f, want in [(1.0, 0x3F80), (1.00390625, 0x3F80), (1.01171875, 0x3F82), (-2.5, 0xC020)]:
        assert O.orc_f32_to_bf16(f) == want
    x = oracle.normal_f32(oracle.key(5, 5), 0, 10000)
    assert np.array_equal(np.array([O.orc_f32_to_bf16(float(v)) for v in x], np.uint16), oracle.f32_to_bf16(x))


def test_e4m3_codebook_roundtrip_and_saturation():
    for c in range(256):
        v = O.orc_e4m3_to_f32(c)
        if np.isnan(v):
            assert c & 0x7F == 0x7F
            continue
        back = O.orc_f32_to_e4m3_satfinite(v)
        assert back == c or (v == 0 and back in (0, 0x80)), (c, v, back)
    assert O.orc_f32_to_e4m3_satfinite(1e6) == 0x7E
    assert O.orc_f32_to_e4m3_satfinite(-500.0) == 0xFE
    assert O.orc_f32_to_e4m3_satfinite(float("inf")) == 0x7E
    assert O.orc_e4m3_to_f32(0x7E) == 448.0
    assert O.orc_e4m3_to_f32(0x01) == 2.0 ** -9
    # ties go to even: 1 + 1/16 lies between 1 and 1.125 -> 1.0 (mantissa 0)
    assert O.orc_f32_to_e4m3_satfinite(1.0625) == 0x38
    assert O.orc_f32_to_e4m3_satfinite(1.1875) == 0x3A    # between 1.125 and 1.25 -> 1.25 (even)


def test_e4m3_nearest():
    codes = np.arange(256)
    vals = np.array([O.orc_e4m3_to_f32(int(c)) for c in codes], np.float64)
    finite = ~np.isnan(vals)
    x = oracle.normal_f32(oracle.key(6, 6), 0, 5000) * np.float32(50)
    for v in x:
        c = O.orc_f32_to_e4m3_satfinite(float(v))
        got = O.orc_e4m3_to_f32(c)
        best = np.min(np.abs(vals[finite] - min(max(float(v), -448), 448)))
        assert abs(got - min(max(float(v), -448), 448)) == pytest.approx(best, abs=0)


# ---- block codecs ---------------------------------------------------------------

def test_q8_0_matches_golden():
    g = np.load(GOLD / "quant_ref.npz")
    x = g["x"]
    enc = np.zeros((len(x), 34), np.uint8)
    xc = np.ascontiguousarray(x)
    O.orc_q8_0_quantize(oracle.ptr(xc), oracle.ptr(enc), x.size)
    assert np.array_equal(enc, g["enc1"])
    dec = np.zeros_like(x)
    O.orc_q8_0_dequantize(oracle.ptr(enc), oracle.ptr(dec), x.size)
    assert np.array_equal(bits(dec), bits(g["dec1"]))


@needs_ref
def test_q8_0_matches_reference_random():
    R = oracle.ref()
    x = oracle.normal_f32(oracle.key(4, 4), 0, 32 * 4096, 100, 20.0)
    x[:32 * 16] *= np.float32(1e-4)                    # tiny blocks: fp16 scale quirk path
    mine = np.zeros(4096 * 34, np.uint8)
    ref = np.zeros(4096 * 34, np.uint8)
    O.orc_q8_0_quantize(oracle.ptr(x), oracle.ptr(mine), x.size)
    R.ct_quant_q8_0(oracle.ptr(x), oracle.ptr(ref), x.size)
    assert np.array_equal(mine, ref)


def test_q8_0_reference_known_answers():
    # quant_test.c:55-145: ramp within rel-err 0.02, constant 1.0 within 0.01, zeros stay zero
    g = np.load(GOLD / "quant_ref.npz")
    x, dec = g["x"], g["dec1"]
    ramp, const, zero = x[0], x[1], x[2]
    nz = np.abs(ramp) > 1e-6
    assert np.all(np.abs(dec[0][nz] - ramp[nz]) / np.abs(ramp[nz]) <= 0.02)
    assert np.all(np.abs(dec[1] - const) <= 0.01)
    assert np.all(dec[2] == 0)
    assert g["enc1"].shape[1] == 34


# ---- per-token codecs -----------------------------------------------------------

def test_int8_token_codec_properties():
    n, dim = 64, 576
    x = oracle.normal_f32(oracle.key(2, 0), 0, n * dim, 100, 20.0)
    codes = np.zeros(n * dim, np.int8)
    sc = np.zeros(n, np.float32)
    O.orc_kv_quant_int8(oracle.ptr(x), n, dim, oracle.ptr(codes), oracle.ptr(sc))
    back = np.zeros_like(x)
    O.orc_kv_dequant_int8(oracle.ptr(codes), oracle.ptr(sc), n, dim, oracle.ptr(back))
    xr, cr = x.reshape(n, dim), codes.reshape(n, dim)
    assert np.all(np.abs(cr).max(axis=1) == 127)
    assert np.all(np.abs(back.reshape(n, dim) - xr) <= sc[:, None] * 0.5 * (1 + 1e-5))
    assert np.allclose(sc, np.abs(xr).max(axis=1) / 127, rtol=1e-7)


def test_e4m3_token_codec_properties():
    n, dim = 64, 576
    x = oracle.normal_f32(oracle.key(2, 1), 0, n * dim, 100, 20.0)
    codes = np.zeros(n * dim, np.uint8)
    sc = np.zeros(n, np.float32)
    O.orc_kv_quant_e4m3(oracle.ptr(x), n, dim, oracle.ptr(codes), oracle.ptr(sc))
    back = np.zeros_like(x)
    O.orc_kv_dequant_e4m3(oracle.ptr(codes), oracle.ptr(sc), n, dim, oracle.ptr(back))
    rel = np.abs(back - x) / np.maximum(np.abs(x), 1e-30)
    big = np.abs(x) > (np.repeat(sc, dim) * 2.0 ** -6)        # normal e4m3 range: rel err <= 2^-4
    assert np.all(rel[big] <= 2.0 ** -4 + 1e-6)
    assert np.all((codes.reshape(n, dim) & 0x7F).max(axis=1) == 0x7E)   # amax -> 448


# ---- attention -------------------------------------------------------------------

def test_attention_matches_golden_bitwise():
    g = np.load(GOLD / "attn_ref.npz")
    ci = 0
    while f"c{ci}" in g:
        n, H, D = (int(v) for v in g[f"c{ci}"])
        o = np.zeros(H * D, np.float32)
        assert O.orc_attn_forward(oracle.ptr(g[f"q{ci}"]), oracle.ptr(g[f"k{ci}"]), oracle.ptr(g[f"v{ci}"]), n, H, D,
                                  float(g[f"s{ci}"][0]), oracle.ptr(o)) == 0
        assert np.array_equal(bits(o), bits(g[f"o{ci}"])), ci
        ci += 1
    y = g["sm_x"].copy()
    O.orc_attn_softmax(oracle.ptr(y), len(y))
    assert np.array_equal(bits(y), bits(g["sm_y"]))


def test_attention_reference_known_answers():
    # attention_test.c:17-39
    x = np.array([1, 2, 3], np.float32)
    O.orc_attn_softmax(oracle.ptr(x), 3)
    assert abs(x.sum() - 1) < 1e-5 and x[2] > x[1] > x[0]
    q = np.array([1, 0, 0, 0], np.float32)
    k = np.array([1, 0, 0, 0], np.float32)
    v = np.array([5, 6, 7, 8], np.float32)
    o = np.zeros(4, np.float32)
    O.orc_attn_forward(oracle.ptr(q), oracle.ptr(k), oracle.ptr(v), 1, 1, 4, 1.0, oracle.ptr(o))
    assert abs(o[0] - 5) < 1e-5
    k2 = np.array([1, 0, 0, 0, 0, 1, 0, 0], np.float32)
    v2 = np.array([5, 0, 0, 0, 0, 9, 0, 0], np.float32)
    O.orc_attn_forward(oracle.ptr(q), oracle.ptr(k2), oracle.ptr(v2), 2, 1, 4, 1.0, oracle.ptr(o))
    assert abs(o[0] - 0.731 * 5) < 1e-2 and o[0] > o[1]


def test_plain_decode_matches_golden_bitwise():
    g = np.load(GOLD / "plain_ref.npz")
    q, k, v = plain_inputs()
    assert np.array_equal(q[:2, 0, :8], g["q_head"]) and np.array_equal(k[:2, 0, :8], g["k_head"])
    L, H, D = 4, 8, 64
    for si, s in enumerate(g["steps"]):
        n = int(s) + 1
        for l in range(L):
            for h in range(H):
                kh = np.ascontiguousarray(k[:n, l, h * D:(h + 1) * D])
                vh = np.ascontiguousarray(v[:n, l, h * D:(h + 1) * D])
                qh = np.ascontiguousarray(q[s, l, h * D:(h + 1) * D])
                o = np.zeros(D, np.float32)
                O.orc_attn_forward(oracle.ptr(qh), oracle.ptr(kh), oracle.ptr(vh), n, 1, D, 0.0, oracle.ptr(o))
                assert np.array_equal(bits(o), bits(g["out"][si, l, h * D:(h + 1) * D])), (s, l, h)


def test_mla_decode_matches_golden_bitwise():
    g = np.load(GOLD / "mla_ref.npz")
    lens = g["lens"]
    H = int(g["heads"])
    pool, bt, q = mla_case(lens, seed=1, H=H)
    assert np.array_equal(pool.reshape(-1)[:64], g["pool_head"]) and np.array_equal(bt, g["bt"])
    out = oracle.mla_decode_paged(pool, bt, lens, q, H, MLA_E, MLA_DV, PAGE, MLA_SCALE)
    assert np.array_equal(bits(out), bits(g["out"]))


def test_mla_skips_unmapped_pages():
    lens = [200]
    pool, bt, q = mla_case(lens, seed=5, H=4)
    full = oracle.mla_decode_paged(pool, bt, lens, q, 4, MLA_E, MLA_DV, PAGE, MLA_SCALE)
    bt2 = bt.copy()
    bt2[0, 0] = -1
    part = oracle.mla_decode_paged(pool, bt2, lens, q, 4, MLA_E, MLA_DV, PAGE, MLA_SCALE)
    # attending only tokens 64..199 equals decoding a sequence made of those tokens
    kv = np.stack([oracle.bf16_to_f32(pool[bt[0, t // PAGE], t % PAGE]) for t in range(64, 200)])
    o = np.zeros((4, MLA_DV), np.float32)
    q0 = np.ascontiguousarray(oracle.bf16_to_f32(q[0]))
    O.orc_mla_decode(oracle.ptr(q0), oracle.ptr(kv), 136, 4, MLA_E,
                     MLA_DV, MLA_SCALE, oracle.ptr(o))
    assert np.array_equal(bits(part[0]), bits(o))
    assert not np.array_equal(part, full)


# ---- contiguous compaction -------------------------------------------------------

def test_compress_matches_golden():
    g = np.load(GOLD / "kv_ref.npz")
    L, H, D, ctx = 2, 4, 8, 16
    for ci in range(5):
        n, ok, m = (int(v) for v in g[f"cmp{ci}"])
        ratio = float(g[f"cmp{ci}_ratio"][0])
        kk = oracle.normal_f32(oracle.key(9, ci), 0, n * L * H * D).reshape(n, L, H * D)
        vv = oracle.normal_f32(oracle.key(9, ci), 1 << 20, n * L * H * D).reshape(n, L, H * D)
        kc = np.zeros((L, ctx, H * D), np.float32)
        vc = np.zeros((L, ctx, H * D), np.float32)
        kc[:, :n] = kk.transpose(1, 0, 2)
        vc[:, :n] = vv.transpose(1, 0, 2)
        if ratio <= 1.0:
            continue
        m2 = O.orc_kv_compress_every_kth(oracle.ptr(kc), oracle.ptr(vc), L, ctx, H * D, n, ratio)
        assert m2 == m and ok == 1
        assert np.array_equal(kc[:, :m], g[f"cmp{ci}_k"]) and np.array_equal(vc[:, :m], g[f"cmp{ci}_v"])


# ---- paged allocator -------------------------------------------------------------

def test_alloc_matches_golden():
    g = np.load(GOLD / "alloc_ref.npz")
    S, P, NP, MP, W = (int(v) for v in g["cfg"])
    rc, bt, owner, ev, last, nfree = oracle.alloc_replay(g["lens"], S, P, NP, MP, W)
    assert rc == 0
    assert np.array_equal(bt, g["bt"]) and np.array_equal(owner, g["owner"])
    assert np.array_equal(np.array(ev, np.int64), g["events"]) and nfree == int(g["n_free"])
    cbt, cmap = oracle.compact_plan(bt)
    assert np.array_equal(cbt, g["compact_bt"]) and np.array_equal(cmap, g["compact_map"])


@pytest.mark.parametrize("S,P,NP,W,lo,hi", [(12, 4, 22, 12, 8, 128), (40, 8, 60, 0, 1, 300), (64, 16, 90, 64, 16, 600)])
def test_alloc_invariants(S, P, NP, W, lo, hi):
    lens = oracle.lengths_loguniform(oracle.key(3, S), S, lo, hi)
    MP = (hi + P - 1) // P + 1
    rc, bt, owner, ev, last, nfree = oracle.alloc_replay(lens, S, P, NP, MP, W)
    assert rc == 0
    live = bt[bt >= 0]
    assert len(np.unique(live)) == len(live) and len(live) + nfree == NP
    for s in range(S):
        mapped = np.nonzero(bt[s] >= 0)[0]
        if len(mapped):
            assert np.all(np.diff(mapped) == 1)                     # one contiguous run
            assert mapped[-1] == (lens[s] - 1) // P                  # tail page always kept
            if W:
                assert (mapped[0] + 1) * P > int(lens[s]) - W             # nothing wholly outside the window
        for lp in mapped:                                            # slot owners agree with the table
            for j in range(P):
                t = lp * P + j
                if t < lens[s]:
                    assert owner[bt[s, lp], j] == (s << 32 | t)
    for (r, s, lp, ph, why) in ev:
        assert why in (1, 2)
        if why == 2:
            assert (lp + 1) * P <= min(int(lens[s]), r + 1)               # LRU takes full pages only


def test_compact_plan_orders_by_seq_then_page():
    bt = np.array([[5, 2, -1], [-1, 7, 0], [3, -1, -1]], np.int32)
    cbt, cmap = oracle.compact_plan(bt)
    assert cbt.tolist() == [[0, 1, -1], [-1, 2, 3], [4, -1, -1]]
    assert cmap.tolist() == [5, 2, 7, 0, 3]


def test_lpt_balances():
    lens = oracle.lengths_loguniform(oracle.key(4, 0), 1024, 512, 65536)
    for R_ in (1, 2, 4, 8):
        r = oracle.lpt(lens, R_)
        load = np.bincount(r, weights=lens, minlength=R_)
        assert load.max() - load.min() <= lens.max()
        assert load.max() / load.mean() < 1.01


def test_reference_engine_runs_on_the_tiny_gguf(tmp_path):
    """The reference engine's transformer forward (compiled from the
    reference sources with oracle/engine_drive.c) loads the synthetic GGUF
    and decodes; its logits are finite and repeat run to run."""
    import subprocess
    from engine_gguf import write_tiny_llama
    exe = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "engine_ref"
    if not exe.exists():
        pytest.skip("engine_ref not built (needs the reference sources at build time)")
    cfg = write_tiny_llama(tmp_path / "tiny.gguf")
    runs = []
    for i in range(2):
        out = tmp_path / f"l{i}.bin"
        r = subprocess.run([str(exe), str(tmp_path / "tiny.gguf"), "12", str(out)], capture_output=True, text=True,
                           timeout=120)
        assert r.returncode == 0, r.stderr
        runs.append(np.fromfile(out, np.float32).reshape(12, cfg["n_vocab"]))
    assert np.isfinite(runs[0]).all() and runs[0].std() > 0.1
    assert np.array_equal(runs[0], runs[1])
