"""GPU: block codecs (the reference ct_quant_* interface) and per-token KV
codecs, bit-exact against the reference's own code and the oracle."""
from pathlib import Path

import numpy as np
import pytest

import cautreo_b200 as ct
import oracle
from gpu_util import dev, empty, host, stream

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"
O = oracle.port()


def same_floats(a, b):
    """Bit-identical, except that any two NaNs match: the reference's decode
    of an Inf scale (0 * Inf) yields the host CPU's default NaN bit pattern,
    the GPU its canonical NaN."""
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    nan = np.isnan(a) & np.isnan(b)
    return bool(np.all(nan | (a.view(np.uint32) == b.view(np.uint32))))


def test_block_codecs_match_reference_golden():
    g = np.load(GOLD / "quant_ref.npz")
    L = ct.lib()
    x = np.ascontiguousarray(g["x"])
    before = ct.launch_count()
    for t, nb in ct.QUANT_BLOCK_BYTES.items():
        enc = np.zeros((len(x), nb), np.uint8)
        for i in range(len(x)):
            blk = np.ascontiguousarray(x[i])
            assert L.ct_quant_do(blk.ctypes.data, enc[i].ctypes.data, 32, t) == nb
        assert np.array_equal(enc, g[f"enc{t}"]), t
        dec = np.zeros_like(x)
        L.ct_quant_undo(enc.ctypes.data, dec.ctypes.data, x.size, t)
        assert same_floats(dec, g[f"dec{t}"]), t
    assert ct.launch_count() > before          # the CUDA kernels ran


def test_block_codec_entry_points_and_errors():
    L = ct.lib()
    x = oracle.normal_f32(oracle.key(4, 1), 0, 32 * 64, 100, 20.0)
    q8 = np.zeros(64 * 34, np.uint8)
    L.ct_quant_q8_0(x.ctypes.data, q8.ctypes.data, x.size)
    want = np.zeros_like(q8)
    O.orc_q8_0_quantize(x.ctypes.data, want.ctypes.data, x.size)
    assert np.array_equal(q8, want)
    out = np.zeros_like(x)
    L.ct_quant_deq8_0(q8.ctypes.data, out.ctypes.data, x.size)
    ref = np.zeros_like(x)
    O.orc_q8_0_dequantize(want.ctypes.data, ref.ctypes.data, x.size)
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))
    assert L.ct_quant_do(x.ctypes.data, q8.ctypes.data, 31, 1) == 0          # n % 32 != 0
    assert L.ct_quant_do(None, q8.ctypes.data, 32, 1) == 0
    assert L.ct_quant_do(x.ctypes.data, q8.ctypes.data, 32, 0) == 0          # FP16 has no block codec


@pytest.mark.skipif(not oracle.ref_available(), reason="reference objects not present")
def test_block_codecs_match_reference_random_quirks():
    R = oracle.ref()
    L = ct.lib()
    x = oracle.normal_f32(oracle.key(4, 2), 0, 32 * 2048, 100, 20.0)
    x[:32 * 64] *= np.float32(3e-4)                 # tiny blocks: Inf / subnormal fp16 scales
    for t, nb in ct.QUANT_BLOCK_BYTES.items():
        mine = np.zeros(2048 * nb, np.uint8)
        ref = np.zeros(2048 * nb, np.uint8)
        assert L.ct_quant_do(x.ctypes.data, mine.ctypes.data, x.size, t) == 2048 * nb
        R.ct_quant_do(x.ctypes.data, ref.ctypes.data, x.size, t)
        assert np.array_equal(mine, ref), t
        a = np.zeros_like(x)
        b = np.zeros_like(x)
        L.ct_quant_undo(mine.ctypes.data, a.ctypes.data, x.size, t)
        R.ct_quant_undo(ref.ctypes.data, b.ctypes.data, x.size, t)
        assert same_floats(a, b), t
        assert np.isnan(a).sum() == np.isnan(b).sum()


@pytest.mark.parametrize("codec", ["int8", "e4m3"])
@pytest.mark.parametrize("src", ["f32", "bf16"])
def test_token_codecs_bit_exact(codec, src):
    L = ct.lib()
    n, dim = 1000, 576
    x = oracle.normal_f32(oracle.key(2, 7), 0, n * dim, 100, 20.0)
    x[:dim] = 0.0                                    # all-zero token: scale 0, codes 0
    if src == "bf16":
        xb = oracle.f32_to_bf16(x)
        xin, xf = dev(xb), oracle.bf16_to_f32(xb)
    else:
        xin, xf = dev(x), x
    codes = empty((n * dim,), np.uint8)
    sc = empty((n,), np.float32)
    fn = L.ct_quant_kv_int8 if codec == "int8" else L.ct_quant_kv_e4m3
    ct.check(fn(xin.data_ptr(), int(src == "bf16"), n, dim, codes.data_ptr(), sc.data_ptr(), stream()))
    want_c = np.zeros(n * dim, np.uint8)
    want_s = np.zeros(n, np.float32)
    (O.orc_kv_quant_int8 if codec == "int8" else O.orc_kv_quant_e4m3)(
        np.ascontiguousarray(xf).ctypes.data, n, dim, want_c.ctypes.data, want_s.ctypes.data)
    got_c, got_s = host(codes, np.uint8), host(sc, np.float32)
    assert np.array_equal(got_s.view(np.uint32), want_s.view(np.uint32))
    assert np.array_equal(got_c, want_c)
    back = empty((n * dim,), np.float32)
    dq = L.ct_dequant_kv_int8 if codec == "int8" else L.ct_dequant_kv_e4m3
    ct.check(dq(codes.data_ptr(), sc.data_ptr(), n, dim, back.data_ptr(), stream()))
    want_b = np.zeros(n * dim, np.float32)
    (O.orc_kv_dequant_int8 if codec == "int8" else O.orc_kv_dequant_e4m3)(
        want_c.ctypes.data, want_s.ctypes.data, n, dim, want_b.ctypes.data)
    assert np.array_equal(host(back, np.float32).view(np.uint32), want_b.view(np.uint32))


def test_e4m3_conversion_matches_oracle_wide_range():
    """Tokens whose absmax is 448 have scale 1, so their codes are the raw
    e4m3 conversion of every value: compare with the oracle's OCP rule."""
    L = ct.lib()
    dim = 256
    vals = np.concatenate([
        (2.0 ** np.linspace(-12, 8.8, 200000)).astype(np.float32),
        oracle.normal_f32(oracle.key(6, 1), 0, 200000) * np.float32(30.0),
        np.array([0.0, -0.0, 2 ** -9, 2 ** -10, 3 * 2 ** -11, 448.0, 464.0, 480.0, -479.0, 1e9], np.float32),
    ]).astype(np.float32)
    per = dim - 1
    n_tok = (len(vals) + per - 1) // per
    x = np.zeros((n_tok, dim), np.float32)
    flat = np.zeros(n_tok * per, np.float32)
    flat[:len(vals)] = np.clip(vals, -448.0, 448.0)
    x[:, :per] = flat.reshape(n_tok, per)
    x[:, per] = 448.0
    codes = empty((n_tok * dim,), np.uint8)
    sc = empty((n_tok,), np.float32)
    xd = dev(x)
    ct.check(L.ct_quant_kv_e4m3(xd.data_ptr(), 0, n_tok, dim, codes.data_ptr(), sc.data_ptr(), stream()))
    got = host(codes, np.uint8).reshape(n_tok, dim)[:, :per].reshape(-1)[:len(vals)]
    assert np.all(host(sc, np.float32) == 1.0)
    want = np.array([O.orc_f32_to_e4m3_satfinite(float(v)) for v in flat[:len(vals)]], np.uint8)
    assert np.array_equal(got, want)


def test_q8_0_device_entry_points():
    L = ct.lib()
    x = oracle.normal_f32(oracle.key(4, 3), 0, 32 * 500, 100, 20.0)
    blk = empty((500 * 34,), np.uint8)
    xd = dev(x)
    ct.check(L.ct_quant_q8_0_dev(xd.data_ptr(), blk.data_ptr(), x.size, stream()))
    want = np.zeros(500 * 34, np.uint8)
    O.orc_q8_0_quantize(x.ctypes.data, want.ctypes.data, x.size)
    assert np.array_equal(host(blk, np.uint8), want)
    back = empty((x.size,), np.float32)
    ct.check(L.ct_dequant_q8_0_dev(blk.data_ptr(), back.data_ptr(), x.size, stream()))
    ref = np.zeros_like(x)
    O.orc_q8_0_dequantize(want.ctypes.data, ref.ctypes.data, x.size)
    assert np.array_equal(host(back, np.float32).view(np.uint32), ref.view(np.uint32))
    assert L.ct_quant_q8_0_dev(xd.data_ptr(), blk.data_ptr(), 33, stream()) == ct.CT_ERR_ARG
