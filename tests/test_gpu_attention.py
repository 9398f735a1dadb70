"""GPU: the reference ct_attn_* interface and the plain contiguous-cache
decode against the reference's own CPU code (golden fixtures)."""
from pathlib import Path

import numpy as np
import pytest
import torch

import cautreo_b200 as ct
import oracle
from gpu_util import dev, empty, host, stream
from helpers import plain_inputs

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"

# fp32 kernels against the reference's fp64-accumulated CPU results
ATTN_TOL = 1e-5          # ct_attn_forward / softmax keep fp64 accumulation
DECODE_TOL = 1e-4        # fp32 FMA online-softmax decode


def test_attn_forward_matches_reference_golden():
    g = np.load(GOLD / "attn_ref.npz")
    L = ct.lib()
    before = ct.launch_count()
    ci = 0
    while f"c{ci}" in g:
        n, H, D = (int(v) for v in g[f"c{ci}"])
        o = np.zeros(H * D, np.float32)
        assert L.ct_attn_forward(g[f"q{ci}"].ctypes.data, g[f"k{ci}"].ctypes.data, g[f"v{ci}"].ctypes.data, n, H, D,
                                 float(g[f"s{ci}"][0]), o.ctypes.data)
        np.testing.assert_allclose(o, g[f"o{ci}"], rtol=ATTN_TOL, atol=ATTN_TOL, err_msg=str(ci))
        o2 = np.zeros(H * D, np.float32)
        assert L.ct_attn_forward_kv(g[f"q{ci}"].ctypes.data, g[f"k{ci}"].ctypes.data, g[f"v{ci}"].ctypes.data, n, H,
                                    D, float(g[f"s{ci}"][0]), o2.ctypes.data)
        assert np.array_equal(o, o2)
        ci += 1
    assert ct.launch_count() > before
    y = g["sm_x"].copy()
    L.ct_attn_softmax(y.ctypes.data, len(y))
    np.testing.assert_allclose(y, g["sm_y"], rtol=ATTN_TOL, atol=1e-9)


@pytest.mark.parametrize("n,H,D", [(20000, 4, 64), (5000, 3, 200), (4096, 2, 1)])
def test_attn_forward_long_contexts_match_reference(n, H, D):
    """From 4096 tokens ct_attn_forward runs split over many CTAs (per-tile
    maxima, sums and value sums in fp64, merged per head); the result stays
    within the tolerance of the reference's own ct_attn_forward."""
    R, L = oracle.ref(), ct.lib()
    rng = np.random.default_rng(n * 7 + H * 3 + D)
    q = rng.standard_normal(H * D).astype(np.float32)
    k = rng.standard_normal(n * D).astype(np.float32)
    v = rng.standard_normal(n * D).astype(np.float32)
    want = np.zeros(H * D, np.float32)
    got = np.zeros(H * D, np.float32)
    assert R.ct_attn_forward(q.ctypes.data, k.ctypes.data, v.ctypes.data, n, H, D, 0.0, want.ctypes.data)
    assert L.ct_attn_forward(q.ctypes.data, k.ctypes.data, v.ctypes.data, n, H, D, 0.0, got.ctypes.data)
    np.testing.assert_allclose(got, want, rtol=ATTN_TOL, atol=ATTN_TOL)


@pytest.mark.parametrize("n", [65536, 300000])
def test_softmax_long_inputs_match_reference(n):
    """From 65536 values ct_attn_softmax runs split over many CTAs; also with
    a NaN after the first value, which the reference's maximum skips but its
    sum does not (the values are then left unnormalised)."""
    R, L = oracle.ref(), ct.lib()
    x = (np.random.default_rng(n).standard_normal(n) * 4).astype(np.float32)
    for case in (x, np.where(np.arange(n) == 70001 % n, np.float32(np.nan), x).astype(np.float32)):
        want, got = case.copy(), case.copy()
        R.ct_attn_softmax(want.ctypes.data, n)
        L.ct_attn_softmax(got.ctypes.data, n)
        assert np.array_equal(np.isnan(got), np.isnan(want))
        ok = ~np.isnan(want)
        np.testing.assert_allclose(got[ok], want[ok], rtol=ATTN_TOL, atol=1e-9)


def test_attention_test_known_answers():
    """attention_test.c:17-39 through the device path."""
    L = ct.lib()
    x = np.array([1, 2, 3], np.float32)
    L.ct_attn_softmax(x.ctypes.data, 3)
    assert abs(x.sum() - 1) < 1e-5 and x[2] > x[1] > x[0]
    q = np.array([1, 0, 0, 0], np.float32)
    k = np.array([1, 0, 0, 0], np.float32)
    v = np.array([5, 6, 7, 8], np.float32)
    o = np.zeros(4, np.float32)
    assert L.ct_attn_forward(q.ctypes.data, k.ctypes.data, v.ctypes.data, 1, 1, 4, 1.0, o.ctypes.data)
    assert abs(o[0] - 5) < 1e-5
    k2 = np.array([1, 0, 0, 0, 0, 1, 0, 0], np.float32)
    v2 = np.array([5, 0, 0, 0, 0, 9, 0, 0], np.float32)
    assert L.ct_attn_forward(q.ctypes.data, k2.ctypes.data, v2.ctypes.data, 2, 1, 4, 1.0, o.ctypes.data)
    assert abs(o[0] - 0.731 * 5) < 1e-2 and o[0] > o[1]
    assert not L.ct_attn_forward(None, k.ctypes.data, v.ctypes.data, 1, 1, 4, 1.0, o.ctypes.data)
    assert not L.ct_attn_forward(q.ctypes.data, k.ctypes.data, v.ctypes.data, 0, 1, 4, 1.0, o.ctypes.data)


def test_plain_decode_run_matches_reference():
    """The CPU-runnable configuration end to end: 256 steps of (append one
    token to 4 layers -> attend over the whole cache), 8 heads x 64, fp32,
    through ct_kv_create + ct_attn_decode_step_contig on the cache's device
    arrays; outputs at the golden steps against the reference path."""
    g = np.load(GOLD / "plain_ref.npz")
    q, k, v = plain_inputs()
    Lyr, H, D, steps = 4, 8, 64, 256
    cache = ct.KvCache(Lyr, H, D, steps, 1.0)
    L = ct.lib()
    kd, vd = L.ct_kv_device_k(cache.h), L.ct_kv_device_v(cache.h)
    qd, kn, vn = dev(q), dev(k), dev(v)
    out = empty((steps, Lyr, H * D), np.float32)
    for s in range(steps):
        ct.check(L.ct_attn_decode_step_contig(qd[s].data_ptr(), kn[s].data_ptr(), vn[s].data_ptr(), kd, vd, Lyr,
                                              steps, H, H, D, s, 0.0, out[s].data_ptr(), stream()))
    got = host(out, np.float32)
    for si, s in enumerate(g["steps"]):
        np.testing.assert_allclose(got[s], g["out"][si], rtol=DECODE_TOL, atol=DECODE_TOL, err_msg=f"step {s}")
    # decode over the filled cache without appending gives the last step again
    out2 = empty((Lyr, H * D), np.float32)
    ct.check(L.ct_attn_decode_contig(qd[255].data_ptr(), kd, vd, Lyr, steps, H, H, D, 256, 0.0, out2.data_ptr(),
                                     stream()))
    np.testing.assert_allclose(host(out2, np.float32), g["out"][-1], rtol=DECODE_TOL, atol=DECODE_TOL)


def test_decode_contig_gqa_matches_reference():
    """Grouped heads: query head h reads KV head h % n_kv (transformer.c:187)."""
    R_ = oracle.port()
    Lyr, Hq, Hkv, D, n, ctx = 2, 8, 2, 64, 77, 100
    kc = oracle.normal_f32(oracle.key(13, 0), 0, Lyr * ctx * Hkv * D).reshape(Lyr, ctx, Hkv * D)
    vc = oracle.normal_f32(oracle.key(13, 1), 0, Lyr * ctx * Hkv * D).reshape(Lyr, ctx, Hkv * D)
    q = oracle.normal_f32(oracle.key(13, 2), 0, Lyr * Hq * D).reshape(Lyr, Hq, D)
    out = empty((Lyr, Hq, D), np.float32)
    qd, kd, vd = dev(q), dev(kc), dev(vc)           # keep the device buffers alive across the calls
    ct.check(ct.lib().ct_attn_decode_contig(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), Lyr, ctx,
                                            Hkv, Hq, D, n, 0.25, out.data_ptr(), stream()))
    got = host(out, np.float32)
    for l in range(Lyr):
        for h in range(Hq):
            kv = h % Hkv
            kh = np.ascontiguousarray(kc[l, :n, kv * D:(kv + 1) * D])
            vh = np.ascontiguousarray(vc[l, :n, kv * D:(kv + 1) * D])
            o = np.zeros(D, np.float32)
            R_.orc_attn_forward(np.ascontiguousarray(q[l, h]).ctypes.data, kh.ctypes.data, vh.ctypes.data, n, 1, D,
                                0.25, o.ctypes.data)
            np.testing.assert_allclose(got[l, h], o, rtol=DECODE_TOL, atol=DECODE_TOL)
    assert ct.lib().ct_attn_decode_contig(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), Lyr, ctx, Hkv,
                                          Hq, D, ctx + 1, 0.25, out.data_ptr(), stream()) == ct.CT_ERR_ARG
