"""GPU: the fused producer (ct_kv_project_write_slots, ct_kv_paged_append_projected):
entry = W . x on the tensor cores, optional RMS norm, append with the pool's
codec.  The projection follows matvec_bf16 (ds4_forward.c:248-272, bf16
weights, fp32 accumulation) and rmsnorm_ip (ds4_forward.c:206-211); the
check is an fp64 restatement on the same bf16 inputs.  Tolerance: fp32
accumulation over n_in products, |got - want| <= 2e-5 * (|want| + rms(row)).
The pool writes after the projection must equal, bit for bit, the fp32
entries passed through each codec (the same kernels as a plain append)."""
import numpy as np
import pytest

import cautreo_b200 as ct
import oracle
from gpu_util import dev, empty, host, stream

pytestmark = pytest.mark.gpu
O = oracle.port()


@pytest.fixture(autouse=True)
def no_expired_waits():
    ct.lib().ct_kv_project_error(1)
    yield
    assert ct.lib().ct_kv_project_error(1) == 0


def inputs(n, n_in, dim, seed):
    x = oracle.normal_bf16(oracle.key(seed, 50), 0, n * n_in).reshape(n, n_in)
    w = oracle.normal_bf16(oracle.key(seed, 51), 0, dim * n_in, 0, 0.02).reshape(dim, n_in)
    return x, w


def want_entries(x, w, norm_w=None, eps=1e-6, norm_dim=0):
    xf = oracle.bf16_to_f32(x).reshape(x.shape).astype(np.float64)
    wf = oracle.bf16_to_f32(w).reshape(w.shape).astype(np.float64)
    e = xf @ wf.T
    if norm_w is not None:
        ss = (e[:, :norm_dim] ** 2).sum(axis=1)
        inv = 1.0 / np.sqrt((ss / norm_dim).astype(np.float32) + np.float32(eps))
        e[:, :norm_dim] = e[:, :norm_dim] * inv[:, None] * norm_w[None, :norm_dim].astype(np.float64)
    return e


def close(got, want, tol=2e-5):
    rms = np.sqrt((want ** 2).mean(axis=1, keepdims=True))
    err = np.abs(got.astype(np.float64) - want)
    return bool(np.all(err <= tol * (np.abs(want) + rms))), float(err.max())


def project(x, w, n, n_in, dim, pool_dtype, norm_w=None, eps=1e-6, norm_dim=0, n_pages=None):
    """Runs the stateless call into a fresh pool; slots 0..n-1 in order."""
    P = 64
    n_pages = n_pages or (n + P - 1) // P
    eb = ct.entry_bytes(pool_dtype, dim)
    pool = empty((n_pages * P * eb,), np.uint8)
    scales = empty((n_pages * P,), np.float32) if pool_dtype in (ct.CT_KV_INT8, ct.CT_KV_E4M3) else None
    dest = dev(np.arange(n, dtype=np.int32))
    xd, wd = dev(x), dev(w)
    nw = dev(np.ascontiguousarray(norm_w, np.float32)) if norm_w is not None else None
    L = ct.lib()
    ct.check(L.ct_kv_project_write_slots(xd.data_ptr(), wd.data_ptr(), nw.data_ptr() if nw is not None else None,
                                         eps, norm_dim, n, n_in, dim, pool.data_ptr(),
                                         scales.data_ptr() if scales is not None else None, pool_dtype,
                                         dest.data_ptr(), stream()))
    codes = host(pool, np.uint8)[:n * eb].reshape(n, eb)
    sc = host(scales, np.float32)[:n] if scales is not None else None
    return codes, sc


@pytest.mark.parametrize("n,n_in,dim", [(1, 512, 576), (37, 4096, 576), (300, 4096, 576), (130, 1024, 512),
                                        (1024, 4096, 576), (8192, 512, 576), (6500, 512, 576),
                                        # two token tiles per CTA with 128- and 64-wide output tiles
                                        # (640 = 10 x 64, 320 = 5 x 64), the second with a ragged tail
                                        (8192, 512, 640), (6500, 512, 320)])
def test_projection_matches_fp64(n, n_in, dim):
    x, w = inputs(n, n_in, dim, 1)
    codes, _ = project(x, w, n, n_in, dim, ct.CT_KV_F32)
    got = codes.view(np.float32).reshape(n, dim)
    ok, mx = close(got, want_entries(x, w))
    assert ok, mx


def test_projection_with_rms_norm():
    n, n_in, dim, nd = 200, 2048, 576, 512
    x, w = inputs(n, n_in, dim, 2)
    norm_w = 1.0 + 0.1 * oracle.normal_f32(oracle.key(2, 52), 0, dim)
    codes, _ = project(x, w, n, n_in, dim, ct.CT_KV_F32, norm_w=norm_w, eps=1e-6, norm_dim=nd)
    got = codes.view(np.float32).reshape(n, dim)
    ok, mx = close(got, want_entries(x, w, norm_w, 1e-6, nd), tol=1e-4)
    assert ok, mx


@pytest.mark.parametrize("pool_dtype", [ct.CT_KV_BF16, ct.CT_KV_INT8, ct.CT_KV_E4M3, ct.CT_KV_Q4_0])
def test_projected_pool_writes_equal_codec_of_fp32(pool_dtype):
    """bf16 / int8 / e4m3 / Q4_0 pools hold exactly what the plain append
    writes for the fp32 entries the projection produced."""
    n, n_in, dim = 100, 1024, 576
    x, w = inputs(n, n_in, dim, 3)
    f32, _ = project(x, w, n, n_in, dim, ct.CT_KV_F32)
    e = np.ascontiguousarray(f32.view(np.float32).reshape(n, dim))
    codes, sc = project(x, w, n, n_in, dim, pool_dtype)
    if pool_dtype == ct.CT_KV_BF16:
        assert np.array_equal(codes.view(np.uint16).reshape(n, dim), oracle.f32_to_bf16(e).reshape(n, dim))
    elif pool_dtype in (ct.CT_KV_INT8, ct.CT_KV_E4M3):
        wc = np.zeros(n * dim, np.uint8)
        ws = np.zeros(n, np.float32)
        fn = O.orc_kv_quant_int8 if pool_dtype == ct.CT_KV_INT8 else O.orc_kv_quant_e4m3
        fn(e.ctypes.data, n, dim, wc.ctypes.data, ws.ctypes.data)
        assert np.array_equal(codes.reshape(-1), wc) and np.array_equal(sc, ws)
    else:
        R = oracle.ref()
        want = np.zeros_like(codes)
        for t in range(n):
            R.ct_quant_q4_0(np.ascontiguousarray(e[t]).ctypes.data, want[t].ctypes.data, dim)
        assert np.array_equal(codes, want)


def test_paged_append_projected_matches_stateless():
    """The paged handle allocates like ct_kv_paged_append (ragged counts,
    page boundaries) and fills the slots with the projected entries."""
    S, P, dim, n_in, NP = 4, 64, 576, 1024, 32
    lens = [1, 64, 65, 130]
    n = sum(lens)
    x, w = inputs(n, n_in, dim, 4)
    h = ct.PagedKV(S, 8, NP, P, dim, 0, ct.CT_KV_BF16, 0, stream())
    h.set_free_order(oracle.permutation(oracle.key(4, 1), NP))
    xd, wd = dev(x), dev(w)
    h.append_projected(list(range(S)), lens, xd.data_ptr(), wd.data_ptr(), n_in)
    f32, _ = project(x, w, n, n_in, dim, ct.CT_KV_F32)
    want = oracle.f32_to_bf16(f32.view(np.float32).reshape(n, dim)).reshape(n, dim)
    off = 0
    for s, c in enumerate(lens):
        out = empty((c, dim), np.uint16)
        h.gather(s, 0, c, out.data_ptr(), ct.CT_KV_BF16)
        assert np.array_equal(host(out, np.uint16), want[off:off + c]), s
        off += c
    h.close()
