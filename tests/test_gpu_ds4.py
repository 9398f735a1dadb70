"""GPU: the MLA-lite cache of ds4_forward.c (store at :1565-1570, attention at
:1572-1627) through ct_ds4_attend, against the oracle's MLA decode on the same
fp32 latents and the bf16-rounded query (scale 1/sqrt(kv_dim), one head, V =
the latent).  Tolerance, elementwise: |got - ref| <= 2e-2 + 1e-2 |ref| (bf16
query and output)."""
import ctypes as C

import numpy as np
import pytest

import cautreo_b200 as ct
import oracle
from helpers import close

pytestmark = pytest.mark.gpu
O = oracle.port()


def expected(cache_rows, q, dim):
    kv = np.ascontiguousarray(np.stack(cache_rows), np.float32)
    qb = oracle.bf16_to_f32(oracle.f32_to_bf16(q)).astype(np.float32)
    out = np.zeros(dim, np.float32)
    assert O.orc_mla_decode(qb.ctypes.data, kv.ctypes.data, len(cache_rows), 1, dim, dim,
                            1.0 / np.sqrt(np.float32(dim)), out.ctypes.data) == 0
    return out


def test_ds4_cache_store_attend_overwrite_and_full_context():
    L = ct.lib()
    n_layers, ctx, dim = 3, 200, 512
    c = L.ct_ds4_cache_create(n_layers, ctx, dim, 0)
    assert c, L.ct_hal_cuda_last_error()
    caches = [[] for _ in range(n_layers)]
    out = np.zeros(dim, np.float32)
    k = oracle.key(60, 0)
    for pos in range(ctx + 30):                        # past ctx: no store, attention over the full cache
        for layer in range(n_layers):
            kv_a = oracle.normal_f32(k, ((pos * n_layers + layer) * 2) * dim, dim)
            q = oracle.normal_f32(k, ((pos * n_layers + layer) * 2 + 1) * dim, dim)
            if pos < ctx:
                caches[layer].append(kv_a)
            ct.check(L.ct_ds4_attend(c, layer, pos, kv_a.ctypes.data, q.ctypes.data, out.ctypes.data))
            if pos % 37 == 0 or pos in (1, 63, 64, 65, ctx - 1, ctx, ctx + 29):
                want = expected(caches[layer][:min(pos + 1, ctx)], q, dim)
                ok, mx, rel = close(out[None, :], want[None, :])
                assert ok, (pos, layer, mx, rel)
    assert [L.ct_ds4_cache_len(c, i) for i in range(n_layers)] == [ctx] * n_layers
    # overwrite position 10 of layer 1, then attend at position 10 and at the end
    new = oracle.normal_f32(oracle.key(60, 1), 0, dim)
    q = oracle.normal_f32(oracle.key(60, 2), 0, dim)
    caches[1][10] = new
    ct.check(L.ct_ds4_attend(c, 1, 10, new.ctypes.data, q.ctypes.data, out.ctypes.data))
    ok, mx, rel = close(out[None, :], expected(caches[1][:11], q, dim)[None, :])
    assert ok, (mx, rel)
    ct.check(L.ct_ds4_attend(c, 1, ctx + 5, None, q.ctypes.data, out.ctypes.data))
    ok, mx, rel = close(out[None, :], expected(caches[1], q, dim)[None, :])
    assert ok, (mx, rel)
    L.ct_ds4_cache_destroy(c)
    # a gap in the positions is refused
    c2 = L.ct_ds4_cache_create(1, 64, dim, 0)
    assert L.ct_ds4_attend(c2, 0, 5, new.ctypes.data, q.ctypes.data, out.ctypes.data) == ct.CT_ERR_ARG
    L.ct_ds4_cache_destroy(c2)
