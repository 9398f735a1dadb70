"""GPU: ct_attn_mla_decode_paged_noalloc, the MLA decode for callers that may
not allocate device memory on their decode path (an engine that reserved
almost all of HBM for its KV pool, or a serving loop that bans allocator
calls once running).  It must give the same results as the planned entry
point (ct_mla_plan_create + ct_attn_mla_decode_paged) and as the oracle,
within the attention tolerance, call after call, without changing the
device's free memory.

This file sorts last so that a run stopping at the first failure has run every
other test first; it also passes on its own in a fresh process."""
import ctypes as C

import numpy as np
import pytest
import torch

import cautreo_b200 as ct
import oracle
from gpu_util import dev, empty, host, stream
from helpers import MLA_DV, MLA_E, MLA_H, MLA_SCALE, PAGE, close, mla_case

pytestmark = pytest.mark.gpu


def free_bytes():
    return int(ct.lib().ct_dist_available_memory(None, 0))


def test_noalloc_matches_planned_decode_twice():
    torch.cuda.set_device(0)
    L = ct.lib()
    lens = np.array([5000, 3, 12000, 700, 0, 64, 4097], np.int32)   # long ones are split across workers
    pool, bt, q = mla_case(lens, seed=8)
    qd, pd, btd, ld = dev(q), dev(pool), dev(bt), dev(lens)
    shape = ct.MlaShape(MLA_H, MLA_E, MLA_DV, PAGE, bt.shape[1], ct.CT_KV_BF16, MLA_SCALE, pool.shape[0])

    plan = ct.MlaPlan(lens, pool.shape[0], max_pages_per_seq=bt.shape[1])
    ref_out = empty((len(lens), MLA_H, MLA_DV), np.uint16)
    ref_lse = empty((len(lens), MLA_H), np.float32)
    plan.decode(qd.data_ptr(), pd.data_ptr(), None, btd.data_ptr(), ld.data_ptr(), ref_out.data_ptr(),
                ref_lse.data_ptr(), stream())
    want = oracle.bf16_to_f32(host(ref_out, np.uint16)).reshape(len(lens), MLA_H, MLA_DV)
    want_lse = host(ref_lse, np.float32)
    oracle_want = oracle.mla_decode_paged(pool, bt, lens, q, MLA_H, MLA_E, MLA_DV, PAGE, MLA_SCALE)

    out = empty((len(lens), MLA_H, MLA_DV), np.uint16)
    lse = empty((len(lens), MLA_H), np.float32)
    free_after = []
    for call in range(2):
        out.fill_(0x7FFF)                         # poison: every value must be rewritten
        lse.fill_(0)
        torch.cuda.synchronize()
        ct.check(L.ct_attn_mla_decode_paged_noalloc(C.byref(shape), lens.ctypes.data, len(lens), qd.data_ptr(),
                                                    pd.data_ptr(), None, btd.data_ptr(), ld.data_ptr(),
                                                    out.data_ptr(), lse.data_ptr(), stream()),
                 "ct_attn_mla_decode_paged_noalloc")
        got = oracle.bf16_to_f32(host(out, np.uint16)).reshape(len(lens), MLA_H, MLA_DV)
        ok, mx, excess = close(got, want)
        assert ok, (call, mx, excess)
        if call == 0:                             # and against the oracle directly
            ok, mx, excess = close(got, oracle_want)
            assert ok, ("oracle", mx, excess)
        assert np.all(got[lens == 0] == 0)
        got_lse = host(lse, np.float32)
        fin = np.isfinite(want_lse)
        assert np.array_equal(fin, np.isfinite(got_lse))
        # split points differ (fewer workers), and the normaliser sums the
        # bf16-rounded probabilities of each chunk: agreement to a few 1e-4
        np.testing.assert_allclose(got_lse[fin], want_lse[fin], rtol=0, atol=5e-3)
        free_after.append(free_bytes())
    assert free_after[0] == free_after[1]         # the second call took no device memory


def test_noalloc_rejects_batches_beyond_its_limits():
    L = ct.lib()
    n = 4097                                      # one more than CT_MLA_NOALLOC_MAX_SEQS
    lens = np.full(n, 10, np.int32)
    shape = ct.MlaShape(MLA_H, MLA_E, MLA_DV, PAGE, 1, ct.CT_KV_BF16, MLA_SCALE, 1)
    buf = torch.empty(16, dtype=torch.int32, device="cuda")
    rc = L.ct_attn_mla_decode_paged_noalloc(C.byref(shape), lens.ctypes.data, n, buf.data_ptr(), buf.data_ptr(),
                                            None, buf.data_ptr(), buf.data_ptr(), buf.data_ptr(), None, stream())
    assert rc == ct.CT_ERR_ARG
    assert b"CT_MLA_NOALLOC_MAX_SEQS" in L.ct_hal_cuda_last_error()
    # heads x value dims too large for the split partials to fit the array
    big = ct.MlaShape(4096, 576, 512, PAGE, 4096, ct.CT_KV_BF16, MLA_SCALE, 1 << 20)
    lens2 = np.full(64, 64 * 4000, np.int32)
    rc = L.ct_attn_mla_decode_paged_noalloc(C.byref(big), lens2.ctypes.data, 64, buf.data_ptr(), buf.data_ptr(),
                                            None, buf.data_ptr(), buf.data_ptr(), buf.data_ptr(), None, stream())
    assert rc == ct.CT_ERR_ARG
    assert b"CT_MLA_NOALLOC_SCRATCH_BYTES" in L.ct_hal_cuda_last_error()
