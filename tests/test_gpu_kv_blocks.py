"""GPU: block-quantised page pools (Q8_0 / Q4_0 / Q2_0 / Q1_0, the cold-tier
codecs of src/quant/quant.c:77-249) in the paged cache.  Every stored entry
must equal, byte for byte, what the reference's own ct_quant_q*_0 writes for
the token's values (oracle/_ref, the reference's quant.c compiled unmodified),
and every gather must equal its ct_quant_deq*_0 output (fp32), or that output
rounded to bf16."""
import numpy as np
import pytest

import cautreo_b200 as ct
import oracle
from gpu_util import dev, empty, host, stream

pytestmark = pytest.mark.gpu
BLOCKS = [ct.CT_KV_Q8_0, ct.CT_KV_Q4_0, ct.CT_KV_Q2_0, ct.CT_KV_Q1_0]
NAME = {ct.CT_KV_Q8_0: "8", ct.CT_KV_Q4_0: "4", ct.CT_KV_Q2_0: "2", ct.CT_KV_Q1_0: "1"}


def ref_encode(dtype, xf):
    """Reference blocks of each row of xf ([n][dim] fp32) -> [n][entry bytes]."""
    R = oracle.ref()
    n, dim = xf.shape
    eb = ct.entry_bytes(dtype, dim)
    out = np.zeros((n, eb), np.uint8)
    fn = getattr(R, f"ct_quant_q{NAME[dtype]}_0")
    for i in range(n):
        row = np.ascontiguousarray(xf[i], np.float32)
        fn(row.ctypes.data, out[i].ctypes.data, dim)
    return out


def ref_decode(dtype, blocks, dim):
    R = oracle.ref()
    n = blocks.shape[0]
    out = np.zeros((n, dim), np.float32)
    fn = getattr(R, f"ct_quant_deq{NAME[dtype]}_0")
    for i in range(n):
        b = np.ascontiguousarray(blocks[i])
        fn(b.ctypes.data, out[i].ctypes.data, dim)
    return out


def entries(n_tok, dim, seed, src):
    # N(0,1) with 1 % of values x20, plus a few all-zero and tiny-magnitude
    # tokens (the reference's fp16 scale maps amax/qmax < 2^-15 to Inf)
    x = oracle.normal_f32(oracle.key(seed, 40), 0, n_tok * dim, 100, 20.0).reshape(n_tok, dim)
    x[min(3, n_tok - 1)] = 0.0
    if n_tok > 7:
        x[7] *= 1e-6
    if src == "bf16":
        xb = oracle.f32_to_bf16(x)
        return dev(xb), oracle.bf16_to_f32(xb).reshape(n_tok, dim), ct.CT_KV_BF16
    return dev(x), x, ct.CT_KV_F32


def pool_bytes(h, n_pages, P, eb):
    L = ct.lib()
    buf = np.zeros(n_pages * P * eb, np.uint8)
    ct.check(L.ct_hal_cuda_memcpy(buf.ctypes.data, h.pool, buf.nbytes, 1, None))
    ct.check(L.ct_hal_cuda_device_sync())
    return buf.reshape(n_pages * P, eb)


def same_bf16(got, want_f32):
    """bf16 outputs equal the reference's fp32 rounded by the bf16 rule, except
    where the reference value is NaN: the rule (no NaN handling, the
    reference's own) turns the GPU's default NaN 0x7FFFFFFF and x86's
    0xFFC00000 into different bit patterns, so NaN positions are not compared."""
    want_f32 = np.asarray(want_f32, np.float32)
    want = oracle.f32_to_bf16(want_f32).reshape(want_f32.shape)
    ok = np.isnan(want_f32) | (np.asarray(got) == want)
    return bool(np.all(ok))


def same_f32(a, b):
    """Bit equality, with every NaN equal to every NaN (Inf scales decode to NaN/Inf)."""
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    both_nan = np.isnan(a) & np.isnan(b)
    return bool(np.all(both_nan | (a.view(np.uint32) == b.view(np.uint32))))


@pytest.mark.parametrize("pool_dtype", BLOCKS)
@pytest.mark.parametrize("src", ["bf16", "f32"])
def test_block_pool_append_and_gather_match_reference(pool_dtype, src):
    S, P, E, NP = 5, 64, 576, 40
    lens = [1, 63, 64, 65, 300]
    total = sum(lens)
    ent, xf, sdt = entries(total, E, 41, src)
    h = ct.PagedKV(S, 8, NP, P, E, 0, pool_dtype, 0, stream())
    h.set_free_order(oracle.permutation(oracle.key(41, 1), NP))
    h.append(list(range(S)), lens, ent.data_ptr(), sdt)
    eb = ct.entry_bytes(pool_dtype, E)
    want_blocks = ref_encode(pool_dtype, xf)
    want_f32 = ref_decode(pool_dtype, want_blocks, E)
    stored = pool_bytes(h, NP, P, eb)
    bt = h.block_table()
    L = ct.lib()
    off = 0
    for s, n in enumerate(lens):
        slots = [bt[s, t // P] * P + t % P for t in range(n)]
        assert np.array_equal(stored[slots], want_blocks[off:off + n]), (s, "stored blocks")
        o32 = empty((n, E), np.float32)
        ct.check(L.ct_kv_paged_gather(h.h, s, 0, n, o32.data_ptr(), ct.CT_KV_F32))
        assert same_f32(host(o32, np.float32), want_f32[off:off + n]), (s, "f32 gather")
        o16 = empty((n, E), np.uint16)
        ct.check(L.ct_kv_paged_gather(h.h, s, 0, n, o16.data_ptr(), ct.CT_KV_BF16))
        assert same_bf16(host(o16, np.uint16), want_f32[off:off + n]), (s, "bf16 gather")
        off += n
    # a sub-range crossing a page boundary, and one past the end
    o = empty((10, E), np.float32)
    ct.check(L.ct_kv_paged_gather(h.h, 4, 60, 10, o.data_ptr(), ct.CT_KV_F32))
    base = sum(lens[:4])
    assert same_f32(host(o, np.float32), want_f32[base + 60:base + 70])
    assert L.ct_kv_paged_gather(h.h, 4, 295, 10, o.data_ptr(), ct.CT_KV_F32) == ct.CT_ERR_ARG
    h.close()


@pytest.mark.parametrize("pool_dtype", [ct.CT_KV_Q4_0, ct.CT_KV_Q1_0])
def test_block_pool_gather_batch_and_odd_word_entries(pool_dtype):
    """gather_batch equals per-sequence gathers; entry_dim 32 x 3 gives
    entries of an odd number of 2-byte words (3 x 18 = 54 B, 3 x 6 = 18 B)
    on pages of 8 tokens."""
    for E, P in ((576, 64), (96, 8)):
        S, NP = 4, 64
        lens = [5, 17, 40, 1]
        ent, xf, sdt = entries(sum(lens), E, 42, "bf16")
        h = ct.PagedKV(S, 16, NP, P, E, 0, pool_dtype, 0, stream())
        h.set_free_order(oracle.permutation(oracle.key(42, 1), NP))
        h.append(list(range(S)), lens, ent.data_ptr(), sdt)
        want = ref_decode(pool_dtype, ref_encode(pool_dtype, xf), E)
        seqs, starts, counts = [3, 1, 2, 2], [0, 2, 7, 39], [1, 15, 30, 1]
        out = empty((sum(counts), E), np.float32)
        h.gather_batch(seqs, starts, counts, out.data_ptr(), ct.CT_KV_F32)
        got = host(out, np.float32)
        off = np.cumsum([0] + lens)
        rows = np.concatenate([np.arange(off[s] + a, off[s] + a + c) for s, a, c in zip(seqs, starts, counts)])
        assert same_f32(got, want[rows]), E
        h.close()


def edge_entries(n, E, seed):
    """N(0,1) tokens with NaN, +-Inf, subnormal, zero, -0 and near-FLT_MAX
    values planted in some of them."""
    x = oracle.normal_f32(oracle.key(seed, 40), 0, n * E, 100, 20.0).reshape(n, E)
    x[1] *= 1e-39                       # subnormal block maxima: 1 / d overflows to Inf
    x[2, 5] = np.nan
    x[2, 32 + 3] = np.inf
    x[2, 64 + 7] = -np.inf
    x[2, 96:128] = 3.0e38               # d = amax / qmax overflows the fp16 scale
    x[3] = 0.0
    x[4] = -0.0
    x[5, :16] = np.nan
    x[6, :32] = np.nan                  # an all-NaN block
    return x


@pytest.mark.parametrize("pool_dtype", BLOCKS)
@pytest.mark.parametrize("src", ["bf16", "f32"])
def test_block_write_slots_edge_values_and_layouts(pool_dtype, src):
    """ct_kv_paged_write_slots into a block pool: slots in reverse order with a
    stride, from a source that is not 16-byte aligned (per-token stores, 2-byte
    staging), then one contiguous run from an odd slot (16-byte stores from an
    offset that is not a multiple of 16).  The tokens hold NaN, +-Inf,
    subnormal, zero and -0 values: the reference's (int)floorf(...) of a NaN or
    out-of-range value is INT_MIN on x86-64, which its clamp turns into -qmax,
    and every stored byte must equal the reference's.  Then an append and the
    gathers of those tokens equal the reference's decode (NaN positions
    excepted, as in same_f32 / same_bf16)."""
    P, E, NP, n = 64, 576, 4, 40
    L = ct.lib()
    x = edge_entries(n, E, 45)
    if src == "bf16":
        raw = oracle.f32_to_bf16(x).reshape(n, E)
        xf, elt, sdt = oracle.bf16_to_f32(raw).reshape(n, E), 2, ct.CT_KV_BF16
    else:
        raw, xf, elt, sdt = x, x, 4, ct.CT_KV_F32
    eb = ct.entry_bytes(pool_dtype, E)
    want = ref_encode(pool_dtype, xf)
    pad = np.zeros(16 // elt, raw.dtype)
    shifted = dev(np.concatenate([pad[:1], raw.reshape(-1), pad]))
    aligned = dev(raw)
    h = ct.PagedKV(1, NP, NP, P, E, 0, pool_dtype, 0, stream())
    for dest, src_ptr in ((5 + 3 * np.arange(n)[::-1], shifted.data_ptr() + elt),
                          (131 + np.arange(n), aligned.data_ptr())):
        d = dev(np.ascontiguousarray(dest, np.int32))
        ct.check(L.ct_kv_paged_write_slots(h.pool, None, pool_dtype, src_ptr, sdt, d.data_ptr(), n, E, stream()))
        stored = pool_bytes(h, NP, P, eb)
        assert np.array_equal(stored[dest], want), (dest[0], "stored blocks")
    h.close()
    g = ct.PagedKV(1, NP, NP, P, E, 0, pool_dtype, 0, stream())
    g.append([0], [n], aligned.data_ptr(), sdt)
    want_f32 = ref_decode(pool_dtype, want, E)
    o32 = empty((n, E), np.float32)
    ct.check(L.ct_kv_paged_gather(g.h, 0, 0, n, o32.data_ptr(), ct.CT_KV_F32))
    assert same_f32(host(o32, np.float32), want_f32)
    o16 = empty((n, E), np.uint16)
    ct.check(L.ct_kv_paged_gather(g.h, 0, 0, n, o16.data_ptr(), ct.CT_KV_BF16))
    assert same_bf16(host(o16, np.uint16), want_f32)
    g.close()


def test_block_pool_checkpoint_fork_compaction(tmp_path):
    """Q2_0 pool: a checkpoint restores the bytes, a fork shares the full
    pages and copies the partial one, compaction keeps every gather."""
    S, P, E, NP = 4, 64, 576, 24
    lens = [150, 70, 0, 0]
    ent, xf, sdt = entries(sum(lens), E, 43, "bf16")
    h = ct.PagedKV(S, 6, NP, P, E, 0, ct.CT_KV_Q2_0, 0, stream())
    h.set_free_order(oracle.permutation(oracle.key(43, 1), NP))
    h.append([0, 1], lens[:2], ent.data_ptr(), sdt)
    L = ct.lib()

    def gather(handle, s, lo, n):
        o = empty((n, E), np.uint16)
        ct.check(L.ct_kv_paged_gather(handle.h, s, lo, n, o.data_ptr(), ct.CT_KV_BF16))
        return host(o, np.uint16)

    want = ref_decode(ct.CT_KV_Q2_0, ref_encode(ct.CT_KV_Q2_0, xf), E)[:150]
    assert same_bf16(gather(h, 0, 0, 150), want)
    h.fork(0, 2, 150)
    bt = h.block_table()
    assert bt[2, 0] == bt[0, 0] and bt[2, 1] == bt[0, 1] and bt[2, 2] != bt[0, 2]
    assert np.array_equal(gather(h, 2, 0, 150), gather(h, 0, 0, 150))
    h.free_seq(1)
    h.compact()
    assert same_bf16(gather(h, 0, 0, 150), want) and same_bf16(gather(h, 2, 0, 150), want)
    path = tmp_path / "q2.ckpt"
    h.save(path)
    g = ct.PagedKV.load(path, device=0, stream=stream())
    for s in (0, 2):
        assert np.array_equal(gather(g, s, 0, 150), gather(h, s, 0, 150))
    h.close()
    g.close()


def test_block_pool_decode_is_unsupported():
    """The decode kernels do not read block pools; the call says so."""
    S, P, E, NP = 1, 64, 576, 4
    ent, _, sdt = entries(64, E, 44, "bf16")
    h = ct.PagedKV(S, 2, NP, P, E, 0, ct.CT_KV_Q4_0, 0, stream())
    h.append([0], [64], ent.data_ptr(), sdt)
    plan = ct.MlaPlan(np.array([64], np.int32), NP, max_pages_per_seq=2, kv_dtype=ct.CT_KV_Q4_0)
    q = dev(oracle.normal_bf16(oracle.key(44, 2), 0, 128 * E))
    out = empty((1, 128, 512), np.uint16)
    rc = ct.lib().ct_attn_mla_decode_paged(plan.h, q.data_ptr(), h.pool, None, h.block_table_dev, h.seq_lens_dev,
                                           out.data_ptr(), None, stream())
    assert rc == ct.CT_ERR_UNSUPPORTED
    h.close()
