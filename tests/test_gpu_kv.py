"""GPU: the reference ct_kv_* interface on device memory, and the paged cache
(append with quantise-on-append, gather with dequantise-on-gather, window /
LRU eviction, compaction) -- bit-exact against the reference and oracle."""
import ctypes as C
import os
from pathlib import Path

import numpy as np
import pytest
import torch

import cautreo_b200 as ct
import oracle
from gpu_util import dev, empty, host, stream
from helpers import MLA_H

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"
O = oracle.port()


# ---- contiguous cache (kv_cache.h part 1) ---------------------------------------

def test_reference_kv_cache_test_scenario(tmp_path):
    """kv_cache_test.c:14-67 through the device-backed library."""
    g = np.load(GOLD / "kv_ref.npz")
    c = ct.KvCache(2, 4, 8, 16, 1.0)
    assert len(c) == 0
    k = np.arange(32, dtype=np.float32)
    v = (np.arange(32) * 2).astype(np.float32)
    assert c.append(0, 0, k, v) and c.append(1, 1, k, v)
    assert len(c) == 2
    k2, v2 = c.get(0, 0)
    assert k2[31] == 31.0 and v2[31] == 62.0
    assert c.get(1, 1) is not None
    assert c.get(0, 2) is None                       # pos >= len
    assert not c.append(2, 0, k, v) and not c.append(0, 16, k, v)
    L = ct.lib()
    st = L.ct_kv_stats(c.h)
    assert st.n_appends == 2 and st.n_reads == 0 and st.bytes_used == 2 * 2 * 32 * 4 * 2 and st.n_tokens == 2
    path = str(tmp_path / "kv.bin")
    assert L.ct_kv_save(c.h, path.encode())
    assert np.array_equal(np.fromfile(path, np.uint8), g["save_bytes"])     # same bytes as the reference
    c2 = ct.KvCache(2, 4, 8, 16, 1.0)
    assert L.ct_kv_load(c2.h, path.encode())
    assert len(c2) == 2 and c2.get(0, 0)[0][0] == 0.0 and c2.get(1, 1)[1][31] == 62.0
    c3 = ct.KvCache(2, 4, 8, 16, 1.0)
    for i in range(8):
        c3.append(0, i, k, v)
    assert len(c3) == 8 and L.ct_kv_compress(c3.h, 4.0) and len(c3) == 2
    assert not L.ct_kv_compress(c3.h, 1.0)
    L.ct_kv_reset(c3.h)
    assert len(c3) == 0 and L.ct_kv_capacity(c3.h) == 16


def test_compress_matches_reference_golden():
    g = np.load(GOLD / "kv_ref.npz")
    L, H, D, ctx = 2, 4, 8, 16
    for ci in range(5):
        n, ok, m = (int(v) for v in g[f"cmp{ci}"])
        ratio = float(g[f"cmp{ci}_ratio"][0])
        c = ct.KvCache(L, H, D, ctx, 1.0)
        kk = oracle.normal_f32(oracle.key(9, ci), 0, n * L * H * D).reshape(n, L, H * D)
        vv = oracle.normal_f32(oracle.key(9, ci), 1 << 20, n * L * H * D).reshape(n, L, H * D)
        for t in range(n):
            for l in range(L):
                c.append(l, t, kk[t, l], vv[t, l])
        assert bool(ct.lib().ct_kv_compress(c.h, ratio)) == bool(ok)
        assert len(c) == m
        for l in range(L):
            for t in range(m):
                kr, vr = c.get(l, t)
                assert np.array_equal(kr, g[f"cmp{ci}_k"][l, t]) and np.array_equal(vr, g[f"cmp{ci}_v"][l, t])
        c.close()


def test_load_short_file_keeps_tail(tmp_path):
    L = ct.lib()
    c = ct.KvCache(1, 1, 4, 4, 1.0)
    for t in range(4):
        c.append(0, t, np.full(4, t + 1, np.float32), np.full(4, -t - 1, np.float32))
    path = str(tmp_path / "short.bin")
    hdr = np.array([1, 1, 4, 4], np.uint32).tobytes() + np.float32(1).tobytes() + np.array([2, 0], np.uint32).tobytes()
    with open(path, "wb") as f:
        f.write(hdr + np.full(4, 9.0, np.float32).tobytes())            # only one K row
    assert L.ct_kv_load(c.h, path.encode())
    assert len(c) == 2
    assert c.get(0, 0)[0].tolist() == [9.0] * 4 and c.get(0, 1)[0].tolist() == [2.0] * 4


# ---- paged cache -------------------------------------------------------------------

def entries_for(n_tok, dim, seed, dtype):
    x = oracle.normal_f32(oracle.key(seed, 20), 0, n_tok * dim, 100, 20.0).reshape(n_tok, dim)
    if dtype == "bf16":
        xb = oracle.f32_to_bf16(x)
        return dev(xb), oracle.bf16_to_f32(xb).reshape(n_tok, dim), ct.CT_KV_BF16
    return dev(x), x, ct.CT_KV_F32


def expected_pool_token(xf, pool_dtype):
    """What one token's entry looks like stored, and read back as fp32."""
    n, dim = xf.shape
    if pool_dtype == ct.CT_KV_BF16:
        return oracle.bf16_to_f32(oracle.f32_to_bf16(xf)).reshape(n, dim)
    if pool_dtype == ct.CT_KV_F32:
        return xf
    codes = np.zeros(n * dim, np.uint8)
    sc = np.zeros(n, np.float32)
    back = np.zeros(n * dim, np.float32)
    xf = np.ascontiguousarray(xf, np.float32)
    if pool_dtype == ct.CT_KV_INT8:
        O.orc_kv_quant_int8(xf.ctypes.data, n, dim, codes.ctypes.data, sc.ctypes.data)
        O.orc_kv_dequant_int8(codes.ctypes.data, sc.ctypes.data, n, dim, back.ctypes.data)
    else:
        O.orc_kv_quant_e4m3(xf.ctypes.data, n, dim, codes.ctypes.data, sc.ctypes.data)
        O.orc_kv_dequant_e4m3(codes.ctypes.data, sc.ctypes.data, n, dim, back.ctypes.data)
    return back.reshape(n, dim)


@pytest.mark.parametrize("pool_dtype", [ct.CT_KV_BF16, ct.CT_KV_F32, ct.CT_KV_INT8, ct.CT_KV_E4M3])
@pytest.mark.parametrize("src", ["bf16", "f32"])
def test_paged_append_gather_bit_exact(pool_dtype, src):
    S, P, E = 5, 64, 576
    lens = [1, 63, 64, 65, 300]                      # page boundary -1 / 0 / +1
    total = sum(lens)
    ent, xf, sdt = entries_for(total, E, 11, src)
    h = ct.PagedKV(S, 8, 40, P, E, 0, pool_dtype, 0, stream())
    h.set_free_order(oracle.permutation(oracle.key(11, 1), 40))
    h.append(list(range(S)), lens, ent.data_ptr(), sdt)
    want_all = expected_pool_token(xf, pool_dtype)
    L = ct.lib()
    off = 0
    for s, n in enumerate(lens):
        for out_dt, npdt in ((ct.CT_KV_F32, np.float32), (ct.CT_KV_BF16, np.uint16)):
            out = empty((n, E), npdt)
            ct.check(L.ct_kv_paged_gather(h.h, s, 0, n, out.data_ptr(), out_dt))
            got = host(out, npdt)
            want = want_all[off:off + n]
            if out_dt == ct.CT_KV_BF16:
                want = oracle.f32_to_bf16(want).reshape(n, E)
                assert np.array_equal(got, want), (s, "bf16 out")
            else:
                assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (s, "f32 out")
        off += n
    # a sub-range crossing a page boundary
    out = empty((10, E), np.float32)
    ct.check(L.ct_kv_paged_gather(h.h, 4, 60, 10, out.data_ptr(), ct.CT_KV_F32))
    assert np.array_equal(host(out, np.float32), want_all[sum(lens[:4]) + 60:sum(lens[:4]) + 70])
    assert L.ct_kv_paged_gather(h.h, 4, 295, 10, out.data_ptr(), ct.CT_KV_F32) == ct.CT_ERR_ARG
    if pool_dtype in (ct.CT_KV_INT8, ct.CT_KV_E4M3):       # codes and scales themselves
        bt = h.block_table()
        nb = 40 * P * E
        buf = np.zeros(nb, np.uint8)
        ct.check(L.ct_hal_cuda_memcpy(buf.ctypes.data, h.pool, nb, 1, None))
        sc = np.zeros(40 * P, np.float32)
        ct.check(L.ct_hal_cuda_memcpy(sc.ctypes.data, h.scales, sc.nbytes, 1, None))
        ct.check(L.ct_hal_cuda_device_sync())
        wc = np.zeros(total * E, np.uint8)
        ws = np.zeros(total, np.float32)
        fn = O.orc_kv_quant_int8 if pool_dtype == ct.CT_KV_INT8 else O.orc_kv_quant_e4m3
        fn(np.ascontiguousarray(xf).ctypes.data, total, E, wc.ctypes.data, ws.ctypes.data)
        off = 0
        for s, n in enumerate(lens):
            for t in range(n):
                slot = bt[s, t // P] * P + t % P
                assert np.array_equal(buf[slot * E:(slot + 1) * E], wc[(off + t) * E:(off + t + 1) * E])
                assert sc[slot] == ws[off + t]
            off += n
    h.close()


@pytest.mark.parametrize("pool_dtype", [ct.CT_KV_BF16, ct.CT_KV_F32, ct.CT_KV_INT8, ct.CT_KV_E4M3])
def test_paged_gather_batch_matches_per_sequence_gathers(pool_dtype):
    """ct_kv_paged_gather_batch: the rows of every range, back to back, bit for
    bit what one ct_kv_paged_gather per range returns (empty and page-crossing
    ranges included); bad ranges fail before anything is written."""
    S, P, E = 6, 64, 576
    lens = [1, 63, 64, 65, 300, 130]
    ent, xf, sdt = entries_for(sum(lens), E, 12, "bf16")
    h = ct.PagedKV(S, 8, 48, P, E, 0, pool_dtype, 0, stream())
    h.set_free_order(oracle.permutation(oracle.key(12, 1), 48))
    h.append(list(range(S)), lens, ent.data_ptr(), sdt)
    L = ct.lib()
    seqs = np.array([4, 0, 3, 5, 1, 2, 4], np.uint32)
    starts = np.array([60, 0, 0, 64, 10, 0, 299], np.uint32)
    counts = np.array([10, 1, 65, 66, 0, 64, 1], np.uint32)
    n_rows = int(counts.sum())
    for out_dt, npdt in ((ct.CT_KV_F32, np.float32), (ct.CT_KV_BF16, np.uint16)):
        out = empty((n_rows, E), npdt)
        ct.check(L.ct_kv_paged_gather_batch(h.h, seqs.ctypes.data, starts.ctypes.data, counts.ctypes.data, len(seqs),
                                            out.data_ptr(), out_dt), "gather_batch")
        got = host(out, npdt)
        row = 0
        for s_, st, n in zip(seqs, starts, counts):
            if n:
                one = empty((int(n), E), npdt)
                ct.check(L.ct_kv_paged_gather(h.h, int(s_), int(st), int(n), one.data_ptr(), out_dt))
                assert np.array_equal(got[row:row + n].view(np.uint8), host(one, npdt).view(np.uint8)), (s_, st, n)
            row += int(n)
    bad = np.array([5], np.uint32)
    assert L.ct_kv_paged_gather_batch(h.h, bad.ctypes.data, np.array([100], np.uint32).ctypes.data,
                                      np.array([40], np.uint32).ctypes.data, 1, out.data_ptr(),
                                      ct.CT_KV_F32) == ct.CT_ERR_ARG          # past the sequence's length
    h.close()


def test_paged_gather_unmapped_is_an_error():
    h = ct.PagedKV(1, 8, 4, 4, 16, 4, ct.CT_KV_BF16, 0, stream())
    ent = dev(oracle.f32_to_bf16(oracle.normal_f32(oracle.key(1, 1), 0, 12 * 16)))
    h.append([0], [12], ent.data_ptr(), ct.CT_KV_BF16)            # window 4 frees pages 0 and 1
    assert h.block_table()[0, :3].tolist() == [-1, -1, 0]      # page 0 freed at len 8, reused at token 8
    out = empty((4, 16), np.float32)
    assert ct.lib().ct_kv_paged_gather(h.h, 0, 0, 4, out.data_ptr(), ct.CT_KV_F32) == ct.CT_ERR_UNMAPPED
    ct.check(ct.lib().ct_kv_paged_gather(h.h, 0, 8, 4, out.data_ptr(), ct.CT_KV_F32))
    h.close()


def pool_tokens(h, n_pages, P, E):
    """Pool contents as bf16 bits [n_pages][P][E]."""
    buf = np.zeros(n_pages * P * E, np.uint16)
    L = ct.lib()
    ct.check(L.ct_hal_cuda_memcpy(buf.ctypes.data, h.pool, buf.nbytes, 1, None))
    ct.check(L.ct_hal_cuda_device_sync())
    return buf.reshape(n_pages, P, E)


@pytest.mark.parametrize("S,P,NP,W,lo,hi,splits", [(12, 4, 22, 12, 8, 128, None), (40, 8, 60, 0, 1, 300, [5, 64]),
                                                    (33, 4, 50, 20, 1, 200, [1, 2, 50])])
def test_paged_eviction_contents_and_compaction(S, P, NP, W, lo, hi, splits):
    """Window + LRU replay with token data: block tables, eviction log and the
    bytes of every live page equal the oracle's; compaction moves them to the
    oracle's (seq, lpage) order."""
    E = 32
    lens = oracle.lengths_loguniform(oracle.key(3, S), S, lo, hi)
    MP = (hi + P - 1) // P + 1
    rc, bt, owner, ev, last, nfree = oracle.alloc_replay(lens, S, P, NP, MP, W)
    assert rc == 0
    # entry values: token t of sequence s is stream element (s << 24 | t) * E + e
    k_ = oracle.key(3, 99)
    vals = {s: oracle.normal_bf16(k_, (s << 24) * E, int(lens[s]) * E).reshape(int(lens[s]), E) for s in range(S)}
    h = ct.PagedKV(S, MP, NP, P, E, W, ct.CT_KV_BF16, 0, stream())
    edges = [0] + list(splits or []) + [int(lens.max())]
    for a, b in zip(edges[:-1], edges[1:]):
        ids = [s for s in range(S) if min(int(lens[s]), b) - a > 0]
        cnt = [min(int(lens[s]), b) - a for s in ids]
        ent = np.concatenate([vals[s][a:a + c] for s, c in zip(ids, cnt)])
        ent_d = dev(ent)
        h.append(ids, cnt, ent_d.data_ptr(), ct.CT_KV_BF16)
    assert np.array_equal(h.block_table(), bt) and h.evict_log() == ev
    pool = pool_tokens(h, NP, P, E)
    for s in range(S):
        for lp in np.nonzero(bt[s] >= 0)[0]:
            ph = bt[s, lp]
            for j in range(P):
                o = int(owner[ph, j])
                if lp * P + j < int(lens[s]):              # a slot of this sequence's history
                    assert o == (s << 32 | (lp * P + j))
                if o == (1 << 64) - 1:
                    continue
                # slots past the sequence's end keep the previous owner's token
                os_, ot = o >> 32, o & 0xFFFFFFFF
                assert np.array_equal(pool[ph, j], vals[os_][ot])
    cbt, cmap = oracle.compact_plan(bt)
    ct.check(ct.lib().ct_kv_paged_compact(h.h))
    assert np.array_equal(h.block_table(), cbt)
    pool2 = pool_tokens(h, NP, P, E)
    assert np.array_equal(pool2[:len(cmap)], pool[cmap])
    st = h.stats()
    assert st.n_compactions == 1 and st.n_pages_free == NP - len(cmap)
    h.close()


def test_eviction_compaction_full_size_contents():
    """The eviction + compaction workload at full size (256 sequences,
    lengths log-uniform 512..32768, 64-token bf16 MLA pages, pool = 60 % of
    demand, window 4096): tables, log and page bytes against the oracle's
    replay, with token contents checked on the device."""
    S, P, W, E = 256, 64, 4096, 576
    lens = oracle.lengths_loguniform(oracle.key(3, 0), S, 512, 32768)
    demand = int(sum((int(n) + P - 1) // P for n in lens))
    NP, MP = int(0.6 * demand), 32768 // P + 1
    rc, bt, owner, ev, last, nfree = oracle.alloc_replay(lens, S, P, NP, MP, W)
    assert rc == 0
    total = int(lens.sum())
    ent = torch.empty(total * E, dtype=torch.int16, device="cuda")
    L = ct.lib()
    ct.check(L.ct_synth_fill(ent.data_ptr(), 0, ct.synth_key(3, 30), 0, total * E, 0, 1.0, stream()))
    h = ct.PagedKV(S, MP, NP, P, E, W, ct.CT_KV_BF16, 0, stream())
    h.append(list(range(S)), lens.tolist(), ent.data_ptr(), ct.CT_KV_BF16)
    assert np.array_equal(h.block_table(), bt) and h.evict_log() == ev
    # every live slot holds the entry of its owner token: gather the expected
    # rows on the device through the oracle's slot owners
    off = np.concatenate([[0], np.cumsum(lens.astype(np.int64))[:-1]])
    live_pages = np.unique(bt[bt >= 0])
    own = owner[live_pages].reshape(-1)
    ok = own != np.uint64((1 << 64) - 1)
    src_rows = (off[(own[ok] >> np.uint64(32)).astype(np.int64)] + (own[ok] & np.uint64(0xFFFFFFFF)).astype(np.int64))
    slots = (live_pages[:, None] * P + np.arange(P)[None, :]).reshape(-1)[ok]
    pool = torch.empty(NP * P * E, dtype=torch.int16, device="cuda")
    ct.check(L.ct_hal_cuda_memcpy(pool.data_ptr(), h.pool, NP * P * E * 2, 2, stream()))
    torch.cuda.synchronize()
    entv, poolv = ent.view(total, E), pool.view(NP * P, E)
    idx_src = torch.from_numpy(src_rows).cuda()
    idx_dst = torch.from_numpy(slots.astype(np.int64)).cuda()
    assert torch.equal(poolv[idx_dst], entv[idx_src])
    cbt, cmap = oracle.compact_plan(bt)
    ct.check(L.ct_kv_paged_compact(h.h))
    assert np.array_equal(h.block_table(), cbt)
    pool2 = torch.empty_like(pool)
    ct.check(L.ct_hal_cuda_memcpy(pool2.data_ptr(), h.pool, NP * P * E * 2, 2, stream()))
    torch.cuda.synchronize()
    pg = pool.view(NP, P * E)
    assert torch.equal(pool2.view(NP, P * E)[:len(cmap)], pg[torch.from_numpy(cmap.astype(np.int64)).cuda()])
    h.close()


@pytest.mark.parametrize("pool_dtype", [ct.CT_KV_BF16, ct.CT_KV_INT8, ct.CT_KV_E4M3])
def test_paged_checkpoint_restores_pages(pool_dtype, tmp_path):
    """ct_kv_paged_save / ct_kv_paged_load with page bytes: every live page
    (codes and scales for quantised pools) comes back at the same physical id,
    gathers are bit-identical, and appends after the load land exactly where
    they land on the original handle."""
    S, P, E, NP = 5, 64, 576, 24
    lens = [1, 63, 64, 65, 300]
    ent, xf, sdt = entries_for(sum(lens), E, 21, "bf16")
    h = ct.PagedKV(S, 8, NP, P, E, 128, pool_dtype, 0, stream())      # window 128 frees early pages
    h.set_free_order(oracle.permutation(oracle.key(21, 1), NP))
    h.append(list(range(S)), lens, ent.data_ptr(), sdt)
    path = tmp_path / "kv.ckpt"
    h.save(path)
    g = ct.PagedKV.load(path, device=0, stream=stream())
    assert np.array_equal(g.block_table(), h.block_table()) and g.evict_log() == h.evict_log()
    L = ct.lib()

    def gathers(handle):
        out = []
        for s, n in enumerate(handle.seq_lens()):
            lo = max(0, int(n) - 128)                              # what the window keeps
            o = empty((int(n) - lo, E), np.uint16)
            ct.check(L.ct_kv_paged_gather(handle.h, s, lo, int(n) - lo, o.data_ptr(), ct.CT_KV_BF16))
            out.append(host(o, np.uint16))
        return out

    for a, b in zip(gathers(h), gathers(g)):
        assert np.array_equal(a, b)
    more, _, _ = entries_for(3 * S, E, 22, "bf16")
    for handle in (h, g):
        handle.append(list(range(S)), [3] * S, more.data_ptr(), ct.CT_KV_BF16)
    assert np.array_equal(g.block_table(), h.block_table())
    for a, b in zip(gathers(h), gathers(g)):
        assert np.array_equal(a, b)
    h.close()
    g.close()


@pytest.mark.parametrize("pool_dtype", [ct.CT_KV_BF16, ct.CT_KV_INT8])
def test_fork_shares_pages_on_device(pool_dtype):
    """A forked sequence reads the same prefix (shared full pages, a copied
    partial page), appends stay private to each sequence, and MLA decode over
    the fork equals decode over the original."""
    S, P, E, NP = 3, 64, 576, 16
    h = ct.PagedKV(S, 6, NP, P, E, 0, pool_dtype, 0, stream())
    h.set_free_order(oracle.permutation(oracle.key(31, 1), NP))
    ent, _, sdt = entries_for(150, E, 31, "bf16")
    h.append([0], [150], ent.data_ptr(), sdt)
    h.fork(0, 1, 150)
    bt = h.block_table()
    assert bt[0, 0] == bt[1, 0] and bt[0, 1] == bt[1, 1] and bt[0, 2] != bt[1, 2]
    L = ct.lib()

    def gather(s, lo, n):
        o = empty((n, E), np.uint16)
        ct.check(L.ct_kv_paged_gather(h.h, s, lo, n, o.data_ptr(), ct.CT_KV_BF16))
        return host(o, np.uint16)

    assert np.array_equal(gather(0, 0, 150), gather(1, 0, 150))
    # identical queries: identical outputs
    q = oracle.normal_bf16(oracle.key(31, 2), 0, 2 * MLA_H * E).reshape(2, MLA_H, E)
    q[1] = q[0]
    qd, out = dev(q), empty((2, MLA_H, 512), np.uint16)
    plan = ct.MlaPlan(np.array([150, 150], np.int32), NP, max_pages_per_seq=6, kv_dtype=pool_dtype,
                      seq_rows=np.array([0, 1], np.uint32))
    plan.decode(qd.data_ptr(), h.pool, h.scales, h.block_table_dev, h.seq_lens_dev, out.data_ptr(), None, stream())
    o = host(out, np.uint16)
    assert np.array_equal(o[0], o[1])
    # private appends: each sequence's new tokens land in its own pages
    a, _, _ = entries_for(5, E, 32, "bf16")
    b, _, _ = entries_for(5, E, 33, "bf16")
    prefix0 = gather(0, 0, 150)
    h.append([0], [5], a.data_ptr(), ct.CT_KV_BF16)
    h.append([1], [5], b.data_ptr(), ct.CT_KV_BF16)
    assert np.array_equal(gather(0, 0, 150), prefix0) and np.array_equal(gather(1, 0, 150), prefix0)
    assert not np.array_equal(gather(0, 150, 5), gather(1, 150, 5))
    h.close()
