"""CPU: the product library loads, exports every declared entry point, and its
host logic (paged allocator bookkeeping, LPT sharding, HAL strategy, fp16
scalar rules, distributed context) matches the oracle / reference -- no GPU
compute is called here."""
import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

import cautreo_b200 as ct
import oracle

ROOT = Path(__file__).resolve().parent.parent
GOLD = ROOT / "tests" / "golden"


def declared_functions():
    names = set()
    for h in sorted((ROOT / "include").glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        text = re.sub(r"static inline[^{]*\{.*?\n\}", "", text, flags=re.S)
        for m in re.finditer(r"\b(ct_[a-z0-9_]+)\s*\(", text):
            names.add(m.group(1))
    return sorted(names)


def test_library_loads_and_exports_every_declared_symbol():
    L = ct.lib()
    names = declared_functions()
    assert len(names) > 90
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    # and every declared function has a ctypes signature in the Python layer
    assert not [n for n in names if n not in ct.SIGNATURES], [n for n in names if n not in ct.SIGNATURES]


def test_version_and_launch_counter():
    L = ct.lib()
    assert b"sm_100a" in L.ct_hal_version()
    assert L.ct_hal_cuda_launch_count() >= 0


def test_fp16_scalar_rules_match_reference_golden():
    g = np.load(GOLD / "quant_ref.npz")
    L = ct.lib()
    enc = np.array([L.ct_quant_f32_to_fp16(float(v)) for v in g["f32"]], np.uint16)
    assert np.array_equal(enc, g["f32_to_fp16"])
    dec = np.array([L.ct_quant_fp16_to_f32(h) for h in range(65536)], np.float32)
    assert np.array_equal(dec.view(np.uint32), g["fp16_to_f32"].view(np.uint32))


def test_bytes_per_float_quirk():
    # quant.h:57-66 integer division: Q8_0 -> 1 (34/32), Q4_0..Q1_0 -> 0; FP16 -> 2
    assert {t: b // 32 for t, b in ct.QUANT_BLOCK_BYTES.items()} == {1: 1, 2: 0, 3: 0, 4: 0}


def test_lpt_matches_oracle():
    lens = oracle.lengths_loguniform(oracle.key(4, 0), 1024, 512, 65536)
    for n_ranks in (1, 2, 3, 4, 8):
        assert np.array_equal(ct.lpt_shard(lens, n_ranks), oracle.lpt(lens, n_ranks))
    ties = np.array([5, 5, 5, 5, 9, 1], np.uint32)
    assert np.array_equal(ct.lpt_shard(ties, 2), oracle.lpt(ties, 2))


def test_rank_sequences():
    L = ct.lib()
    rank_of = np.array([1, 0, 1, 2, 0], np.int32)
    out = np.zeros(5, np.uint32)
    n = L.ct_dist_rank_sequences(rank_of.ctypes.data, 5, 0, out.ctypes.data)
    assert n == 2 and out[:2].tolist() == [1, 4]


def test_distributed_context_mirrors_reference():
    # distributed_test.c: defaults to one device, rank 0 leads, collectives succeed
    L = ct.lib()
    ctx = L.ct_dist_init(None)
    assert L.ct_dist_n_devices(ctx) == 1 and L.ct_dist_device_id(ctx) == 0 and L.ct_dist_is_leader(ctx)
    buf = np.ones(4, np.float32)
    assert L.ct_dist_allreduce(ctx, buf.ctypes.data, 4)
    assert not L.ct_dist_allreduce(ctx, None, 4)
    assert L.ct_dist_broadcast(ctx, buf.ctypes.data, 4, 0)
    L.ct_dist_destroy(ctx)


def test_hal_strategy_matches_reference_rule():
    """With the RAM budget pinned and no GPU, ct_hal_set_model follows the
    reference's strategy rule (hal.c:285-305): resident up to 80 % of the
    budget, otherwise stream when the SSD reads >= 500 MB/s."""
    L = ct.lib()
    sc = L.ct_hal_detect().contents
    assert sc.cpu_cores_logical >= 1 and sc.ram_total_bytes > 0
    budget = 10 << 30
    L.ct_hal_set_ram_budget(budget)
    assert L.ct_hal_get().contents.ram_model_budget == int(budget * 0.8)
    assert L.ct_hal_set_model(int(budget * 0.8), 1, False) == 0            # RESIDENT
    big = L.ct_hal_set_model(int(budget * 0.9), 1, True)
    gpu = L.ct_hal_get().contents
    if not gpu.gpu_present:
        assert big == 1                                                     # STREAM (ssd 3000 MB/s)
    if oracle.ref_available():
        R = C.CDLL(str(oracle.REF_LIB))
        R.ct_hal_set_ram_budget.argtypes = [C.c_uint64]
        R.ct_hal_set_model.argtypes = [C.c_uint64, C.c_uint64, C.c_bool]
        R.ct_hal_detect()
        R.ct_hal_set_ram_budget(budget)
        assert R.ct_hal_set_model(int(budget * 0.8), 1, False) == 0
        if not gpu.gpu_present:
            assert R.ct_hal_set_model(int(budget * 0.9), 1, True) == big
    L.ct_hal_set_ram_budget(0)


# ---- paged allocator bookkeeping (host-only handle) --------------------------

def host_paged(S, MP, NP, P, W):
    return ct.PagedKV(S, MP, NP, page_tokens=P, entry_dim=16, window_tokens=W, dtype=ct.CT_KV_BF16, device=-1)


def replay_product(lens, S, P, NP, MP, W, splits=None):
    h = host_paged(S, MP, NP, P, W)
    lens = np.asarray(lens, np.int64)
    edges = [0] + list(splits or []) + [int(lens.max())]
    for a, b in zip(edges[:-1], edges[1:]):
        ids = [s for s in range(S) if lens[s] > a]
        cnt = [min(int(lens[s]), b) - a for s in ids]
        ids = [s for s, c in zip(ids, cnt) if c > 0]
        cnt = [c for c in cnt if c > 0]
        if ids:
            h.append(ids, cnt)
    return h


@pytest.mark.parametrize("splits", [None, [1, 2, 3, 17, 40, 41]])
def test_product_allocator_matches_golden(splits):
    g = np.load(GOLD / "alloc_ref.npz")
    S, P, NP, MP, W = (int(v) for v in g["cfg"])
    h = replay_product(g["lens"], S, P, NP, MP, W, splits)
    assert np.array_equal(h.block_table(), g["bt"])
    ev = np.array(h.evict_log(), np.int64)
    assert np.array_equal(ev, g["events"])
    assert np.array_equal(h.last_access().astype(np.uint32), g["last"])
    st = h.stats()
    assert st.n_pages_free == int(g["n_free"])
    assert st.n_evict_window + st.n_evict_lru == len(ev)
    assert ct.lib().ct_kv_paged_compact(h.h) == 0
    assert np.array_equal(h.block_table(), g["compact_bt"])
    h.close()


@pytest.mark.parametrize("S,P,NP,W,lo,hi", [(40, 8, 60, 0, 1, 300), (64, 16, 90, 64, 16, 600),
                                            (33, 4, 50, 20, 1, 200)])
def test_product_allocator_matches_oracle(S, P, NP, W, lo, hi):
    lens = oracle.lengths_loguniform(oracle.key(3, S), S, lo, hi)
    MP = (hi + P - 1) // P + 1
    rc, bt, owner, ev, last, nfree = oracle.alloc_replay(lens, S, P, NP, MP, W)
    assert rc == 0
    h = replay_product(lens, S, P, NP, MP, W)
    assert np.array_equal(h.block_table(), bt)
    assert h.evict_log() == ev
    assert np.array_equal(h.seq_lens(), lens)
    h.close()


def test_product_allocator_eviction_compaction_full_size():
    """The eviction + compaction workload at full size: 256 sequences with
    log-uniform lengths 512..32768, 64-token pages, a pool of 60 % of the
    pages demanded, sliding window 4096 -- tables and eviction log identical."""
    S, P, W = 256, 64, 4096
    lens = oracle.lengths_loguniform(oracle.key(3, 0), S, 512, 32768)
    demand = int(sum((int(n) + P - 1) // P for n in lens))
    NP = int(0.6 * demand)
    MP = 32768 // P + 1
    rc, bt, owner, ev, last, nfree = oracle.alloc_replay(lens, S, P, NP, MP, W)
    assert rc == 0
    h = replay_product(lens, S, P, NP, MP, W)
    assert np.array_equal(h.block_table(), bt)
    assert h.evict_log() == ev
    cbt, cmap = oracle.compact_plan(bt)
    assert ct.lib().ct_kv_paged_compact(h.h) == 0
    assert np.array_equal(h.block_table(), cbt)
    h.close()


def test_product_allocator_full_pool_errors():
    h = host_paged(2, 4, 1, 4, 0)
    h.append([0], [2])                          # the only page, partly filled
    with pytest.raises(RuntimeError):
        h.append([1], [1])                      # only a partial tail page exists: nothing evictable
    h.close()
    h = host_paged(2, 4, 1, 4, 0)
    h.append([0], [4])                          # the only page, full
    h.append([1], [1])                          # -> LRU takes it
    assert h.evict_log() == [(4, 0, 0, 0, 2)]
    assert h.block_table()[0].tolist() == [-1] * 4 and h.block_table()[1, 0] == 0
    h.close()


def test_product_allocator_free_and_evict_api():
    h = host_paged(3, 8, 6, 4, 0)
    h.append([0, 1, 2], [8, 4, 6])              # 2 + 1 + 2 pages = 5 of 6
    L = ct.lib()
    assert L.ct_kv_paged_evict_lru(h.h, 2) == 2
    ev = h.evict_log()
    # all three appended in the same rounds; round of last access: seq0 -> 7, seq1 -> 3, seq2 -> 5
    assert [(e[1], e[2]) for e in ev] == [(1, 0), (2, 0)]
    assert L.ct_kv_paged_free_seq(h.h, 0) == 0
    assert h.seq_lens().tolist() == [0, 4, 6] and (h.block_table()[0] < 0).all()
    assert h.stats().n_pages_free == 6 - 1
    h.close()


# ---- paged checkpoint (tables only: host-only handle) ------------------------

def _state(h):
    st = h.stats()
    return (h.block_table().tolist(), h.seq_lens().tolist(), h.last_access().tolist(), h.evict_log(),
            (st.n_appends, st.n_evict_window, st.n_evict_lru, st.n_pages_live, st.n_pages_free, st.clock))


def test_paged_checkpoint_round_trip_and_resume(tmp_path):
    """Save mid-run under window and LRU pressure, load into a new handle:
    same tables, lengths, clocks, eviction log and statistics, and the same
    future -- further appends evict and place pages exactly as on the
    original handle."""
    S, P, NP, W = 33, 4, 50, 20
    lens = oracle.lengths_loguniform(oracle.key(3, S), S, 1, 200)
    MP = (200 + P - 1) // P + 1
    h = host_paged(S, MP, NP, P, W)
    h.set_free_order(oracle.permutation(oracle.key(9, 1), NP))
    half = [int(n) // 2 for n in lens]
    ids = [s for s in range(S) if half[s] > 0]
    h.append(ids, [half[s] for s in ids])
    path = tmp_path / "kv.ckpt"
    h.save(path)
    g = ct.PagedKV.load(path, device=-1)
    assert _state(g) == _state(h)
    rest = [int(n) - half[s] for s, n in enumerate(lens)]
    ids2 = [s for s in range(S) if rest[s] > 0]
    for handle in (h, g):
        handle.append(ids2, [rest[s] for s in ids2])
    assert _state(g) == _state(h)
    assert ct.lib().ct_kv_paged_compact(h.h) == 0 and ct.lib().ct_kv_paged_compact(g.h) == 0
    assert _state(g) == _state(h)
    h.close()
    g.close()


def test_paged_checkpoint_rejects_damage(tmp_path):
    h = host_paged(4, 8, 10, 4, 0)
    h.append([0, 1, 2], [5, 9, 1])
    path = tmp_path / "kv.ckpt"
    h.save(path)
    raw = bytearray(path.read_bytes())
    L = ct.lib()
    for pos in (0, 20, len(raw) // 2, len(raw) - 1):       # magic, config, tables, checksum
        bad = bytearray(raw)
        bad[pos] ^= 0x5A
        (tmp_path / "bad.ckpt").write_bytes(bytes(bad))
        assert not L.ct_kv_paged_load(str(tmp_path / "bad.ckpt").encode(), -1)
    (tmp_path / "short.ckpt").write_bytes(bytes(raw[:-9]))
    assert not L.ct_kv_paged_load(str(tmp_path / "short.ckpt").encode(), -1)
    assert not L.ct_kv_paged_load(str(tmp_path / "missing.ckpt").encode(), -1)
    assert L.ct_kv_paged_save(h.h, str(tmp_path / "no_such_dir" / "x").encode()) == ct.CT_ERR_IO
    h.close()


def _fnv1a64(data):
    h = 0xCBF29CE484222325
    for b in data:
        h = ((h ^ b) * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


def test_paged_checkpoint_rejects_inconsistent_free_set(tmp_path):
    """A checkpoint whose checksum is right but whose free set names a page
    the block table maps (or names a page twice) is rejected: loading it
    would let the allocator hand a live page to another sequence."""
    S, MP, NP, P = 4, 8, 10, 4
    h = host_paged(S, MP, NP, P, 0)
    h.append([0, 1, 2], [5, 9, 1])                # 2 + 3 + 1 = 6 live pages, 4 free
    path = tmp_path / "kv.ckpt"
    h.save(path)
    raw = bytes(path.read_bytes())
    # header 104 B, then len / lo / hi (4 B each per seq), last_access (8 B),
    # the block table, the free order (4 B per page), then free_n and the ids
    off_free = 104 + S * (4 + 4 + 4 + 8) + S * MP * 4 + NP * 4
    free_n = int(np.frombuffer(raw[off_free:off_free + 4], np.uint32)[0])
    assert free_n == NP - 6
    ids = np.frombuffer(raw[off_free + 4:off_free + 4 + 4 * free_n], np.int32).copy()
    live = int(h.block_table()[0, 0])
    L = ct.lib()
    for bad_ids in (np.array([live] + ids[1:].tolist(), np.int32),        # a mapped page marked free
                    np.array([ids[1]] + ids[1:].tolist(), np.int32)):     # a free page listed twice
        body = bytearray(raw[:-8])
        body[off_free + 4:off_free + 4 + 4 * free_n] = bad_ids.tobytes()
        (tmp_path / "bad.ckpt").write_bytes(bytes(body) + _fnv1a64(body).to_bytes(8, "little"))
        assert not L.ct_kv_paged_load(str(tmp_path / "bad.ckpt").encode(), -1)
    # the untouched bytes re-signed the same way still load (the layout above is right)
    body = bytearray(raw[:-8])
    (tmp_path / "ok.ckpt").write_bytes(bytes(body) + _fnv1a64(body).to_bytes(8, "little"))
    g = ct.PagedKV.load(tmp_path / "ok.ckpt", device=-1)
    assert _state(g) == _state(h)
    g.close()
    h.close()


# ---- prefix sharing (tables only) ---------------------------------------------

def test_fork_shares_full_pages_copies_the_partial_one():
    h = host_paged(4, 8, 20, 4, 0)
    h.append([0], [10])                                   # pages 0, 1 full, page 2 holds 2 tokens
    bt = h.block_table()
    p0, p1, p2 = bt[0, :3]
    h.fork(0, 1, 10)
    bt = h.block_table()
    assert bt[1, 0] == p0 and bt[1, 1] == p1 and bt[1, 2] not in (p0, p1, p2)
    assert [h.page_refs(p) for p in (p0, p1, p2, bt[1, 2])] == [2, 2, 1, 1]
    h.fork(0, 2, 8)                                       # page-aligned prefix: nothing copied
    bt = h.block_table()
    assert bt[2, :3].tolist() == [p0, p1, -1] and h.page_refs(p0) == 3
    assert h.seq_lens()[:3].tolist() == [10, 10, 8]
    live = h.stats().n_pages_live
    h.append([2], [1])                                    # opens its own page 2
    assert h.block_table()[2, 2] not in (p0, p1, p2) and h.stats().n_pages_live == live + 1
    ct.check(ct.lib().ct_kv_paged_free_seq(h.h, 0))
    assert h.page_refs(p0) == 2 and h.page_refs(p2) == 0  # shared pages stay; seq 0's own page is free
    ct.check(ct.lib().ct_kv_paged_free_seq(h.h, 1))
    ct.check(ct.lib().ct_kv_paged_free_seq(h.h, 2))
    assert h.stats().n_pages_live == 0 and h.stats().n_pages_free == 20
    h.close()


def test_fork_errors():
    h = host_paged(4, 8, 20, 4, 8)                        # window 8
    h.append([0, 1], [6, 30])
    L = ct.lib()
    assert L.ct_kv_paged_fork(h.h, 0, 0, 2) == ct.CT_ERR_ARG         # src == dst
    assert L.ct_kv_paged_fork(h.h, 0, 1, 2) == ct.CT_ERR_ARG         # dst not empty
    assert L.ct_kv_paged_fork(h.h, 0, 2, 7) == ct.CT_ERR_ARG         # longer than src
    assert L.ct_kv_paged_fork(h.h, 1, 2, 30) == ct.CT_ERR_UNMAPPED   # window dropped src's prefix
    h.close()


def test_fork_pages_are_not_lru_victims():
    """Under pool pressure LRU takes only pages one sequence maps."""
    h = host_paged(3, 8, 6, 4, 0)
    h.append([0], [12])                                   # 3 full pages, oldest access
    h.fork(0, 1, 8)                                       # shares pages 0 and 1 of seq 0
    h.append([2], [12])                                   # 3 more pages: the pool is full
    bt0 = h.block_table()[0].copy()
    h.append([2], [1])                                    # needs a page: seq 0's lowest is shared...
    ev = h.evict_log()
    assert len(ev) == 1 and ev[0][1] == 2 and ev[0][4] == 2   # ...so seq 2's own oldest page goes
    assert np.array_equal(h.block_table()[0], bt0)
    h.close()


def test_fork_window_releases_references():
    h = host_paged(2, 16, 30, 4, 8)                       # window 8
    h.append([0], [8])
    h.fork(0, 1, 8)
    p0, p1 = h.block_table()[0, :2]
    h.append([1], [8])                                    # seq 1's window moves past the shared pages
    assert h.block_table()[1, :2].tolist() == [-1, -1]
    assert h.page_refs(p0) == 1 and h.page_refs(p1) == 1  # still seq 0's
    h.close()


def test_fork_survives_compaction_and_checkpoint(tmp_path):
    h = host_paged(3, 8, 24, 4, 0)
    h.set_free_order(oracle.permutation(oracle.key(5, 1), 24))
    h.append([0, 2], [9, 5])
    h.fork(0, 1, 9)
    h.append([1], [3])
    assert ct.lib().ct_kv_paged_compact(h.h) == 0
    bt = h.block_table()
    assert bt[0, 0] == bt[1, 0] and bt[0, 1] == bt[1, 1] and bt[0, 2] != bt[1, 2]
    refs = [h.page_refs(p) for p in range(24)]
    assert sorted(set(bt[bt >= 0].tolist())) == list(range(sum(r > 0 for r in refs)))   # dense after compaction
    path = tmp_path / "kv.ckpt"
    h.save(path)
    g = ct.PagedKV.load(path, device=-1)
    assert [g.page_refs(p) for p in range(24)] == refs
    assert np.array_equal(g.block_table(), bt)
    for handle in (h, g):
        ct.check(ct.lib().ct_kv_paged_free_seq(handle.h, 0))
        handle.append([2], [6])
    assert np.array_equal(g.block_table(), h.block_table())
    h.close()
    g.close()


def test_block_pool_creation_rules():
    """Block-quantised pools (quant.h codecs): entry_dim a multiple of 32 and
    at most 4096, pages a multiple of 16 bytes; the entry sizes follow the
    block structs (34 / 18 / 10 / 6 B per 32 values)."""
    assert [ct.entry_bytes(d, 576) for d in (ct.CT_KV_Q8_0, ct.CT_KV_Q4_0, ct.CT_KV_Q2_0, ct.CT_KV_Q1_0)] == \
        [612, 324, 180, 108]
    ok = ct.PagedKV(2, 4, 8, page_tokens=64, entry_dim=576, dtype=ct.CT_KV_Q4_0, device=-1)
    ok.close()
    L = ct.lib()
    for dim, P, dt in ((48, 64, ct.CT_KV_Q4_0),      # not a multiple of 32
                       (8192, 64, ct.CT_KV_Q8_0),    # more than 4096 values
                       (32, 4, ct.CT_KV_Q4_0),       # 4 x 18 B pages are not 16-byte multiples
                       (576, 64, 8)):                # no such dtype
        cfg = ct.PagedConfig(2, 4, 8, P, dim, 0, dt, -1)
        assert not L.ct_kv_paged_create(C.byref(cfg)), (dim, P, dt)


def _fnv64(b):
    h = 0xCBF29CE484222325
    for x in b:
        h ^= x
        h = (h * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


def test_token_ids_prefix_match_fork_and_checkpoint(tmp_path):
    """KV reuse across turns: recorded token ids, longest cached prefix,
    fork of that prefix (ids come along), free_seq drops them, and the
    checkpoint carries them (version 2; version 1 files still load)."""
    S, MP, NP, P = 4, 8, 32, 16
    h = host_paged(S, MP, NP, P, 0)
    h.append([0, 1], [40, 20])
    ids0 = np.arange(100, 140, dtype=np.int32)
    ids1 = np.concatenate([np.arange(100, 110), np.arange(900, 910)]).astype(np.int32)
    h.set_tokens(0, 0, ids0[:30])
    h.set_tokens(0, 30, ids0[30:])
    h.set_tokens(1, 0, ids1)
    assert np.array_equal(h.tokens(0), ids0) and np.array_equal(h.tokens(1), ids1)
    L = ct.lib()
    # gaps and positions past the cached length are refused
    assert L.ct_kv_paged_set_tokens(h.h, 1, 25, ids1.ctypes.data, 1) == ct.CT_ERR_ARG
    assert L.ct_kv_paged_set_tokens(h.h, 1, 15, ids1.ctypes.data, 10) == ct.CT_ERR_ARG
    prompt = np.concatenate([np.arange(100, 125), [7, 7]]).astype(np.int32)
    assert h.match_prefix(prompt) == (0, 25)
    assert h.match_prefix(np.array([900], np.int32))[1] == 0
    assert h.match_prefix(np.concatenate([np.arange(100, 110), [900]]).astype(np.int32)) == (1, 11)
    s, n = h.match_prefix(prompt)
    h.fork(s, 2, n)
    assert np.array_equal(h.tokens(2), ids0[:25]) and h.seq_lens()[2] == 25
    h.free_seq(1)
    assert len(h.tokens(1)) == 0
    path = tmp_path / "t.ckpt"
    h.save(path)
    g = ct.PagedKV.load(path, device=-1)
    for s in range(S):
        assert np.array_equal(g.tokens(s), h.tokens(s))
    assert g.match_prefix(prompt) == (0, 25)
    g.close()
    # the same state written as version 1 (no token section): loads, without ids
    raw = path.read_bytes()
    body = bytearray(raw[:-8])
    tok_bytes = sum(4 + 4 * len(h.tokens(s)) for s in range(S))
    body = body[:-tok_bytes]
    body[8:12] = (1).to_bytes(4, "little")
    v1 = tmp_path / "v1.ckpt"
    v1.write_bytes(bytes(body) + _fnv64(bytes(body)).to_bytes(8, "little"))
    g1 = ct.PagedKV.load(v1, device=-1)
    assert np.array_equal(g1.block_table(), h.block_table()) and len(g1.tokens(0)) == 0
    g1.close()
    h.close()
