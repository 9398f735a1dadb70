"""GPU: paged absorbed-MLA decode (ct_attn_mla_decode_paged) against the
oracle, whose MLA numerics are pinned bit-exactly to the reference's own
ct_attn_forward (tests/test_oracle.py).  Tolerance (bf16 inputs, fp32
accumulation), elementwise: |got - ref| <= 2e-2 + 1e-2 |ref| (helpers.close)."""
from pathlib import Path

import numpy as np
import pytest
import torch

import cautreo_b200 as ct
import oracle
from gpu_util import dev, empty, host, stream
from helpers import ATOL, MLA_DV, MLA_E, MLA_H, MLA_SCALE, PAGE, RTOL, close, mla_case

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"
O = oracle.port()


@pytest.fixture(autouse=True)
def no_expired_waits():
    """Every test leaves the tensor-core kernel's error word at 0."""
    ct.lib().ct_mla_tc_error(1)
    yield
    assert ct.lib().ct_mla_tc_error(1) == 0


def run_decode(pool, bt, lens, q, H=MLA_H, E=MLA_E, Dv=MLA_DV, P=PAGE, dtype=ct.CT_KV_BF16, scales=None,
               want_lse=False):
    lens = np.asarray(lens, np.int32)
    plan = ct.MlaPlan(lens, pool.shape[0], n_heads=H, entry_dim=E, v_dim=Dv, page_tokens=P, max_pages_per_seq=bt.shape[1],
                      kv_dtype=dtype, scale=MLA_SCALE)
    out = empty((len(lens), H, Dv), np.uint16)
    lse = empty((len(lens), H), np.float32) if want_lse else None
    pd, qd, btd, ld = dev(pool), dev(q), dev(bt), dev(lens)       # alive until the results are read
    sd = dev(scales) if scales is not None else None
    plan.decode(qd.data_ptr(), pd.data_ptr(), sd.data_ptr() if sd is not None else None,
                btd.data_ptr(), ld.data_ptr(), out.data_ptr(), lse.data_ptr() if lse is not None else None,
                stream())
    got = oracle.bf16_to_f32(host(out, np.uint16)).reshape(len(lens), H, Dv)
    return (got, host(lse, np.float32), plan) if want_lse else (got, plan)


def oracle_decode_f32(poolf, bt, lens, qf, H, E, Dv, P):
    out = np.zeros((len(lens), H, Dv), np.float32)
    for s, n in enumerate(lens):
        rows = [poolf[bt[s, t // P], t % P] for t in range(int(n)) if bt[s, t // P] >= 0]
        if not rows:
            continue
        kv = np.ascontiguousarray(np.stack(rows), np.float32)
        qs = np.ascontiguousarray(qf[s], np.float32)
        assert O.orc_mla_decode(qs.ctypes.data, kv.ctypes.data, len(rows), H, E, Dv, MLA_SCALE,
                                out[s].ctypes.data) == 0
    return out


@pytest.mark.parametrize("lens", [[1, 63, 64, 65, 130, 0, 200], [4096], [1], [0, 0], [777, 1500, 64 * 17 + 3]])
def test_mla_small_cases(lens):
    pool, bt, q = mla_case(lens, seed=1)
    before = ct.launch_count()
    got, plan = run_decode(pool, bt, lens, q)
    assert ct.launch_count() > before
    assert plan.tensor_cores and plan.workers >= 64        # the tcgen05 kernel ran
    want = oracle.mla_decode_paged(pool, bt, lens, q, MLA_H, MLA_E, MLA_DV, PAGE, MLA_SCALE)
    ok, mx, rel = close(got, want)
    assert ok, (mx, rel)
    for s, n in enumerate(lens):
        if n == 0:
            assert np.all(got[s] == 0)


def test_mla_matches_reference_golden_16_heads():
    """16-head case of mla_ref.npz, computed by the reference's own
    ct_attn_forward over gathered pages (runs the CUDA-core kernel)."""
    g = np.load(GOLD / "mla_ref.npz")
    lens = g["lens"]
    H = int(g["heads"])
    pool, bt, q = mla_case(lens, seed=1, H=H)
    got, plan = run_decode(pool, bt, lens, q, H=H)
    assert not plan.tensor_cores
    ok, mx, rel = close(got, g["out"])
    assert ok, (mx, rel)


def test_mla_lse_and_splits():
    lens = [5000, 3, 12000]
    pool, bt, q = mla_case(lens, seed=3)
    got, lse, plan = run_decode(pool, bt, lens, q, want_lse=True)
    assert plan.n_chunks > len(lens)                 # long sequences were split across workers
    want = oracle.mla_decode_paged(pool, bt, lens, q, MLA_H, MLA_E, MLA_DV, PAGE, MLA_SCALE)
    ok, mx, rel = close(got, want)
    assert ok, (mx, rel)
    # log-sum-exp of the scaled scores, from the oracle's fp64 scores.  The
    # kernels sum the probabilities as rounded to bf16 for the P.V product
    # (so the normaliser matches the weights actually applied): a few 1e-4.
    for s, n in enumerate(lens):
        kv = np.stack([oracle.bf16_to_f32(pool[bt[s, t // PAGE], t % PAGE]) for t in range(n)]).astype(np.float64)
        sc = (oracle.bf16_to_f32(q[s]).astype(np.float64) @ kv.T) * MLA_SCALE
        m = sc.max(axis=1)
        ref = m + np.log(np.exp(sc - m[:, None]).sum(axis=1))
        np.testing.assert_allclose(lse[s], ref, rtol=0, atol=5e-3)


def test_mla_output_16_byte_aligned_equals_32_byte_aligned():
    """An output that starts 16 bytes past a 32-byte boundary takes the
    epilogue's 16-byte stores instead of its 32-byte ones: same bytes."""
    lens = [700, 64, 2500, 1]
    pool, bt, q = mla_case(lens, seed=6)
    L = np.asarray(lens, np.int32)
    plan = ct.MlaPlan(L, pool.shape[0], max_pages_per_seq=bt.shape[1], scale=MLA_SCALE)
    n_out = len(lens) * MLA_H * MLA_DV
    buf = empty((n_out + 16,), np.uint16)                 # 256-B aligned base
    pd, qd, btd, ld = dev(pool), dev(q), dev(bt), dev(L)
    outs = []
    for off in (0, 8):                                    # 0 and 16 bytes in
        buf.zero_()
        plan.decode(qd.data_ptr(), pd.data_ptr(), None, btd.data_ptr(), ld.data_ptr(), buf.data_ptr() + 2 * off,
                    None, stream())
        outs.append(host(buf, np.uint16)[off:off + n_out].copy())
    assert plan.tensor_cores
    np.testing.assert_array_equal(outs[0], outs[1])
    want = oracle.mla_decode_paged(pool, bt, lens, q, MLA_H, MLA_E, MLA_DV, PAGE, MLA_SCALE)
    ok, mx, rel = close(oracle.bf16_to_f32(outs[1]).reshape(len(lens), MLA_H, MLA_DV), want)
    assert ok, (mx, rel)


def test_mla_evicted_pages_are_skipped():
    lens = [300, 300]
    pool, bt, q = mla_case(lens, seed=4)
    bt = bt.copy()
    bt[0, 1] = -1                                    # an LRU-evicted page
    bt[1, 0] = -1                                    # a window-freed head
    got, _ = run_decode(pool, bt, lens, q)
    want = oracle.mla_decode_paged(pool, bt, lens, q, MLA_H, MLA_E, MLA_DV, PAGE, MLA_SCALE)
    ok, mx, rel = close(got, want)
    assert ok, (mx, rel)


@pytest.mark.parametrize("dtype", [ct.CT_KV_INT8, ct.CT_KV_E4M3])
def test_mla_quantised_pool(dtype):
    """Decode over int8 / e4m3 pages (dequantised on load) against the oracle
    run on the dequantised codes and scales; latent ~N(0,1) with 1 % x20."""
    lens = [700, 64, 2049]
    pool16, bt, q = mla_case(lens, seed=2, outlier_bp=100, outlier_mul=20.0)
    NP = pool16.shape[0]
    xf = oracle.bf16_to_f32(pool16.reshape(-1)).reshape(NP * PAGE, MLA_E)
    codes = np.zeros(NP * PAGE * MLA_E, np.uint8)
    sc = np.zeros(NP * PAGE, np.float32)
    back = np.zeros(NP * PAGE * MLA_E, np.float32)
    xf = np.ascontiguousarray(xf)
    if dtype == ct.CT_KV_INT8:
        O.orc_kv_quant_int8(xf.ctypes.data, NP * PAGE, MLA_E, codes.ctypes.data, sc.ctypes.data)
        O.orc_kv_dequant_int8(codes.ctypes.data, sc.ctypes.data, NP * PAGE, MLA_E, back.ctypes.data)
    else:
        O.orc_kv_quant_e4m3(xf.ctypes.data, NP * PAGE, MLA_E, codes.ctypes.data, sc.ctypes.data)
        O.orc_kv_dequant_e4m3(codes.ctypes.data, sc.ctypes.data, NP * PAGE, MLA_E, back.ctypes.data)
    got, plan = run_decode(codes.reshape(NP, PAGE, MLA_E), bt, lens, q, dtype=dtype, scales=sc)
    assert plan.tensor_cores                         # codes widened to bf16 in shared memory, tcgen05 GEMMs
    want = oracle_decode_f32(back.reshape(NP, PAGE, MLA_E), bt, lens, oracle.bf16_to_f32(q.reshape(-1)).reshape(
        q.shape), MLA_H, MLA_E, MLA_DV, PAGE)
    ok, mx, rel = close(got, want)
    assert ok, (mx, rel)
    # stale slots past each sequence's end hold NaN codes and NaN scales: no effect
    codes2 = codes.reshape(NP * PAGE, MLA_E).copy()
    sc2 = sc.copy()
    for s_, n in enumerate(lens):
        for t in range(n, ((n + PAGE - 1) // PAGE) * PAGE):
            slot = bt[s_, t // PAGE] * PAGE + t % PAGE
            codes2[slot] = 0x7F if dtype == ct.CT_KV_E4M3 else 0x80
            sc2[slot] = np.nan
    got2, _ = run_decode(codes2.reshape(NP, PAGE, MLA_E), bt, lens, q, dtype=dtype, scales=sc2)
    assert np.array_equal(np.isnan(got2), np.zeros_like(got2, bool))
    ok, mx, rel = close(got2, want)
    assert ok, (mx, rel)


@pytest.mark.parametrize("dtype", [ct.CT_KV_INT8, ct.CT_KV_E4M3])
def test_mla_quantised_pool_long(dtype):
    """Quantised pages through the full tensor-core pipeline: sequences long
    enough to be split across workers (combine path) and to cycle every page
    stage many times."""
    lens = [9000, 4097, 31, 12800]
    pool16, bt, q = mla_case(lens, seed=5, outlier_bp=100, outlier_mul=20.0)
    NP = pool16.shape[0]
    xf = np.ascontiguousarray(oracle.bf16_to_f32(pool16.reshape(-1)).reshape(NP * PAGE, MLA_E))
    codes = np.zeros(NP * PAGE * MLA_E, np.uint8)
    sc = np.zeros(NP * PAGE, np.float32)
    back = np.zeros(NP * PAGE * MLA_E, np.float32)
    quant = O.orc_kv_quant_int8 if dtype == ct.CT_KV_INT8 else O.orc_kv_quant_e4m3
    dequant = O.orc_kv_dequant_int8 if dtype == ct.CT_KV_INT8 else O.orc_kv_dequant_e4m3
    quant(xf.ctypes.data, NP * PAGE, MLA_E, codes.ctypes.data, sc.ctypes.data)
    dequant(codes.ctypes.data, sc.ctypes.data, NP * PAGE, MLA_E, back.ctypes.data)
    got, plan = run_decode(codes.reshape(NP, PAGE, MLA_E), bt, lens, q, dtype=dtype, scales=sc)
    assert plan.tensor_cores
    want = oracle_decode_f32(back.reshape(NP, PAGE, MLA_E), bt, lens, oracle.bf16_to_f32(q.reshape(-1)).reshape(
        q.shape), MLA_H, MLA_E, MLA_DV, PAGE)
    ok, mx, rel = close(got, want)
    assert ok, (mx, rel)


def test_mla_full_size_batch32_ctx4096():
    """The MLA paged decode configuration at full size: 32 sequences x 4096
    tokens, 128 heads, 576-d bf16 entries, 64-token pages in one random
    permutation of the pool.  Parity on 4 sequences against the oracle, and
    size-independent checks on all 32: a zero query attends uniformly (output
    = mean of the latents), and permuting the pages does not change results."""
    S, T = 32, 4096
    lens = [T] * S
    pool, bt, q = mla_case(lens, seed=1)
    got, plan = run_decode(pool, bt, lens, q)
    assert plan.n_chunks >= S
    sub = [0, 9, 22, 31]
    want = oracle.mla_decode_paged(pool, bt[sub], [T] * len(sub), q[sub], MLA_H, MLA_E, MLA_DV, PAGE, MLA_SCALE)
    ok, mx, rel = close(got[sub], want)
    assert ok, (mx, rel)
    # zero query -> uniform softmax -> mean latent (all heads)
    q0 = np.zeros_like(q)
    got0, _ = run_decode(pool, bt, lens, q0)
    pd = torch.from_numpy(pool.view(np.int16)).cuda().view(torch.bfloat16).float()
    btd = torch.from_numpy(bt.astype(np.int64)).cuda()
    mean = pd[btd].reshape(S, T, MLA_E)[:, :, :MLA_DV].mean(dim=1).cpu().numpy()
    assert np.abs(got0 - mean[:, None, :]).max() < 2e-2
    # re-permute physical pages
    perm = oracle.permutation(oracle.key(1, 77), pool.shape[0])
    inv = np.argsort(perm)
    pool2 = pool[perm]
    bt2 = inv[bt].astype(np.int32)
    got2, _ = run_decode(pool2, bt2, lens, q)
    assert np.array_equal(got2, got)


def test_mla_variable_lengths_sharded_shape():
    """Log-uniform lengths (the sequence-sharded serving shape, reduced to 48
    sequences of 512..16384 tokens); parity on a stratified subset."""
    lens = oracle.lengths_loguniform(oracle.key(4, 0), 48, 512, 16384).astype(np.int32)
    pool, bt, q = mla_case(lens, seed=4)
    got, plan = run_decode(pool, bt, lens, q)
    order = np.argsort(lens)
    sub = sorted(set(order[[0, 12, 24, 36, 47]].tolist()))
    want = oracle.mla_decode_paged(pool, bt[sub], lens[sub], q[sub], MLA_H, MLA_E, MLA_DV, PAGE, MLA_SCALE)
    ok, mx, rel = close(got[sub], want)
    assert ok, (mx, rel)


@pytest.mark.parametrize("zero_q", [False, True])
def test_mla_many_short_sequences(zero_q):
    """Many short sequences: every worker runs several chunks of one to three
    pages back to back, so chunk boundaries (query reloads, epilogues, the
    split-KV combine) come every few tiles.  A zero query makes every
    softmax uniform (output = mean of the latents)."""
    k = oracle.key(31, 600)
    lens = oracle.lengths_loguniform(k, 600, 1, 200).astype(np.int32)
    pool, bt, q = mla_case(lens, seed=31)
    if zero_q:
        q = np.zeros_like(q)
    got, plan = run_decode(pool, bt, lens, q)
    assert plan.tensor_cores
    want = oracle.mla_decode_paged(pool, bt, lens, q, MLA_H, MLA_E, MLA_DV, PAGE, MLA_SCALE)
    ok, mx, rel = close(got, want)
    assert ok, (mx, rel)


def test_mla_plan_follows_device_lengths():
    """A plan splits the work on the device from the lengths it is given at
    each decode: the same plan decodes sequences that grew (new pages), that
    shrank, and that became empty, as a serving loop reuses one plan."""
    cap = [3000, 700, 64, 5000, 1]
    pool, bt, q = mla_case(cap, seed=41)
    plan = ct.MlaPlan(np.array([10, 10, 10, 10, 10], np.int32), pool.shape[0], max_pages_per_seq=bt.shape[1])
    pd, qd, btd = dev(pool), dev(q), dev(bt)
    for lens in ([10, 10, 10, 10, 1], [2999, 65, 64, 4097, 0], [3000, 700, 64, 5000, 1], [1, 0, 63, 129, 1]):
        lens = np.array(lens, np.int32)
        ld = dev(lens)
        out = empty((len(lens), MLA_H, MLA_DV), np.uint16)
        plan.decode(qd.data_ptr(), pd.data_ptr(), None, btd.data_ptr(), ld.data_ptr(), out.data_ptr(), None, stream())
        got = oracle.bf16_to_f32(host(out, np.uint16)).reshape(len(lens), MLA_H, MLA_DV)
        want = oracle.mla_decode_paged(pool, bt, lens, q, MLA_H, MLA_E, MLA_DV, PAGE, MLA_SCALE)
        ok, mx, rel = close(got, want)
        assert ok, (lens.tolist(), mx, rel)
        assert np.all(got[lens == 0] == 0)


def test_mla_decode_graph_replay_follows_appends():
    """A serving loop: the decode (plan, decode kernel, combine) is captured
    once into a CUDA graph; between replays the sequences grow through
    ct_kv_paged_append, some across page boundaries.  Each replay equals an
    ordinary decode of the same state, bit for bit."""
    S, E, NP, MP = 6, MLA_E, 80, 40
    lens0 = [70, 1, 300, 64, 129, 2000]
    grow = [1, 63, 1, 1, 64, 5]
    steps = 3
    x = oracle.normal_bf16(oracle.key(8, 3), 0, (sum(lens0) + steps * sum(grow)) * E).reshape(-1, E)
    h = ct.PagedKV(S, MP, NP, PAGE, E, 0, ct.CT_KV_BF16, 0, stream())
    h.set_free_order(oracle.permutation(oracle.key(8, 4), NP))
    xd = dev(x)
    h.append(list(range(S)), lens0, xd.data_ptr(), ct.CT_KV_BF16)
    qd = dev(oracle.normal_bf16(oracle.key(8, 5), 0, S * MLA_H * E))
    plan = ct.MlaPlan(np.array(lens0, np.int32), NP, max_pages_per_seq=MP)
    out_g = empty((S, MLA_H, MLA_DV), np.uint16)
    out_e = empty((S, MLA_H, MLA_DV), np.uint16)
    side = torch.cuda.Stream()

    def decode(out, st):
        plan.decode(qd.data_ptr(), h.pool, None, h.block_table_dev, h.seq_lens_dev, out.data_ptr(), None, st)

    torch.cuda.synchronize()
    with torch.cuda.stream(side):
        decode(out_g, side.cuda_stream)                  # first call outside the capture (attributes, maps)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        decode(out_g, side.cuda_stream)
    off = sum(lens0)
    for _ in range(steps):
        h.append(list(range(S)), grow, xd.data_ptr() + off * E * 2, ct.CT_KV_BF16)
        off += sum(grow)
        torch.cuda.synchronize()
        g.replay()
        torch.cuda.synchronize()
        decode(out_e, stream())
        assert np.array_equal(host(out_g, np.uint16), host(out_e, np.uint16))
    assert h.seq_lens().tolist() == [l + steps * d for l, d in zip(lens0, grow)]
    del g
    h.close()


def test_mla_through_paged_handle():
    """Append through ct_kv_paged_append, then decode the handle's pool."""
    S, E = 3, MLA_E
    lens = [100, 64, 257]
    total = sum(lens)
    x = oracle.normal_bf16(oracle.key(6, 3), 0, total * E).reshape(total, E)
    h = ct.PagedKV(S, 8, 20, PAGE, E, 0, ct.CT_KV_BF16, 0, stream())
    h.set_free_order(oracle.permutation(oracle.key(6, 4), 20))
    xd = dev(x)
    h.append(list(range(S)), lens, xd.data_ptr(), ct.CT_KV_BF16)
    q = oracle.normal_bf16(oracle.key(6, 5), 0, S * MLA_H * E).reshape(S, MLA_H, E)
    plan = ct.MlaPlan(lens, 20, max_pages_per_seq=8)
    out = empty((S, MLA_H, MLA_DV), np.uint16)
    qd = dev(q)
    plan.decode(qd.data_ptr(), h.pool, None, h.block_table_dev, h.seq_lens_dev, out.data_ptr(), None, stream())
    got = oracle.bf16_to_f32(host(out, np.uint16)).reshape(S, MLA_H, MLA_DV)
    bt = h.block_table()
    pool = np.zeros((20, PAGE, E), np.uint16)
    off = 0
    for s, n in enumerate(lens):
        for t in range(n):
            pool[bt[s, t // PAGE], t % PAGE] = x[off + t]
        off += n
    want = oracle.mla_decode_paged(pool, bt, lens, q, MLA_H, E, MLA_DV, PAGE, MLA_SCALE)
    ok, mx, rel = close(got, want)
    assert ok, (mx, rel)
    h.close()


def _pinned(a):
    t = torch.from_numpy(np.ascontiguousarray(a).view(np.int16).copy())
    return t.pin_memory()


@pytest.mark.parametrize("n_seq", [4, 96])
def test_mla_step_host(n_seq):
    """ct_attn_mla_decode_step_host: append each sequence's new token from
    host memory, decode, copy the outputs to host memory.  96 sequences move
    about 27 MB per step, enough for the copies of one sequence group to run
    during the decode of another; 4 sequences run in one group."""
    k = oracle.key(21, n_seq)
    lens = oracle.lengths_loguniform(k, n_seq, 64, 3000).astype(np.int32)
    lens_after = lens + 1
    pool, bt, q = mla_case(lens_after, seed=21)
    slots = np.array([bt[s, n // PAGE] * PAGE + n % PAGE for s, n in enumerate(lens)], np.int32)
    new = np.stack([pool[sl // PAGE, sl % PAGE] for sl in slots])
    before = pool.copy()
    for sl in slots:
        before[sl // PAGE, sl % PAGE] = 0x7FC0          # NaN until the step writes the token
    plan = ct.MlaPlan(lens_after, pool.shape[0], max_pages_per_seq=bt.shape[1], scale=MLA_SCALE)
    pd, btd, ld, sd = dev(before), dev(bt), dev(lens_after), dev(slots)
    qh, eh = _pinned(q), _pinned(new)
    oh = torch.empty((n_seq, MLA_H, MLA_DV), dtype=torch.int16).pin_memory()
    plan.step_host(qh, eh, sd, pd, None, btd, ld, oh, stream())
    assert np.array_equal(host(pd, np.uint16), pool)              # every new token landed bit-exactly
    got = oracle.bf16_to_f32(oh.numpy().view(np.uint16)).reshape(n_seq, MLA_H, MLA_DV)
    # the same decode on the device path
    ref_dev, _ = run_decode(pool, bt, lens_after, q)
    ok, mx, rel = close(got, ref_dev)
    assert ok, (mx, rel)
    sub = sorted(set(np.argsort(lens)[[0, n_seq // 2, n_seq - 1]].tolist()))
    want = oracle.mla_decode_paged(pool, bt[sub], lens_after[sub], q[sub], MLA_H, MLA_E, MLA_DV, PAGE, MLA_SCALE)
    ok, mx, rel = close(got[sub], want)
    assert ok, (mx, rel)
    if n_seq == 4:                                               # one group: the plan's own chunks
        assert np.array_equal(got, ref_dev)
    # a second call on the same plan, without appends, repeats the outputs
    oh2 = torch.empty_like(oh).pin_memory()
    plan.step_host(qh, None, None, pd, None, btd, ld, oh2, stream())
    assert torch.equal(oh, oh2)


@pytest.mark.parametrize("dtype", [ct.CT_KV_INT8, ct.CT_KV_E4M3])
def test_mla_step_host_quantised_pool(dtype):
    """The host-buffer step over an int8 / e4m3 pool: the new tokens are
    quantised on append exactly as the oracle codes them (codes and scales
    bit-exact), and the decode, cut into sequence groups on two streams,
    matches the oracle on the dequantised pool (a sample of the sequences)."""
    n_seq = 40                                                  # ~11 MB of copies: three sequence groups
    lens = oracle.lengths_loguniform(oracle.key(23, 1), n_seq, 64, 2000).astype(np.int32)
    lens_after = lens + 1
    pool16, bt, q = mla_case(lens_after, seed=23, outlier_bp=100, outlier_mul=20.0)
    NP = pool16.shape[0]
    xf = np.ascontiguousarray(oracle.bf16_to_f32(pool16.reshape(-1)).reshape(NP * PAGE, MLA_E))
    codes = np.zeros(NP * PAGE * MLA_E, np.uint8)
    sc = np.zeros(NP * PAGE, np.float32)
    quant = O.orc_kv_quant_int8 if dtype == ct.CT_KV_INT8 else O.orc_kv_quant_e4m3
    quant(xf.ctypes.data, NP * PAGE, MLA_E, codes.ctypes.data, sc.ctypes.data)
    codes = codes.reshape(NP * PAGE, MLA_E)
    slots = np.array([bt[s, n // PAGE] * PAGE + n % PAGE for s, n in enumerate(lens)], np.int32)
    new = pool16.reshape(NP * PAGE, MLA_E)[slots]
    codes_before, sc_before = codes.copy(), sc.copy()
    codes_before[slots] = 0x7F if dtype == ct.CT_KV_E4M3 else 0x80   # stale until the step writes the token
    sc_before[slots] = np.nan
    plan = ct.MlaPlan(lens_after, NP, max_pages_per_seq=bt.shape[1], kv_dtype=dtype, scale=MLA_SCALE)
    pd, sd_, btd, ld, slotd = dev(codes_before), dev(sc_before), dev(bt), dev(lens_after), dev(slots)
    qh, eh = _pinned(q), _pinned(new)
    oh = torch.empty((n_seq, MLA_H, MLA_DV), dtype=torch.int16).pin_memory()
    plan.step_host(qh, eh, slotd, pd, sd_, btd, ld, oh, stream())
    assert np.array_equal(host(pd, np.uint8).reshape(NP * PAGE, MLA_E), codes)
    assert np.array_equal(host(sd_, np.float32), sc)
    got = oracle.bf16_to_f32(oh.numpy().view(np.uint16)).reshape(n_seq, MLA_H, MLA_DV)
    back = np.zeros(NP * PAGE * MLA_E, np.float32)
    dequant = O.orc_kv_dequant_int8 if dtype == ct.CT_KV_INT8 else O.orc_kv_dequant_e4m3
    cc = np.ascontiguousarray(codes.reshape(-1))
    dequant(cc.ctypes.data, sc.ctypes.data, NP * PAGE, MLA_E, back.ctypes.data)
    sub = sorted(set(np.argsort(lens)[[0, 1, n_seq // 3, n_seq // 2, n_seq - 2, n_seq - 1]].tolist()))
    qf = oracle.bf16_to_f32(q.reshape(-1)).reshape(q.shape)
    want = oracle_decode_f32(back.reshape(NP, PAGE, MLA_E), bt[sub], lens_after[sub], qf[sub], MLA_H, MLA_E, MLA_DV,
                             PAGE)
    ok, mx, rel = close(got[sub], want)
    assert ok, (mx, rel)
