"""GPU: parity at the full sizes of the two largest configurations.

* Sequence-sharded serving (one GPU's whole share at N=1): 1024 sequences,
  context lengths log-uniform 512..65536 (seed 4), bf16 MLA latent cache in
  64-token pages of one random permutation, 128 heads, scale 1/sqrt(192).
  The whole batch is decoded on the device; the oracle checks a subset that
  holds the longest and the shortest sequence, a stratified sample of the
  lengths, and sequences the work plan splits across workers (so their
  partial results go through the split-KV combine).  The oracle reads back
  exactly the pages the kernel read.
* Quantised pools: 64 sequences x 8192 tokens, latents N(0,1) with 1 % of the
  values x20 (seed 2), quantise-on-append to int8 and to fp8-e4m3 with one
  fp32 scale per token.  Codes and scales of all 524,288 tokens must equal
  the oracle's bit for bit; attention is checked on a subset against the
  oracle run on the dequantised codes and scales.

Tolerance for attention: elementwise |got - ref| <= 2e-2 + 1e-2 |ref|."""
import numpy as np
import pytest
import torch

import cautreo_b200 as ct
import oracle
from gpu_util import dev, empty, host, stream
from helpers import MLA_DV, MLA_E, MLA_H, MLA_SCALE, PAGE, close

pytestmark = pytest.mark.gpu
O = oracle.port()


@pytest.fixture(autouse=True)
def no_expired_waits():
    ct.lib().ct_mla_tc_error(1)
    yield
    assert ct.lib().ct_mla_tc_error(1) == 0


def split_sequences(lens, workers, page=PAGE):
    """Sequences the work plan cuts across workers: the sequences' pages laid
    end to end, worker w takes the pages [w*Q, (w+1)*Q) with
    Q = ceil(total / workers) (the planning kernel's rule)."""
    pages = [(int(n) + page - 1) // page for n in lens]
    total = sum(pages)
    q = max(1, -(-total // workers))
    out, cp = [], 0
    for s, n in enumerate(pages):
        if n and (cp + n - 1) // q != cp // q:
            out.append(s)
        cp += n
    return out


def gather_subset(pool_dev, bt, lens, subset, page=PAGE, E=MLA_E):
    """The subset's pages copied back from the device into a compact pool,
    with the block table renumbered to it."""
    pool2 = pool_dev.view(-1, page * E)
    rows, bt_sub = [], np.full((len(subset), bt.shape[1]), -1, np.int32)
    nxt = 0
    for i, s in enumerate(subset):
        pages = (int(lens[s]) + page - 1) // page
        rows.append(torch.from_numpy(bt[s, :pages].astype(np.int64)))
        bt_sub[i, :pages] = np.arange(nxt, nxt + pages, dtype=np.int32)
        nxt += pages
    idx = torch.cat(rows).cuda()
    sub = pool2[idx].cpu().numpy().view(np.uint16).reshape(nxt, page, E)
    return sub, bt_sub


def test_mla_full_size_sharded_serving_workload():
    L = ct.lib()
    S = 1024
    lens = oracle.lengths_loguniform(oracle.key(4, 0), S, 512, 65536).astype(np.int32)
    pages = (lens + PAGE - 1) // PAGE
    NP, MP = int(pages.sum()), int(pages.max())
    perm = oracle.permutation(oracle.key(4, 12), NP)
    bt = np.full((S, MP), -1, np.int32)
    off = np.concatenate([[0], np.cumsum(pages)])
    for s in range(S):
        bt[s, :pages[s]] = perm[off[s]:off[s + 1]]
    sp = stream()
    pool = torch.empty(NP * PAGE * MLA_E, dtype=torch.int16, device="cuda")     # 15.8 GB
    btd, ld = dev(bt), dev(lens)
    ct.check(L.ct_synth_fill_paged(pool.data_ptr(), None, ct.CT_KV_BF16, btd.data_ptr(), MP, None, ld.data_ptr(), S,
                                   int(lens.max()), PAGE, MLA_E, ct.synth_key(4, 10), 0, 1.0, sp), "fill")
    q = torch.empty(S * MLA_H * MLA_E, dtype=torch.int16, device="cuda")
    ct.check(L.ct_synth_fill(q.data_ptr(), 0, ct.synth_key(4, 11), 0, S * MLA_H * MLA_E, 0, 1.0, sp))
    plan = ct.MlaPlan(lens, NP, max_pages_per_seq=MP)
    assert plan.tensor_cores
    out = empty((S, MLA_H, MLA_DV), np.uint16)
    lse = empty((S, MLA_H), np.float32)
    plan.decode(q.data_ptr(), pool.data_ptr(), None, btd.data_ptr(), ld.data_ptr(), out.data_ptr(), lse.data_ptr(),
                sp)
    got = oracle.bf16_to_f32(host(out, np.uint16)).reshape(S, MLA_H, MLA_DV)
    got_lse = host(lse, np.float32)
    assert np.isfinite(got).all() and np.isfinite(got_lse).all()

    order = np.argsort(lens, kind="stable")
    split = split_sequences(lens, plan.workers)
    assert len(split) >= plan.workers // 2            # the balanced plan cuts many sequences
    subset = {int(order[-1]), int(order[0])}           # longest, shortest
    subset |= {int(order[i]) for i in np.linspace(0, S - 1, 6).astype(int)[1:-1]}
    subset |= {split[0], split[len(split) // 2], split[-1]}
    subset = sorted(subset)
    sub_pool, sub_bt = gather_subset(pool, bt, lens, subset)
    qh = q.view(S, MLA_H * MLA_E)[torch.tensor(subset).cuda()].cpu().numpy().view(np.uint16)
    want = oracle.mla_decode_paged(sub_pool, sub_bt, lens[subset], qh.reshape(len(subset), MLA_H, MLA_E), MLA_H,
                                   MLA_E, MLA_DV, PAGE, MLA_SCALE)
    ok, mx, excess = close(got[subset], want)
    assert ok, (mx, excess)


@pytest.mark.parametrize("dtype", [ct.CT_KV_INT8, ct.CT_KV_E4M3])
def test_quantised_pools_full_size(dtype):
    L = ct.lib()
    B, T = 64, 8192
    n_tok = B * T
    pages_per = T // PAGE
    NP = B * pages_per
    sp = stream()
    src = torch.empty(n_tok * MLA_E, dtype=torch.int16, device="cuda")
    ct.check(L.ct_synth_fill(src.data_ptr(), 0, ct.synth_key(2, 10), 0, n_tok * MLA_E, 100, 20.0, sp))
    kv = ct.PagedKV(B, pages_per, NP, PAGE, MLA_E, 0, dtype, 0, sp)
    kv.set_free_order(oracle.permutation(oracle.key(2, 12), NP))
    kv.append(list(range(B)), [T] * B, src.data_ptr(), ct.CT_KV_BF16)      # tokens of seq s = rows s*T ...
    torch.cuda.synchronize()
    bt = kv.block_table()
    # codes and scales of every token, against the oracle's codec of the same bf16 values
    xf = np.ascontiguousarray(oracle.bf16_to_f32(src.cpu().numpy().view(np.uint16)))
    want_c = np.empty(n_tok * MLA_E, np.uint8)
    want_s = np.empty(n_tok, np.float32)
    quant = O.orc_kv_quant_int8 if dtype == ct.CT_KV_INT8 else O.orc_kv_quant_e4m3
    quant(xf.ctypes.data, n_tok, MLA_E, want_c.ctypes.data, want_s.ctypes.data)
    nbytes = NP * PAGE * MLA_E
    codes = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    scales = torch.empty(NP * PAGE, dtype=torch.float32, device="cuda")
    ct.check(L.ct_hal_cuda_memcpy(codes.data_ptr(), kv.pool, nbytes, 2, sp), "copy codes")
    ct.check(L.ct_hal_cuda_memcpy(scales.data_ptr(), kv.scales, NP * PAGE * 4, 2, sp), "copy scales")
    slot = (bt[:, :, None].astype(np.int64) * PAGE + np.arange(PAGE)[None, None, :]).reshape(-1)   # token order
    got_c = host(codes, np.uint8).reshape(NP * PAGE, MLA_E)[slot]
    got_s = host(scales, np.float32)[slot]
    assert np.array_equal(got_s.view(np.uint32), want_s.view(np.uint32))
    assert np.array_equal(got_c, want_c.reshape(n_tok, MLA_E))
    # decode every sequence over the quantised pages; oracle on a subset
    q = torch.empty(B * MLA_H * MLA_E, dtype=torch.int16, device="cuda")
    ct.check(L.ct_synth_fill(q.data_ptr(), 0, ct.synth_key(2, 11), 0, B * MLA_H * MLA_E, 0, 1.0, sp))
    plan = ct.MlaPlan(np.full(B, T, np.int32), NP, kv_dtype=dtype, max_pages_per_seq=pages_per)
    assert plan.tensor_cores
    out = empty((B, MLA_H, MLA_DV), np.uint16)
    plan.decode(q.data_ptr(), kv.pool, kv.scales, kv.block_table_dev, kv.seq_lens_dev, out.data_ptr(), None, sp)
    got = oracle.bf16_to_f32(host(out, np.uint16)).reshape(B, MLA_H, MLA_DV)
    assert np.isfinite(got).all()
    subset = [0, 21, 63]
    back = np.empty(len(subset) * T * MLA_E, np.float32)
    codes_sub = np.ascontiguousarray(want_c.reshape(B, T * MLA_E)[subset])
    scales_sub = np.ascontiguousarray(want_s.reshape(B, T)[subset])
    dequant = O.orc_kv_dequant_int8 if dtype == ct.CT_KV_INT8 else O.orc_kv_dequant_e4m3
    dequant(codes_sub.ctypes.data, scales_sub.ctypes.data, len(subset) * T, MLA_E, back.ctypes.data)
    qf = oracle.bf16_to_f32(q.cpu().numpy().view(np.uint16)).reshape(B, MLA_H, MLA_E)
    want = np.zeros((len(subset), MLA_H, MLA_DV), np.float32)
    kvs = back.reshape(len(subset), T, MLA_E)
    for i, s in enumerate(subset):
        qs = np.ascontiguousarray(qf[s])
        kvi = np.ascontiguousarray(kvs[i])
        assert O.orc_mla_decode(qs.ctypes.data, kvi.ctypes.data, T, MLA_H, MLA_E, MLA_DV, MLA_SCALE,
                                want[i].ctypes.data) == 0
    ok, mx, excess = close(got[subset], want)
    assert ok, (mx, excess)
    plan.close()
    kv.close()
