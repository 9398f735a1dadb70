"""Generate the golden fixtures in tests/golden/ from the reference's own
CPU code (oracle/_ref/libctref.so, compiled from the reference sources by
oracle/Makefile) and, for the paged allocator that has no reference code,
from the oracle restatement.

    make -C oracle && python tests/golden/make_golden.py

Fixtures (numpy .npz):
  quant_ref.npz   Q8_0/Q4_0/Q2_0/Q1_0 encodings and decodings of edge-case
                  blocks; ct_quant_f32_to_fp16 over sample floats and
                  ct_quant_fp16_to_f32 over all 65536 halves.
  attn_ref.npz    ct_attn_forward / ct_attn_softmax on seeded inputs.
  kv_ref.npz      ct_kv_save bytes and ct_kv_compress results.
  plain_ref.npz   the plain decode run (4 layers x 8 heads x 64, 256 steps,
                  seed 0) through ct_kv_append + ct_kv_get + ct_attn_forward,
                  outputs at selected steps.
  mla_ref.npz     paged MLA decode through the reference ct_attn_forward
                  (every head reads the same [n][576] entries, so with 576-d
                  heads it is exactly absorbed-MLA attention; the first 512
                  output values are the result), small ragged case.
  alloc_ref.npz   the oracle allocator replay (window + LRU) for a small
                  pressure case.
"""
from __future__ import annotations

import ctypes as C
import os
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))
sys.path.insert(0, str(HERE.parent))

import oracle  # noqa: E402
from helpers import MLA_DV, MLA_E, MLA_SCALE, PAGE, mla_case, plain_inputs, reference_plain_decode  # noqa: E402

QTYPES = {1: 34, 2: 18, 3: 10, 4: 6}


def quant_blocks():
    blocks = []
    blocks.append([(i - 16) * 0.5 for i in range(32)])                    # quant_test.c ramp
    blocks.append([1.0] * 32)                                              # constant
    blocks.append([0.0] * 32)                                              # zero block
    blocks.append([1.0 if i < 16 else -1.0 for i in range(32)])           # sign pattern
    blocks.append([float(i - 16) for i in range(32)])                      # generic dispatch case
    blocks.append([1e-3 * (i - 16) for i in range(32)])                    # amax/127 < 2^-15: Inf scale quirk
    blocks.append([2.0 ** -15 * 127 * (1 + i / 64) * (-1) ** i for i in range(32)])  # exponent-112 scale
    blocks.append([65504.0 * (i / 31) for i in range(32)])                # fp16 overflow range
    blocks.append([0.5 * (-1) ** i for i in range(32)])                    # ties at x*id + 0.5
    rng = oracle.normal_f32(oracle.key(7, 0), 0, 32 * 8)
    rng[5] *= 20.0
    rng[77] *= -20.0
    for b in range(8):
        blocks.append(list(rng[b * 32:(b + 1) * 32]))
    return np.asarray(blocks, np.float32)


def make_quant(R):
    x = quant_blocks()
    out = {"x": x}
    for t, nb in QTYPES.items():
        enc = np.zeros((len(x), nb), np.uint8)
        dec = np.zeros_like(x)
        for i, blk in enumerate(x):
            blk = np.ascontiguousarray(blk)
            w = R.ct_quant_do(blk.ctypes.data, enc[i].ctypes.data, 32, t)
            assert w == nb
            R.ct_quant_undo(enc[i].ctypes.data, dec[i].ctypes.data, 32, t)
        out[f"enc{t}"] = enc
        out[f"dec{t}"] = dec
    # fp16 conversions
    f = np.concatenate([
        np.array([0.0, -0.0, 1.0, -1.0, 3.140625, 0.5, -0.5, 65504.0, 0.001, 1e-5, 3.0517578125e-05,
                  6.103515625e-05, 65520.0, 1e30, np.inf, -np.inf], np.float32),
        oracle.normal_f32(oracle.key(7, 1), 0, 2048) * np.float32(100.0),
        (2.0 ** np.linspace(-30, 17, 2048)).astype(np.float32),
    ]).astype(np.float32)
    out["f32"] = f
    out["f32_to_fp16"] = np.array([R.ct_quant_f32_to_fp16(float(v)) for v in f], np.uint16)
    out["fp16_to_f32"] = np.array([R.ct_quant_fp16_to_f32(h) for h in range(65536)], np.float32)
    np.savez_compressed(HERE / "quant_ref.npz", **out)


def make_attn(R):
    cases = [(1, 1, 4), (2, 1, 4), (7, 3, 16), (33, 8, 64), (300, 2, 64), (129, 4, 96), (5, 16, 576)]
    out = {}
    for ci, (n, H, D) in enumerate(cases):
        k_ = oracle.key(8, ci)
        q = oracle.normal_f32(k_, 0, H * D)
        kk = oracle.normal_f32(k_, 1 << 20, n * D)
        vv = oracle.normal_f32(k_, 2 << 20, n * D)
        o = np.zeros(H * D, np.float32)
        scale = 0.0 if ci % 2 == 0 else 0.3
        assert R.ct_attn_forward(q.ctypes.data, kk.ctypes.data, vv.ctypes.data, n, H, D, scale, o.ctypes.data)
        out[f"c{ci}"] = np.array([n, H, D], np.int64)
        out[f"s{ci}"] = np.array([scale], np.float32)
        out[f"q{ci}"], out[f"k{ci}"], out[f"v{ci}"], out[f"o{ci}"] = q, kk, vv, o
    x = oracle.normal_f32(oracle.key(8, 99), 0, 1000) * np.float32(5.0)
    y = x.copy()
    R.ct_attn_softmax(y.ctypes.data, len(y))
    out["sm_x"], out["sm_y"] = x, y
    np.savez_compressed(HERE / "attn_ref.npz", **out)


def make_kv(R):
    out = {}
    L, H, D, ctx = 2, 4, 8, 16
    cfg = oracle.KvConfig(L, H, D, ctx, 1.0)
    c = R.ct_kv_create(C.byref(cfg))
    k = np.arange(32, dtype=np.float32)
    v = (np.arange(32) * 2).astype(np.float32)
    assert R.ct_kv_append(c, 0, 0, k.ctypes.data, v.ctypes.data)
    assert R.ct_kv_append(c, 1, 1, k.ctypes.data, v.ctypes.data)
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "kv.bin")
        assert R.ct_kv_save(c, path.encode())
        out["save_bytes"] = np.frombuffer(open(path, "rb").read(), np.uint8)
    R.ct_kv_destroy(c)
    # compress: random contents, several lengths and ratios
    for ci, (n, ratio) in enumerate([(8, 4.0), (13, 3.0), (16, 2.0), (5, 1.5), (9, 7.9)]):
        c = R.ct_kv_create(C.byref(cfg))
        kk = oracle.normal_f32(oracle.key(9, ci), 0, n * L * H * D).reshape(n, L, H * D)
        vv = oracle.normal_f32(oracle.key(9, ci), 1 << 20, n * L * H * D).reshape(n, L, H * D)
        for t in range(n):
            for l in range(L):
                R.ct_kv_append(c, l, t, np.ascontiguousarray(kk[t, l]).ctypes.data,
                               np.ascontiguousarray(vv[t, l]).ctypes.data)
        ok = R.ct_kv_compress(c, ratio)
        m = R.ct_kv_len(c)
        got_k = np.zeros((L, m, H * D), np.float32)
        got_v = np.zeros((L, m, H * D), np.float32)
        for l in range(L):
            for t in range(m):
                R.ct_kv_get(c, l, t, got_k[l, t].ctypes.data, got_v[l, t].ctypes.data)
        out[f"cmp{ci}"] = np.array([n, ok, m], np.int64)
        out[f"cmp{ci}_ratio"] = np.array([ratio], np.float32)
        out[f"cmp{ci}_k"], out[f"cmp{ci}_v"] = got_k, got_v
        R.ct_kv_destroy(c)
    np.savez_compressed(HERE / "kv_ref.npz", **out)


PLAIN_STEPS = [0, 1, 2, 63, 64, 65, 127, 128, 200, 255]


def make_plain():
    q, k, v = plain_inputs()
    outs = reference_plain_decode(q, k, v, keep_steps=set(PLAIN_STEPS))
    np.savez_compressed(HERE / "plain_ref.npz", steps=np.array(PLAIN_STEPS), out=np.stack([outs[s] for s in PLAIN_STEPS]),
                        q_head=q[:2, 0, :8], k_head=k[:2, 0, :8], v_head=v[:2, 0, :8])


MLA_LENS = [1, 63, 64, 65, 130, 0, 200]
MLA_HEADS = 16


def make_mla(R):
    pool, bt, q = mla_case(MLA_LENS, seed=1, H=MLA_HEADS)
    out = np.zeros((len(MLA_LENS), MLA_HEADS, MLA_DV), np.float32)
    for s, n in enumerate(MLA_LENS):
        if n == 0:
            continue
        kv = np.zeros((n, MLA_E), np.float32)
        for t in range(n):
            kv[t] = oracle.bf16_to_f32(pool[bt[s, t // PAGE], t % PAGE])
        qf = oracle.bf16_to_f32(q[s]).astype(np.float32)
        o = np.zeros((MLA_HEADS, MLA_E), np.float32)
        assert R.ct_attn_forward(qf.ctypes.data, kv.ctypes.data, kv.ctypes.data, n, MLA_HEADS, MLA_E,
                                 MLA_SCALE, o.ctypes.data)
        out[s] = o[:, :MLA_DV]
    np.savez_compressed(HERE / "mla_ref.npz", lens=np.array(MLA_LENS), heads=MLA_HEADS, out=out,
                        pool_head=pool.reshape(-1)[:64], q_head=q.reshape(-1)[:64], bt=bt)


ALLOC = dict(n_seqs=12, page_tokens=4, n_pages=22, max_pages=40, window=12)


def make_alloc():
    lens = oracle.lengths_loguniform(oracle.key(3, 0), ALLOC["n_seqs"], 8, 128)
    rc, bt, owner, ev, last, nfree = oracle.alloc_replay(lens, ALLOC["n_seqs"], ALLOC["page_tokens"],
                                                         ALLOC["n_pages"], ALLOC["max_pages"], ALLOC["window"])
    assert rc == 0, rc
    cbt, cmap = oracle.compact_plan(bt)
    np.savez_compressed(HERE / "alloc_ref.npz", lens=lens, bt=bt, owner=owner, events=np.array(ev, np.int64),
                        last=last, n_free=nfree, compact_bt=cbt, compact_map=cmap,
                        cfg=np.array([ALLOC[k] for k in ("n_seqs", "page_tokens", "n_pages", "max_pages", "window")]))


def main():
    R = oracle.ref()
    make_quant(R)
    make_attn(R)
    make_kv(R)
    make_plain()
    make_mla(R)
    make_alloc()
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
