"""Shared input generators and reference drivers for the tests.

Inputs are the seeded SplitMix64 / Box-Muller streams of the oracle
(oracle/ct_oracle.c), so the same values can be regenerated anywhere.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

import oracle

# Plain cache decode, the CPU-runnable configuration: 4 layers, 8 heads,
# head_dim 64, fp32, batch 1, 256 steps, q/k/v ~ N(0,1), seed 0.
PLAIN = dict(L=4, H=8, D=64, steps=256, seed=0)
# MLA shapes: 128 heads, 512 latent + 64 rope, 64-token pages.
MLA_H, MLA_E, MLA_DV, PAGE = 128, 576, 512, 64
MLA_SCALE = float(1.0 / np.sqrt(192.0))

ATOL, RTOL = 2e-2, 1e-2           # attention parity: |got - ref| <= ATOL + RTOL * |ref| elementwise


def plain_inputs(steps=None, L=4, H=8, D=64, seed=0):
    """q, k, v of the plain decode run as [steps][L][H*D] fp32."""
    steps = steps or PLAIN["steps"]
    n = steps * L * H * D
    q = oracle.normal_f32(oracle.key(seed, 0), 0, n).reshape(steps, L, H * D)
    k = oracle.normal_f32(oracle.key(seed, 1), 0, n).reshape(steps, L, H * D)
    v = oracle.normal_f32(oracle.key(seed, 2), 0, n).reshape(steps, L, H * D)
    return q, k, v


def reference_plain_decode(q, k, v, L=4, H=8, D=64, keep_steps=None):
    """The reference CPU path, step by step: ct_kv_append for every layer,
    then per layer and head a gather of that head's K/V rows through ct_kv_get
    and ct_attn_forward (src/kv_cache/kv_cache.c, src/attention/attention.c,
    compiled from the reference tree).  Returns {step: out [L][H*D]}."""
    R = oracle.ref()
    steps = q.shape[0]
    cfg = oracle.KvConfig(L, H, D, steps, 1.0)
    c = R.ct_kv_create(C.byref(cfg))
    krow = np.empty(H * D, np.float32)
    vrow = np.empty(H * D, np.float32)
    outs = {}
    try:
        for s in range(steps):
            for l in range(L):
                assert R.ct_kv_append(c, l, s, k[s, l].ctypes.data, v[s, l].ctypes.data)
            if keep_steps is not None and s not in keep_steps:
                continue
            out = np.empty((L, H * D), np.float32)
            n = s + 1
            for l in range(L):
                kh = np.empty((H, n, D), np.float32)
                vh = np.empty((H, n, D), np.float32)
                for t in range(n):
                    assert R.ct_kv_get(c, l, t, krow.ctypes.data, vrow.ctypes.data)
                    kh[:, t] = krow.reshape(H, D)
                    vh[:, t] = vrow.reshape(H, D)
                for h in range(H):
                    qh = np.ascontiguousarray(q[s, l, h * D:(h + 1) * D])
                    o = np.empty(D, np.float32)
                    assert R.ct_attn_forward(qh.ctypes.data, np.ascontiguousarray(kh[h]).ctypes.data,
                                             np.ascontiguousarray(vh[h]).ctypes.data, n, 1, D, 0.0, o.ctypes.data)
                    out[l, h * D:(h + 1) * D] = o
            outs[s] = out
    finally:
        R.ct_kv_destroy(c)
    return outs


def mla_case(lens, seed=1, H=MLA_H, E=MLA_E, page=PAGE, extra_pages=0, outlier_bp=0, outlier_mul=1.0):
    """A paged MLA cache: bf16 pool with randomly permuted pages (one
    permutation of all pages), block table, q.  Entry value e of token t of
    sequence s is element (s << 24 | t) * E + e of stream (seed, 10); q is
    stream (seed, 11); the page permutation is stream (seed, 12)."""
    lens = np.asarray(lens, np.int32)
    pages = [(int(n) + page - 1) // page for n in lens]
    max_pages = max(1, max(pages) if len(pages) else 1)
    n_pages = sum(pages) + extra_pages
    perm = oracle.permutation(oracle.key(seed, 12), max(n_pages, 1))
    bt = np.full((len(lens), max_pages), -1, np.int32)
    pool = np.zeros((max(n_pages, 1), page, E), np.uint16)
    k_kv = oracle.key(seed, 10)
    nxt = 0
    for s, n in enumerate(lens):
        n = int(n)
        for lp in range(pages[s]):
            bt[s, lp] = perm[nxt]
            nxt += 1
        if n == 0:
            continue
        # tokens of sequence s are contiguous in the stream: index (s<<24 | t)*E + e
        vals = oracle.normal_bf16(k_kv, (s << 24) * E, n * E, outlier_bp, outlier_mul).reshape(n, E)
        for lp in range(pages[s]):
            t0 = lp * page
            cnt = min(page, n - t0)
            pool[bt[s, lp], :cnt] = vals[t0:t0 + cnt]
    q = oracle.normal_bf16(oracle.key(seed, 11), 0, len(lens) * H * E).reshape(len(lens), H, E)
    return pool, bt, q


def close(got, want, atol=ATOL, rtol=RTOL):
    """Attention parity, elementwise: |got - want| <= atol + rtol * |want|
    (2e-2 absolute, 1e-2 relative), the combined absolute/relative bound the
    decode path is held to.  A pure 2e-2 absolute bound cannot hold for
    bf16 outputs beyond 8 in magnitude, whose rounding step alone is 2^-4
    (outlier-heavy caches produce such outputs), hence the relative term.
    Returns (ok, max |err|, max excess over the bound)."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    err = np.abs(got - want)
    bound = atol + rtol * np.abs(want)
    mx = float(err.max()) if err.size else 0.0
    excess = float((err - bound).max()) if err.size else -1.0
    return bool(np.all(err <= bound)), mx, excess
