"""CPU oracle for the KV-cache / decode-attention hot path.

TEST INFRASTRUCTURE ONLY.  Only tests/, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of bench.py may import this
package, and only as the checker or the timed CPU baseline.  The product
(``cautreo_b200``) never imports it.

Two libraries, both built by ``oracle/Makefile``:
  * ``_ref/libctref.so`` -- the reference's own src/kv_cache/kv_cache.c,
    src/attention/attention.c, src/quant/quant.c and src/hal/hal.c compiled
    from the reference tree (``ref()``);
  * ``_build/liboracle.so`` -- this repository's C11 restatement of the parts
    the reference lacks (``port()``); see ct_oracle.h for the file:line each
    function follows.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REF_LIB = HERE / "_ref" / "libctref.so"
PORT_LIB = HERE / "_build" / "liboracle.so"

P, F, U32, I32, U64, I64, SZ, B, V, I, D = (C.c_void_p, C.c_float, C.c_uint32, C.c_int32, C.c_uint64,
                                             C.c_int64, C.c_size_t, C.c_bool, None, C.c_int, C.c_double)


class KvConfig(C.Structure):
    _fields_ = [("n_layers", C.c_uint32), ("n_kv_heads", C.c_uint32), ("head_dim", C.c_uint32),
                ("max_ctx", C.c_uint32), ("compress_ratio", C.c_float)]


class KvStats(C.Structure):
    _fields_ = [("n_appends", C.c_uint64), ("n_reads", C.c_uint64), ("bytes_used", C.c_uint64),
                ("n_tokens", C.c_uint32)]


class AllocCfg(C.Structure):
    _fields_ = [("n_seqs", C.c_uint32), ("page_tokens", C.c_uint32), ("n_pages", C.c_uint32),
                ("max_pages_per_seq", C.c_uint32), ("window_tokens", C.c_uint32)]


class EvictEvent(C.Structure):
    _fields_ = [("round", C.c_uint32), ("seq", C.c_uint32), ("lpage", C.c_uint32), ("phys", C.c_int32),
                ("reason", C.c_uint32)]


REF_SIGS = {
    "ct_kv_create": (P, [C.POINTER(KvConfig)]),
    "ct_kv_destroy": (V, [P]),
    "ct_kv_append": (B, [P, U32, U32, P, P]),
    "ct_kv_get": (B, [P, U32, U32, P, P]),
    "ct_kv_len": (U32, [P]),
    "ct_kv_capacity": (U32, [P]),
    "ct_kv_reset": (V, [P]),
    "ct_kv_save": (B, [P, C.c_char_p]),
    "ct_kv_load": (B, [P, C.c_char_p]),
    "ct_kv_compress": (B, [P, F]),
    "ct_kv_stats": (KvStats, [P]),
    "ct_attn_forward": (B, [P, P, P, U32, U32, U32, F, P]),
    "ct_attn_forward_kv": (B, [P, P, P, U32, U32, U32, F, P]),
    "ct_attn_softmax": (V, [P, U32]),
    "ct_quant_q8_0": (V, [P, P, I64]),
    "ct_quant_q4_0": (V, [P, P, I64]),
    "ct_quant_q2_0": (V, [P, P, I64]),
    "ct_quant_q1_0": (V, [P, P, I64]),
    "ct_quant_deq8_0": (V, [P, P, I64]),
    "ct_quant_deq4_0": (V, [P, P, I64]),
    "ct_quant_deq2_0": (V, [P, P, I64]),
    "ct_quant_deq1_0": (V, [P, P, I64]),
    "ct_quant_do": (SZ, [P, P, I64, I]),
    "ct_quant_undo": (V, [P, P, I64, I]),
    "ct_quant_f32_to_fp16": (C.c_uint16, [F]),
    "ct_quant_fp16_to_f32": (F, [C.c_uint16]),
}

PORT_SIGS = {
    "orc_mix64": (U64, [U64]),
    "orc_key": (U64, [U64, U64]),
    "orc_u64": (U64, [U64, U64]),
    "orc_unit": (D, [U64, U64]),
    "orc_normal": (F, [U64, U64]),
    "orc_outlier": (I, [U64, U64, U32]),
    "orc_fill_normal_f32": (V, [U64, U64, U64, U32, F, P]),
    "orc_fill_normal_bf16": (V, [U64, U64, U64, U32, F, P]),
    "orc_permutation": (V, [U64, U32, P]),
    "orc_lengths_loguniform": (V, [U64, U32, U32, U32, P]),
    "orc_f32_to_bf16": (C.c_uint16, [F]),
    "orc_bf16_to_f32": (F, [C.c_uint16]),
    "orc_ct_f32_to_fp16": (C.c_uint16, [F]),
    "orc_ct_fp16_to_f32": (F, [C.c_uint16]),
    "orc_f32_to_e4m3_satfinite": (C.c_uint8, [F]),
    "orc_e4m3_to_f32": (F, [C.c_uint8]),
    "orc_q8_0_quantize": (V, [P, P, I64]),
    "orc_q8_0_dequantize": (V, [P, P, I64]),
    "orc_kv_quant_int8": (V, [P, U32, U32, P, P]),
    "orc_kv_dequant_int8": (V, [P, P, U32, U32, P]),
    "orc_kv_quant_e4m3": (V, [P, U32, U32, P, P]),
    "orc_kv_dequant_e4m3": (V, [P, P, U32, U32, P]),
    "orc_attn_softmax": (V, [P, U32]),
    "orc_attn_forward": (I, [P, P, P, U32, U32, U32, F, P]),
    "orc_mla_decode": (I, [P, P, U32, U32, U32, U32, F, P]),
    "orc_paged_gather_bf16_f32": (I, [P, P, U32, U32, U32, P]),
    "orc_mla_decode_paged_bf16": (I, [P, P, U32, P, U32, P, U32, U32, U32, U32, F, I, P]),
    "orc_kv_compress_every_kth": (U32, [P, P, U32, U32, U32, U32, F]),
    "orc_alloc_replay": (I, [C.POINTER(AllocCfg), P, P, P, P, U32, P, P, P]),
    "orc_compact_plan": (U32, [P, U32, U32, P]),
    "orc_lpt_assign": (V, [P, U32, U32, P]),
}

_REF = None
_PORT = None


def build() -> None:
    """Build the restatement, and the reference objects when the reference
    sources are present (they are not on every machine that runs tests)."""
    subprocess.run(["make", "-s", "-C", str(HERE), "port"], check=True)
    # where the reference sources lie is the Makefile's REF (overridable from
    # the environment); `have-ref` succeeds when they are there
    if subprocess.run(["make", "-s", "-C", str(HERE), "have-ref"], capture_output=True).returncode == 0:
        subprocess.run(["make", "-s", "-C", str(HERE), "ref"], check=True)
        # the reference's own unit-test programs, built from its sources
        subprocess.run(["make", "-s", "-C", str(HERE), "ref-tests"], check=True)
        # the reference's unit tests linked against this repository's library
        if (HERE.parent / "cautreo_b200" / "libcautreo_b200.so").exists():
            subprocess.run(["make", "-s", "-C", str(HERE), "ours-tests"], check=True)
            # the reference engine's transformer forward, against either KV cache
            subprocess.run(["make", "-s", "-C", str(HERE), "engine"], check=True)


def _load(path, sigs):
    L = C.CDLL(str(path))
    for name, (res, args) in sigs.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    return L


def ref_available() -> bool:
    return REF_LIB.exists()


def ref():
    """The reference's own CPU code (oracle/_ref/libctref.so)."""
    global _REF
    if _REF is None:
        if not REF_LIB.exists():
            raise RuntimeError(f"{REF_LIB} missing: build it with `make -C oracle ref` where the reference exists")
        _REF = _load(REF_LIB, REF_SIGS)
    return _REF


def port():
    """The C11 restatement (oracle/_build/liboracle.so)."""
    global _PORT
    if _PORT is None:
        if not PORT_LIB.exists():
            build()
        _PORT = _load(PORT_LIB, PORT_SIGS)
    return _PORT


def ptr(a):
    return None if a is None else a.ctypes.data


# ---- convenience -------------------------------------------------------------

def key(seed: int, stream: int) -> int:
    return int(port().orc_key(seed, stream))


def normal_bf16(k: int, start: int, n: int, outlier_bp: int = 0, mul: float = 1.0) -> np.ndarray:
    out = np.empty(n, np.uint16)
    port().orc_fill_normal_bf16(k, start, n, outlier_bp, mul, ptr(out))
    return out


def normal_f32(k: int, start: int, n: int, outlier_bp: int = 0, mul: float = 1.0) -> np.ndarray:
    out = np.empty(n, np.float32)
    port().orc_fill_normal_f32(k, start, n, outlier_bp, mul, ptr(out))
    return out


def bf16_to_f32(a: np.ndarray) -> np.ndarray:
    return (a.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(a: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def permutation(k: int, n: int) -> np.ndarray:
    out = np.empty(n, np.int32)
    port().orc_permutation(k, n, ptr(out))
    return out


def lengths_loguniform(k: int, n: int, lo: int, hi: int) -> np.ndarray:
    out = np.empty(n, np.uint32)
    port().orc_lengths_loguniform(k, n, lo, hi, ptr(out))
    return out


def mla_decode_paged(pool_bf16, bt, seq_lens, q_bf16, H, E, Dv, page_tokens, scale, n_threads=0):
    n_seq = len(seq_lens)
    out = np.empty((n_seq, H, Dv), np.float32)
    bt = np.ascontiguousarray(bt, np.int32)
    lens = np.ascontiguousarray(seq_lens, np.int32)
    pool_c = np.ascontiguousarray(pool_bf16)        # keep references for the duration of the call
    q_c = np.ascontiguousarray(q_bf16)
    rc = port().orc_mla_decode_paged_bf16(ptr(pool_c), ptr(bt), bt.shape[1], ptr(lens), n_seq, ptr(q_c), H, E, Dv,
                                          page_tokens, scale, n_threads, ptr(out))
    if rc != 0:
        raise RuntimeError("oracle mla decode failed")
    return out


def alloc_replay(lengths, n_seqs, page_tokens, n_pages, max_pages, window, max_events=1 << 22):
    cfg = AllocCfg(n_seqs, page_tokens, n_pages, max_pages, window)
    lens = np.ascontiguousarray(lengths, np.uint32)
    bt = np.empty((n_seqs, max_pages), np.int32)
    owner = np.empty((n_pages, page_tokens), np.uint64)
    events = (EvictEvent * max_events)()
    n_ev = C.c_uint32(0)
    last = np.empty(n_seqs, np.uint32)
    n_free = C.c_uint32(0)
    rc = port().orc_alloc_replay(C.byref(cfg), ptr(lens), ptr(bt), ptr(owner), C.cast(events, C.c_void_p),
                                 max_events, C.cast(C.pointer(n_ev), C.c_void_p), ptr(last),
                                 C.cast(C.pointer(n_free), C.c_void_p))
    ev = [(e.round, e.seq, e.lpage, e.phys, e.reason) for e in events[:n_ev.value]]
    return rc, bt, owner, ev, last, n_free.value


def compact_plan(bt):
    bt = np.array(bt, np.int32, copy=True)
    m = np.empty(bt.size, np.int32)
    n = port().orc_compact_plan(ptr(bt), bt.shape[0], bt.shape[1], ptr(m))
    return bt, m[:n]


def lpt(lengths, n_ranks):
    lens = np.ascontiguousarray(lengths, np.uint32)
    out = np.empty(len(lens), np.int32)
    port().orc_lpt_assign(ptr(lens), len(lens), n_ranks, ptr(out))
    return out
