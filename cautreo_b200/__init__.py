"""cautreo_b200 -- the KV-cache / decode-attention hot path of Cautreo on B200.

The product is the C-ABI library ``libcautreo_b200.so`` (headers in
``include/``): the reference's ``ct_kv_*``, ``ct_attn_*``, ``ct_quant_*``,
``ct_hal_*`` and ``ct_dist_*`` interfaces plus the paged / MLA / per-token
codec entry points, all backed by sm_100a CUDA kernels.  This module loads
that library with ctypes, declares every signature, and offers thin Python
wrappers that tests and the benchmark call.  There is no Python or CPU
compute path: if the library is missing, :func:`lib` raises.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libcautreo_b200.so"

# ct_status_t
CT_OK, CT_ERR_ARG, CT_ERR_CUDA, CT_ERR_NOMEM, CT_ERR_FULL, CT_ERR_UNMAPPED, CT_ERR_UNSUPPORTED, CT_ERR_IO = (
    0, -1, -2, -3, -4, -5, -6, -7)
# ct_kv_dtype_t
CT_KV_BF16, CT_KV_F32, CT_KV_INT8, CT_KV_E4M3 = 0, 1, 2, 3
CT_KV_Q8_0, CT_KV_Q4_0, CT_KV_Q2_0, CT_KV_Q1_0 = 4, 5, 6, 7      # block codecs of quant.h, 32 values per block
BLOCK_BYTES = {CT_KV_Q8_0: 34, CT_KV_Q4_0: 18, CT_KV_Q2_0: 10, CT_KV_Q1_0: 6}


def entry_bytes(dtype: int, dim: int) -> int:
    """Bytes of one token's entry in a pool of `dtype`."""
    if dtype in BLOCK_BYTES:
        return dim // 32 * BLOCK_BYTES[dtype]
    return dim * {CT_KV_BF16: 2, CT_KV_F32: 4, CT_KV_INT8: 1, CT_KV_E4M3: 1}[dtype]
# ct_quant_type_t
CT_QUANT_FP16, CT_QUANT_Q8_0, CT_QUANT_Q4_0, CT_QUANT_Q2_0, CT_QUANT_Q1_0 = 0, 1, 2, 3, 4
QUANT_BLOCK_BYTES = {CT_QUANT_Q8_0: 34, CT_QUANT_Q4_0: 18, CT_QUANT_Q2_0: 10, CT_QUANT_Q1_0: 6}


class KvConfig(C.Structure):
    """ct_kv_config_t (kv_cache.h:22-28)."""
    _fields_ = [("n_layers", C.c_uint32), ("n_kv_heads", C.c_uint32), ("head_dim", C.c_uint32),
                ("max_ctx", C.c_uint32), ("compress_ratio", C.c_float)]


class KvStats(C.Structure):
    """ct_kv_stats_t (kv_cache.h:59-64)."""
    _fields_ = [("n_appends", C.c_uint64), ("n_reads", C.c_uint64), ("bytes_used", C.c_uint64),
                ("n_tokens", C.c_uint32)]


class PagedConfig(C.Structure):
    _fields_ = [("n_seqs", C.c_uint32), ("max_pages_per_seq", C.c_uint32), ("n_pages", C.c_uint32),
                ("page_tokens", C.c_uint32), ("entry_dim", C.c_uint32), ("window_tokens", C.c_uint32),
                ("dtype", C.c_uint32), ("device", C.c_int32)]


class PagedStats(C.Structure):
    _fields_ = [("n_appends", C.c_uint64), ("n_evict_window", C.c_uint64), ("n_evict_lru", C.c_uint64),
                ("n_compactions", C.c_uint64), ("bytes_compacted", C.c_uint64), ("n_pages_live", C.c_uint32),
                ("n_pages_free", C.c_uint32), ("clock", C.c_uint64)]


class EvictEvent(C.Structure):
    _fields_ = [("round", C.c_uint32), ("seq", C.c_uint32), ("lpage", C.c_uint32), ("phys", C.c_int32),
                ("reason", C.c_uint32)]


class MlaShape(C.Structure):
    _fields_ = [("n_heads", C.c_uint32), ("entry_dim", C.c_uint32), ("v_dim", C.c_uint32),
                ("page_tokens", C.c_uint32), ("max_pages_per_seq", C.c_uint32), ("kv_dtype", C.c_uint32),
                ("scale", C.c_float), ("n_pages", C.c_uint32)]


class Scorecard(C.Structure):
    """ct_hardware_scorecard_t (hal.h:116-145)."""
    _fields_ = [("ram_total_bytes", C.c_uint64), ("ram_avail_bytes", C.c_uint64),
                ("ram_model_budget", C.c_uint64), ("cpu_cores_physical", C.c_uint32),
                ("cpu_cores_logical", C.c_uint32), ("cpu_simd", C.c_int), ("cpu_ghz", C.c_double),
                ("gpu_present", C.c_bool), ("gpu_type", C.c_int), ("gpu_vram_bytes", C.c_uint64),
                ("ssd_type", C.c_int), ("ssd_read_mbps", C.c_double), ("ssd_read_iops", C.c_double),
                ("suggested_strategy", C.c_int), ("model_size_bytes", C.c_uint64),
                ("model_n_params", C.c_uint64), ("model_is_moe", C.c_bool)]


P, F, U32, I32, U64, I64, SZ, B, V, I = (C.c_void_p, C.c_float, C.c_uint32, C.c_int32, C.c_uint64, C.c_int64,
                                          C.c_size_t, C.c_bool, None, C.c_int)
CCP = C.c_char_p

# name: (restype, [argtypes])
SIGNATURES = {
    # kv_cache.h part 1
    "ct_kv_create": (P, [C.POINTER(KvConfig)]),
    "ct_kv_destroy": (V, [P]),
    "ct_kv_append": (B, [P, U32, U32, P, P]),
    "ct_kv_get": (B, [P, U32, U32, P, P]),
    "ct_kv_len": (U32, [P]),
    "ct_kv_capacity": (U32, [P]),
    "ct_kv_reset": (V, [P]),
    "ct_kv_save": (B, [P, CCP]),
    "ct_kv_load": (B, [P, CCP]),
    "ct_kv_compress": (B, [P, F]),
    "ct_kv_stats": (KvStats, [P]),
    "ct_kv_device_k": (P, [P]),
    "ct_kv_device_v": (P, [P]),
    # kv_cache.h part 2
    "ct_kv_paged_create": (P, [C.POINTER(PagedConfig)]),
    "ct_kv_paged_destroy": (V, [P]),
    "ct_kv_paged_set_stream": (I, [P, P]),
    "ct_kv_paged_set_free_order": (I, [P, P]),
    "ct_kv_paged_append": (I, [P, P, P, U32, P, U32]),
    "ct_kv_paged_free_seq": (I, [P, U32]),
    "ct_kv_paged_append_projected": (I, [P, P, P, U32, P, P, U32, P, F, U32]),
    "ct_kv_project_write_slots": (I, [P, P, P, F, U32, U32, U32, U32, P, P, U32, P, P]),
    "ct_kv_project_error": (I, [I]),
    "ct_kv_paged_set_tokens": (I, [P, U32, U32, P, U32]),
    "ct_kv_paged_tokens": (U32, [P, U32, P, U32]),
    "ct_kv_paged_match_prefix": (I, [P, P, U32, P, P]),
    "ct_ds4_cache_create": (P, [U32, U32, U32, I]),
    "ct_ds4_cache_destroy": (V, [P]),
    "ct_ds4_cache_len": (U32, [P, U32]),
    "ct_ds4_attend": (I, [P, U32, U32, P, P, P]),
    "ct_kv_paged_evict_lru": (I, [P, U32]),
    "ct_kv_paged_compact": (I, [P]),
    "ct_kv_paged_gather": (I, [P, U32, U32, U32, P, U32]),
    "ct_kv_paged_gather_batch": (I, [P, P, P, P, U32, P, U32]),
    "ct_kv_paged_save": (I, [P, C.c_char_p]),
    "ct_kv_paged_fork": (I, [P, U32, U32, U32]),
    "ct_kv_paged_page_refs": (U32, [P, I32]),
    "ct_kv_paged_load": (P, [C.c_char_p, C.c_int]),
    "ct_kv_paged_block_table": (I, [P, P]),
    "ct_kv_paged_seq_lens": (I, [P, P]),
    "ct_kv_paged_last_access": (I, [P, P]),
    "ct_kv_paged_evict_log": (U32, [P, P, U32]),
    "ct_kv_paged_stats": (PagedStats, [P]),
    "ct_kv_paged_config": (C.POINTER(PagedConfig), [P]),
    "ct_kv_paged_pool": (P, [P]),
    "ct_kv_paged_scales": (P, [P]),
    "ct_kv_paged_block_table_dev": (P, [P]),
    "ct_kv_paged_seq_lens_dev": (P, [P]),
    "ct_kv_paged_write_slots": (I, [P, P, U32, P, U32, P, U32, U32, P]),
    "ct_kv_paged_move_pages": (I, [P, P, P, P, P, U32, SZ, U32, P]),
    # attention.h
    "ct_attn_forward": (B, [P, P, P, U32, U32, U32, F, P]),
    "ct_attn_forward_kv": (B, [P, P, P, U32, U32, U32, F, P]),
    "ct_attn_softmax": (V, [P, U32]),
    "ct_attn_decode_contig": (I, [P, P, P, U32, U32, U32, U32, U32, U32, F, P, P]),
    "ct_attn_decode_step_contig": (I, [P, P, P, P, P, U32, U32, U32, U32, U32, U32, F, P, P]),
    "ct_mla_plan_create": (P, [C.POINTER(MlaShape), P, P, U32, I]),
    "ct_mla_plan_destroy": (V, [P]),
    "ct_mla_plan_chunks": (U32, [P]),
    "ct_mla_plan_scratch_bytes": (SZ, [P]),
    "ct_attn_mla_decode_paged": (I, [P, P, P, P, P, P, P, P, P]),
    "ct_mla_plan_launches": (U32, [P]),
    "ct_mla_plan_workers": (U32, [P]),
    "ct_mla_plan_tensor_cores": (I, [P]),
    "ct_attn_mla_decode_step_host": (I, [P, P, P, P, P, P, P, P, P, P]),
    "ct_attn_mla_decode_paged_noalloc": (I, [C.POINTER(MlaShape), P, U32, P, P, P, P, P, P, P, P]),
    "ct_mla_tc_error": (I, [I]),
    # quant.h
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
    "ct_quant_kv_int8": (I, [P, I, U32, U32, P, P, P]),
    "ct_quant_kv_e4m3": (I, [P, I, U32, U32, P, P, P]),
    "ct_dequant_kv_int8": (I, [P, P, U32, U32, P, P]),
    "ct_dequant_kv_e4m3": (I, [P, P, U32, U32, P, P]),
    "ct_quant_q8_0_dev": (I, [P, P, I64, P]),
    "ct_dequant_q8_0_dev": (I, [P, P, I64, P]),
    # hal.h
    "ct_hal_detect": (C.POINTER(Scorecard), []),
    "ct_hal_redetect": (C.POINTER(Scorecard), []),
    "ct_hal_set_model": (I, [U64, U64, B]),
    "ct_hal_set_ram_budget": (I, [U64]),
    "ct_hal_get": (C.POINTER(Scorecard), []),
    "ct_hal_print": (V, [C.POINTER(Scorecard)]),
    "ct_hal_cuda_device_count": (I, []),
    "ct_hal_cuda_set_device": (I, [I]),
    "ct_hal_cuda_device_info": (I, [I, C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_uint64)]),
    "ct_hal_cuda_alloc": (P, [SZ]),
    "ct_hal_cuda_free": (V, [P]),
    "ct_hal_cuda_alloc_host": (P, [SZ]),
    "ct_hal_cuda_free_host": (V, [P]),
    "ct_hal_cuda_memcpy": (I, [P, P, SZ, I, P]),
    "ct_hal_cuda_memset": (I, [P, I, SZ, P]),
    "ct_hal_cuda_stream_create": (P, []),
    "ct_hal_cuda_stream_destroy": (V, [P]),
    "ct_hal_cuda_stream_sync": (I, [P]),
    "ct_hal_cuda_device_sync": (I, []),
    "ct_hal_cuda_event_create": (P, []),
    "ct_hal_cuda_event_destroy": (V, [P]),
    "ct_hal_cuda_event_record": (I, [P, P]),
    "ct_hal_cuda_event_elapsed_ms": (F, [P, P]),
    "ct_hal_cuda_last_error": (CCP, []),
    "ct_hal_cuda_launch_count": (U64, []),
    "ct_hal_version": (CCP, []),
    # distributed.h
    "ct_dist_init": (P, [P]),
    "ct_dist_destroy": (V, [P]),
    "ct_dist_n_devices": (U32, [P]),
    "ct_dist_device_id": (U32, [P]),
    "ct_dist_is_leader": (B, [P]),
    "ct_dist_allreduce": (B, [P, P, SZ]),
    "ct_dist_broadcast": (B, [P, P, SZ, U32]),
    "ct_dist_send": (B, [P, P, SZ, U32]),
    "ct_dist_recv": (B, [P, P, SZ, U32]),
    "ct_dist_available_memory": (U64, [P, U32]),
    "ct_dist_shard_lpt": (I, [P, U32, U32, P]),
    "ct_dist_rank_sequences": (U32, [P, U32, U32, P]),
    "ct_dist_nccl_unique_id": (I, [P]),
    "ct_dist_init_nccl": (P, [P, P, I]),
    "ct_dist_gather_rows": (I, [P, P, U32, SZ, P, U32, P, P]),
    "ct_dist_gather_stats": (I, [P, P, P]),
    # synth.h
    "ct_synth_key": (U64, [U64, U64]),
    "ct_synth_fill": (I, [P, U32, U64, U64, U64, U32, F, P]),
    "ct_synth_fill_paged": (I, [P, P, U32, P, U32, P, P, U32, U32, U32, U32, U64, U32, F, P]),
}

_LIB = None


def lib() -> C.CDLL:
    """Load libcautreo_b200.so (built by ``python -m cautreo_b200.build``)."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: run `python -m cautreo_b200.build` (no CPU fallback exists)")
        L = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def check(rc: int, what: str = "") -> None:
    """Raise on a negative ct_status_t."""
    if rc < 0:
        raise RuntimeError(f"{what} failed: status {rc}: {lib().ct_hal_cuda_last_error().decode()}")


def ptr(a) -> int:
    """Address of a numpy array, torch tensor, or int."""
    if a is None:
        return None
    if isinstance(a, int):
        return a
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    return a.data_ptr()


def launch_count() -> int:
    return int(lib().ct_hal_cuda_launch_count())


# ---- thin wrappers ----------------------------------------------------------

class KvCache:
    """ct_kv_* handle (contiguous fp32 cache in HBM)."""

    def __init__(self, n_layers, n_kv_heads, head_dim, max_ctx=0, compress_ratio=1.0):
        self.cfg = KvConfig(n_layers, n_kv_heads, head_dim, max_ctx, compress_ratio)
        self.h = lib().ct_kv_create(C.byref(self.cfg))
        if not self.h:
            raise RuntimeError("ct_kv_create failed: " + lib().ct_hal_cuda_last_error().decode())
        self.stride = n_kv_heads * head_dim

    def close(self):
        if self.h:
            lib().ct_kv_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except (TypeError, AttributeError):   # interpreter shutdown: module globals already cleared
            pass

    def append(self, layer, pos, k, v) -> bool:
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        return bool(lib().ct_kv_append(self.h, layer, pos, ptr(k), ptr(v)))

    def get(self, layer, pos):
        k = np.zeros(self.stride, np.float32)
        v = np.zeros(self.stride, np.float32)
        ok = lib().ct_kv_get(self.h, layer, pos, ptr(k), ptr(v))
        return (k, v) if ok else None

    def __len__(self):
        return int(lib().ct_kv_len(self.h))


class PagedKV:
    """ct_kv_paged_* handle."""

    def __init__(self, n_seqs, max_pages_per_seq, n_pages, page_tokens=64, entry_dim=576, window_tokens=0,
                 dtype=CT_KV_BF16, device=0, stream=None, _handle=None):
        self.cfg = PagedConfig(n_seqs, max_pages_per_seq, n_pages, page_tokens, entry_dim, window_tokens, dtype,
                               device)
        self.h = _handle if _handle is not None else lib().ct_kv_paged_create(C.byref(self.cfg))
        if not self.h:
            raise RuntimeError("ct_kv_paged_create failed: " + lib().ct_hal_cuda_last_error().decode())
        if stream is not None:
            check(lib().ct_kv_paged_set_stream(self.h, stream), "set_stream")

    def fork(self, src, dst, n_tokens):
        check(lib().ct_kv_paged_fork(self.h, src, dst, n_tokens), "ct_kv_paged_fork")

    def page_refs(self, page):
        return int(lib().ct_kv_paged_page_refs(self.h, page))

    def save(self, path):
        check(lib().ct_kv_paged_save(self.h, str(path).encode()), "ct_kv_paged_save")

    @classmethod
    def load(cls, path, device=0, stream=None):
        h = lib().ct_kv_paged_load(str(path).encode(), device)
        if not h:
            raise RuntimeError("ct_kv_paged_load failed: " + lib().ct_hal_cuda_last_error().decode())
        c = lib().ct_kv_paged_config(h).contents
        return cls(c.n_seqs, c.max_pages_per_seq, c.n_pages, c.page_tokens, c.entry_dim, c.window_tokens, c.dtype,
                   device, stream, _handle=h)

    def close(self):
        if self.h:
            lib().ct_kv_paged_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except (TypeError, AttributeError):   # interpreter shutdown: module globals already cleared
            pass

    def set_free_order(self, order):
        order = np.ascontiguousarray(order, np.int32)
        check(lib().ct_kv_paged_set_free_order(self.h, ptr(order)), "set_free_order")

    def append(self, seq_ids, counts, entries=None, src_dtype=CT_KV_BF16):
        seq_ids = np.ascontiguousarray(seq_ids, np.uint32)
        counts = np.ascontiguousarray(counts, np.uint32)
        rc = lib().ct_kv_paged_append(self.h, ptr(seq_ids), ptr(counts), len(seq_ids), ptr(entries), src_dtype)
        check(rc, "ct_kv_paged_append")

    def block_table(self):
        out = np.zeros((self.cfg.n_seqs, self.cfg.max_pages_per_seq), np.int32)
        check(lib().ct_kv_paged_block_table(self.h, ptr(out)))
        return out

    def gather(self, seq, start, n, out, out_dtype=CT_KV_BF16):
        """Tokens [start, start+n) of `seq` into device rows `out`."""
        check(lib().ct_kv_paged_gather(self.h, seq, start, n, ptr(out), out_dtype), "ct_kv_paged_gather")

    def gather_batch(self, seqs, starts, counts, out, out_dtype=CT_KV_BF16):
        """Several (seq, start, count) ranges, back to back, in one launch."""
        seqs, starts, counts = (np.ascontiguousarray(a, np.uint32) for a in (seqs, starts, counts))
        check(lib().ct_kv_paged_gather_batch(self.h, ptr(seqs), ptr(starts), ptr(counts), len(seqs), ptr(out),
                                              out_dtype), "ct_kv_paged_gather_batch")

    def append_projected(self, seq_ids, counts, x, w, n_in, norm_w=None, eps=1e-6, norm_dim=0):
        """Append tokens whose entries are W . x (+ RMS norm), computed on the device."""
        seq_ids = np.ascontiguousarray(seq_ids, np.uint32)
        counts = np.ascontiguousarray(counts, np.uint32)
        check(lib().ct_kv_paged_append_projected(self.h, ptr(seq_ids), ptr(counts), len(seq_ids), ptr(x), ptr(w),
                                                 n_in, ptr(norm_w), eps, norm_dim), "ct_kv_paged_append_projected")

    def set_tokens(self, seq, start, ids):
        ids = np.ascontiguousarray(ids, np.int32)
        check(lib().ct_kv_paged_set_tokens(self.h, seq, start, ptr(ids), len(ids)), "ct_kv_paged_set_tokens")

    def tokens(self, seq):
        n = int(lib().ct_kv_paged_tokens(self.h, seq, None, 0))
        out = np.zeros(n, np.int32)
        lib().ct_kv_paged_tokens(self.h, seq, ptr(out), n)
        return out

    def match_prefix(self, ids):
        """(seq, length) of the longest cached prefix of ids."""
        ids = np.ascontiguousarray(ids, np.int32)
        s, n = C.c_uint32(0), C.c_uint32(0)
        check(lib().ct_kv_paged_match_prefix(self.h, ptr(ids), len(ids), C.byref(s), C.byref(n)),
              "ct_kv_paged_match_prefix")
        return int(s.value), int(n.value)

    def free_seq(self, seq):
        check(lib().ct_kv_paged_free_seq(self.h, seq), "ct_kv_paged_free_seq")

    def compact(self):
        check(lib().ct_kv_paged_compact(self.h), "ct_kv_paged_compact")

    def seq_lens(self):
        out = np.zeros(self.cfg.n_seqs, np.uint32)
        check(lib().ct_kv_paged_seq_lens(self.h, ptr(out)))
        return out

    def last_access(self):
        out = np.zeros(self.cfg.n_seqs, np.uint64)
        check(lib().ct_kv_paged_last_access(self.h, ptr(out)))
        return out

    def evict_log(self):
        n = lib().ct_kv_paged_evict_log(self.h, None, 0)
        arr = (EvictEvent * max(n, 1))()
        n = lib().ct_kv_paged_evict_log(self.h, C.cast(arr, C.c_void_p), n)
        return [(e.round, e.seq, e.lpage, e.phys, e.reason) for e in arr[:n]]

    def stats(self) -> PagedStats:
        return lib().ct_kv_paged_stats(self.h)

    @property
    def pool(self):
        return lib().ct_kv_paged_pool(self.h)

    @property
    def scales(self):
        return lib().ct_kv_paged_scales(self.h)

    @property
    def block_table_dev(self):
        return lib().ct_kv_paged_block_table_dev(self.h)

    @property
    def seq_lens_dev(self):
        return lib().ct_kv_paged_seq_lens_dev(self.h)


class MlaPlan:
    """ct_mla_plan_t for a fixed set of sequence lengths."""

    def __init__(self, seq_lens, n_pages, n_heads=128, entry_dim=576, v_dim=512, page_tokens=64,
                 max_pages_per_seq=None, kv_dtype=CT_KV_BF16, scale=None, seq_rows=None, device=0):
        seq_lens = np.ascontiguousarray(seq_lens, np.int32)
        if max_pages_per_seq is None:
            max_pages_per_seq = int(max(1, (int(seq_lens.max(initial=0)) + page_tokens - 1) // page_tokens))
        if scale is None:
            scale = 1.0 / np.sqrt(192.0)
        self.shape = MlaShape(n_heads, entry_dim, v_dim, page_tokens, max_pages_per_seq, kv_dtype, scale, n_pages)
        rows = None if seq_rows is None else np.ascontiguousarray(seq_rows, np.uint32)
        self._rows = rows
        self.n_seq = len(seq_lens)
        self.h = lib().ct_mla_plan_create(C.byref(self.shape), ptr(rows), ptr(seq_lens), self.n_seq, device)
        if not self.h:
            raise RuntimeError("ct_mla_plan_create failed: " + lib().ct_hal_cuda_last_error().decode())

    def close(self):
        if self.h:
            lib().ct_mla_plan_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except (TypeError, AttributeError):   # interpreter shutdown: module globals already cleared
            pass

    @property
    def n_chunks(self):
        return int(lib().ct_mla_plan_chunks(self.h))

    @property
    def launches(self):
        return int(lib().ct_mla_plan_launches(self.h))

    @property
    def workers(self):
        return int(lib().ct_mla_plan_workers(self.h))

    @property
    def tensor_cores(self):
        return bool(lib().ct_mla_plan_tensor_cores(self.h))

    def decode(self, q, pool, scales, block_table, seq_lens, out, lse=None, stream=None):
        rc = lib().ct_attn_mla_decode_paged(self.h, ptr(q), ptr(pool), ptr(scales), ptr(block_table),
                                            ptr(seq_lens), ptr(out), ptr(lse), stream)
        check(rc, "ct_attn_mla_decode_paged")

    def step_host(self, q_host, entries_host, dest_slot, pool, scales, block_table, seq_lens, out_host,
                  stream=None):
        """One step with host buffers (ct_attn_mla_decode_step_host): append
        entries_host at dest_slot (device; None skips), decode, fill out_host."""
        rc = lib().ct_attn_mla_decode_step_host(self.h, ptr(q_host), ptr(entries_host), ptr(dest_slot), ptr(pool),
                                                ptr(scales), ptr(block_table), ptr(seq_lens), ptr(out_host),
                                                stream)
        check(rc, "ct_attn_mla_decode_step_host")


class DistConfig(C.Structure):
    _fields_ = [("mode", C.c_int), ("n_devices", C.c_uint32), ("device_id", C.c_uint32), ("device_names", C.c_void_p)]


class DistStats(C.Structure):
    _fields_ = [("kv_tokens", C.c_uint64), ("bytes", C.c_uint64), ("decode_us", C.c_double), ("error", C.c_int32),
                ("n_seqs", C.c_uint32)]


class NcclContext:
    """ct_dist_init_nccl: an NCCL communicator over world processes, one GPU
    each; `uid` is the 128-byte id rank 0 made with nccl_unique_id()."""

    def __init__(self, rank, world, uid, device):
        self.cfg = DistConfig(0, world, rank, None)
        buf = (C.c_uint8 * 128).from_buffer_copy(bytes(uid))
        self.h = lib().ct_dist_init_nccl(C.byref(self.cfg), buf, device)
        if not self.h:
            raise RuntimeError("ct_dist_init_nccl failed: " + lib().ct_hal_cuda_last_error().decode())
        self.rank, self.world = rank, world

    def gather_rows(self, rows, n_rows, row_bytes, global_ids, n_global, out, stream=None):
        ids = np.ascontiguousarray(global_ids, np.uint32)
        check(lib().ct_dist_gather_rows(self.h, ptr(rows), n_rows, row_bytes, ptr(ids), n_global, ptr(out), stream),
              "ct_dist_gather_rows")

    def gather_stats(self, mine):
        out = (DistStats * self.world)()
        check(lib().ct_dist_gather_stats(self.h, C.byref(mine), C.cast(out, C.c_void_p) if self.rank == 0 else None),
              "ct_dist_gather_stats")
        return list(out) if self.rank == 0 else None

    def close(self):
        if self.h:
            lib().ct_dist_destroy(self.h)
            self.h = None


def nccl_unique_id() -> bytes:
    buf = (C.c_uint8 * 128)()
    check(lib().ct_dist_nccl_unique_id(buf), "ct_dist_nccl_unique_id")
    return bytes(buf)


def lpt_shard(lengths, n_ranks):
    lengths = np.ascontiguousarray(lengths, np.uint32)
    out = np.zeros(len(lengths), np.int32)
    check(lib().ct_dist_shard_lpt(ptr(lengths), len(lengths), n_ranks, ptr(out)), "ct_dist_shard_lpt")
    return out


def synth_key(seed, stream):
    return int(lib().ct_synth_key(seed, stream))
