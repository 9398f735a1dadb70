"""A tiny llama-style model as a GGUF v3 file (public GGUF layout: header,
metadata key/values, tensor infos, 32-byte aligned tensor data), for
driving the reference engine's transformer.c against the library.  Weights
are seeded normals (the oracle's SplitMix64 / Box-Muller stream), F32."""
from __future__ import annotations

import struct

import numpy as np

import oracle

# GGUF metadata value types (public spec)
U32, F32, STR = 4, 6, 8

CFG = dict(n_layers=2, n_embd=64, n_head=8, n_head_kv=2, n_ff=96, n_vocab=40, ctx=64)


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def write_tiny_llama(path, seed=7, **over):
    c = dict(CFG, **over)
    E, V, F, L = c["n_embd"], c["n_vocab"], c["n_ff"], c["n_layers"]
    kvd = c["n_head_kv"] * (E // c["n_head"])
    meta = [("general.architecture", STR, "llama"), ("llama.block_count", U32, L), ("llama.embedding_length", U32, E),
            ("llama.attention.head_count", U32, c["n_head"]), ("llama.attention.head_count_kv", U32, c["n_head_kv"]),
            ("llama.context_length", U32, c["ctx"]), ("llama.vocab_size", U32, V),
            ("llama.feed_forward_length", U32, F), ("llama.rope.freq_base", F32, 10000.0)]
    # (name, dims as ne0 (input, contiguous), ne1 (output)); norms are 1-D
    tensors = [("token_embd.weight", (E, V)), ("output_norm.weight", (E,)), ("output.weight", (E, V))]
    for l in range(L):
        tensors += [(f"blk.{l}.attn_norm.weight", (E,)), (f"blk.{l}.attn_q.weight", (E, E)),
                    (f"blk.{l}.attn_k.weight", (E, kvd)), (f"blk.{l}.attn_v.weight", (E, kvd)),
                    (f"blk.{l}.attn_output.weight", (E, E)), (f"blk.{l}.ffn_norm.weight", (E,)),
                    (f"blk.{l}.ffn_gate.weight", (E, F)), (f"blk.{l}.ffn_up.weight", (E, F)),
                    (f"blk.{l}.ffn_down.weight", (F, E))]
    key = oracle.key(seed, 77)
    data, infos, off, start = [], [], 0, 0
    for name, dims in tensors:
        n = int(np.prod(dims))
        x = oracle.normal_f32(key, start, n)
        start += n
        x = (1.0 + 0.1 * x) if len(dims) == 1 else x * np.float32(1.0 / np.sqrt(dims[0]))
        raw = np.ascontiguousarray(x, np.float32).tobytes()
        infos.append((name, dims, off))
        data.append(raw)
        off += (len(raw) + 31) // 32 * 32
    out = bytearray()
    out += struct.pack("<IIQQ", 0x46554747, 3, len(tensors), len(meta))
    for k, t, v in meta:
        out += _str(k) + struct.pack("<I", t)
        out += _str(v) if t == STR else struct.pack("<I", v) if t == U32 else struct.pack("<f", v)
    for name, dims, o in infos:
        out += _str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        out += struct.pack("<IQ", 0, o)                   # type F32, offset within the data section
    out += b"\0" * ((32 - len(out) % 32) % 32)
    for raw in data:                                      # offsets above are these 32-byte padded runs
        out += raw + b"\0" * ((32 - len(raw) % 32) % 32)
    open(path, "wb").write(bytes(out))
    return c
