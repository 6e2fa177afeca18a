"""A minimal GGUF v2/v3 writer for the tests: the layout the reference's
parser reads (gguf.js:146-183): magic, version, tensor count, metadata
count, typed metadata, tensor infos, padding to the alignment, then each
tensor's bytes at an aligned offset inside the data section."""
from __future__ import annotations

import struct
from typing import List, Sequence, Tuple

import numpy as np

U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_FMT = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<B", U64: "<Q",
        I64: "<q", F64: "<d"}


def _str(s: str) -> bytes:
    b = s.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def _value(t: int, v) -> bytes:
    if t == STRING:
        return _str(v)
    if t == ARRAY:
        et, items = v
        return struct.pack("<IQ", et, len(items)) + b"".join(_value(et, x) for x in items)
    return struct.pack(_FMT[t], int(v) if t not in (F32, F64) else float(v))


def write_gguf(path: str, metadata: Sequence[Tuple[str, int, object]],
               tensors: Sequence[Tuple[str, Sequence[int], int, bytes]], version: int = 3, alignment: int = 32,
               truncate: int = 0) -> None:
    """metadata: (key, type, value), arrays as (ARRAY, (elem_type, items));
    tensors: (name, dims, ggml_type, raw bytes).  `truncate` drops that many
    bytes from the end (for error tests)."""
    head = struct.pack("<IIQQ", 0x46554747, version, len(tensors), len(metadata))
    for k, t, v in metadata:
        head += _str(k) + struct.pack("<I", t) + _value(t, v)
    offs: List[int] = []
    rel = 0
    for name, dims, gt, raw in tensors:
        rel = (rel + alignment - 1) // alignment * alignment
        offs.append(rel)
        rel += len(raw)
    for (name, dims, gt, raw), off in zip(tensors, offs):
        head += _str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        head += struct.pack("<IQ", gt, off)
    start = (len(head) + alignment - 1) // alignment * alignment
    body = bytearray(rel)
    for (name, dims, gt, raw), off in zip(tensors, offs):
        body[off:off + len(raw)] = raw
    data = head + b"\0" * (start - len(head)) + bytes(body)
    if truncate:
        data = data[:-truncate]
    with open(path, "wb") as f:
        f.write(data)


def llama_metadata(dim, hidden, layers, heads, kv_heads, ctx_len, vocab, theta=10000.0, eps=1e-5, arch="llama",
                   extra=()):
    """The llama.* keys extractConfig reads, and a token list of `vocab` entries."""
    md = [("general.architecture", STRING, arch), ("general.name", STRING, "test-model"),
          (f"{arch}.embedding_length", U32, dim), (f"{arch}.feed_forward_length", U32, hidden),
          (f"{arch}.block_count", U32, layers), (f"{arch}.attention.head_count", U32, heads),
          (f"{arch}.attention.head_count_kv", U32, kv_heads), (f"{arch}.context_length", U32, ctx_len),
          (f"{arch}.attention.layer_norm_rms_epsilon", F32, eps), (f"{arch}.rope.freq_base", F32, theta),
          ("tokenizer.ggml.model", STRING, "llama"),
          ("tokenizer.ggml.tokens", ARRAY, (STRING, [f"tok{i}" for i in range(vocab)])),
          ("tokenizer.ggml.bos_token_id", U32, 1), ("tokenizer.ggml.eos_token_id", U32, 2)]
    return md + list(extra)


def f32_bytes(a) -> bytes:
    return np.ascontiguousarray(a, np.float32).tobytes()
