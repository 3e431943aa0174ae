"""A minimal GGUF (version 3) writer, for the loader's tests and its probe: metadata keys of the
common value types, tensor infos, tensor data at `general.alignment` boundaries. The format is
llama.cpp's GGUF; the values are whatever the caller passes.

    write_gguf(path, [("blk.0.attn_q.weight", GGML_Q8_0, [4096, 4096], q8_bytes), ...],
               kv={"general.architecture": "qwen35"})
"""
from __future__ import annotations

import struct

import numpy as np

GGML_F32, GGML_F16, GGML_Q8_0, GGML_BF16 = 0, 1, 8, 30
_U32, _U64, _F32, _STR, _ARR = 4, 10, 6, 8, 9


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(v) -> bytes:
    if isinstance(v, bool) or isinstance(v, int):
        return struct.pack("<I", _U32) + struct.pack("<I", int(v)) if 0 <= int(v) < 2 ** 32 else \
            struct.pack("<I", _U64) + struct.pack("<Q", int(v))
    if isinstance(v, float):
        return struct.pack("<I", _F32) + struct.pack("<f", v)
    if isinstance(v, str):
        return struct.pack("<I", _STR) + _str(v)
    if isinstance(v, (list, tuple)):
        if all(isinstance(e, str) for e in v):
            return struct.pack("<I", _ARR) + struct.pack("<IQ", _STR, len(v)) + b"".join(_str(e) for e in v)
        return struct.pack("<I", _ARR) + struct.pack("<IQ", _U32, len(v)) + b"".join(struct.pack("<I", e) for e in v)
    raise TypeError(f"metadata value {v!r}")


def write_gguf(path: str, tensors: list, kv: dict | None = None, alignment: int = 32, shared: dict | None = None) -> list:
    """tensors: (name, ggml type, dims fastest-first, data bytes). shared: {name: other name} makes
    `name`'s tensor info point at `other`'s data (a tied matrix; its data argument is ignored).
    Returns each tensor's offset from the start of the file."""
    kv = dict(kv or {})
    kv["general.alignment"] = alignment
    shared = shared or {}
    rel, off, blobs = {}, 0, []
    for name, typ, dims, data in tensors:
        if name in shared:
            continue
        off = (off + alignment - 1) // alignment * alignment
        rel[name] = off
        blobs.append((off, bytes(data)))
        off += len(data)
    for name, other in shared.items():
        rel[name] = rel[other]
    head = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(kv))
    for k, v in kv.items():
        head += _str(k) + _value(v)
    for name, typ, dims, _ in tensors:
        head += _str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        head += struct.pack("<IQ", typ, rel[name])
    start = (len(head) + alignment - 1) // alignment * alignment
    with open(path, "wb") as f:
        f.write(head + b"\0" * (start - len(head)))
        pos = 0
        for o, b in blobs:
            f.write(b"\0" * (o - pos))
            f.write(b)
            pos = o + len(b)
        end = start + pos
        f.write(b"\0" * ((end + alignment - 1) // alignment * alignment - end))
    return [start + rel[name] for name, *_ in tensors]


def file_sum(path: str) -> int:
    """The file's position-weighted sum: sum of word_i * (2i + 1) mod 2^64 over its 8-byte words
    (a partial last word counts with zero bytes)."""
    raw = np.fromfile(path, dtype=np.uint8)
    pad = (-len(raw)) % 8
    w = np.concatenate([raw, np.zeros(pad, np.uint8)]).view(np.uint64)
    i = np.arange(len(w), dtype=np.uint64)
    with np.errstate(over="ignore"):
        return int(np.sum(w * (np.uint64(2) * i + np.uint64(1)), dtype=np.uint64))
