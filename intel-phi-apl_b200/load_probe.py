"""Times the weight loader (rt_b200_load_gguf) on a synthetic GGUF file of the decode shapes:

    python intel-phi-apl_b200/load_probe.py [--layers 4] [--dir /tmp]

writes `layers` decode layers (QKV, out, gate, up, down; Q8_0, random quants and fp16 scales) plus
the 151936 x 4096 head to a GGUF file, loads it into HBM (O_DIRECT reads into pinned buffers,
copies overlapping the reads, the file's sum and the in-place repacks on the GPU) and prints one
JSON line: bytes, seconds, GB/s, the repack's share and whether the reads bypassed the page cache.
The reference measures its own load at 3.05-3.29 GB/s for the transfer and 9.27 GB/s for the
repack (its docs/measurements.md).
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

import gguf_synth as G  # noqa: E402
import rtb200  # noqa: E402
import workload as WL  # noqa: E402


def q8_bytes(rows: int, cols: int, rng) -> bytes:
    blocks = rows * cols // 32
    raw = np.empty((blocks, 34), dtype=np.uint8)
    raw[:, 2:] = rng.integers(0, 256, size=(blocks, 32), dtype=np.uint8)
    d = (rng.random(blocks, dtype=np.float32) * 1e-3 + 1e-4).astype(np.float16)
    raw[:, :2] = d.view(np.uint8).reshape(blocks, 2)
    return raw.tobytes()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--dir", default="/tmp")
    a = ap.parse_args()
    import torch
    rng = np.random.default_rng(1)
    tensors = []
    for L in range(a.layers):
        for name, rows, cols in (("attn_qkv", WL.QKV, WL.D), ("attn_output", WL.D, WL.D), ("ffn_gate", WL.FF, WL.D),
                                 ("ffn_up", WL.FF, WL.D), ("ffn_down", WL.D, WL.FF)):
            tensors.append((f"blk.{L}.{name}.weight", G.GGML_Q8_0, [cols, rows], q8_bytes(rows, cols, rng)))
    tensors.append(("output.weight", G.GGML_Q8_0, [WL.D, WL.VOCAB], q8_bytes(WL.VOCAB, WL.D, rng)))
    path = os.path.join(a.dir, "rtb_load_probe.gguf")
    G.write_gguf(path, tensors, kv={"general.architecture": "qwen35"})
    size = os.path.getsize(path)
    arena = torch.empty((size + 4095) // 4096 * 4096, dtype=torch.uint8, device="cuda")
    with rtb200.Runtime() as rt:
        rt.load_gguf(path, arena.data_ptr(), arena.numel())  # warm-up (driver, pinned buffers)
        table, st = rt.load_gguf(path, arena.data_ptr(), arena.numel())
    ok = st["file_sum"] == G.file_sum(path)
    os.remove(path)
    print(json.dumps({"file_bytes": size, "seconds": round(st["seconds"], 4), "GB_s": round(size / st["seconds"] / 1e9, 2),
                      "repack_seconds": round(st["seconds_repack"], 5),
                      "repack_GB_s": round(size / st["seconds_repack"] / 1e9, 1) if st["seconds_repack"] else None,
                      "o_direct": bool(st["direct"]), "q8_matrices": st["q8_matrices"], "sum_ok": ok,
                      "tensors": len(table)}))


if __name__ == "__main__":
    main()
