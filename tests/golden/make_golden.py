"""Makes the committed golden fixtures of this directory from the reference itself.

    make -C oracle && python tests/golden/make_golden.py

Needs the reference source tree ($REF_ROOT, by default a checkout named `reference` beside this
repository) and oracle/_ref/libq8ref.so, the
reference's own host-model kernels compiled from its sources by oracle/Makefile. Writes:

* ref_gates.json -- the reference's golden known answers for the up-conversions, fma and tree
  sum the Q8_0 product is built from (tests/golden/gate-2.1.txt and gate-a.txt of the reference),
  parsed into JSON;
* ref_vectors.npz -- for a set of seeded Q8_0 products, the y the reference's gemv_i_thread /
  gemm_i_thread computes (as uint32 bit patterns), with sha256 digests of the exact input bytes
  (the GGUF Q8_0 weights and the fp32 x) so the generator that rebuilds them is pinned too. The
  smallest cases also carry their input bytes outright.

The GPU host has no reference tree: tests read only these fixtures there.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle as O  # noqa: E402

REF_ROOT = O.REF_ROOT

# (name, rows, cols, t, seed, weight stream, x stream). rows % 16 == 0 (the reference's form I).
CASES = [
    ("gemv_64x512", 64, 512, 1, 11, 1, 2),
    ("gemv_48x1024", 48, 1024, 1, 12, 1, 2),
    ("gemv_16x32", 16, 32, 1, 13, 1, 2),
    ("gemm_32x256_t3", 32, 256, 3, 14, 1, 2),
    ("gemm_16x512_t9", 16, 512, 9, 15, 1, 2),
    ("gemm_16x32_t17", 16, 32, 17, 16, 1, 2),
    ("gemm_48x4128_t2", 48, 4128, 2, 17, 1, 2),
    ("gemv_4096x4096", 4096, 4096, 1, 1, 1, 2),
    ("gemm_1024x12288_t2", 1024, 12288, 2, 3, 5, 6), # a down-projection slice, verify M = 2
]
INLINE_MAX = 64 * 1024  # input bytes stored outright up to this size


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def gates() -> dict:
    out = {"source": "reference tests/golden/gate-2.1.txt and gate-a.txt"}
    g21 = {}
    with open(os.path.join(REF_ROOT, "tests/golden/gate-2.1.txt")) as f:
        for line in f:
            p = line.split()
            g21[p[0]] = {"n": int(p[2]), "hash": p[4]}
    out["gate_2_1"] = g21
    with open(os.path.join(REF_ROOT, "tests/golden/gate-a.txt")) as f:
        p = f.read().split()
    out["gate_a"] = {"n": int(p[1]), "hash": p[3], "c0": p[5], "c1": p[7], "clast": p[9]}
    return out


def main() -> None:
    if not O.ref_available():
        sys.exit("oracle/_ref/libq8ref.so missing: run make -C oracle ref (needs the reference tree)")
    with open(os.path.join(HERE, "ref_gates.json"), "w") as f:
        json.dump(gates(), f, indent=1)
        f.write("\n")
    arrays = {}
    meta = []
    for name, rows, cols, t, seed, ws, xs in CASES:
        q8 = O.synth_q8_0(rows, cols, seed, ws)
        x = np.stack([O.synth_f32(cols, seed, xs + 1000 * k) for k in range(t)]).astype(np.float32)
        m = O.RefMatrix(q8, rows, cols)
        y = m.gemv(x[0])[None, :] if t == 1 else m.gemm(x, t)
        arrays[f"{name}.y"] = y.view(np.uint32)
        if q8.nbytes <= INLINE_MAX:
            arrays[f"{name}.q8"] = q8
            arrays[f"{name}.x"] = x
        meta.append({"name": name, "rows": rows, "cols": cols, "t": t, "seed": seed, "w_stream": ws, "x_stream": xs,
                     "q8_sha256": sha(q8), "x_sha256": sha(x)})
        print(f"{name}: y[0][:3] = {y.reshape(-1)[:3]}")
    arrays["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(os.path.join(HERE, "ref_vectors.npz"), **arrays)
    print("wrote", os.path.join(HERE, "ref_vectors.npz"))


if __name__ == "__main__":
    main()
