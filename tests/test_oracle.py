"""The CPU oracle against the reference's own known answers (CPU only).

The oracle (oracle/q8_oracle.c) restates the reference's Q8_0 product; these tests pin it:
  * to the reference's golden hashes for the conversions and fma the product is built from
    (gate 2.1 and gate A: tests/golden/gate-2.1.txt, gate-a.txt of the reference);
  * to y vectors the reference's own gemv_i_thread / gemm_i_thread produced from its sources
    (tests/golden/ref_vectors.npz, made by tests/golden/make_golden.py), bit for bit;
  * and, where the reference tree is present, to the reference's host model run live.
"""
from __future__ import annotations

import hashlib
import json
import os

import numpy as np
import pytest

import oracle as O
from conftest import GOLDEN


def _vectors():
    z = np.load(os.path.join(GOLDEN, "ref_vectors.npz"))
    meta = json.loads(bytes(z["meta"]).decode())
    return z, meta


def _sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_gate_2_1_hashes(oracle):
    """int8 and fp16 up-conversions, the {1to16} fma and the tree sum: the reference's golden file."""
    gold = json.load(open(os.path.join(GOLDEN, "ref_gates.json")))["gate_2_1"]
    names = ["s8", "u8fma", "u8mul", "b16", "bcast", "f16", "hsum"]
    got = oracle.gate21_hashes()
    for n, h in zip(names, got):
        assert f"{h:016x}" == gold[n]["hash"], n


def test_gate_a_fma(oracle):
    gold = json.load(open(os.path.join(GOLDEN, "ref_gates.json")))["gate_a"]
    h, words = oracle.gate_a()
    assert f"{h:016x}" == gold["hash"]
    assert [f"{w:08x}" for w in words] == [gold["c0"], gold["c1"], gold["clast"]]


def test_half_decode_all_patterns(oracle):
    """The exact fp16 -> fp32 decode over all 65,536 patterns (tests/host/t_knc_half.c)."""
    lib = oracle.port()
    h = np.arange(65536, dtype=np.uint16)
    want = h.view(np.float16).astype(np.float32).view(np.uint32)
    got = np.array([lib.q8o_half(int(v)) for v in h], dtype=np.float32).view(np.uint32)
    exp = (h >> 10) & 31
    nan = (exp == 31) & ((h & 1023) != 0)
    assert np.array_equal(got[~nan], want[~nan])
    # NaN: same sign and payload, the quiet bit aside (as the reference's own test allows)
    assert np.all(((got[nan] ^ want[nan]) & ~np.uint32(0x00400000)) == 0)


@pytest.mark.parametrize("case", range(9))
def test_port_matches_reference_vectors(oracle, case):
    """The restatement computes the reference's y bit for bit, and rebuilds its exact inputs."""
    z, meta = _vectors()
    m = meta[case]
    rows, cols, t = m["rows"], m["cols"], m["t"]
    q8 = oracle.synth_q8_0(rows, cols, m["seed"], m["w_stream"])
    x = np.stack([oracle.synth_f32(cols, m["seed"], m["x_stream"] + 1000 * k) for k in range(t)])
    assert _sha(q8) == m["q8_sha256"], "the seeded Q8_0 generator changed"
    assert _sha(x) == m["x_sha256"], "the seeded x generator changed"
    if f"{m['name']}.q8" in z:
        assert np.array_equal(z[f"{m['name']}.q8"], q8)
        assert np.array_equal(z[f"{m['name']}.x"], x)
    y = oracle.gemm(q8, rows, cols, x, t)
    assert np.array_equal(y.view(np.uint32), z[f"{m['name']}.y"])


def test_f64_restatement_close(oracle):
    """The F64 check (exact dequant, double sums) agrees with the fp32 order to fp32 rounding."""
    rows, cols = 256, 4096
    q8 = oracle.synth_q8_0(rows, cols, 5, 1)
    x = oracle.synth_f32(cols, 5, 2)
    y = oracle.gemv(q8, rows, cols, x)
    y64 = oracle.gemm_f64(q8, rows, cols, x, 1)[0]
    rms = np.sqrt(np.mean(y64 ** 2))
    assert np.max(np.abs(y - y64) / np.maximum(np.abs(y64), rms)) < 1e-5


def test_split_layout_round_trip(oracle):
    for rows, cols in [(3, 32), (5, 96), (16, 4096), (2, 4128)]:
        q8 = oracle.synth_q8_0(rows, cols, 9, 3)
        s = oracle.repack_split(q8, rows, cols)
        assert s.nbytes == oracle.port().q8o_split_bytes(rows, cols)
        rb = oracle.port().q8o_split_row_bytes(cols)
        assert rb % 16 == 0
        if (cols // 32) % 8 == 0:
            assert rb == cols // 32 * 34, "rows keep their GGUF length: in-place repack"
        assert np.array_equal(oracle.unpack_split(s, rows, cols), q8)
        # quants first, then the scales, in every row
        r1 = s[rb:2 * rb]
        blk = q8[(cols // 32) * 34:(cols // 32) * 34 + 34]
        assert np.array_equal(r1[:32], blk[2:])
        assert np.array_equal(r1[cols:cols + 2], blk[:2])


def test_threaded_generator_is_the_same_matrix(oracle):
    """The bench's CPU baseline fills its matrices on host threads: the same bytes, any split."""
    a = oracle.synth_q8_0(37, 4096, 5, 9, row0=3)
    for threads in (2, 5, 64):
        assert np.array_equal(oracle.synth_q8_0(37, 4096, 5, 9, row0=3, threads=threads), a)


def test_generator_distribution(oracle):
    x = oracle.synth_f32(200000, 3, 4)
    assert abs(x.mean()) < 0.01 and abs(x.std() - 1.0) < 0.01
    q8 = oracle.synth_q8_0(64, 4096, 3, 5).reshape(-1, 34)
    q = q8[:, 2:].view(np.int8)
    assert q.min() >= -127 and q.max() == 127  # d = amax/127: every block reaches |q| = 127
    d = q8[:, :2].copy().view(np.float16).astype(np.float32)
    assert 1e-4 < float(np.median(d)) < 1e-3  # sigma 0.02: amax ~ 0.04..0.07 over 32 draws


def test_gather_and_gemm_port(oracle):
    rows, cols = 64, 256
    q8 = oracle.synth_q8_0(rows, cols, 21, 1)
    x = oracle.synth_f32(cols, 21, 2)
    idx = np.array([5, 0, 63, 5, 17], dtype=np.int32)
    y = oracle.gemv(q8, rows, cols, x)
    assert np.array_equal(oracle.gemv_rows(q8, cols, idx, x).view(np.uint32), y[idx].view(np.uint32))
    X = np.stack([x, -x, 2 * x])
    Y = oracle.gemm(q8, rows, cols, X, 3)
    assert np.array_equal(Y[0].view(np.uint32), y.view(np.uint32))


@pytest.mark.skipif(not os.path.exists(os.path.join(O.REF_ROOT, "src/card/gemv.c")), reason="reference tree absent")
def test_port_against_live_reference(oracle):
    """Where the reference tree is present: its compiled host model, live, on fresh shapes."""
    import subprocess
    subprocess.run(["make", "-C", os.path.join(os.path.dirname(GOLDEN), "..", "oracle"), "ref"], check=True,
                   capture_output=True)
    for rows, cols, t, seed in [(16, 64, 1, 31), (80, 2048, 5, 32), (32, 4096, 16, 33)]:
        q8 = oracle.synth_q8_0(rows, cols, seed, 1)
        x = np.stack([oracle.synth_f32(cols, seed, 2 + k) for k in range(t)])
        ref = oracle.RefMatrix(q8, rows, cols)
        want = ref.gemm(x, t) if t > 1 else ref.gemv(x[0])[None]
        got = oracle.gemm(q8, rows, cols, x, t)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


PRIM_SHAPES = [  # h, n1, c, t (history), r (state rows), m, k
    (8, 2, 64, 37, 19, 24, 40),
    (16, 4, 256, 300, 128, 128, 128),
    (3, 3, 8, 1, 1, 1, 8),
    (40, 1, 72, 130, 5, 9, 16),
]


def _prim_inputs(shape, seed):
    h, n1, c, t, r, m, k = shape
    rng = np.random.default_rng(seed)
    f = lambda n: rng.standard_normal(n).astype(np.float32)
    l = np.array([(7 * q + 1) % n1 for q in range(h)], dtype=np.int64)
    return dict(kv=f(t * n1 * c), b=f(h * c), l=l, a=f(h * t), A=f(h * r * c), s=f(m * k), av=f(m), bv=f(k))


@pytest.mark.skipif(not O.hostref_available(), reason="oracle/_ref/libhostref.so not built (reference tree absent)")
@pytest.mark.parametrize("shape", PRIM_SHAPES)
def test_prims_port_matches_reference(oracle, shape):
    """The C restatement of the host-half primitives (prims_oracle.c) against the reference's own
    src/host/rt_host.c compiled from its sources: every output bit for bit."""
    h, n1, c, t, r, m, k = shape
    d = _prim_inputs(shape, 5)
    cases = [
        (lambda u: oracle.ip21_kv(d["kv"], n1, c, d["l"], h, t, d["b"], use_ref=u)),
        (lambda u: oracle.ip12_kv(d["a"], d["kv"], n1, c, d["l"], h, t, use_ref=u)),
        (lambda u: oracle.ip21(d["A"], h, r, c, d["b"], use_ref=u)),
        (lambda u: oracle.scale_outer(d["s"], 0.9375, d["av"], d["bv"], m, k, use_ref=u)),
    ]
    for f in cases:
        assert np.array_equal(f(False).view(np.uint32), f(True).view(np.uint32))


def test_prims_port_order(oracle):
    """The restatement's lane order, on inputs where it shows: 8-lane sums differ from a plain
    left-to-right sum, and ip12_kv is one ordered chain."""
    c = 16
    row = np.array([1e8, 1, -1e8, 1, 3, 0, 0, 0, 0.5, 0, 0, 0, 0, 0, 0, 0], dtype=np.float32)
    b = np.ones(c, dtype=np.float32)
    z = oracle.ip21(row, 1, 1, c, b)
    lanes = [float(np.float32(row[j]) + np.float32(row[j + 8])) for j in range(8)]
    want = np.float32((np.float32(lanes[0] + lanes[4]) + np.float32(lanes[2] + lanes[6])) +
                      np.float32(np.float32(lanes[1] + lanes[5]) + np.float32(lanes[3] + lanes[7])))
    assert z[0] == want
    a = np.array([1e8, 1.0, -1e8], dtype=np.float32)
    kv = np.ones(3 * 8, dtype=np.float32)
    z = oracle.ip12_kv(a, kv, 1, 8, np.zeros(1, dtype=np.int64), 1, 3)
    assert z[0] == np.float32(np.float32(np.float32(1e8) + 1.0) - np.float32(1e8))
