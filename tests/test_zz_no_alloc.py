"""rt_gemm_static: the tensor-core product for callers that cannot allocate device memory.

Some engines reserve all of HBM up front or forbid allocation while serving, so they can't let
the library cudaMalloc the scratch its tensor-core path needs (the fp16 copy of x). rt_gemm_static
runs the same kernel with that scratch in a fixed device array inside the library. These tests
call it through the C ABI and hold it to the ordinary entry point (rt_gemm at t >= 16) within the
tensor-core tolerance, on two calls in a row, and to the CPU oracle (the reference's rounding
order in fp32) within the same tolerance; and check that it refuses sizes beyond its limits.
This file is collected last on purpose: if it fails, a run that stops at the first failure has
already run every other test.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SEED = 20261201
TC_TOL = 2e-3
STATIC_LIMIT = 4 * 1024 * 1024  # t * cols: the 8 MiB fp16 copy of x
STATIC_ROWS = 1024 * 1024       # rows: one scale exponent byte per row


def rel_err(y, ref) -> float:
    ref = ref.astype(np.float64)
    rms = float(np.sqrt(np.mean(ref ** 2))) or 1.0
    return float(np.max(np.abs(y.astype(np.float64) - ref) / np.maximum(np.abs(ref), rms)))


def _matrix(torch, rtb, rows, cols, stream):
    w = torch.empty(rtb.gemv_s_bytes(rows, cols), dtype=torch.uint8, device="cuda")
    rtb.synth_q8_0(w.data_ptr(), 0, rows, cols, SEED, stream)
    return w


def _x(torch, rtb, t, cols, stream):
    x = torch.empty(t * cols, dtype=torch.float32, device="cuda")
    rtb.synth_f32(x.data_ptr(), t * cols, SEED, stream)
    return x


def test_static_gemm_matches_rt_gemm_two_calls(cuda, runtime, rtb):
    lib = rtb.load()
    # two calls in a row, different shapes and inputs: the second must not see the first's state
    for rows, cols, t, stream in [(4096, 4096, 40, 201), (1000, 12288, 300, 202)]:
        w = _matrix(cuda, rtb, rows, cols, stream)
        x = _x(cuda, rtb, t, cols, stream + 50)
        y_static = cuda.full((t, rows), float("nan"), dtype=cuda.float32, device="cuda")
        y_ref = cuda.full((t, rows), float("nan"), dtype=cuda.float32, device="cuda")
        cuda.cuda.synchronize()
        rc = lib.rt_gemm_static(w.data_ptr(), rows, cols, x.data_ptr(), t, y_static.data_ptr(), None)
        assert rc == 0, rc
        runtime.gemm(w.data_ptr(), rows, cols, x.data_ptr(), t, y_ref.data_ptr())
        got, want = y_static.cpu().numpy(), y_ref.cpu().numpy()
        assert np.isfinite(got).all()
        assert rel_err(got, want) < TC_TOL


def test_static_gemm_matches_the_oracle(cuda, rtb, oracle):
    """Against the CPU oracle (the reference's fp32 rounding order) rather than the library itself."""
    lib = rtb.load()
    rows, cols, t = 1024, 4096, 48
    q8 = oracle.synth_q8_0(rows, cols, SEED, 211)
    w = cuda.from_numpy(oracle.repack_split(q8, rows, cols)).cuda()
    x = np.stack([oracle.synth_f32(cols, SEED, 212 + k) for k in range(t)]).astype(np.float32)
    xd = cuda.from_numpy(x).cuda()
    for _ in range(2):
        y = cuda.full((t, rows), float("nan"), dtype=cuda.float32, device="cuda")
        cuda.cuda.synchronize()
        assert lib.rt_gemm_static(w.data_ptr(), rows, cols, xd.data_ptr(), t, y.data_ptr(), None) == 0
        assert rel_err(y.cpu().numpy(), oracle.gemm(q8, rows, cols, x, t)) < TC_TOL


def test_static_gemm_refuses_what_it_cannot_hold(cuda, runtime, rtb):
    lib = rtb.load()
    rows, cols = 256, 8192
    w = _matrix(cuda, rtb, rows, cols, 203)
    t_over = STATIC_LIMIT // cols + 1
    x = cuda.zeros(t_over * cols, dtype=cuda.float32, device="cuda")
    y = cuda.zeros((t_over, rows), dtype=cuda.float32, device="cuda")
    assert lib.rt_gemm_static(w.data_ptr(), rows, cols, x.data_ptr(), t_over, y.data_ptr(), None) == 1
    assert lib.rt_gemm_static(w.data_ptr(), rows, cols, x.data_ptr(), 8, y.data_ptr(), None) == 1  # t < 16
    assert lib.rt_gemm_static(w.data_ptr(), rows, 33, x.data_ptr(), 16, y.data_ptr(), None) == 1
    # more rows than the exponent bytes hold (checked before anything is read)
    assert lib.rt_gemm_static(w.data_ptr(), STATIC_ROWS + 1, cols, x.data_ptr(), 16, y.data_ptr(), None) == 1
    # at the limit it runs
    t_max = STATIC_LIMIT // cols
    assert lib.rt_gemm_static(w.data_ptr(), rows, cols, x.data_ptr(), t_max, y.data_ptr(), None) == 0
