"""Parity of the B200 products with the reference (GPU).

Every product goes through the C ABI of librt_b200.so (rt_gemv, rt_gemm, the queued round, ...)
on device buffers; the checker is the CPU oracle (oracle/), itself pinned to the reference's own
host-model output (tests/test_oracle.py), and for the golden cases the reference's y directly.

Bar: for t < 16 tokens the CUDA-core path computes the reference's rounding sequence, so y must
equal the reference bit for bit (compared as uint32 patterns). The fused SwiGLU adds an fp32
silu(g)*u after two exact products: within 1e-5 relative (rms floor) of the F64 value. From
t = 16 the tensor cores run the product on fp16 operands with fp32 sums: within TC_TOL = 2e-3
as max |y - ref| / max(|ref|, rms(ref)) against the reference's fp32 y.
"""
from __future__ import annotations

import json
import os

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu

SEED = 20261201
TC_MIN_T = 16
TC_TOL = 2e-3


def rel_err(y: np.ndarray, ref: np.ndarray) -> float:
    """max |y - ref| / max(|ref|, rms(ref)): relative error with an rms floor for outputs near 0."""
    ref = ref.astype(np.float64)
    rms = float(np.sqrt(np.mean(ref ** 2))) or 1.0
    return float(np.max(np.abs(y.astype(np.float64) - ref) / np.maximum(np.abs(ref), rms)))


def bits_equal(a: np.ndarray, b: np.ndarray) -> bool:
    return np.array_equal(np.ascontiguousarray(a, dtype=np.float32).view(np.uint32),
                          np.ascontiguousarray(b, dtype=np.float32).view(np.uint32))


class Mat:
    """A seeded Q8_0 matrix on the device (row-split layout, made by the GPU generator) and the
    same matrix's GGUF bytes on the host (made by the CPU generator)."""

    def __init__(self, torch, rtb, oracle, rows, cols, stream, host=True):
        self.rows, self.cols = rows, cols
        self.dev = torch.empty(rtb.gemv_s_bytes(rows, cols), dtype=torch.uint8, device="cuda")
        rtb.synth_q8_0(self.dev.data_ptr(), 0, rows, cols, SEED, stream)
        self.q8 = oracle.synth_q8_0(rows, cols, SEED, stream) if host else None

    @property
    def ptr(self) -> int:
        return self.dev.data_ptr()


def dev(torch, a: np.ndarray):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def xs(oracle, t, cols, stream):
    return np.stack([oracle.synth_f32(cols, SEED, stream + 1000 * k) for k in range(t)]).astype(np.float32)


# ---------------------------------------------------------------- inputs and layout

@pytest.mark.parametrize("rows,cols", [(1, 32), (5, 96), (64, 4096), (3, 4128)])
def test_gpu_generator_matches_cpu(cuda, rtb, oracle, rows, cols):
    m = Mat(cuda, rtb, oracle, rows, cols, 7)
    assert np.array_equal(m.dev.cpu().numpy(), oracle.repack_split(m.q8, rows, cols))
    x = cuda.empty(1000, dtype=cuda.float32, device="cuda")
    rtb.synth_f32(x.data_ptr(), 1000, SEED, 9)
    assert bits_equal(x.cpu().numpy(), oracle.synth_f32(1000, SEED, 9))


@pytest.mark.parametrize("rows,cols,in_place", [(37, 4096, True), (16, 96, False), (9, 12288, True), (4, 4128, False)])
def test_repack(cuda, rtb, oracle, rows, cols, in_place):
    q8 = oracle.synth_q8_0(rows, cols, SEED, 3)
    want = oracle.repack_split(q8, rows, cols)
    src = dev(cuda, q8)
    if in_place:
        rtb.gemv_s_repack(src.data_ptr(), rows, cols, src.data_ptr())
        got = src
    else:
        got = cuda.empty(rtb.gemv_s_bytes(rows, cols), dtype=cuda.uint8, device="cuda")
        rtb.gemv_s_repack(src.data_ptr(), rows, cols, got.data_ptr())
    assert np.array_equal(got.cpu().numpy(), want)


def test_reference_load_names_repack(cuda, rtb, oracle):
    """gemv_i_repack_thread as the engine's load site runs it (a team body; thread 0 repacks in
    place on the GPU) and gemv_i_repack out of place: the row-split layout under the reference's
    names (src/card/gemv.h:51-67)."""
    import ctypes as C
    lib = rtb.load()
    rows, cols = 300, 4096
    q8 = oracle.synth_q8_0(rows, cols, SEED, 4)
    want = oracle.repack_split(q8, rows, cols)
    w = dev(cuda, q8)

    class Job(C.Structure):
        _fields_ = [("w", C.c_void_p), ("rows", C.c_long), ("cols", C.c_long), ("tmp", C.c_void_p)]

    job = Job(w.data_ptr(), rows, cols, None)
    for tid in (2, 1, 0):
        lib.gemv_i_repack_thread(C.cast(C.byref(job), C.c_void_p), tid, 3)
    assert rtb.last_error(None)[0] == 0
    assert np.array_equal(w.cpu().numpy(), want)
    src = dev(cuda, q8)
    out = cuda.empty(lib.gemv_i_bytes(rows, cols), dtype=cuda.uint8, device="cuda")
    lib.gemv_i_repack(src.data_ptr(), rows, cols, out.data_ptr())
    assert rtb.last_error(None)[0] == 0
    assert np.array_equal(out.cpu().numpy(), want)


# ---------------------------------------------------------------- the reference's golden y

def _golden():
    z = np.load(os.path.join(GOLDEN, "ref_vectors.npz"))
    return z, json.loads(bytes(z["meta"]).decode())


@pytest.mark.parametrize("case", range(9))
def test_reference_golden_vectors(cuda, runtime, rtb, oracle, case):
    """y of the reference's own gemv_i_thread / gemm_i_thread, reproduced bit for bit on B200."""
    z, meta = _golden()
    m = meta[case]
    rows, cols, t = m["rows"], m["cols"], m["t"]
    q8 = oracle.synth_q8_0(rows, cols, m["seed"], m["w_stream"])
    x = np.stack([oracle.synth_f32(cols, m["seed"], m["x_stream"] + 1000 * k) for k in range(t)])
    w = dev(cuda, oracle.repack_split(q8, rows, cols))
    xd = dev(cuda, x)
    y = cuda.full((t, rows), float("nan"), dtype=cuda.float32, device="cuda")
    if t == 1:
        runtime.gemv(w.data_ptr(), rows, cols, xd.data_ptr(), y.data_ptr())
    else:
        runtime.gemm(w.data_ptr(), rows, cols, xd.data_ptr(), t, y.data_ptr())
    if t < TC_MIN_T:
        assert np.array_equal(y.cpu().numpy().view(np.uint32), z[f"{m['name']}.y"])
    else:  # tensor cores: fp16 operands
        assert rel_err(y.cpu().numpy(), z[f"{m['name']}.y"].view(np.float32)) < TC_TOL


# ---------------------------------------------------------------- gemv

@pytest.mark.parametrize("rows,cols", [
    (4096, 4096),
    (8192, 4096),    # fused QKV
    (4096, 12288),   # down
    (1, 32), (7, 64), (13, 4096), (100, 12288), (33, 4128), (9, 8192), (257, 1056),
])
def test_gemv_bit_exact(cuda, runtime, rtb, oracle, rows, cols):
    m = Mat(cuda, rtb, oracle, rows, cols, 11)
    x = xs(oracle, 1, cols, 12)
    xd = dev(cuda, x)
    y = cuda.full((rows,), float("nan"), dtype=cuda.float32, device="cuda")
    runtime.gemv(m.ptr, rows, cols, xd.data_ptr(), y.data_ptr())
    assert bits_equal(y.cpu().numpy(), oracle.gemv(m.q8, rows, cols, x[0]))


@pytest.mark.parametrize("rows,cols", [
    (14208, 4096),   # 1776 stages: the smallest one-token launch that runs two CTAs per SM
    (12288, 8192),   # two CTAs per SM, rows longer than a stage (two chunks each)
    (14200, 4096),   # 1775 stages: one CTA per SM, just under the switch
])
def test_gemv_two_ctas_per_sm(cuda, runtime, rtb, oracle, rows, cols):
    """Launches long enough to run two CTAs per SM (12 stages per SM on 148 SMs), and the one
    just under the switch, bit for bit."""
    m = Mat(cuda, rtb, oracle, rows, cols, 15)
    x = xs(oracle, 1, cols, 16)
    xd = dev(cuda, x)
    y = cuda.full((rows,), float("nan"), dtype=cuda.float32, device="cuda")
    runtime.gemv(m.ptr, rows, cols, xd.data_ptr(), y.data_ptr())
    assert bits_equal(y.cpu().numpy(), oracle.gemv(m.q8, rows, cols, x[0]))


def test_round_through_host_buffers(cuda, runtime, rtb, oracle):
    """The engine's link crossing (link_pull / link_push of src/card/link.c:86-118): x pulled from
    pinned host memory, the product enqueued, y pushed back; push returns with y on the host."""
    rows, cols = 512, 4096
    m = Mat(cuda, rtb, oracle, rows, cols, 31)
    x = xs(oracle, 1, cols, 32)[0]
    hx = cuda.from_numpy(x).pin_memory()
    hy = cuda.zeros(rows, dtype=cuda.float32).pin_memory()
    xd = cuda.empty(cols, dtype=cuda.float32, device="cuda")
    yd = cuda.empty(rows, dtype=cuda.float32, device="cuda")
    runtime.set_async(True)
    for _ in range(3):  # repeated rounds on the same buffers
        hy.zero_()
        runtime.pull(xd.data_ptr(), hx.data_ptr(), 4 * cols)
        runtime.gemv(m.ptr, rows, cols, xd.data_ptr(), yd.data_ptr())
        runtime.push(hy.data_ptr(), yd.data_ptr(), 4 * rows)
        assert bits_equal(hy.numpy(), oracle.gemv(m.q8, rows, cols, x))
    runtime.set_async(False)
    with pytest.raises(rtb.RtError):
        runtime.push(hy.data_ptr(), 0, 4 * rows)


@pytest.mark.parametrize("blocking", [False, True])
def test_opened_round(cuda, rtb, oracle, blocking):
    """The reference's opened round (src/card/rt.c:267-285, placed by src/apl/compiler/em.apl:
    1014-1046): products queued, rt_gemv_open before x has landed (the CUDA-core products are
    launched and stream their weights, their compute gated on the device), x pulled from pinned
    host memory, rt_gemv_go, y pushed back. A plain gemv, a SwiGLU pair, a row gather, a 2-token
    gemm and a 16-token tensor-core gemm (launched at go) in one round, over three rounds."""
    cols = 4096
    a = Mat(cuda, rtb, oracle, 8192, cols, 191)
    g = Mat(cuda, rtb, oracle, 512, cols, 192)
    u = Mat(cuda, rtb, oracle, 512, cols, 193)
    idx = np.array([8191, 0, 4000, 17, 17], dtype=np.int32)
    idx_d = dev(cuda, idx)
    xd = cuda.empty((16, cols), dtype=cuda.float32, device="cuda")
    ya = cuda.empty(8192, dtype=cuda.float32, device="cuda")
    h = cuda.empty(512, dtype=cuda.float32, device="cuda")
    yr = cuda.empty(5, dtype=cuda.float32, device="cuda")
    y2 = cuda.empty((2, 8192), dtype=cuda.float32, device="cuda")
    y16 = cuda.empty((16, 8192), dtype=cuda.float32, device="cuda")
    hy = cuda.zeros(8192, dtype=cuda.float32).pin_memory()
    with rtb.Runtime() as rt:
        rt.set_async(not blocking)
        for k in range(3):
            x = xs(oracle, 16, cols, 194 + k)
            hx = cuda.from_numpy(x).pin_memory()
            rt.gemv_q(a.ptr, 8192, cols, xd.data_ptr(), ya.data_ptr())
            rt.gemm_silu_q(g.ptr, u.ptr, 512, cols, xd.data_ptr(), 1, h.data_ptr())
            rt.gemv_rows_q(a.ptr, 8192, idx_d.data_ptr(), 5, cols, xd.data_ptr(), yr.data_ptr())
            rt.gemm_q(a.ptr, 8192, cols, xd.data_ptr(), 2, y2.data_ptr())
            rt.gemm_q(a.ptr, 8192, cols, xd.data_ptr(), 16, y16.data_ptr())
            rt.gemv_open()
            rt.pull(xd.data_ptr(), hx.data_ptr(), 4 * 16 * cols)
            rt.gemv_go()
            rt.push(hy.data_ptr(), ya.data_ptr(), 4 * 8192)
            want = oracle.gemm(a.q8, 8192, cols, x, 16)
            assert bits_equal(hy.numpy(), want[0])
            assert bits_equal(ya.cpu().numpy(), want[0])
            assert bits_equal(yr.cpu().numpy(), want[0][idx])
            assert bits_equal(y2.cpu().numpy(), want[:2])
            assert rel_err(y16.cpu().numpy(), want) < TC_TOL
            yg = oracle.gemv(g.q8, 512, cols, x[0]).astype(np.float64)
            yu = oracle.gemv(u.q8, 512, cols, x[0]).astype(np.float64)
            assert rel_err(h.cpu().numpy(), yg / (1 + np.exp(-yg)) * yu) < 1e-5


def test_opened_round_without_go_gives_up_and_recovers(cuda, rtb, oracle):
    """An opened round whose go never comes: the pre-launched kernel's wait for its x gives up
    after about a second and reports it (RTB_EKERNEL, naming the missing go); the runtime then
    runs the next round bit for bit. No GPU fault: the wait is bounded."""
    rows, cols = 1024, 4096
    m = Mat(cuda, rtb, oracle, rows, cols, 201)
    x = xs(oracle, 1, cols, 202)
    xd = dev(cuda, x)
    y = cuda.full((rows,), float("nan"), dtype=cuda.float32, device="cuda")
    with rtb.Runtime() as rt:
        rt.set_async(True)
        rt.gemv_q(m.ptr, rows, cols, xd.data_ptr(), y.data_ptr())
        rt.gemv_open()
        with pytest.raises(rtb.RtError) as e:
            rt.sync()
        assert e.value.code == 3 and "never landed" in str(e.value), str(e.value)
        rt.set_async(False)
        rt.gemv_q(m.ptr, rows, cols, xd.data_ptr(), y.data_ptr())
        rt.gemv_open()
        rt.gemv_go()
        assert bits_equal(y.cpu().numpy(), oracle.gemv(m.q8, rows, cols, x[0]))


def test_direct_push(cuda, rtb, oracle):
    """rt_b200_set_push_direct: a round of one product, held back by rt_gemv_go, then pushed into
    mapped pinned host memory, writes y there from its own kernel and raises a host flag; push
    returns with y whole on the host. The product runs as a CUDA graph cached by its arguments:
    the later rounds reuse the graphs, with new x pulled into the same buffer. Checked bit for bit on the host and in device memory over
    back-to-back rounds (a gemv, a SwiGLU pair, a row gather, a 2-token product, the 151936-row
    head), and the rounds that must take the usual path: a push of part of y, a push into
    pageable memory, a held round followed by another call instead of a push, and a 16-token
    tensor-core product (never held)."""
    cols = 4096
    a = Mat(cuda, rtb, oracle, 8192, cols, 211)
    g = Mat(cuda, rtb, oracle, 512, cols, 212)
    u = Mat(cuda, rtb, oracle, 512, cols, 213)
    hd = Mat(cuda, rtb, oracle, 151936, cols, 214)
    idx = np.array([8191, 0, 4000, 17, 17], dtype=np.int32)
    idx_d = dev(cuda, idx)
    xd = cuda.empty((16, cols), dtype=cuda.float32, device="cuda")
    ya = cuda.full((8192,), float("nan"), dtype=cuda.float32, device="cuda")
    y2 = cuda.full((2, 8192), float("nan"), dtype=cuda.float32, device="cuda")
    h = cuda.full((512,), float("nan"), dtype=cuda.float32, device="cuda")
    yr = cuda.full((5,), float("nan"), dtype=cuda.float32, device="cuda")
    yh = cuda.full((151936,), float("nan"), dtype=cuda.float32, device="cuda")
    y16 = cuda.full((16, 8192), float("nan"), dtype=cuda.float32, device="cuda")
    host = cuda.full((2 * 151936,), float("nan"), dtype=cuda.float32).pin_memory()
    pageable = np.full(8192, np.nan, dtype=np.float32)

    def fresh():
        host.fill_(float("nan"))

    with rtb.Runtime() as rt:
        rt.set_async(True)
        rt.set_push_direct(True)
        hx = cuda.empty((16, cols), dtype=cuda.float32).pin_memory()
        for k in range(3):  # the same buffers each time: from the second, the rounds' cached graphs
            x = xs(oracle, 16, cols, 215 + k)
            hx.copy_(cuda.from_numpy(x))
            want = oracle.gemm(a.q8, 8192, cols, x, 2)
            # a gemv, pushed whole into pinned memory: direct
            fresh()
            rt.gemv_q(a.ptr, 8192, cols, xd.data_ptr(), ya.data_ptr())
            rt.pull(xd.data_ptr(), hx.data_ptr(), 4 * 16 * cols)
            rt.gemv_go()
            rt.push(host.data_ptr(), ya.data_ptr(), 4 * 8192)
            assert bits_equal(host[:8192].numpy(), want[0]), k
            assert bits_equal(ya.cpu().numpy(), want[0]), k
            # 2 tokens
            fresh()
            rt.gemm_q(a.ptr, 8192, cols, xd.data_ptr(), 2, y2.data_ptr())
            rt.gemv_go()
            rt.push(host.data_ptr(), y2.data_ptr(), 4 * 2 * 8192)
            assert bits_equal(host[:2 * 8192].numpy().reshape(2, 8192), want), k
            # a SwiGLU pair
            fresh()
            rt.gemm_silu_q(g.ptr, u.ptr, 512, cols, xd.data_ptr(), 1, h.data_ptr())
            rt.gemv_go()
            rt.push(host.data_ptr(), h.data_ptr(), 4 * 512)
            yg = oracle.gemv(g.q8, 512, cols, x[0]).astype(np.float64)
            yu = oracle.gemv(u.q8, 512, cols, x[0]).astype(np.float64)
            hs = host[:512].numpy()
            assert np.allclose(hs, (yg / (1.0 + np.exp(-yg)) * yu).astype(np.float32), rtol=1e-6, atol=1e-30), k
            assert bits_equal(h.cpu().numpy(), hs), k
            # a row gather
            fresh()
            rt.gemv_rows_q(a.ptr, 8192, idx_d.data_ptr(), 5, cols, xd.data_ptr(), yr.data_ptr())
            rt.gemv_go()
            rt.push(host.data_ptr(), yr.data_ptr(), 4 * 5)
            assert bits_equal(host[:5].numpy(), want[0][idx]), k
            # the head: 607 KB of y from 296 CTAs
            fresh()
            rt.gemv_q(hd.ptr, 151936, cols, xd.data_ptr(), yh.data_ptr())
            rt.gemv_go()
            rt.push(host.data_ptr(), yh.data_ptr(), 4 * 151936)
            assert bits_equal(host[:151936].numpy(), oracle.gemv(hd.q8, 151936, cols, x[0])), k
        # the usual path: part of y; pageable memory; another call first; tensor cores
        x = xs(oracle, 16, cols, 219)
        xd.copy_(cuda.from_numpy(x))
        want = oracle.gemm(a.q8, 8192, cols, x, 16)
        fresh()
        ya.fill_(float("nan"))
        rt.gemv_q(a.ptr, 8192, cols, xd.data_ptr(), ya.data_ptr())
        rt.gemv_go()
        rt.push(host.data_ptr(), ya.data_ptr(), 4 * 4096)
        assert bits_equal(host[:4096].numpy(), want[0][:4096])
        assert np.isnan(host[4096:8192].numpy()).all()
        assert bits_equal(ya.cpu().numpy(), want[0])
        rt.gemv_q(a.ptr, 8192, cols, xd.data_ptr(), ya.data_ptr())
        rt.gemv_go()
        rt.push(pageable.ctypes.data, ya.data_ptr(), 4 * 8192)
        assert bits_equal(pageable, want[0])
        ya.fill_(float("nan"))
        rt.gemv_q(a.ptr, 8192, cols, xd.data_ptr(), ya.data_ptr())
        rt.gemv_go()
        rt.sync()  # launches the held round, as any call on R does
        assert bits_equal(ya.cpu().numpy(), want[0])
        rt.gemm_q(a.ptr, 8192, cols, xd.data_ptr(), 16, y16.data_ptr())
        rt.gemv_go()
        rt.push(host.data_ptr(), y16.data_ptr(), 4 * 16 * 8192)
        assert rel_err(host[:16 * 8192].numpy().reshape(16, 8192), want) < TC_TOL


def test_gemv_output_head_full_size(cuda, runtime, rtb, oracle):
    """BASELINE config 2's output head, 151936 x 4096, every output bit for bit."""
    rows, cols = 151936, 4096
    m = Mat(cuda, rtb, oracle, rows, cols, 13)
    x = xs(oracle, 1, cols, 14)
    xd = dev(cuda, x)
    y = cuda.empty((rows,), dtype=cuda.float32, device="cuda")
    runtime.gemv(m.ptr, rows, cols, xd.data_ptr(), y.data_ptr())
    assert bits_equal(y.cpu().numpy(), oracle.gemv(m.q8, rows, cols, x[0]))


# ---------------------------------------------------------------- gemm on CUDA cores (t < 16)

@pytest.mark.parametrize("t", [2, 3, 4, 5, 8, 9, 15])
@pytest.mark.parametrize("rows,cols", [(256, 4096), (40, 12288), (17, 96)])
def test_gemm_small_t_bit_exact(cuda, runtime, rtb, oracle, t, rows, cols):
    m = Mat(cuda, rtb, oracle, rows, cols, 21)
    x = xs(oracle, t, cols, 22)
    xd = dev(cuda, x)
    y = cuda.full((t, rows), float("nan"), dtype=cuda.float32, device="cuda")
    runtime.gemm(m.ptr, rows, cols, xd.data_ptr(), t, y.data_ptr())
    assert bits_equal(y.cpu().numpy(), oracle.gemm(m.q8, rows, cols, x, t))


@pytest.mark.parametrize("t", [2, 3, 4])
def test_gemm_wide_rows_many_tiles_per_cta(cuda, runtime, rtb, oracle, t):
    """Rows of four 4096-column chunks, 3-4 row tiles per CTA: the two chain warps take alternate
    tiles, each tile as long as the ring of partial-sum buffers (so each chain warp skips a whole
    ring's worth of the other's stages between its own). Bit for bit."""
    rows, cols = 4096, 16384
    m = Mat(cuda, rtb, oracle, rows, cols, 25)
    x = xs(oracle, t, cols, 26)
    xd = dev(cuda, x)
    y = cuda.full((t, rows), float("nan"), dtype=cuda.float32, device="cuda")
    runtime.gemm(m.ptr, rows, cols, xd.data_ptr(), t, y.data_ptr())
    assert bits_equal(y.cpu().numpy(), oracle.gemm(m.q8, rows, cols, x, t))


def test_gemm_each_token_equals_gemv(cuda, runtime, rtb, oracle):
    """The reference's gate: gemm of t tokens == one gemv per token, bit for bit
    (scripts/check.sh:132-149 of the reference)."""
    rows, cols, t = 1888, 512, 9
    m = Mat(cuda, rtb, oracle, rows, cols, 23, host=False)
    x = dev(cuda, xs(oracle, t, cols, 24))
    y = cuda.empty((t, rows), dtype=cuda.float32, device="cuda")
    runtime.gemm(m.ptr, rows, cols, x.data_ptr(), t, y.data_ptr())
    for k in range(t):
        y1 = cuda.empty((rows,), dtype=cuda.float32, device="cuda")
        runtime.gemv(m.ptr, rows, cols, x[k].data_ptr(), y1.data_ptr())
        assert bits_equal(y[k].cpu().numpy(), y1.cpu().numpy())


# ---------------------------------------------------------------- fused products

@pytest.mark.parametrize("t", [1, 2, 5])
def test_swiglu_fused(cuda, runtime, rtb, oracle, t):
    rows, cols = 1536, 4096
    g = Mat(cuda, rtb, oracle, rows, cols, 31)
    u = Mat(cuda, rtb, oracle, rows, cols, 32)
    x = xs(oracle, t, cols, 33)
    xd = dev(cuda, x)
    h = cuda.full((t, rows), float("nan"), dtype=cuda.float32, device="cuda")
    runtime.gemm_silu(g.ptr, u.ptr, rows, cols, xd.data_ptr(), t, h.data_ptr())
    yg = oracle.gemm(g.q8, rows, cols, x, t).astype(np.float64)
    yu = oracle.gemm(u.q8, rows, cols, x, t).astype(np.float64)
    want = yg / (1.0 + np.exp(-yg)) * yu
    assert rel_err(h.cpu().numpy(), want) < 1e-5


def test_draft_head_gather(cuda, runtime, rtb, oracle):
    """32,768 seeded rows of the 151,936 x 4096 output matrix."""
    rows, cols, n = 151936, 4096, 32768
    m = Mat(cuda, rtb, oracle, rows, cols, 41, host=False)
    idx = np.sort(np.random.default_rng(SEED).choice(rows, n, replace=False)).astype(np.int32)
    idx = np.random.default_rng(SEED + 1).permutation(idx).astype(np.int32)
    x = xs(oracle, 1, cols, 42)
    idx_d, xd = dev(cuda, idx), dev(cuda, x)  # held: a freed tensor's memory can be reused at once
    y = cuda.empty((n,), dtype=cuda.float32, device="cuda")
    runtime.gemv_rows(m.ptr, rows, idx_d.data_ptr(), n, cols, xd.data_ptr(), y.data_ptr())
    rb = rtb.gemv_s_bytes(1, cols)
    sel = m.dev.view(rows, rb)[cuda.from_numpy(idx.astype(np.int64)).cuda()].cpu().numpy().reshape(-1)
    q8 = oracle.unpack_split(sel, n, cols)
    assert bits_equal(y.cpu().numpy(), oracle.gemv(q8, n, cols, x[0]))


def test_queued_round(cuda, runtime, rtb, oracle):
    """One round (rt_gemv_q ... rt_gemv_go): products of several shapes, a SwiGLU pair, a gather
    and a 2-token gemm run in one go, each exact."""
    cols = 4096
    a = Mat(cuda, rtb, oracle, 8192, cols, 51)
    b = Mat(cuda, rtb, oracle, 4096, cols, 52)
    g = Mat(cuda, rtb, oracle, 512, cols, 53)
    u = Mat(cuda, rtb, oracle, 512, cols, 54)
    x = xs(oracle, 2, cols, 55)
    xd = dev(cuda, x)
    ya = cuda.empty(8192, dtype=cuda.float32, device="cuda")
    yb = cuda.empty((2, 4096), dtype=cuda.float32, device="cuda")
    h = cuda.empty(512, dtype=cuda.float32, device="cuda")
    idx = np.array([4095, 0, 17, 17, 2048], dtype=np.int32)
    yr = cuda.empty(5, dtype=cuda.float32, device="cuda")
    runtime.gemv_q(a.ptr, 8192, cols, xd.data_ptr(), ya.data_ptr())
    runtime.gemm_q(b.ptr, 4096, cols, xd.data_ptr(), 2, yb.data_ptr())
    runtime.gemm_silu_q(g.ptr, u.ptr, 512, cols, xd.data_ptr(), 1, h.data_ptr())
    idx_d = dev(cuda, idx)
    runtime.gemv_rows_q(b.ptr, 4096, idx_d.data_ptr(), 5, cols, xd.data_ptr(), yr.data_ptr())
    runtime.gemv_open()
    runtime.gemv_go()
    assert bits_equal(ya.cpu().numpy(), oracle.gemv(a.q8, 8192, cols, x[0]))
    yb_ref = oracle.gemm(b.q8, 4096, cols, x, 2)
    assert bits_equal(yb.cpu().numpy(), yb_ref)
    assert bits_equal(yr.cpu().numpy(), yb_ref[0][idx])
    yg = oracle.gemv(g.q8, 512, cols, x[0]).astype(np.float64)
    yu = oracle.gemv(u.q8, 512, cols, x[0]).astype(np.float64)
    assert rel_err(h.cpu().numpy(), yg / (1 + np.exp(-yg)) * yu) < 1e-5


# ---------------------------------------------------------------- rt_q8_row, modes, errors

def test_q8_row(cuda, rtb, oracle):
    rows, cols = 40, 4128
    m = Mat(cuda, rtb, oracle, rows, cols, 61)
    z = cuda.empty(cols, dtype=cuda.float32, device="cuda")
    for r in (0, 17, 39):
        rtb.q8_row(m.ptr, cols, r, z.data_ptr())
        blk = m.q8.reshape(rows, cols // 32, 34)[r]
        d = blk[:, :2].copy().view(np.float16).astype(np.float32)
        q = blk[:, 2:].view(np.int8).astype(np.float32)
        assert bits_equal(z.cpu().numpy(), (q * d).reshape(-1))


def test_async_mode_and_stream(cuda, rtb, oracle):
    rt = rtb.Runtime()
    try:
        rt.set_async(True)
        rows, cols = 2048, 4096
        m = Mat(cuda, rtb, oracle, rows, cols, 71)
        x = xs(oracle, 3, cols, 72)
        xd = dev(cuda, x)
        ys = [cuda.empty(rows, dtype=cuda.float32, device="cuda") for _ in range(3)]
        for k in range(3):
            rt.gemv(m.ptr, rows, cols, xd[k].data_ptr(), ys[k].data_ptr())
        rt.sync()
        want = oracle.gemm(m.q8, rows, cols, x, 3)
        for k in range(3):
            assert bits_equal(ys[k].cpu().numpy(), want[k])
    finally:
        rt.close()


def test_back_to_back_launches(cuda, rtb, oracle):
    """24 products back to back, overlapping (programmatic launch: each streams its weights while
    the previous one finishes), of sizes around the one/two-CTA-per-SM switch and with rows of one
    to three 4096-column chunks; then the same sequence replayed as a CUDA graph three times:
    every y bit for bit."""
    shapes = [(4096, 4096), (2368, 4096), (2360, 4096), (8192, 4096), (512, 12288), (12288, 4096)]
    mats = [Mat(cuda, rtb, oracle, r, c, 211 + i) for i, (r, c) in enumerate(shapes)]
    xs_ = {c: xs(oracle, 1, c, 217 + c) for c in {c for _, c in shapes}}
    xd = {c: dev(cuda, x) for c, x in xs_.items()}
    want = [oracle.gemv(m.q8, m.rows, m.cols, xs_[m.cols][0]) for m in mats]
    ys = [cuda.full((mats[k % len(mats)].rows,), float("nan"), dtype=cuda.float32, device="cuda") for k in range(24)]
    with rtb.Runtime() as rt:
        rt.set_async(True)
        rt.set_overlap(True)

        def run():
            for k in range(24):
                m = mats[k % len(mats)]
                rt.gemv(m.ptr, m.rows, m.cols, xd[m.cols].data_ptr(), ys[k].data_ptr())

        run()
        rt.sync()
        for k in range(24):
            assert bits_equal(ys[k].cpu().numpy(), want[k % len(mats)]), k
        g = cuda.cuda.CUDAGraph()
        st = cuda.cuda.Stream()
        st.wait_stream(cuda.cuda.current_stream())
        with cuda.cuda.stream(st):
            with cuda.cuda.graph(g, stream=st):
                rt.set_stream(cuda.cuda.current_stream().cuda_stream)
                run()
        cuda.cuda.current_stream().wait_stream(st)
        rt.set_stream(cuda.cuda.current_stream().cuda_stream)
        for _ in range(3):
            for y in ys:
                y.fill_(float("nan"))
            g.replay()
            cuda.cuda.synchronize()
            for k in range(24):
                assert bits_equal(ys[k].cpu().numpy(), want[k % len(mats)]), k
        rt.sync()
        del g


def test_bad_arguments_raise_and_leave_the_gpu_usable(cuda, runtime, rtb, oracle):
    m = Mat(cuda, rtb, oracle, 16, 64, 81)
    x = dev(cuda, xs(oracle, 1, 64, 82))
    y = cuda.empty(16, dtype=cuda.float32, device="cuda")
    with pytest.raises(rtb.RtError) as e:
        runtime.gemv(m.ptr, 16, 33, x.data_ptr(), y.data_ptr())
    assert e.value.code == 1
    with pytest.raises(rtb.RtError):
        runtime.gemv(m.ptr, 0, 64, x.data_ptr(), y.data_ptr())
    with pytest.raises(rtb.RtError):
        runtime.gemv(m.ptr, 16, 64, x.data_ptr() + 4, y.data_ptr())  # x not 16-byte aligned
    with pytest.raises(rtb.RtError):
        runtime.gemm(m.ptr, 16, 64, x.data_ptr(), 0, y.data_ptr())
    runtime.gemv(m.ptr, 16, 64, x.data_ptr(), y.data_ptr())  # still works
    assert bits_equal(y.cpu().numpy(), oracle.gemv(m.q8, 16, 64, x.cpu().numpy()[0]))


def test_gather_index_out_of_range_is_reported_not_read(cuda, runtime, rtb, oracle):
    """An index outside [0, w_rows) is never copied: its y is NaN and the call reports
    RTB_EKERNEL; the other rows are exact and the runtime stays usable."""
    rows, cols = 64, 256
    m = Mat(cuda, rtb, oracle, rows, cols, 91)
    x = xs(oracle, 1, cols, 92)
    xd = dev(cuda, x)
    idx = np.array([3, rows, 5, -1, 63], dtype=np.int32)
    idx_d = dev(cuda, idx)
    y = cuda.zeros(5, dtype=cuda.float32, device="cuda")
    with pytest.raises(rtb.RtError) as e:
        runtime.gemv_rows(m.ptr, rows, idx_d.data_ptr(), 5, cols, xd.data_ptr(), y.data_ptr())
    assert e.value.code == 3
    got = y.cpu().numpy()
    assert np.isnan(got[1]) and np.isnan(got[3])
    want = oracle.gemv(m.q8, rows, cols, x[0])
    assert bits_equal(got[[0, 2, 4]], want[[3, 5, 63]])
    ok = np.array([1, 2], dtype=np.int32)
    ok_d = dev(cuda, ok)
    runtime.gemv_rows(m.ptr, rows, ok_d.data_ptr(), 2, cols, xd.data_ptr(), y.data_ptr())
    assert bits_equal(y.cpu().numpy()[:2], want[[1, 2]])


# ---------------------------------------------------------------- gemm on tensor cores (t >= 16)

@pytest.mark.parametrize("t", [16, 17, 40, 64, 100, 300])
@pytest.mark.parametrize("rows,cols", [(4096, 4096), (200, 12288), (129, 96), (1, 4128)])
def test_gemm_tensor_cores(cuda, runtime, rtb, oracle, t, rows, cols):
    """BASELINE config 4 sizes and ragged ones: row tiles cut by the matrix end, K not a
    multiple of the 64-column stage, several token passes (t = 300 > 256). Tiles of up to 64
    tokens run two CTAs per SM; t = 100 (a 112-token tile) and more run one, with two
    accumulators up to 128 tokens."""
    m = Mat(cuda, rtb, oracle, rows, cols, 101)
    x = xs(oracle, t, cols, 102)
    xd = dev(cuda, x)
    y = cuda.full((t, rows), float("nan"), dtype=cuda.float32, device="cuda")
    runtime.gemm(m.ptr, rows, cols, xd.data_ptr(), t, y.data_ptr())
    got = y.cpu().numpy()
    assert np.isfinite(got).all()
    assert rel_err(got, oracle.gemm(m.q8, rows, cols, x, t)) < TC_TOL


@pytest.mark.parametrize("rows,cols", [(12288, 4096), (4096, 12288)])
def test_gemm_prompt_512(cuda, runtime, rtb, oracle, rows, cols):
    """BASELINE config 4 at M = 512 on gate/up and down shapes; checked on a row sample (the CPU
    oracle over all rows would take minutes) plus full-output properties."""
    t = 512
    m = Mat(cuda, rtb, oracle, rows, cols, 111, host=False)
    x = xs(oracle, t, cols, 112)
    xd = dev(cuda, x)
    y = cuda.full((t, rows), float("nan"), dtype=cuda.float32, device="cuda")
    runtime.gemm(m.ptr, rows, cols, xd.data_ptr(), t, y.data_ptr())
    got = y.cpu().numpy()
    assert np.isfinite(got).all()
    sel = np.sort(np.random.default_rng(3).choice(rows, 96, replace=False))
    q8 = np.concatenate([oracle.synth_q8_0(1, cols, SEED, 111, row0=int(r)) for r in sel])
    want = oracle.gemm(q8, len(sel), cols, x, t)
    assert rel_err(got[:, sel], want) < TC_TOL


@pytest.mark.parametrize("t", [16, 48])
def test_swiglu_tensor_cores(cuda, runtime, rtb, oracle, t):
    rows, cols = 1536, 4096
    g = Mat(cuda, rtb, oracle, rows, cols, 121)
    u = Mat(cuda, rtb, oracle, rows, cols, 122)
    x = xs(oracle, t, cols, 123)
    xd = dev(cuda, x)
    h = cuda.full((t, rows), float("nan"), dtype=cuda.float32, device="cuda")
    runtime.gemm_silu(g.ptr, u.ptr, rows, cols, xd.data_ptr(), t, h.data_ptr())
    yg = oracle.gemm(g.q8, rows, cols, x, t).astype(np.float64)
    yu = oracle.gemm(u.q8, rows, cols, x, t).astype(np.float64)
    assert rel_err(h.cpu().numpy(), yg / (1.0 + np.exp(-yg)) * yu) < 2 * TC_TOL


def test_tensor_core_round_mixed_with_cuda_core(cuda, runtime, rtb, oracle):
    """A queued round holding a t = 1 product, a t = 2 product and a t = 24 product."""
    cols = 4096
    a = Mat(cuda, rtb, oracle, 1024, cols, 131)
    x = xs(oracle, 24, cols, 132)
    xd = dev(cuda, x)
    y1 = cuda.empty(1024, dtype=cuda.float32, device="cuda")
    y2 = cuda.empty((2, 1024), dtype=cuda.float32, device="cuda")
    y24 = cuda.empty((24, 1024), dtype=cuda.float32, device="cuda")
    runtime.gemv_q(a.ptr, 1024, cols, xd.data_ptr(), y1.data_ptr())
    runtime.gemm_q(a.ptr, 1024, cols, xd.data_ptr(), 2, y2.data_ptr())
    runtime.gemm_q(a.ptr, 1024, cols, xd.data_ptr(), 24, y24.data_ptr())
    runtime.gemv_go()
    want = oracle.gemm(a.q8, 1024, cols, x, 24)
    assert bits_equal(y1.cpu().numpy(), want[0])
    assert bits_equal(y2.cpu().numpy(), want[:2])
    assert rel_err(y24.cpu().numpy(), want) < TC_TOL


@pytest.mark.parametrize("overlap", [False, True])
def test_dependent_chain_async(cuda, rtb, oracle, overlap):
    """Products whose x is the previous product's y, enqueued back to back (async; with overlap the
    kernels are launched so that the next one streams its weights while the previous finishes):
    every y must still see its x complete."""
    rows = cols = 4096
    a = Mat(cuda, rtb, oracle, rows, cols, 141)
    b = Mat(cuda, rtb, oracle, rows, cols, 142)
    x = xs(oracle, 16, cols, 143)
    rt = rtb.Runtime()
    try:
        rt.set_async(True)
        rt.set_overlap(overlap)
        xd = dev(cuda, x)
        ys = [cuda.empty((16, rows), dtype=cuda.float32, device="cuda") for _ in range(4)]
        # t = 1 chain: x -> A -> B -> A -> B
        rt.gemv(a.ptr, rows, cols, xd[0].data_ptr(), ys[0][0].data_ptr())
        rt.gemv(b.ptr, rows, cols, ys[0][0].data_ptr(), ys[1][0].data_ptr())
        rt.gemv(a.ptr, rows, cols, ys[1][0].data_ptr(), ys[2][0].data_ptr())
        rt.gemv(b.ptr, rows, cols, ys[2][0].data_ptr(), ys[3][0].data_ptr())
        rt.sync()
        want = x[0]
        for k, m in enumerate([a, b, a, b]):
            want = oracle.gemv(m.q8, rows, cols, want)
            assert bits_equal(ys[k][0].cpu().numpy(), want), k
        # t = 16 chain on the tensor cores: X -> A -> B
        rt.gemm(a.ptr, rows, cols, xd.data_ptr(), 16, ys[0].data_ptr())
        rt.gemm(b.ptr, rows, cols, ys[0].data_ptr(), 16, ys[1].data_ptr())
        rt.sync()
        y0 = ys[0].cpu().numpy()
        assert rel_err(y0, oracle.gemm(a.q8, rows, cols, x, 16)) < TC_TOL
        assert rel_err(ys[1].cpu().numpy(), oracle.gemm(b.q8, rows, cols, y0, 16)) < TC_TOL
    finally:
        rt.close()


# ---------------------------------------------------------------- tensor cores: any fp32 x, any fp16 scale

def _banded_q8(oracle, bands, cols, stream):
    """GGUF Q8_0 rows in bands of different weight scales, [(rows, sigma), ...]."""
    return np.concatenate([oracle.synth_q8_0(r, cols, SEED, stream + 7 * k, sigma=s) for k, (r, s) in enumerate(bands)])


def _worst_block_err(got, ref, cuts):
    """rel_err per (token, row band), each with its own rms floor: a band of tiny weights is held to
    the same 2e-3 as the others instead of hiding under their magnitude."""
    return max(rel_err(got[k, a:b], ref[k, a:b]) for k in range(got.shape[0]) for a, b in zip(cuts[:-1], cuts[1:]))


@pytest.mark.parametrize("t,cols", [(16, 4096), (40, 4096), (100, 4096), (24, 12288)])
def test_tensor_cores_take_any_fp32_range(cuda, runtime, rtb, oracle, t, cols):
    """The reference takes any fp32 x and any fp16 scale (src/card/gemm.c:271-294). Rows whose
    scales are ~2e-7 (fp16 subnormals: q*d underflows fp16) or ~2000 (q*d overflows it) sit in the
    same tiles as ordinary rows, and tokens hold entries of +-1e5 (beyond fp16), values ~1e-6
    (fp16 subnormals) or ~1e4 throughout. Each (token, row band) is within 2e-3 of the reference's
    fp32 y. (cols = 12288 with few row tiles: the K range is split, partial sums reduced.)"""
    bands = [(160, 0.02), (96, 1e-5), (64, 1e5), (200, 0.02), (33, 3e-6)]
    rows = sum(r for r, _ in bands)
    cuts = np.cumsum([0] + [r for r, _ in bands])
    q8 = _banded_q8(oracle, bands, cols, 161)
    w = dev(cuda, oracle.repack_split(q8, rows, cols))
    x = xs(oracle, t, cols, 162)
    x[0, ::97] = 1e5
    x[1, 5] = -1e5
    x[2] *= 1e-6
    x[3] *= 1e4
    x[4, :] = 0.0
    xd = dev(cuda, x)
    y = cuda.full((t, rows), float("nan"), dtype=cuda.float32, device="cuda")
    runtime.gemm(w.data_ptr(), rows, cols, xd.data_ptr(), t, y.data_ptr())
    got = y.cpu().numpy()
    want = oracle.gemm(q8, rows, cols, x, t)
    assert np.isfinite(got).all()
    assert np.array_equal(got[4], np.zeros(rows, dtype=np.float32))
    assert _worst_block_err(got, want, cuts) < TC_TOL


def test_tensor_core_swiglu_takes_any_fp32_range(cuda, runtime, rtb, oracle):
    """The SwiGLU pair with gate and up rows of very different scales and x with outliers."""
    t, cols = 16, 4096
    gate_bands, up_bands = [(64, 0.02), (64, 1e-5)], [(64, 1e3), (64, 0.02)]
    rows = 128
    gq, uq = _banded_q8(oracle, gate_bands, cols, 171), _banded_q8(oracle, up_bands, cols, 172)
    g, u = dev(cuda, oracle.repack_split(gq, rows, cols)), dev(cuda, oracle.repack_split(uq, rows, cols))
    x = xs(oracle, t, cols, 173)
    x[0, 11] = 3e4
    x[1] *= 1e-6
    xd = dev(cuda, x)
    h = cuda.full((t, rows), float("nan"), dtype=cuda.float32, device="cuda")
    runtime.gemm_silu(g.data_ptr(), u.data_ptr(), rows, cols, xd.data_ptr(), t, h.data_ptr())
    yg = oracle.gemm(gq, rows, cols, x, t).astype(np.float64)
    yu = oracle.gemm(uq, rows, cols, x, t).astype(np.float64)
    got = h.cpu().numpy()
    assert np.isfinite(got).all()
    assert _worst_block_err(got, yg / (1.0 + np.exp(-yg)) * yu, [0, 64, 128]) < 2 * TC_TOL


# ---------------------------------------------------------------- BASELINE configs 3a and 4 at their own shapes

CONFIG_SHAPES = {"qkv": (8192, 4096), "out": (4096, 4096), "down": (4096, 12288), "head": (151936, 4096)}


def _row_sample(rows: int, n: int = 96, seed: int = 5) -> np.ndarray:
    """A seeded sample of output rows plus both ends of the matrix (the first and last row tiles)."""
    sel = set(np.random.default_rng(seed).choice(rows, n, replace=False).tolist()) | {0, 1, rows - 2, rows - 1}
    return np.array(sorted(sel))


def _sample_q8(oracle, sel, cols, stream):
    return np.concatenate([oracle.synth_q8_0(1, cols, SEED, stream, row0=int(r)) for r in sel])


@pytest.mark.parametrize("t", [2, 4, 16, 40])
@pytest.mark.parametrize("shape", ["qkv", "out", "down", "head"])
def test_config_shapes_on_a_row_sample(cuda, runtime, rtb, oracle, shape, t):
    """The verify pass (M = 2, config 3a), M = 4, and the prompt products at M = 16 and 40 (config
    4) on the full BASELINE matrices, the 151936 x 4096 head included: the sampled rows bit for bit
    below 16 tokens, within 2e-3 from 16 (the two-CTA tensor-core shape)."""
    rows, cols = CONFIG_SHAPES[shape]
    m = Mat(cuda, rtb, oracle, rows, cols, 151, host=False)
    x = xs(oracle, t, cols, 152)
    xd = dev(cuda, x)
    y = cuda.full((t, rows), float("nan"), dtype=cuda.float32, device="cuda")
    runtime.gemm(m.ptr, rows, cols, xd.data_ptr(), t, y.data_ptr())
    got = y.cpu().numpy()
    assert np.isfinite(got).all()
    sel = _row_sample(rows)
    want = oracle.gemm(_sample_q8(oracle, sel, cols, 151), len(sel), cols, x, t)
    if t < TC_MIN_T:
        assert bits_equal(got[:, sel], want)
    else:
        assert rel_err(got[:, sel], want) < TC_TOL


@pytest.mark.parametrize("t", [1, 2, 16, 40])
def test_gate_up_config_shape_on_a_row_sample(cuda, runtime, rtb, oracle, t):
    """The fused gate+up+SiLU pair at its BASELINE shape (2 x 12288 x 4096) on a row sample."""
    rows, cols = 12288, 4096
    g = Mat(cuda, rtb, oracle, rows, cols, 181, host=False)
    u = Mat(cuda, rtb, oracle, rows, cols, 182, host=False)
    x = xs(oracle, t, cols, 183)
    xd = dev(cuda, x)
    h = cuda.full((t, rows), float("nan"), dtype=cuda.float32, device="cuda")
    runtime.gemm_silu(g.ptr, u.ptr, rows, cols, xd.data_ptr(), t, h.data_ptr())
    sel = _row_sample(rows)
    yg = oracle.gemm(_sample_q8(oracle, sel, cols, 181), len(sel), cols, x, t).astype(np.float64)
    yu = oracle.gemm(_sample_q8(oracle, sel, cols, 182), len(sel), cols, x, t).astype(np.float64)
    tol = 1e-5 if t < TC_MIN_T else 2 * TC_TOL
    assert rel_err(h.cpu().numpy()[:, sel], yg / (1.0 + np.exp(-yg)) * yu) < tol
