"""Chained launches (rt_b200_chain_begin / rt_b200_chain_end, GPU).

A chain runs recorded rounds as one persistent launch; a round waits on the device for every
earlier round whose y its x reads, or whose x or y its y overwrites. In the decode-layer tests
each round feeds the next (x of round r+1 is y of round r, with
the shapes of a decode layer), so a round that read its x early would read the NaNs the buffers
start with. Every product is checked bit for bit against the oracle applied to the x the GPU
actually fed it (the SwiGLU pair within 1e-5, as in test_gpu_products).
"""
from __future__ import annotations

import numpy as np
import pytest

from test_gpu_products import Mat, bits_equal, dev, rel_err, xs

pytestmark = pytest.mark.gpu


def _layer(cuda, rtb, oracle):
    D, Q, F = 4096, 8192, 1536
    m = {"qkv": Mat(cuda, rtb, oracle, Q, D, 61), "out": Mat(cuda, rtb, oracle, D, Q, 62),
         "gate": Mat(cuda, rtb, oracle, F, D, 63), "up": Mat(cuda, rtb, oracle, F, D, 64),
         "down": Mat(cuda, rtb, oracle, D, F, 65)}
    nan = float("nan")
    buf = {"x0": dev(cuda, xs(oracle, 1, D, 66)), "y0": cuda.full((Q,), nan, device="cuda"),
           "y1": cuda.full((D,), nan, device="cuda"), "h": cuda.full((F,), nan, device="cuda"),
           "y3": cuda.full((D,), nan, device="cuda"), "y4": cuda.full((1000,), nan, device="cuda")}
    idx = np.random.default_rng(7).choice(Q, 1000, replace=False).astype(np.int32)
    buf["idx"] = dev(cuda, idx)
    return m, buf, idx


def _record(rt, m, buf):
    D, Q, F = 4096, 8192, 1536
    rt.gemv(m["qkv"].ptr, Q, D, buf["x0"].data_ptr(), buf["y0"].data_ptr())
    rt.gemv(m["out"].ptr, D, Q, buf["y0"].data_ptr(), buf["y1"].data_ptr())  # two 4096-column stages per row
    rt.gemm_silu(m["gate"].ptr, m["up"].ptr, F, D, buf["y1"].data_ptr(), 1, buf["h"].data_ptr())
    rt.gemv(m["down"].ptr, D, F, buf["h"].data_ptr(), buf["y3"].data_ptr())
    rt.gemv_rows(m["qkv"].ptr, Q, buf["idx"].data_ptr(), 1000, D, buf["y3"].data_ptr(), buf["y4"].data_ptr())


def _check(oracle, m, buf, idx):
    D, Q, F = 4096, 8192, 1536
    host = {k: v.cpu().numpy() for k, v in buf.items()}
    assert bits_equal(host["y0"], oracle.gemv(m["qkv"].q8, Q, D, host["x0"][0]))
    assert bits_equal(host["y1"], oracle.gemv(m["out"].q8, D, Q, host["y0"]))
    g = oracle.gemv(m["gate"].q8, F, D, host["y1"]).astype(np.float64)
    u = oracle.gemv(m["up"].q8, F, D, host["y1"]).astype(np.float64)
    assert rel_err(host["h"], g / (1.0 + np.exp(-g)) * u) < 1e-5
    assert bits_equal(host["y3"], oracle.gemv(m["down"].q8, D, F, host["h"]))
    assert bits_equal(host["y4"], oracle.gemv_rows(m["qkv"].q8, D, idx, host["y3"]))


@pytest.mark.parametrize("serial", [True, False])
def test_chain_of_dependent_rounds(cuda, rtb, oracle, serial):
    """serial: every round waits for the one before; else the waits come from the x/y overlaps."""
    m, buf, idx = _layer(cuda, rtb, oracle)
    with rtb.Runtime() as rt:
        rt.chain_begin()
        _record(rt, m, buf)
        rt.chain_end(serial=serial)
    _check(oracle, m, buf, idx)


def test_chain_replayed_as_cuda_graph(cuda, rtb, oracle):
    """The round counters are reset inside the captured work: every replay waits afresh."""
    m, buf, idx = _layer(cuda, rtb, oracle)
    with rtb.Runtime() as rt:
        rt.set_async(True)
        g = cuda.cuda.CUDAGraph()
        s = cuda.cuda.Stream()
        s.wait_stream(cuda.cuda.current_stream())
        with cuda.cuda.stream(s):
            with cuda.cuda.graph(g, stream=s):
                rt.set_stream(cuda.cuda.current_stream().cuda_stream)
                rt.chain_begin()
                _record(rt, m, buf)
                rt.chain_end(serial=True)
        cuda.cuda.current_stream().wait_stream(s)
        rt.set_stream(cuda.cuda.current_stream().cuda_stream)
        for _ in range(3):
            for k in ("y0", "y1", "h", "y3", "y4"):
                buf[k].fill_(float("nan"))
            g.replay()
            cuda.cuda.synchronize()
            _check(oracle, m, buf, idx)
        rt.sync()
        del g


def test_chain_with_unchainable_rounds_runs_them_in_order(cuda, rtb, oracle):
    """t = 16 goes to the tensor cores: the chain falls back to one launch per round, in order."""
    D, Q, t = 4096, 1024, 16
    a = Mat(cuda, rtb, oracle, Q, D, 71)
    b = Mat(cuda, rtb, oracle, D, Q, 72)
    x = dev(cuda, xs(oracle, t, D, 73))
    y0 = cuda.full((t, Q), float("nan"), device="cuda")
    y1 = cuda.full((t, D), float("nan"), device="cuda")
    with rtb.Runtime() as rt:
        rt.chain_begin()
        rt.gemm(a.ptr, Q, D, x.data_ptr(), t, y0.data_ptr())
        rt.gemm(b.ptr, D, Q, y0.data_ptr(), t, y1.data_ptr())
        rt.chain_end()
    h0, h1 = y0.cpu().numpy(), y1.cpu().numpy()
    assert rel_err(h0, oracle.gemm_f64(a.q8, Q, D, x.cpu().numpy(), t)) < 2e-3
    assert rel_err(h1, oracle.gemm_f64(b.q8, D, Q, h0, t)) < 2e-3


def test_chain_misuse_is_an_error(cuda, rtb):
    with rtb.Runtime() as rt:
        with pytest.raises(rtb.RtError):
            rt.chain_end()
        rt.chain_begin()
        with pytest.raises(rtb.RtError):
            rt.chain_begin()
        rt.chain_end()


def test_chain_fan_in_waits_for_every_writer(cuda, rtb, oracle):
    """Round C reads one buffer whose halves rounds A and B write. B finishes first (A's tiles are
    four stages long and ten CTAs run two of them), so C must wait for both writers, not only the
    latest: otherwise the CTAs with one A tile read A's last rows before they are written."""
    ra, rb_, ca, cb = 1264, 784, 16384, 4096  # 158 and 98 eight-row tiles
    a = Mat(cuda, rtb, oracle, ra, ca, 81)
    b = Mat(cuda, rtb, oracle, rb_, cb, 82)
    cm = Mat(cuda, rtb, oracle, 512, ra + rb_, 83)
    xa, xb = dev(cuda, xs(oracle, 1, ca, 84)), dev(cuda, xs(oracle, 1, cb, 85))
    ybuf = cuda.full((ra + rb_,), float("nan"), device="cuda")
    yc = cuda.full((512,), float("nan"), device="cuda")
    with rtb.Runtime() as rt:
        rt.chain_begin()
        rt.gemv(a.ptr, ra, ca, xa.data_ptr(), ybuf.data_ptr())
        rt.gemv(b.ptr, rb_, cb, xb.data_ptr(), ybuf.data_ptr() + 4 * ra)
        rt.gemv(cm.ptr, 512, ra + rb_, ybuf.data_ptr(), yc.data_ptr())
        rt.chain_end(serial=False)
    y = ybuf.cpu().numpy()
    assert bits_equal(y[:ra], oracle.gemv(a.q8, ra, ca, xa.cpu().numpy()[0]))
    assert bits_equal(y[ra:], oracle.gemv(b.q8, rb_, cb, xb.cpu().numpy()[0]))
    assert bits_equal(yc.cpu().numpy(), oracle.gemv(cm.q8, 512, ra + rb_, y))


def test_chain_write_after_read_waits_for_the_reader(cuda, rtb, oracle):
    """Round R writes into the last 4096 columns of round Q's x. Q's tiles are eight stages long
    and 74 CTAs run two of them, reading that part of x last; the other CTAs reach R after one Q
    tile. R must wait for Q, or Q's late tiles read R's output instead of their x."""
    rq, cq, rr, cr = 1776, 32768, 4096, 4096  # Q: 222 eight-row tiles of 8 stages
    qm = Mat(cuda, rtb, oracle, rq, cq, 91)
    rm = Mat(cuda, rtb, oracle, rr, cr, 92)
    x_host = xs(oracle, 1, cq, 93)[0]
    xq = dev(cuda, x_host)
    xr = dev(cuda, xs(oracle, 1, cr, 94))
    yq = cuda.full((rq,), float("nan"), device="cuda")
    with rtb.Runtime() as rt:
        rt.chain_begin()
        rt.gemv(qm.ptr, rq, cq, xq.data_ptr(), yq.data_ptr())
        rt.gemv(rm.ptr, rr, cr, xr.data_ptr(), xq.data_ptr() + 4 * (cq - rr))
        rt.chain_end(serial=False)
    assert bits_equal(yq.cpu().numpy(), oracle.gemv(qm.q8, rq, cq, x_host))
    x_after = xq.cpu().numpy()
    assert bits_equal(x_after[:cq - rr], x_host[:cq - rr])
    assert bits_equal(x_after[cq - rr:], oracle.gemv(rm.q8, rr, cr, xr.cpu().numpy()[0]))
