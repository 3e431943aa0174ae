"""The host-half primitives beside the products (src/host/rt_host.c:128-279) on the GPU, through
the C ABI: every output bit for bit against the oracle's restatement (oracle/prims_oracle.c,
itself pinned to the reference's compiled rt_host.c by tests/test_oracle.py), on decode-sized
and ragged shapes, grouped-query head maps, and the calls that must be refused."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def bits_equal(a, b) -> bool:
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


def _dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


# h query heads, n1 kv heads, c columns, t history rows, r state rows, m x k outer product
SHAPES = [
    (16, 4, 256, 4096, 128, 128, 128),  # a 9B-class decode step's head sizes over a 4096-token history
    (32, 8, 128, 1000, 128, 256, 128),
    (5, 2, 8, 1, 1, 1, 8),              # the smallest
    (40, 1, 72, 130, 13, 9, 5),         # 40 heads on one kv head (three groups), c % 32 != 0, ragged t
    (3, 3, 40, 0, 2, 4, 24),            # an empty history
    (64, 8, 128, 2048, 300, 64, 8),     # one thread per output for the dot products (131072 of them)
    (7, 7, 16, 4098, 3, 2, 8),          # t % 4 != 0: the weights' rows are copied 4 bytes at a time
    (6, 8, 64, 300, 5, 7, 9),           # kv heads 1 and 6 never read
    (64, 128, 8, 1200, 2, 3, 8),        # half the kv heads read, 76800 outputs
    (4, 4, 8192, 3, 1, 2, 8),           # 128 KB history rows, 256 ip12_kv slices of 32 columns
]


@pytest.mark.parametrize("shape", SHAPES)
def test_prims_bit_exact(cuda, rtb, oracle, shape):
    h, n1, c, t, r, m, k = shape
    rng = np.random.default_rng(h * 1000 + c)
    f = lambda n: rng.standard_normal(n).astype(np.float32)
    l = np.array([(5 * q + 3) % n1 for q in range(h)], dtype=np.int64)
    kv, b, a, A = f(t * n1 * c), f(h * c), f(h * t), f(h * r * c)
    s, av, bv = f(m * k), f(m), f(k)
    kv_d, b_d, a_d, A_d = (_dev(cuda, v) for v in (kv, b, a, A))
    s_d, av_d, bv_d = (_dev(cuda, v) for v in (s, av, bv))
    z1 = cuda.full((max(h * t, 1),), float("nan"), device="cuda")
    z2 = cuda.full((h * c,), float("nan"), device="cuda")
    z3 = cuda.full((h * r,), float("nan"), device="cuda")
    z4 = cuda.full((m * k,), float("nan"), device="cuda")
    with rtb.Runtime() as rt:
        for async_mode in (False, True):
            rt.set_async(async_mode)
            rt.ip21_kv(z1.data_ptr(), kv_d.data_ptr(), n1, c, l, h, t, b_d.data_ptr())
            rt.ip12_kv(z2.data_ptr(), a_d.data_ptr(), kv_d.data_ptr(), n1, c, l, h, t)
            rt.ip21(z3.data_ptr(), A_d.data_ptr(), h, r, c, b_d.data_ptr())
            rt.scale_outer(z4.data_ptr(), s_d.data_ptr(), 0.9375, av_d.data_ptr(), bv_d.data_ptr(), m, k)
            rt.sync()
            if t:
                assert bits_equal(z1.cpu().numpy()[:h * t], oracle.ip21_kv(kv, n1, c, l, h, t, b)), async_mode
            assert bits_equal(z2.cpu().numpy(), oracle.ip12_kv(a, kv, n1, c, l, h, t)), async_mode
            assert bits_equal(z3.cpu().numpy(), oracle.ip21(A, h, r, c, b)), async_mode
            assert bits_equal(z4.cpu().numpy(), oracle.scale_outer(s, 0.9375, av, bv, m, k)), async_mode
            for z in (z1, z2, z3, z4):
                z.fill_(float("nan"))


def test_prims_refuse_bad_calls(cuda, rtb):
    """c not a multiple of 8, a kv head outside [0, n1), too many heads, a misaligned kv: each is
    refused with RTB_EINVAL and nothing runs; the runtime stays usable."""
    kv = cuda.zeros(4096, device="cuda")
    z = cuda.zeros(4096, device="cuda")
    b = cuda.zeros(4096, device="cuda")
    with rtb.Runtime() as rt:
        with pytest.raises(rtb.RtError) as e:
            rt.ip21_kv(z.data_ptr(), kv.data_ptr(), 1, 12, [0], 1, 4, b.data_ptr())
        assert e.value.code == 1  # RTB_EINVAL
        with pytest.raises(rtb.RtError):
            rt.ip12_kv(z.data_ptr(), b.data_ptr(), kv.data_ptr(), 2, 8, [0, 2], 2, 4)
        with pytest.raises(rtb.RtError):
            rt.ip21(z.data_ptr(), kv.data_ptr(), 129, 1, 8, b.data_ptr())
        with pytest.raises(rtb.RtError):
            rt.ip12_kv(z.data_ptr(), b.data_ptr(), kv.data_ptr() + 4, 1, 8, [0], 1, 4)
        rt.ip21(z.data_ptr(), kv.data_ptr(), 1, 1, 8, b.data_ptr())
        rt.sync()


def test_ip12_kv_unaligned_weights(cuda, rtb, oracle):
    """a 4 bytes off a 16-byte boundary (allowed: 4-byte alignment): the weights then go through
    shared memory 4 bytes at a time; bit for bit all the same."""
    h, n1, c, t = 6, 2, 64, 512
    rng = np.random.default_rng(3)
    kv = rng.standard_normal(t * n1 * c).astype(np.float32)
    a = rng.standard_normal(h * t).astype(np.float32)
    l = np.array([0, 1, 1, 0, 1, 0], dtype=np.int64)
    kv_d = _dev(cuda, kv)
    a_buf = cuda.empty(h * t + 4, device="cuda")
    a_buf[1:1 + h * t] = _dev(cuda, a)
    z = cuda.full((h * c,), float("nan"), device="cuda")
    with rtb.Runtime() as rt:
        rt.ip12_kv(z.data_ptr(), a_buf.data_ptr() + 4, kv_d.data_ptr(), n1, c, l, h, t)
    assert bits_equal(z.cpu().numpy(), oracle.ip12_kv(a, kv, n1, c, l, h, t))
