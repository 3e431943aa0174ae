"""Failure detection on the GPU without a fault: every device wait in the product kernels is
bounded and reports through the context's error word. Here a kernel waits on a device counter that
nothing advances and on an mbarrier that nothing arrives on; each wait gives up after about a
second, the host reads RTB_EKERNEL with both waits named, and the same runtime then computes a
product bit for bit. Collected after the product tests, as it spends about two seconds waiting.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SEED = 20261201


def test_stuck_waits_give_up_and_leave_the_runtime_usable(cuda, rtb, oracle):
    with rtb.Runtime() as rt:
        code, msg = rt.wait_probe()
        assert code == 3, (code, msg)  # RTB_EKERNEL
        assert "chained round's dependency never completed" in msg and "bulk copy never completed" in msg, msg
        assert rtb.last_error(rt)[0] == 0  # the record was read and cleared
        rows, cols = 64, 4096
        q8 = oracle.synth_q8_0(rows, cols, SEED, 301)
        w = cuda.from_numpy(oracle.repack_split(q8, rows, cols)).cuda()
        x = oracle.synth_f32(cols, SEED, 302)
        xd = cuda.from_numpy(x).cuda()
        y = cuda.empty(rows, dtype=cuda.float32, device="cuda")
        rt.gemv(w.data_ptr(), rows, cols, xd.data_ptr(), y.data_ptr())
        assert np.array_equal(y.cpu().numpy().view(np.uint32), oracle.gemv(q8, rows, cols, x).view(np.uint32))
