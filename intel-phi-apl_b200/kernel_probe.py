"""Runs one product kernel a few times on a BASELINE shape, through the C ABI, for profiler
captures (ncu) and quick timing:

    python intel-phi-apl_b200/kernel_probe.py --shape head --t 1 --launches 3

Shapes are those of intel-phi-apl_b200/workload.py (gate_up_silu, down, qkv, out, head,
draft_head). Prints one JSON line with the mean CUDA-event time per launch and the algorithmic
bytes and flops of one launch.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

import rtb200  # noqa: E402
import workload as WL  # noqa: E402


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--shape", default="head", choices=[p.name for p in WL.SWEEP] + ["draft_head"])
    ap.add_argument("--t", type=int, default=1)
    ap.add_argument("--launches", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=1)
    a = ap.parse_args()
    import numpy as np
    import torch

    p = WL.DRAFT if a.shape == "draft_head" else next(q for q in WL.SWEEP if q.name == a.shape)
    rt = rtb200.Runtime()
    rt.set_async(True)
    rt.set_stream(torch.cuda.current_stream().cuda_stream)
    nb = rtb200.gemv_s_bytes(p.rows, p.cols)
    w = torch.empty(nb, dtype=torch.uint8, device="cuda")
    rtb200.synth_q8_0(w.data_ptr(), 0, p.rows, p.cols, 1, 1)
    w2 = None
    if p.kind == "silu":
        w2 = torch.empty(nb, dtype=torch.uint8, device="cuda")
        rtb200.synth_q8_0(w2.data_ptr(), 0, p.rows, p.cols, 1, 2)
    x = torch.empty(a.t * p.cols, dtype=torch.float32, device="cuda")
    rtb200.synth_f32(x.data_ptr(), a.t * p.cols, 1, 3)
    nout = p.nsel if p.kind == "rows" else p.rows
    y = torch.empty(a.t * nout, dtype=torch.float32, device="cuda")
    idx = None
    if p.kind == "rows":
        idx = torch.from_numpy(np.random.default_rng(1).choice(p.rows, p.nsel, replace=False).astype(np.int32)).cuda()

    def launch():
        if p.kind == "silu":
            rt.gemm_silu(w.data_ptr(), w2.data_ptr(), p.rows, p.cols, x.data_ptr(), a.t, y.data_ptr())
        elif p.kind == "rows":
            rt.gemv_rows(w.data_ptr(), p.rows, idx.data_ptr(), p.nsel, p.cols, x.data_ptr(), y.data_ptr())
        else:
            rt.gemm(w.data_ptr(), p.rows, p.cols, x.data_ptr(), a.t, y.data_ptr())

    for _ in range(a.warmup):
        launch()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(a.launches)]
    for e0, e1 in ev:
        e0.record()
        launch()
        e1.record()
    torch.cuda.synchronize()
    rt.sync()
    us = sum(e0.elapsed_time(e1) for e0, e1 in ev) / len(ev) * 1e3
    print(json.dumps({"shape": p.name, "rows": p.rows, "cols": p.cols, "t": a.t, "us_per_launch": round(us, 2),
                      "bytes": p.bytes(a.t), "flops": p.flops(a.t), "GB_s": round(p.bytes(a.t) / us / 1e3, 1)}))
    rt.close()


if __name__ == "__main__":
    main()
