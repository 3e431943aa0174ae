"""Row sharding over ranks (CPU, gloo, world size 2).

The library's multi-GPU contract (include/rt_b200.h, rt_b200_shard): with `world` ranks, rank k
holds rows [k*rows/world, (k+1)*rows/world) of every matrix, computes those outputs, and an
all-gather in rank order rebuilds the whole y on every rank. These tests run that contract on CPU
ranks: each rank asks the library for its shard (rt_b200_shard_rows, the split its products use),
loads those rows with the oracle's generator, computes them with the oracle, and gloo all-gathers;
the rebuilt y must be the unsharded product bit for bit. bench.py shards the same way.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ORACLE, PKG


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, case: dict, out) -> None:
    import sys
    sys.path.insert(0, ORACLE)
    sys.path.insert(0, PKG)
    import oracle as O
    import rtb200
    import workload as WL
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rows, cols, t = case["rows"], case["cols"], case["t"]
        r0, n = rtb200.shard_rows(rows, rank, world)  # the library's split
        assert (r0, n) == WL.shard_rows(rows, rank, world)  # the bench's allocation agrees
        q8 = O.synth_q8_0(n, cols, 7, 3, row0=r0)  # this rank's shard only
        x = np.stack([O.synth_f32(cols, 7, 4 + k) for k in range(t)])
        y_local = O.gemm(q8, n, cols, x, t, threads=2)  # [t][n]
        parts = [torch.empty((t, n), dtype=torch.float32) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(y_local))
        y = torch.cat(parts, dim=1).numpy()  # [t][rows], ranks' slices in rank order
        if rank == 0:
            out.put(y)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case", [{"rows": 64, "cols": 256, "t": 1}, {"rows": 96, "cols": 512, "t": 3}])
def test_row_shards_all_gather_rebuild_the_product(case, oracle):
    world = 2
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, case, out)) for r in range(world)]
    for p in procs:
        p.start()
    y = out.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    q8 = oracle.synth_q8_0(case["rows"], case["cols"], 7, 3)
    x = np.stack([oracle.synth_f32(case["cols"], 7, 4 + k) for k in range(case["t"])])
    want = oracle.gemm(q8, case["rows"], case["cols"], x, case["t"])
    assert np.array_equal(y.view(np.uint32), want.view(np.uint32))


def test_shard_rows_partition(rtb):
    import workload as WL
    for rows, world in [(4096, 1), (4096, 2), (151936, 8), (12288, 4)]:
        parts = [rtb.shard_rows(rows, k, world) for k in range(world)]
        assert parts == [WL.shard_rows(rows, k, world) for k in range(world)]
        assert parts[0][0] == 0 and sum(n for _, n in parts) == rows
        assert all(parts[k][0] + parts[k][1] == parts[k + 1][0] for k in range(world - 1))
    with pytest.raises(ValueError):
        WL.shard_rows(100, 0, 8)
    for bad in [(100, 0, 8), (64, 2, 2), (64, -1, 2), (64, 0, 0)]:
        with pytest.raises(rtb.RtError):
            rtb.shard_rows(*bad)


def test_every_baseline_shape_shards_over_8():
    import workload as WL
    for p in WL.SWEEP + [WL.DRAFT]:
        for world in (2, 4, 8):
            WL.shard_rows(p.rows, 0, world)


def _gpu_rank_main(rank: int, world: int, nid: bytes, out) -> None:
    import sys
    sys.path.insert(0, ORACLE)
    sys.path.insert(0, PKG)
    import oracle as O
    import rtb200
    import workload as WL
    torch.cuda.set_device(rank)
    rows, cols, t = 8192, 4096, 2
    r0, n = WL.shard_rows(rows, rank, world)
    w = torch.empty(rtb200.gemv_s_bytes(n, cols), dtype=torch.uint8, device="cuda")
    rtb200.synth_q8_0(w.data_ptr(), r0, n, cols, 11, 5)
    w2 = torch.empty_like(w)
    rtb200.synth_q8_0(w2.data_ptr(), r0, n, cols, 11, 7)
    x = torch.from_numpy(np.stack([O.synth_f32(cols, 11, 6 + k) for k in range(16)])).cuda()
    y = torch.full((t, rows), float("nan"), dtype=torch.float32, device="cuda")
    y1 = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
    ys = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
    y16 = torch.full((16, rows), float("nan"), dtype=torch.float32, device="cuda")
    rounds = []
    with rtb200.Runtime() as rt:
        rt.shard(rank, world, nid)
        peer = rt.peer_gather()
        rt.gemm(w.data_ptr(), rows, cols, x.data_ptr(), t, y.data_ptr())
        rt.gemv(w.data_ptr(), rows, cols, x.data_ptr(), y1.data_ptr())
        rt.gemm_silu(w.data_ptr(), w2.data_ptr(), rows, cols, x.data_ptr(), 1, ys.data_ptr())
        rt.gemm(w.data_ptr(), rows, cols, x.data_ptr(), 16, y16.data_ptr())  # tensor cores, NCCL gather
        # rounds back to back (alternating staging images), each on its own x row, blocking
        for k in range(5):
            yk = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
            rt.gemv(w.data_ptr(), rows, cols, x[k].data_ptr(), yk.data_ptr())
            rounds.append(yk)
        # and async, 21 rounds: the gathers run in batches of 8 on a side stream, the staging
        # images (16) come round again; then a product whose x is part of the last y (not
        # gathered yet: it waits for that gather)
        rt.set_async(True)
        for k in range(21):
            yk = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
            rt.gemv(w.data_ptr(), rows, cols, x[(7 + k) % 16].data_ptr(), yk.data_ptr())
            rounds.append(yk)
        ya = torch.full((rows // 2,), float("nan"), dtype=torch.float32, device="cuda")
        rt.gemv(w.data_ptr(), rows // 2, cols, rounds[-1].data_ptr(), ya.data_ptr())  # x: part of the pending y
        rt.sync()
        rt.set_async(False)
        # one round captured as a CUDA graph and replayed twice: the round count lives on the GPU
        yg = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
        rt.set_async(True)
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                rt.set_stream(torch.cuda.current_stream().cuda_stream)
                rt.gemv(w.data_ptr(), rows, cols, x[6].data_ptr(), yg.data_ptr())
                rt.flush()  # the graph finishes its own last gather
        torch.cuda.current_stream().wait_stream(s)
        rt.set_stream(torch.cuda.current_stream().cuda_stream)
        for _ in range(2):
            yg.fill_(float("nan"))
            g.replay()
            torch.cuda.synchronize()
        rt.sync()
        del g
    out.put((rank, peer, y.cpu().numpy(), y1.cpu().numpy(), ys.cpu().numpy(), y16.cpu().numpy(),
             [r.cpu().numpy() for r in rounds], yg.cpu().numpy(), ya.cpu().numpy()))


@pytest.mark.gpu
def test_row_shards_on_two_gpus(cuda, rtb, oracle):
    """rt_b200_shard on 2 GPUs: each rank computes its rows and y is gathered over NVLink, in
    the product's own kernel for single products of <= 4 tokens (peer stores + flags), through
    NCCL for the tensor-core path. Every rank ends with the whole product, bit for bit (the
    tensor-core one within its tolerance), over repeated rounds and CUDA-graph replays."""
    if cuda.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    nid = rtb.nccl_id()
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    procs = [ctx.Process(target=_gpu_rank_main, args=(r, world, nid, out)) for r in range(world)]
    for p in procs:
        p.start()
    res = [out.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    rows, cols, t = 8192, 4096, 2
    q8 = oracle.synth_q8_0(rows, cols, 11, 5)
    q8u = oracle.synth_q8_0(rows, cols, 11, 7)
    x = np.stack([oracle.synth_f32(cols, 11, 6 + k) for k in range(16)])
    want = oracle.gemm(q8, rows, cols, x[:t], t)
    g = oracle.gemv(q8, rows, cols, x[0])
    u = oracle.gemv(q8u, rows, cols, x[0])
    want_silu = (g / (1.0 + np.exp(-g.astype(np.float64))) * u).astype(np.float32)
    want16 = oracle.gemm_f64(q8, rows, cols, x, 16)
    for _, peer, y, y1, ys, y16, rounds, yg, ya in res:
        assert peer, "the in-kernel gather was not set up"
        assert np.array_equal(y.view(np.uint32), want.view(np.uint32))
        assert np.array_equal(y1.view(np.uint32), want[0].view(np.uint32))
        assert np.max(np.abs(ys - want_silu) / np.maximum(np.abs(want_silu), 1e-3)) < 1e-4
        rms = np.sqrt(np.mean(want16 ** 2))
        assert np.max(np.abs(y16 - want16)) / rms < 2e-3
        for k, yk in enumerate(rounds):
            xk = x[k] if k < 5 else x[(7 + k - 5) % 16]
            assert np.array_equal(yk.view(np.uint32), oracle.gemv(q8, rows, cols, xk).view(np.uint32)), k
        # the product of rows // 2 rows over each rank's first rows // 4 shard rows, its x the first
        # cols entries of the last async round's y: every rank's product is the big matrix's rows
        # [k * rows/2, k * rows/2 + rows/4) for rank k
        xa = rounds[-1][:cols]
        want_a = np.concatenate([oracle.gemv(oracle.synth_q8_0(rows // 4, cols, 11, 5, row0=k * rows // 2), rows // 4,
                                             cols, xa) for k in range(2)])
        assert np.array_equal(ya.view(np.uint32), want_a.view(np.uint32))
        assert np.array_equal(yg.view(np.uint32), oracle.gemv(q8, rows, cols, x[6]).view(np.uint32))
