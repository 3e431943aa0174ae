"""Benchmark of the B200 Q8_0 weight products ("Q8_0 GEMV HBM GB/s and 9B
weight-product tok/s at 1/2/4/8 B200").

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P bench.py --gpus N ...

A step is one 9B-class decode step's weight products: 32 layers of
(QKV 8192x4096, out 4096x4096, gate+up 2x12288x4096 fused with SiLU, down 4096x12288) and the
151936x4096 output head, M = 1 token, synthetic seeded Q8_0 weights (7.5 GB, larger than L2) in
HBM. Every product is one launch of the exact CUDA-core kernel through the library's C ABI; with
N GPUs each holds a row shard of every matrix and each round ends in an NCCL all-gather of y.
The step is captured once as a CUDA graph and replayed (the kernels and collectives it holds are
the ones the eager C-ABI calls launch).

value = algorithmic bytes of the whole step (all ranks' products: N*K*34/32 + x + y per product)
divided by the step time (CUDA events on the launching stream, max over ranks). tok_s = steps/s.

Also reported (rank 0): the M = 2 verify step; e2e through the C ABI with host buffers (per
round: pinned H2D of x, the product, D2H of y, as the reference engine crosses its link each
phase); the config-2 per-shape sweep (N = 1); the config-4 prompt products at M = 16, 40, 512 on the
tensor-core path (N = 1; TFLOP/s and fraction of the measured bf16 peak; --no-prompt skips it); the
roofline of the gemv kernel on the output head; the reference's own CPU implementation on a sample
(oracle/_ref, N = 1); SM clocks sampled during the timed region.

--impl reference: the reference's CPU implementation of the product (its host-model gemv_i_thread
built from its sources, oracle/_ref) on all host cores, same metric and unit, each step a bounded
sample (five decode layers' five products each). Rank 0 only.

Two single-purpose modes, for profiler captures and the loader (one JSON line each, 1 GPU):

    python bench.py --probe SHAPE [--t T] [--launches N]   one product kernel on a BASELINE shape
        (gate_up_silu, down, qkv, out, head, draft_head) through the C ABI, N timed launches
    python bench.py --load [--load-layers L] [--dir DIR]    rt_b200_load_gguf on a synthetic GGUF of
        L decode layers plus the head (written to DIR, then removed)
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "intel-phi-apl_b200")
sys.path.insert(0, PKG)

import workload as WL  # noqa: E402

SEED = 20261201
METRIC = "Q8_0 weight-product GB/s, 9B decode step (M=1)"
PEAKS_PATH = os.path.join(ROOT, "MEASURED_PEAKS.json")
TRAFFIC_PATH = os.path.join(ROOT, "profiles", "gemv_exact_head_151936x4096.md")
STEP_TRAFFIC_PATH = os.path.join(ROOT, "profiles", "gemv_exact_down_gateup_m1.md")


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def peaks() -> tuple[float, str]:
    try:
        with open(PEAKS_PATH) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def tensor_peak() -> tuple[float, str]:
    """Dense bf16 TFLOP/s: the burst cuBLAS figure (a kernel timed alone)."""
    try:
        with open(PEAKS_PATH) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 1590.0, "fallback"


# ---------------------------------------------------------------- the reference's CPU path

CPU_LAYERS = 5  # 5 x 214 MB of distinct matrices: larger than a server CPU's L3, so DRAM-bound as the step is
CPU_MIN_SECONDS = 10.0  # the B200 arm's CPU baseline times at least this much work


def cpu_sample_matrices(layers: int = CPU_LAYERS):
    """`layers` decode layers' five products each (QKV, out, gate, up, down) as GGUF Q8_0 bytes
    from the seeded CPU generator (distinct matrices per layer), plus fp32 x vectors."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    threads = len(os.sched_getaffinity(0))
    mats = []
    for layer in range(layers):
        for i, (name, rows, cols) in enumerate([("qkv", WL.QKV, WL.D), ("out", WL.D, WL.D), ("gate", WL.FF, WL.D),
                                                ("up", WL.FF, WL.D), ("down", WL.D, WL.FF)]):
            q8 = O.synth_q8_0(rows, cols, SEED, 500 + 10 * layer + i, threads=threads)
            x = O.synth_f32(cols, SEED, 600 + 10 * layer + i)
            mats.append((name, rows, cols, q8, x))
    return O, mats


def cpu_model() -> str:
    """The host CPU's model name (/proc/cpuinfo), for the baseline's description."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown CPU"


def reference_cpu(steps: int, warmup: int, min_seconds: float = 0.0) -> dict:
    """The reference's host implementation (oracle/_ref: its gemv_i_repack + gemv_i_thread over
    the lane-exact host model, team of all host threads pinned to CPUs 0..n-1). One sample is one
    pass over CPU_LAYERS layers' products; at least `steps` samples are timed, and more until
    `min_seconds` of timed work."""
    O, mats = cpu_sample_matrices()
    if not O.ref_available():
        raise RuntimeError("oracle/_ref/libq8ref.so missing (make -C oracle ref, with the reference tree)")
    threads = len(os.sched_getaffinity(0))
    refs = []
    while mats:  # each GGUF copy is dropped once its form-I copy exists
        _, rows, cols, q8, x = mats.pop(0)
        refs.append((O.RefMatrix(q8, rows, cols, threads=threads), x, rows, cols))
    nbytes = sum(rows * cols * 34 // 32 + 4 * cols + 4 * rows for _, _, rows, cols in refs)
    times = []
    k = 0
    while len(times) < steps or sum(times) < min_seconds:
        t0 = time.perf_counter()
        for m, x, rows, cols in refs:
            m.gemv(x)
        dt = time.perf_counter() - t0
        if k >= warmup:
            times.append(dt)
        k += 1
    med = statistics.median(times)
    return {"value": nbytes / med / 1e9, "unit": "GB/s", "cores": threads, "kind": "reference",
            "sample": f"{CPU_LAYERS} decode layers' 5 Q8_0 products each (QKV, out, gate, up, down; distinct "
                      f"matrices, {nbytes / 1e6:.0f} MB, larger than the host's L3) at M=1, median of {len(times)} "
                      f"samples ({sum(times):.1f} s timed) after {warmup} warm-up, the reference's gemv_i_thread "
                      f"on a team of {threads} pinned threads ({cpu_model()})", "ms_per_sample": med * 1e3}


# ---------------------------------------------------------------- clocks

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus: list[int]):
        self.proc = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", ",".join(map(str, gpus)), "-lms", "50"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        none = {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}  # no nvidia-smi, or too short
        if self.proc is None:
            return none
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, smax, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            p = [s.strip() for s in line.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                smax = max(smax, float(p[2]))
            except ValueError:
                continue
            for n, v in zip(names, p[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return none
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- the B200 arm

class Bench:
    def __init__(self, args, rank: int, world: int):
        import torch

        import rtb200
        self.torch, self.rtb = torch, rtb200
        self.args, self.rank, self.world = args, rank, world
        self.layers = args.layers
        self.rt = rtb200.Runtime()
        if world > 1:
            nid = torch.zeros(128, dtype=torch.uint8, device="cuda")
            if rank == 0:
                nid.copy_(torch.frombuffer(bytearray(rtb200.nccl_id()), dtype=torch.uint8))
            torch.distributed.broadcast(nid, 0)
            self.rt.shard(rank, world, bytes(nid.cpu().numpy().tobytes()))
        self.launches_per_step = 0
        self._alloc()

    def _mat(self, rows: int, cols: int, stream: int):
        r0, n = WL.shard_rows(rows, self.rank, self.world)
        t = self.torch.empty(self.rtb.gemv_s_bytes(n, cols), dtype=self.torch.uint8, device="cuda")
        self.rtb.synth_q8_0(t.data_ptr(), r0, n, cols, SEED, stream)
        return t

    def _alloc(self):
        torch = self.torch
        self.w = []
        for layer in range(self.layers):
            s = 1000 * (layer + 1)
            self.w.append({"qkv": self._mat(WL.QKV, WL.D, s + 1), "out": self._mat(WL.D, WL.D, s + 2),
                           "gate": self._mat(WL.FF, WL.D, s + 3), "up": self._mat(WL.FF, WL.D, s + 4),
                           "down": self._mat(WL.D, WL.FF, s + 5)})
        self.head = self._mat(WL.VOCAB, WL.D, 99)
        self.x = {}
        self.y = {}
        for m in (1, 2):
            for name, cols in (("d", WL.D), ("ff", WL.FF)):
                t = torch.empty(m * cols, dtype=torch.float32, device="cuda")
                self.rtb.synth_f32(t.data_ptr(), m * cols, SEED, 7 + cols + m)
                self.x[(name, m)] = t
            for name, rows in (("qkv", WL.QKV), ("out", WL.D), ("h", WL.FF), ("down", WL.D), ("head", WL.VOCAB)):
                self.y[(name, m)] = torch.empty(m * rows, dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()

    def step(self, m: int) -> int:
        """One decode step's products through the C ABI (async: enqueued on the runtime's stream).
        Returns the launches it made."""
        rt, x, y = self.rt, self.x, self.y
        xd, xf = x[("d", m)].data_ptr(), x[("ff", m)].data_ptr()
        for L in self.w:
            rt.gemm(L["qkv"].data_ptr(), WL.QKV, WL.D, xd, m, y[("qkv", m)].data_ptr())
            rt.gemm(L["out"].data_ptr(), WL.D, WL.D, xd, m, y[("out", m)].data_ptr())
            rt.gemm_silu(L["gate"].data_ptr(), L["up"].data_ptr(), WL.FF, WL.D, xd, m, y[("h", m)].data_ptr())
            rt.gemm(L["down"].data_ptr(), WL.D, WL.FF, xf, m, y[("down", m)].data_ptr())
        rt.gemm(self.head.data_ptr(), WL.VOCAB, WL.D, xd, m, y[("head", m)].data_ptr())
        rt.flush()  # with row shards: the step waits for its last gathers (side stream)
        n = 4 * len(self.w) + 1
        return n + ((n + 7) // 8 if self.world > 1 and rt.peer_gather() else 0)  # + a gather per 8 rounds

    def barrier(self):
        if self.world > 1:
            self.torch.distributed.barrier()

    def max_over_ranks(self, v: float) -> float:
        if self.world == 1:
            return v
        t = self.torch.tensor([v], dtype=self.torch.float64, device="cuda")
        self.torch.distributed.all_reduce(t, op=self.torch.distributed.ReduceOp.MAX)
        return float(t.item())

    def capture(self, m: int):
        torch = self.torch
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                self.rt.set_stream(torch.cuda.current_stream().cuda_stream)
                n = self.step(m)
        torch.cuda.current_stream().wait_stream(s)
        self.rt.set_stream(torch.cuda.current_stream().cuda_stream)
        return g, n

    def timed(self, g, steps: int) -> float:
        torch = self.torch
        self.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        self.barrier()
        return self.max_over_ranks(e0.elapsed_time(e1) / steps)

    def run(self) -> dict:
        torch, args = self.torch, self.args
        rt = self.rt
        rt.set_async(True)
        rt.set_overlap(True)  # weights are read-only through the step: products overlap (PDL)
        rt.set_stream(torch.cuda.current_stream().cuda_stream)
        for m in (1, 2):  # eager warm-up through the C ABI (also sets kernel attributes)
            for _ in range(args.warmup):
                self.step(m)
        torch.cuda.synchronize()
        rt.sync()
        g1, n1 = self.capture(1)
        g2, n2 = self.capture(2)
        for _ in range(args.warmup):
            g1.replay()
            g2.replay()
        torch.cuda.synchronize()
        clocks = ClockSampler(list(range(self.world))) if self.rank == 0 else None
        ms1 = self.timed(g1, args.steps)
        ms2 = self.timed(g2, args.steps)
        clk = clocks.stop() if clocks else None
        rt.sync()
        res = {"ms1": ms1, "ms2": ms2, "launches": args.steps * (n1 + n2), "clocks": clk}
        del g1, g2  # graphs holding NCCL work go before the process group
        torch.cuda.synchronize()
        res["head_launch"] = self.head_launch(args.steps)
        res["e2e"] = self.e2e(max(3, min(args.steps, 10)), args.warmup)
        if self.world == 1 and self.rank == 0:
            clocks = ClockSampler([0])
            res["sweep"] = self.sweep()
            res["sweep"]["clocks"] = clocks.stop()
            if not self.args.no_prompt:
                clocks = ClockSampler([0])
                res["prompt"] = self.prompt()
                res["prompt"]["clocks"] = clocks.stop()
            clocks = ClockSampler([0])
            res["prims"] = self.prims()
            res["prims"]["clocks"] = clocks.stop()
        return res

    def head_launch(self, steps: int) -> dict:
        """The gemv kernel alone on the output head (this rank's shard, 661 MB at N=1: larger
        than L2), each launch timed with CUDA events on its stream."""
        torch = self.torch
        rt = self.rtb.Runtime()  # unsharded: the local product alone, no collective
        rt.set_stream(torch.cuda.current_stream().cuda_stream)
        rt.set_async(True)
        rt.set_overlap(True)
        r0, n = WL.shard_rows(WL.VOCAB, self.rank, self.world)
        yl = torch.empty(n, dtype=torch.float32, device="cuda")
        xd = self.x[("d", 1)].data_ptr()
        for _ in range(3):
            rt.gemv(self.head.data_ptr(), n, WL.D, xd, yl.data_ptr())
        torch.cuda.synchronize()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for a, b in ev:
            a.record()
            rt.gemv(self.head.data_ptr(), n, WL.D, xd, yl.data_ptr())
            b.record()
        torch.cuda.synchronize()
        rt.sync()
        rt.close()
        dur = statistics.mean(a.elapsed_time(b) for a, b in ev) / 1e3
        nbytes = n * WL.D * 34 // 32 + 4 * WL.D + 4 * n
        peak, how = peaks()
        traffic = None  # ncu dram read+write of one full-head launch, scaled to this shard's rows
        try:
            with open(TRAFFIC_PATH) as f:
                for line in f:
                    if line.startswith("traffic_bytes_per_launch:"):
                        traffic = int(int(line.split(":")[1]) * n / WL.VOCAB)
        except (OSError, ValueError):
            pass
        achieved = nbytes / dur / 1e9
        return {"kernel": "gemv_exact_kernel<1>", "shape": f"{n}x{WL.D} M=1 (output head shard)",
                "achieved": round(achieved, 1), "peak": peak, "peak_kind": how, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": traffic, "algorithmic_bytes": nbytes,
                "us_per_launch": round(dur * 1e6, 2)}

    def e2e(self, steps: int, warmup: int) -> dict:
        """The reference-facing path with host buffers, one round at a time as the reference engine
        runs them, driven from C (intel-phi-apl_b200/engine_rounds.c, eng_run_rounds) against the C
        ABI on the runtime's own stream: per round the product is queued (rt_gemv_q /
        rt_gemm_silu_q), x goes host->device from pinned memory (rt_b200_pull, the engine's
        link_pull), the round runs (rt_gemv_go) and y comes back device->host (rt_b200_push, the
        engine's link_push), which returns once y is on the host. Wall-clock time of whole steps,
        after `warmup` steps. Also timed: the same rounds with direct pushes
        (rt_b200_set_push_direct: the product kernel stores y into the pinned host buffer itself
        and raises a host flag, which push polls), and opened before x is pulled (rt_gemv_open:
        the round's kernel is launched at once and streams its weights, gated on the GPU until
        go). Both measure slower in this loop, where each round's pull follows the previous
        round at once."""
        import ctypes as C
        torch, rt = self.torch, self.rt
        rt.set_async(True)
        rt.set_stream(None)  # the runtime's own stream, as a C engine uses it
        torch.cuda.synchronize()
        hx = {k: v.cpu().pin_memory() for k, v in self.x.items() if k[1] == 1}
        hy = {k: torch.empty(v.numel(), dtype=torch.float32).pin_memory() for k, v in self.y.items() if k[1] == 1}
        xd, xf = self.x[("d", 1)], self.x[("ff", 1)]
        y = self.y

        class Round(C.Structure):
            _fields_ = [("kind", C.c_int), ("open", C.c_int), ("w", C.c_void_p), ("w2", C.c_void_p),
                        ("rows", C.c_long), ("cols", C.c_long), ("t", C.c_long), ("x_dev", C.c_void_p),
                        ("x_host", C.c_void_p), ("x_bytes", C.c_size_t), ("y_dev", C.c_void_p),
                        ("y_host", C.c_void_p), ("y_bytes", C.c_size_t)]

        spec = []  # (kind, w, w2, rows, cols, x name, y name); every round opened until the plain run
        for L in self.w:
            spec += [(0, L["qkv"], None, WL.QKV, WL.D, "d", "qkv"), (0, L["out"], None, WL.D, WL.D, "d", "out"),
                     (1, L["gate"], L["up"], WL.FF, WL.D, "d", "h"), (0, L["down"], None, WL.D, WL.FF, "ff", "down")]
        spec.append((0, self.head, None, WL.VOCAB, WL.D, "d", "head"))
        rounds = (Round * len(spec))()
        for i, (kind, w, w2, rows, cols, nx, ny) in enumerate(spec):
            xdev = xd if nx == "d" else xf
            rounds[i] = Round(kind, 1, w.data_ptr(), w2.data_ptr() if w2 is not None else None, rows, cols, 1,
                              xdev.data_ptr(), hx[(nx, 1)].data_ptr(), xdev.numel() * 4, y[(ny, 1)].data_ptr(),
                              hy[(ny, 1)].data_ptr(), y[(ny, 1)].numel() * 4)
        h2d = sum(r.x_bytes for r in rounds)
        d2h = sum(r.y_bytes for r in rounds)
        eng = C.CDLL(os.path.join(PKG, "libengine_rounds.so"))
        eng.eng_run_rounds.argtypes = [C.POINTER(self.rtb.StructRt), C.POINTER(Round), C.c_int, C.c_int]
        eng.eng_run_rounds.restype = C.c_int

        def timed(n: int) -> float:
            if eng.eng_run_rounds(rt._ref, rounds, len(spec), warmup):
                rt.sync()  # raises with the runtime's message
            self.barrier()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            if eng.eng_run_rounds(rt._ref, rounds, len(spec), n):
                rt.sync()
            torch.cuda.synchronize()
            return self.max_over_ranks((time.perf_counter() - t0) / n)

        dt_open = timed(steps)
        for r in rounds:
            r.open = 0
        dt = timed(steps)
        rt.set_push_direct(True)
        dt_direct = timed(steps)
        rt.set_push_direct(False)
        total = WL.step_bytes(1, self.layers)
        return {"value": round(total / dt / 1e9, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": round(dt * 1e3, 3), "tok_s": round(1.0 / dt, 1),
                "path": "per round, from C (engine_rounds.c): rt_gemv_q / rt_gemm_silu_q, rt_b200_pull of x, "
                        "rt_gemv_go, rt_b200_push of y (pinned host buffers)",
                "direct_pushes": {"ms_per_step": round(dt_direct * 1e3, 3), "value": round(total / dt_direct / 1e9, 1),
                                  "path": "the same with rt_b200_set_push_direct: y written to the host buffer by the "
                                          "product kernel, push polls its host flag"},
                "opened_rounds": {"ms_per_step": round(dt_open * 1e3, 3), "value": round(total / dt_open / 1e9, 1),
                                  "path": "the same with rt_gemv_open before the pull"}}

    def _graph(self, fns):
        """The calls captured as one CUDA graph on a side stream (the runtime follows the stream)."""
        torch, rt = self.torch, self.rt
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                rt.set_stream(torch.cuda.current_stream().cuda_stream)
                for f in fns:
                    f()
        torch.cuda.current_stream().wait_stream(s)
        rt.set_stream(torch.cuda.current_stream().cuda_stream)
        return g

    def _time_graph(self, g, reps: int) -> float:
        """ms per replay (CUDA events on the current stream), after one untimed replay."""
        torch = self.torch
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    def prompt(self) -> dict:
        """the prompt products at M = 16, 40 and 512 tokens on the config-2
        shapes, through rt_gemm / rt_gemm_silu (the tensor-core path at M >= 16). The 32 layer
        copies of a shape run back to back as one CUDA graph (weights larger than L2); the head
        runs twice per graph. M = 512 is judged by TFLOP/s against the measured bf16 peak, M = 16
        and 40 (HBM-bound) by GB/s against the measured copy bandwidth."""
        torch, rt = self.torch, self.rt
        rt.set_async(True)
        rt.set_stream(torch.cuda.current_stream().cuda_stream)
        tpeak, tkind = tensor_peak()
        hpeak, hkind = peaks()
        out = {"peaks": {"bf16_tflops": tpeak, "hbm_gbs": hpeak, "kind": tkind}}
        for m in (16, 40, 512):
            xd = torch.empty(m * WL.D, dtype=torch.float32, device="cuda")
            xf = torch.empty(m * WL.FF, dtype=torch.float32, device="cuda")
            self.rtb.synth_f32(xd.data_ptr(), m * WL.D, SEED, 91 + m)
            self.rtb.synth_f32(xf.data_ptr(), m * WL.FF, SEED, 92 + m)
            ys = {p.name: torch.empty(m * p.rows, dtype=torch.float32, device="cuda") for p in WL.SWEEP}
            calls = {
                "gate_up_silu": lambda L: rt.gemm_silu(L["gate"].data_ptr(), L["up"].data_ptr(), WL.FF, WL.D,
                                                       xd.data_ptr(), m, ys["gate_up_silu"].data_ptr()),
                "down": lambda L: rt.gemm(L["down"].data_ptr(), WL.D, WL.FF, xf.data_ptr(), m, ys["down"].data_ptr()),
                "qkv": lambda L: rt.gemm(L["qkv"].data_ptr(), WL.QKV, WL.D, xd.data_ptr(), m, ys["qkv"].data_ptr()),
                "out": lambda L: rt.gemm(L["out"].data_ptr(), WL.D, WL.D, xd.data_ptr(), m, ys["out"].data_ptr()),
            }
            row = {}
            tot_f = tot_t = 0.0
            for p in WL.SWEEP:
                if p.name == "head":
                    fns = [lambda: rt.gemm(self.head.data_ptr(), WL.VOCAB, WL.D, xd.data_ptr(), m,
                                           ys["head"].data_ptr())] * 2
                else:
                    fns = [(lambda L=L, p=p: calls[p.name](L)) for L in self.w]
                for f in fns[:2]:  # eager first: kernel attributes and scratch
                    f()
                torch.cuda.synchronize()
                g = self._graph(fns)
                us = self._time_graph(g, 2) * 1e3 / len(fns)
                del g
                fl, by = p.flops(m), p.bytes(m)
                tot_f += fl * len(fns)
                tot_t += us * len(fns)
                row[p.name] = {"us": round(us, 2), "TFLOP_s": round(fl / us / 1e6, 1), "GB_s": round(by / us / 1e3, 1),
                               "tensor_frac": round(fl / us / 1e6 / tpeak, 3), "hbm_frac": round(by / us / 1e3 / hpeak, 3)}
            row["all_shapes"] = {"TFLOP_s": round(tot_f / tot_t / 1e6, 1),
                                 "tensor_frac": round(tot_f / tot_t / 1e6 / tpeak, 3)}
            out[f"m{m}"] = row
            del xd, xf, ys
        rt.sync()
        return out

    def prims(self) -> dict:
        """The host-half primitives beside the products (rt_ip21_kv, rt_ip12_kv, rt_ip21,
        rt_scale_outer; src/host/rt_host.c:128-279) at a 9B-class decode step's sizes: attention
        over a 4096-token history (16 query heads on 4 kv heads, 256 columns: 16 MB of keys or
        values per call) and the delta rule's state (32 heads of 128 x 128: 2 MB per call). Each
        call reads its own buffer from a rotation larger than L2, 24 calls per CUDA graph; GB/s
        of algorithmic bytes (inputs read once, outputs written once). Beside each, the
        reference's own host code (oracle/_ref, src/host/rt_host.c, one thread) on one call."""
        import numpy as np
        torch, rt = self.torch, self.rt
        rt.set_async(True)
        rt.set_stream(torch.cuda.current_stream().cuda_stream)
        hpeak, hkind = peaks()
        h, n1, c, t = 16, 4, 256, 4096
        hs, r, cs = 32, 128, 128
        l = [q * n1 // h for q in range(h)]
        kv_bytes = t * n1 * c * 4
        nkv = 12  # 12 x 16 MB > L2
        gen = torch.Generator(device="cuda").manual_seed(7)
        kvs = [torch.randn(t * n1 * c, device="cuda", generator=gen) for _ in range(nkv)]
        states = [torch.randn(hs * r * cs, device="cuda", generator=gen) for _ in range(96)]  # 96 x 2 MB
        q = torch.randn(h * c, device="cuda", generator=gen)
        p = torch.randn(h * t, device="cuda", generator=gen)
        bs = torch.randn(hs * cs, device="cuda", generator=gen)
        av = torch.randn(hs * r, device="cuda", generator=gen)
        bv = torch.randn(hs * cs, device="cuda", generator=gen)
        zs = torch.empty(h * t, device="cuda")
        zo = torch.empty(h * c, device="cuda")
        zd = torch.empty(hs * r, device="cuda")
        zu = [torch.empty(hs * r * cs, device="cuda") for _ in range(2)]
        n = 24
        calls = {
            "ip21_kv": (lambda i: rt.ip21_kv(zs.data_ptr(), kvs[i % nkv].data_ptr(), n1, c, l, h, t, q.data_ptr()),
                        kv_bytes + h * c * 4 + h * t * 4),
            "ip12_kv": (lambda i: rt.ip12_kv(zo.data_ptr(), p.data_ptr(), kvs[i % nkv].data_ptr(), n1, c, l, h, t),
                        kv_bytes + h * t * 4 + h * c * 4),
            "ip21": (lambda i: rt.ip21(zd.data_ptr(), states[i % 96].data_ptr(), hs, r, cs, bs.data_ptr()),
                     hs * r * cs * 4 + hs * cs * 4 + hs * r * 4),
            "scale_outer": (lambda i: rt.scale_outer(zu[i % 2].data_ptr(), states[i % 96].data_ptr(), 0.97, av.data_ptr(),
                                                     bv.data_ptr(), hs * r, cs),
                            2 * hs * r * cs * 4 + hs * r * 4 + cs * 4),
        }
        out = {"shapes": {"attention": {"h": h, "n1": n1, "c": c, "t": t}, "delta_rule": {"h": hs, "r": r, "c": cs}},
               "peak_gbs": hpeak, "peak_kind": hkind}
        for name, (f, nbytes) in calls.items():
            fns = [(lambda i=i, f=f: f(i)) for i in range(n)]
            for g in fns:
                g()
            torch.cuda.synchronize()
            gr = self._graph(fns)
            us = self._time_graph(gr, 3) * 1e3 / n
            del gr
            out[name] = {"us": round(us, 2), "GB_s": round(nbytes / us / 1e3, 1), "hbm_frac": round(nbytes / us / 1e3 / hpeak, 3),
                         "bytes": nbytes}
        rt.sync()
        try:  # the reference's own host code, one call each (the CPU leg: the checker library)
            sys.path.insert(0, os.path.join(ROOT, "oracle"))
            import oracle as O
            if O.hostref_available():
                A = O._f32  # 64-byte aligned copies: the reference's AVX2 loads need 32
                kvh, qh, ph = A(kvs[0].cpu().numpy()), A(q.cpu().numpy()), A(p.cpu().numpy())
                sh, bsh, avh, bvh = A(states[0].cpu().numpy()), A(bs.cpu().numpy()), A(av.cpu().numpy()), A(bv.cpu().numpy())
                la = np.array(l, dtype=np.int64)
                zsh, zoh, zdh, zuh = O._aligned(h * t), O._aligned(h * c), O._aligned(hs * r), O._aligned(hs * r * cs)
                lib, rref = O.hostref()
                R = O.C.byref(rref)
                refs = {"ip21_kv": lambda: lib.rt_ip21_kv(R, zsh, kvh, n1, c, la, h, t, qh),
                        "ip12_kv": lambda: lib.rt_ip12_kv(R, zoh, ph, kvh, n1, c, la, h, t),
                        "ip21": lambda: lib.rt_ip21(R, zdh, sh, hs, r, cs, bsh),
                        "scale_outer": lambda: lib.rt_scale_outer(R, zuh, sh, 0.97, avh, bvh, hs * r, cs)}
                for name, f in refs.items():
                    f()
                    t0 = time.perf_counter()
                    f()
                    out[name]["cpu_reference_us"] = round((time.perf_counter() - t0) * 1e6, 1)
        except OSError:
            pass
        del kvs, states
        return out

    def sweep(self) -> dict:
        """BASELINE configs 2 and 3: each decode shape alone at M = 1 and at M = 2 (the verify pass),
        GB/s. The 32 layer copies of a shape run back to back as one CUDA graph (1.1-3.4 GB: larger
        than L2); the head is one 661 MB matrix, 8 launches per graph. Config 3's draft-head gather
        (32,768 of the head's 151,936 rows, 142.6 MB) rotates over four disjoint seeded row sets,
        8 launches per graph, so consecutive launches read different rows."""
        import numpy as np
        torch, rt = self.torch, self.rt
        rt.set_async(True)
        rt.set_stream(torch.cuda.current_stream().cuda_stream)
        hpeak, _ = peaks()
        out = {}
        y = self.y

        def run(fns, reps=3):
            for f in fns:  # eager once (kernel attributes), then the launches as one CUDA graph
                f()
            torch.cuda.synchronize()
            g = self._graph(fns)
            us = self._time_graph(g, reps) * 1e3 / len(fns)
            del g
            return us

        for m in (1, 2):
            xd, xf = self.x[("d", m)].data_ptr(), self.x[("ff", m)].data_ptr()
            calls = {
                "gate_up_silu": lambda L: rt.gemm_silu(L["gate"].data_ptr(), L["up"].data_ptr(), WL.FF, WL.D, xd, m,
                                                       y[("h", m)].data_ptr()),
                "down": lambda L: rt.gemm(L["down"].data_ptr(), WL.D, WL.FF, xf, m, y[("down", m)].data_ptr()),
                "qkv": lambda L: rt.gemm(L["qkv"].data_ptr(), WL.QKV, WL.D, xd, m, y[("qkv", m)].data_ptr()),
                "out": lambda L: rt.gemm(L["out"].data_ptr(), WL.D, WL.D, xd, m, y[("out", m)].data_ptr()),
            }
            row = {}
            for p in WL.SWEEP:
                if p.name == "head":
                    fns = [lambda: rt.gemm(self.head.data_ptr(), WL.VOCAB, WL.D, xd, m, y[("head", m)].data_ptr())] * 8
                else:
                    fns = [(lambda L=L, p=p: calls[p.name](L)) for L in self.w]
                us = run(fns)
                row[p.name] = {"shape": f"{p.rows}x{p.cols}" + (" x2 +silu" if p.kind == "silu" else ""),
                               "us": round(us, 2), "GB_s": round(p.bytes(m) / us / 1e3, 1),
                               "hbm_frac": round(p.bytes(m) / us / 1e3 / hpeak, 3)}
            out[f"m{m}"] = row
        # config 3: the draft head's gather (M = 1)
        perm = np.random.default_rng(SEED).permutation(WL.VOCAB).astype(np.int32)
        sets = [torch.from_numpy(perm[k * WL.HOT:(k + 1) * WL.HOT].copy()).cuda() for k in range(4)]
        yd = torch.empty(WL.HOT, dtype=torch.float32, device="cuda")
        xd = self.x[("d", 1)].data_ptr()
        fns = [(lambda k=k: rt.gemv_rows(self.head.data_ptr(), WL.VOCAB, sets[k % 4].data_ptr(), WL.HOT, WL.D, xd,
                                         yd.data_ptr())) for k in range(8)]
        us = run(fns)
        p = WL.DRAFT
        out["draft_head_gather"] = {"shape": f"{WL.HOT} of {WL.VOCAB} rows x{WL.D}", "us": round(us, 2),
                                    "GB_s": round(p.bytes(1) / us / 1e3, 1),
                                    "hbm_frac": round(p.bytes(1) / us / 1e3 / hpeak, 3)}
        rt.sync()
        return out


# ---------------------------------------------------------------- single-purpose modes

def probe(args) -> None:
    """One product kernel on a BASELINE shape through the C ABI, `args.launches` launches each
    timed with CUDA events after one warm-up launch: for profiler captures and quick timing.
    Prints the mean time per launch and one launch's algorithmic bytes and flops."""
    import numpy as np
    import torch

    import rtb200
    p = WL.DRAFT if args.probe == "draft_head" else next(q for q in WL.SWEEP if q.name == args.probe)
    t = args.t
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
    x = torch.empty(t * p.cols, dtype=torch.float32, device="cuda")
    rtb200.synth_f32(x.data_ptr(), t * p.cols, 1, 3)
    nout = p.nsel if p.kind == "rows" else p.rows
    y = torch.empty(t * nout, dtype=torch.float32, device="cuda")
    idx = None
    if p.kind == "rows":
        idx = torch.from_numpy(np.random.default_rng(1).choice(p.rows, p.nsel, replace=False).astype(np.int32)).cuda()

    def launch():
        if p.kind == "silu":
            rt.gemm_silu(w.data_ptr(), w2.data_ptr(), p.rows, p.cols, x.data_ptr(), t, y.data_ptr())
        elif p.kind == "rows":
            rt.gemv_rows(w.data_ptr(), p.rows, idx.data_ptr(), p.nsel, p.cols, x.data_ptr(), y.data_ptr())
        else:
            rt.gemm(w.data_ptr(), p.rows, p.cols, x.data_ptr(), t, y.data_ptr())

    launch()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.launches)]
    for e0, e1 in ev:
        e0.record()
        launch()
        e1.record()
    torch.cuda.synchronize()
    rt.sync()
    us = sum(e0.elapsed_time(e1) for e0, e1 in ev) / len(ev) * 1e3
    print(json.dumps({"probe": p.name, "rows": p.rows, "cols": p.cols, "t": t, "us_per_launch": round(us, 2),
                      "bytes": p.bytes(t), "flops": p.flops(t), "GB_s": round(p.bytes(t) / us / 1e3, 1)}), flush=True)
    rt.close()


def prim_probe(args) -> None:
    """One host-half primitive at the prims section's attention sizes (16 query heads on 4 kv
    heads, 256 columns, a history of `args.t` rows, 4096 unless given) through the C ABI,
    `args.launches` launches each timed with CUDA events after one warm-up launch: for profiler
    captures. Prints the mean time per launch and its algorithmic bytes."""
    import torch

    import rtb200
    h, n1, c = 16, 4, 256
    t = args.t if args.t > 1 else 4096
    l = [q * n1 // h for q in range(h)]
    gen = torch.Generator(device="cuda").manual_seed(7)
    kv = torch.randn(t * n1 * c, device="cuda", generator=gen)
    q = torch.randn(h * c, device="cuda", generator=gen)
    a = torch.randn(h * t, device="cuda", generator=gen)
    z = torch.empty(h * max(t, c), device="cuda")
    rt = rtb200.Runtime()
    rt.set_async(True)
    rt.set_stream(torch.cuda.current_stream().cuda_stream)
    if args.probe == "ip21_kv":
        launch = lambda: rt.ip21_kv(z.data_ptr(), kv.data_ptr(), n1, c, l, h, t, q.data_ptr())  # noqa: E731
    else:
        launch = lambda: rt.ip12_kv(z.data_ptr(), a.data_ptr(), kv.data_ptr(), n1, c, l, h, t)  # noqa: E731
    launch()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.launches)]
    for e0, e1 in ev:
        e0.record()
        launch()
        e1.record()
    torch.cuda.synchronize()
    rt.sync()
    us = sum(e0.elapsed_time(e1) for e0, e1 in ev) / len(ev) * 1e3
    nbytes = (t * n1 * c + h * c + h * t) * 4
    print(json.dumps({"probe": args.probe, "h": h, "n1": n1, "c": c, "t": t, "us_per_launch": round(us, 2),
                      "bytes": nbytes, "GB_s": round(nbytes / us / 1e3, 1)}), flush=True)
    rt.close()


def load_probe(args) -> None:
    """rt_b200_load_gguf on a synthetic GGUF of `args.load_layers` decode layers (QKV, out, gate, up,
    down; Q8_0 with random quants and fp16 scales) plus the 151936 x 4096 head: O_DIRECT reads into
    pinned buffers, copies overlapping the reads, the file's sum and the in-place repacks on the
    GPU. The reference measures its own load at 3.05-3.29 GB/s for the transfer and 9.27 GB/s for
    the repack (its docs/measurements.md). The GGUF writer is the tests' (tests/gguf_synth.py)."""
    import numpy as np
    import torch

    import rtb200
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import gguf_synth as G

    def q8_bytes(rows: int, cols: int, rng) -> bytes:
        blocks = rows * cols // 32
        raw = np.empty((blocks, 34), dtype=np.uint8)
        raw[:, 2:] = rng.integers(0, 256, size=(blocks, 32), dtype=np.uint8)
        d = (rng.random(blocks, dtype=np.float32) * 1e-3 + 1e-4).astype(np.float16)
        raw[:, :2] = d.view(np.uint8).reshape(blocks, 2)
        return raw.tobytes()

    rng = np.random.default_rng(1)
    tensors = []
    for L in range(args.load_layers):
        for name, rows, cols in (("attn_qkv", WL.QKV, WL.D), ("attn_output", WL.D, WL.D), ("ffn_gate", WL.FF, WL.D),
                                 ("ffn_up", WL.FF, WL.D), ("ffn_down", WL.D, WL.FF)):
            tensors.append((f"blk.{L}.{name}.weight", G.GGML_Q8_0, [cols, rows], q8_bytes(rows, cols, rng)))
    tensors.append(("output.weight", G.GGML_Q8_0, [WL.D, WL.VOCAB], q8_bytes(WL.VOCAB, WL.D, rng)))
    path = os.path.join(args.dir, "rtb_load_probe.gguf")
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
                      "tensors": len(table)}), flush=True)


def profile_figure(path: str, key: str):
    """An integer `key: value` line of a committed profile summary, or None."""
    try:
        with open(path) as f:
            for line in f:
                if line.startswith(key + ":"):
                    return int(line.split(":", 1)[1].split()[0])
    except (OSError, ValueError, IndexError):
        pass
    return None


def step_roofline(total: int, ms1: float, world: int, res: dict, layers: int = WL.LAYERS) -> dict:
    """The roofline of the decode step, the metric's own workload: its 129 gemv_exact_kernel
    launches (each rank streams its row shard) against one GPU's measured HBM copy bandwidth.
    achieved = the step's algorithmic bytes per GPU / the step time. traffic = ncu DRAM read+write
    bytes of one step's launches (profiles/gemv_exact_down_gateup_m1.md, 1 GPU), per step.
    per_shape (1 GPU): each shape's launch alone (the sweep's graph of 32 copies), its fraction of
    the peak and its share of the step (launches per step x time / step time)."""
    peak, how = peaks()
    achieved = total / world / (ms1 * 1e6)
    out = {"kernel": "gemv_exact_kernel (the decode step's 129 launches, graph-replayed)", "bound": "hbm",
           "achieved": round(achieved, 1), "peak": peak, "peak_kind": how, "unit": "GB/s",
           "frac": round(achieved / peak, 4),
           "traffic": profile_figure(STEP_TRAFFIC_PATH, "traffic_bytes_per_step") if world == 1 else None,
           "algorithmic_bytes": total // world, "us_per_launch": round(ms1 * 1e3 / len(WL.step_rounds(layers)), 2)}
    sw = res.get("sweep", {}).get("m1")
    if sw:
        counts = {p.name: sum(1 for q in WL.step_rounds(layers) if q.name == p.name) for p in WL.SWEEP}
        out["per_shape"] = {k: {"us": v["us"], "GB_s": v["GB_s"], "frac": v["hbm_frac"],
                                "share_of_step": round(counts[k] * v["us"] / (ms1 * 1e3), 3)} for k, v in sw.items()}
    out["head_launch"] = res["head_launch"]
    return out


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)  # ~0.4 s (M=1) + ~0.6 s (M=2) timed: clock samples
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--layers", type=int, default=WL.LAYERS)
    ap.add_argument("--no-prompt", action="store_true", help="skip the config-4 prompt gemm section")
    ap.add_argument("--probe", choices=[p.name for p in WL.SWEEP] + ["draft_head", "ip21_kv", "ip12_kv"],
                    help="time one product kernel on this BASELINE shape, or one host-half primitive at "
                         "the prims section's attention sizes (profiler captures)")
    ap.add_argument("--t", type=int, default=1, help="--probe: tokens")
    ap.add_argument("--launches", type=int, default=3, help="--probe: timed launches")
    ap.add_argument("--load", action="store_true", help="time the weight loader on a synthetic GGUF file")
    ap.add_argument("--load-layers", type=int, default=4, help="--load: decode layers in the file")
    ap.add_argument("--dir", default="/tmp", help="--load: where the file is written")
    args = ap.parse_args()
    if args.probe:
        (prim_probe if args.probe in ("ip21_kv", "ip12_kv") else probe)(args)
        return 0
    if args.load:
        load_probe(args)
        return 0
    args.warmup = max(3, args.warmup)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return 0
        cpu = reference_cpu(args.steps, args.warmup)
        line = {"metric": METRIC, "value": round(cpu["value"], 3), "unit": "GB/s", "impl": "reference",
                "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(cpu["ms_per_sample"], 3), "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded Q8_0, w ~ 0.02*N(0,1), x ~ N(0,1))",
                "config": {"workload": f"BASELINE config 5 sample: {CPU_LAYERS} 9B-class decode layers' weight "
                                       f"products (QKV, out, gate, up, down; distinct matrices), M=1",
                           "parallelism": "host threads"},
                "cpu_baseline": {**{k: cpu[k] for k in ("unit", "cores", "kind", "sample")},
                                 "value": round(cpu["value"], 3)},
                "e2e": {"value": round(cpu["value"], 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0

    import torch
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        os.environ.setdefault("NCCL_DEBUG", "WARN")  # stdout carries the one JSON line only
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    b = Bench(args, rank, world)
    res = b.run()
    total = WL.step_bytes(1, args.layers)
    total2 = WL.step_bytes(2, args.layers)
    ms1, ms2 = res["ms1"], res["ms2"]
    cpu = None
    if world == 1 and rank == 0:
        try:
            cpu = reference_cpu(5, 1, CPU_MIN_SECONDS)
        except Exception as e:  # noqa: BLE001 -- reported, not fatal: the GPU numbers stand alone
            log("cpu baseline unavailable:", e)
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(total / ms1 / 1e6, 1), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms1, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded Q8_0, w ~ 0.02*N(0,1), x ~ N(0,1))",
            "config": {"workload": f"BASELINE config 5: 9B-class decode step weight products, {args.layers} layers + "
                                   f"151936x4096 head, M=1", "bytes_per_step": total,
                       "parallelism": (f"row-shard x{world} + per-round gather of y "
                                + ("in the product kernel over NVLink" if b.rt.peer_gather() else "by NCCL all-gather"))
                               if world > 1 else "1 GPU",
                       "l2": "inputs larger than L2 (7.5 GB of weights per step)", "graph": "step captured as a CUDA graph"},
            "tok_s": round(1e3 / ms1, 1),
            "verify_m2": {"ms_per_step": round(ms2, 4), "GB_s": round(total2 / ms2 / 1e6, 1),
                          "tok_s_max": round(2e3 / ms2, 1)},
            "roofline": step_roofline(total, ms1, world, res, args.layers), "e2e": res["e2e"], "gpu_launches": res["launches"],
            "clocks": res["clocks"],
        }
        if cpu:
            line["cpu_baseline"] = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")}
        if "sweep" in res:
            line["sweep"] = res["sweep"]
        if "prompt" in res:
            line["prompt"] = res["prompt"]
        if "prims" in res:
            line["prims"] = res["prims"]
        print(json.dumps(line), flush=True)
    b.rt.close()
    if world > 1:
        torch.distributed.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
