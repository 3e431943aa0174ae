"""ctypes binding of librt_b200.so (include/rt_b200.h) for Python callers: the tests and bench.py.

It mirrors the reference runtime's product interface (src/card/rt.h:39, 62-72, 85): the same
names (rt_init, rt_gemv, rt_gemv_q, rt_gemv_open, rt_gemv_go, rt_gemm, rt_gemm_q, rt_q8_row), the
same argument meaning and order. Arguments are device addresses (ints, e.g. a torch tensor's
``data_ptr()``). Where the reference has no error path (its functions are void), this binding
raises ``RtError`` with the library's recorded message after a call that could not run.

There is no fallback: if the CUDA library is missing, ``load()`` raises.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "librt_b200.so")

RT_BATCH = 8
RTB_OK = 0
CUDA_STREAM_LEGACY = 0x1  # cudaStreamLegacy
ERRORS = {1: "RTB_EINVAL", 2: "RTB_ECUDA", 3: "RTB_EKERNEL", 4: "RTB_ENOMEM", 5: "RTB_ENOTINIT", 6: "RTB_EQUEUE",
          7: "RTB_ENCCL"}

# The entry points include/rt_b200.h declares, all of which the library must export.
EXPORTS = ("rt_init", "rt_gemv", "rt_gemv_q", "rt_gemv_open", "rt_gemv_go", "rt_gemm", "rt_gemm_q", "rt_q8_row",
           "gemv_s_bytes", "gemv_s_repack", "rt_gemm_silu_q", "rt_gemm_silu", "rt_gemv_rows_q", "rt_gemv_rows",
           "rt_b200_last_error", "rt_b200_set_overlap", "rt_b200_set_async", "rt_b200_sync", "rt_b200_stream", "rt_b200_set_stream",
           "rt_b200_free", "rt_b200_nccl_id", "rt_b200_shard", "rt_b200_peer_gather", "rt_b200_chain_begin",
           "rt_b200_chain_end", "rtb_gguf_info", "rt_b200_load_gguf", "rtb_load_error", "rtb_synth_q8_0",
           "rtb_synth_f32", "rt_gemm_static", "rt_b200_pull", "rt_b200_push", "rt_b200_wait_probe", "gemv_i_bytes",
           "gemv_i_repack", "gemv_i_repack_thread", "rt_b200_shard_rows", "rt_b200_flush",
           "rt_b200_set_push_direct", "rt_ip21", "rt_ip21_kv", "rt_ip12_kv", "rt_scale_outer")


class RtError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{ERRORS.get(code, code)}: {msg}")
        self.code = code


class StructRt(C.Structure):
    """struct rt of src/card/rt.h:19-26, field for field."""
    _fields_ = [("team", C.c_void_p), ("frame", C.c_char_p), ("chain", C.c_void_p), ("gemm_chain", C.c_void_p),
                ("threads", C.c_int), ("last", C.c_int)]


_lib = None
_L = C.c_long
_P = C.c_void_p


class Tensor(C.Structure):
    """rtb_tensor of include/rt_b200.h: one GGUF tensor's table entry."""
    _fields_ = [("name", C.c_char * 96), ("type", C.c_int), ("n_dims", C.c_int), ("dim", C.c_longlong * 4),
                ("offset", C.c_ulonglong), ("bytes", C.c_ulonglong), ("dev", C.c_void_p), ("repacked", C.c_int),
                ("pad_", C.c_int)]


class LoadStats(C.Structure):
    """rtb_load_stats of include/rt_b200.h."""
    _fields_ = [("file_bytes", C.c_ulonglong), ("file_sum", C.c_ulonglong), ("seconds", C.c_double),
                ("seconds_repack", C.c_double), ("direct", C.c_int), ("q8_matrices", C.c_int)]


def load() -> C.CDLL:
    """The CUDA library; raises if it has not been built (python intel-phi-apl_b200/build.py)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise FileNotFoundError(f"{LIB_PATH} missing: build it with intel-phi-apl_b200/build.py")
    lib = C.CDLL(LIB_PATH)
    R = C.POINTER(StructRt)
    sig = {
        "rt_init": ([R, C.c_int], C.c_int),
        "rt_gemv": ([R, _P, _L, _L, _P, _P], None),
        "rt_gemv_q": ([R, _P, _L, _L, _P, _P], None),
        "rt_gemv_open": ([R], None),
        "rt_gemv_go": ([R], None),
        "rt_gemm": ([R, _P, _L, _L, _P, _L, _P], None),
        "rt_gemm_q": ([R, _P, _L, _L, _P, _L, _P], None),
        "rt_q8_row": ([_P, _L, _L, _P], None),
        "rt_ip21": ([R, _P, _P, _L, _L, _L, _P], None),
        "rt_ip21_kv": ([R, _P, _P, _L, _L, _P, _L, _L, _P], None),
        "rt_ip12_kv": ([R, _P, _P, _P, _L, _L, _P, _L, _L], None),
        "rt_scale_outer": ([R, _P, _P, C.c_float, _P, _P, _L, _L], None),
        "gemv_s_bytes": ([_L, _L], _L),
        "gemv_s_repack": ([_P, _L, _L, _P], C.c_int),
        "gemv_i_bytes": ([_L, _L], _L),
        "gemv_i_repack": ([_P, _L, _L, _P], None),
        "gemv_i_repack_thread": ([_P, C.c_int, C.c_int], None),
        "rt_gemm_silu_q": ([R, _P, _P, _L, _L, _P, _L, _P], None),
        "rt_gemm_silu": ([R, _P, _P, _L, _L, _P, _L, _P], None),
        "rt_gemv_rows_q": ([R, _P, _L, _P, _L, _L, _P, _P], None),
        "rt_gemv_rows": ([R, _P, _L, _P, _L, _L, _P, _P], None),
        "rt_b200_last_error": ([R, C.c_char_p, C.c_size_t], C.c_int),
        "rt_b200_set_async": ([R, C.c_int], None),
        "rt_b200_set_overlap": ([R, C.c_int], None),
        "rt_b200_sync": ([R], C.c_int),
        "rt_b200_pull": ([R, _P, _P, C.c_size_t], C.c_int),
        "rt_b200_push": ([R, _P, _P, C.c_size_t], C.c_int),
        "rt_b200_stream": ([R], _P),
        "rt_b200_set_stream": ([R, _P], None),
        "rt_b200_free": ([R], None),
        "rt_b200_nccl_id": ([_P], C.c_int),
        "rt_b200_shard": ([R, C.c_int, C.c_int, _P], C.c_int),
        "rt_b200_peer_gather": ([R], C.c_int),
        "rt_b200_flush": ([R], C.c_int),
        "rt_b200_set_push_direct": ([R, C.c_int], None),
        "rt_b200_shard_rows": ([_L, C.c_int, C.c_int, C.POINTER(_L), C.POINTER(_L)], C.c_int),
        "rt_b200_wait_probe": ([R], C.c_int),
        "rt_b200_chain_begin": ([R], C.c_int),
        "rt_b200_chain_end": ([R, C.c_int], C.c_int),
        "rtb_gguf_info": ([C.c_char_p, C.POINTER(Tensor), C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_ulonglong)],
                          C.c_int),
        "rt_b200_load_gguf": ([R, C.c_char_p, _P, C.c_ulonglong, C.POINTER(Tensor), C.c_int, C.POINTER(C.c_int),
                               C.POINTER(LoadStats)], C.c_int),
        "rtb_load_error": ([], C.c_char_p),
        "rtb_synth_q8_0": ([_P, _L, _L, _L, C.c_uint64, C.c_uint64, C.c_float], C.c_int),
        "rtb_synth_f32": ([_P, _L, C.c_uint64, C.c_uint64, C.c_float], C.c_int),
        "rt_gemm_static": ([_P, _L, _L, _P, _L, _P, _P], C.c_int),
    }
    for name, (args, res) in sig.items():
        f = getattr(lib, name)
        f.argtypes = args
        f.restype = res
    _lib = lib
    return lib


def shard_rows(rows: int, rank: int, world: int) -> tuple[int, int]:
    """rt_b200_shard_rows: (first row, row count) of rank's shard, as the library splits products."""
    r0, n = C.c_long(0), C.c_long(0)
    code = load().rt_b200_shard_rows(rows, rank, world, C.byref(r0), C.byref(n))
    if code:
        raise RtError(code, last_error(None)[1])
    return r0.value, n.value


def last_error(rt: "Runtime | None" = None) -> tuple[int, str]:
    buf = C.create_string_buffer(256)
    code = load().rt_b200_last_error(C.byref(rt.R) if rt is not None else None, buf, 256)
    return code, buf.value.decode(errors="replace")


def _check(rt: "Runtime | None") -> None:
    code, msg = last_error(rt)
    if code != RTB_OK:
        raise RtError(code, msg)


def gguf_info(path: str) -> tuple[list[dict], int]:
    """The tensor table of a GGUF file (host only) and the file's size."""
    lib = load()
    n, fb = C.c_int(0), C.c_ulonglong(0)
    code = lib.rtb_gguf_info(path.encode(), None, 0, C.byref(n), C.byref(fb))
    if code:
        raise RtError(code, lib.rtb_load_error().decode(errors="replace"))
    arr = (Tensor * max(1, n.value))()
    code = lib.rtb_gguf_info(path.encode(), arr, n.value, C.byref(n), C.byref(fb))
    if code:
        raise RtError(code, lib.rtb_load_error().decode(errors="replace"))
    return [_tensor_dict(arr[i]) for i in range(n.value)], fb.value


def _tensor_dict(t: Tensor) -> dict:
    return {"name": t.name.decode(), "type": t.type, "dims": [t.dim[d] for d in range(t.n_dims)],
            "offset": t.offset, "bytes": t.bytes, "dev": t.dev or 0, "repacked": bool(t.repacked)}


def gemv_s_bytes(rows: int, cols: int) -> int:
    return load().gemv_s_bytes(rows, cols)


def gemv_s_repack(q8: int, rows: int, cols: int, out: int) -> None:
    code = load().gemv_s_repack(q8, rows, cols, out)
    if code:
        _check(None)
        raise RtError(code, "gemv_s_repack")


def q8_row(w: int, cols: int, row: int, z: int) -> None:
    load().rt_q8_row(w, cols, row, z)
    _check(None)


def synth_q8_0(dst: int, row0: int, rows: int, cols: int, seed: int, stream: int, sigma: float = 0.02) -> None:
    code = load().rtb_synth_q8_0(dst, row0, rows, cols, seed, stream, sigma)
    if code:
        raise RtError(code, "rtb_synth_q8_0")


def synth_f32(dst: int, n: int, seed: int, stream: int, sigma: float = 1.0) -> None:
    code = load().rtb_synth_f32(dst, n, seed, stream, sigma)
    if code:
        raise RtError(code, "rtb_synth_f32")


def nccl_id() -> bytes:
    buf = C.create_string_buffer(128)
    code = load().rt_b200_nccl_id(buf)
    if code:
        raise RtError(code, "rt_b200_nccl_id")
    return buf.raw


class Runtime:
    """One struct rt bound to the current CUDA device (rt_init)."""

    def __init__(self, threads: int = 1):
        self.lib = load()
        self.R = StructRt()
        if self.lib.rt_init(C.byref(self.R), threads) != 0:
            raise RtError(5, "rt_init failed (no CUDA device?)")
        self._ref = C.byref(self.R)

    def close(self) -> None:
        if self.R.chain:
            self.lib.rt_b200_free(self._ref)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # -- the reference's products (device addresses)
    def gemv(self, w: int, rows: int, cols: int, x: int, y: int) -> None:
        self.lib.rt_gemv(self._ref, w, rows, cols, x, y)
        _check(self)

    def gemv_q(self, w: int, rows: int, cols: int, x: int, y: int) -> None:
        self.lib.rt_gemv_q(self._ref, w, rows, cols, x, y)
        _check(self)

    def gemv_open(self) -> None:
        self.lib.rt_gemv_open(self._ref)
        _check(self)

    def gemv_go(self) -> None:
        self.lib.rt_gemv_go(self._ref)
        _check(self)

    def gemm(self, w: int, rows: int, cols: int, x: int, t: int, y: int) -> None:
        self.lib.rt_gemm(self._ref, w, rows, cols, x, t, y)
        _check(self)

    def gemm_q(self, w: int, rows: int, cols: int, x: int, t: int, y: int) -> None:
        self.lib.rt_gemm_q(self._ref, w, rows, cols, x, t, y)
        _check(self)

    # -- fused products
    def gemm_silu(self, wg: int, wu: int, rows: int, cols: int, x: int, t: int, h: int) -> None:
        self.lib.rt_gemm_silu(self._ref, wg, wu, rows, cols, x, t, h)
        _check(self)

    def gemm_silu_q(self, wg: int, wu: int, rows: int, cols: int, x: int, t: int, h: int) -> None:
        self.lib.rt_gemm_silu_q(self._ref, wg, wu, rows, cols, x, t, h)
        _check(self)

    def gemv_rows(self, w: int, w_rows: int, idx: int, n: int, cols: int, x: int, y: int) -> None:
        self.lib.rt_gemv_rows(self._ref, w, w_rows, idx, n, cols, x, y)
        _check(self)

    def gemv_rows_q(self, w: int, w_rows: int, idx: int, n: int, cols: int, x: int, y: int) -> None:
        self.lib.rt_gemv_rows_q(self._ref, w, w_rows, idx, n, cols, x, y)
        _check(self)

    # -- controls
    def set_async(self, on: bool) -> None:
        self.lib.rt_b200_set_async(self._ref, 1 if on else 0)

    def set_overlap(self, on: bool) -> None:
        """Weights are read-only between products: launch products so they overlap (PDL)."""
        self.lib.rt_b200_set_overlap(self._ref, 1 if on else 0)

    # ---- the host-half primitives (device pointers; l: the kv head of each query head, host ints)
    def ip21(self, z: int, a: int, h: int, r: int, c: int, b: int) -> None:
        """rt_ip21: z[h][i] = a[h][i][:] . b[h][:] (the delta rule's state product)."""
        self.lib.rt_ip21(self._ref, z, a, h, r, c, b)
        _check(self)

    def ip21_kv(self, z: int, kv: int, n1: int, c: int, l, h: int, t: int, b: int) -> None:
        """rt_ip21_kv: z[h][s] = kv[s][l[h]][:] . b[h][:] (scores over a head's history)."""
        la = (C.c_long * h)(*[int(v) for v in l])
        self.lib.rt_ip21_kv(self._ref, z, kv, n1, c, la, h, t, b)
        _check(self)

    def ip12_kv(self, z: int, a: int, kv: int, n1: int, c: int, l, h: int, t: int) -> None:
        """rt_ip12_kv: z[h][:] = sum over s in order of a[h][s] * kv[s][l[h]][:]."""
        la = (C.c_long * h)(*[int(v) for v in l])
        self.lib.rt_ip12_kv(self._ref, z, a, kv, n1, c, la, h, t)
        _check(self)

    def scale_outer(self, z: int, s: int, g: float, a: int, b: int, m: int, k: int) -> None:
        """rt_scale_outer: z[i][q] = g * s[i][q] + a[i] * b[q] (one fma, the product rounded first)."""
        self.lib.rt_scale_outer(self._ref, z, s, g, a, b, m, k)
        _check(self)

    def set_push_direct(self, on: bool) -> None:
        """rt_b200_set_push_direct: go holds a one-product round back for push, which then takes y
        straight from the product kernel into mapped pinned host memory."""
        self.lib.rt_b200_set_push_direct(self._ref, 1 if on else 0)

    def sync(self) -> None:
        code = self.lib.rt_b200_sync(self._ref)
        if code:
            _check(self)
            raise RtError(code, "rt_b200_sync")

    def pull(self, dev: int, host: int, nbytes: int) -> None:
        """Host -> device copy of nbytes on the runtime's stream, or while a round is open on its
        link stream (returns at once)."""
        code = self.lib.rt_b200_pull(self._ref, dev, host, nbytes)
        if code:
            _check(self)
            raise RtError(code, "rt_b200_pull")

    def push(self, host: int, dev: int, nbytes: int) -> None:
        """Device -> host copy of nbytes; returns once they are on the host."""
        code = self.lib.rt_b200_push(self._ref, host, dev, nbytes)
        if code:
            _check(self)
            raise RtError(code, "rt_b200_push")

    def stream(self) -> int:
        return self.lib.rt_b200_stream(self._ref) or 0

    def set_stream(self, stream: int | None) -> None:
        """Run on `stream` (a cudaStream_t handle, e.g. torch's ``cuda_stream``). Handle 0 is the
        legacy default stream and goes to the library as cudaStreamLegacy; None restores the
        runtime's own stream."""
        if stream is None:
            self.lib.rt_b200_set_stream(self._ref, None)
        else:
            self.lib.rt_b200_set_stream(self._ref, stream if stream != 0 else CUDA_STREAM_LEGACY)

    def shard(self, rank: int, world: int, nid: bytes | None) -> None:
        buf = C.create_string_buffer(nid, 128) if nid is not None else None
        code = self.lib.rt_b200_shard(self._ref, rank, world, buf)
        if code:
            _check(self)
            raise RtError(code, "rt_b200_shard")

    def chain_begin(self) -> None:
        code = self.lib.rt_b200_chain_begin(self._ref)
        if code:
            _check(self)
            raise RtError(code, "rt_b200_chain_begin")

    def chain_end(self, serial: bool = True) -> None:
        code = self.lib.rt_b200_chain_end(self._ref, 1 if serial else 0)
        if code:
            _check(self)
            raise RtError(code, "rt_b200_chain_end")

    def load_gguf(self, path: str, arena: int, arena_bytes: int) -> tuple[list[dict], dict]:
        """rt_b200_load_gguf: the file into the device arena, Q8_0 matrices repacked in place."""
        tensors, _ = gguf_info(path)
        arr = (Tensor * max(1, len(tensors)))()
        n, st = C.c_int(0), LoadStats()
        code = self.lib.rt_b200_load_gguf(self._ref, path.encode(), arena, arena_bytes, arr, len(tensors), C.byref(n),
                                          C.byref(st))
        if code:
            raise RtError(code, self.lib.rtb_load_error().decode(errors="replace"))
        stats = {k: getattr(st, k) for k, _ in LoadStats._fields_}
        return [_tensor_dict(arr[i]) for i in range(n.value)], stats

    def flush(self) -> None:
        """rt_b200_flush: enqueue the finish of a pending row-sharded gather (capturable)."""
        code = self.lib.rt_b200_flush(self._ref)
        if code:
            _check(self)
            raise RtError(code, "rt_b200_flush")

    def peer_gather(self) -> bool:
        """True when single products gather y in their own kernel (else through NCCL)."""
        return bool(self.lib.rt_b200_peer_gather(self._ref))

    def wait_probe(self) -> tuple[int, str]:
        """The failure path's self-test: a kernel whose two bounded waits never complete. Returns
        the library's code (RTB_EKERNEL expected) and the recorded message, which it clears."""
        code = self.lib.rt_b200_wait_probe(self._ref)
        return code, last_error(self)[1]
