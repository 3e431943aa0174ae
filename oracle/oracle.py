"""TEST INFRASTRUCTURE ONLY: ctypes access to the CPU oracles.

Three libraries, all built by ``oracle/Makefile``:

* ``libq8oracle.so`` -- this repository's C restatement of the reference's Q8_0 products
  (``oracle/q8_oracle.c``; the header says which reference lines each function follows);
* ``_ref/libq8ref.so`` -- the reference's own host-model kernels (src/card/gemv.c, gemm.c,
  team.c) compiled from its sources, behind ``oracle/ref_harness.c``;
* ``_ref/libhostref.so`` -- the reference's own host-half primitives (src/host/rt_host.c).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg import this
module; the product path never does.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_PATH = os.path.join(HERE, "libq8oracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libq8ref.so")
# The reference's source tree (read only; only oracle/Makefile's `ref` target and the fixture
# script read it): $REF_ROOT, else a checkout named `reference` beside this repository.
REF_ROOT = os.environ.get("REF_ROOT") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")

_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_lp = np.ctypeslib.ndpointer(dtype=np.int64, flags="C_CONTIGUOUS")
_L = C.c_long

_port = None
_ref = None


def port() -> C.CDLL:
    """The C restatement (always available once ``make -C oracle port`` has run)."""
    global _port
    if _port is None:
        lib = C.CDLL(PORT_PATH)
        lib.q8o_half.argtypes = [C.c_uint16]
        lib.q8o_half.restype = C.c_float
        lib.q8o_to_half.argtypes = [C.c_float]
        lib.q8o_to_half.restype = C.c_uint16
        for name in ("q8o_gguf_bytes", "q8o_split_bytes"):
            getattr(lib, name).argtypes = [_L, _L]
            getattr(lib, name).restype = _L
        lib.q8o_split_scale_stride.argtypes = [_L]
        lib.q8o_split_scale_stride.restype = _L
        lib.q8o_repack_split.argtypes = [_u8p, _L, _L, _u8p]
        lib.q8o_unpack_split.argtypes = [_u8p, _L, _L, _u8p]
        lib.q8o_normal.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64]
        lib.q8o_normal.restype = C.c_float
        lib.q8o_fill_f32.argtypes = [_f32p, _L, C.c_uint64, C.c_uint64, C.c_float]
        lib.q8o_fill_q8_0.argtypes = [_u8p, _L, _L, _L, C.c_uint64, C.c_uint64, C.c_float]
        lib.q8o_gemv.argtypes = [_u8p, _L, _L, _f32p, _f32p, C.c_int]
        lib.q8o_gemm.argtypes = [_u8p, _L, _L, _f32p, _L, _f32p, C.c_int]
        lib.q8o_gemv_rows.argtypes = [_u8p, _L, _i32p, _L, _f32p, _f32p, C.c_int]
        lib.q8o_gemm_f64.argtypes = [_u8p, _L, _L, _f32p, _L, _f64p, C.c_int]
        lib.q8o_gate21_hashes.argtypes = [np.ctypeslib.ndpointer(dtype=np.uint64, flags="C_CONTIGUOUS")]
        lib.q8o_gate_a.argtypes = [C.POINTER(C.c_uint64), np.ctypeslib.ndpointer(dtype=np.uint32, flags="C_CONTIGUOUS")]
        lib.q8o_ip21_kv.argtypes = [_f32p, _f32p, _L, _L, _lp, _L, _L, _f32p]
        lib.q8o_ip12_kv.argtypes = [_f32p, _f32p, _f32p, _L, _L, _lp, _L, _L]
        lib.q8o_ip21.argtypes = [_f32p, _f32p, _L, _L, _L, _f32p]
        lib.q8o_scale_outer.argtypes = [_f32p, _f32p, C.c_float, _f32p, _f32p, _L, _L]
        _port = lib
    return _port


def ref_available() -> bool:
    return os.path.exists(REF_PATH)


HOSTREF_PATH = os.path.join(HERE, "_ref", "libhostref.so")
_hostref = None


class _StructRt(C.Structure):
    # the reference's struct rt (src/card/rt.h:19-26); team = NULL: the one-thread path
    _fields_ = [("team", C.c_void_p), ("frame", C.c_char_p), ("chain", C.c_void_p), ("gemm_chain", C.c_void_p),
                ("threads", C.c_int), ("last", C.c_int)]


def hostref_available() -> bool:
    return os.path.exists(HOSTREF_PATH)


def hostref() -> tuple[C.CDLL, C.c_void_p]:
    """The reference's own host-half primitives (src/host/rt_host.c), and a struct rt without a
    team for them (its one-thread path: the same arithmetic per output)."""
    global _hostref
    if _hostref is None:
        lib = C.CDLL(HOSTREF_PATH)
        R = C.POINTER(_StructRt)
        lib.rt_ip21_kv.argtypes = [R, _f32p, _f32p, _L, _L, _lp, _L, _L, _f32p]
        lib.rt_ip12_kv.argtypes = [R, _f32p, _f32p, _f32p, _L, _L, _lp, _L, _L]
        lib.rt_ip21.argtypes = [R, _f32p, _f32p, _L, _L, _L, _f32p]
        lib.rt_scale_outer.argtypes = [R, _f32p, _f32p, C.c_float, _f32p, _f32p, _L, _L]
        rt = _StructRt()
        _hostref = (lib, rt)
    return _hostref


def ref() -> C.CDLL:
    """The reference's own host-model kernels (built here from the reference's sources)."""
    global _ref
    if _ref is None:
        lib = C.CDLL(REF_PATH)
        lib.refh_team.argtypes = [C.c_int]
        lib.refh_team.restype = C.c_int
        lib.refh_form_i_bytes.argtypes = [_L, _L]
        lib.refh_form_i_bytes.restype = _L
        lib.refh_repack.argtypes = [_u8p, _L, _L, _u8p]
        lib.refh_gemv.argtypes = [_u8p, _L, _L, _f32p, _f32p]
        lib.refh_gemm.argtypes = [_u8p, _L, _L, _f32p, _L, _f32p]
        _ref = lib
    return _ref


THREADS = max(1, min(os.cpu_count() or 1, 64))


# ---------------------------------------------------------------- inputs

def gguf_bytes(rows: int, cols: int) -> int:
    return rows * (cols // 32) * 34


def synth_q8_0(rows: int, cols: int, seed: int, stream: int, sigma: float = 0.02, row0: int = 0,
               threads: int = 1) -> np.ndarray:
    """Rows [row0, row0+rows) of a seeded synthetic Q8_0 matrix, GGUF layout (uint8). With
    threads > 1 the rows are filled in ranges on host threads (the C fill runs without the GIL);
    every value depends only on its own index, so the bytes are the same."""
    out = np.empty(gguf_bytes(rows, cols), dtype=np.uint8)
    rb = gguf_bytes(1, cols)
    n = max(1, min(threads, rows))
    if n == 1:
        port().q8o_fill_q8_0(out, row0, rows, cols, seed, stream, sigma)
        return out
    from concurrent.futures import ThreadPoolExecutor
    cuts = [rows * k // n for k in range(n + 1)]
    with ThreadPoolExecutor(n) as pool:
        list(pool.map(lambda k: port().q8o_fill_q8_0(out[cuts[k] * rb:cuts[k + 1] * rb], row0 + cuts[k],
                                                     cuts[k + 1] - cuts[k], cols, seed, stream, sigma), range(n)))
    return out


def synth_f32(n: int, seed: int, stream: int, sigma: float = 1.0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    port().q8o_fill_f32(out, n, seed, stream, sigma)
    return out


def repack_split(q8: np.ndarray, rows: int, cols: int) -> np.ndarray:
    out = np.empty(port().q8o_split_bytes(rows, cols), dtype=np.uint8)
    port().q8o_repack_split(np.ascontiguousarray(q8), rows, cols, out)
    return out


def unpack_split(split: np.ndarray, rows: int, cols: int) -> np.ndarray:
    out = np.empty(gguf_bytes(rows, cols), dtype=np.uint8)
    port().q8o_unpack_split(np.ascontiguousarray(split), rows, cols, out)
    return out


# ---------------------------------------------------------------- products (the port)

def gemv(q8: np.ndarray, rows: int, cols: int, x: np.ndarray, threads: int = THREADS) -> np.ndarray:
    y = np.empty(rows, dtype=np.float32)
    port().q8o_gemv(np.ascontiguousarray(q8), rows, cols, np.ascontiguousarray(x, dtype=np.float32), y, threads)
    return y


def gemm(q8: np.ndarray, rows: int, cols: int, x: np.ndarray, t: int, threads: int = THREADS) -> np.ndarray:
    """x [t, cols] -> y [t, rows]"""
    y = np.empty((t, rows), dtype=np.float32)
    port().q8o_gemm(np.ascontiguousarray(q8), rows, cols, np.ascontiguousarray(x, dtype=np.float32).reshape(-1), t,
                    y.reshape(-1), threads)
    return y


def gemv_rows(q8: np.ndarray, cols: int, idx: np.ndarray, x: np.ndarray, threads: int = THREADS) -> np.ndarray:
    idx = np.ascontiguousarray(idx, dtype=np.int32)
    y = np.empty(len(idx), dtype=np.float32)
    port().q8o_gemv_rows(np.ascontiguousarray(q8), cols, idx, len(idx), np.ascontiguousarray(x, dtype=np.float32), y,
                         threads)
    return y


def gemm_f64(q8: np.ndarray, rows: int, cols: int, x: np.ndarray, t: int, threads: int = THREADS) -> np.ndarray:
    y = np.empty((t, rows), dtype=np.float64)
    port().q8o_gemm_f64(np.ascontiguousarray(q8), rows, cols, np.ascontiguousarray(x, dtype=np.float32).reshape(-1), t,
                        y.reshape(-1), threads)
    return y


def gate21_hashes() -> list[int]:
    out = np.zeros(7, dtype=np.uint64)
    port().q8o_gate21_hashes(out)
    return [int(v) for v in out]


def gate_a() -> tuple[int, list[int]]:
    h = C.c_uint64(0)
    w = np.zeros(3, dtype=np.uint32)
    port().q8o_gate_a(C.byref(h), w)
    return int(h.value), [int(v) for v in w]


# ---------------------------------------------------------------- products (the reference itself)

class RefMatrix:
    """A GGUF Q8_0 matrix repacked to form I by the reference's gemv_i_repack, ready for its
    gemv_i_thread / gemm_i_thread (rows % 16 == 0)."""

    def __init__(self, q8: np.ndarray, rows: int, cols: int, threads: int = THREADS):
        if rows % 16 or cols % 32:
            raise ValueError("the reference's form I needs rows % 16 == 0 and cols % 32 == 0")
        lib = ref()
        if lib.refh_team(threads) < 0:
            raise RuntimeError("refh_team failed")
        self.rows, self.cols = rows, cols
        self.form_i = np.empty(lib.refh_form_i_bytes(rows, cols), dtype=np.uint8)
        lib.refh_repack(np.ascontiguousarray(q8), rows, cols, self.form_i)

    def gemv(self, x: np.ndarray, y: np.ndarray | None = None) -> np.ndarray:
        if y is None:
            y = np.empty(self.rows, dtype=np.float32)
        ref().refh_gemv(self.form_i, self.rows, self.cols, np.ascontiguousarray(x, dtype=np.float32), y)
        return y

    def gemm(self, x: np.ndarray, t: int) -> np.ndarray:
        y = np.empty((t, self.rows), dtype=np.float32)
        ref().refh_gemm(self.form_i, self.rows, self.cols, np.ascontiguousarray(x, dtype=np.float32).reshape(-1), t,
                        y.reshape(-1))
        return y


# ---------------------------------------------------------------- host-half primitives
# (prims_oracle.c restates src/host/rt_host.c:128-279; the same calls on the reference itself
# through hostref())

def _f32(a):
    """A float32 copy on a 64-byte boundary: the reference's AVX2 code uses aligned loads and
    stores (_mm256_load_ps / _mm256_store_ps), which fault on less."""
    a = np.asarray(a, dtype=np.float32).ravel()
    out = _aligned(a.size)
    out[:] = a
    return out


def _aligned(n: int) -> np.ndarray:
    buf = np.empty(n + 16, dtype=np.float32)
    off = (-buf.ctypes.data % 64) // 4
    return buf[off:off + n]


def ip21_kv(kv: np.ndarray, n1: int, c: int, l: np.ndarray, h: int, t: int, b: np.ndarray, use_ref: bool = False) -> np.ndarray:
    z = _aligned(h * t)
    l64 = np.ascontiguousarray(l, dtype=np.int64)
    if use_ref:
        lib, rt = hostref()
        lib.rt_ip21_kv(C.byref(rt), z, _f32(kv), n1, c, l64, h, t, _f32(b))
    else:
        port().q8o_ip21_kv(z, _f32(kv), n1, c, l64, h, t, _f32(b))
    return z


def ip12_kv(a: np.ndarray, kv: np.ndarray, n1: int, c: int, l: np.ndarray, h: int, t: int, use_ref: bool = False) -> np.ndarray:
    z = _aligned(h * c)
    l64 = np.ascontiguousarray(l, dtype=np.int64)
    if use_ref:
        lib, rt = hostref()
        lib.rt_ip12_kv(C.byref(rt), z, _f32(a), _f32(kv), n1, c, l64, h, t)
    else:
        port().q8o_ip12_kv(z, _f32(a), _f32(kv), n1, c, l64, h, t)
    return z


def ip21(a: np.ndarray, h: int, r: int, c: int, b: np.ndarray, use_ref: bool = False) -> np.ndarray:
    z = _aligned(h * r)
    if use_ref:
        lib, rt = hostref()
        lib.rt_ip21(C.byref(rt), z, _f32(a), h, r, c, _f32(b))
    else:
        port().q8o_ip21(z, _f32(a), h, r, c, _f32(b))
    return z


def scale_outer(s: np.ndarray, g: float, a: np.ndarray, b: np.ndarray, m: int, k: int, use_ref: bool = False) -> np.ndarray:
    z = _aligned(m * k)
    if use_ref:
        lib, rt = hostref()
        lib.rt_scale_outer(C.byref(rt), z, _f32(s), g, _f32(a), _f32(b), m, k)
    else:
        port().q8o_scale_outer(z, _f32(s), g, _f32(a), _f32(b), m, k)
    return z
