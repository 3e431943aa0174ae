"""The weight loader (rtb_gguf_info on CPU, rt_b200_load_gguf on the GPU).

A synthetic GGUF file holds Q8_0 matrices of the decode shapes' widths (their GGUF bytes from the
oracle's generator), an F32 vector, a tied entry that shares another matrix's data, and metadata
of every value kind. The loaded arena must hold: every Q8_0 matrix in the row-split layout
(equal to the oracle's repack of the same GGUF bytes), every other tensor as in the file, and the
file's position-weighted sum (the engine's "file sum", src/bench/arena.h:26-44).
"""
from __future__ import annotations

import os

import numpy as np
import pytest

import gguf_synth as G

SEED = 20261201


@pytest.fixture(scope="module")
def synth_file(tmp_path_factory, oracle):
    path = str(tmp_path_factory.mktemp("gguf") / "tiny.gguf")
    mats = {"blk.0.attn_qkv.weight": (512, 4096, 81), "blk.0.ffn_down.weight": (256, 12288, 82),
            "token_embd.weight": (300, 4096, 83)}
    tensors = []
    for name, (rows, cols, stream) in mats.items():
        tensors.append((name, G.GGML_Q8_0, [cols, rows], oracle.synth_q8_0(rows, cols, SEED, stream).tobytes()))
    norm = oracle.synth_f32(4096, SEED, 84)
    tensors.append(("blk.0.attn_norm.weight", G.GGML_F32, [4096], norm.tobytes()))
    tensors.append(("output.weight", G.GGML_Q8_0, [4096, 300], b""))  # tied to token_embd
    offs = G.write_gguf(path, tensors, kv={"general.architecture": "qwen35", "general.name": "synthetic",
                                           "tokenizer.ggml.tokens": ["a", "bb", "ccc"],
                                           "qwen35.block_count": 1, "qwen35.rope.freq_base": 1e6,
                                           "qwen35.list": [1, 2, 3]},
                        shared={"output.weight": "token_embd.weight"})
    return path, mats, norm, offs


def test_gguf_info_reads_the_table(rtb, synth_file):
    path, mats, norm, offs = synth_file
    table, size = rtb.gguf_info(path)
    assert size == os.path.getsize(path)
    names = [t["name"] for t in table]
    assert names == list(mats) + ["blk.0.attn_norm.weight", "output.weight"]
    for t, off in zip(table, offs):
        assert t["offset"] == off and off % 32 == 0
    for t in table[:3]:
        rows, cols, _ = mats[t["name"]]
        assert t["type"] == G.GGML_Q8_0 and t["dims"] == [cols, rows] and t["bytes"] == rows * cols // 32 * 34
    assert table[3]["type"] == G.GGML_F32 and table[3]["bytes"] == 4 * 4096
    assert table[4]["offset"] == table[2]["offset"]


def test_gguf_info_rejects_what_is_not_gguf(rtb, tmp_path):
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGML" + bytes(60))
    with pytest.raises(rtb.RtError):
        rtb.gguf_info(str(bad))
    short = tmp_path / "short.gguf"
    short.write_bytes(b"GGUF" + bytes(6))
    with pytest.raises(rtb.RtError):
        rtb.gguf_info(str(short))


def one_tensor_gguf(path, dims, typ, rel_offset, data: bytes, alignment: int = 32) -> None:
    """A GGUF holding one tensor info with the given raw fields (sizes as an engine file would
    never hold them), then `data` at the aligned data start."""
    import struct
    name = b"t"
    head = b"GGUF" + struct.pack("<IQQ", 3, 1, 1)
    key = b"general.alignment"
    head += struct.pack("<Q", len(key)) + key + struct.pack("<II", 4, alignment)
    head += struct.pack("<Q", len(name)) + name + struct.pack("<I", len(dims))
    head += b"".join(struct.pack("<Q", d % 2 ** 64) for d in dims) + struct.pack("<IQ", typ, rel_offset % 2 ** 64)
    a = alignment if alignment > 0 and alignment & (alignment - 1) == 0 else 32
    start = (len(head) + a - 1) // a * a
    with open(path, "wb") as f:
        f.write(head + b"\0" * (start - len(head)) + data)


def test_gguf_info_takes_a_well_formed_one_tensor_file(rtb, tmp_path):
    p = str(tmp_path / "ok.gguf")
    one_tensor_gguf(p, [256, 2], G.GGML_Q8_0, 0, bytes(2 * 8 * 34))
    table, _ = rtb.gguf_info(p)
    assert table[0]["dims"] == [256, 2] and table[0]["bytes"] == 2 * 8 * 34


@pytest.mark.parametrize("case", ["dims_overflow", "dim_huge", "offset_wraps", "past_end", "ragged_q8_rows",
                                  "alignment_not_pow2", "alignment_zero"])
def test_gguf_info_rejects_crafted_sizes(rtb, tmp_path, case):
    """Sizes that would wrap the loader's arithmetic or send the in-place repack outside the file:
    refused while parsing the header, before anything is read into the arena."""
    p = str(tmp_path / f"{case}.gguf")
    data = bytes(2 * 8 * 34)
    args = {
        "dims_overflow": ([2 ** 32, 2 ** 32, 32], G.GGML_Q8_0, 0, data),  # the product wraps to 0
        "dim_huge": ([32, 2 ** 45], G.GGML_Q8_0, 0, data),
        "offset_wraps": ([256, 2], G.GGML_Q8_0, -32, data),  # offset + bytes wraps past 2^64
        "past_end": ([256, 4], G.GGML_Q8_0, 0, data),
        "ragged_q8_rows": ([48, 2], G.GGML_Q8_0, 0, data),  # 96 weights, but rows of 1.5 blocks
        "alignment_not_pow2": ([256, 2], G.GGML_Q8_0, 0, data),
        "alignment_zero": ([256, 2], G.GGML_Q8_0, 0, data),
    }[case]
    alignment = {"alignment_not_pow2": 48, "alignment_zero": 0}.get(case, 32)
    one_tensor_gguf(p, *args, alignment=alignment)
    with pytest.raises(rtb.RtError) as e:
        rtb.gguf_info(p)
    assert e.value.code == 1


def test_file_sum_is_position_weighted(tmp_path):
    p = tmp_path / "w.bin"
    w = np.array([3, 5, 7], dtype=np.uint64)
    w.tofile(str(p))
    assert G.file_sum(str(p)) == 3 * 1 + 5 * 3 + 7 * 5
    np.array([1, 2], dtype=np.uint64)[::-1].copy().tofile(str(p))
    assert G.file_sum(str(p)) == 2 * 1 + 1 * 3  # the order counts


def test_load_gguf_refuses_a_mis_tied_matrix(rtb, oracle, tmp_path):
    """A tensor sharing a repacked Q8_0 matrix's bytes with other dims (a crafted or mis-tied file):
    the in-place repack would rewrite bytes the other tensor reads, so the load refuses the file
    before it reads anything or touches the arena (no GPU needed: the arena address is never used)."""
    import ctypes as C
    p = str(tmp_path / "mistied.gguf")
    q8 = oracle.synth_q8_0(300, 4096, SEED, 86).tobytes()
    G.write_gguf(p, [("token_embd.weight", G.GGML_Q8_0, [4096, 300], q8),
                     ("output.weight", G.GGML_Q8_0, [4096, 200], b"")],
                 shared={"output.weight": "token_embd.weight"})
    lib = rtb.load()
    arr = (rtb.Tensor * 2)()
    n, st = C.c_int(0), rtb.LoadStats()
    code = lib.rt_b200_load_gguf(None, p.encode(), 1 << 30, 1 << 40, arr, 2, C.byref(n), C.byref(st))
    assert code == 1  # RTB_EINVAL
    assert b"share bytes" in lib.rtb_load_error()


@pytest.mark.gpu
def test_load_gguf_into_hbm(cuda, rtb, oracle, synth_file):
    path, mats, norm, offs = synth_file
    size = os.path.getsize(path)
    arena = cuda.zeros((size + 4095) // 4096 * 4096, dtype=cuda.uint8, device="cuda")
    with rtb.Runtime() as rt:
        table, stats = rt.load_gguf(path, arena.data_ptr(), arena.numel())
        assert stats["file_bytes"] == size
        assert stats["file_sum"] == G.file_sum(path)
        assert stats["q8_matrices"] == 3  # the tied entry shares token_embd's repack
        host = arena.cpu().numpy()
        for t in table[:3]:
            rows, cols, stream = mats[t["name"]]
            assert t["repacked"] and t["dev"] == arena.data_ptr() + t["offset"]
            got = host[t["offset"]:t["offset"] + t["bytes"]]
            want = oracle.repack_split(oracle.synth_q8_0(rows, cols, SEED, stream), rows, cols)
            assert np.array_equal(got, want.reshape(-1))
        f32 = host[table[3]["offset"]:table[3]["offset"] + 4 * 4096].view(np.float32)
        assert np.array_equal(f32.view(np.uint32), norm.view(np.uint32))
        assert table[4]["repacked"] and table[4]["dev"] == table[2]["dev"]
        # a product straight off the loaded arena
        rows, cols, stream = mats["blk.0.attn_qkv.weight"]
        x = oracle.synth_f32(cols, SEED, 85)
        xd = cuda.from_numpy(x).cuda()
        y = cuda.empty((rows,), dtype=cuda.float32, device="cuda")
        rt.gemv(table[0]["dev"], rows, cols, xd.data_ptr(), y.data_ptr())
        want = oracle.gemv(oracle.synth_q8_0(rows, cols, SEED, stream), rows, cols, x)
        assert np.array_equal(y.cpu().numpy().view(np.uint32), want.view(np.uint32))


@pytest.mark.gpu
def test_load_gguf_refuses_a_small_arena(cuda, rtb, synth_file):
    path = synth_file[0]
    arena = cuda.zeros(4096, dtype=cuda.uint8, device="cuda")
    with rtb.Runtime() as rt:
        with pytest.raises(rtb.RtError):
            rt.load_gguf(path, arena.data_ptr(), arena.numel())
