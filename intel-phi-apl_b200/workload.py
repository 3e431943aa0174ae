"""The benchmark workloads of BASELINE.json, as data: the 9B-class Q8_0 matrices and the decode
step that runs them, with their algorithmic byte and flop counts.

Shapes (N x K, N output rows, K = cols), from the reference model's products
(src/apl/qwen35.apl:92-98, 116-126, 158-160, 170-172) at the 9B sizes BASELINE.json names:
fused QKV 8192 x 4096, out 4096 x 4096, gate and up 12288 x 4096 (run fused with SiLU), down
4096 x 12288, output head 151936 x 4096, draft head 32768 of the head's rows.

Algorithmic units: a product reads N*K*34/32 weight bytes (Q8_0), 4*M*K of x and writes 4*M*N
of y; a gather adds 4 bytes per selected row; flops = 2*M*N*K. A SwiGLU pair counts both
matrices and writes one h.
"""
from __future__ import annotations

from dataclasses import dataclass

D, FF, QKV, VOCAB, HOT, LAYERS = 4096, 12288, 8192, 151936, 32768, 32


@dataclass(frozen=True)
class Product:
    name: str
    rows: int          # N, whole product (all shards)
    cols: int          # K
    kind: str          # "gemv" (plain), "silu" (gate+up pair), "rows" (gather)
    nsel: int = 0      # gather: rows selected

    def weight_bytes(self) -> int:
        n = self.nsel if self.kind == "rows" else self.rows
        mats = 2 if self.kind == "silu" else 1
        return mats * n * self.cols * 34 // 32

    def bytes(self, m: int = 1) -> int:
        n = self.nsel if self.kind == "rows" else self.rows
        extra = 4 * n if self.kind == "rows" else 0
        return self.weight_bytes() + 4 * m * self.cols + 4 * m * n + extra

    def flops(self, m: int = 1) -> int:
        n = self.nsel if self.kind == "rows" else self.rows
        mats = 2 if self.kind == "silu" else 1
        return 2 * m * mats * n * self.cols


# BASELINE config 2 (the decode shapes, batch 1)
SWEEP = [
    Product("gate_up_silu", FF, D, "silu"),
    Product("down", D, FF, "gemv"),
    Product("qkv", QKV, D, "gemv"),
    Product("out", D, D, "gemv"),
    Product("head", VOCAB, D, "gemv"),
]

# one decode step's weight products, in the order a layer runs them. Each
# entry is one round (one launch; under sharding one all-gather).
LAYER = [SWEEP[2], SWEEP[3], SWEEP[0], SWEEP[1]]
HEAD = SWEEP[4]
DRAFT = Product("draft_head", VOCAB, D, "rows", HOT)


def step_rounds(layers: int = LAYERS) -> list[Product]:
    return [p for _ in range(layers) for p in LAYER] + [HEAD]


def step_bytes(m: int = 1, layers: int = LAYERS) -> int:
    return sum(p.bytes(m) for p in step_rounds(layers))


def step_weight_bytes(layers: int = LAYERS) -> int:
    return sum(p.weight_bytes() for p in step_rounds(layers))


def shard_rows(rows: int, rank: int, world: int) -> tuple[int, int]:
    """(first row, row count) of this rank's shard: rows split into world consecutive slices,
    rank-major. The products' all-gather restores y in the same order."""
    if rows % world:
        raise ValueError(f"{rows} rows do not split over {world} ranks")
    n = rows // world
    return rank * n, n
