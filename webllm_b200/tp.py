"""Row-sharded (tensor-parallel) quantized MUL_MAT across the GPUs of one node.

A weight's M output rows split into contiguous shards, one per rank (rank r
holds rows [start_r, start_r + count_r)). Blocks never split, because the
shards cut along M, not K. Every rank holds the full activation vectors x.
Each rank computes its rows with the library's device GEMV. The ranks then
all-gather the row shards over NCCL (NVLink), so every rank ends with the
full output y[m + M*n].

The reference runs this op on one browser GPU and has no multi-device path;
the sharding here follows the row independence of dst[m + M*n] = sum_k
W[m,k] x[k,n] (src/inference/jsep/ops/matmul.ts:10-17).

Only the local GEMV touches the GPU; the shard arithmetic and the gather
assembly are plain host code, so the CPU tests exercise them with gloo
ranks and a CPU stand-in for the local GEMV.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Sequence

__all__ = ["RowShard", "row_shard", "shard_bytes", "gather_rows", "TPMulMat"]


@dataclass(frozen=True)
class RowShard:
    start: int   # first row of this rank
    count: int   # rows of this rank (the last ranks may hold fewer, or none)
    padded: int  # rows every rank reserves in the gather buffer (ceil(M / world))


def row_shard(M: int, world: int, rank: int) -> RowShard:
    """Contiguous split of M rows over `world` ranks; ranks 0.. take
    ceil(M / world) rows each until the rows run out."""
    if M <= 0 or world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad shard request M={M} world={world} rank={rank}")
    padded = -(-M // world)
    start = min(M, rank * padded)
    count = max(0, min(M, start + padded) - start)
    return RowShard(start, count, padded)


def shard_bytes(weight_rows: bytes | memoryview, row_bytes: int, shard: RowShard) -> memoryview:
    """The raw GGUF rows of one shard (a view, no copy)."""
    mv = memoryview(weight_rows)
    return mv[shard.start * row_bytes:(shard.start + shard.count) * row_bytes]


def gather_rows(y_shard, M: int, N: int, world: int, all_gather: Callable):
    """Assemble the full output from every rank's row shard.

    `y_shard` is this rank's [N, padded] tensor (rows past its count are
    ignored); `all_gather(out, inp)` is torch.distributed.all_gather_into_tensor
    (or a stand-in) filling `out` [world * N * padded] with every rank's `inp`
    in rank order. Returns the [N, M] output in ggml order (row m of vector n
    at [n, m])."""
    import torch

    padded = y_shard.shape[-1]
    flat = torch.empty(world * N * padded, dtype=y_shard.dtype, device=y_shard.device)
    all_gather(flat, y_shard.reshape(-1).contiguous())
    parts = flat.view(world, N, padded).permute(1, 0, 2).reshape(N, world * padded)
    return parts[:, :M]


class TPMulMat:
    """One row-sharded MUL_MAT: this rank's weight rows plus the gather.

    `local(x, y_shard)` computes y_shard[n, r] = sum_k W[start + r, k] x[n, k]
    for r < count (on the GPU: webllm_b200.jsep.mul_mat_device on the rank's
    shard; in the CPU tests: the oracle)."""

    def __init__(self, M: int, N: int, world: int, rank: int, local: Callable, all_gather: Callable):
        self.M, self.N, self.world, self.rank = M, N, world, rank
        self.shard = row_shard(M, world, rank)
        self.local = local
        self.all_gather = all_gather

    def forward(self, x, y_shard=None):
        import torch

        if y_shard is None:
            y_shard = torch.zeros(self.N, self.shard.padded, dtype=torch.float32, device=x.device)
        if self.shard.count:
            self.local(x, y_shard)
        return gather_rows(y_shard, self.M, self.N, self.world, self.all_gather)


def shards_cover(M: int, world: int) -> Sequence[RowShard]:
    """All ranks' shards (for checks)."""
    return [row_shard(M, world, r) for r in range(world)]
