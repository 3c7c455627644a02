"""Row partitioning of the hot-path ops across GPUs (one process per GPU).

Every op on the path is row-independent, so ranks own disjoint row ranges and exchange nothing on the data path:

- RMSNorm, residual add + RMSNorm, SiLU*up, row argmax: contiguous, equal-count row ranges (`row_ranges`);
- q/k RMSNorm + RoPE: contiguous token ranges; a rank's first token sits at global position `start`, so RoPE angles
  stay those of the unsharded batch (`token_shard`);
- causal softmax: a row q of a [matrices, Q, K] score tensor reads q + 1 values and writes K, so equal row counts
  give unequal bytes; `causal_row_ranges` cuts the flattened rows where the cumulative algorithmic bytes reach
  rank / world of the total.

`copy_back` is the one data movement between ranks: every rank's output rows land in one buffer on rank 0 by
point-to-point transfers (NVLink peer traffic under NCCL, TCP under gloo). bench.py (`--gpus N`) partitions one global
batch with these functions and times the ops with and without the copy-back; tests/test_sharding.py runs the same
partition and copy-back on world-size-2 gloo ranks on the CPU.
"""

from __future__ import annotations

from bisect import bisect_left
from dataclasses import dataclass


def row_ranges(rows: int, world: int) -> list[tuple[int, int]]:
    """Contiguous [start, end) ranges covering `rows`, sizes differing by at most one (larger ranges first)."""
    if world <= 0:
        raise ValueError("world size must be positive")
    if rows < 0:
        raise ValueError("rows must be non-negative")
    base, extra = divmod(rows, world)
    out = []
    start = 0
    for r in range(world):
        size = base + (1 if r < extra else 0)
        out.append((start, start + size))
        start += size
    return out


@dataclass(frozen=True)
class TokenShard:
    start: int  # first global token row of this rank
    end: int
    position_offset: int  # RoPE position of the first row (global position of `start`)

    @property
    def tokens(self) -> int:
        return self.end - self.start


def token_shard(tokens: int, world: int, rank: int, position_offset: int = 0) -> TokenShard:
    """This rank's token rows of a `tokens`-row batch whose first row sits at `position_offset`."""
    start, end = row_ranges(tokens, world)[rank]
    return TokenShard(start, end, position_offset + start)


def causal_row_bytes(query_index: int, key_len: int, element_size: int = 4) -> int:
    """Algorithmic bytes of one causal-softmax row: visible keys read plus the whole row written."""
    return (min(query_index + 1, key_len) + key_len) * element_size


def causal_row_ranges(matrices: int, query_len: int, key_len: int, world: int,
                      element_size: int = 4) -> list[tuple[int, int]]:
    """Contiguous ranges of the flattened [matrices * query_len] rows with (nearly) equal algorithmic bytes."""
    if world <= 0:
        raise ValueError("world size must be positive")
    rows = matrices * query_len
    per_matrix = [0]
    for q in range(query_len):
        per_matrix.append(per_matrix[-1] + causal_row_bytes(q, key_len, element_size))
    matrix_bytes = per_matrix[-1]
    total = matrix_bytes * matrices

    def prefix(row: int) -> int:  # bytes of rows [0, row)
        m, q = divmod(row, query_len)
        return m * matrix_bytes + per_matrix[q]

    cuts = [0]
    for r in range(1, world):
        target = total * r / world
        # smallest row whose prefix reaches the target (binary search over the monotone prefix)
        lo, hi = cuts[-1], rows
        while lo < hi:
            mid = (lo + hi) // 2
            if prefix(mid) < target:
                lo = mid + 1
            else:
                hi = mid
        cuts.append(lo)
    cuts.append(rows)
    return [(cuts[i], cuts[i + 1]) for i in range(world)]


def range_bytes(rng: tuple[int, int], query_len: int, key_len: int, element_size: int = 4) -> int:
    return sum(causal_row_bytes(row % query_len, key_len, element_size) for row in range(*rng))


def owner_of(row: int, ranges: list[tuple[int, int]]) -> int:
    """Rank owning global row `row`."""
    starts = [s for s, _ in ranges]
    r = bisect_left(starts, row + 1) - 1
    if r < 0 or not (ranges[r][0] <= row < ranges[r][1]):
        raise IndexError(f"row {row} is outside the partition")
    return r


@dataclass(frozen=True)
class SoftmaxPiece:
    """A run of consecutive rows of one [Q, K] score matrix: rows [query_start, query_start + rows) of `matrix`."""

    matrix: int
    query_start: int
    rows: int


def softmax_pieces(rng: tuple[int, int], query_len: int) -> list[SoftmaxPiece]:
    """Splits a range of flattened [matrices * query_len] rows at matrix boundaries; each piece is one launch of the
    position-aware causal softmax (query offset = query_start), whole matrices are pieces with query_start 0."""
    start, end = rng
    out = []
    row = start
    while row < end:
        m, q = divmod(row, query_len)
        n = min(end - row, query_len - q)
        out.append(SoftmaxPiece(m, q, n))
        row += n
    return out


def copy_back(local, dst, ranges: list[tuple[int, int]], rank: int, group=None) -> None:
    """Gathers every rank's rows into `dst` on rank 0: rank r's `local` holds rows ranges[r] of the global tensor
    (split along dim 0); rank 0 passes the global tensor as `dst` (others pass None). Rank 0 copies its own rows and
    receives the others' directly into their rows of `dst` (one batch of concurrent point-to-point transfers, so
    unequal shard sizes need no padding); the call returns once this rank's transfers are complete."""
    import torch.distributed as dist

    world = len(ranges)
    if rank == 0:
        s, e = ranges[0]
        if e > s:
            dst[s:e].copy_(local[: e - s])
        ops = [dist.P2POp(dist.irecv, dst[ranges[r][0]:ranges[r][1]], r, group)
               for r in range(1, world) if ranges[r][1] > ranges[r][0]]
    else:
        s, e = ranges[rank]
        ops = [dist.P2POp(dist.isend, local[: e - s].contiguous(), 0, group)] if e > s else []
    if ops:
        for work in dist.batch_isend_irecv(ops):
            work.wait()
