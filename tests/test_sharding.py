"""Row sharding across ranks: partition arithmetic, and world-size-2 gloo runs on the CPU in which every rank computes
its rows with the oracle and rank 0 checks the gathered result against the unsharded computation (the same
partition bench.py uses on GPUs, where each rank runs the device kernels instead)."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from cppinf_b200.shard import (causal_row_bytes, causal_row_ranges, owner_of, range_bytes, row_ranges,
                               softmax_pieces, token_shard)


@pytest.mark.parametrize("rows,world", [(2048, 1), (2048, 2), (2048, 8), (7, 3), (0, 4), (3, 8)])
def test_row_ranges_cover_rows_exactly_once(rows, world):
    ranges = row_ranges(rows, world)
    assert len(ranges) == world
    assert ranges[0][0] == 0 and ranges[-1][1] == rows
    for (s0, e0), (s1, _) in zip(ranges, ranges[1:]):
        assert e0 == s1
    sizes = [e - s for s, e in ranges]
    assert max(sizes) - min(sizes) <= 1


def test_token_shard_keeps_global_positions():
    shards = [token_shard(16384, 8, r, position_offset=0) for r in range(8)]
    assert [s.position_offset for s in shards] == [r * 2048 for r in range(8)]
    assert all(s.tokens == 2048 for s in shards)
    assert token_shard(10, 4, 3, position_offset=100).position_offset == 100 + 8


@pytest.mark.parametrize("world", [2, 4, 8])
def test_causal_row_ranges_balance_bytes(world):
    ranges = causal_row_ranges(16, 2048, 2048, world)
    assert ranges[0][0] == 0 and ranges[-1][1] == 16 * 2048
    loads = [range_bytes(r, 2048, 2048) for r in ranges]
    assert max(loads) / min(loads) < 1.01
    assert sum(loads) == 16 * sum(causal_row_bytes(q, 2048) for q in range(2048))


def test_causal_row_ranges_single_matrix_split_is_not_equal_count():
    ranges = causal_row_ranges(1, 1000, 1000, 2)
    # the later rows read more keys, so the first rank gets more rows
    assert ranges[0][1] - ranges[0][0] > ranges[1][1] - ranges[1][0]
    assert owner_of(0, ranges) == 0 and owner_of(999, ranges) == 1


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_softmax_pieces_tile_each_rank_range(world):
    for rng_ in causal_row_ranges(5, 64, 64, world):
        pieces = softmax_pieces(rng_, 64)
        assert sum(p.rows for p in pieces) == rng_[1] - rng_[0]
        row = rng_[0]
        for p in pieces:
            assert p.matrix * 64 + p.query_start == row and 0 < p.rows and p.query_start + p.rows <= 64
            row += p.rows


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, result_path: str) -> None:
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(repo))
    import torch

    from cppinf_b200.shard import causal_row_ranges, copy_back, row_ranges, softmax_pieces, token_shard
    from oracle.oracle import Oracle, f32_to_bf16

    os.environ["OMP_NUM_THREADS"] = "1"
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    oracle = Oracle()
    rng = np.random.default_rng(42)  # every rank draws the same global batch and keeps its own rows
    q = f32_to_bf16(rng.standard_normal((64, 4, 128)).astype(np.float32))
    k = f32_to_bf16(rng.standard_normal((64, 2, 128)).astype(np.float32))
    qw = f32_to_bf16((1 + 0.1 * rng.standard_normal(128)).astype(np.float32))
    kw = f32_to_bf16((1 + 0.1 * rng.standard_normal(128)).astype(np.float32))
    x = f32_to_bf16(rng.standard_normal((50, 256)).astype(np.float32))
    w = f32_to_bf16((1 + 0.1 * rng.standard_normal(256)).astype(np.float32))
    scores = (rng.standard_normal((3, 40, 40)) * 2).astype(np.float32)

    # q/k: token rows with global RoPE positions
    q_ranges = row_ranges(64, world)
    shard = token_shard(64, world, rank, position_offset=7)
    assert (shard.start, shard.end) == q_ranges[rank]
    q_out, k_out = oracle.qk_norm_rope(q[shard.start:shard.end], k[shard.start:shard.end], qw, kw, 1e-6,
                                       shard.position_offset, 1e6)
    # RMSNorm: equal row counts
    x_ranges = row_ranges(50, world)
    s0, e0 = x_ranges[rank]
    y = oracle.rms_norm(x[s0:e0], w, 1e-6)
    # causal softmax: byte-balanced rows, computed per piece of one matrix at its query offset
    c_ranges = causal_row_ranges(3, 40, 40, world)
    flat = scores.reshape(-1, 40)
    parts = []
    for piece in softmax_pieces(c_ranges[rank], 40):
        rows = scores[piece.matrix, piece.query_start:piece.query_start + piece.rows]
        parts.append(oracle.position_causal_softmax(rows[None, None], 0.125, [piece.query_start], [piece.rows],
                                                    [40])[0, 0])
    probs = np.concatenate(parts) if parts else np.zeros((0, 40), np.float32)
    assert probs.shape[0] == c_ranges[rank][1] - c_ranges[rank][0]

    # copy-back of every rank's rows into one buffer on rank 0 (bench.py does the same over NCCL)
    def bits(a):
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16) if a.dtype == np.uint16 else a)

    out = {}
    for name, local, ranges, shape, dtype in (("q", q_out, q_ranges, q.shape, torch.int16),
                                              ("k", k_out, q_ranges, k.shape, torch.int16),
                                              ("y", y, x_ranges, x.shape, torch.int16),
                                              ("p", probs, c_ranges, flat.shape, torch.float32)):
        dst = torch.zeros(shape, dtype=dtype) if rank == 0 else None
        copy_back(bits(local), dst, ranges, rank)
        out[name] = dst
    t = torch.tensor([float(rank + 1)], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)  # the max-over-ranks timing reduction bench.py uses
    if rank == 0:
        full_q, full_k = oracle.qk_norm_rope(q, k, qw, kw, 1e-6, 7, 1e6)

        def same(t_, a):
            return np.array_equal(t_.numpy().view(np.uint16) if t_.dtype == torch.int16 else t_.numpy(), a)

        ok = (same(out["q"], full_q) and same(out["k"], full_k) and same(out["y"], oracle.rms_norm(x, w, 1e-6))
              and same(out["p"], oracle.scaled_causal_softmax(scores, 0.125).reshape(-1, 40))
              and t.item() == float(world))
        Path(result_path).write_text("ok" if ok else "mismatch")
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_gloo_ranks_reassemble_the_unsharded_result(tmp_path, world):
    result = tmp_path / "result.txt"
    mp.start_processes(_worker, args=(world, _free_port(), str(result)), nprocs=world, start_method="spawn",
                       join=True)
    assert result.read_text() == "ok"
