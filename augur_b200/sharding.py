"""Sequence sharding across the GPUs of one box.

Every sequence's K/V and block table are private, so the path shards by
whole sequence: each rank (one process per GPU) owns a block pool and an
allocator and moves only its own sequences; no collective touches cache
data. The only communication is the report at the end (bytes moved and
device time per rank), gathered over the process group.

Assignment is longest-processing-time first: sequences sorted by length
(longest first, ties by index) each go to the rank with the fewest tokens so
far (ties to the lowest rank). Every rank computes the same plan from the
same lengths, so no plan needs to be sent.
"""

from __future__ import annotations

import heapq
from dataclasses import asdict, dataclass
from collections.abc import Sequence

import numpy as np


def lpt_assign(lengths: Sequence[int], n_shards: int) -> list[list[int]]:
    """Sequence indices per shard, each list in increasing index order."""
    if n_shards <= 0:
        raise ValueError("n_shards must be positive")
    lens = np.asarray(lengths, dtype=np.int64)
    if lens.size and lens.min() < 0:
        raise ValueError("lengths must be non-negative")
    order = sorted(range(lens.size), key=lambda i: (-int(lens[i]), i))
    heap = [(0, r) for r in range(n_shards)]
    shards: list[list[int]] = [[] for _ in range(n_shards)]
    for i in order:
        load, r = heapq.heappop(heap)
        shards[r].append(i)
        heapq.heappush(heap, (load + int(lens[i]), r))
    return [sorted(s) for s in shards]


def shard_tokens(shards: Sequence[Sequence[int]], lengths: Sequence[int]) -> list[int]:
    lens = np.asarray(lengths, dtype=np.int64)
    return [int(lens[list(s)].sum()) if len(s) else 0 for s in shards]


def box_lengths(n_seqs: int = 2048, seed: int = 0, median: float = 1024.0, sigma: float = 0.8,
                lo: int = 64, hi: int = 8192) -> np.ndarray:
    """Scale-out workload lengths: lognormal(ln median, sigma) clipped to [lo, hi]."""
    rng = np.random.default_rng(seed)
    return np.clip(np.round(rng.lognormal(np.log(median), sigma, size=n_seqs)), lo, hi).astype(np.int64)


@dataclass
class ShardReport:
    rank: int
    sequences: int
    tokens: int
    bytes_moved: int
    device_ms: float


def gather_reports(report: ShardReport, group=None) -> list[ShardReport]:
    """All ranks' reports, in rank order (every rank must call this)."""
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized():
        return [report]
    out: list[dict | None] = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, asdict(report), group=group)
    return [ShardReport(**r) for r in out]  # type: ignore[arg-type]


def aggregate(reports: Sequence[ShardReport]) -> dict:
    """Whole-job numbers: the job ends when the slowest rank ends."""
    if not reports:
        raise ValueError("no reports")
    total = sum(r.bytes_moved for r in reports)
    slowest = max(r.device_ms for r in reports)
    tokens = [r.tokens for r in reports]
    mean = sum(tokens) / len(tokens)
    return {
        "ranks": len(reports),
        "bytes": total,
        "max_device_ms": slowest,
        "GBps": total / (slowest / 1e3) / 1e9 if slowest > 0 else float("inf"),
        "token_imbalance": (max(tokens) / mean) if mean > 0 else 1.0,
    }
