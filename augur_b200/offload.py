"""Offload KV-cache blocks to pinned host memory and restore them.

augur keeps a prefix's K/V in a PrefixCacheEntry on the device where it was
computed (augur/prefix_cache.py:13-22, cache_prefix :78-98), and its paged
pool has no way out of HBM. Here blocks leave the pool and come back in one
augur_kv_copy_runs launch each way:

- offload gathers the chosen pool blocks, all layers with K and V, straight
  into a pinned host buffer laid out like the pool, `[layers, n_blocks,
  kv_heads, block_size, head_dim]`. The device writes host memory in place
  over the host link, so there is no staging buffer and no extra HBM pass.
- restore scatters such a buffer back into any pool blocks, which the
  allocator may pick anew; again the device reads host memory in place.

Host memory is reached through the CUDA unified address space (pinned
allocations are device-addressable). The copy uses the run-copy vector path,
with 16-byte loads and stores; the TMA bulk path is not used on host memory.
Block contents round-trip bit-exactly. Only each block's valid rows move;
the rest of a host block is left as allocated.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass, field

import numpy as np
import torch
from torch import Tensor

from . import _lib, _ops
from .batched import _to_device_runs, split_runs
from .paged_kv_cache import PagedKVCache, SequenceBlockTable
from .prefix_cache import PrefixCacheEntry


@dataclass
class HostKV:
    """K/V blocks in pinned host memory, in pool layout.

    keys / values: pinned CPU ``[layers, n_blocks, kv_heads, block_size, head_dim]``.
    rows[i]: valid rows of block i (the rest were not copied).
    done: CUDA event recorded after the offload copy; wait() before reading on the host.
    """

    keys: Tensor
    values: Tensor
    rows: np.ndarray
    block_size: int
    done: torch.cuda.Event | None = field(default=None, repr=False)

    @property
    def n_blocks(self) -> int:
        return int(self.rows.shape[0])

    @property
    def n_tokens(self) -> int:
        return int(self.rows.sum())

    @property
    def nbytes(self) -> int:
        """Bytes of K and V moved by one offload or restore of these blocks."""
        L, _, H, _, D = self.keys.shape
        return 2 * L * H * D * self.keys.element_size() * self.n_tokens

    def wait(self) -> None:
        if self.done is not None:
            self.done.synchronize()


def host_buffer(cache: PagedKVCache, n_blocks: int) -> tuple[Tensor, Tensor]:
    """Pinned host K and V buffers for n_blocks blocks of this pool (reusable)."""
    L, _, H, bs, D = cache.keys.shape
    shape = (L, n_blocks, H, bs, D)
    return (torch.empty(shape, dtype=cache.keys.dtype, pin_memory=True),
            torch.empty(shape, dtype=cache.values.dtype, pin_memory=True))


def _rows(cache: PagedKVCache, n: int, rows) -> np.ndarray:
    bs = cache.keys.shape[3]
    r = np.full(n, bs, np.int64) if rows is None else np.broadcast_to(np.asarray(rows, np.int64), (n,)).copy()
    if n and (r.min() < 0 or r.max() > bs):
        raise ValueError("rows per block must be in [0, block_size]")
    return r


def _copy(src_k, src_v, dst_k, dst_v, runs: np.ndarray, cache: PagedKVCache, stream) -> None:
    L, _, H, bs, D = cache.keys.shape
    max_rows = _ops.max_rows_for(D, cache.keys.element_size(), cap_rows=bs)
    runs_t = _to_device_runs(split_runs(runs, max_rows), cache.keys.device)
    st = lambda t: (t.stride(0), t.stride(1), t.stride(3), t.stride(2))  # noqa: E731
    pairs = ([(src_k, src_v, dst_k, dst_v)] if src_k.stride() == src_v.stride() and dst_k.stride() == dst_v.stride()
             else [(src_k, None, dst_k, None), (src_v, None, dst_v, None)])
    for sk, sv, dk, dv in pairs:
        _ops.copy_runs(
            src_k=sk, src_v=sv, src_strides=st(sk), src_majors=sk.shape[1], src_rows_per_major=sk.shape[3],
            dst_k=dk, dst_v=dv, dst_strides=st(dk), dst_majors=dk.shape[1], dst_rows_per_major=dk.shape[3],
            runs=runs_t, max_rows=max_rows, n_layers=L, n_heads=H, head_dim=D,
            flags=_lib.COPY_VECTOR, stream=stream, allow_pinned_host=True)


def offload_blocks(
    cache: PagedKVCache,
    block_ids: Sequence[int],
    rows: Sequence[int] | int | None = None,
    out: tuple[Tensor, Tensor] | None = None,
    stream: torch.cuda.Stream | None = None,
) -> HostKV:
    """Copy pool blocks ``block_ids`` (rows [0, rows[i]) of each; all by default) to pinned host memory.

    Stream-ordered on ``stream`` (the current stream by default); the result's
    ``done`` event marks completion. ``out`` reuses buffers from host_buffer().
    """
    _ops.require_cuda("offload_blocks", cache.keys, cache.values)
    n = len(block_ids)
    r = _rows(cache, n, rows)
    ids = np.asarray(block_ids, dtype=np.int64).reshape(-1)
    if n and (ids.min() < 0 or ids.max() >= cache.keys.shape[1]):
        raise ValueError("block id outside the pool")
    hk, hv = out if out is not None else host_buffer(cache, n)
    if hk.shape[1] < n or hk.shape[0] != cache.keys.shape[0] or hk.shape[2:] != cache.keys.shape[2:]:
        raise ValueError("host buffer does not match the pool's layout or block count")
    st = stream if stream is not None else torch.cuda.current_stream(cache.keys.device)
    if n:
        runs = np.zeros((n, 5), dtype=np.int64)
        runs[:, 0] = ids
        runs[:, 2] = np.arange(n)
        runs[:, 4] = r
        _copy(cache.keys, cache.values, hk, hv, runs, cache, st)
    done = torch.cuda.Event()
    done.record(st)
    return HostKV(keys=hk, values=hv, rows=r, block_size=cache.keys.shape[3], done=done)


def restore_blocks(
    cache: PagedKVCache,
    host: HostKV,
    dst_block_ids: Sequence[int],
    stream: torch.cuda.Stream | None = None,
) -> None:
    """Copy every offloaded block i back into pool block dst_block_ids[i] (its valid rows)."""
    _ops.require_cuda("restore_blocks", cache.keys, cache.values)
    if len(dst_block_ids) != host.n_blocks:
        raise ValueError("one destination block per offloaded block is required")
    if host.keys.shape[0] != cache.keys.shape[0] or host.keys.shape[2:] != cache.keys.shape[2:]:
        raise ValueError("offloaded blocks do not match the pool's layout")
    ids = np.asarray(dst_block_ids, dtype=np.int64).reshape(-1)
    if host.n_blocks and (ids.min() < 0 or ids.max() >= cache.keys.shape[1]):
        raise ValueError("block id outside the pool")
    st = stream if stream is not None else torch.cuda.current_stream(cache.keys.device)
    if host.n_blocks:
        runs = np.zeros((host.n_blocks, 5), dtype=np.int64)
        runs[:, 0] = np.arange(host.n_blocks)
        runs[:, 2] = ids
        runs[:, 4] = host.rows
        _copy(host.keys, host.values, cache.keys, cache.values, runs, cache, st)


def offload_sequence(cache: PagedKVCache, table: SequenceBlockTable,
                     stream: torch.cuda.Stream | None = None) -> HostKV:
    """Offload positions [0, table.seq_len) of a sequence (its used blocks, valid rows only)."""
    bs = table.block_size
    if bs != cache.keys.shape[3]:
        raise ValueError("block table block_size must equal the cache block size")
    n = -(-table.seq_len // bs)
    if n > len(table.block_ids):
        raise ValueError("position exceeds block table capacity")
    rows = np.minimum(bs, table.seq_len - np.arange(n) * bs)
    return offload_blocks(cache, table.block_ids[:n], rows, stream=stream)


def restore_sequence(cache: PagedKVCache, host: HostKV,
                     stream: torch.cuda.Stream | None = None) -> SequenceBlockTable:
    """Allocate blocks from the pool's allocator, restore an offloaded sequence into them and
    return its new block table (seq_len = the offloaded tokens)."""
    ids = cache.allocator.allocate_many(host.n_blocks)
    restore_blocks(cache, host, ids, stream=stream)
    return SequenceBlockTable(block_ids=ids, block_size=host.block_size, seq_len=host.n_tokens)


def offload_prefix_entry(entry: PrefixCacheEntry) -> PrefixCacheEntry:
    """The same prefix entry with its K/V (and logits) in pinned host memory.

    copy_prefix_into_cache reads such an entry in place, without staging it in
    device memory first.
    """
    pin = lambda t: t if t.device.type == "cpu" and t.is_pinned() else t.to("cpu").pin_memory()  # noqa: E731
    return PrefixCacheEntry(token_ids=entry.token_ids, keys=pin(entry.keys), values=pin(entry.values),
                            logits=pin(entry.logits))
