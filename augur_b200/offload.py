"""Offload KV-cache blocks to pinned host memory and restore them.

augur keeps a prefix's K/V in a PrefixCacheEntry on the device where it was
computed (augur/prefix_cache.py:13-22, cache_prefix :78-98), and its paged
pool has no way out of HBM. Here blocks leave the pool and come back:

- The host format is block-major, ``[n_blocks, layers, kv_heads,
  block_size, head_dim]`` for K and for V, in pinned memory. Each block is one
  self-contained slab of all its layers.
- "staged" path (large transfers): SMs gather blocks into a double-buffered
  staging area in HBM with augur_kv_copy_runs, at HBM speed, while the copy
  engine streams the previous chunk over the host link. Restore runs the
  mirror image: the copy engine fills a staging chunk, SMs scatter it into
  the pool. The SMs stay free for most of the transfer, and the link runs at
  copy-engine speed.
- "direct" path (small transfers): one augur_kv_copy_runs launch reads or
  writes the pinned host buffer in place, through the CUDA unified address
  space, with the vector path's 16-byte accesses. The TMA bulk path is never
  used on host memory.

Block contents round-trip bit-exactly. Only each block's valid rows are
gathered or scattered.
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

    keys / values: pinned CPU ``[n_blocks, layers, kv_heads, block_size, head_dim]``.
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
        """Bytes of K and V in the valid rows of these blocks."""
        _, L, H, _, D = self.keys.shape
        return 2 * L * H * D * self.keys.element_size() * self.n_tokens

    def wait(self) -> None:
        if self.done is not None:
            self.done.synchronize()


def host_buffer(cache: PagedKVCache, n_blocks: int) -> tuple[Tensor, Tensor]:
    """Pinned host K and V buffers for n_blocks blocks of this pool (reusable)."""
    L, _, H, bs, D = cache.keys.shape
    shape = (n_blocks, L, H, bs, D)
    return (torch.empty(shape, dtype=cache.keys.dtype, pin_memory=True),
            torch.empty(shape, dtype=cache.values.dtype, pin_memory=True))


def _rows(cache: PagedKVCache, n: int, rows) -> np.ndarray:
    bs = cache.keys.shape[3]
    r = np.full(n, bs, np.int64) if rows is None else np.broadcast_to(np.asarray(rows, np.int64), (n,)).copy()
    if n and (r.min() < 0 or r.max() > bs):
        raise ValueError("rows per block must be in [0, block_size]")
    return r


def _strides(t: Tensor) -> tuple[int, int, int, int]:
    """(layer, major = block, row, head) element strides of a pool or of a block-major buffer."""
    if t.dim() != 5:
        raise ValueError("expected a 5-d KV tensor")
    return (t.stride(0), t.stride(1), t.stride(3), t.stride(2))


def _block_major_strides(t: Tensor) -> tuple[int, int, int, int]:
    return (t.stride(1), t.stride(0), t.stride(3), t.stride(2))


def _device_runs(cache: PagedKVCache, runs: np.ndarray) -> tuple[Tensor, int, np.ndarray]:
    """Runs (one per block) cut to max_rows and uploaded once; also max_rows and, per block,
    the index of its first piece (length n + 1) so chunks of blocks slice the upload."""
    L, _, H, bs, D = cache.keys.shape
    max_rows = _ops.max_rows_for(D, cache.keys.element_size(), cap_rows=bs)
    pieces = np.maximum(1, -(-runs[:, 4] // max_rows))
    first = np.concatenate([[0], np.cumsum(pieces)])
    return _to_device_runs(split_runs(runs, max_rows), cache.keys.device), max_rows, first


def _copy(src, dst, src_st, dst_st, runs_t: Tensor, max_rows: int, cache: PagedKVCache, stream, host: bool) -> None:
    """copy_runs of device runs from (src_k, src_v) to (dst_k, dst_v) with the given stride maps."""
    L, _, H, bs, D = cache.keys.shape
    (sk, sv), (dk, dv) = src, dst
    majors = lambda t, st: t.shape[0] if st is _block_major_strides else t.shape[1]  # noqa: E731
    pairs = ([(sk, sv, dk, dv)] if sk.stride() == sv.stride() and dk.stride() == dv.stride()
             else [(sk, None, dk, None), (sv, None, dv, None)])
    for a, b, c, d in pairs:
        _ops.copy_runs(
            src_k=a, src_v=b, src_strides=src_st(a), src_majors=majors(a, src_st), src_rows_per_major=bs,
            dst_k=c, dst_v=d, dst_strides=dst_st(c), dst_majors=majors(c, dst_st), dst_rows_per_major=bs,
            runs=runs_t, max_rows=max_rows, n_layers=L, n_heads=H, head_dim=D,
            flags=_lib.COPY_VECTOR if host else _lib.COPY_AUTO, stream=stream, allow_pinned_host=host)


# Staging for the staged path: per (device, dtype, block shape) two chunks of
# K and V, block-major, reused across calls, and the side stream the copy
# engine runs on.
STAGE_BYTES = 16 << 20  # per chunk, for K (and again for V)
_stages: dict[tuple, tuple[Tensor, Tensor]] = {}
_copy_streams: dict[int, torch.cuda.Stream] = {}


def _stage(cache: PagedKVCache, per_chunk: int) -> tuple[Tensor, Tensor]:
    L, _, H, bs, D = cache.keys.shape
    key = (cache.keys.device, cache.keys.dtype, L, H, bs, D)
    st = _stages.get(key)
    if st is None or st[0].shape[1] < per_chunk:
        shape = (2, per_chunk, L, H, bs, D)
        st = (torch.empty(shape, dtype=cache.keys.dtype, device=cache.keys.device),
              torch.empty(shape, dtype=cache.values.dtype, device=cache.values.device))
        _stages[key] = st
    return st


def _copy_stream(device: torch.device) -> torch.cuda.Stream:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    cs = _copy_streams.get(idx)
    if cs is None:
        cs = torch.cuda.Stream(device=torch.device("cuda", idx))
        _copy_streams[idx] = cs
    return cs


def _block_bytes(cache: PagedKVCache) -> int:
    L, _, H, bs, D = cache.keys.shape
    return L * H * bs * D * cache.keys.element_size()


def _choose(path: str, cache: PagedKVCache, n: int) -> str:
    if path not in ("auto", "direct", "staged"):
        raise ValueError(f"unknown path {path!r}")
    if path == "auto":
        return "staged" if n * _block_bytes(cache) >= (4 << 20) else "direct"
    return path


def offload_blocks(
    cache: PagedKVCache,
    block_ids: Sequence[int],
    rows: Sequence[int] | int | None = None,
    out: tuple[Tensor, Tensor] | None = None,
    stream: torch.cuda.Stream | None = None,
    path: str = "auto",
) -> HostKV:
    """Copy pool blocks ``block_ids`` (rows [0, rows[i]) of each; all by default) to pinned host memory.

    Ordered after earlier work on ``stream`` (the current stream by default),
    which may reuse the blocks as soon as the call returns; the result's
    ``done`` event marks the host copy complete. ``out`` reuses buffers from
    host_buffer(). path: "auto" (staged from 4 MB up), "staged" or "direct".
    """
    _ops.require_cuda("offload_blocks", cache.keys, cache.values)
    n = len(block_ids)
    r = _rows(cache, n, rows)
    ids = np.asarray(block_ids, dtype=np.int64).reshape(-1)
    if n and (ids.min() < 0 or ids.max() >= cache.keys.shape[1]):
        raise ValueError("block id outside the pool")
    hk, hv = out if out is not None else host_buffer(cache, n)
    L, _, H, bs, D = cache.keys.shape
    if hk.shape[0] < n or tuple(hk.shape[1:]) != (L, H, bs, D) or hv.shape != hk.shape:
        raise ValueError("host buffer does not match the pool's layout or block count")
    if any(t.device.type != "cpu" or not t.is_pinned() for t in (hk, hv)):
        raise ValueError("host buffers must be in pinned memory (tensor.pin_memory())")
    st = stream if stream is not None else torch.cuda.current_stream(cache.keys.device)
    done = torch.cuda.Event()
    if n and _choose(path, cache, n) == "direct":
        runs = np.zeros((n, 5), dtype=np.int64)
        runs[:, 0] = ids
        runs[:, 2] = np.arange(n)
        runs[:, 4] = r
        runs_t, max_rows, _ = _device_runs(cache, runs)
        _copy((cache.keys, cache.values), (hk, hv), _strides, _block_major_strides, runs_t, max_rows, cache, st,
              host=True)
        done.record(st)
    elif n:
        per = max(1, STAGE_BYTES // _block_bytes(cache))
        sk, sv = _stage(cache, min(per, n))
        # every chunk's runs go up in one copy before any wait is queued, so the
        # host never blocks on the stream while it issues the pipeline
        runs = np.zeros((n, 5), dtype=np.int64)
        runs[:, 0] = ids
        runs[:, 2] = np.arange(n) % per
        runs[:, 4] = r
        runs_t, max_rows, first = _device_runs(cache, runs)
        cs = _copy_stream(cache.keys.device)
        cs.wait_stream(st)  # staging is free of earlier calls' work on either stream
        st.wait_stream(cs)
        freed = [None, None]
        for g, g0 in enumerate(range(0, n, per)):
            m, buf = min(per, n - g0), g % 2
            if freed[buf] is not None:
                st.wait_event(freed[buf])
            _copy((cache.keys, cache.values), (sk[buf], sv[buf]), _strides, _block_major_strides,
                  runs_t[first[g0] : first[g0 + m]], max_rows, cache, st, host=False)
            gathered = torch.cuda.Event()
            gathered.record(st)
            cs.wait_event(gathered)
            with torch.cuda.stream(cs):
                hk[g0 : g0 + m].copy_(sk[buf, :m], non_blocking=True)
                hv[g0 : g0 + m].copy_(sv[buf, :m], non_blocking=True)
            freed[buf] = torch.cuda.Event()
            freed[buf].record(cs)
        done.record(cs)
    else:
        done.record(st)
    return HostKV(keys=hk, values=hv, rows=r, block_size=bs, done=done)


def restore_blocks(
    cache: PagedKVCache,
    host: HostKV,
    dst_block_ids: Sequence[int],
    stream: torch.cuda.Stream | None = None,
    path: str = "auto",
) -> None:
    """Copy every offloaded block i back into pool block dst_block_ids[i] (its valid rows).

    The pool writes are ordered on ``stream`` (later work on it sees them).
    """
    _ops.require_cuda("restore_blocks", cache.keys, cache.values)
    n = host.n_blocks
    if len(dst_block_ids) != n:
        raise ValueError("one destination block per offloaded block is required")
    L, _, H, bs, D = cache.keys.shape
    if tuple(host.keys.shape[1:]) != (L, H, bs, D):
        raise ValueError("offloaded blocks do not match the pool's layout")
    ids = np.asarray(dst_block_ids, dtype=np.int64).reshape(-1)
    if n and (ids.min() < 0 or ids.max() >= cache.keys.shape[1]):
        raise ValueError("block id outside the pool")
    st = stream if stream is not None else torch.cuda.current_stream(cache.keys.device)
    if n == 0:
        return
    if host.done is not None:
        st.wait_event(host.done)  # an offload still in flight finishes first
    if _choose(path, cache, n) == "direct":
        runs = np.zeros((n, 5), dtype=np.int64)
        runs[:, 0] = np.arange(n)
        runs[:, 2] = ids
        runs[:, 4] = host.rows
        runs_t, max_rows, _ = _device_runs(cache, runs)
        _copy((host.keys, host.values), (cache.keys, cache.values), _block_major_strides, _strides, runs_t, max_rows,
              cache, st, host=True)
        return
    per = max(1, STAGE_BYTES // _block_bytes(cache))
    sk, sv = _stage(cache, min(per, n))
    runs = np.zeros((n, 5), dtype=np.int64)
    runs[:, 0] = np.arange(n) % per
    runs[:, 2] = ids
    runs[:, 4] = host.rows
    runs_t, max_rows, first = _device_runs(cache, runs)  # uploaded before any wait is queued
    cs = _copy_stream(cache.keys.device)
    cs.wait_stream(st)
    consumed = [None, None]
    for g, g0 in enumerate(range(0, n, per)):
        m, buf = min(per, n - g0), g % 2
        if consumed[buf] is not None:
            cs.wait_event(consumed[buf])
        with torch.cuda.stream(cs):
            sk[buf, :m].copy_(host.keys[g0 : g0 + m], non_blocking=True)
            sv[buf, :m].copy_(host.values[g0 : g0 + m], non_blocking=True)
        landed = torch.cuda.Event()
        landed.record(cs)
        st.wait_event(landed)
        _copy((sk[buf], sv[buf]), (cache.keys, cache.values), _block_major_strides, _strides,
              runs_t[first[g0] : first[g0 + m]], max_rows, cache, st, host=False)
        consumed[buf] = torch.cuda.Event()
        consumed[buf].record(st)
    cs.wait_stream(st)  # the next user of the staging chunks on the copy stream waits for the scatters


def offload_sequence(cache: PagedKVCache, table: SequenceBlockTable,
                     stream: torch.cuda.Stream | None = None, path: str = "auto") -> HostKV:
    """Offload positions [0, table.seq_len) of a sequence (its used blocks, valid rows only)."""
    bs = table.block_size
    if bs != cache.keys.shape[3]:
        raise ValueError("block table block_size must equal the cache block size")
    n = -(-table.seq_len // bs)
    if n > len(table.block_ids):
        raise ValueError("position exceeds block table capacity")
    rows = np.minimum(bs, table.seq_len - np.arange(n) * bs)
    return offload_blocks(cache, table.block_ids[:n], rows, stream=stream, path=path)


def restore_sequence(cache: PagedKVCache, host: HostKV,
                     stream: torch.cuda.Stream | None = None, path: str = "auto") -> SequenceBlockTable:
    """Allocate blocks from the pool's allocator, restore an offloaded sequence into them and
    return its new block table (seq_len = the offloaded tokens)."""
    ids = cache.allocator.allocate_many(host.n_blocks)
    restore_blocks(cache, host, ids, stream=stream, path=path)
    return SequenceBlockTable(block_ids=ids, block_size=host.block_size, seq_len=host.n_tokens)


def offload_prefix_entry(entry: PrefixCacheEntry) -> PrefixCacheEntry:
    """The same prefix entry with its K/V (and logits) in pinned host memory.

    copy_prefix_into_cache reads such an entry in place, without staging it in
    device memory first.
    """
    pin = lambda t: t if t.device.type == "cpu" and t.is_pinned() else t.to("cpu").pin_memory()  # noqa: E731
    return PrefixCacheEntry(token_ids=entry.token_ids, keys=pin(entry.keys), values=pin(entry.values),
                            logits=pin(entry.logits))
