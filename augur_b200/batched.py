"""Batched, all-layer entry points for the prefill -> decode cache path.

augur calls its cache once per layer per sequence from attention
(augur/attention.py:57-72). These entry points move the same bytes for many
sequences and all layers in one launch each:

  write_paged_kv_batch     slot-mapped scatter of [layers, tokens, heads, dim]
  write_paged_kv_prefill   right-padded prefill [layers, batch, seq, heads, dim] into tables
  append_decode            one new token per sequence per layer (decode step)
  handoff_contiguous_to_paged  finished prefill in a contiguous KVCache -> paged pool
  fork_prefix / cow_partial_blocks  refcounted prefix sharing and copy-on-write
  copy_blocks              explicit block copies (all layers, K and V)
  read_paged_kv_batch      logical-order gather of many sequences, all layers

Each is, byte for byte, the reference's write_paged_kv / read_paged_kv
(augur/paged_kv_cache.py:167-221) applied per sequence and per layer; the
parity tests check exactly that composition. Host bookkeeping (block
allocation, table growth) happens here, before the launch, in the same order
the per-token reference loop would perform it.
"""

from __future__ import annotations

import math
from collections.abc import Sequence

import numpy as np
import torch
from torch import Tensor

from . import _lib, _ops
from .kv_cache import KVCache
from .paged_kv_cache import PagedKVCache, SequenceBlockTable, pool_strides


def _to_device_i64(a: np.ndarray | Tensor, device: torch.device) -> Tensor:
    t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.int64)) if isinstance(a, np.ndarray) else a
    return t.to(device=device, dtype=torch.int64)


def _to_device_runs(a: np.ndarray | Tensor, device: torch.device) -> Tensor:
    t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)) if isinstance(a, np.ndarray) else a
    return t.to(device=device, dtype=torch.int32).contiguous()


def _kv_pairs(sk: Tensor, sv: Tensor, dk: Tensor, dv: Tensor):
    """One launch for K and V together when their layouts agree, else one each."""
    if sk.stride() == sv.stride() and sk.dtype == sv.dtype and dk.stride() == dv.stride():
        return [(sk, sv, dk, dv)]
    return [(sk, None, dk, None), (sv, None, dv, None)]


# ---------------------------------------------------------------------------
# scatter family
# ---------------------------------------------------------------------------


def write_paged_kv_batch(
    cache: PagedKVCache,
    key: Tensor,
    value: Tensor,
    slot_mapping: Tensor | np.ndarray,
    layer_idx: int | None = None,
    stream: torch.cuda.Stream | None = None,
) -> None:
    """Scatter tokens into the pool by slot: token t -> slot_mapping[t] (-1 skips it).

    key/value: ``[layers, tokens, kv_heads, head_dim]`` with layer_idx None
    (all cache layers in one launch), or ``[tokens, kv_heads, head_dim]`` for
    one layer. slot_mapping: int64 ``[tokens]`` on the cache's device,
    slot = block_id * block_size + offset; a host numpy array of at most 32
    slots is passed to the kernel by value (larger ones are copied over).
    """
    if key.shape != value.shape:
        raise ValueError("key and value must have the same shape")
    _ops.require_cuda("write_paged_kv_batch", cache.keys, cache.values, key, value,
                      None if isinstance(slot_mapping, np.ndarray) else slot_mapping)
    pool_k, pool_v = cache.keys, cache.values
    if layer_idx is None:
        if key.dim() != 4 or key.shape[0] != pool_k.shape[0]:
            raise ValueError("key/value must be [layers, tokens, kv_heads, head_dim] for all layers")
        n_layers = key.shape[0]
        src = lambda t: (t.stride(0), 0, t.stride(1), t.stride(2))  # noqa: E731
        dst_layer_view = False
    else:
        if not 0 <= layer_idx < pool_k.shape[0]:
            raise ValueError("layer_idx is outside the cache layer range")
        if key.dim() != 3:
            raise ValueError("key/value must be [tokens, kv_heads, head_dim] for one layer")
        key, value = key.unsqueeze(0), value.unsqueeze(0)
        pool_k, pool_v = pool_k[layer_idx : layer_idx + 1], pool_v[layer_idx : layer_idx + 1]
        n_layers = 1
        src = lambda t: (0, 0, t.stride(1), t.stride(2))  # noqa: E731
        dst_layer_view = False
    _, n_tokens, num_heads, head_dim = key.shape
    if (num_heads, head_dim) != (pool_k.shape[2], pool_k.shape[4]):
        raise ValueError("key/value shape does not match cache shape")
    if tuple(slot_mapping.shape) != (n_tokens,):
        raise ValueError("slot_mapping must have shape [tokens]")
    if isinstance(slot_mapping, np.ndarray):
        slot_mapping = np.ascontiguousarray(slot_mapping, dtype=np.int64)
        if not (_ops.host_index_ok(n_tokens, key, pool_k) and value.dtype == key.dtype):
            slot_mapping = _to_device_i64(slot_mapping, pool_k.device)
    elif slot_mapping.dtype != torch.int64:
        slot_mapping = slot_mapping.to(torch.int64)
    for sk, sv, dk, dv in _kv_pairs(key, value, pool_k, pool_v):
        _ops.scatter(
            src_k=sk, src_v=sv, src_k_strides=src(sk), src_v_strides=None if sv is None else src(sv),
            tokens_per_row=max(1, n_tokens),
            dst_k=dk, dst_v=dv, dst_strides=pool_strides(dk, dst_layer_view),
            rows_per_major=cache.block_size, num_majors=dk.shape[1],
            index=slot_mapping, index_strides=(0, 1 if isinstance(slot_mapping, np.ndarray) else slot_mapping.stride(0)),
            index_row_base=0, n_tokens=n_tokens, n_layers=n_layers, n_heads=num_heads, head_dim=head_dim,
            stream=stream,
        )


def prefill_slot_mapping(
    tables: Sequence[SequenceBlockTable],
    seq_lens: Sequence[int],
    allocator,
    max_len: int | None = None,
    start_positions: Sequence[int] | None = None,
) -> np.ndarray:
    """Grow each table for positions [start, start + len) and return int64 slots ``[B, max_len]``.

    Padding (beyond a sequence's length) is -1. Blocks are allocated sequence
    by sequence in table order, as the reference's per-sequence
    write_paged_kv calls would allocate them.
    """
    lens = np.asarray(seq_lens, dtype=np.int64)
    if lens.size and lens.min() < 0:
        raise ValueError("seq_lens must be non-negative")
    width = int(max_len if max_len is not None else (lens.max() if lens.size else 0))
    if lens.size and lens.max() > width:
        raise ValueError("a sequence is longer than max_len")
    starts = np.zeros_like(lens) if start_positions is None else np.asarray(start_positions, np.int64)
    out = np.full((len(tables), width), -1, dtype=np.int64)
    for b, table in enumerate(tables):
        n = int(lens[b])
        if n == 0:
            continue
        s0 = int(starts[b])
        table.ensure_position(s0 + n - 1, allocator)
        pos = np.arange(s0, s0 + n, dtype=np.int64)
        ids = np.asarray(table.block_ids, dtype=np.int64)
        bs = table.block_size
        out[b, :n] = ids[pos // bs] * bs + pos % bs
    return out


def write_paged_kv_prefill(
    cache: PagedKVCache,
    key: Tensor,
    value: Tensor,
    slot_mapping: Tensor,
    stream: torch.cuda.Stream | None = None,
) -> None:
    """Scatter right-padded prefill K/V ``[layers, batch, seq, kv_heads, head_dim]`` by slot.

    slot_mapping: int64 ``[batch, seq]`` on the device (prefill_slot_mapping
    builds it; -1 marks padding). All layers in one launch.
    """
    if key.shape != value.shape:
        raise ValueError("key and value must have the same shape")
    _ops.require_cuda("write_paged_kv_prefill", cache.keys, cache.values, key, value, slot_mapping)
    if key.dim() != 5 or key.shape[0] != cache.keys.shape[0]:
        raise ValueError("key/value must be [layers, batch, seq, kv_heads, head_dim]")
    n_layers, batch, seq, num_heads, head_dim = key.shape
    if (num_heads, head_dim) != (cache.keys.shape[2], cache.keys.shape[4]):
        raise ValueError("key/value shape does not match cache shape")
    if slot_mapping.shape != (batch, seq) or slot_mapping.dtype != torch.int64:
        raise ValueError("slot_mapping must be int64 [batch, seq]")
    src = lambda t: (t.stride(0), t.stride(1), t.stride(2), t.stride(3))  # noqa: E731
    for sk, sv, dk, dv in _kv_pairs(key, value, cache.keys, cache.values):
        _ops.scatter(
            src_k=sk, src_v=sv, src_k_strides=src(sk), src_v_strides=None if sv is None else src(sv),
            tokens_per_row=max(1, seq),
            dst_k=dk, dst_v=dv, dst_strides=pool_strides(dk, False),
            rows_per_major=cache.block_size, num_majors=dk.shape[1],
            index=slot_mapping, index_strides=(slot_mapping.stride(0), slot_mapping.stride(1)),
            index_row_base=0, n_tokens=batch * seq, n_layers=n_layers, n_heads=num_heads,
            head_dim=head_dim, stream=stream,
        )


def decode_slot_mapping(tables: Sequence[SequenceBlockTable], allocator) -> np.ndarray:
    """Grow each table by one position (its seq_len) and return the int64 slots ``[B]``."""
    out = np.empty(len(tables), dtype=np.int64)
    for b, table in enumerate(tables):
        pos = table.seq_len
        table.ensure_position(pos, allocator)
        out[b] = table.block_ids[pos // table.block_size] * table.block_size + pos % table.block_size
    return out


def append_decode(
    cache: PagedKVCache,
    tables: Sequence[SequenceBlockTable] | None,
    key: Tensor,
    value: Tensor,
    slot_mapping: Tensor | None = None,
    stream: torch.cuda.Stream | None = None,
) -> Tensor:
    """Append one token per sequence, all layers: key/value ``[layers, batch, kv_heads, head_dim]``.

    With slot_mapping None, each table grows by one position (allocating a
    block when it crosses a boundary) and the slots are built here; pass a
    prebuilt device slot_mapping (tables may then be None) to keep the step
    free of host work, e.g. inside a CUDA graph. Returns the slot tensor used.
    """
    if slot_mapping is None:
        if tables is None:
            raise ValueError("append_decode needs tables or a slot_mapping")
        slots = decode_slot_mapping(tables, cache.allocator)
        if _ops.host_index_ok(len(slots), key, cache.keys) and key.dtype == value.dtype:
            slot_mapping = slots  # few sequences: slots go to the kernel by value
        else:
            slot_mapping = _to_device_i64(slots, cache.keys.device)
    write_paged_kv_batch(cache, key, value, slot_mapping, stream=stream)
    return slot_mapping


# ---------------------------------------------------------------------------
# run family
# ---------------------------------------------------------------------------


def split_runs(runs: np.ndarray, max_rows: int) -> np.ndarray:
    """Cut runs longer than max_rows rows into consecutive pieces."""
    runs = np.asarray(runs, dtype=np.int64).reshape(-1, 5)
    if runs.shape[0] == 0 or runs[:, 4].max(initial=0) <= max_rows:
        return runs.astype(np.int32)
    pieces = np.maximum(1, -(-runs[:, 4] // max_rows))
    rep = np.repeat(runs, pieces, axis=0)
    k = np.arange(rep.shape[0]) - np.repeat(np.cumsum(pieces) - pieces, pieces)
    rep[:, 1] += k * max_rows
    rep[:, 3] += k * max_rows
    rep[:, 4] = np.minimum(max_rows, rep[:, 4] - k * max_rows)
    return rep.astype(np.int32)


def handoff_runs(
    tables: Sequence[SequenceBlockTable], seq_lens: Sequence[int], batch_rows: Sequence[int] | None = None
) -> np.ndarray:
    """Runs moving positions [0, n_b) of contiguous batch row b into table b's blocks."""
    lens = np.asarray(seq_lens, dtype=np.int64)
    rows = np.arange(len(tables), dtype=np.int64) if batch_rows is None else np.asarray(batch_rows, np.int64)
    if len(tables) == 0:
        return np.zeros((0, 5), dtype=np.int32)
    bs = tables[0].block_size
    if any(t.block_size != bs for t in tables):
        raise ValueError("all block tables must share one block_size")
    nblk = -(-lens // bs)
    total = int(nblk.sum())
    b_idx = np.repeat(np.arange(len(tables)), nblk)
    j = np.arange(total) - np.repeat(np.cumsum(nblk) - nblk, nblk)
    dst = np.concatenate(
        [np.asarray(t.block_ids[: int(n)], dtype=np.int64) for t, n in zip(tables, nblk)]
    ) if total else np.zeros(0, np.int64)
    runs = np.empty((total, 5), dtype=np.int64)
    runs[:, 0] = rows[b_idx]
    runs[:, 1] = j * bs
    runs[:, 2] = dst
    runs[:, 3] = 0
    runs[:, 4] = np.minimum(bs, lens[b_idx] - j * bs)
    return runs.astype(np.int32)


def copy_runs_between(
    src_k: Tensor,
    src_v: Tensor,
    src_layout: str,
    dst_k: Tensor,
    dst_v: Tensor,
    dst_layout: str,
    runs: Tensor,
    max_rows: int,
    flags: int = _lib.COPY_AUTO,
    stream: torch.cuda.Stream | None = None,
) -> None:
    """copy_runs between two all-layer caches; layout is "paged" or "contiguous".

    paged:      [layers, blocks, heads, block_size, dim] (major = block)
    contiguous: [layers, batch, heads, max_seq, dim]     (major = batch row)
    Both have (layer, major, head, row, dim) order, so strides map the same way.
    """
    for name in (src_layout, dst_layout):
        if name not in ("paged", "contiguous"):
            raise ValueError(f"unknown layout {name!r}")
    num_layers, _, num_heads, _, head_dim = src_k.shape
    if dst_k.shape[0] != num_layers or (dst_k.shape[2], dst_k.shape[4]) != (num_heads, head_dim):
        raise ValueError("source and destination caches have different layer/head/dim shapes")
    st = lambda t: (t.stride(0), t.stride(1), t.stride(3), t.stride(2))  # noqa: E731
    for sk, sv, dk, dv in _kv_pairs(src_k, src_v, dst_k, dst_v):
        _ops.copy_runs(
            src_k=sk, src_v=sv, src_strides=st(sk), src_majors=sk.shape[1], src_rows_per_major=sk.shape[3],
            dst_k=dk, dst_v=dv, dst_strides=st(dk), dst_majors=dk.shape[1], dst_rows_per_major=dk.shape[3],
            runs=runs, max_rows=max_rows, n_layers=num_layers, n_heads=num_heads, head_dim=head_dim,
            flags=flags, stream=stream,
        )


def _run_max_rows(cache_keys: Tensor, rows: int) -> int:
    return _ops.max_rows_for(cache_keys.shape[4], cache_keys.element_size(), cap_rows=rows)


def handoff_contiguous_to_paged(
    src: KVCache,
    dst: PagedKVCache,
    tables: Sequence[SequenceBlockTable],
    seq_lens: Sequence[int],
    batch_rows: Sequence[int] | None = None,
    flags: int = _lib.COPY_AUTO,
    stream: torch.cuda.Stream | None = None,
) -> Tensor:
    """Move each finished prefill (batch row b, positions [0, n_b)) into table b's blocks.

    Grows each table to n_b positions (allocating blocks in table order),
    then copies every layer, K and V, in one launch: a full block is one
    2 KiB run per (layer, head) on both sides at the augur shape. Equal, byte
    for byte, to augur's write_paged_kv(dst, l, table_b, arange(n_b),
    src.keys[l, b:b+1, :, :n_b], ...) for every layer. Returns the device
    runs tensor (reusable for a repeated identical handoff).
    """
    _ops.require_cuda("handoff_contiguous_to_paged", src.keys, src.values, dst.keys, dst.values)
    if len(tables) != len(seq_lens):
        raise ValueError("tables and seq_lens must have the same length")
    for table, n in zip(tables, seq_lens):
        if n < 0 or n > src.max_seq_len:
            raise ValueError("seq_len outside the contiguous cache capacity")
        if table.block_size != dst.block_size:
            raise ValueError("block table block_size must equal the cache block size")
        if n > 0:
            table.ensure_position(int(n) - 1, dst.allocator)
    max_rows = _run_max_rows(dst.keys, dst.block_size)
    runs = split_runs(handoff_runs(tables, seq_lens, batch_rows), max_rows)
    runs_t = _to_device_runs(runs, dst.keys.device)
    copy_runs_between(src.keys, src.values, "contiguous", dst.keys, dst.values, "paged", runs_t,
                      max_rows, flags=flags, stream=stream)
    return runs_t


def copy_blocks(
    cache: PagedKVCache,
    src_blocks: Sequence[int],
    dst_blocks: Sequence[int],
    n_rows: Sequence[int] | int | None = None,
    flags: int = _lib.COPY_AUTO,
    stream: torch.cuda.Stream | None = None,
) -> None:
    """Copy rows [0, n) of block src -> block dst, every layer, K and V, in one launch."""
    _ops.require_cuda("copy_blocks", cache.keys, cache.values)
    if len(src_blocks) != len(dst_blocks):
        raise ValueError("src_blocks and dst_blocks must have the same length")
    bs = cache.block_size
    n = len(src_blocks)
    if n == 0:
        return
    rows = np.full(n, bs, np.int64) if n_rows is None else np.broadcast_to(np.asarray(n_rows, np.int64), (n,))
    runs = np.zeros((n, 5), dtype=np.int64)
    runs[:, 0] = np.asarray(src_blocks, np.int64)
    runs[:, 2] = np.asarray(dst_blocks, np.int64)
    runs[:, 4] = rows
    # the longest run bounds the copy's rows (short copy-on-write runs let the
    # kernel give each warp several planes)
    max_rows = min(_run_max_rows(cache.keys, bs), max(1, int(rows.max())))
    runs_t = _to_device_runs(split_runs(runs, max_rows), cache.keys.device)
    copy_runs_between(cache.keys, cache.values, "paged", cache.keys, cache.values, "paged", runs_t,
                      max_rows, flags=flags, stream=stream)


def fork_prefix(cache: PagedKVCache, table: SequenceBlockTable, n_forks: int) -> list[SequenceBlockTable]:
    """``n_forks`` tables sharing every block of ``table`` (refcount++); no data moves."""
    if n_forks < 0:
        raise ValueError("n_forks must be non-negative")
    return [table.fork(cache.allocator) for _ in range(n_forks)]


def cow_partial_blocks(
    cache: PagedKVCache,
    tables: Sequence[SequenceBlockTable],
    stream: torch.cuda.Stream | None = None,
) -> int:
    """Copy-on-write the shared, partially filled last block of each table before it is appended to.

    For every table whose seq_len ends inside a block held by more than one
    table, allocate a private block, copy the block's written rows (all
    layers, K and V) and swap it into the table. One launch for all tables.
    Returns the number of blocks copied.
    """
    alloc = cache.allocator
    src, dst, rows = [], [], []
    for table in tables:
        r = table.seq_len % table.block_size
        if r == 0 or not table.block_ids:
            continue
        j = (table.seq_len - 1) // table.block_size
        old = table.block_ids[j]
        if alloc.refcount(old) <= 1:
            continue
        new = alloc.allocate()
        table.block_ids[j] = new
        alloc.free(old)  # drops this table's hold on the shared block
        src.append(old)
        dst.append(new)
        rows.append(r)
    if src:
        copy_blocks(cache, src, dst, rows, stream=stream)
    return len(src)


def read_paged_kv_batch(
    cache: PagedKVCache,
    tables: Sequence[SequenceBlockTable],
    seq_lens: Sequence[int] | None = None,
    out: tuple[Tensor, Tensor] | None = None,
    stream: torch.cuda.Stream | None = None,
) -> tuple[Tensor, Tensor]:
    """Gather positions [0, n_b) of every table, all layers, into ``[layers, batch, heads, max_n, dim]``.

    Rows past a sequence's length are left as they were in ``out`` (fresh,
    uninitialised memory when out is None).
    """
    _ops.require_cuda("read_paged_kv_batch", cache.keys, cache.values)
    lens = [t.seq_len for t in tables] if seq_lens is None else [int(n) for n in seq_lens]
    for t, n in zip(tables, lens):
        if n < 0 or math.ceil(n / t.block_size) > len(t.block_ids):
            raise ValueError("position exceeds block table capacity")
        if t.block_size != cache.block_size:
            raise ValueError("block table block_size must equal the cache block size")
    L, _, H, bs, D = cache.keys.shape
    width = max(lens, default=0)
    if out is None:
        shape = (L, len(tables), H, width, D)
        out = (torch.empty(shape, device=cache.keys.device, dtype=cache.keys.dtype),
               torch.empty(shape, device=cache.keys.device, dtype=cache.keys.dtype))
    ok, ov = out
    if ok.shape[:3] != (L, len(tables), H) or ok.shape[3] < width or ok.shape[4] != D:
        raise ValueError("out tensors have the wrong shape")
    # gather runs = handoff runs with source and destination swapped
    runs = handoff_runs(tables, lens)
    runs = runs[:, [2, 3, 0, 1, 4]]
    max_rows = _run_max_rows(cache.keys, bs)
    runs_t = _to_device_runs(split_runs(runs, max_rows), cache.keys.device)
    if runs_t.shape[0]:
        copy_runs_between(cache.keys, cache.values, "paged", ok, ov, "contiguous", runs_t, max_rows,
                          stream=stream)
    return ok, ov
