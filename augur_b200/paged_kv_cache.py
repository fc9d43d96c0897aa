"""Paged KV cache — drop-in for augur/paged_kv_cache.py.

Host bookkeeping (allocator free-list order, block tables, the prefix-block
hash index) behaves exactly like augur/paged_kv_cache.py:10-139; the data
movement of write_paged_kv and read_paged_kv runs as one sm_100a kernel
launch per call instead of the reference's per-token Python loops
(paged_kv_cache.py:188-192, :217-220).

Additions that the reference does not have, used by fork / copy-on-write:
BlockAllocator keeps a reference count for shared blocks (incref/refcount),
and SequenceBlockTable.fork shares a table's blocks with a new table. For a
block nobody shares, allocate/free order is the reference's.
"""

from __future__ import annotations

import math
from collections import deque
from dataclasses import dataclass

import numpy as np
import torch
from torch import Tensor

from . import _ops
from ._ops import keep_last
from .config import QwenConfig


class BlockAllocator:
    """Free list of block ids: allocate takes the front, free puts back at the front.

    Same order as augur/paged_kv_cache.py:10-22 (a deque instead of a list, so
    both ends are O(1)). Blocks shared through incref() return to the free list
    only when their last holder frees them.
    """

    def __init__(self, num_blocks: int) -> None:
        if num_blocks <= 0:
            raise ValueError("num_blocks must be positive")
        self.num_blocks = num_blocks
        self._free_blocks: deque[int] = deque(range(num_blocks))
        self._shared: dict[int, int] = {}  # block id -> holders, only while > 1

    def allocate(self) -> int:
        if not self._free_blocks:
            raise RuntimeError("no free KV cache blocks")
        return self._free_blocks.popleft()

    def allocate_many(self, count: int) -> list[int]:
        """``count`` blocks in allocate() order; all or nothing."""
        if count < 0:
            raise ValueError("count must be non-negative")
        if count > len(self._free_blocks):
            raise RuntimeError("no free KV cache blocks")
        return [self._free_blocks.popleft() for _ in range(count)]

    def free(self, block_id: int) -> None:
        holders = self._shared.get(block_id)
        if holders is not None:
            if holders > 2:
                self._shared[block_id] = holders - 1
            else:
                del self._shared[block_id]
            return
        self._free_blocks.appendleft(block_id)

    def incref(self, block_id: int) -> None:
        """Record one more holder of an allocated block (a fork)."""
        self._shared[block_id] = self._shared.get(block_id, 1) + 1

    def refcount(self, block_id: int) -> int:
        """Holders of an allocated block: 1 unless it was shared with incref()."""
        return self._shared.get(block_id, 1)

    @property
    def num_free(self) -> int:
        return len(self._free_blocks)


@dataclass
class PagedKVCache:
    """Block pool ``[layers, num_blocks, kv_heads, block_size, head_dim]`` (paged_kv_cache.py:25-30)."""

    keys: Tensor
    values: Tensor
    block_size: int
    allocator: BlockAllocator


@dataclass
class PagedKVCacheState:
    cache: PagedKVCache
    block_table: "SequenceBlockTable"


@dataclass
class PagedPrefixCacheMatch:
    block_ids: list[int]
    matched_tokens: int


class PagedPrefixCache:
    """Hash-chained index of full prefix blocks (paged_kv_cache.py:45-85).

    A block's key is (parent hash, its tokens); its hash is Python's hash of
    that pair, which is deterministic for tuples of ints and None, so chains
    built here and in augur agree.
    """

    def __init__(self) -> None:
        self._blocks: dict[tuple[int | None, tuple[int, ...]], tuple[int, int]] = {}

    def add_block(self, parent_hash: int | None, block_tokens: list[int], block_id: int) -> int:
        if not block_tokens:
            raise ValueError("block_tokens must not be empty")
        block_key = tuple(block_tokens)
        block_hash = self._hash_block(parent_hash, block_key)
        self._blocks[(parent_hash, block_key)] = (block_hash, block_id)
        return block_hash

    def match_prefix(self, token_ids: list[int], block_size: int) -> PagedPrefixCacheMatch:
        if block_size <= 0:
            raise ValueError("block_size must be positive")
        parent_hash: int | None = None
        block_ids: list[int] = []
        for block_idx in range(len(token_ids) // block_size):
            start = block_idx * block_size
            entry = self._blocks.get((parent_hash, tuple(token_ids[start : start + block_size])))
            if entry is None:
                break
            parent_hash, block_id = entry
            block_ids.append(block_id)
        return PagedPrefixCacheMatch(block_ids=block_ids, matched_tokens=len(block_ids) * block_size)

    def lookup(self, parent_hash: int | None, block_tokens: list[int]) -> tuple[int, int] | None:
        """(hash, block id) of a registered block, or None (an addition to augur's API)."""
        return self._blocks.get((parent_hash, tuple(block_tokens)))

    def remove_block(self, parent_hash: int | None, block_tokens: list[int]) -> int | None:
        """Unregister a block and return its id, or None (an addition to augur's API).
        Blocks chained after it can no longer be matched."""
        entry = self._blocks.pop((parent_hash, tuple(block_tokens)), None)
        return None if entry is None else entry[1]

    def _hash_block(self, parent_hash: int | None, block_tokens: tuple[int, ...]) -> int:
        return hash((parent_hash, block_tokens))


@dataclass
class SequenceBlockTable:
    """Logical->physical block list of one sequence (paged_kv_cache.py:88-139)."""

    block_ids: list[int]
    block_size: int
    seq_len: int = 0

    @classmethod
    def empty(cls, block_size: int) -> "SequenceBlockTable":
        if block_size <= 0:
            raise ValueError("block_size must be positive")
        return cls(block_ids=[], block_size=block_size)

    @classmethod
    def allocate(
        cls, allocator: BlockAllocator, max_seq_len: int, block_size: int
    ) -> "SequenceBlockTable":
        if max_seq_len <= 0:
            raise ValueError("max_seq_len must be positive")
        if block_size <= 0:
            raise ValueError("block_size must be positive")
        num_required_blocks = math.ceil(max_seq_len / block_size)
        return cls(
            block_ids=[allocator.allocate() for _ in range(num_required_blocks)],
            block_size=block_size,
            seq_len=max_seq_len,
        )

    def ensure_position(self, position: int, allocator: BlockAllocator) -> None:
        if position < 0:
            raise ValueError("position must be non-negative")
        required_blocks = position // self.block_size + 1
        while len(self.block_ids) < required_blocks:
            self.block_ids.append(allocator.allocate())
        self.seq_len = max(self.seq_len, position + 1)

    def free(self, allocator: BlockAllocator) -> None:
        for block_id in reversed(self.block_ids):
            allocator.free(block_id)
        self.block_ids.clear()
        self.seq_len = 0

    def position_to_block_offset(self, position: int) -> tuple[int, int]:
        if position < 0:
            raise ValueError("position must be non-negative")
        logical_block = position // self.block_size
        if logical_block >= len(self.block_ids):
            raise ValueError("position exceeds block table capacity")
        return self.block_ids[logical_block], position % self.block_size

    def fork(self, allocator: BlockAllocator) -> "SequenceBlockTable":
        """A new table holding the same blocks (each gains a holder); no data moves."""
        for block_id in self.block_ids:
            allocator.incref(block_id)
        return SequenceBlockTable(
            block_ids=list(self.block_ids), block_size=self.block_size, seq_len=self.seq_len
        )


def new_paged_kv_cache(
    cfg: QwenConfig,
    num_blocks: int,
    block_size: int,
    device: torch.device,
    dtype: torch.dtype,
) -> PagedKVCache:
    """Allocate an uninitialised block pool and its allocator (paged_kv_cache.py:142-164)."""
    if block_size <= 0:
        raise ValueError("block_size must be positive")
    shape = (cfg.num_hidden_layers, num_blocks, cfg.num_key_value_heads, block_size, cfg.head_dim)
    return PagedKVCache(
        keys=torch.empty(shape, device=device, dtype=dtype),
        values=torch.empty(shape, device=device, dtype=dtype),
        block_size=block_size,
        allocator=BlockAllocator(num_blocks),
    )


# ---------------------------------------------------------------------------
# host helpers shared with the batched entry points
# ---------------------------------------------------------------------------


def ensure_positions(
    block_table: SequenceBlockTable, positions: np.ndarray, allocator: BlockAllocator
) -> tuple[int, Exception | None]:
    """Apply the reference's per-token ensure_position to ``positions`` in order.

    Returns (n, err): the first n tokens are the ones augur's loop
    (paged_kv_cache.py:188-192) writes before it raises err (None if all are
    written). Allocation order and the table's final block_ids / seq_len match
    calling ensure_position token by token, because a token only ever extends
    the table to cover the running maximum position.
    """
    n = int(positions.shape[0])
    if n == 0:
        return 0, None
    neg = np.flatnonzero(positions < 0)
    limit = int(neg[0]) if neg.size else n
    err: Exception | None = None
    if limit:
        runmax = np.maximum.accumulate(positions[:limit])
        try:
            block_table.ensure_position(int(runmax[-1]), allocator)
        except RuntimeError as exc:  # pool exhausted part-way
            covered = len(block_table.block_ids)
            need = runmax // block_table.block_size + 1
            limit = int(np.searchsorted(need, covered, side="right"))
            if limit:
                block_table.seq_len = max(block_table.seq_len, int(runmax[limit - 1]) + 1)
            err = exc
    if err is None and limit < n:
        err = ValueError("position must be non-negative")
    return limit, err


def slots_for_positions(block_table: SequenceBlockTable, positions: np.ndarray) -> np.ndarray:
    """slot = block_ids[p // block_size] * block_size + p % block_size, as int64."""
    bs = block_table.block_size
    table = np.asarray(block_table.block_ids, dtype=np.int64)
    return table[positions // bs] * bs + positions % bs


def pool_strides(pool_layer_or_all: Tensor, per_layer: bool) -> tuple[int, int, int, int]:
    """(layer, major=block, row=offset, head) element strides of a pool tensor or layer view."""
    t = pool_layer_or_all
    if per_layer:
        return (0, t.stride(0), t.stride(2), t.stride(1))
    return (t.stride(0), t.stride(1), t.stride(3), t.stride(2))


def _device_runs(block_table: SequenceBlockTable, key: tuple, build, device) -> Tensor:
    """Device copy of a table-derived runs array, cached on the table object."""
    cached = getattr(block_table, "_augur_runs", None)
    if cached is not None and cached[0] == key:
        return cached[1]
    runs = torch.from_numpy(build()).to(device=device)
    try:
        block_table._augur_runs = (key, runs)  # type: ignore[attr-defined]
    except AttributeError:
        pass
    return runs


def gather_runs(block_ids, block_size: int, seq_len: int, max_rows: int) -> np.ndarray:
    """Runs copying logical positions [0, seq_len) of a table into a dense [seq_len] row range."""
    out = []
    for j in range(math.ceil(seq_len / block_size)):
        base = j * block_size
        n = min(block_size, seq_len - base)
        for r0 in range(0, n, max_rows):
            out.append((block_ids[j], r0, 0, base + r0, min(max_rows, n - r0)))
    return np.asarray(out, dtype=np.int32).reshape(-1, 5)


# ---------------------------------------------------------------------------
# data movement (drop-in)
# ---------------------------------------------------------------------------


def write_paged_kv(
    cache: PagedKVCache,
    layer_idx: int,
    block_table: SequenceBlockTable,
    position_ids: Tensor,
    key: Tensor,
    value: Tensor,
) -> None:
    """Write ``key``/``value`` ``[1, kv_heads, seq, head_dim]`` at ``position_ids`` through the table.

    Same checks, messages, lazy block allocation and partial-write-on-error
    behaviour as augur's write_paged_kv (paged_kv_cache.py:167-192); the data
    moves in one augur_kv_scatter launch. Reading position_ids is a host sync
    when it lives on the GPU, as in the reference (.tolist()). A position given
    twice keeps the later token's K/V, as the reference's loop does.
    """
    if key.shape != value.shape:
        raise ValueError("key and value must have the same shape")

    batch, num_heads, seq, head_dim = key.shape
    if batch != 1:
        raise ValueError("paged KV cache currently supports batch size 1")
    if position_ids.shape != (batch, seq):
        raise ValueError("position_ids must have shape [batch, seq]")
    if not 0 <= layer_idx < cache.keys.shape[0]:
        raise ValueError("layer_idx is outside the cache layer range")
    if (num_heads, head_dim) != (cache.keys.shape[2], cache.keys.shape[4]):
        raise ValueError("key/value shape does not match cache shape")
    _ops.require_cuda("write_paged_kv", cache.keys, cache.values)

    positions = np.asarray(position_ids[0].tolist(), dtype=np.int64)
    n_ok, err = ensure_positions(block_table, positions, cache.allocator)
    if n_ok:
        if block_table.block_size > cache.keys.shape[3]:
            raise IndexError("block table block_size exceeds the cache block size")
        slots = keep_last(slots_for_positions(block_table, positions[:n_ok]))
        if not (_ops.host_index_ok(n_ok, key, cache.keys) and key.dtype == value.dtype):
            slots = torch.from_numpy(slots).to(device=cache.keys.device)
        scatter_slots_one_layer(cache, layer_idx, key[0], value[0], slots, block_table.block_size)
    if err is not None:
        raise err


def scatter_slots_one_layer(
    cache: PagedKVCache,
    layer_idx: int,
    key: Tensor,
    value: Tensor,
    slots: Tensor | np.ndarray,
    block_size: int | None = None,
) -> None:
    """key/value ``[kv_heads, seq, head_dim]``: token t goes to slot slots[t] of one layer.

    Only the first len(slots) tokens move. A slot < 0 skips its token.
    `slots` is an int64 CUDA tensor, or a host int64 array of at most 32
    slots (passed by value).
    """
    device = cache.keys.device
    # torch's slice assignment in the reference accepts a source on another
    # device; bring it over first (a transfer, not a fallback).
    if key.device != device:
        key = key.to(device)
    if value.device != device:
        value = value.to(device)
    if key.stride(-1) != 1:
        key = key.contiguous()
    if value.stride(-1) != 1:
        value = value.contiguous()
    kc, vc = cache.keys[layer_idx], cache.values[layer_idx]
    bs = block_size if block_size is not None else cache.block_size
    n_tokens = int(slots.shape[0])
    num_heads, _, head_dim = key.shape
    common = dict(
        tokens_per_row=max(1, n_tokens),
        rows_per_major=bs,
        num_majors=kc.shape[0],
        index=slots,
        index_strides=(0, 1 if isinstance(slots, np.ndarray) else slots.stride(0)),
        index_row_base=0,
        n_tokens=n_tokens,
        n_layers=1,
        n_heads=num_heads,
        head_dim=head_dim,
    )
    # Slot s lives at block s // bs, row s % bs of the pool, bs being the
    # table's block size (the reference indexes the pool the same way).
    if bs > kc.shape[2]:
        raise IndexError("block table block_size exceeds the cache block size")
    k_strides = (0, 0, key.stride(1), key.stride(0))
    v_strides = (0, 0, value.stride(1), value.stride(0))
    if key.dtype == value.dtype and kc.stride() == vc.stride():
        _ops.scatter(
            src_k=key, src_v=value, src_k_strides=k_strides, src_v_strides=v_strides,
            dst_k=kc, dst_v=vc, dst_strides=pool_strides(kc, True), **common,
        )
    else:
        for src, strides, dst in ((key, k_strides, kc), (value, v_strides, vc)):
            _ops.scatter(
                src_k=src, src_v=None, src_k_strides=strides, src_v_strides=None,
                dst_k=dst, dst_v=None, dst_strides=pool_strides(dst, True), **common,
            )


def read_paged_kv(
    cache: PagedKVCache,
    layer_idx: int,
    block_table: SequenceBlockTable,
    seq_len: int | None = None,
) -> tuple[Tensor, Tensor]:
    """Gather positions [0, seq_len) of one layer into fresh ``[1, kv_heads, seq_len, head_dim]``.

    Same checks and messages as augur's read_paged_kv (paged_kv_cache.py:195-221);
    the copy is one augur_kv_copy_runs launch over whole blocks.
    """
    if seq_len is None:
        seq_len = block_table.seq_len
    if seq_len <= 0:
        raise ValueError("seq_len must be positive")
    if not 0 <= layer_idx < cache.keys.shape[0]:
        raise ValueError("layer_idx is outside the cache layer range")
    _ops.require_cuda("read_paged_kv", cache.keys, cache.values)
    bs = block_table.block_size
    if math.ceil(seq_len / bs) > len(block_table.block_ids):
        raise ValueError("position exceeds block table capacity")
    if bs > cache.keys.shape[3]:
        raise IndexError("block table block_size exceeds the cache block size")

    kc, vc = cache.keys[layer_idx], cache.values[layer_idx]
    num_heads, head_dim = kc.shape[1], kc.shape[3]
    key = torch.empty(1, num_heads, seq_len, head_dim, device=kc.device, dtype=kc.dtype)
    value = torch.empty_like(key)
    max_rows = _ops.max_rows_for(head_dim, kc.element_size(), cap_rows=bs)
    n_blocks = math.ceil(seq_len / bs)
    ids = block_table.block_ids[:n_blocks]
    runs = _device_runs(
        block_table,
        ("gather", kc.device, tuple(ids), bs, seq_len, max_rows),
        lambda: gather_runs(ids, bs, seq_len, max_rows),
        kc.device,
    )
    dst_strides = (0, 0, key.stride(2), key.stride(1))
    if kc.stride() == vc.stride():
        pairs = [((kc, vc), (key, value))]
    else:
        pairs = [((kc, None), (key, None)), ((vc, None), (value, None))]
    for (sk, sv), (dk, dv) in pairs:
        _ops.copy_runs(
            src_k=sk, src_v=sv, src_strides=pool_strides(sk, True),
            src_majors=sk.shape[0], src_rows_per_major=sk.shape[2],
            dst_k=dk, dst_v=dv, dst_strides=dst_strides,
            dst_majors=1, dst_rows_per_major=seq_len,
            runs=runs, max_rows=max_rows, n_layers=1, n_heads=num_heads, head_dim=head_dim,
        )
    return key, value
