"""PagedSequences host bookkeeping: prefix matching, block sharing, forks, release and
eviction (no device work; the data side is tests/test_gpu_sequences.py)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import augur_b200 as ab
from augur_b200.sequences import PagedSequences


def _pool(num_blocks: int = 32, bs: int = 4) -> ab.PagedKVCache:
    return ab.PagedKVCache(keys=torch.empty(1, num_blocks, 1, bs, 2), values=torch.empty(1, num_blocks, 1, bs, 2),
                           block_size=bs, allocator=ab.BlockAllocator(num_blocks))


def test_prefix_blocks_are_shared_and_returned_when_nobody_holds_them():
    pool = _pool()
    alloc = pool.allocator
    seqs = PagedSequences(pool)
    a = seqs.admit(range(10))  # blocks of tokens 0-3, 4-7, 8-9
    assert a.cached_tokens == 0
    np.testing.assert_array_equal(a.slots, np.arange(10))  # blocks 0, 1, 2 in allocate() order
    assert seqs.publish_prefix(a.seq_id) == 2  # the two full blocks
    ta = seqs.tables[a.seq_id]
    assert [alloc.refcount(x) for x in ta.block_ids] == [2, 2, 1]

    b = seqs.admit(list(range(8)) + [100, 101, 102])
    tb = seqs.tables[b.seq_id]
    assert b.cached_tokens == 8 and tb.block_ids[:2] == ta.block_ids[:2]
    np.testing.assert_array_equal(b.slots, tb.block_ids[2] * 4 + np.arange(3))
    # a prompt made only of cached blocks still prefills its last block
    c = seqs.admit(range(8))
    tc = seqs.tables[c.seq_id]
    assert c.cached_tokens == 4 and tc.block_ids[0] == ta.block_ids[0] and tc.block_ids[1] != ta.block_ids[1]
    assert len(c.slots) == 4
    assert seqs.publish_prefix(b.seq_id) == 0  # its full blocks are already registered
    assert alloc.refcount(ta.block_ids[0]) == 4  # cache, a, b, c

    forks = seqs.fork(b.seq_id, 2)
    assert all(seqs.tables[f].block_ids == tb.block_ids for f in forks)
    assert alloc.refcount(tb.block_ids[2]) == 3

    for sid in [a.seq_id, b.seq_id, c.seq_id, *forks]:
        seqs.release(sid)
    assert alloc.num_free == 32 - 2  # the prefix cache still holds two blocks
    assert seqs.prefix_cache.match_prefix(list(range(12)), 4).matched_tokens == 8
    assert seqs.evict_prefixes() == 2
    assert alloc.num_free == 32
    assert seqs.prefix_cache.match_prefix(list(range(12)), 4).matched_tokens == 0


def test_admission_is_all_or_nothing():
    pool = _pool(num_blocks=4)
    seqs = PagedSequences(pool)
    a = seqs.admit(range(8))
    seqs.publish_prefix(a.seq_id)
    held = [pool.allocator.refcount(x) for x in seqs.tables[a.seq_id].block_ids]
    with pytest.raises(RuntimeError, match="no free KV cache blocks"):
        seqs.admit(list(range(4)) + list(range(50, 62)))  # one shared block + 3 new > 2 free
    assert pool.allocator.num_free == 2
    assert [pool.allocator.refcount(x) for x in seqs.tables[a.seq_id].block_ids] == held
    with pytest.raises(ValueError, match="at least one token"):
        seqs.admit([])


def test_evicting_a_chain_keeps_blocks_in_use():
    pool = _pool()
    seqs = PagedSequences(pool)
    a = seqs.admit(range(13))
    seqs.publish_prefix(a.seq_id)  # 3 full blocks
    b = seqs.admit(range(6))  # shares the first block
    seqs.release(a.seq_id)
    assert seqs.evict_prefixes() == 2  # the second and third; the first is still b's
    assert seqs.prefix_cache.match_prefix(list(range(13)), 4).matched_tokens == 4
    seqs.release(b.seq_id)
    assert seqs.evict_prefixes() == 1
    assert pool.allocator.num_free == 32
