"""KV blocks offloaded to pinned host memory and restored (bit-exact round trips).

The host copy of a block is the pool's block, all layers, block-major (the
oracle is the pool itself gathered on the CPU); restoring into other blocks
reproduces every valid row and leaves the rest of the destination untouched.
Both paths run: direct (the device reads and writes pinned memory in place)
and staged (SM gather / scatter through HBM chunks plus copy-engine
transfers), the staged one with chunks small enough to cycle the two buffers.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import augur_b200 as ab
from augur_b200 import _lib, _ops, batched
from augur_b200 import offload
from augur_b200.offload import (offload_blocks, offload_sequence, restore_blocks, restore_sequence)
from tests.conftest import assert_bits_equal, poison_

pytestmark = pytest.mark.gpu


def _pool(cuda, NB, dtype, L=3, H=2, bs=16, D=64, fill=True, seed=0):
    g = torch.Generator(device=cuda).manual_seed(seed)
    if fill:
        k = torch.randn(L, NB, H, bs, D, generator=g, device=cuda).to(dtype)
        v = torch.randn(L, NB, H, bs, D, generator=g, device=cuda).to(dtype)
    else:
        k = poison_(torch.empty(L, NB, H, bs, D, dtype=dtype, device=cuda))
        v = poison_(torch.empty(L, NB, H, bs, D, dtype=dtype, device=cuda))
    return ab.PagedKVCache(keys=k, values=v, block_size=bs, allocator=ab.BlockAllocator(NB))


@pytest.fixture
def small_chunks(monkeypatch):
    """Staging chunks of two blocks (at 3 layers x 2 heads x 16 x 64), so a transfer cycles both buffers."""
    monkeypatch.setattr(offload, "STAGE_BYTES", 2 * 3 * 2 * 16 * 64 * 4)


@pytest.mark.parametrize("path", ["direct", "staged"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_offload_then_restore_elsewhere(cuda, small_chunks, dtype, path):
    src = _pool(cuda, 40, dtype)
    ids = [7, 3, 31, 0, 12]
    rows = [16, 16, 5, 16, 1]
    host = offload_blocks(src, ids, rows, path=path)
    host.wait()
    assert host.keys.is_pinned() and host.n_tokens == sum(rows)
    assert host.keys.shape == (5, 3, 2, 16, 64)
    for i, (b, r) in enumerate(zip(ids, rows)):
        assert_bits_equal(host.keys[i, :, :, :r], src.keys[:, b, :, :r].cpu(), f"host keys block {b}")
        assert_bits_equal(host.values[i, :, :, :r], src.values[:, b, :, :r].cpu(), f"host values block {b}")
    dst = _pool(cuda, 40, dtype, fill=False)
    dst_ids = [39, 1, 2, 20, 8]
    restore_blocks(dst, host, dst_ids, path=path)
    torch.cuda.synchronize(cuda)
    for b, d, r in zip(ids, dst_ids, rows):
        assert_bits_equal(dst.keys[:, d, :, :r], src.keys[:, b, :, :r], f"restored keys {b}->{d}")
        assert_bits_equal(dst.values[:, d, :, :r], src.values[:, b, :, :r], f"restored values {b}->{d}")
        assert bool((dst.keys[:, d, :, r:].contiguous().view(torch.uint8) == 0xFF).all())
    untouched = [b for b in range(40) if b not in dst_ids]
    assert bool((dst.keys[:, untouched].contiguous().view(torch.uint8) == 0xFF).all())
    assert _ops.read_status(cuda) == _lib.OK


@pytest.mark.parametrize("path", ["direct", "staged"])
def test_sequence_round_trip_through_the_allocator(cuda, small_chunks, path):
    """A sequence written by the batched scatter, offloaded, freed, restored into newly
    allocated blocks: the logical gather is unchanged."""
    pool = _pool(cuda, 64, torch.bfloat16, fill=False)
    lens = [37, 16, 100]
    tables = [ab.SequenceBlockTable.empty(16) for _ in lens]
    sm = batched.prefill_slot_mapping(tables, lens, pool.allocator)
    g = torch.Generator(device=cuda).manual_seed(3)
    T = sum(lens)
    k = torch.randn(3, T, 2, 64, generator=g, device=cuda).to(torch.bfloat16)
    v = torch.randn(3, T, 2, 64, generator=g, device=cuda).to(torch.bfloat16)
    flat = np.concatenate([sm[b, :n] for b, n in enumerate(lens)])
    batched.write_paged_kv_batch(pool, k, v, torch.from_numpy(flat).to(cuda))
    before = batched.read_paged_kv_batch(pool, tables, seq_lens=lens)
    hosts = [offload_sequence(pool, t, path=path) for t in tables]
    for t in tables:
        t.free(pool.allocator)
    pool.keys.view(torch.uint8).fill_(0xFF)  # the freed blocks are reused and overwritten
    pool.values.view(torch.uint8).fill_(0xFF)
    new_tables = [restore_sequence(pool, h, path=path) for h in hosts]
    assert [t.seq_len for t in new_tables] == lens
    after = batched.read_paged_kv_batch(pool, new_tables, seq_lens=lens)
    for b, n in enumerate(lens):
        assert_bits_equal(after[0][:, b, :, :n], before[0][:, b, :, :n], f"keys seq {b}")
        assert_bits_equal(after[1][:, b, :, :n], before[1][:, b, :, :n], f"values seq {b}")
    assert _ops.read_status(cuda) == _lib.OK


def test_host_buffers_must_be_pinned(cuda):
    pool = _pool(cuda, 4, torch.bfloat16)
    out = (torch.empty(2, 3, 2, 16, 64, dtype=torch.bfloat16), torch.empty(2, 3, 2, 16, 64, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="pinned"):
        offload_blocks(pool, [0, 1], out=out)
    with pytest.raises(ValueError, match="block id outside"):
        offload_blocks(pool, [4])


@pytest.mark.parametrize("path", ["direct", "staged"])
def test_blocks_cut_into_several_runs(cuda, monkeypatch, path):
    """float32, head_dim 128, block 64: a block is several copy runs; staged chunks of 3 blocks."""
    monkeypatch.setattr(offload, "STAGE_BYTES", 3 * 2 * 2 * 64 * 128 * 4)
    src = _pool(cuda, 12, torch.float32, L=2, H=2, bs=64, D=128)
    ids, rows = [11, 0, 5, 6, 2, 9, 3], [64, 63, 1, 64, 17, 64, 40]
    host = offload_blocks(src, ids, rows, path=path)
    dst = _pool(cuda, 12, torch.float32, L=2, H=2, bs=64, D=128, fill=False)
    dst_ids = [0, 1, 2, 3, 4, 5, 6]
    restore_blocks(dst, host, dst_ids, path=path)
    torch.cuda.synchronize(cuda)
    for b, d, r in zip(ids, dst_ids, rows):
        assert_bits_equal(dst.keys[:, d, :, :r], src.keys[:, b, :, :r], f"keys {b}->{d}")
        assert_bits_equal(dst.values[:, d, :, :r], src.values[:, b, :, :r], f"values {b}->{d}")
        assert bool((dst.values[:, d, :, r:].contiguous().view(torch.uint8) == 0xFF).all())
