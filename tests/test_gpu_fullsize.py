"""Full-size workloads (the benchmark configurations), checked through properties.

At these sizes the CPU oracle is used on sampled sequences only; the rest is
checked with size-independent properties on the device:
  * scatter then gather returns the source exactly (round trip);
  * every pool row that was not a destination still holds the 0xFF poison
    (nothing written out of place), counted per pool;
  * handoff then gather equals the contiguous source on valid rows;
  * decode appends land at the sequence ends and nowhere else;
  * forked sequences (shared prefix blocks + copy-on-write) read back as
    prefix followed by their own suffix.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import augur_b200 as ab
from augur_b200 import _lib, _ops, batched
from bench import BS, D, H, L, config2_batch, config3_lengths
from tests.conftest import assert_bits_equal, poison_

pytestmark = pytest.mark.gpu


def _poison_count(t: torch.Tensor) -> int:
    return int((t.view(torch.int16) == -1).sum().item())


def _pool(nb, device):
    return ab.PagedKVCache(keys=poison_(torch.empty(L, nb, H, BS, D, dtype=torch.bfloat16, device=device)),
                           values=poison_(torch.empty(L, nb, H, BS, D, dtype=torch.bfloat16, device=device)),
                           block_size=BS, allocator=ab.BlockAllocator(nb))


def test_config2_full_scatter_round_trip(cuda, oracle):
    """8192 tokens x 24 layers into a 65,536-block pool (12.9 GB)."""
    lens, slots, k, v, _ = config2_batch(seed=0)
    pool = _pool(65536, cuda)
    kd, vd, sd = k.to(cuda), v.to(cuda), torch.from_numpy(slots).to(cuda)
    batched.write_paged_kv_batch(pool, kd, vd, sd)
    assert _ops.read_status(cuda) == _lib.OK
    # round trip through the logical tables
    perm_tables, pos0 = [], 0
    for n in lens:
        ids = (slots[pos0 : pos0 + n : BS] // BS).tolist()
        perm_tables.append(ab.SequenceBlockTable(block_ids=ids, block_size=BS, seq_len=int(n)))
        pos0 += int(n)
    gk, gv = batched.read_paged_kv_batch(pool, perm_tables)
    pos0 = 0
    for b, n in enumerate(lens):
        src_k = kd[:, pos0 : pos0 + n].permute(0, 2, 1, 3)  # [L, H, n, D]
        src_v = vd[:, pos0 : pos0 + n].permute(0, 2, 1, 3)
        assert torch.equal(gk[:, b, :, :n].view(torch.int16), src_k.reshape(L, H, n, D).view(torch.int16))
        assert torch.equal(gv[:, b, :, :n].view(torch.int16), src_v.reshape(L, H, n, D).view(torch.int16))
        pos0 += int(n)
    # nothing outside the 8192 destination slots changed
    written = 8192 * L * H * D
    assert _poison_count(pool.keys) == pool.keys.numel() - written
    assert _poison_count(pool.values) == pool.values.numel() - written
    # oracle on three sampled sequences, through their own blocks only
    for b in (0, 31, 63):
        start = int(lens[:b].sum())
        n = int(lens[b])
        ids = perm_tables[b].block_ids
        ek = poison_(torch.empty(L, len(ids), H, BS, D, dtype=torch.bfloat16))
        ev = poison_(torch.empty(L, len(ids), H, BS, D, dtype=torch.bfloat16))
        local = np.arange(n, dtype=np.int64)
        oracle.scatter_slots(k[:, start : start + n].contiguous(), v[:, start : start + n].contiguous(),
                             local, ek, ev, BS)
        got_k = pool.keys[:, ids].cpu()
        got_v = pool.values[:, ids].cpu()
        assert_bits_equal(got_k, ek, f"seq {b} keys")
        assert_bits_equal(got_v, ev, f"seq {b} values")


def test_config3_full_handoff_and_256_appends(cuda):
    """32 prompts of U[512,2048] tokens: handoff (both copy paths) then 256 decode steps."""
    lens = config3_lengths()
    B, Lmax = len(lens), int(lens.max())
    g = torch.Generator(device=cuda).manual_seed(3)
    src = ab.KVCache(keys=torch.randn(L, B, H, Lmax, D, generator=g, device=cuda).to(torch.bfloat16),
                     values=torch.randn(L, B, H, Lmax, D, generator=g, device=cuda).to(torch.bfloat16))
    results = []
    for flags in (_lib.COPY_VECTOR, _lib.COPY_BULK):
        pool = _pool(8192, cuda)
        tables = [ab.SequenceBlockTable.empty(BS) for _ in lens]
        batched.handoff_contiguous_to_paged(src, pool, tables, lens, flags=flags)
        results.append((pool, tables))
    (pa, ta), (pb, tb) = results
    assert [t.block_ids for t in ta] == [t.block_ids for t in tb]
    assert torch.equal(pa.keys.view(torch.int16), pb.keys.view(torch.int16))
    assert torch.equal(pa.values.view(torch.int16), pb.values.view(torch.int16))
    del results, pb, tb
    gk, gv = batched.read_paged_kv_batch(pa, ta)
    for b, n in enumerate(lens):
        assert torch.equal(gk[:, b, :, :n].view(torch.int16), src.keys[:, b, :, :n].view(torch.int16))
        assert torch.equal(gv[:, b, :, :n].view(torch.int16), src.values[:, b, :, :n].view(torch.int16))
    del gk, gv
    # 256 decode appends, one token per sequence per step, all layers
    steps = 256
    nk = torch.randn(steps, L, B, H, D, generator=g, device=cuda).to(torch.bfloat16)
    nv = torch.randn(steps, L, B, H, D, generator=g, device=cuda).to(torch.bfloat16)
    for s in range(steps):
        batched.append_decode(pa, ta, nk[s], nv[s])
    assert [t.seq_len for t in ta] == [int(n) + steps for n in lens]
    gk, gv = batched.read_paged_kv_batch(pa, ta)
    for b, n in enumerate(lens):
        n = int(n)
        assert torch.equal(gk[:, b, :, :n].view(torch.int16), src.keys[:, b, :, :n].view(torch.int16))
        want_k = nk[:, :, b].permute(1, 2, 0, 3)  # [L, H, steps, D]
        want_v = nv[:, :, b].permute(1, 2, 0, 3)
        assert torch.equal(gk[:, b, :, n : n + steps].view(torch.int16), want_k.reshape(L, H, steps, D).view(torch.int16))
        assert torch.equal(gv[:, b, :, n : n + steps].view(torch.int16), want_v.reshape(L, H, steps, D).view(torch.int16))
    written = (int(lens.sum()) + steps * B) * L * H * D
    assert _poison_count(pa.keys) == pa.keys.numel() - written
    assert _ops.read_status(cuda) == _lib.OK


@pytest.mark.parametrize("prefix_len", [1024, 1000])
def test_config4_full_fork_cow_suffix(cuda, prefix_len):
    """One prefix shared by 256 forks; copy-on-write of a partial last block; 128-token suffixes."""
    g = torch.Generator(device=cuda).manual_seed(4)
    pool = _pool(8192, cuda)
    parent = ab.SequenceBlockTable.empty(BS)
    sm = batched.prefill_slot_mapping([parent], [prefix_len], pool.allocator)[0]
    pk = torch.randn(L, prefix_len, H, D, generator=g, device=cuda).to(torch.bfloat16)
    pv = torch.randn(L, prefix_len, H, D, generator=g, device=cuda).to(torch.bfloat16)
    batched.write_paged_kv_batch(pool, pk, pv, torch.from_numpy(sm).to(cuda))
    forks = batched.fork_prefix(pool, parent, 256)
    copied = batched.cow_partial_blocks(pool, forks)
    assert copied == (256 if prefix_len % BS else 0)
    full = prefix_len // BS
    assert all(f.block_ids[:full] == parent.block_ids[:full] for f in forks)
    assert all(pool.allocator.refcount(b) == 257 for b in parent.block_ids[:full])
    suffix = batched.prefill_slot_mapping(forks, [128] * 256, pool.allocator,
                                          start_positions=[prefix_len] * 256).reshape(-1)
    sk = torch.randn(L, 256 * 128, H, D, generator=g, device=cuda).to(torch.bfloat16)
    sv = torch.randn(L, 256 * 128, H, D, generator=g, device=cuda).to(torch.bfloat16)
    batched.write_paged_kv_batch(pool, sk, sv, torch.from_numpy(suffix).to(cuda))
    gk, gv = batched.read_paged_kv_batch(pool, forks)
    want_pk = pk.permute(0, 2, 1, 3)
    want_pv = pv.permute(0, 2, 1, 3)
    for f in range(256):
        assert torch.equal(gk[:, f, :, :prefix_len].view(torch.int16), want_pk.reshape(L, H, prefix_len, D).view(torch.int16))
        assert torch.equal(gv[:, f, :, :prefix_len].view(torch.int16), want_pv.reshape(L, H, prefix_len, D).view(torch.int16))
        ws = sk[:, f * 128 : (f + 1) * 128].permute(0, 2, 1, 3).reshape(L, H, 128, D)
        assert torch.equal(gk[:, f, :, prefix_len:].view(torch.int16), ws.view(torch.int16))
    # the parent still reads back as the prefix alone (its partial block was never written past it)
    rk, _ = batched.read_paged_kv_batch(pool, [parent])
    assert torch.equal(rk[:, 0].view(torch.int16), want_pk.reshape(L, H, prefix_len, D).view(torch.int16))
    assert _ops.read_status(cuda) == _lib.OK
