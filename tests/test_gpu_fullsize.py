"""Full-size workloads (the benchmark configurations) against the oracle.

Every check here compares the device pool itself, copied back with plain
tensor indexing, with what the oracle (the reference's write_paged_kv loop
and block bookkeeping, restated in oracle/) builds on the host from the same
inputs; nothing is read back through the library's own gather.
  * config 2: all 64 sequences' blocks, plus the count of rows that must
    still hold the 0xFF poison (nothing written out of place);
  * config 3: the whole pool, bit for bit, after the contiguous -> paged
    handoff (both copy paths) and again after 256 decode appends, with the
    block tables the reference's allocator produces;
  * config 4: the block holding the first position after the prefix, for
    all 256 forks (the copy-on-write copy plus the suffix rows), the parent's
    blocks, and a seeded sample of forks position by position against the
    oracle's private-table write of prefix then suffix.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import augur_b200 as ab
from augur_b200 import _lib, _ops, batched
from bench import BS, D, H, L, config2_batch, config3_lengths, oracle_check_sequences
from tests.conftest import assert_bits_equal, poison_

pytestmark = pytest.mark.gpu


def _poison_count(t: torch.Tensor) -> int:
    return int((t.view(torch.int16) == -1).sum().item())


def _pool(nb, device):
    return ab.PagedKVCache(keys=poison_(torch.empty(L, nb, H, BS, D, dtype=torch.bfloat16, device=device)),
                           values=poison_(torch.empty(L, nb, H, BS, D, dtype=torch.bfloat16, device=device)),
                           block_size=BS, allocator=ab.BlockAllocator(nb))


def _host_pool(nb):
    return (poison_(torch.empty(L, nb, H, BS, D, dtype=torch.bfloat16)),
            poison_(torch.empty(L, nb, H, BS, D, dtype=torch.bfloat16)))


def _ref_slots(oracle, table, alloc, positions) -> np.ndarray:
    """The reference's per-token ensure_position + position_to_block_offset, as slots."""
    out = np.empty(len(positions), dtype=np.int64)
    for i, p in enumerate(positions):
        table.ensure_position(int(p), alloc)
        blk, off = table.position_to_block_offset(int(p))
        out[i] = blk * BS + off
    return out


def test_config2_full_scatter_all_sequences(cuda):
    """8192 tokens x 24 layers into a 65,536-block pool (12.9 GB): every sequence's blocks."""
    lens, slots, k, v, _ = config2_batch(seed=0)
    pool = _pool(65536, cuda)
    batched.write_paged_kv_batch(pool, k.to(cuda), v.to(cuda), torch.from_numpy(slots).to(cuda))
    assert _ops.read_status(cuda) == _lib.OK
    samples, pos0 = [], 0
    for n in lens:
        n = int(n)
        sl = slots[pos0 : pos0 + n]
        samples.append({"ids": (sl[::BS] // BS).tolist(), "k": k[:, pos0 : pos0 + n].contiguous(),
                        "v": v[:, pos0 : pos0 + n].contiguous(), "pre": sl})
        pos0 += n
    ok, tokens = oracle_check_sequences(pool, samples)
    assert ok and tokens == 8192
    written = 8192 * L * H * D
    assert _poison_count(pool.keys) == pool.keys.numel() - written
    assert _poison_count(pool.values) == pool.values.numel() - written


def test_config3_full_handoff_and_256_appends(cuda, oracle):
    """32 prompts of U[512,2048] tokens: handoff (both copy paths), then 256 decode steps,
    the whole pool against the oracle's after each phase."""
    lens = config3_lengths()
    B, Lmax, NB = len(lens), int(lens.max()), 8192
    g = torch.Generator(device=cuda).manual_seed(3)
    src = ab.KVCache(keys=torch.randn(L, B, H, Lmax, D, generator=g, device=cuda).to(torch.bfloat16),
                     values=torch.randn(L, B, H, Lmax, D, generator=g, device=cuda).to(torch.bfloat16))
    results = []
    for flags in (_lib.COPY_VECTOR, _lib.COPY_BULK):
        pool = _pool(NB, cuda)
        tables = [ab.SequenceBlockTable.empty(BS) for _ in lens]
        batched.handoff_contiguous_to_paged(src, pool, tables, lens, flags=flags)
        results.append((pool, tables))
    (pa, ta), (pb, tb) = results
    assert [t.block_ids for t in ta] == [t.block_ids for t in tb]
    assert torch.equal(pa.keys.view(torch.int16), pb.keys.view(torch.int16))
    assert torch.equal(pa.values.view(torch.int16), pb.values.view(torch.int16))
    del results, pb, tb
    # oracle: the handoff is write_paged_kv(pool, l, table_b, arange(n_b), keys[l, b:b+1, :, :n_b])
    # for every layer, sequence by sequence (blocks allocated at the first layer)
    hk, hv = _host_pool(NB)
    alloc = oracle.RefBlockAllocator(NB)
    ref_tables = [oracle.RefBlockTable([], BS) for _ in lens]
    sk_host, sv_host = src.keys.cpu(), src.values.cpu()
    for b, n in enumerate(lens):
        n = int(n)
        sl = _ref_slots(oracle, ref_tables[b], alloc, range(n))
        oracle.scatter_slots(sk_host[:, b, :, :n].permute(0, 2, 1, 3).contiguous(),
                             sv_host[:, b, :, :n].permute(0, 2, 1, 3).contiguous(), sl, hk, hv, BS)
    assert [t.block_ids for t in ta] == [t.block_ids for t in ref_tables]
    assert_bits_equal(pa.keys, hk, "handoff keys")
    assert_bits_equal(pa.values, hv, "handoff values")
    del sk_host, sv_host
    # 256 decode appends, one token per sequence per step, all layers
    steps = 256
    nk = torch.randn(steps, L, B, H, D, generator=g, device=cuda).to(torch.bfloat16)
    nv = torch.randn(steps, L, B, H, D, generator=g, device=cuda).to(torch.bfloat16)
    for s in range(steps):
        batched.append_decode(pa, ta, nk[s], nv[s])
    nk_host, nv_host = nk.cpu(), nv.cpu()
    for s in range(steps):
        sl = np.array([_ref_slots(oracle, rt, alloc, [int(n) + s])[0] for rt, n in zip(ref_tables, lens)])
        oracle.scatter_slots(nk_host[s], nv_host[s], sl, hk, hv, BS)
    assert [t.block_ids for t in ta] == [t.block_ids for t in ref_tables]
    assert [t.seq_len for t in ta] == [int(n) + steps for n in lens]
    assert_bits_equal(pa.keys, hk, "keys after appends")
    assert_bits_equal(pa.values, hv, "values after appends")
    assert _ops.read_status(cuda) == _lib.OK


@pytest.mark.parametrize("prefix_len", [1024, 1000])
def test_config4_full_fork_cow_suffix(cuda, oracle, prefix_len):
    """One prefix shared by 256 forks; copy-on-write of a partial last block; 128-token suffixes."""
    g = torch.Generator(device=cuda).manual_seed(4)
    NB, n_forks, suf = 8192, 256, 128
    pool = _pool(NB, cuda)
    parent = ab.SequenceBlockTable.empty(BS)
    sm = batched.prefill_slot_mapping([parent], [prefix_len], pool.allocator)[0]
    pk = torch.randn(L, prefix_len, H, D, generator=g, device=cuda).to(torch.bfloat16)
    pv = torch.randn(L, prefix_len, H, D, generator=g, device=cuda).to(torch.bfloat16)
    batched.write_paged_kv_batch(pool, pk, pv, torch.from_numpy(sm).to(cuda))
    forks = batched.fork_prefix(pool, parent, n_forks)
    copied = batched.cow_partial_blocks(pool, forks)
    rows = prefix_len % BS
    assert copied == (n_forks if rows else 0)
    full = prefix_len // BS
    assert all(f.block_ids[:full] == parent.block_ids[:full] for f in forks)
    assert all(pool.allocator.refcount(b) == n_forks + 1 for b in parent.block_ids[:full])
    suffix = batched.prefill_slot_mapping(forks, [suf] * n_forks, pool.allocator,
                                          start_positions=[prefix_len] * n_forks).reshape(-1)
    sk = torch.randn(L, n_forks * suf, H, D, generator=g, device=cuda).to(torch.bfloat16)
    sv = torch.randn(L, n_forks * suf, H, D, generator=g, device=cuda).to(torch.bfloat16)
    batched.write_paged_kv_batch(pool, sk, sv, torch.from_numpy(suffix).to(cuda))
    assert _ops.read_status(cuda) == _lib.OK
    pk_h, pv_h, sk_h, sv_h = pk.cpu(), pv.cpu(), sk.cpu(), sv.cpu()

    # (1) all forks: the block holding position prefix_len is the copy-on-write copy of the
    # parent's partial block (rows [0, rows)) followed by the fork's first suffix tokens
    tail = slice(full * BS, prefix_len)
    head = BS - rows
    toks_k = torch.cat([torch.cat([pk_h[:, tail], sk_h[:, f * suf : f * suf + head]], dim=1)
                        for f in range(n_forks)], dim=1)
    toks_v = torch.cat([torch.cat([pv_h[:, tail], sv_h[:, f * suf : f * suf + head]], dim=1)
                        for f in range(n_forks)], dim=1)
    ek, ev = (poison_(torch.empty(L, n_forks, H, BS, D, dtype=torch.bfloat16)) for _ in range(2))
    oracle.scatter_slots(toks_k.contiguous(), toks_v.contiguous(), np.arange(n_forks * BS, dtype=np.int64),
                         ek, ev, BS)
    boundary = torch.tensor([f.block_ids[full] for f in forks], device=cuda)
    assert len(set(boundary.tolist())) == n_forks  # every fork owns its boundary block
    assert_bits_equal(pool.keys.index_select(1, boundary), ek, "boundary blocks keys")
    assert_bits_equal(pool.values.index_select(1, boundary), ev, "boundary blocks values")

    # (2) the parent's blocks: the prefix, and its partial block untouched past `rows`
    pids = np.asarray(parent.block_ids, dtype=np.int64)
    ok, _ = oracle_check_sequences(pool, [{"ids": pids.tolist(), "k": pk_h, "v": pv_h,
                                           "pre": np.arange(prefix_len) % BS + pids[np.arange(prefix_len) // BS] * BS}])
    assert ok, "parent blocks"

    # (3) a seeded sample of forks, position by position, against the reference's
    # composition: write_paged_kv of the prefix, then of the suffix, into a private table
    pick = np.random.default_rng(44).choice(n_forks, size=8, replace=False).tolist() + [n_forks - 1]
    for f in pick:
        rk, rv = _host_pool(-(-(prefix_len + suf) // BS))
        alloc = oracle.RefBlockAllocator(rk.shape[1])
        rt = oracle.RefBlockTable([], BS)
        oracle.scatter_slots(pk_h, pv_h, _ref_slots(oracle, rt, alloc, range(prefix_len)), rk, rv, BS)
        oracle.scatter_slots(sk_h[:, f * suf : (f + 1) * suf].contiguous(),
                             sv_h[:, f * suf : (f + 1) * suf].contiguous(),
                             _ref_slots(oracle, rt, alloc, range(prefix_len, prefix_len + suf)), rk, rv, BS)
        n = prefix_len + suf
        p = torch.arange(n)
        ids = torch.tensor(forks[f].block_ids, device=cuda)
        blk, off = ids[(p // BS).to(cuda)], (p % BS).to(cuda)
        for pool_t, ref_t, what in ((pool.keys, rk, "keys"), (pool.values, rv, "values")):
            got = pool_t.permute(0, 1, 3, 2, 4)[:, blk, off].cpu()  # [L, n, H, D] in position order
            want = torch.stack([oracle.read_paged_kv(ref_t, ref_t, layer, rt, n)[0][0] for layer in range(L)])
            assert_bits_equal(got, want.permute(0, 2, 1, 3), f"fork {f} {what}")

    # nothing written out of place: prefix once, per fork the COW copy and its suffix
    written = (prefix_len + n_forks * (rows + suf)) * L * H * D
    assert _poison_count(pool.keys) == pool.keys.numel() - written
    assert _poison_count(pool.values) == pool.values.numel() - written
