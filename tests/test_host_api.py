"""Host-side behaviour of the drop-in API (CPU only, no kernel launches).

Bookkeeping, byte accounting and every validation error must match augur's
(the messages are the reference's, from augur/kv_cache.py,
augur/paged_kv_cache.py and augur/prefix_cache.py); data movement on CPU
tensors must refuse loudly instead of falling back.
"""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

import augur_b200 as ab
from augur_b200 import batched, paged_kv_cache, prefix_cache


def tiny_cfg(**kw):
    base = dict(vocab_size=16, hidden_size=8, intermediate_size=16, num_hidden_layers=2,
                num_attention_heads=2, num_key_value_heads=1)
    base.update(kw)
    return ab.QwenConfig(**base)


# --- contiguous cache (reference tests/test_kv_cache.py) --------------------


def test_new_kv_cache_shapes():
    cache = ab.new_kv_cache(tiny_cfg(), batch_size=3, max_seq_len=5, device=torch.device("cpu"),
                            dtype=torch.float32)
    assert cache.keys.shape == (2, 3, 1, 5, 4) and cache.values.shape == (2, 3, 1, 5, 4)
    assert cache.seq_len == 0 and cache.max_seq_len == 5


def test_kv_cache_nbytes_and_format():
    cfg = tiny_cfg(hidden_size=4, num_hidden_layers=3)
    assert ab.kv_cache_nbytes(cfg, batch_size=2, max_seq_len=5, dtype=torch.float32) == 480
    assert ab.kv_cache_nbytes(cfg, batch_size=2, max_seq_len=5, dtype=torch.float16) == 240
    with pytest.raises(ValueError, match="batch_size"):
        ab.kv_cache_nbytes(cfg, batch_size=0, max_seq_len=5, dtype=torch.float32)
    with pytest.raises(ValueError, match="max_seq_len"):
        ab.kv_cache_nbytes(cfg, batch_size=1, max_seq_len=0, dtype=torch.float32)
    assert ab.format_bytes(512) == "512 B"
    assert ab.format_bytes(1536) == "1.50 KiB"
    assert ab.format_bytes(1024**2) == "1.00 MiB"
    # augur/kv_cache.py:67-72 stops dividing after TiB, so a PiB-sized count
    # prints its TiB magnitude with the PiB label; kept bit-compatible.
    assert ab.format_bytes(3 * 1024**5) == "3072.00 PiB"
    with pytest.raises(ValueError, match="non-negative"):
        ab.format_bytes(-1)


def test_config_validation_matches_reference():
    with pytest.raises(ValueError, match="only silu"):
        ab.QwenConfig(hidden_act="gelu")
    with pytest.raises(ValueError, match="divisible by num_attention_heads"):
        ab.QwenConfig(hidden_size=10, num_attention_heads=3)
    assert ab.QwenConfig().head_dim == 64 and ab.QwenConfig().num_key_value_groups == 7


def _cpu_cache(batch=1, max_seq=4):
    return ab.new_kv_cache(tiny_cfg(), batch_size=batch, max_seq_len=max_seq,
                           device=torch.device("cpu"), dtype=torch.float32)


@pytest.mark.parametrize(
    "kwargs, message",
    [
        (dict(key=torch.zeros(1, 1, 2, 4), value=torch.zeros(1, 1, 3, 4)), "same shape"),
        (dict(layer_idx=2), "layer_idx 2 is outside the cache layer range"),
        (dict(position_ids=torch.tensor([[0, 1, 2]])), r"position_ids must have shape \[batch, seq\]"),
        (dict(key=torch.zeros(2, 1, 2, 4), value=torch.zeros(2, 1, 2, 4),
              position_ids=torch.zeros(2, 2, dtype=torch.long)), "does not match cache shape"),
    ],
)
def test_write_kv_validation_messages(kwargs, message):
    args = dict(layer_idx=0, position_ids=torch.tensor([[0, 1]]), key=torch.zeros(1, 1, 2, 4),
                value=torch.zeros(1, 1, 2, 4))
    args.update(kwargs)
    with pytest.raises(ValueError, match=message):
        ab.write_kv(_cpu_cache(), **args)


def test_write_kv_on_cpu_refuses_instead_of_falling_back():
    with pytest.raises(ValueError, match="needs CUDA tensors"):
        ab.write_kv(_cpu_cache(), 0, torch.tensor([[0]]), torch.zeros(1, 1, 1, 4), torch.zeros(1, 1, 1, 4))


def test_paged_write_and_read_on_cpu_refuse():
    cfg = tiny_cfg()
    pool = ab.new_paged_kv_cache(cfg, num_blocks=2, block_size=4, device=torch.device("cpu"),
                                 dtype=torch.float32)
    table = ab.SequenceBlockTable.empty(4)
    with pytest.raises(ValueError, match="needs CUDA tensors"):
        ab.write_paged_kv(pool, 0, table, torch.tensor([[0]]), torch.zeros(1, 1, 1, 4), torch.zeros(1, 1, 1, 4))
    assert table.block_ids == []  # nothing was allocated before the refusal
    table.ensure_position(0, pool.allocator)
    with pytest.raises(ValueError, match="needs CUDA tensors"):
        ab.read_paged_kv(pool, 0, table)


def test_paged_validation_messages():
    cfg = tiny_cfg()
    pool = ab.new_paged_kv_cache(cfg, num_blocks=2, block_size=4, device=torch.device("cpu"),
                                 dtype=torch.float32)
    t = ab.SequenceBlockTable.empty(4)
    z = torch.zeros(1, 1, 2, 4)
    with pytest.raises(ValueError, match="same shape"):
        ab.write_paged_kv(pool, 0, t, torch.tensor([[0, 1]]), z, torch.zeros(1, 1, 3, 4))
    with pytest.raises(ValueError, match="batch size 1"):
        ab.write_paged_kv(pool, 0, t, torch.tensor([[0, 1]]), torch.zeros(2, 1, 2, 4), torch.zeros(2, 1, 2, 4))
    with pytest.raises(ValueError, match=r"shape \[batch, seq\]"):
        ab.write_paged_kv(pool, 0, t, torch.tensor([[0]]), z, z)
    with pytest.raises(ValueError, match="layer_idx is outside"):
        ab.write_paged_kv(pool, 5, t, torch.tensor([[0, 1]]), z, z)
    with pytest.raises(ValueError, match="does not match cache shape"):
        ab.write_paged_kv(pool, 0, t, torch.tensor([[0, 1]]), torch.zeros(1, 1, 2, 3), torch.zeros(1, 1, 2, 3))
    with pytest.raises(ValueError, match="seq_len must be positive"):
        ab.read_paged_kv(pool, 0, t)
    with pytest.raises(ValueError, match="layer_idx is outside"):
        ab.read_paged_kv(pool, 9, t, seq_len=1)


def test_new_paged_kv_cache_storage():
    cfg = tiny_cfg(hidden_size=4)
    cache = ab.new_paged_kv_cache(cfg, num_blocks=3, block_size=4, device=torch.device("cpu"),
                                  dtype=torch.float32)
    assert cache.keys.shape == (2, 3, 1, 4, 2) and cache.block_size == 4
    assert cache.allocator.allocate() == 0
    with pytest.raises(ValueError, match="block_size must be positive"):
        ab.new_paged_kv_cache(cfg, num_blocks=3, block_size=0, device=torch.device("cpu"), dtype=torch.float32)


# --- bookkeeping, against the reference's inline tests and golden script ----


def test_allocator_and_tables_follow_reference(golden):
    log = dict((entry[0], entry[1:]) for entry in golden["bookkeeping"])
    a = ab.BlockAllocator(12)
    got = [a.allocate() for _ in range(4)]
    assert got == log["allocate4"][0]
    a.free(got[1])
    a.free(got[3])
    assert list(a._free_blocks) == log["after_free_1_3"][0]
    assert [a.allocate() for _ in range(3)] == log["allocate3"][0]
    t = ab.SequenceBlockTable.empty(4)
    t.ensure_position(13, a)
    assert (t.block_ids, t.seq_len) == tuple(log["ensure13"])
    t.free(a)
    assert list(a._free_blocks) == log["free_table"][0]
    t2 = ab.SequenceBlockTable.allocate(a, max_seq_len=9, block_size=4)
    assert (t2.block_ids, t2.seq_len) == tuple(log["table_allocate9"])


def test_prefix_hash_index_follows_reference(golden):
    log = dict((entry[0], entry[1:]) for entry in golden["bookkeeping"])
    pc = ab.PagedPrefixCache()
    h1 = pc.add_block(None, [1, 2, 3, 4], 7)
    h2 = pc.add_block(h1, [5, 6, 7, 8], 9)
    h3 = pc.add_block(h2, [9, 10, 11, 12], 3)
    hx = pc.add_block(None, [5, 6, 7, 8], 11)
    assert [h1, h2, h3, hx] == log["hashes"][0]
    matches = [pc.match_prefix(ids, 4) for ids in ([1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13],
                                                   [1, 2, 3, 4, 5, 6, 7], [5, 6, 7, 8, 1, 2, 3, 4],
                                                   [9, 9, 9, 9])]
    assert [(m.block_ids, m.matched_tokens) for m in matches] == [tuple(x) for x in log["matches"][0]]
    with pytest.raises(ValueError, match="block_tokens must not be empty"):
        pc.add_block(None, [], 1)
    with pytest.raises(ValueError, match="block_size must be positive"):
        pc.match_prefix([1], 0)


def test_allocator_errors_and_refcounts():
    a = ab.BlockAllocator(2)
    with pytest.raises(ValueError, match="num_blocks must be positive"):
        ab.BlockAllocator(0)
    b0 = a.allocate()
    a.incref(b0)
    a.incref(b0)
    assert a.refcount(b0) == 3
    a.free(b0)
    a.free(b0)
    assert a.num_free == 1 and a.refcount(b0) == 1
    a.free(b0)
    assert a.num_free == 2 and a.allocate() == b0
    a.allocate()
    with pytest.raises(RuntimeError, match="no free KV cache blocks"):
        a.allocate()
    with pytest.raises(RuntimeError, match="no free KV cache blocks"):
        ab.BlockAllocator(1).allocate_many(2)


def test_table_fork_shares_blocks():
    a = ab.BlockAllocator(8)
    t = ab.SequenceBlockTable.empty(4)
    t.ensure_position(9, a)
    forks = batched.fork_prefix(SimpleNamespace(allocator=a), t, 3)
    assert all(f.block_ids == t.block_ids and f.seq_len == 10 for f in forks)
    assert [a.refcount(b) for b in t.block_ids] == [4, 4, 4]
    for f in forks:
        f.free(a)
    assert [a.refcount(b) for b in t.block_ids] == [1, 1, 1] and a.num_free == 5


@pytest.mark.parametrize("seed", range(12))
def test_ensure_positions_equals_per_token_loop(oracle, seed):
    """The vectorised allocation + partial-write rule equals the reference's per-token loop."""
    rng = np.random.default_rng(seed)
    bs = int(rng.integers(1, 6))
    nb = int(rng.integers(1, 10))
    n = int(rng.integers(0, 20))
    pos = rng.integers(-1 if seed % 3 == 0 else 0, nb * bs + 3, size=n).astype(np.int64)
    ref_alloc, ref_table = oracle.RefBlockAllocator(nb), oracle.RefBlockTable([], bs)
    written, ref_err = 0, None
    for p in pos.tolist():
        try:
            ref_table.ensure_position(p, ref_alloc)
            ref_table.position_to_block_offset(p)
        except (ValueError, RuntimeError) as exc:
            ref_err = exc
            break
        written += 1
    a, t = ab.BlockAllocator(nb), ab.SequenceBlockTable.empty(bs)
    got, err = paged_kv_cache.ensure_positions(t, pos, a)
    assert got == written
    assert (type(err), str(err)) == (type(ref_err), str(ref_err))
    assert t.block_ids == ref_table.block_ids and t.seq_len == ref_table.seq_len
    assert list(a._free_blocks) == ref_alloc.free_blocks
    if got:
        expect = []
        for p in pos[:got].tolist():
            blk, off = ref_table.position_to_block_offset(p)
            expect.append(blk * bs + off)
        assert paged_kv_cache.slots_for_positions(t, pos[:got]).tolist() == expect


def test_batched_host_helpers(oracle):
    a = ab.BlockAllocator(64)
    tables = [ab.SequenceBlockTable.empty(16) for _ in range(3)]
    slots = batched.prefill_slot_mapping(tables, [37, 16, 1], a)
    assert slots.shape == (3, 37)
    assert [t.block_ids for t in tables] == [[0, 1, 2], [3], [4]]
    assert slots[0, 36] == 2 * 16 + 4 and slots[1, 15] == 3 * 16 + 15 and slots[1, 16] == -1
    assert slots[2, 0] == 64 and (slots[2, 1:] == -1).all()
    runs = batched.handoff_runs(tables, [37, 16, 1])
    assert runs.tolist() == [[0, 0, 0, 0, 16], [0, 16, 1, 0, 16], [0, 32, 2, 0, 5],
                             [1, 0, 3, 0, 16], [2, 0, 4, 0, 1]]
    split = batched.split_runs(np.array([[1, 0, 2, 3, 10], [4, 5, 6, 7, 3]]), 4)
    assert split.tolist() == [[1, 0, 2, 3, 4], [1, 4, 2, 7, 4], [1, 8, 2, 11, 2], [4, 5, 6, 7, 3]]
    dec = batched.decode_slot_mapping(tables, a)
    assert dec.tolist() == [2 * 16 + 5, 5 * 16 + 0, 4 * 16 + 1]
    assert tables[1].block_ids == [3, 5] and tables[1].seq_len == 17


def test_prefix_cache_lookup_and_cache_prefix(monkeypatch):
    pc = ab.PrefixCache()
    e = lambda ids: ab.PrefixCacheEntry(token_ids=torch.tensor(ids), keys=torch.empty(0),  # noqa: E731
                                        values=torch.empty(0), logits=torch.empty(0))
    short, long, miss = e([1, 2]), e([1, 2, 3]), e([2, 3])
    for x in (short, long, miss):
        pc.add(x)
    assert pc.longest_prefix(torch.tensor([[1, 2, 3, 4]])) is long
    assert pc.longest_prefix(torch.tensor([[9, 2, 3]])) is None
    with pytest.raises(ValueError, match="batch size 1"):
        pc.longest_prefix(torch.tensor([[1], [2]]))
    with pytest.raises(ValueError, match="max_entries must be positive"):
        ab.PrefixCache(max_entries=0)
    bounded = ab.PrefixCache(max_entries=1)
    bounded.add(short)
    bounded.add(long)
    assert bounded.longest_prefix(torch.tensor([[1, 2, 3]])) is long and len(bounded._entries) == 1

    cfg = tiny_cfg(hidden_size=4)

    def fake_model(input_ids, w, cfg, cache=None, position_ids=None):
        assert position_ids.tolist() == [[0, 1, 2]]
        cache.keys[:, 0, :, :3, :] = 11
        cache.values[:, 0, :, :3, :] = 22
        cache.seq_len = 3
        logits = torch.zeros(1, 3, cfg.vocab_size)
        logits[:, -1, 5] = 1
        return logits

    monkeypatch.setattr(prefix_cache, "model", fake_model)
    # the entry's K/V leave the cache through the library's copy kernel: CUDA only
    with pytest.raises(ValueError, match="CUDA"):
        ab.cache_prefix(torch.tensor([[1, 2, 3]]),
                        SimpleNamespace(embed_tokens=torch.empty(0, dtype=torch.float32)), cfg)


def test_copy_prefix_validation():
    cache = _cpu_cache(batch=1, max_seq=5)
    entry = ab.PrefixCacheEntry(token_ids=torch.tensor([1, 2, 3]), keys=torch.zeros(2, 1, 3, 4),
                                values=torch.zeros(2, 1, 3, 4), logits=torch.empty(0))
    with pytest.raises(ValueError, match="batch_idx is outside"):
        ab.copy_prefix_into_cache(entry, cache, batch_idx=1)
    long = ab.PrefixCacheEntry(token_ids=torch.arange(6), keys=torch.zeros(2, 1, 6, 4),
                               values=torch.zeros(2, 1, 6, 4), logits=torch.empty(0))
    with pytest.raises(ValueError, match="exceeds cache capacity"):
        ab.copy_prefix_into_cache(long, cache)
    bad = ab.PrefixCacheEntry(token_ids=torch.tensor([1, 2, 3]), keys=torch.zeros(2, 1, 3, 3),
                              values=torch.zeros(2, 1, 3, 3), logits=torch.empty(0))
    with pytest.raises(ValueError, match="do not match cache shape"):
        ab.copy_prefix_into_cache(bad, cache)
    with pytest.raises(ValueError, match="needs CUDA tensors"):
        ab.copy_prefix_into_cache(entry, cache)


def test_paged_decode_attention_refuses_cpu_and_bad_shapes():
    from augur_b200.attention import DecodeTables, paged_decode_attention

    cfg = ab.QwenConfig()
    cpu = ab.new_paged_kv_cache(cfg, num_blocks=2, block_size=16, device=torch.device("cpu"), dtype=torch.bfloat16)
    t = ab.SequenceBlockTable(block_ids=[0], block_size=16, seq_len=3)
    with pytest.raises(ValueError, match="needs CUDA tensors"):
        paged_decode_attention(torch.zeros(1, 14, 64, dtype=torch.bfloat16), cpu, 0, [t])
    with pytest.raises(ValueError, match="one query token"):
        paged_decode_attention(torch.zeros(1, 14, 2, 64, dtype=torch.bfloat16), cpu, 0, [t])
    with pytest.raises(ValueError, match="block table capacity"):
        DecodeTables([ab.SequenceBlockTable(block_ids=[0], block_size=16, seq_len=17)], torch.device("cpu"))


def test_decode_step_packs_its_arrays_into_one_buffer():
    """A decode step's positions, slots, block tables and lengths are views of one buffer,
    filled by one copy, with the values the per-array builders give."""
    from augur_b200.attention import DecodeTables
    from augur_b200.decode import DecodeStep

    cpu = ab.new_paged_kv_cache(ab.QwenConfig(), num_blocks=8, block_size=4, device=torch.device("cpu"),
                                dtype=torch.bfloat16)
    tables = [ab.SequenceBlockTable(block_ids=[], block_size=4, seq_len=0) for _ in range(3)]
    for t, n in zip(tables, (4, 6, 1)):  # the first grows a block at the step, the others do not
        t.ensure_position(n - 1, cpu.allocator)
        t.seq_len = n
    twins = [ab.SequenceBlockTable(block_ids=list(t.block_ids), block_size=4, seq_len=t.seq_len) for t in tables]
    step = DecodeStep(cpu, tables)
    assert step.positions.tolist() == [4, 6, 1] and step.max_position == 6 and step.batch == 3
    assert step.slots.tolist() == [t.block_ids[p // 4] * 4 + p % 4 for t, p in zip(tables, (4, 6, 1))]
    assert step.slots.dtype == step.positions.dtype == torch.int64
    for t in twins:
        t.seq_len += 1
        t.block_ids = next(u for u in tables if u.block_ids[: len(t.block_ids)] == t.block_ids).block_ids
    ref = DecodeTables(twins, torch.device("cpu"))
    assert torch.equal(step.tables.blocks, ref.blocks) and torch.equal(step.tables.lens, ref.lens)
    assert step.tables.lens.tolist() == [5, 7, 2] and step.tables.max_seq_len == 7
    base = step.positions.untyped_storage().data_ptr()
    assert step.tables.blocks.untyped_storage().data_ptr() == base == step.tables.lens.untyped_storage().data_ptr()
    empty = DecodeStep(cpu, [])
    assert empty.batch == 0 and empty.positions.numel() == 0 and empty.tables.blocks.shape == (0, 1)
    # a table's ids are converted again whenever its list changes, in place too (copy-on-write)
    tables[1].block_ids[0] = 7
    assert DecodeTables(tables, torch.device("cpu")).blocks[1, 0] == 7
    tables[1].block_ids = [5, 6]
    assert DecodeTables(tables, torch.device("cpu")).blocks[1].tolist()[:2] == [5, 6]
    assert tables[1] == ab.SequenceBlockTable(block_ids=[5, 6], block_size=4, seq_len=7)


def test_rope_tables_follow_the_reference_formula(oracle):
    """The product's cos/sin tables equal the oracle's (pinned to augur/rope.py) bit for bit."""
    from augur_b200.rope import rope_tables

    for dt in (torch.float32, torch.bfloat16, torch.float16):
        cos, sin = rope_tables(64, 1000000.0, dt, 5000, torch.device("cpu"))
        assert cos.shape == (8192, 32) and cos.dtype == dt
        rc, rs = oracle.rope_table(64, 1000000.0, 8192, dt)
        assert torch.equal(cos.view(torch.uint8), rc.view(torch.uint8))
        assert torch.equal(sin.view(torch.uint8), rs.view(torch.uint8))
    with pytest.raises(ValueError, match="even"):
        rope_tables(63, 10000.0, torch.float32, 8, torch.device("cpu"))


def test_rope_writes_refuse_cpu_and_bad_shapes():
    from augur_b200.rope import rope_write_kv, rope_write_paged_kv, write_paged_kv_batch_rope

    cfg = ab.QwenConfig()
    pool = ab.new_paged_kv_cache(cfg, num_blocks=4, block_size=16, device=torch.device("cpu"), dtype=torch.bfloat16)
    t = ab.SequenceBlockTable.empty(16)
    q = torch.zeros(1, 14, 3, 64, dtype=torch.bfloat16)
    kv = torch.zeros(1, 2, 3, 64, dtype=torch.bfloat16)
    pos = torch.arange(3).unsqueeze(0)
    with pytest.raises(ValueError, match="needs CUDA tensors"):
        rope_write_paged_kv(pool, 0, t, pos, q, kv, kv, 1e6)
    assert t.block_ids == []  # nothing allocated before the refusal
    with pytest.raises(ValueError, match="batch size 1"):
        rope_write_paged_kv(pool, 0, t, pos.repeat(2, 1), q.repeat(2, 1, 1, 1), kv.repeat(2, 1, 1, 1),
                            kv.repeat(2, 1, 1, 1), 1e6)
    with pytest.raises(ValueError, match="q must be"):
        rope_write_paged_kv(pool, 0, t, pos, q[:, :, :2], kv, kv, 1e6)
    cache = ab.new_kv_cache(cfg, batch_size=1, max_seq_len=8, device=torch.device("cpu"), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="needs CUDA tensors"):
        rope_write_kv(cache, 0, pos, q, kv, kv, 1e6)
    with pytest.raises(ValueError, match="exceeds cache capacity|needs CUDA"):
        rope_write_kv(cache, 0, pos + 8, q, kv, kv, 1e6)
    with pytest.raises(ValueError, match="slot_mapping and positions"):
        write_paged_kv_batch_rope(pool, q[0].transpose(0, 1), kv[0].transpose(0, 1), kv[0].transpose(0, 1),
                                  torch.zeros(2, dtype=torch.int64), torch.zeros(3, dtype=torch.int64), 1e6, 0)


def test_decode_graph_step_refuses_a_cpu_cache():
    from augur_b200.decode import DecodeGraphStep

    cpu = ab.PagedKVCache(keys=torch.zeros(1, 4, 2, 16, 64, dtype=torch.bfloat16),
                          values=torch.zeros(1, 4, 2, 16, 64, dtype=torch.bfloat16),
                          block_size=16, allocator=ab.BlockAllocator(4))
    with pytest.raises(ValueError, match="needs CUDA tensors"):
        DecodeGraphStep(cpu, batch=2, max_blocks=2, n_q_heads=14, rope_theta=1e6)


def test_keep_last_marks_earlier_repeats():
    from augur_b200.paged_kv_cache import keep_last

    x = np.array([3, 5, 3, 7, 5, 9, 3], dtype=np.int64)
    assert keep_last(x).tolist() == [-1, -1, -1, 7, 5, 9, 3]
    y = np.array([4, 1, 2], dtype=np.int64)
    assert keep_last(y) is y  # no repeats: unchanged, no copy
    assert keep_last(np.array([6], dtype=np.int64)).tolist() == [6]


def test_position_range_reads_repeats_per_row():
    from augur_b200.kv_cache import keep_last_per_row, position_range

    pos = torch.tensor([[2, 4, 2, 9], [0, 1, 2, 3]])
    assert position_range(pos) == (9, 0, True)
    assert position_range(torch.tensor([[2, 4], [2, 4]])) == (4, 2, False)  # repeats across rows are fine
    assert position_range(torch.tensor([[7], [3]])) == (7, 3, False)
    assert keep_last_per_row(pos).tolist() == [[-1, 4, 2, 9], [0, 1, 2, 3]]
