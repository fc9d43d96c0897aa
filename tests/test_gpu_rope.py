"""RoPE fused with the cache write vs the reference (bit-exact).

The reference rotates q and k with apply_rope (augur/rope.py:12-40) and then
writes k and v into the cache (augur/attention.py:53-71). With cos/sin tables
built by the reference's formula the kernel rounds exactly where the
reference's dtype ops round, so every comparison here is bitwise: against
fixtures produced by the reference itself, and against the oracle's
restatement on seeded batches.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import augur_b200 as ab
from augur_b200 import _lib, _ops
from augur_b200.rope import rope_write_kv, rope_write_paged_kv, write_paged_kv_batch_rope
from tests.conftest import assert_bits_equal, poison_

pytestmark = pytest.mark.gpu

THETA = 1000000.0


def _is_poison(t: torch.Tensor) -> bool:
    return bool((t.contiguous().view(torch.uint8) == 0xFF).all())


@pytest.mark.parametrize("case", ["f32", "bf16", "f16"])
def test_golden_rope_write_paged_kv(cuda, golden, case):
    c = golden["rope"][f"paged_{case}"]
    dt = c["calls"][0]["q"].dtype
    NB = c["num_blocks"]
    pool = ab.PagedKVCache(keys=poison_(torch.empty(1, NB, 2, 16, 64, dtype=dt, device=cuda)),
                           values=poison_(torch.empty(1, NB, 2, 16, 64, dtype=dt, device=cuda)),
                           block_size=16, allocator=ab.BlockAllocator(NB))
    for _ in range(c["prior_allocated"]):
        pool.allocator.allocate()
    table = ab.SequenceBlockTable.empty(16)
    for call in c["calls"]:
        q_out = rope_write_paged_kv(pool, 0, table, call["position_ids"], call["q"].to(cuda), call["k"].to(cuda),
                                    call["v"].to(cuda), c["theta"])
        assert q_out.shape == call["q"].shape
        assert_bits_equal(q_out, call["q_embed"], "rotated q")
    assert table.block_ids == c["block_ids"]
    assert_bits_equal(pool.keys[:, c["touched_blocks"]], c["keys"], "keys")
    assert_bits_equal(pool.values[:, c["touched_blocks"]], c["values"], "values")
    others = [b for b in range(NB) if b not in c["touched_blocks"]]
    assert _is_poison(pool.keys[:, others]) and _is_poison(pool.values[:, others])
    assert _ops.read_status(cuda) == _lib.OK


@pytest.mark.parametrize("case", ["f32", "bf16", "f16"])
def test_golden_rope_write_kv(cuda, golden, case):
    c = golden["rope"][f"contig_{case}"]
    dt = c["q"].dtype
    cache = ab.KVCache(keys=poison_(torch.empty(c["keys"].shape, dtype=dt, device=cuda)),
                       values=poison_(torch.empty(c["values"].shape, dtype=dt, device=cuda)))
    q_out, kview, vview = rope_write_kv(cache, 0, c["position_ids"], c["q"].to(cuda), c["k"].to(cuda),
                                        c["v"].to(cuda), c["theta"])
    assert_bits_equal(q_out, c["q_embed"], "rotated q")
    assert_bits_equal(cache.keys, c["keys"], "keys")
    assert_bits_equal(cache.values, c["values"], "values")
    assert cache.seq_len == c["seq_len"] and kview.shape[2] == c["seq_len"]
    assert kview.data_ptr() == cache.keys.data_ptr() and vview.data_ptr() == cache.values.data_ptr()


@pytest.mark.parametrize("case", ["f32", "bf16", "f16"])
def test_golden_far_positions(cuda, golden, case):
    """Positions 0, 1, 4095, 8191, 32767: large angles, table rows far apart."""
    c = golden["rope"][f"far_{case}"]
    dt = c["q"].dtype
    pool = ab.PagedKVCache(keys=poison_(torch.empty(1, 1, 2, 16, 64, dtype=dt, device=cuda)),
                           values=poison_(torch.empty(1, 1, 2, 16, 64, dtype=dt, device=cuda)),
                           block_size=16, allocator=ab.BlockAllocator(1))
    q = c["q"][0].transpose(0, 1).to(cuda)  # [tokens, heads, D]
    k = c["k"][0].transpose(0, 1).to(cuda)
    pos = c["position_ids"][0].to(cuda)
    q_out = write_paged_kv_batch_rope(pool, q, k, k, torch.arange(5, device=cuda), pos, c["theta"], 0)
    assert_bits_equal(q_out, c["q_embed"][0].transpose(0, 1), "rotated q")
    assert_bits_equal(pool.keys[0, 0, :, :5], c["k_embed"][0], "rotated k")
    assert_bits_equal(pool.values[0, 0, :, :5], c["k"][0], "v copied unrotated")
    assert _ops.read_status(cuda) == _lib.OK


def _batch_case(cuda, oracle, dtype, T, Hq, Hkv, D, seed, head_stride_pad=0):
    g = torch.Generator().manual_seed(seed)
    rng = np.random.default_rng(seed)
    NB, bs = 64, 16
    q = torch.randn(T, Hq, D + head_stride_pad, generator=g).to(dtype)[..., :D]
    k = torch.randn(T, Hkv, D, generator=g).to(dtype)
    v = torch.randn(T, Hkv, D, generator=g).to(dtype)
    pos = torch.from_numpy(rng.integers(0, 8192, size=T).astype(np.int64))
    slots = rng.permutation(NB * bs)[:T].astype(np.int64)
    slots[rng.random(T) < 0.1] = -1  # padding tokens: no cache write, q still rotated
    pool = ab.PagedKVCache(keys=poison_(torch.empty(1, NB, Hkv, bs, D, dtype=dtype, device=cuda)),
                           values=poison_(torch.empty(1, NB, Hkv, bs, D, dtype=dtype, device=cuda)),
                           block_size=bs, allocator=ab.BlockAllocator(NB))
    q_out = write_paged_kv_batch_rope(pool, q.to(cuda), k.to(cuda), v.to(cuda), torch.from_numpy(slots).to(cuda),
                                      pos.to(cuda), THETA, 0, max_position=8191)
    # oracle: table-indexed apply_rope on [1, heads, T, D] views, then the slot scatter
    table = oracle.rope_table(D, THETA, 8192, dtype)
    qe, ke = oracle.apply_rope(q.transpose(0, 1)[None], k.transpose(0, 1)[None], pos[None], THETA, table=table)
    assert_bits_equal(q_out, qe[0].transpose(0, 1), "rotated q")
    rk, rv = poison_(torch.empty(1, NB, Hkv, bs, D, dtype=dtype)), poison_(torch.empty(1, NB, Hkv, bs, D, dtype=dtype))
    keep = slots >= 0
    oracle.scatter_slots(ke[0].transpose(0, 1)[keep][None], v[keep][None], slots[keep], rk, rv, bs)
    assert_bits_equal(pool.keys, rk, "pool keys")
    assert_bits_equal(pool.values, rv, "pool values")
    assert _ops.read_status(cuda) == _lib.OK


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("Hq, Hkv, D", [(14, 2, 64), (8, 2, 128), (4, 4, 64), (12, 4, 128), (28, 4, 64)])
def test_batch_matches_oracle(cuda, oracle, dtype, Hq, Hkv, D):
    _batch_case(cuda, oracle, dtype, 300, Hq, Hkv, D, 5)


def test_unaligned_rows_take_the_element_path(cuda, oracle):
    """head_dim 40 (a half row of 40 bytes) and a q with padded head stride."""
    _batch_case(cuda, oracle, torch.bfloat16, 77, 6, 2, 40, 6)
    _batch_case(cuda, oracle, torch.bfloat16, 77, 14, 2, 64, 7, head_stride_pad=4)


def test_decode_step_through_rope_write_paged_kv(cuda, oracle):
    """One token per call at growing positions, bf16, augur's shape."""
    pool = ab.PagedKVCache(keys=poison_(torch.empty(1, 8, 2, 16, 64, dtype=torch.bfloat16, device=cuda)),
                           values=poison_(torch.empty(1, 8, 2, 16, 64, dtype=torch.bfloat16, device=cuda)),
                           block_size=16, allocator=ab.BlockAllocator(8))
    rk = poison_(torch.empty(1, 8, 2, 16, 64, dtype=torch.bfloat16))
    rv = poison_(torch.empty(1, 8, 2, 16, 64, dtype=torch.bfloat16))
    ra = oracle.RefBlockAllocator(8)
    rt = oracle.RefBlockTable([], 16)
    table = ab.SequenceBlockTable.empty(16)
    g = torch.Generator().manual_seed(8)
    for p in (0, 1, 15, 16, 17, 100):
        q = torch.randn(1, 1, 14, 64, generator=g).to(torch.bfloat16).permute(0, 2, 1, 3)
        k = torch.randn(1, 1, 2, 64, generator=g).to(torch.bfloat16).permute(0, 2, 1, 3)
        v = torch.randn(1, 1, 2, 64, generator=g).to(torch.bfloat16).permute(0, 2, 1, 3)
        pos = torch.tensor([[p]])
        got = rope_write_paged_kv(pool, 0, table, pos, q.to(cuda), k.to(cuda), v.to(cuda), THETA)
        qe, ke = oracle.apply_rope(q, k, pos, THETA)
        oracle.write_paged_kv(rk, rv, ra, 0, rt, [p], ke, v)
        assert_bits_equal(got, qe, f"q at {p}")
    assert table.block_ids == rt.block_ids
    assert_bits_equal(pool.keys, rk, "keys")
    assert_bits_equal(pool.values, rv, "values")


def test_capacity_error_writes_the_tokens_before_it(cuda):
    """Pool exhaustion mid-chunk: like write_paged_kv, earlier tokens are written, then the error."""
    pool = ab.PagedKVCache(keys=poison_(torch.empty(1, 2, 2, 16, 64, dtype=torch.bfloat16, device=cuda)),
                           values=poison_(torch.empty(1, 2, 2, 16, 64, dtype=torch.bfloat16, device=cuda)),
                           block_size=16, allocator=ab.BlockAllocator(2))
    table = ab.SequenceBlockTable.empty(16)
    q = torch.randn(1, 14, 40, 64, device=cuda).to(torch.bfloat16)
    kv = torch.randn(1, 2, 40, 64, device=cuda).to(torch.bfloat16)
    with pytest.raises(RuntimeError, match="no free KV cache blocks"):
        rope_write_paged_kv(pool, 0, table, torch.arange(40).unsqueeze(0), q, kv, kv, THETA)
    assert table.block_ids == [0, 1]
    assert not _is_poison(pool.values[0, :, :, :, :])  # the first 32 tokens landed
    assert torch.equal(pool.values[0, 1, :, 15].view(torch.int16), kv[0, :, 31].view(torch.int16))


def test_position_outside_table_is_reported(cuda):
    pool = ab.PagedKVCache(keys=poison_(torch.empty(1, 1, 2, 16, 64, dtype=torch.bfloat16, device=cuda)),
                           values=poison_(torch.empty(1, 1, 2, 16, 64, dtype=torch.bfloat16, device=cuda)),
                           block_size=16, allocator=ab.BlockAllocator(1))
    q = torch.randn(2, 14, 64, device=cuda).to(torch.bfloat16)
    k = torch.randn(2, 2, 64, device=cuda).to(torch.bfloat16)
    # max_position understates the positions: a fresh table (a theta no other test
    # uses) has 4096 rows, so position 5000 is outside it
    write_paged_kv_batch_rope(pool, q, k, k, torch.tensor([0, 1], device=cuda),
                              torch.tensor([3, 5000], device=cuda), 12345.0, 0, max_position=10)
    assert _ops.read_status(cuda) == _lib.EBOUNDS
    assert _is_poison(pool.keys[0, 0, :, 1]) and not _is_poison(pool.keys[0, 0, :, 0])


@pytest.mark.parametrize("positions_on", ["device", "host"])
def test_rope_writes_keep_the_last_duplicate(cuda, oracle, positions_on):
    """Repeated positions in one call: every q is rotated; the cache keeps the later token
    (apply_rope then write_kv / write_paged_kv, as the reference runs them)."""
    g = torch.Generator().manual_seed(21)
    B, H, Hq, S, D, M = 2, 2, 4, 6, 64, 16
    pos = torch.tensor([[4, 1, 4, 2, 1, 9], [0, 0, 3, 3, 5, 0]])
    q = torch.randn(B, Hq, S, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, H, S, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, H, S, D, generator=g).to(torch.bfloat16)
    qe, ke = oracle.apply_rope(q, k, pos, THETA)
    p_arg = pos if positions_on == "host" else pos.to(cuda)
    # contiguous cache
    cache = ab.KVCache(keys=poison_(torch.empty(2, B, H, M, D, dtype=torch.bfloat16, device=cuda)),
                       values=poison_(torch.empty(2, B, H, M, D, dtype=torch.bfloat16, device=cuda)))
    ck = poison_(torch.empty(2, B, H, M, D, dtype=torch.bfloat16))
    cv = poison_(torch.empty(2, B, H, M, D, dtype=torch.bfloat16))
    q_out, _, _ = rope_write_kv(cache, 1, p_arg, q.to(cuda), k.to(cuda), v.to(cuda), THETA)
    oracle.write_kv(ck, cv, 1, pos, ke, v)
    assert_bits_equal(q_out, qe, "rotated q")
    assert_bits_equal(cache.keys, ck, "keys")
    assert_bits_equal(cache.values, cv, "values")
    # paged cache, batch 1
    pool = ab.PagedKVCache(keys=poison_(torch.empty(1, 4, H, 4, D, dtype=torch.bfloat16, device=cuda)),
                           values=poison_(torch.empty(1, 4, H, 4, D, dtype=torch.bfloat16, device=cuda)),
                           block_size=4, allocator=ab.BlockAllocator(4))
    table = ab.SequenceBlockTable.empty(4)
    rk = poison_(torch.empty(1, 4, H, 4, D, dtype=torch.bfloat16))
    rv = poison_(torch.empty(1, 4, H, 4, D, dtype=torch.bfloat16))
    q_out = rope_write_paged_kv(pool, 0, table, p_arg[:1], q[:1].to(cuda), k[:1].to(cuda), v[:1].to(cuda), THETA)
    rt = oracle.RefBlockTable([], 4)
    oracle.write_paged_kv(rk, rv, oracle.RefBlockAllocator(4), 0, rt, pos[0].tolist(), ke[:1], v[:1])
    assert table.block_ids == rt.block_ids
    assert_bits_equal(q_out, qe[:1], "paged rotated q")
    assert_bits_equal(pool.keys, rk, "paged keys")
    assert_bits_equal(pool.values, rv, "paged values")
    assert _ops.read_status(cuda) == _lib.OK
