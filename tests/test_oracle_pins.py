"""Pin the CPU oracle to the reference before trusting it (CPU only).

Two sources of truth, both from semioz/augur itself:
  * the known-answer cases written inline in the reference's tests
    (tests/test_kv_cache.py, tests/test_paged_kv_cache.py,
    tests/test_prefix_cache.py), restated here;
  * tests/golden/*.pt, produced by running the reference's own functions
    (tests/golden/make_golden.py) from 0xFF-poisoned caches.
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

from tests.conftest import assert_bits_equal, poison_


def _pool(shape, dtype):
    return poison_(torch.empty(shape, dtype=dtype))


# --- inline known answers of the reference's tests -------------------------


def test_allocator_reuses_freed_block(oracle):
    # reference tests/test_paged_kv_cache.py:16-29
    a = oracle.RefBlockAllocator(3)
    first, second = a.allocate(), a.allocate()
    assert (first, second) == (0, 1)
    a.free(first)
    assert a.allocate() == 0


def test_table_free_order_reallocates_in_order(oracle):
    # reference tests/test_paged_kv_cache.py:121-133
    a = oracle.RefBlockAllocator(4)
    t = oracle.RefBlockTable([], 4)
    t.ensure_position(8, a)
    assert t.block_ids == [0, 1, 2] and t.seq_len == 9
    t.free(a)
    assert [a.allocate(), a.allocate(), a.allocate()] == [0, 1, 2]


def test_position_to_block_offset(oracle):
    # reference tests/test_paged_kv_cache.py:136-141
    t = oracle.RefBlockTable([7, 1, 4], 4)
    assert t.position_to_block_offset(0) == (7, 0)
    assert t.position_to_block_offset(6) == (1, 2)
    assert t.position_to_block_offset(9) == (4, 1)


def test_prefix_hash_chain(oracle):
    # reference tests/test_paged_kv_cache.py:32-57
    blocks = {}
    h1 = oracle.ref_block_hash(None, [1, 2, 3, 4])
    blocks[(None, (1, 2, 3, 4))] = (h1, 7)
    assert oracle.ref_match_prefix(blocks, [1, 2, 3, 4, 5, 6], 4) == ([7], 4)
    h2 = oracle.ref_block_hash(h1, [5, 6, 7, 8])
    blocks[(h1, (5, 6, 7, 8))] = (h2, 9)
    assert oracle.ref_match_prefix(blocks, [1, 2, 3, 4, 5, 6, 7, 8, 99], 4) == ([7, 9], 8)
    assert oracle.ref_match_prefix(blocks, [1, 2, 3, 4, 5, 6], 4) == ([7], 4)


def test_paged_scatter_into_permuted_table(oracle):
    # reference tests/test_paged_kv_cache.py:168-202
    pk, pv = torch.zeros(2, 3, 1, 4, 2), torch.zeros(2, 3, 1, 4, 2)
    a = oracle.RefBlockAllocator(3)
    t = oracle.RefBlockTable([2, 0, 1], 4)
    key = torch.tensor([[[[10.0, 11.0], [20.0, 21.0], [30.0, 31.0]]]])
    value = torch.tensor([[[[110.0, 111.0], [120.0, 121.0], [130.0, 131.0]]]])
    oracle.write_paged_kv(pk, pv, a, 1, t, [3, 4, 9], key, value)
    rk, rv = oracle.read_paged_kv(pk, pv, 1, t, 10)
    assert torch.equal(pk[1, 2, :, 3, :], key[0, :, 0, :])
    assert torch.equal(pk[1, 0, :, 0, :], key[0, :, 1, :])
    assert torch.equal(pk[1, 1, :, 1, :], key[0, :, 2, :])
    assert torch.equal(rk[:, :, [3, 4, 9], :], key)
    assert torch.equal(rv[:, :, [3, 4, 9], :], value)


def test_paged_lazy_allocation(oracle):
    # reference tests/test_paged_kv_cache.py:205-236
    pk, pv = torch.zeros(2, 3, 1, 4, 2), torch.zeros(2, 3, 1, 4, 2)
    a = oracle.RefBlockAllocator(3)
    t = oracle.RefBlockTable([], 4)
    key = torch.tensor([[[[10.0, 11.0], [20.0, 21.0]]]])
    oracle.write_paged_kv(pk, pv, a, 1, t, [0, 4], key, key + 100)
    assert t.block_ids == [0, 1]
    assert torch.equal(pk[1, 0, :, 0, :], key[0, :, 0, :])
    assert torch.equal(pk[1, 1, :, 0, :], key[0, :, 1, :])


def test_paged_read_matches_contiguous(oracle):
    # reference tests/test_paged_kv_cache.py:239-320
    ck, cv = torch.zeros(2, 1, 1, 6, 2), torch.zeros(2, 1, 1, 6, 2)
    pk, pv = torch.zeros(2, 2, 1, 4, 2), torch.zeros(2, 2, 1, 4, 2)
    key = torch.arange(12, dtype=torch.float32).view(1, 1, 6, 2)
    value = torch.arange(100, 112, dtype=torch.float32).view(1, 1, 6, 2)
    pos = torch.tensor([[0, 1, 2, 3, 4, 5]])
    oracle.write_kv(ck, cv, 1, pos, key, value)
    t = oracle.RefBlockTable([1, 0], 4)
    oracle.write_paged_kv(pk, pv, oracle.RefBlockAllocator(2), 1, t, list(range(6)), key, value)
    rk, rv = oracle.read_paged_kv(pk, pv, 1, t, 6)
    assert torch.equal(rk, ck[1, :, :, :6, :])
    assert torch.equal(rv, cv[1, :, :, :6, :])


def test_write_kv_positions(oracle):
    # reference tests/test_kv_cache.py:71-97 (values at the written positions)
    ck, cv = torch.zeros(2, 1, 1, 4, 4), torch.zeros(2, 1, 1, 4, 4)
    g = torch.Generator().manual_seed(0)
    k1, v1 = torch.randn(1, 1, 3, 4, generator=g), torch.randn(1, 1, 3, 4, generator=g)
    k2, v2 = torch.randn(1, 1, 1, 4, generator=g), torch.randn(1, 1, 1, 4, generator=g)
    oracle.write_kv(ck, cv, 1, torch.tensor([[0, 1, 2]]), k1, v1)
    oracle.write_kv(ck, cv, 1, torch.tensor([[3]]), k2, v2)
    assert torch.equal(ck[1, :, :, :3], k1) and torch.equal(ck[1, :, :, 3:], k2)
    assert torch.equal(cv[1, :, :, :3], v1) and torch.equal(cv[1, :, :, 3:], v2)


def test_copy_prefix(oracle):
    # reference tests/test_prefix_cache.py:52-81
    ck, cv = torch.zeros(2, 1, 1, 5, 2), torch.zeros(2, 1, 1, 5, 2)
    ek = torch.arange(12, dtype=torch.float32).view(2, 1, 3, 2)
    ev = torch.arange(100, 112, dtype=torch.float32).view(2, 1, 3, 2)
    oracle.copy_prefix_into_cache(ek, ev, ck, cv, 0)
    assert torch.equal(ck[:, 0, :, :3, :], ek) and torch.equal(cv[:, 0, :, :3, :], ev)


# --- golden fixtures produced by the reference ------------------------------


@pytest.mark.parametrize("case", ["f32", "bf16", "f16"])
def test_golden_write_kv(oracle, golden, case):
    c = golden["write_kv"][case]
    L, B, H, S, D = c["cfg"]
    ck, cv = _pool((L, B, H, S, D), c["keys"].dtype), _pool((L, B, H, S, D), c["keys"].dtype)
    for call in c["calls"]:
        # recorded K/V are contiguous [B, H, S, D]; feed them token-major-strided like the reference saw
        oracle.write_kv(ck, cv, call["layer"], call["positions"], call["key"], call["value"])
    assert_bits_equal(ck, c["keys"], "keys")
    assert_bits_equal(cv, c["values"], "values")


def test_golden_paged(oracle, golden):
    for name, c in golden["paged"].items():
        dtype = c["keys"].dtype
        L, NB, H, bs, D = c["keys"].shape
        pk, pv = _pool(c["keys"].shape, dtype), _pool(c["keys"].shape, dtype)
        a = oracle.RefBlockAllocator(c["num_blocks"])
        t = oracle.RefBlockTable(c["initial_table"] or [], c["block_size"])
        for call in c["calls"]:
            err = None
            try:
                oracle.write_paged_kv(pk, pv, a, call["layer"], t, call["positions"], call["key"], call["value"])
            except (ValueError, RuntimeError) as exc:
                err = f"{type(exc).__name__}: {exc}"
            assert err == call["error"], name
            assert t.block_ids == call["block_ids"] and t.seq_len == call["seq_len"], name
        assert_bits_equal(pk, c["keys"], f"{name} keys")
        assert_bits_equal(pv, c["values"], f"{name} values")
        assert a.free_blocks == c["free_after"], name
        for layer, r in c["reads"].items():
            rk, rv = oracle.read_paged_kv(pk, pv, layer, t)
            assert_bits_equal(rk, r["key"], f"{name} read key {layer}")
            assert_bits_equal(rv, r["value"], f"{name} read value {layer}")


@pytest.mark.parametrize("case", ["bf16", "f32_to_bf16", "f32"])
def test_golden_prefix(oracle, golden, case):
    c = golden["prefix"][case]
    ck, cv = _pool(c["keys"].shape, c["keys"].dtype), _pool(c["keys"].shape, c["keys"].dtype)
    oracle.copy_prefix_into_cache(c["entry_keys"], c["entry_values"], ck, cv, c["batch_idx"])
    assert_bits_equal(ck, c["keys"], "keys")
    assert_bits_equal(cv, c["values"], "values")


def _handoff_runs(tables, lens, bs):
    runs = []
    for b, (ids, n) in enumerate(zip(tables, lens)):
        for j in range(-(-n // bs)):
            runs.append((b, j * bs, ids[j], 0, min(bs, n - j * bs)))
    return np.asarray(runs, dtype=np.int32)


def test_golden_handoff_runs_and_scatter(oracle, golden):
    c = golden["handoff"]
    src_k, src_v = c["src_keys"], c["src_values"]
    bs = c["keys"].shape[3]
    # as whole-block runs
    pk, pv = _pool(c["keys"].shape, src_k.dtype), _pool(c["keys"].shape, src_k.dtype)
    oracle.copy_runs(src_k, src_v, pk, pv, _handoff_runs(c["tables"], c["lens"], bs), threads=4)
    assert_bits_equal(pk, c["keys"], "runs keys")
    assert_bits_equal(pv, c["values"], "runs values")
    # as a slot scatter, one sequence (batch row) at a time
    pk2, pv2 = _pool(c["keys"].shape, src_k.dtype), _pool(c["keys"].shape, src_k.dtype)
    for b, (ids, n) in enumerate(zip(c["tables"], c["lens"])):
        pos = np.arange(n)
        slots = np.asarray(ids, np.int64)[pos // bs] * bs + pos % bs
        tok_k = src_k[:, b, :, :n, :].permute(0, 2, 1, 3).contiguous()  # [L, n, H, D]
        tok_v = src_v[:, b, :, :n, :].permute(0, 2, 1, 3).contiguous()
        oracle.scatter_slots(tok_k, tok_v, slots, pk2, pv2, bs, threads=3)
    assert_bits_equal(pk2, c["keys"], "scatter keys")
    assert_bits_equal(pv2, c["values"], "scatter values")


def test_golden_fork_with_cow(oracle, golden):
    """Shared prefix blocks + copy-on-write of the partial block == private per-fork writes."""
    c = golden["fork"]
    P, S = c["prefix_len"], c["suffix_len"]
    pk_in, pv_in = c["prefix_keys"], c["prefix_values"]
    L, _, H, _, D = pk_in.shape
    bs, NB = 4, 32
    pk, pv = _pool((L, NB, H, bs, D), pk_in.dtype), _pool((L, NB, H, bs, D), pk_in.dtype)
    a = oracle.RefBlockAllocator(NB)
    parent = oracle.RefBlockTable([], bs)
    for layer in range(L):
        oracle.write_paged_kv(pk, pv, a, layer, parent, list(range(P)), pk_in[layer], pv_in[layer])
    for f, per_layer in enumerate(c["reads"]):
        t = oracle.RefBlockTable(list(parent.block_ids), bs, parent.seq_len)
        # copy-on-write: the last prefix block is partial and shared
        new = a.allocate()
        runs = np.asarray([(t.block_ids[-1], 0, new, 0, P % bs)], dtype=np.int32)
        oracle.copy_runs(pk, pv, pk, pv, runs)
        t.block_ids[-1] = new
        for layer in range(L):
            oracle.write_paged_kv(pk, pv, a, layer, t, list(range(P, P + S)),
                                  c["suffix_keys"][f, layer], c["suffix_values"][f, layer])
        for layer in range(L):
            rk, rv = oracle.read_paged_kv(pk, pv, layer, t)
            assert_bits_equal(rk, per_layer[layer]["key"], f"fork {f} layer {layer} key")
            assert_bits_equal(rv, per_layer[layer]["value"], f"fork {f} layer {layer} value")


def test_golden_bookkeeping(oracle, golden):
    log = dict((entry[0], entry[1:]) for entry in golden["bookkeeping"])
    a = oracle.RefBlockAllocator(12)
    got = [a.allocate() for _ in range(4)]
    assert got == log["allocate4"][0]
    a.free(got[1])
    a.free(got[3])
    assert a.free_blocks == log["after_free_1_3"][0]
    assert [a.allocate() for _ in range(3)] == log["allocate3"][0]
    t = oracle.RefBlockTable([], 4)
    t.ensure_position(13, a)
    assert (t.block_ids, t.seq_len) == tuple(log["ensure13"])
    t.free(a)
    assert a.free_blocks == log["free_table"][0]
    h1 = oracle.ref_block_hash(None, [1, 2, 3, 4])
    h2 = oracle.ref_block_hash(h1, [5, 6, 7, 8])
    h3 = oracle.ref_block_hash(h2, [9, 10, 11, 12])
    hx = oracle.ref_block_hash(None, [5, 6, 7, 8])
    assert [h1, h2, h3, hx] == log["hashes"][0]


def test_golden_config1_replay(oracle, config1_golden):
    """Replaying the reference's recorded write_kv calls reproduces its final cache bytes."""
    c = config1_golden
    L, T, H, D = c["keys"].shape
    ck, cv = _pool((L, 1, H, c["max_seq_len"], D), torch.float32), _pool((L, 1, H, c["max_seq_len"], D), torch.float32)
    off = 0
    for n in c["call_sizes"]:
        for layer in range(L):
            pos = c["positions"][layer, off : off + n].unsqueeze(0)
            k = c["keys"][layer, off : off + n].permute(1, 0, 2).unsqueeze(0)
            v = c["values"][layer, off : off + n].permute(1, 0, 2).unsqueeze(0)
            oracle.write_kv(ck, cv, layer, pos, k, v)
        off += n
    assert c["seq_len"] == 160
    assert hashlib.sha256(ck.numpy().tobytes()).hexdigest() == c["sha256_keys"]
    assert hashlib.sha256(cv.numpy().tobytes()).hexdigest() == c["sha256_values"]


@pytest.mark.parametrize("case", ["f32", "bf16"])
def test_golden_decode_attention(oracle, golden, case):
    """The oracle's attention equals the reference's own attention() on its paged cache."""
    c = golden["attention"][case]
    got = oracle.decode_attention(c["q"], c["k"], c["v"])
    assert_bits_equal(got, c["out"], "attention output")


# --- RoPE fused with the cache write ----------------------------------------


@pytest.mark.parametrize("case", ["f32", "bf16", "f16"])
def test_golden_rope_far_positions(oracle, golden, case):
    """apply_rope restated, from the reference's formula and from a position-indexed
    table, equals the reference's apply_rope bit for bit, large angles included."""
    c = golden["rope"][f"far_{case}"]
    dt = c["q"].dtype
    for table in (None, oracle.rope_table(64, c["theta"], 32768, dt)):
        q, k = oracle.apply_rope(c["q"], c["k"], c["position_ids"], c["theta"], table=table)
        assert_bits_equal(q, c["q_embed"], "q")
        assert_bits_equal(k, c["k_embed"], "k")


@pytest.mark.parametrize("case", ["f32", "bf16", "f16"])
def test_golden_rope_then_write_paged_kv(oracle, golden, case):
    """apply_rope then write_paged_kv, replayed on the oracle from the recorded inputs,
    reproduces the reference's pool blocks, block table and rotated q."""
    c = golden["rope"][f"paged_{case}"]
    dt = c["calls"][0]["q"].dtype
    pk, pv = _pool((1, c["num_blocks"], 2, 16, 64), dt), _pool((1, c["num_blocks"], 2, 16, 64), dt)
    alloc = oracle.RefBlockAllocator(c["num_blocks"])
    for _ in range(c["prior_allocated"]):
        alloc.allocate()
    table = oracle.RefBlockTable([], 16)
    for call in c["calls"]:
        q, k = oracle.apply_rope(call["q"], call["k"], call["position_ids"], c["theta"])
        assert_bits_equal(q, call["q_embed"], "q")
        oracle.write_paged_kv(pk, pv, alloc, 0, table, call["position_ids"][0].tolist(), k, call["v"])
    assert table.block_ids == c["block_ids"]
    assert_bits_equal(pk[:, c["touched_blocks"]], c["keys"], "keys")
    assert_bits_equal(pv[:, c["touched_blocks"]], c["values"], "values")


@pytest.mark.parametrize("case", ["f32", "bf16"])
def test_golden_duplicate_positions(oracle, golden, case):
    """A position given twice in one call: the reference keeps the later token's K/V, in
    write_kv (per-row index_put) and in write_paged_kv (per-token loop); so does the oracle."""
    c = golden["duplicates"][f"write_kv_{case}"]
    L, B, H, S, D = c["cfg"]
    ck, cv = _pool((L, B, H, S, D), c["keys"].dtype), _pool((L, B, H, S, D), c["keys"].dtype)
    oracle.write_kv(ck, cv, c["layer"], c["positions"], c["key"], c["value"])
    assert_bits_equal(ck, c["keys"], "write_kv keys")
    assert_bits_equal(cv, c["values"], "write_kv values")
    # the later duplicate is the one the reference kept
    b, s_late = 1, 4  # row 1 writes position 0 at tokens 0, 1, 2 and 4
    assert_bits_equal(c["keys"][c["layer"], b, :, 0], c["key"][b, :, s_late], "last duplicate kept")
    p = golden["duplicates"][f"write_paged_kv_{case}"]
    pk, pv = _pool(p["keys"].shape, p["keys"].dtype), _pool(p["keys"].shape, p["keys"].dtype)
    a = oracle.RefBlockAllocator(p["num_blocks"])
    t = oracle.RefBlockTable([], p["block_size"])
    oracle.write_paged_kv(pk, pv, a, p["layer"], t, p["positions"][0].tolist(), p["key"], p["value"])
    assert t.block_ids == p["block_ids"] and t.seq_len == p["seq_len"]
    assert_bits_equal(pk, p["keys"], "write_paged_kv keys")
    assert_bits_equal(pv, p["values"], "write_paged_kv values")


def test_torch_loop_write_paged_kv_matches_golden(oracle, golden):
    """The torch-loop restatement (timed as the reference's own CPU path) writes what the
    reference wrote, including the duplicate-position case."""
    for name in ("bf16", "f32"):
        p = golden["duplicates"][f"write_paged_kv_{name}"]
        pk, pv = _pool(p["keys"].shape, p["keys"].dtype), _pool(p["keys"].shape, p["keys"].dtype)
        a = oracle.RefBlockAllocator(p["num_blocks"])
        t = oracle.RefBlockTable([], p["block_size"])
        oracle.write_paged_kv_torch_loop(pk, pv, a, p["layer"], t, p["positions"], p["key"], p["value"])
        assert t.block_ids == p["block_ids"]
        assert_bits_equal(pk, p["keys"], f"{name} keys")
        assert_bits_equal(pv, p["values"], f"{name} values")


@pytest.mark.parametrize("case", ["f32_prefix", "bf16_prefix", "bf16_plain"])
def test_golden_prefill_attention(oracle, golden, case):
    """The oracle's prefill attention (causal mask with past_len = key_len - query_len)
    equals the reference's own attention() for a call of several new tokens on a paged
    cache, with and without a cached prefix; its gather equals read_paged_kv's."""
    c = golden["prefill_attention"][case]
    t = oracle.RefBlockTable(c["block_ids"], 16, c["seq_len"])
    kk, vv = oracle.read_paged_kv(c["keys"], c["values"], 0, t)
    assert_bits_equal(kk, c["k"], "gathered keys")
    assert_bits_equal(vv, c["v"], "gathered values")
    got = oracle.prefill_attention(c["q"], kk, vv)
    assert_bits_equal(got, c["out"], "attention output")
