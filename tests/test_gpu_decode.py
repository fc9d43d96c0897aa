"""Batched paged decode layer vs the reference's per-sequence paged branch.

For each sequence the oracle runs what augur/attention.py:53-86 runs with a
paged cache for its new token: apply_rope, write_paged_kv, read_paged_kv, the
GQA repeat and the attention. The pool must match bit for bit; the attention
output within the bf16 tolerance of the decode-attention tests.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import augur_b200 as ab
from augur_b200 import _lib, _ops, batched
from augur_b200.decode import DecodeStep, paged_decode_layer
from tests.conftest import assert_bits_equal, poison_

pytestmark = pytest.mark.gpu

THETA = 1000000.0


@pytest.mark.parametrize("path", ["prepared", "general", "mixed", "side"])
def test_decode_layers_match_the_reference_branch(cuda, oracle, path):
    """path: the step's prepared launches, the general wrappers (an explicit stream), or
    both in one step (a later layer's q is a strided view, which the prepared arguments
    do not describe, so that layer takes the general path); side: the prepared launches
    with another stream current than the one the step uploaded its arrays on (they wait
    for the upload, and through it for the prompt writes before it)."""
    L, H, Hq, D, bs, NB = 2, 2, 14, 64, 16, 64
    prior = [0, 1, 15, 16, 300]
    g = torch.Generator().manual_seed(12)
    pool = ab.PagedKVCache(keys=poison_(torch.empty(L, NB, H, bs, D, dtype=torch.bfloat16, device=cuda)),
                           values=poison_(torch.empty(L, NB, H, bs, D, dtype=torch.bfloat16, device=cuda)),
                           block_size=bs, allocator=ab.BlockAllocator(NB))
    rk = poison_(torch.empty(L, NB, H, bs, D, dtype=torch.bfloat16))
    rv = poison_(torch.empty(L, NB, H, bs, D, dtype=torch.bfloat16))
    # the prompts, written through the batched scatter on the device and by the oracle
    tables = [ab.SequenceBlockTable.empty(bs) for _ in prior]
    sm = batched.prefill_slot_mapping(tables, prior, pool.allocator)
    T = sum(prior)
    pk = torch.randn(L, T, H, D, generator=g).to(torch.bfloat16)
    pv = torch.randn(L, T, H, D, generator=g).to(torch.bfloat16)
    flat = np.concatenate([sm[b, :n] for b, n in enumerate(prior)])
    batched.write_paged_kv_batch(pool, pk.to(cuda), pv.to(cuda), torch.from_numpy(flat).to(cuda))
    oracle.scatter_slots(pk, pv, flat, rk, rv, bs)
    ref_tables = [oracle.RefBlockTable(list(t.block_ids), bs, t.seq_len) for t in tables]
    ref_alloc = oracle.RefBlockAllocator(NB)
    for _ in range(NB - len(pool.allocator._free_blocks)):
        ref_alloc.allocate()  # the same blocks are taken on both sides

    step = DecodeStep(pool, tables)
    for layer in range(L):
        q = torch.randn(len(prior), Hq, 1, D, generator=g).to(torch.bfloat16)
        k = torch.randn(len(prior), H, 1, D, generator=g).to(torch.bfloat16)
        v = torch.randn(len(prior), H, 1, D, generator=g).to(torch.bfloat16)
        stream = torch.cuda.current_stream(cuda) if path == "general" else None
        qd = q.to(cuda)
        if path == "mixed" and layer == 1:
            wide = torch.empty(len(prior), Hq, 2, D, dtype=torch.bfloat16, device=cuda)
            wide[:, :, :1] = qd
            qd = wide[:, :, :1]
            assert qd.stride() != q.stride()
        if path == "side":
            side = torch.cuda.Stream(cuda)
            with torch.cuda.stream(side):
                out = paged_decode_layer(step, pool, layer, qd, k.to(cuda), v.to(cuda), THETA)
            torch.cuda.current_stream(cuda).wait_stream(side)
        else:
            out = paged_decode_layer(step, pool, layer, qd, k.to(cuda), v.to(cuda), THETA, stream=stream)
        assert out.shape == (len(prior), Hq, 1, D)
        for b, n in enumerate(prior):
            pos = torch.tensor([[n]])
            qe, ke = oracle.apply_rope(q[b : b + 1], k[b : b + 1], pos, THETA)
            rt = ref_tables[b]
            if layer == 0:
                oracle.write_paged_kv(rk, rv, ref_alloc, layer, rt, [n], ke, v[b : b + 1])
            else:
                blk, off = rt.block_ids[n // bs], n % bs
                rk[layer, blk, :, off] = ke[0, :, 0]
                rv[layer, blk, :, off] = v[b, :, 0]
            kk, vv = oracle.read_paged_kv(rk, rv, layer, oracle.RefBlockTable(rt.block_ids, bs, n + 1))
            want = oracle.decode_attention(qe, kk, vv)[0, :, 0, :]
            torch.testing.assert_close(out[b, :, 0].float().cpu(), want.float(), rtol=1e-2, atol=1e-2,
                                       msg=f"layer {layer} seq {b}")
    assert [t.block_ids for t in tables] == [rt.block_ids for rt in ref_tables]
    assert [t.seq_len for t in tables] == [n + 1 for n in prior]
    assert_bits_equal(pool.keys, rk, "pool keys")
    assert_bits_equal(pool.values, rv, "pool values")
    assert _ops.read_status(cuda) == _lib.OK


@pytest.mark.parametrize("early", [False, True])
def test_graph_step_replays_match_eager_steps(cuda, early):
    """A CUDA graph captured once over DecodeGraphStep.layer calls, replayed after each
    update(), gives the eager DecodeStep results: the same pool bits, the same block tables,
    attention outputs within the bf16 tolerance (the launch plan sees the step's capacity
    instead of its longest sequence); padding rows write nothing and return zeros.
    early: the graph's layers read lengths, tables and pool before the previous layer's
    launch has finished."""
    from augur_b200.decode import DecodeGraphStep

    L, H, Hq, D, bs, NB = 2, 2, 14, 64, 16, 96
    prior = [0, 1, 15, 16, 300]
    cap_seqs, max_blocks = 6, 24
    g = torch.Generator().manual_seed(31)

    def fresh():
        pool = ab.PagedKVCache(keys=poison_(torch.empty(L, NB, H, bs, D, dtype=torch.bfloat16, device=cuda)),
                               values=poison_(torch.empty(L, NB, H, bs, D, dtype=torch.bfloat16, device=cuda)),
                               block_size=bs, allocator=ab.BlockAllocator(NB))
        tables = [ab.SequenceBlockTable.empty(bs) for _ in prior]
        return pool, tables

    pool_e, tabs_e = fresh()
    pool_g, tabs_g = fresh()
    T = sum(prior)
    pk = torch.randn(L, T, H, D, generator=g).to(torch.bfloat16).to(cuda)
    pv = torch.randn(L, T, H, D, generator=g).to(torch.bfloat16).to(cuda)
    for pool, tabs in ((pool_e, tabs_e), (pool_g, tabs_g)):
        sm = batched.prefill_slot_mapping(tabs, prior, pool.allocator)
        flat = np.concatenate([sm[b, :n] for b, n in enumerate(prior)])
        batched.write_paged_kv_batch(pool, pk, pv, torch.from_numpy(flat).to(cuda))
    B = len(prior)
    steps = 3
    qs = torch.randn(steps, L, B, Hq, 1, D, generator=g).to(torch.bfloat16).to(cuda)
    ks = torch.randn(steps, L, B, H, 1, D, generator=g).to(torch.bfloat16).to(cuda)
    vs = torch.randn(steps, L, B, H, 1, D, generator=g).to(torch.bfloat16).to(cuda)

    # static inputs of the graph: rows past B are padding
    q_in = torch.zeros(L, cap_seqs, Hq, 1, D, dtype=torch.bfloat16, device=cuda)
    k_in = torch.zeros(L, cap_seqs, H, 1, D, dtype=torch.bfloat16, device=cuda)
    v_in = torch.zeros(L, cap_seqs, H, 1, D, dtype=torch.bfloat16, device=cuda)
    gs = DecodeGraphStep(pool_g, cap_seqs, max_blocks, Hq, THETA, early_reads=early)
    graph = torch.cuda.CUDAGraph()
    cs = torch.cuda.Stream(cuda)
    cs.wait_stream(torch.cuda.current_stream(cuda))
    outs_g = None
    for s in range(steps):
        # eager reference step
        step = DecodeStep(pool_e, tabs_e)
        outs_e = [paged_decode_layer(step, pool_e, layer, qs[s, layer], ks[s, layer], vs[s, layer], THETA)
                  for layer in range(L)]
        # graph step
        with torch.cuda.stream(cs):
            q_in[:, :B].copy_(qs[s])
            k_in[:, :B].copy_(ks[s])
            v_in[:, :B].copy_(vs[s])
            gs.update(tabs_g)
            if s == 0:
                with torch.cuda.graph(graph, stream=cs):
                    outs_g = [gs.layer(layer, q_in[layer], k_in[layer], v_in[layer]) for layer in range(L)]
            graph.replay()
        torch.cuda.synchronize(cuda)
        for layer in range(L):
            torch.testing.assert_close(outs_g[layer][:B].float(), outs_e[layer].float(), rtol=1e-2, atol=1e-2,
                                       msg=f"step {s} layer {layer}")
            assert int(outs_g[layer][B:].abs().sum()) == 0, "padding rows must return zeros"
    graph.reset()
    assert [t.block_ids for t in tabs_g] == [t.block_ids for t in tabs_e]
    assert [t.seq_len for t in tabs_g] == [n + steps for n in prior]
    assert_bits_equal(pool_g.keys, pool_e.keys.cpu(), "pool keys")
    assert_bits_equal(pool_g.values, pool_e.values.cpu(), "pool values")
    assert _ops.read_status(cuda) == _lib.OK


def test_graph_step_rows_follow_reordered_batches(cuda):
    """DecodeGraphStep keeps each staging row of the block tables until that row's block ids
    change. The same captured step, replayed after the batch's sequences change rows from
    step to step, matches eager steps in the same order: the same pool bits, outputs within
    the bf16 tolerance."""
    from augur_b200.decode import DecodeGraphStep

    L, H, Hq, D, bs, NB = 2, 2, 14, 64, 16, 96
    prior = [3, 15, 16, 40, 300]
    orders = [[0, 1, 2, 3, 4], [4, 0, 1, 2, 3], [2, 4, 0, 3, 1], [2, 4, 0, 3, 1], [1, 0, 4, 2, 3]]
    g = torch.Generator().manual_seed(57)

    def fresh():
        pool = ab.PagedKVCache(keys=poison_(torch.empty(L, NB, H, bs, D, dtype=torch.bfloat16, device=cuda)),
                               values=poison_(torch.empty(L, NB, H, bs, D, dtype=torch.bfloat16, device=cuda)),
                               block_size=bs, allocator=ab.BlockAllocator(NB))
        return pool, [ab.SequenceBlockTable.empty(bs) for _ in prior]

    (pool_e, tabs_e), (pool_g, tabs_g) = fresh(), fresh()
    T = sum(prior)
    pk = torch.randn(L, T, H, D, generator=g).to(torch.bfloat16).to(cuda)
    pv = torch.randn(L, T, H, D, generator=g).to(torch.bfloat16).to(cuda)
    for pool, tabs in ((pool_e, tabs_e), (pool_g, tabs_g)):
        sm = batched.prefill_slot_mapping(tabs, prior, pool.allocator)
        flat = np.concatenate([sm[b, :n] for b, n in enumerate(prior)])
        batched.write_paged_kv_batch(pool, pk, pv, torch.from_numpy(flat).to(cuda))
    B = len(prior)
    q_in = torch.zeros(L, B, Hq, 1, D, dtype=torch.bfloat16, device=cuda)
    k_in = torch.zeros(L, B, H, 1, D, dtype=torch.bfloat16, device=cuda)
    v_in = torch.zeros(L, B, H, 1, D, dtype=torch.bfloat16, device=cuda)
    gs = DecodeGraphStep(pool_g, B, 24, Hq, THETA)
    graph = torch.cuda.CUDAGraph()
    cs = torch.cuda.Stream(cuda)
    cs.wait_stream(torch.cuda.current_stream(cuda))
    outs_g = None
    for s, order in enumerate(orders):
        q = torch.randn(L, B, Hq, 1, D, generator=g).to(torch.bfloat16).to(cuda)
        k = torch.randn(L, B, H, 1, D, generator=g).to(torch.bfloat16).to(cuda)
        v = torch.randn(L, B, H, 1, D, generator=g).to(torch.bfloat16).to(cuda)
        step = DecodeStep(pool_e, [tabs_e[i] for i in order])
        outs_e = [paged_decode_layer(step, pool_e, layer, q[layer], k[layer], v[layer], THETA) for layer in range(L)]
        with torch.cuda.stream(cs):
            q_in.copy_(q)
            k_in.copy_(k)
            v_in.copy_(v)
            gs.update([tabs_g[i] for i in order])
            if s == 0:
                with torch.cuda.graph(graph, stream=cs):
                    outs_g = [gs.layer(layer, q_in[layer], k_in[layer], v_in[layer]) for layer in range(L)]
            graph.replay()
        torch.cuda.synchronize(cuda)
        for layer in range(L):
            torch.testing.assert_close(outs_g[layer].float(), outs_e[layer].float(), rtol=1e-2, atol=1e-2,
                                       msg=lambda m, s=s, layer=layer: f"step {s} layer {layer}: {m}")
    graph.reset()
    assert [t.block_ids for t in tabs_g] == [t.block_ids for t in tabs_e]
    assert_bits_equal(pool_g.keys, pool_e.keys.cpu(), "pool keys")
    assert_bits_equal(pool_g.values, pool_e.values.cpu(), "pool values")
    assert _ops.read_status(cuda) == _lib.OK


def test_graph_step_rejects_what_it_cannot_describe(cuda):
    from augur_b200.decode import DecodeGraphStep

    pool = ab.PagedKVCache(keys=torch.zeros(1, 8, 2, 16, 64, dtype=torch.bfloat16, device=cuda),
                           values=torch.zeros(1, 8, 2, 16, 64, dtype=torch.bfloat16, device=cuda),
                           block_size=16, allocator=ab.BlockAllocator(8))
    gs = DecodeGraphStep(pool, 2, 2, 14, THETA)
    with pytest.raises(ValueError, match="at most 2 sequences"):
        gs.update([ab.SequenceBlockTable.empty(16) for _ in range(3)])
    full = ab.SequenceBlockTable.empty(16)
    full.seq_len = 32
    with pytest.raises(ValueError, match="capacity of 32 positions"):
        gs.update([full])
    with pytest.raises(ValueError, match="contiguous"):
        gs.layer(0, torch.zeros(2, 14, 1, 64, dtype=torch.float16, device=cuda),
                 torch.zeros(2, 2, 1, 64, dtype=torch.bfloat16, device=cuda),
                 torch.zeros(2, 2, 1, 64, dtype=torch.bfloat16, device=cuda))


@pytest.mark.parametrize("early", [False, True])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("head_dim", [64, 128])
def test_fused_decode_layer_matches_separate_launches(cuda, dtype, head_dim, early):
    """augur_kv_decode_layer rotates q and the new k inside the attention launch and writes
    the new k / v rows itself (bf16 / fp16); the general path runs the RoPE write and the
    attention as two launches. Both must leave the same pool bits and return the same
    outputs bit for bit, step after step. float32 takes the two-launch form in both.
    early: the prepared layers read lengths, tables and pool rows before the previous
    layer's launch has finished (the new token's row after it); the two-launch form drops
    the early reads."""
    L, H, Hq, bs, NB = 4, 2, 14, 16, 96
    prior = [1, 15, 16, 47, 300]
    g = torch.Generator().manual_seed(77)

    def setup():
        pool = ab.PagedKVCache(keys=poison_(torch.empty(L, NB, H, bs, head_dim, dtype=dtype, device=cuda)),
                               values=poison_(torch.empty(L, NB, H, bs, head_dim, dtype=dtype, device=cuda)),
                               block_size=bs, allocator=ab.BlockAllocator(NB))
        tables = [ab.SequenceBlockTable.empty(bs) for _ in prior]
        return pool, tables

    pools = [setup(), setup()]
    T = sum(prior)
    pk = torch.randn(L, T, H, head_dim, generator=g).to(dtype).to(cuda)
    pv = torch.randn(L, T, H, head_dim, generator=g).to(dtype).to(cuda)
    for pool, tables in pools:
        sm = batched.prefill_slot_mapping(tables, prior, pool.allocator)
        flat = np.concatenate([sm[b, :n] for b, n in enumerate(prior)])
        batched.write_paged_kv_batch(pool, pk, pv, torch.from_numpy(flat).to(cuda))
    B = len(prior)
    for s in range(3):
        q = torch.randn(L, B, Hq, 1, head_dim, generator=g).to(dtype).to(cuda)
        k = torch.randn(L, B, H, 1, head_dim, generator=g).to(dtype).to(cuda)
        v = torch.randn(L, B, H, 1, head_dim, generator=g).to(dtype).to(cuda)
        outs = []
        for i, (pool, tables) in enumerate(pools):
            step = DecodeStep(pool, tables, early_reads=early and i == 0)
            stream = torch.cuda.current_stream(cuda) if i == 1 else None
            outs.append([paged_decode_layer(step, pool, layer, q[layer], k[layer], v[layer], THETA, stream=stream)
                         for layer in range(L)])
            if i == 0:  # the prepared call: one launch per layer when the attention kernel fuses the write
                assert step._fast[4].launches == (2 if dtype == torch.float32 else 1)
        torch.cuda.synchronize(cuda)
        for layer in range(L):
            assert_bits_equal(outs[0][layer], outs[1][layer], f"step {s} layer {layer} output")
    assert_bits_equal(pools[0][0].keys, pools[1][0].keys, "pool keys")
    assert_bits_equal(pools[0][0].values, pools[1][0].values, "pool values")
    assert _ops.read_status(cuda) == _lib.OK


@pytest.mark.parametrize("field", ["positions", "slots"])
def test_fused_decode_layer_flags_positions_or_slots_off_the_table(cuda, field):
    """The one-launch layer takes each new token's position from seq_len - 1 and its slot
    from the block table; a caller's positions or slots that disagree are reported as
    AUGUR_KV_EBOUNDS (the kernel still writes where the table says)."""
    L, H, Hq, D, bs, NB = 1, 2, 14, 64, 16, 32
    pool = ab.PagedKVCache(keys=torch.zeros(L, NB, H, bs, D, dtype=torch.bfloat16, device=cuda),
                           values=torch.zeros(L, NB, H, bs, D, dtype=torch.bfloat16, device=cuda),
                           block_size=bs, allocator=ab.BlockAllocator(NB))
    tables = [ab.SequenceBlockTable.empty(bs) for _ in range(3)]
    batched.prefill_slot_mapping(tables, [5, 16, 40], pool.allocator)
    g = torch.Generator(device=cuda).manual_seed(3)
    q = torch.randn(3, Hq, 1, D, generator=g, device=cuda).to(torch.bfloat16)
    k = torch.randn(3, H, 1, D, generator=g, device=cuda).to(torch.bfloat16)
    _ops.read_status(cuda)
    step = DecodeStep(pool, tables)
    assert step.layer(pool, 0, q, k, k, THETA) is not None
    torch.cuda.synchronize()
    assert _ops.read_status(cuda) == _lib.OK  # consistent step: no report
    getattr(step, field)[1] += 1  # sequence 1's position or slot no longer matches its table
    assert step.layer(pool, 0, q, k, k, THETA) is not None
    torch.cuda.synchronize()
    assert _ops.read_status(cuda) == _lib.EBOUNDS
