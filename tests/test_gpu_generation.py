"""Batched paged generation against the reference's batch-1 paged path, sequence by sequence.

augur runs its paged branch for a batch of one and refuses a prefix cache
under the paged backend (augur/generation.py:35-40): each request prefills its
whole prompt (augur/attention.py:53-86: apply_rope, write_paged_kv,
read_paged_kv, attention) and then decodes token by token. Here the same
requests run as one batch through the repo's entry points:
  * PagedSequences admits the prompts; later prompts share the first one's
    cached full blocks, and one prompt is forked (its half-full last block is
    copied on the forks' first step);
  * each prompt's new tokens go through the fused RoPE write
    (write_paged_kv_batch_rope) and the prefill attention reading the pool in
    place (paged_prefill_attention);
  * every decode step is one fused RoPE append + attention launch per layer
    (DecodeStep / paged_decode_layer) for the whole batch, across block
    boundaries.
The oracle runs every sequence alone on a private table, as the reference
would. The K/V each sequence reads back must equal the reference's bit for
bit; the prefill and decode attention outputs agree within the bf16
tolerance (1e-2), as the kernels sum in another order.
"""

from __future__ import annotations

import pytest
import torch

import augur_b200 as ab
from augur_b200 import _lib, _ops
from augur_b200.attention import paged_prefill_attention
from augur_b200.decode import paged_decode_layer
from augur_b200.rope import write_paged_kv_batch_rope
from augur_b200.sequences import PagedSequences
from tests.conftest import assert_bits_equal, poison_

pytestmark = pytest.mark.gpu

L, H, HQ, D, BS, NB = 2, 2, 14, 64, 16, 256
THETA = 1000000.0
DT = torch.bfloat16
PREFIX = list(range(1000, 1040))  # 2 full blocks + 8 tokens
PROMPTS = [PREFIX + list(range(7)), PREFIX + list(range(200, 233)), PREFIX[:35], PREFIX + list(range(300, 320))]
N_FORKS = 2  # of the last prompt (60 tokens: its last block holds 12 of 16 rows)
STEPS = 20


def _qkv(tokens: list[int], layer: int):
    """q [HQ, D], k / v [H, D] of the last of `tokens` in one layer: a function of the tokens
    so far, as a causal model's are, so shared prefixes have equal K/V."""
    g = torch.Generator().manual_seed((hash(tuple(tokens)) * 31 + layer) & 0x7FFFFFFF)
    return (torch.randn(HQ, D, generator=g).to(DT), torch.randn(H, D, generator=g).to(DT),
            torch.randn(H, D, generator=g).to(DT))


def _new_token(i: int, step: int) -> int:
    return 5000 + 101 * i + step


def _device_run(cuda, early: bool):
    pool = ab.PagedKVCache(keys=poison_(torch.empty(L, NB, H, BS, D, dtype=DT, device=cuda)),
                           values=poison_(torch.empty(L, NB, H, BS, D, dtype=DT, device=cuda)),
                           block_size=BS, allocator=ab.BlockAllocator(NB))
    seqs = PagedSequences(pool)
    ids, prefill = [], {}
    for toks in PROMPTS:
        adm = seqs.admit(toks)
        n0 = adm.cached_tokens
        slots = torch.from_numpy(adm.slots).to(cuda)
        positions = torch.arange(n0, len(toks), device=cuda)
        table = seqs.tables[adm.seq_id]
        outs = []
        for layer in range(L):
            qkv = [_qkv(toks[: p + 1], layer) for p in range(n0, len(toks))]
            q, k, v = (torch.stack([x[j] for x in qkv]).to(cuda) for j in range(3))
            q_rot = write_paged_kv_batch_rope(pool, q, k, v, slots, positions, THETA, layer,
                                              max_position=len(toks) - 1)
            outs.append(paged_prefill_attention(q_rot, pool, layer, [table], [len(toks) - n0]))
        prefill[adm.seq_id] = (n0, outs)
        seqs.publish_prefix(adm.seq_id)
        ids.append(adm.seq_id)
    assert [prefill[s][0] for s in ids] == [0, 32, 32, 32], "later prompts share the prefix's 2 full blocks"
    ids += seqs.fork(ids[-1], N_FORKS)
    tokens = {sid: list(seqs.prompts[sid]) for sid in ids}
    decode = []
    for st in range(STEPS):
        for i, sid in enumerate(ids):
            tokens[sid].append(_new_token(i, st))
        step = seqs.decode_step(ids, early_reads=early)
        assert seqs.last_cow_blocks == (N_FORKS if st == 0 else 0)
        outs = []
        for layer in range(L):
            qkv = [_qkv(tokens[sid], layer) for sid in ids]
            q, k, v = (torch.stack([x[j] for x in qkv]).unsqueeze(2).to(cuda) for j in range(3))
            outs.append(paged_decode_layer(step, pool, layer, q, k, v, THETA))
        decode.append(outs)
    gathered = {sid: [ab.read_paged_kv(pool, layer, seqs.tables[sid]) for layer in range(L)] for sid in ids}
    torch.cuda.synchronize(cuda)
    assert _ops.read_status(cuda) == _lib.OK
    prompts = {sid: seqs.prompts[sid] for sid in ids}
    for sid in ids:
        seqs.release(sid)
    seqs.evict_prefixes()
    assert pool.allocator.num_free == NB, "every block returns to the pool"
    return ids, prompts, prefill, decode, gathered


@pytest.mark.parametrize("early", [False, True])
def test_batched_generation_matches_the_reference_one_sequence_at_a_time(cuda, oracle, early):
    """early: every decode layer reads lengths, tables and pool rows before the launch ahead
    of it has finished (the new tokens' rows after it)."""
    ids, prompts, prefill, decode, gathered = _device_run(cuda, early)
    NBR = 512
    rk = poison_(torch.empty(L, NBR, H, BS, D, dtype=DT))
    rv = poison_(torch.empty(L, NBR, H, BS, D, dtype=DT))
    alloc = oracle.RefBlockAllocator(NBR)
    for i, sid in enumerate(ids):
        toks = list(prompts[sid])
        table = oracle.RefBlockTable([], BS)
        n = len(toks)
        # the reference's prompt call: every prompt token (no prefix cache under the paged backend)
        for layer in range(L):
            qkv = [_qkv(toks[: p + 1], layer) for p in range(n)]
            q, k, v = (torch.stack([x[j] for x in qkv], 1).unsqueeze(0) for j in range(3))  # [1, heads, n, D]
            qe, ke = oracle.apply_rope(q, k, torch.arange(n).unsqueeze(0), THETA)
            oracle.write_paged_kv(rk, rv, alloc, layer, table, list(range(n)), ke, v)
            kk, vv = oracle.read_paged_kv(rk, rv, layer, table)
            want = oracle.prefill_attention(qe, kk, vv)[0].transpose(0, 1)  # [n, HQ, D]
            if sid in prefill:  # forks have no prompt call of their own on the device
                n0, outs = prefill[sid]
                torch.testing.assert_close(outs[layer].float().cpu(), want[n0:].float(), rtol=1e-2, atol=1e-2,
                                           msg=lambda m, sid=sid, layer=layer: f"prefill seq {sid} layer {layer}: {m}")
        for st in range(STEPS):
            toks.append(_new_token(i, st))
            pos = len(toks) - 1
            for layer in range(L):
                q, k, v = (x.unsqueeze(0).unsqueeze(2) for x in _qkv(toks, layer))  # [1, heads, 1, D]
                qe, ke = oracle.apply_rope(q, k, torch.tensor([[pos]]), THETA)
                oracle.write_paged_kv(rk, rv, alloc, layer, table, [pos], ke, v)
                kk, vv = oracle.read_paged_kv(rk, rv, layer, table)
                want = oracle.decode_attention(qe, kk, vv)[0, :, 0]  # [HQ, D]
                got = decode[st][layer][i, :, 0].float().cpu()
                torch.testing.assert_close(got, want.float(), rtol=1e-2, atol=1e-2,
                                           msg=lambda m, st=st, sid=sid, layer=layer: f"step {st} seq {sid} layer {layer}: {m}")
        assert table.seq_len == len(prompts[sid]) + STEPS
        for layer in range(L):
            kk, vv = oracle.read_paged_kv(rk, rv, layer, table)
            gk, gv = gathered[sid][layer]
            assert_bits_equal(gk, kk, f"seq {sid} layer {layer} keys")
            assert_bits_equal(gv, vv, f"seq {sid} layer {layer} values")
