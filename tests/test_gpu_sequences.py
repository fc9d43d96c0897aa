"""Prefix sharing, forks and copy-on-write are invisible in the data.

The same requests run twice: through PagedSequences with a prefix cache (later
prompts share the first prompt's cached blocks, one prompt is forked in the
middle of a block, so the forks' first decode step copies that block), and
through private tables on a twin pool (no prefix cache, each fork given its
own copy of the prompt). Every sequence's gathered K/V must match bit for bit
and the decode outputs exactly (same kernels on the same values); both pools
end with every block free.
"""

from __future__ import annotations

import pytest
import torch

import augur_b200 as ab
from augur_b200 import _lib, _ops, batched
from augur_b200.decode import DecodeGraphStep, paged_decode_layer
from augur_b200.sequences import PagedSequences
from tests.conftest import assert_bits_equal, poison_

pytestmark = pytest.mark.gpu

L, H, HQ, D, BS, NB = 2, 2, 14, 64, 16, 128
THETA = 1000000.0


def _kv(tokens: list[int], lo: int, hi: int) -> tuple[torch.Tensor, torch.Tensor]:
    """K/V [L, hi - lo, H, D] of prompt positions lo..hi-1, a function of the tokens up to
    each position (as a causal model's are), so equal prefixes give equal K/V."""
    ks, vs = [], []
    for p in range(lo, hi):
        g = torch.Generator().manual_seed(hash(tuple(tokens[: p + 1])) & 0x7FFFFFFF)
        ks.append(torch.randn(L, H, D, generator=g))
        vs.append(torch.randn(L, H, D, generator=g))
    return torch.stack(ks, 1).to(torch.bfloat16), torch.stack(vs, 1).to(torch.bfloat16)


def _pool(cuda) -> ab.PagedKVCache:
    return ab.PagedKVCache(keys=poison_(torch.empty(L, NB, H, BS, D, dtype=torch.bfloat16, device=cuda)),
                           values=poison_(torch.empty(L, NB, H, BS, D, dtype=torch.bfloat16, device=cuda)),
                           block_size=BS, allocator=ab.BlockAllocator(NB))


PREFIX = list(range(1000, 1040))  # 2 full blocks + 8 tokens
PROMPTS = [PREFIX + list(range(7)), PREFIX + list(range(200, 221)), PREFIX]
N_FORKS = 2  # of the last prompt, whose last block holds 8 of 16 rows
STEPS = 3


def _run(cuda, shared: bool, graph: bool = False):
    pool = _pool(cuda)
    seqs = PagedSequences(pool)
    ids = []
    for i, toks in enumerate(PROMPTS if shared else PROMPTS + [PROMPTS[-1]] * N_FORKS):
        adm = seqs.admit(toks)
        k, v = _kv(toks, adm.cached_tokens, len(toks))
        batched.write_paged_kv_batch(pool, k.to(cuda), v.to(cuda), torch.from_numpy(adm.slots).to(cuda))
        if shared:
            seqs.publish_prefix(adm.seq_id)
            if i > 0:
                assert adm.cached_tokens == 32
        ids.append(adm.seq_id)
    if shared:
        ids += seqs.fork(ids[-1], N_FORKS)
        first = seqs.tables[ids[0]].block_ids[0]
        assert pool.allocator.refcount(first) == 1 + len(ids)  # the prefix cache and every sequence
    g = torch.Generator().manual_seed(9)
    outs = []
    if graph:  # the decode steps replay one captured graph (DecodeGraphStep)
        gstep = DecodeGraphStep(pool, len(ids), 16, HQ, THETA)
        q_in = torch.empty(L, len(ids), HQ, 1, D, dtype=torch.bfloat16, device=cuda)
        k_in = torch.empty(L, len(ids), H, 1, D, dtype=torch.bfloat16, device=cuda)
        v_in = torch.empty(L, len(ids), H, 1, D, dtype=torch.bfloat16, device=cuda)
        cg = torch.cuda.CUDAGraph()
        cs = torch.cuda.Stream(cuda)
        cs.wait_stream(torch.cuda.current_stream(cuda))
    for st in range(STEPS):
        q = torch.randn(L, len(ids), HQ, 1, D, generator=g).to(torch.bfloat16).to(cuda)
        k = torch.randn(L, len(ids), H, 1, D, generator=g).to(torch.bfloat16).to(cuda)
        v = torch.randn(L, len(ids), H, 1, D, generator=g).to(torch.bfloat16).to(cuda)
        if graph:
            with torch.cuda.stream(cs):
                q_in.copy_(q)
                k_in.copy_(k)
                v_in.copy_(v)
                seqs.update_graph_step(gstep, ids)
                if st == 0:
                    with torch.cuda.graph(cg, stream=cs):
                        g_outs = [gstep.layer(layer, q_in[layer], k_in[layer], v_in[layer]) for layer in range(L)]
                cg.replay()
            torch.cuda.synchronize(cuda)
            outs.append([o.clone() for o in g_outs])
        else:
            step = seqs.decode_step(ids)
            outs.append([paged_decode_layer(step, pool, layer, q[layer], k[layer], v[layer], THETA)
                         for layer in range(L)])
        # the forked prompt's half-full last block: two of its three holders copy it
        assert seqs.last_cow_blocks == (2 if shared and st == 0 else 0)
    if graph:
        cg.reset()
    gathered = []
    for sid in ids:
        t = seqs.tables[sid]
        gathered.append([ab.read_paged_kv(pool, layer, t) for layer in range(L)])
    torch.cuda.synchronize(cuda)
    assert _ops.read_status(cuda) == _lib.OK
    lens = [seqs.tables[s].seq_len for s in ids]
    for sid in ids:
        seqs.release(sid)
    seqs.evict_prefixes()
    assert pool.allocator.num_free == NB, "every block returns to the pool"
    return outs, gathered, lens



def test_shared_prefixes_forks_and_cow_match_private_tables(cuda):
    outs_s, kv_s, lens_s = _run(cuda, shared=True)
    outs_p, kv_p, lens_p = _run(cuda, shared=False)
    assert lens_s == lens_p == [len(p) + STEPS for p in PROMPTS] + [len(PROMPTS[-1]) + STEPS] * N_FORKS
    for b in range(len(lens_s)):
        for layer in range(L):
            assert_bits_equal(kv_s[b][layer][0], kv_p[b][layer][0], f"seq {b} layer {layer} keys")
            assert_bits_equal(kv_s[b][layer][1], kv_p[b][layer][1], f"seq {b} layer {layer} values")
    for s in range(STEPS):
        for layer in range(L):
            assert_bits_equal(outs_s[s][layer], outs_p[s][layer], f"step {s} layer {layer} output")


def test_graph_replayed_steps_with_shared_prefixes_match_eager_steps(cuda):
    """The same requests, forks and copy-on-write, with the decode layers captured once in a
    CUDA graph and replayed after each PagedSequences.update_graph_step: the pools' K/V
    match the eager run bit for bit, the outputs within the bf16 attention tolerance (the
    graph's launch is sized for its buffers' capacity)."""
    outs_e, kv_e, lens_e = _run(cuda, shared=True)
    outs_g, kv_g, lens_g = _run(cuda, shared=True, graph=True)
    assert lens_e == lens_g
    for b in range(len(lens_e)):
        for layer in range(L):
            assert_bits_equal(kv_g[b][layer][0], kv_e[b][layer][0], f"seq {b} layer {layer} keys")
            assert_bits_equal(kv_g[b][layer][1], kv_e[b][layer][1], f"seq {b} layer {layer} values")
    for s in range(len(outs_e)):
        for layer in range(L):
            torch.testing.assert_close(outs_g[s][layer].float(), outs_e[s][layer].float(), rtol=1e-2, atol=1e-2)
