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

import numpy as np
import pytest
import torch

import augur_b200 as ab
from augur_b200 import _lib, _ops, batched
from augur_b200.decode import paged_decode_layer
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


def test_shared_prefixes_forks_and_cow_match_private_tables(cuda):
    prefix = list(range(1000, 1040))  # 2 full blocks + 8 tokens
    prompts = [prefix + list(range(7)), prefix + list(range(200, 221)), prefix]
    n_forks = 2  # of the last prompt, whose last block holds 8 of 16 rows
    steps = 3

    def run(shared: bool):
        pool = _pool(cuda)
        seqs = PagedSequences(pool)
        ids = []
        for i, toks in enumerate(prompts if shared else prompts + [prompts[-1]] * n_forks):
            adm = seqs.admit(toks)
            k, v = _kv(toks, adm.cached_tokens, len(toks))
            batched.write_paged_kv_batch(pool, k.to(cuda), v.to(cuda), torch.from_numpy(adm.slots).to(cuda))
            if shared:
                seqs.publish_prefix(adm.seq_id)
                if i > 0:
                    assert adm.cached_tokens == 32
            ids.append(adm.seq_id)
        if shared:
            ids += seqs.fork(ids[-1], n_forks)
            first = seqs.tables[ids[0]].block_ids[0]
            assert pool.allocator.refcount(first) == 1 + len(ids)  # the prefix cache and every sequence
        g = torch.Generator().manual_seed(9)
        outs = []
        for st in range(steps):
            step = seqs.decode_step(ids)
            # the forked prompt's half-full last block: two of its three holders copy it
            assert seqs.last_cow_blocks == (2 if shared and st == 0 else 0)
            q = torch.randn(L, len(ids), HQ, 1, D, generator=g).to(torch.bfloat16).to(cuda)
            k = torch.randn(L, len(ids), H, 1, D, generator=g).to(torch.bfloat16).to(cuda)
            v = torch.randn(L, len(ids), H, 1, D, generator=g).to(torch.bfloat16).to(cuda)
            outs.append([paged_decode_layer(step, pool, layer, q[layer], k[layer], v[layer], THETA)
                         for layer in range(L)])
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

    outs_s, kv_s, lens_s = run(shared=True)
    outs_p, kv_p, lens_p = run(shared=False)
    assert lens_s == lens_p == [len(p) + steps for p in prompts] + [len(prompts[-1]) + steps] * n_forks
    for b in range(len(lens_s)):
        for layer in range(L):
            assert_bits_equal(kv_s[b][layer][0], kv_p[b][layer][0], f"seq {b} layer {layer} keys")
            assert_bits_equal(kv_s[b][layer][1], kv_p[b][layer][1], f"seq {b} layer {layer} values")
    for s in range(steps):
        for layer in range(L):
            assert_bits_equal(outs_s[s][layer], outs_p[s][layer], f"step {s} layer {layer} output")
