"""Prefill attention over the paged pool vs the reference (tolerance tests).

The reference's paged branch (augur/attention.py:53-86) writes a call's new
tokens, gathers the whole sequence with read_paged_kv and attends with its
causal mask (past_len = key_len - query_len). The kernels read the pool in
place. Checked against:
  * the reference's own attention() outputs (golden: a suffix call after a
    cached prefix, and a plain prefill), on the pool the reference left;
  * the oracle (oracle.prefill_attention, pinned bit for bit to those
    goldens) on seeded batches: several sequences per launch, prefixes that
    end inside a block, suffixes of one token (a decode step) up to several
    16-token tiles, both head dims, GQA groups of 1 to 8 heads, bf16 / fp16
    on the tcgen05 and mma.sync kernels and float32 on the CUDA-core kernel;
  * a prompt admitted through PagedSequences with its prefix shared from the
    prefix index: its suffix attends to the shared blocks in place.
Tolerance: 1e-2 for bf16 / fp16 (the reference's bf16-kernel tolerance),
1e-5 for float32 (its attention tests' tolerance).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import augur_b200 as ab
from augur_b200 import _lib, _ops, batched
from augur_b200.attention import DecodeTables, paged_attention, paged_prefill_attention
from augur_b200.sequences import PagedSequences
from tests.conftest import poison_

pytestmark = pytest.mark.gpu


def _tol(dtype):
    return dict(rtol=1e-5, atol=1e-5) if dtype == torch.float32 else dict(rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("case", ["f32_prefix", "bf16_prefix", "bf16_plain"])
@pytest.mark.parametrize("kernel", ["auto", "tcgen05", "mma_sync", "generic"])
def test_golden_prefill_attention(cuda, golden, case, kernel):
    """The reference's own attention() output for a call of several tokens on a paged cache
    (its pool as the reference left it: rows never written stay 0xFF and are never read)."""
    c = golden["prefill_attention"][case]
    pool = ab.PagedKVCache(keys=c["keys"].to(cuda), values=c["values"].to(cuda), block_size=16,
                           allocator=ab.BlockAllocator(c["keys"].shape[1]))
    table = ab.SequenceBlockTable(block_ids=list(c["block_ids"]), block_size=16, seq_len=c["seq_len"])
    if kernel in ("tcgen05", "mma_sync") and c["q"].dtype == torch.float32:
        with pytest.raises(ab.KVLibraryError, match="needs bf16/fp16"):
            paged_attention(c["q"].to(cuda), pool, 0, table, kernel=kernel)
        return
    out = paged_attention(c["q"].to(cuda), pool, 0, table, kernel=kernel)
    assert out.shape == c["out"].shape
    torch.testing.assert_close(out.float().cpu(), c["out"].float(), **_tol(c["q"].dtype))
    assert _ops.read_status(cuda) == _lib.OK


def _batch(cuda, oracle, dtype, D, Hq, Hkv, prefixes, suffixes, seed, kernel="auto", bs=16):
    """Sequences with the given cached prefixes and new suffixes in one pool; the suffix
    tokens' attention from one launch against the oracle, sequence by sequence."""
    g = torch.Generator().manual_seed(seed)
    seq_lens = [p + s for p, s in zip(prefixes, suffixes)]
    NB = sum(-(-n // bs) for n in seq_lens) + 5
    L = 2
    pool = ab.PagedKVCache(keys=poison_(torch.empty(L, NB, Hkv, bs, D, dtype=dtype, device=cuda)),
                           values=poison_(torch.empty(L, NB, Hkv, bs, D, dtype=dtype, device=cuda)),
                           block_size=bs, allocator=ab.BlockAllocator(NB))
    pool.allocator.allocate_many(3)  # ids differ from positions
    tables = [ab.SequenceBlockTable.empty(bs) for _ in seq_lens]
    sm = batched.prefill_slot_mapping(tables, seq_lens, pool.allocator)
    T = sum(seq_lens)
    k = torch.randn(L, T, Hkv, D, generator=g).to(dtype)
    v = torch.randn(L, T, Hkv, D, generator=g).to(dtype)
    flat = np.concatenate([sm[b, :n] for b, n in enumerate(seq_lens)])
    batched.write_paged_kv_batch(pool, k.to(cuda), v.to(cuda), torch.from_numpy(flat).to(cuda))
    q = torch.randn(sum(suffixes), Hq, D, generator=g).to(dtype)
    layer = 1
    out = paged_prefill_attention(q.to(cuda), pool, layer, tables, suffixes, kernel=kernel)
    assert _ops.read_status(cuda) == _lib.OK
    hk, hv = pool.keys.cpu(), pool.values.cpu()
    q0 = 0
    for b, (n, S) in enumerate(zip(suffixes, seq_lens)):
        if n == 0:
            continue
        kk, vv = oracle.read_paged_kv(hk, hv, layer, oracle.RefBlockTable(tables[b].block_ids, bs, S))
        want = oracle.prefill_attention(q[q0 : q0 + n].transpose(0, 1)[None], kk, vv)[0].transpose(0, 1)
        torch.testing.assert_close(out[q0 : q0 + n].float().cpu(), want.float(), **_tol(dtype),
                                   msg=lambda m, b=b: f"sequence {b}: {m}")
        q0 += n
    return out


PREFIXES = [0, 21, 200, 700, 16, 5]
SUFFIXES = [37, 16, 45, 1, 64, 3]


@pytest.mark.parametrize("kernel", ["tcgen05", "mma_sync"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D, Hq, Hkv", [(64, 14, 2), (128, 8, 2), (64, 8, 8), (64, 16, 2)])
def test_batch_matches_oracle(cuda, oracle, dtype, D, Hq, Hkv, kernel):
    _batch(cuda, oracle, dtype, D, Hq, Hkv, PREFIXES, SUFFIXES, seed=D + Hq, kernel=kernel)


@pytest.mark.parametrize("kernel", ["tcgen05", "mma_sync", "generic"])
@pytest.mark.parametrize("bs", [8, 32, 12])
def test_block_sizes(cuda, oracle, bs, kernel):
    """Block sizes other than 16: powers of two take the shift, 12 the division, in every
    kernel's block-table lookup."""
    _batch(cuda, oracle, torch.bfloat16, 64, 14, 2, PREFIXES, SUFFIXES, seed=bs, kernel=kernel, bs=bs)


def test_float32_takes_the_generic_kernel(cuda, oracle):
    _batch(cuda, oracle, torch.float32, 64, 14, 2, PREFIXES[:4], SUFFIXES[:4], seed=3)


def test_the_three_kernels_agree(cuda, oracle):
    a = _batch(cuda, oracle, torch.bfloat16, 64, 14, 2, PREFIXES, SUFFIXES, seed=9, kernel="mma_sync")
    b = _batch(cuda, oracle, torch.bfloat16, 64, 14, 2, PREFIXES, SUFFIXES, seed=9, kernel="generic")
    c = _batch(cuda, oracle, torch.bfloat16, 64, 14, 2, PREFIXES, SUFFIXES, seed=9, kernel="tcgen05")
    torch.testing.assert_close(a.float(), b.float(), rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(c.float(), b.float(), rtol=1e-2, atol=1e-2)


def test_a_long_prefix_and_a_sequence_with_no_new_tokens(cuda, oracle):
    # 2,000 cached positions before a 40-token suffix; a sequence with no query tokens in
    # the batch is skipped
    _batch(cuda, oracle, torch.bfloat16, 64, 14, 2, [2000, 50, 0], [40, 0, 20], seed=11)


def test_lengths_that_disagree_are_reported(cuda):
    """More query tokens than cached positions (a table not written first): the Python
    entry refuses it for plain tables, the C entry refuses a launch whose longest query
    exceeds max_seq_len, and on the device the sequence is skipped with AUGUR_KV_EBOUNDS
    while the others are computed."""
    pool = ab.PagedKVCache(keys=torch.zeros(1, 8, 2, 16, 64, dtype=torch.bfloat16, device=cuda),
                           values=torch.zeros(1, 8, 2, 16, 64, dtype=torch.bfloat16, device=cuda),
                           block_size=16, allocator=ab.BlockAllocator(8))
    short = ab.SequenceBlockTable(block_ids=[0, 1], block_size=16, seq_len=3)
    longer = ab.SequenceBlockTable(block_ids=[2, 3], block_size=16, seq_len=20)
    q = torch.zeros(5, 14, 64, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(ValueError, match="more query tokens than cached positions"):
        paged_prefill_attention(q, pool, 0, [short], [5])
    with pytest.raises(ab.KVLibraryError, match="bad sizes"):
        paged_prefill_attention(q, pool, 0, DecodeTables([short], cuda), [5])
    _ops.read_status(cuda)
    out = paged_prefill_attention(torch.zeros(7, 14, 64, dtype=torch.bfloat16, device=cuda), pool, 0,
                                  DecodeTables([short, longer], cuda), [5, 2])
    torch.cuda.synchronize()
    assert _ops.read_status(cuda) == _lib.EBOUNDS
    assert torch.equal(out[5:].float().cpu(), torch.zeros(2, 14, 64))  # zero K/V: the mean of zeros


def test_suffix_prefill_over_a_shared_prefix(cuda, oracle):
    """PagedSequences.admit shares the cached full blocks of a prompt's prefix; the suffix
    tokens are written and attend to the shared blocks in place, as the reference's
    attention over a private copy of the whole prompt does."""
    L, H, Hq, D, bs, NB = 1, 2, 14, 64, 16, 64
    g = torch.Generator().manual_seed(31)
    pool = ab.PagedKVCache(keys=poison_(torch.empty(L, NB, H, bs, D, dtype=torch.bfloat16, device=cuda)),
                           values=poison_(torch.empty(L, NB, H, bs, D, dtype=torch.bfloat16, device=cuda)),
                           block_size=bs, allocator=ab.BlockAllocator(NB))
    seqs = PagedSequences(pool)
    prefix = list(range(500, 548))  # 3 full blocks
    first = seqs.admit(prefix + [1, 2, 3])
    pk = torch.randn(L, len(prefix) + 3, H, D, generator=g).to(torch.bfloat16)
    batched.write_paged_kv_batch(pool, pk.to(cuda), pk.to(cuda), torch.from_numpy(first.slots).to(cuda))
    seqs.publish_prefix(first.seq_id)
    second = seqs.admit(prefix + list(range(40)))
    assert second.cached_tokens == 48  # the prefix's 3 blocks are shared, not written again
    n = 40
    sk = torch.randn(L, n, H, D, generator=g).to(torch.bfloat16)
    sv = torch.randn(L, n, H, D, generator=g).to(torch.bfloat16)
    batched.write_paged_kv_batch(pool, sk.to(cuda), sv.to(cuda), torch.from_numpy(second.slots).to(cuda))
    table = seqs.tables[second.seq_id]
    assert table.block_ids[:3] == seqs.tables[first.seq_id].block_ids[:3] and table.seq_len == 88
    q = torch.randn(n, Hq, D, generator=g).to(torch.bfloat16)
    out = paged_prefill_attention(q.to(cuda), pool, 0, [table], [n])
    # reference composition: the whole prompt in a private table, then the suffix call's attention
    kk = torch.cat([pk[0, :48], sk[0]], 0).transpose(0, 1)[None]  # [1, H, 88, D]
    vv = torch.cat([pk[0, :48], sv[0]], 0).transpose(0, 1)[None]
    want = oracle.prefill_attention(q.transpose(0, 1)[None], kk, vv)[0].transpose(0, 1)
    torch.testing.assert_close(out.float().cpu(), want.float(), rtol=1e-2, atol=1e-2)
    assert _ops.read_status(cuda) == _lib.OK
