"""The bench's multi-GPU parity check (bench.oracle_check_sequences), on CPU.

The check runs the oracle's scatter for a sample of sequences into a compact,
poisoned host pool and compares it with the same blocks of the pool under
test. Here the pool under test is written by plain torch indexing (slot ->
block, row) from a poisoned start, so the check must pass; one flipped
element, or a row written to the wrong slot, must make it fail.
"""

from __future__ import annotations

import numpy as np
import torch

import bench
from augur_b200.paged_kv_cache import BlockAllocator, PagedKVCache


def _pool(nb: int) -> PagedKVCache:
    k = torch.empty(bench.L, nb, bench.H, bench.BS, bench.D, dtype=torch.bfloat16)
    v = torch.empty_like(k)
    k.view(torch.uint8).fill_(0xFF)
    v.view(torch.uint8).fill_(0xFF)
    return PagedKVCache(keys=k, values=v, block_size=bench.BS, allocator=BlockAllocator(nb))


def _write(pool, src_k, src_v, slots):
    for t, s in enumerate(slots.tolist()):
        pool.keys[:, s // bench.BS, :, s % bench.BS] = src_k[:, t]
        pool.values[:, s // bench.BS, :, s % bench.BS] = src_v[:, t]


def _samples(pool, rng, g):
    perm = rng.permutation(pool.keys.shape[1])
    out, cur = [], 0
    for n in (5, 16, 37):
        nb = -(-(n + 3) // bench.BS)
        ids = perm[cur : cur + nb].tolist()
        cur += nb
        pos = np.arange(n + 3)
        slots = np.asarray(ids)[pos // bench.BS] * bench.BS + pos % bench.BS
        k = torch.randn(bench.L, n, bench.H, bench.D, generator=g).to(torch.bfloat16)
        v = torch.randn(bench.L, n, bench.H, bench.D, generator=g).to(torch.bfloat16)
        ak = torch.randn(bench.L, 3, bench.H, bench.D, generator=g).to(torch.bfloat16)
        av = torch.randn(bench.L, 3, bench.H, bench.D, generator=g).to(torch.bfloat16)
        out.append({"ids": ids, "k": k, "v": v, "pre": slots[:n], "ak": ak, "av": av, "app": slots[n:]})
    return out


def test_parity_check_accepts_a_correct_pool_and_rejects_a_wrong_one():
    rng, g = np.random.default_rng(3), torch.Generator().manual_seed(3)
    pool = _pool(40)
    samples = _samples(pool, rng, g)
    for x in samples:
        _write(pool, x["k"], x["v"], x["pre"])
        _write(pool, x["ak"], x["av"], x["app"])
    ok, tokens = bench.oracle_check_sequences(pool, samples)
    assert ok and tokens == sum(5 + 16 + 37 for _ in [0]) + 9
    # one element changed
    pool.values[3, samples[1]["ids"][0], 1, 2, 7] += 1
    assert not bench.oracle_check_sequences(pool, samples)[0]


def test_parity_check_rejects_a_row_in_the_wrong_slot():
    rng, g = np.random.default_rng(4), torch.Generator().manual_seed(4)
    pool = _pool(40)
    samples = _samples(pool, rng, g)
    for i, x in enumerate(samples):
        pre = x["pre"].copy()
        if i == 2:
            pre[[0, 1]] = pre[[1, 0]]  # two tokens swapped
        _write(pool, x["k"], x["v"], pre)
        _write(pool, x["ak"], x["av"], x["app"])
    assert not bench.oracle_check_sequences(pool, samples)[0]
