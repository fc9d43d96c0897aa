"""Disaggregated prefill -> decode push between two GPUs (two processes).

Rank 1 (decode) exports its block pool, a ready flag and the destination
blocks its own allocator picked, and queues a device-side wait on the flag
followed by a gather of those blocks; rank 0 (prefill) scatters seeded K/V
into its local pool, opens rank 1's pool through CUDA IPC, pushes the blocks
with one kernel (plain stores over NVLink) and signals the flag. Rank 1 then
compares its whole pool, bit for bit, with the same tokens written locally
through write_paged_kv_batch (pushed rows must match, every other row must
still hold the poison), and the gather that waited on the flag must have
seen the pushed data.
Needs two GPUs; skipped on one.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

L, H, D, BS, NB = 6, 2, 64, 16, 96


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _workload():
    rng = np.random.default_rng(11)
    lens = rng.integers(1, 120, size=7)
    g = torch.Generator().manual_seed(11)
    T = int(lens.sum())
    k = torch.randn(L, T, H, D, generator=g).to(torch.bfloat16)
    v = torch.randn(L, T, H, D, generator=g).to(torch.bfloat16)
    return lens, k, v


def _poisoned_pool(ab, dev):
    pool = ab.PagedKVCache(keys=torch.empty(L, NB, H, BS, D, dtype=torch.bfloat16, device=dev),
                           values=torch.empty(L, NB, H, BS, D, dtype=torch.bfloat16, device=dev),
                           block_size=BS, allocator=ab.BlockAllocator(NB))
    pool.keys.view(torch.uint8).fill_(0xFF)
    pool.values.view(torch.uint8).fill_(0xFF)
    return pool


def _worker(rank: int, port: int, q) -> None:
    import datetime

    import torch.distributed as dist

    import augur_b200 as ab
    from augur_b200 import _lib, _ops, batched, peer

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=60))
    try:
        lens, k, v = _workload()
        pool = _poisoned_pool(ab, dev)
        # 1. the decode rank picks destination blocks with its own allocator and exports its pool
        obj = [None]
        if rank == 1:
            pool.allocator.allocate_many(5)  # decode pool already holds other work
            dst_tables = [ab.SequenceBlockTable.empty(BS) for _ in lens]
            batched.prefill_slot_mapping(dst_tables, lens, pool.allocator)
            flags = peer.new_flags(dev)
            obj = [(peer.export_pool(pool, flags), [t.block_ids for t in dst_tables])]
        dist.broadcast_object_list(obj, src=1)
        exported, dst_ids = obj[0]
        if rank == 1:
            # queue, before the push has happened, a device-side wait for the
            # prefill rank's ready flag and then a gather of the pushed blocks
            w0, w1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            w0.record()
            peer.wait(flags, 1, timeout_s=30.0)
            w1.record()
            early = batched.read_paged_kv_batch(
                pool, [ab.SequenceBlockTable(block_ids=list(ids), block_size=BS, seq_len=int(n))
                       for ids, n in zip(dst_ids, lens)])
        # 2. the prefill rank scatters locally, then pushes block by block into the peer pool
        if rank == 0:
            src_tables = [ab.SequenceBlockTable.empty(BS) for _ in lens]
            sm = batched.prefill_slot_mapping(src_tables, lens, pool.allocator)
            flat = np.concatenate([sm[b, :n] for b, n in enumerate(lens)])
            batched.write_paged_kv_batch(pool, k.to(dev), v.to(dev), torch.from_numpy(flat).to(dev))
            remote = peer.open_pool(exported, dev)
            src_b, dst_b, rows = [], [], []
            for t_src, ids, n in zip(src_tables, dst_ids, lens):
                for j in range(-(-int(n) // BS)):
                    src_b.append(t_src.block_ids[j])
                    dst_b.append(ids[j])
                    rows.append(min(BS, int(n) - j * BS))
            moved = peer.push_blocks(pool, src_b, remote, dst_b, rows)
            peer.signal(remote, 1)  # stream-ordered after the push
            torch.cuda.synchronize(dev)
            assert _ops.read_status(dev) == _lib.OK
        dist.barrier()  # push complete
        # 3. the decode rank checks its whole pool against a local write of the same tokens
        if rank == 1:
            ref = _poisoned_pool(ab, dev)
            tables = [ab.SequenceBlockTable(block_ids=list(ids), block_size=BS) for ids in dst_ids]
            pos = [np.arange(int(n)) for n in lens]
            flat = np.concatenate([np.asarray(t.block_ids)[p // BS] * BS + p % BS for t, p in zip(tables, pos)])
            batched.write_paged_kv_batch(ref, k.to(dev), v.to(dev), torch.from_numpy(flat).to(dev))
            torch.cuda.synchronize(dev)
            same_k = torch.equal(pool.keys.view(torch.int16), ref.keys.view(torch.int16))
            same_v = torch.equal(pool.values.view(torch.int16), ref.values.view(torch.int16))
            # the gather queued behind the device wait saw the pushed data
            # (valid rows of each sequence; rows past a length are not written)
            rk, rv = batched.read_paged_kv_batch(ref, tables, seq_lens=[int(n) for n in lens])
            same_early = all(
                torch.equal(early[0][:, b, :, :n].view(torch.int16), rk[:, b, :, :n].view(torch.int16))
                and torch.equal(early[1][:, b, :, :n].view(torch.int16), rv[:, b, :, :n].view(torch.int16))
                for b, n in enumerate(int(x) for x in lens))
            status = _ops.read_status(dev)
            q.put(("decode", {"same_k": bool(same_k), "same_v": bool(same_v), "same_early": bool(same_early),
                              "status": status, "wait_ms": w0.elapsed_time(w1), "flag": int(flags[0].item())},
                   int(lens.sum())))
        dist.barrier()  # checks done; the importer may unmap now
        if rank == 0:
            remote.close()
            q.put(("prefill", moved))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_push_blocks_between_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(2):
        item = q.get(timeout=300)
        got[item[0]] = item[1:]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    checks, tokens = got["decode"]
    msg = " ".join(f"{k}={v}" for k, v in checks.items())
    assert checks["same_k"] and checks["same_v"], msg
    assert checks["same_early"] and checks["status"] == 0 and checks["flag"] == 1, msg
    assert got["prefill"][0] == tokens * L * 2 * H * D * 2
