"""Paged decode attention vs the reference's attention (floating point, tolerance-based).

Tolerances: float32 rtol = atol = 1e-5 (the reference's own tolerance for
cached vs uncached and paged vs contiguous attention, tests/test_attention.py);
bf16 / fp16 rtol = atol = 1e-2 (the reference's tolerance for its bf16
kernel, tests/test_kernels/test_rms_norm.py). The kernels round where the
reference rounds but sum in another order, so results are not bit-exact.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import augur_b200 as ab
from augur_b200 import _lib, _ops
from augur_b200.attention import DecodeTables, paged_decode_attention
from tests.conftest import assert_bits_equal

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-5, torch.bfloat16: 1e-2, torch.float16: 1e-2}


def _close(got, want, dtype, what=""):
    tol = TOL[dtype]
    torch.testing.assert_close(got.float().cpu(), want.float().cpu(), rtol=tol, atol=tol, msg=what)


@pytest.mark.parametrize("case, generic", [("f32", False), ("bf16", False), ("bf16", True)])
def test_reference_golden(cuda, golden, case, generic):
    """The reference's own attention() on its paged cache (14 query heads, 2 KV heads, head_dim 64)."""
    c = golden["attention"][case]
    dtype = c["keys"].dtype
    pool = ab.PagedKVCache(keys=c["keys"].to(cuda), values=c["values"].to(cuda), block_size=16,
                           allocator=ab.BlockAllocator(c["keys"].shape[1]))
    table = ab.SequenceBlockTable(block_ids=list(c["block_ids"]), block_size=16, seq_len=c["seq_len"])
    out = paged_decode_attention(c["q"].to(cuda), pool, 0, [table], generic=generic)
    assert out.shape == c["out"].shape and out.dtype == dtype
    _close(out, c["out"], dtype, f"{case} generic={generic}")
    assert _ops.read_status(cuda) == _lib.OK


def _case(cuda, oracle, dtype, B, Hq, Hkv, D, bs, lens, seed, generic):
    g = torch.Generator().manual_seed(seed)
    rng = np.random.default_rng(seed)
    nblk = [-(-int(n) // bs) for n in lens]
    NB = sum(nblk) + 7
    kp = torch.randn(1, NB, Hkv, bs, D, generator=g).to(dtype)
    vp = torch.randn(1, NB, Hkv, bs, D, generator=g).to(dtype)
    perm = rng.permutation(NB).tolist()
    tables, cur = [], 0
    for n, nb in zip(lens, nblk):
        tables.append(ab.SequenceBlockTable(block_ids=perm[cur : cur + nb], block_size=bs, seq_len=int(n)))
        cur += nb
    q = torch.randn(B, Hq, D, generator=g).to(dtype)
    pool = ab.PagedKVCache(keys=kp.to(cuda), values=vp.to(cuda), block_size=bs, allocator=ab.BlockAllocator(NB))
    got = paged_decode_attention(q.to(cuda), pool, 0, tables, generic=generic)
    for b, (t, n) in enumerate(zip(tables, lens)):
        if n == 0:
            continue
        rt = oracle.RefBlockTable(t.block_ids, bs, int(n))
        k, v = oracle.read_paged_kv(kp, vp, 0, rt)
        want = oracle.decode_attention(q[b : b + 1].unsqueeze(2), k, v)[0, :, 0, :]
        _close(got[b], want, dtype, f"seq {b} len {n}")
    assert _ops.read_status(cuda) == _lib.OK


@pytest.mark.parametrize("generic", [False, True])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_augur_shape_batch(cuda, oracle, dtype, generic):
    """augur's GQA shape, a batch with lengths around tile and block edges and a long one."""
    lens = [1, 15, 16, 17, 100, 513, 2049, 33]
    _case(cuda, oracle, dtype, len(lens), 14, 2, 64, 16, lens, 1, generic)


@pytest.mark.parametrize(
    "Hq, Hkv, D, bs",
    [(2, 2, 64, 16), (16, 1, 64, 16), (8, 2, 128, 16), (7, 1, 64, 8), (4, 2, 64, 32), (28, 4, 128, 4),
     (14, 2, 64, 12), (14, 2, 64, 1), (14, 2, 64, 64), (16, 2, 128, 48)],
)
def test_shapes_tensor_core_path(cuda, oracle, Hq, Hkv, D, bs):
    """Block sizes that are and are not powers of two, smaller and larger than a 32-token stage."""
    _case(cuda, oracle, torch.bfloat16, 3, Hq, Hkv, D, bs, [5, 70, 300], 2, False)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_empty_and_chunk_edge_lengths(cuda, oracle, dtype):
    """A zero-length sequence next to lengths at 32-token stage and 128-token chunk edges."""
    lens = [0, 31, 32, 33, 127, 128, 129, 255, 256, 257, 1000, 3000]
    _case(cuda, oracle, dtype, len(lens), 14, 2, 64, 16, lens, 6, False)


@pytest.mark.parametrize(
    "dtype, Hq, Hkv, D, bs",
    [(torch.float32, 14, 2, 64, 16), (torch.float32, 4, 4, 32, 4), (torch.bfloat16, 3, 1, 40, 16),
     (torch.bfloat16, 32, 1, 64, 16)],
)
def test_shapes_generic_path(cuda, oracle, dtype, Hq, Hkv, D, bs):
    """float32, head_dim not 64/128 and groups over 16 take the CUDA-core kernel."""
    _case(cuda, oracle, dtype, 3, Hq, Hkv, D, bs, [1, 37, 260], 3, False)


def test_long_sequence_and_4d_query(cuda, oracle):
    """An 8192-token sequence (the scale-out workload's longest), query as [B, H, 1, D]."""
    g = torch.Generator().manual_seed(9)
    n, bs, NB = 8192, 16, 600
    kp = torch.randn(1, NB, 2, bs, 64, generator=g).to(torch.bfloat16)
    vp = torch.randn(1, NB, 2, bs, 64, generator=g).to(torch.bfloat16)
    ids = np.random.default_rng(9).permutation(NB)[: n // bs].tolist()
    t = ab.SequenceBlockTable(block_ids=ids, block_size=bs, seq_len=n)
    q = torch.randn(1, 14, 1, 64, generator=g).to(torch.bfloat16)
    pool = ab.PagedKVCache(keys=kp.to(cuda), values=vp.to(cuda), block_size=bs, allocator=ab.BlockAllocator(NB))
    dt = DecodeTables([t], cuda)
    got = paged_decode_attention(q.to(cuda), pool, 0, dt)
    assert got.shape == (1, 14, 1, 64)
    k, v = oracle.read_paged_kv(kp, vp, 0, oracle.RefBlockTable(ids, bs, n))
    _close(got, oracle.decode_attention(q, k, v), torch.bfloat16, "8192 tokens")


def test_bad_block_id_is_reported(cuda):
    pool = ab.PagedKVCache(keys=torch.randn(1, 4, 2, 16, 64, device=cuda).to(torch.bfloat16),
                           values=torch.randn(1, 4, 2, 16, 64, device=cuda).to(torch.bfloat16),
                           block_size=16, allocator=ab.BlockAllocator(4))
    t = ab.SequenceBlockTable(block_ids=[1, 9], block_size=16, seq_len=20)  # block 9 is outside the pool
    out = paged_decode_attention(torch.randn(1, 14, 64, device=cuda).to(torch.bfloat16), pool, 0, [t])
    assert _ops.read_status(cuda) == _lib.EBOUNDS
    assert torch.isfinite(out.float()).all()



def _raw_call(cuda, q, pool, dt, out, counters, scratch, max_seq=None):
    """The C-ABI entry point with explicit counters and scratch (tensors or None)."""
    lib = _lib.load()
    kc, vc = pool.keys[0], pool.values[0]
    B, Hq, D = q.shape
    code = lib.augur_kv_paged_decode_attention(
        q.data_ptr(), _lib.i64_array((q.stride(0), q.stride(1))), kc.data_ptr(), vc.data_ptr(),
        _lib.i64_array((kc.stride(0), kc.stride(1), kc.stride(2))), kc.shape[0], kc.shape[2],
        dt.blocks.data_ptr(), dt.blocks.stride(0), dt.blocks.shape[1], dt.lens.data_ptr(),
        dt.max_seq_len if max_seq is None else max_seq, B, Hq, kc.shape[1], D, _ops.dtype_code(q),
        out.data_ptr(), _lib.i64_array((out.stride(0), out.stride(1))), _lib.ATTN_AUTO,
        None if counters is None else counters.data_ptr(), 0 if counters is None else counters.numel() * 4,
        None if scratch is None else scratch.data_ptr(), 0 if scratch is None else scratch.numel(),
        _ops.status_word(cuda).data_ptr(), torch.cuda.current_stream(cuda).cuda_stream)
    _lib.check(code, "augur_kv_paged_decode_attention")


def _long_batch(cuda, seed, lens, bs=16):
    g = torch.Generator().manual_seed(seed)
    nblk = [-(-n // bs) for n in lens]
    NB = sum(nblk) + 3
    kp = torch.randn(1, NB, 2, bs, 64, generator=g).to(torch.bfloat16)
    vp = torch.randn(1, NB, 2, bs, 64, generator=g).to(torch.bfloat16)
    perm = np.random.default_rng(seed).permutation(NB).tolist()
    tables, cur = [], 0
    for n, nb in zip(lens, nblk):
        tables.append(ab.SequenceBlockTable(block_ids=perm[cur : cur + nb], block_size=bs, seq_len=n))
        cur += nb
    q = torch.randn(len(lens), 14, 64, generator=g).to(torch.bfloat16)
    pool = ab.PagedKVCache(keys=kp.to(cuda), values=vp.to(cuda), block_size=bs, allocator=ab.BlockAllocator(NB))
    return kp, vp, tables, q, pool


def test_workspace_sizes_and_counters(cuda, oracle):
    """No counters (static items, unsplit), counters without scratch (dynamic items, unsplit)
    and the full workspace (split into chunks) give the oracle's result within tolerance;
    every launch leaves the counters zero."""
    from augur_b200.attention import workspace_bytes

    lens = [4000, 17, 2500, 129]
    kp, vp, tables, q, pool = _long_batch(cuda, 21, lens)
    dt = DecodeTables(tables, cuda)
    qd = q.to(cuda)
    lib = _lib.load()
    need_c, need_s = workspace_bytes(lib, (len(lens), 14, 2, 64, max(lens), _lib.BF16, _lib.ATTN_AUTO))
    assert need_c > 256 and need_s > 0
    want = []
    for b, (t, n) in enumerate(zip(tables, lens)):
        k, v = oracle.read_paged_kv(kp, vp, 0, oracle.RefBlockTable(t.block_ids, 16, n))
        want.append(oracle.decode_attention(q[b : b + 1].unsqueeze(2), k, v)[0, :, 0, :])
    for c_bytes, s_bytes in ((0, 0), (256, 0), (need_c, need_s // 2), (need_c, need_s)):
        cnt = torch.zeros(max(1, c_bytes // 4), dtype=torch.int32, device=cuda) if c_bytes else None
        scr = torch.empty(s_bytes, dtype=torch.uint8, device=cuda) if s_bytes else None
        out = torch.full_like(qd, float("nan"))
        for _ in range(2):  # the second launch relies on the first having reset the counters
            _raw_call(cuda, qd, pool, dt, out, cnt, scr)
        torch.cuda.synchronize(cuda)
        assert _ops.read_status(cuda) == _lib.OK
        if cnt is not None:
            assert int(cnt.count_nonzero()) == 0, "counters not left zero"
        for b in range(len(lens)):
            _close(out[b], want[b], torch.bfloat16, f"counters {c_bytes} scratch {s_bytes} seq {b}")


def test_counters_shared_across_sizes(cuda, oracle):
    """One counters buffer and one scratch buffer serve launches of different sizes in turn
    (head_dim 128 then 64, few then many sequences): counters never hold data."""
    from augur_b200.attention import workspace_bytes

    lib = _lib.load()
    cnt = torch.zeros(1 << 16, dtype=torch.int32, device=cuda)
    scr = torch.empty(64 << 20, dtype=torch.uint8, device=cuda)
    g = torch.Generator().manual_seed(44)
    for Hq, Hkv, D, nseq in ((16, 2, 128, 3), (14, 2, 64, 300), (8, 1, 64, 40)):
        lens = [int(x) for x in np.random.default_rng(nseq).integers(1, 900, size=nseq)]
        nblk = [-(-n // 16) for n in lens]
        NB = sum(nblk) + 1
        kp = torch.randn(1, NB, Hkv, 16, D, generator=g).to(torch.bfloat16)
        vp = torch.randn(1, NB, Hkv, 16, D, generator=g).to(torch.bfloat16)
        tabs, cur = [], 0
        for n, nb in zip(lens, nblk):
            tabs.append(ab.SequenceBlockTable(block_ids=list(range(cur, cur + nb)), block_size=16, seq_len=n))
            cur += nb
        pool = ab.PagedKVCache(keys=kp.to(cuda), values=vp.to(cuda), block_size=16, allocator=ab.BlockAllocator(NB))
        q = torch.randn(nseq, Hq, D, generator=g).to(torch.bfloat16)
        need_c, need_s = workspace_bytes(lib, (nseq, Hq, Hkv, D, max(lens), _lib.BF16, _lib.ATTN_AUTO))
        assert need_c <= cnt.numel() * 4 and need_s <= scr.numel()
        out = torch.empty(nseq, Hq, D, dtype=torch.bfloat16, device=cuda)
        _raw_call(cuda, q.to(cuda), pool, DecodeTables(tabs, cuda), out, cnt, scr)
        torch.cuda.synchronize(cuda)
        assert int(cnt.count_nonzero()) == 0
        for b in range(0, nseq, max(1, nseq // 20)):
            k, v = oracle.read_paged_kv(kp, vp, 0, oracle.RefBlockTable(tabs[b].block_ids, 16, lens[b]))
            want = oracle.decode_attention(q[b : b + 1].unsqueeze(2), k, v)[0, :, 0, :]
            _close(out[b], want, torch.bfloat16, f"D {D} seq {b}")


def test_seq_len_above_max_is_reported(cuda):
    from augur_b200.attention import workspace_bytes

    lens = [300, 40]
    kp, vp, tables, q, pool = _long_batch(cuda, 22, lens)
    dt = DecodeTables(tables, cuda)
    out = torch.empty_like(q.to(cuda))
    lib = _lib.load()
    need_c, need_s = workspace_bytes(lib, (2, 14, 2, 64, 200, _lib.BF16, _lib.ATTN_AUTO))
    cnt = torch.zeros(need_c // 4, dtype=torch.int32, device=cuda)
    scr = torch.empty(max(16, need_s), dtype=torch.uint8, device=cuda)
    _raw_call(cuda, q.to(cuda), pool, dt, out, cnt, scr, max_seq=200)
    torch.cuda.synchronize(cuda)
    assert _ops.read_status(cuda) == _lib.EBOUNDS
    assert torch.isfinite(out.float()).all()
    assert int(cnt.count_nonzero()) == 0


def test_large_batch_scheduling_paths(cuda, oracle):
    """300 sequences: beyond the register-held lengths (256) and item counts (128), so the
    plan re-reads lengths and the item search walks seq_lens; several chunk sizes and
    dynamic item scheduling are exercised against the oracle."""
    rng = np.random.default_rng(30)
    lens = [int(x) for x in rng.integers(0, 700, size=300)]
    lens[7] = 4000  # one long sequence split over many chunks
    _case(cuda, oracle, torch.bfloat16, len(lens), 14, 2, 64, 16, lens, 30, False)


def test_back_to_back_launches_share_the_workspace(cuda, oracle):
    """Three launches on one stream reuse the cached workspace: the scheduler and arrival
    counters each launch leaves at zero must serve the next."""
    for seed in (41, 42, 43):
        lens = [int(x) for x in np.random.default_rng(seed).integers(100, 3000, size=20)]
        _case(cuda, oracle, torch.float16, len(lens), 14, 2, 64, 16, lens, seed, False)


@pytest.mark.parametrize("nseq", [5, 40, 300, 1000])
def test_early_reads_back_to_back_layers(cuda, oracle, nseq):
    """AUGUR_KV_ATTN_EARLY_READS: each layer's launch reads lengths, tables and pool rows
    before the previous layer's launch (which shares its workspace) has finished. Six
    layers back to back, twice over, give the same outputs bit for bit both times, and the
    outputs of launches without early reads and the oracle's within tolerance (a small
    batch's plan may take fewer, longer chunks with early reads, so the summation order can
    differ). Five sequences leave most CTAs without an item (they exit through the
    scheduler's counters); 300 take several items per CTA; 1,000 short ones are more
    (sequence, KV head) units than the plan's item bound, so every sequence runs unsplit."""
    L, Hq, Hkv, D, bs = 6, 14, 2, 64, 16
    rng = np.random.default_rng(nseq)
    hi = 2500 if nseq < 100 else (900 if nseq < 1000 else 64)
    lens = [int(x) for x in rng.integers(1, hi, size=nseq)]
    nblk = [-(-n // bs) for n in lens]
    NB = sum(nblk) + 3
    g = torch.Generator().manual_seed(nseq)
    kp = torch.randn(L, NB, Hkv, bs, D, generator=g).to(torch.bfloat16)
    vp = torch.randn(L, NB, Hkv, bs, D, generator=g).to(torch.bfloat16)
    perm = rng.permutation(NB).tolist()
    tables, cur = [], 0
    for n, nb in zip(lens, nblk):
        tables.append(ab.SequenceBlockTable(block_ids=perm[cur : cur + nb], block_size=bs, seq_len=n))
        cur += nb
    pool = ab.PagedKVCache(keys=kp.to(cuda), values=vp.to(cuda), block_size=bs, allocator=ab.BlockAllocator(NB))
    dt = DecodeTables(tables, cuda)
    q = torch.randn(L, nseq, Hq, D, generator=g).to(torch.bfloat16)
    qd = q.to(cuda)
    plain = torch.stack([paged_decode_attention(qd[layer], pool, layer, dt) for layer in range(L)])
    first = None
    for _ in range(2):
        outs = torch.full_like(qd, float("nan"))
        for layer in range(L):
            paged_decode_attention(qd[layer], pool, layer, dt, out=outs[layer], early_reads=True)
        torch.cuda.synchronize(cuda)
        if first is None:
            first = outs
            _close(outs, plain, torch.bfloat16, "early reads against plain launches")
        else:
            assert_bits_equal(outs, first, "early reads, second pass")
    assert _ops.read_status(cuda) == _lib.OK
    for layer in (0, L - 1):
        for b in range(0, nseq, max(1, nseq // 10)):
            k, v = oracle.read_paged_kv(kp, vp, layer, oracle.RefBlockTable(tables[b].block_ids, bs, lens[b]))
            want = oracle.decode_attention(q[layer, b : b + 1].unsqueeze(2), k, v)[0, :, 0, :]
            _close(outs[layer, b], want, torch.bfloat16, f"layer {layer} seq {b}")


def test_early_reads_flag_is_checked(cuda):
    """The early-reads bit combines with AUTO or GENERIC only; other values are refused."""
    lens = [40, 3]
    kp, vp, tables, q, pool = _long_batch(cuda, 23, lens)
    dt = DecodeTables(tables, cuda)
    qd = q.to(cuda)
    out = torch.empty_like(qd)
    lib = _lib.load()
    for flags, ok in ((_lib.ATTN_EARLY_READS, True), (_lib.ATTN_GENERIC | _lib.ATTN_EARLY_READS, True),
                      (_lib.ATTN_EARLY_READS | 2, False), (32, False)):
        code = lib.augur_kv_paged_decode_attention(
            qd.data_ptr(), _lib.i64_array((qd.stride(0), qd.stride(1))), pool.keys[0].data_ptr(),
            pool.values[0].data_ptr(), _lib.i64_array(pool.keys[0].stride()[:3]), pool.keys.shape[1], 16,
            dt.blocks.data_ptr(), dt.blocks.stride(0), dt.blocks.shape[1], dt.lens.data_ptr(), dt.max_seq_len,
            2, 14, 2, 64, _lib.BF16, out.data_ptr(), _lib.i64_array((out.stride(0), out.stride(1))), flags,
            None, 0, None, 0, _ops.status_word(cuda).data_ptr(), torch.cuda.current_stream(cuda).cuda_stream)
        assert (code == _lib.OK) == ok, flags
    torch.cuda.synchronize(cuda)
    assert _ops.read_status(cuda) == _lib.OK
