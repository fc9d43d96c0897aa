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



def _raw_call(cuda, q, pool, dt, out, workspace, ws_bytes, max_seq=None):
    """The C-ABI entry point with an explicit workspace."""
    lib = _lib.load()
    kc, vc = pool.keys[0], pool.values[0]
    B, Hq, D = q.shape
    code = lib.augur_kv_paged_decode_attention(
        q.data_ptr(), _lib.i64_array((q.stride(0), q.stride(1))), kc.data_ptr(), vc.data_ptr(),
        _lib.i64_array((kc.stride(0), kc.stride(1), kc.stride(2))), kc.shape[0], kc.shape[2],
        dt.blocks.data_ptr(), dt.blocks.stride(0), dt.blocks.shape[1], dt.lens.data_ptr(),
        dt.max_seq_len if max_seq is None else max_seq, B, Hq, kc.shape[1], D, _ops.dtype_code(q),
        out.data_ptr(), _lib.i64_array((out.stride(0), out.stride(1))), _lib.ATTN_AUTO,
        workspace, ws_bytes, _ops.status_word(cuda).data_ptr(), torch.cuda.current_stream(cuda).cuda_stream)
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
    """No workspace and a too-small one (each sequence unsplit) and the full size (split into
    chunks) give the oracle's result within tolerance; every launch leaves the counters zero."""
    lens = [4000, 17, 2500, 129]
    kp, vp, tables, q, pool = _long_batch(cuda, 21, lens)
    dt = DecodeTables(tables, cuda)
    qd = q.to(cuda)
    lib = _lib.load()
    full = lib.augur_kv_paged_decode_attention_workspace(len(lens), 14, 2, 64, max(lens), _lib.BF16, _lib.ATTN_AUTO)
    assert full > 0
    want = []
    for b, (t, n) in enumerate(zip(tables, lens)):
        k, v = oracle.read_paged_kv(kp, vp, 0, oracle.RefBlockTable(t.block_ids, 16, n))
        want.append(oracle.decode_attention(q[b : b + 1].unsqueeze(2), k, v)[0, :, 0, :])
    for nbytes in (0, full // 3, full):
        ws = torch.zeros(max(nbytes, 16), dtype=torch.uint8, device=cuda)
        out = torch.full_like(qd, float("nan"))
        for _ in range(2):  # the second launch relies on the first having reset the counters
            _raw_call(cuda, qd, pool, dt, out, ws.data_ptr() if nbytes else None, nbytes)
        torch.cuda.synchronize(cuda)
        assert _ops.read_status(cuda) == _lib.OK
        assert int(ws[:512].count_nonzero()) == 0, "scheduler / arrival counters not reset"
        for b in range(len(lens)):
            _close(out[b], want[b], torch.bfloat16, f"workspace {nbytes} seq {b}")


def test_seq_len_above_max_is_reported(cuda):
    lens = [300, 40]
    kp, vp, tables, q, pool = _long_batch(cuda, 22, lens)
    dt = DecodeTables(tables, cuda)
    out = torch.empty_like(q.to(cuda))
    lib = _lib.load()
    nbytes = lib.augur_kv_paged_decode_attention_workspace(2, 14, 2, 64, 200, _lib.BF16, _lib.ATTN_AUTO)
    ws = torch.zeros(max(nbytes, 16), dtype=torch.uint8, device=cuda)
    _raw_call(cuda, q.to(cuda), pool, dt, out, ws.data_ptr(), nbytes, max_seq=200)
    torch.cuda.synchronize(cuda)
    assert _ops.read_status(cuda) == _lib.EBOUNDS
    assert torch.isfinite(out.float()).all()
    assert int(ws[:256].count_nonzero()) == 0
