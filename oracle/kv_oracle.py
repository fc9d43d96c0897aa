"""CPU oracle for augur's KV-cache data movement — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module; it is the checker, never the thing measured or shipped, and
augur_b200/ never imports it.

It restates semioz/augur's cache algorithm:
  * host bookkeeping in plain Python, statement for statement the reference's
    order of effects: RefBlockAllocator (augur/paged_kv_cache.py:10-22),
    RefBlockTable (:88-139), ref_block_hash (:84-85);
  * data movement through liboracle_kv.so (kv_oracle.c), one C function per
    reference loop, on torch CPU tensors;
  * write_paged_kv_torch_loop: the reference's per-token torch loop itself,
    restated only so the CPU baseline can time the reference's own path.

Parity pin: tests/test_oracle_pins.py checks every function here against the
known-answer cases of the reference's own tests (tests/test_kv_cache.py,
tests/test_paged_kv_cache.py, tests/test_prefix_cache.py) and against golden
fixtures produced by running the reference itself (tests/golden/make_golden.py).
"""

from __future__ import annotations

import ctypes
import math
import os
import subprocess

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle_kv.so")

_DTYPES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}

_lib: ctypes.CDLL | None = None


def build(force: bool = False) -> str:
    """Compile liboracle_kv.so with the committed Makefile (gcc, pthreads)."""
    src = os.path.join(HERE, "kv_oracle.c")
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(src) > os.path.getmtime(LIB_PATH):
        subprocess.run(["make", "-s", "-C", HERE, "-B" if force else "liboracle_kv.so"], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        build()
        l = ctypes.CDLL(LIB_PATH)
        P, I64, I32, I64P, I32P = (ctypes.c_void_p, ctypes.c_int64, ctypes.c_int,
                                   ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int32))
        l.oracle_write_kv.argtypes = [P, I64P, I32, P, I64P, I32, I64, I64P, I64P, I64, I64, I64, I64]
        l.oracle_write_paged_tokens.argtypes = [P, I64P, I32, P, I64P, I32, I64, I64P, I64P, I64, I64, I64]
        l.oracle_read_paged.argtypes = [P, I64P, I32, I64, I64P, I64, I64, P, I64P, I64, I64]
        l.oracle_copy_prefix.argtypes = [P, I64P, I32, P, I64P, I32, I64, I64, I64, I64, I64]
        l.oracle_scatter_slots.argtypes = [P, P, I64P, P, P, I64P, I64, I64P, I64, I64, I64, I64, I64, I32]
        l.oracle_copy_runs.argtypes = [P, P, I64P, P, P, I64P, I64, I32P, I64, I64, I64, I64, I32]
        l.oracle_max_threads.restype = ctypes.c_int
        for fn in ("oracle_write_kv", "oracle_write_paged_tokens", "oracle_read_paged",
                   "oracle_copy_prefix", "oracle_scatter_slots", "oracle_copy_runs"):
            getattr(l, fn).restype = None
        _lib = l
    return _lib


def max_threads() -> int:
    return int(lib().oracle_max_threads())


def _i64(vals) -> ctypes.Array:
    vals = [int(v) for v in vals]
    return (ctypes.c_int64 * max(1, len(vals)))(*vals)


def _cpu(t: torch.Tensor) -> torch.Tensor:
    if t.device.type != "cpu":
        raise ValueError("the oracle runs on CPU tensors")
    if t.stride(-1) != 1:
        raise ValueError("the oracle needs head_dim contiguous")
    return t


def _i64_ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_int64))


# ---------------------------------------------------------------------------
# restated host bookkeeping
# ---------------------------------------------------------------------------


class RefBlockAllocator:
    """augur/paged_kv_cache.py:10-22: list free list, pop(0) / insert(0, ...)."""

    def __init__(self, num_blocks: int) -> None:
        if num_blocks <= 0:
            raise ValueError("num_blocks must be positive")
        self.free_blocks = list(range(num_blocks))

    def allocate(self) -> int:
        if not self.free_blocks:
            raise RuntimeError("no free KV cache blocks")
        return self.free_blocks.pop(0)

    def free(self, block_id: int) -> None:
        self.free_blocks.insert(0, block_id)


class RefBlockTable:
    """augur/paged_kv_cache.py:88-139."""

    def __init__(self, block_ids: list[int], block_size: int, seq_len: int = 0) -> None:
        self.block_ids = list(block_ids)
        self.block_size = block_size
        self.seq_len = seq_len

    def ensure_position(self, position: int, allocator: RefBlockAllocator) -> None:
        if position < 0:
            raise ValueError("position must be non-negative")
        required = position // self.block_size + 1
        while len(self.block_ids) < required:
            self.block_ids.append(allocator.allocate())
        self.seq_len = max(self.seq_len, position + 1)

    def free(self, allocator: RefBlockAllocator) -> None:
        for block_id in reversed(self.block_ids):
            allocator.free(block_id)
        self.block_ids.clear()
        self.seq_len = 0

    def position_to_block_offset(self, position: int) -> tuple[int, int]:
        if position < 0:
            raise ValueError("position must be non-negative")
        logical = position // self.block_size
        if logical >= len(self.block_ids):
            raise ValueError("position exceeds block table capacity")
        return self.block_ids[logical], position % self.block_size


def ref_block_hash(parent_hash: int | None, block_tokens) -> int:
    """augur/paged_kv_cache.py:84-85: Python hash of (parent hash, token tuple)."""
    return hash((parent_hash, tuple(block_tokens)))


def ref_match_prefix(blocks: dict, token_ids: list[int], block_size: int) -> tuple[list[int], int]:
    """augur/paged_kv_cache.py:63-82 over a {(parent, tokens): (hash, block)} dict."""
    parent: int | None = None
    ids: list[int] = []
    for b in range(len(token_ids) // block_size):
        entry = blocks.get((parent, tuple(token_ids[b * block_size : (b + 1) * block_size])))
        if entry is None:
            break
        parent, block_id = entry
        ids.append(block_id)
    return ids, len(ids) * block_size


# ---------------------------------------------------------------------------
# composed data movement (torch CPU tensors)
# ---------------------------------------------------------------------------


def write_kv(cache_k, cache_v, layer: int, position_ids, key, value) -> None:
    """augur/kv_cache.py:103-106 for already-validated positions."""
    pos = np.ascontiguousarray(position_ids.to(torch.int64).numpy())
    pstr = _i64([s // 8 for s in pos.strides])
    batch, heads, seq, head_dim = key.shape
    for src, dst in ((key, cache_k), (value, cache_v)):
        src, dst = _cpu(src), _cpu(dst)
        lib().oracle_write_kv(src.data_ptr(), _i64(src.stride()), _DTYPES[src.dtype], dst.data_ptr(),
                              _i64(dst.stride()), _DTYPES[dst.dtype], layer, _i64_ptr(pos), pstr,
                              batch, heads, seq, head_dim)


def write_paged_kv(pool_k, pool_v, allocator: RefBlockAllocator, layer: int, table: RefBlockTable,
                   positions: list[int], key, value) -> None:
    """augur/paged_kv_cache.py:188-192: per token ensure_position, resolve, copy.

    Like the reference, tokens before a failing one are written and the
    error is raised afterwards.
    """
    blocks, offsets, err = [], [], None
    for p in positions:
        try:
            table.ensure_position(p, allocator)
            blk, off = table.position_to_block_offset(p)
        except (ValueError, RuntimeError) as exc:
            err = exc
            break
        blocks.append(blk)
        offsets.append(off)
    n = len(blocks)
    if n:
        b = np.asarray(blocks, dtype=np.int64)
        o = np.asarray(offsets, dtype=np.int64)
        heads, head_dim = key.shape[1], key.shape[3]
        for src, dst in ((key, pool_k), (value, pool_v)):
            src, dst = _cpu(src), _cpu(dst)
            lib().oracle_write_paged_tokens(src.data_ptr(), _i64(src.stride()), _DTYPES[src.dtype],
                                            dst.data_ptr(), _i64(dst.stride()), _DTYPES[dst.dtype],
                                            layer, _i64_ptr(b), _i64_ptr(o), n, heads, head_dim)
    if err is not None:
        raise err


def write_paged_kv_torch_loop(pool_k, pool_v, allocator: RefBlockAllocator, layer: int, table: RefBlockTable,
                              position_ids: torch.Tensor, key: torch.Tensor, value: torch.Tensor) -> None:
    """augur/paged_kv_cache.py:188-192 as the reference runs it: a Python loop over the tokens
    with one torch row assignment per token for K and one for V. Used to time the reference's
    own CPU path on hosts where the reference package is not installed; the C restatement
    (write_paged_kv above) is the checker."""
    for token_idx, position in enumerate(position_ids[0].tolist()):
        table.ensure_position(position, allocator)
        physical_block, offset = table.position_to_block_offset(position)
        pool_k[layer, physical_block, :, offset, :] = key[0, :, token_idx, :]
        pool_v[layer, physical_block, :, offset, :] = value[0, :, token_idx, :]


def read_paged_kv(pool_k, pool_v, layer: int, table: RefBlockTable, seq_len: int | None = None):
    """augur/paged_kv_cache.py:207-221."""
    if seq_len is None:
        seq_len = table.seq_len
    if seq_len <= 0:
        raise ValueError("seq_len must be positive")
    if math.ceil(seq_len / table.block_size) > len(table.block_ids):
        raise ValueError("position exceeds block table capacity")
    heads, head_dim = pool_k.shape[2], pool_k.shape[4]
    ids = np.asarray(table.block_ids, dtype=np.int64)
    outs = []
    for pool in (pool_k, pool_v):
        out = torch.empty(1, heads, seq_len, head_dim, dtype=pool.dtype)
        lib().oracle_read_paged(_cpu(pool).data_ptr(), _i64(pool.stride()), _DTYPES[pool.dtype], layer,
                                _i64_ptr(ids), table.block_size, seq_len, out.data_ptr(),
                                _i64(out.stride()), heads, head_dim)
        outs.append(out)
    return outs[0], outs[1]


def copy_prefix_into_cache(entry_k, entry_v, cache_k, cache_v, batch_idx: int = 0) -> None:
    """augur/prefix_cache.py:66-73 (shape checks are the caller's)."""
    layers, heads, prefix_len, head_dim = entry_k.shape
    for src, dst in ((entry_k, cache_k), (entry_v, cache_v)):
        src, dst = _cpu(src), _cpu(dst)
        lib().oracle_copy_prefix(src.data_ptr(), _i64(src.stride()), _DTYPES[src.dtype], dst.data_ptr(),
                                 _i64(dst.stride()), _DTYPES[dst.dtype], batch_idx, prefix_len,
                                 layers, heads, head_dim)


def scatter_slots(src_k, src_v, slots: np.ndarray, pool_k, pool_v, block_size: int,
                  threads: int = 1) -> None:
    """write_paged_kv over all layers of [layers, tokens, heads, dim] by resolved slot."""
    layers, tokens, heads, head_dim = src_k.shape
    slots = np.ascontiguousarray(slots, dtype=np.int64)
    sstr = _i64((src_k.stride(0), src_k.stride(1), src_k.stride(2)))
    pstr = _i64((pool_k.stride(0), pool_k.stride(1), pool_k.stride(2), pool_k.stride(3)))
    assert src_v is None or src_v.stride() == src_k.stride()
    assert pool_v is None or pool_v.stride() == pool_k.stride()
    lib().oracle_scatter_slots(_cpu(src_k).data_ptr(), None if src_v is None else _cpu(src_v).data_ptr(),
                               sstr, _cpu(pool_k).data_ptr(),
                               None if pool_v is None else _cpu(pool_v).data_ptr(), pstr,
                               src_k.element_size(), _i64_ptr(slots), block_size, layers, tokens,
                               heads, head_dim, int(threads))


def copy_runs(src_k, src_v, dst_k, dst_v, runs: np.ndarray, threads: int = 1) -> None:
    """Row runs between two (layers, major, heads, rows, dim) caches of one dtype."""
    runs = np.ascontiguousarray(runs, dtype=np.int32).reshape(-1, 5)
    layers, _, heads, _, head_dim = src_k.shape
    assert src_k.dtype == dst_k.dtype
    st = lambda t: _i64((t.stride(0), t.stride(1), t.stride(2), t.stride(3)))  # noqa: E731
    lib().oracle_copy_runs(_cpu(src_k).data_ptr(), None if src_v is None else _cpu(src_v).data_ptr(),
                           st(src_k), _cpu(dst_k).data_ptr(),
                           None if dst_v is None else _cpu(dst_v).data_ptr(), st(dst_k),
                           src_k.element_size(), runs.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                           runs.shape[0], layers, heads, head_dim, int(threads))


def poison_(t: torch.Tensor) -> torch.Tensor:
    """Fill every byte with 0xFF (a NaN pattern for every float dtype); in place."""
    t.view(torch.uint8).fill_(0xFF)
    return t


def bits(t: torch.Tensor) -> torch.Tensor:
    """Bit view for exact comparison (NaNs and -0 compare by bits)."""
    return t.contiguous().view(torch.int16 if t.element_size() == 2 else torch.int32)


# ---------------------------------------------------------------------------
# decode attention over a paged cache (floating point; torch on CPU)
# ---------------------------------------------------------------------------


def decode_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """Attention of one decode query per sequence, restating augur/attention.py:74-86.

    q [B, Hq, 1, D] (after RoPE), k / v [B, Hkv, S, D] (the cache gathered in
    logical order, read_paged_kv). K/V heads are repeated for the query heads
    of their group; scores are q k^T / sqrt(D) in the input dtype; the
    softmax runs in float32 and its result is cast back before the product
    with V. The decode query is the last position, so the causal mask
    (attention.py:80-81) hides nothing.
    """
    groups = q.shape[1] // k.shape[1]
    k = k.repeat_interleave(groups, dim=1)
    v = v.repeat_interleave(groups, dim=1)
    scores = torch.matmul(q, k.transpose(-2, -1)) / math.sqrt(q.shape[-1])
    probs = torch.softmax(scores, dim=-1, dtype=torch.float32).to(q.dtype)
    return torch.matmul(probs, v)


def prefill_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """Attention of a call's n query tokens over the whole cached sequence, restating
    augur/attention.py:74-86 with _causal_mask (:15-19).

    q [B, Hq, n, D] (after RoPE), k / v [B, Hkv, S, D] (read_paged_kv: the cache
    in logical order, the n new tokens last). Query i sits at position
    S - n + i (past_len = key_len - query_len) and key positions above it are
    masked with -inf before the float32 softmax; otherwise as decode_attention.
    """
    groups = q.shape[1] // k.shape[1]
    k = k.repeat_interleave(groups, dim=1)
    v = v.repeat_interleave(groups, dim=1)
    scores = torch.matmul(q, k.transpose(-2, -1)) / math.sqrt(q.shape[-1])
    n, S = q.shape[2], k.shape[2]
    query_positions = torch.arange(n).unsqueeze(-1) + (S - n)
    key_positions = torch.arange(S).unsqueeze(0)
    scores = scores.masked_fill(key_positions > query_positions, float("-inf"))
    probs = torch.softmax(scores, dim=-1, dtype=torch.float32).to(q.dtype)
    return torch.matmul(probs, v)


def rope_inv_freq(head_dim: int, rope_theta: float) -> torch.Tensor:
    """augur/rope.py:29-32: 1 / theta^(arange(0, D, 2) / D), float32."""
    return 1.0 / (rope_theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))


def _agreeing(fn, attempts: int = 4):
    """fn()'s tuple of tensors, computed until two computations agree bit for bit.

    A long vectorised torch CPU loop on the GPU hosts has been seen to return,
    rarely, a run of slightly wrong values (the same call repeated is exact);
    the checker's floating-point tables and rotations must not inherit them.
    """
    def same(a, b):
        return a.shape == b.shape and a.dtype == b.dtype and torch.equal(
            a.contiguous().view(torch.uint8), b.contiguous().view(torch.uint8))

    first = fn()
    for _ in range(attempts):
        second = fn()
        if all(same(a, b) for a, b in zip(first, second)):
            return first
        first = second
    raise RuntimeError("oracle: the host's floating-point results disagree between attempts")


def rope_table(head_dim: int, rope_theta: float, n_positions: int, dtype: torch.dtype):
    """cos / sin [n_positions, head_dim // 2] in `dtype`, as augur/rope.py:33-36 forms them
    for positions 0..n_positions-1 (float32 angles, cos/sin in float32, cast); computed
    until two computations agree (_agreeing)."""
    def once():
        freqs = torch.arange(n_positions, dtype=torch.float32).unsqueeze(-1) * rope_inv_freq(head_dim, rope_theta)
        return freqs.cos().to(dtype), freqs.sin().to(dtype)

    return _agreeing(once)


def apply_rope(q: torch.Tensor, k: torch.Tensor, position_ids: torch.Tensor, rope_theta: float,
               table: tuple[torch.Tensor, torch.Tensor] | None = None):
    """Restates augur/rope.py:12-40 on the CPU: x * cos + rotate_half(x) * sin, every op in
    the input dtype. q [B, Hq, S, D], k [B, Hkv, S, D], position_ids [B, S].

    table=None computes cos/sin from the positions exactly as the reference does;
    a (cos, sin) table [P, D/2] (rope_table) is indexed by position instead, which
    is what the kernel consumes.
    """
    q, k, position_ids = _cpu(q), _cpu(k), _cpu(position_ids)
    head_dim = q.shape[-1]

    def rotate_half(x):
        half = x.shape[-1] // 2
        return torch.cat((-x[..., half:], x[..., :half]), dim=-1)

    def once():
        if table is None:
            freqs = position_ids.to(torch.float32).unsqueeze(-1) * rope_inv_freq(head_dim, rope_theta)
            emb = torch.cat((freqs, freqs), dim=-1)
            cos = emb.cos().unsqueeze(1).to(q.dtype)
            sin = emb.sin().unsqueeze(1).to(q.dtype)
        else:
            c, s = table[0][position_ids.long()], table[1][position_ids.long()]
            cos = torch.cat((c, c), dim=-1).unsqueeze(1).to(q.dtype)
            sin = torch.cat((s, s), dim=-1).unsqueeze(1).to(q.dtype)
        return (q * cos) + (rotate_half(q) * sin), (k * cos) + (rotate_half(k) * sin)

    return _agreeing(once)
