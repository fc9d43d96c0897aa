"""Decode attention that reads the paged KV pool in place.

augur's attention gathers the whole cached sequence out of the pool position
by position (read_paged_kv, augur/attention.py:72), repeats each KV head for
its query heads (:75-76) and runs q.k^T, a float32 softmax and P.V eagerly
(:78-86), one sequence and one layer at a time. paged_decode_attention does
the same computation for a decode step of a whole batch in one launch per
layer (augur_kv_paged_decode_attention), reading every K/V row once straight
from its block. Results match the reference's within floating-point
tolerance: the kernels round where the reference rounds (scores and
probabilities in the cache dtype, softmax in float32) but sum in another
order.
"""

from __future__ import annotations

import contextlib
import ctypes
from collections.abc import Sequence

import numpy as np
import torch
from torch import Tensor

from . import _lib, _ops
from .paged_kv_cache import PagedKVCache, SequenceBlockTable


# Counters (zeroed once; every launch leaves them zero) and scratch of the split
# kernel, one pair per (device, stream): launches on one stream run in order,
# so they can share them whatever their sizes.
_workspaces: dict[tuple[int, int], tuple[Tensor, Tensor]] = {}


_workspace_sizes: dict[tuple, tuple[int, int]] = {}


def workspace_bytes(lib, sizes: tuple) -> tuple[int, int]:
    """(counters, scratch) bytes augur_kv_paged_decode_attention needs for these sizes on the
    current device (cached per device and sizes)."""
    key = (torch.cuda.current_device(),) + tuple(sizes)
    got = _workspace_sizes.get(key)
    if got is None:
        cnt, scr = ctypes.c_int64(0), ctypes.c_int64(0)
        _lib.check(lib.augur_kv_paged_decode_attention_workspace(*sizes, ctypes.byref(cnt), ctypes.byref(scr)),
                   "augur_kv_paged_decode_attention_workspace")
        got = _workspace_sizes[key] = (cnt.value, scr.value)
    return got


def _workspace(lib, device: torch.device, st: torch.cuda.Stream, sizes: tuple) -> tuple[Tensor | None, Tensor | None]:
    """Counters and scratch tensors large enough for these sizes (None when not needed)."""
    need_c, need_s = workspace_bytes(lib, sizes)
    if need_c == 0 and need_s == 0:
        return None, None
    key = (device.index, st.cuda_stream)
    cnt, scr = _workspaces.get(key, (None, None))
    grow_c = cnt is None or cnt.numel() * 4 < need_c
    grow_s = need_s > 0 and (scr is None or scr.numel() < need_s)
    if grow_c or grow_s:
        with torch.cuda.stream(st):
            if grow_c:
                cnt = torch.zeros(max(1, -(-need_c // 4)), dtype=torch.int32, device=device)
            if grow_s:
                scr = torch.empty(need_s, dtype=torch.uint8, device=device)
        if not torch.cuda.is_current_stream_capturing():  # a graph owns what its capture allocates
            _workspaces[key] = (cnt, scr)
    return cnt, scr


class DecodeTables:
    """Device copy of a batch's block tables and lengths, reusable across layers.

    blocks: int32 [batch, max_blocks] (unused entries -1), lens: int32 [batch]: views of
    one device buffer filled by one copy (rows, then lengths).
    """

    def __init__(self, tables: Sequence[SequenceBlockTable], device: torch.device,
                 seq_lens: Sequence[int] | None = None, stream: torch.cuda.Stream | None = None) -> None:
        """stream: the stream the copy is ordered on (the current one by default); launches
        on another stream must wait for it."""
        lens = [t.seq_len for t in tables] if seq_lens is None else [int(n) for n in seq_lens]
        if len(lens) != len(tables):
            raise ValueError("seq_lens and tables must have the same length")
        host, width = _table_rows(tables, lens, 0)
        self._set(upload_int32(host, device, stream), 0, tables, lens, width)

    def _set(self, dev: Tensor, offset: int, tables: Sequence[SequenceBlockTable], lens: list[int],
             width: int) -> None:
        """Views of dev laid out as _table_rows packs them from int32 element `offset` on."""
        B = len(tables)
        self.blocks = dev[offset: offset + B * width].view(B, width)
        self.lens = dev[offset + B * width: offset + B * width + B]
        self.block_size = tables[0].block_size if tables else 1
        self.max_seq_len = max(lens, default=0)
        self.batch = B


def _table_rows(tables: Sequence[SequenceBlockTable], lens: list[int], offset: int) -> tuple[np.ndarray, int]:
    """An int32 host array of `offset` leading elements (left for the caller), then the block
    ids ``[batch, width]`` row by row (unused entries -1), then the lengths; and width.
    Checks that each length fits its table and that the tables share one block_size."""
    B = len(tables)
    width = max([len(t.block_ids) for t in tables] + [1])
    host = np.empty(offset + B * width + B, dtype=np.int32)
    rows = host[offset: offset + B * width].reshape(B, width)
    rows.fill(-1)
    for b, t in enumerate(tables):
        if lens[b] < 0 or -(-lens[b] // t.block_size) > len(t.block_ids):
            raise ValueError("position exceeds block table capacity")
        rows[b, : len(t.block_ids)] = _int32_row(t)
    host[offset + B * width:] = lens
    if any(t.block_size != tables[0].block_size for t in tables):
        raise ValueError("all block tables must share one block_size")
    return host, width


def _int32_row(t: SequenceBlockTable) -> np.ndarray:
    """t.block_ids as int32, converted again only when the list has changed. Converting
    Python ints is most of a batch's host work (about 35 ns an id), while a table gains at
    most one block a decode step; the table keeps its last conversion beside a copy of the
    list it was made from (a hidden attribute: not a field, so equality and repr ignore it),
    and comparing the list with that copy is all an unchanged table costs."""
    ids = t.block_ids
    kept = t.__dict__.get("_int32_ids")
    if kept is not None and kept[0] == ids:
        return kept[1]
    row = np.array(ids, dtype=np.int32)
    t.__dict__["_int32_ids"] = (list(ids), row)
    return row


def upload_int32(host: np.ndarray, device: torch.device, stream: torch.cuda.Stream | None = None) -> Tensor:
    """A 1-D int32 host array on device in one copy. To a GPU it goes through pinned memory
    as a copy ordered on `stream` (the current stream when None) that the host does not wait
    for: kernels on that stream see it, another stream must wait on that one first. The
    staging block is not reused before the copy has run (torch's pinned allocator records
    the copy)."""
    t = torch.from_numpy(host)
    if torch.device(device).type != "cuda" or t.numel() == 0:
        return t.to(device)
    with torch.cuda.stream(stream) if stream is not None else contextlib.nullcontext():
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("host data cannot be uploaded inside a CUDA graph capture: "
                               "build the device tables before capturing")
        return t.pin_memory().to(device, non_blocking=True)


def paged_decode_attention(
    q: Tensor,
    cache: PagedKVCache,
    layer_idx: int,
    tables: Sequence[SequenceBlockTable] | DecodeTables,
    out: Tensor | None = None,
    generic: bool = False,
    stream: torch.cuda.Stream | None = None,
    early_reads: bool = False,
) -> Tensor:
    """Attention of each sequence's decode query over its cached K/V (one layer).

    q: ``[batch, n_q_heads, head_dim]`` or ``[batch, n_q_heads, 1, head_dim]``
    (after RoPE), in the cache dtype. tables: one SequenceBlockTable per
    sequence (its seq_len positions are attended) or a prepared DecodeTables.
    Returns the attention output in q's shape (before the output projection,
    heads not yet concatenated). generic=True forces the CUDA-core kernel.
    early_reads=True lets the launch read the lengths, the block tables and
    the pool before the kernel ahead of it on the stream has finished
    (AUGUR_KV_ATTN_EARLY_READS): only when that kernel writes none of them,
    e.g. when it is the previous layer's attention.
    """
    squeeze = q.dim() == 4
    if squeeze:
        if q.shape[2] != 1:
            raise ValueError("paged_decode_attention takes one query token per sequence")
        q3 = q[:, :, 0, :]
    elif q.dim() == 3:
        q3 = q
    else:
        raise ValueError("q must be [batch, heads, head_dim] or [batch, heads, 1, head_dim]")
    _ops.require_cuda("paged_decode_attention", q3, cache.keys, cache.values)
    if not 0 <= layer_idx < cache.keys.shape[0]:
        raise ValueError("layer_idx is outside the cache layer range")
    L, NB, Hkv, bs, D = cache.keys.shape
    B, Hq, Dq = q3.shape
    if Dq != D or Hq % Hkv != 0:
        raise ValueError("query shape does not match the cache (head_dim, or heads not a multiple of KV heads)")
    if q3.dtype != cache.keys.dtype:
        raise ValueError("query and cache dtypes differ")
    if q3.stride(-1) != 1:
        q3 = q3.contiguous()
    dt = tables if isinstance(tables, DecodeTables) else DecodeTables(tables, cache.keys.device, stream=stream)
    if dt.batch != B:
        raise ValueError("one block table per sequence is required")
    if dt.block_size != bs:
        raise ValueError("block table block_size must equal the cache block size")
    if out is None:
        out3 = torch.empty(B, Hq, D, dtype=q3.dtype, device=q3.device)
    else:
        out3 = out[:, :, 0, :] if out.dim() == 4 else out
    if B == 0:
        return out if out is not None else (out3.unsqueeze(2) if squeeze else out3)
    kc, vc = cache.keys[layer_idx], cache.values[layer_idx]
    if kc.stride() != vc.stride():
        raise ValueError("keys and values must share one layout")
    lib = _lib.load()
    device = kc.device
    st = stream if stream is not None else torch.cuda.current_stream(device)
    kind = _lib.ATTN_GENERIC if generic else _lib.ATTN_AUTO
    flags = kind | (_lib.ATTN_EARLY_READS if early_reads else 0)
    dcode = _ops.dtype_code(q3)
    with _ops._DeviceGuard(device):
        cnt, scr = _workspace(lib, device, st, (B, Hq, Hkv, D, dt.max_seq_len, dcode, kind))
        code = lib.augur_kv_paged_decode_attention(
            q3.data_ptr(), _lib.i64_array((q3.stride(0), q3.stride(1))),
            kc.data_ptr(), vc.data_ptr(), _lib.i64_array((kc.stride(0), kc.stride(1), kc.stride(2))),
            NB, bs, dt.blocks.data_ptr(), dt.blocks.stride(0), dt.blocks.shape[1],
            dt.lens.data_ptr(), dt.max_seq_len, B, Hq, Hkv, D, dcode,
            out3.data_ptr(), _lib.i64_array((out3.stride(0), out3.stride(1))), flags,
            cnt.data_ptr() if cnt is not None else None, cnt.numel() * 4 if cnt is not None else 0,
            scr.data_ptr() if scr is not None else None, scr.numel() if scr is not None else 0,
            _ops.status_word(device).data_ptr(), st.cuda_stream)
    _lib.check(code, "augur_kv_paged_decode_attention")
    _ops.launch_count += 1
    _ops.keep_until_done(st, q3, dt.blocks, dt.lens, cnt, scr)
    if out is not None:
        return out
    return out3.unsqueeze(2) if squeeze else out3


class PrefillQueries:
    """Device copy of a batch's query-token counts, reusable across layers (and inside a
    CUDA graph, where no host data may be uploaded): starts int32 [batch + 1], sequence b's
    query tokens being rows [starts[b], starts[b + 1]) of q."""

    def __init__(self, q_lens: Sequence[int], device: torch.device,
                 stream: torch.cuda.Stream | None = None) -> None:
        """stream: the stream the copy is ordered on (the current one by default)."""
        lens = np.asarray(q_lens, dtype=np.int64)
        if lens.size and lens.min() < 0:
            raise ValueError("q_lens must be non-negative")
        starts = np.zeros(lens.size + 1, dtype=np.int32)
        np.cumsum(lens, out=starts[1:])
        self.lens = lens
        self.total = int(starts[-1])
        self.max_len = int(lens.max(initial=0))
        self.starts = upload_int32(starts, device, stream)


def paged_prefill_attention(
    q: Tensor,
    cache: PagedKVCache,
    layer_idx: int,
    tables: Sequence[SequenceBlockTable] | DecodeTables,
    q_lens: Sequence[int] | PrefillQueries,
    out: Tensor | None = None,
    generic: bool = False,
    stream: torch.cuda.Stream | None = None,
    kernel: str = "auto",
) -> Tensor:
    """Attention of a batch's new tokens over the pool (one layer, one launch).

    q: ``[tokens, n_q_heads, head_dim]`` after RoPE, the sequences' new tokens
    concatenated in table order (q_lens[b] of them for sequence b; pass a
    PrefillQueries, with a DecodeTables, to reuse both across layers). Each
    table's seq_len counts its cached positions with the new tokens included,
    so write them first (write_paged_kv_batch, or its RoPE form). New token i
    of sequence b sits at position seq_len - q_lens[b] + i and attends to
    positions [0, that position]: a plain prefill when q_lens[b] == seq_len, the
    suffix of a prompt whose prefix blocks were shared from the prefix index
    otherwise. Returns ``[tokens, n_q_heads, head_dim]`` (heads not yet
    concatenated). kernel: "auto" (the 5th-generation tensor cores with
    accumulators in tensor memory for bf16/fp16 at head_dim 64 or 128 with
    16-byte aligned rows, the mma.sync kernel for those shapes otherwise, CUDA
    cores for the rest), "tcgen05" or "mma_sync" (force one tensor-core
    kernel) or "generic" (CUDA cores, any dtype); generic=True is
    kernel="generic".
    """
    if kernel not in ("auto", "tcgen05", "mma_sync", "generic"):
        raise ValueError("kernel must be 'auto', 'tcgen05', 'mma_sync' or 'generic'")
    if q.dim() != 3:
        raise ValueError("q must be [tokens, n_q_heads, head_dim]")
    _ops.require_cuda("paged_prefill_attention", q, cache.keys, cache.values)
    if not 0 <= layer_idx < cache.keys.shape[0]:
        raise ValueError("layer_idx is outside the cache layer range")
    L, NB, Hkv, bs, D = cache.keys.shape
    T, Hq, Dq = q.shape
    if Dq != D or Hq % Hkv != 0:
        raise ValueError("query shape does not match the cache (head_dim, or heads not a multiple of KV heads)")
    if q.dtype != cache.keys.dtype:
        raise ValueError("query and cache dtypes differ")
    pq = q_lens if isinstance(q_lens, PrefillQueries) else PrefillQueries(q_lens, cache.keys.device, stream=stream)
    lens = pq.lens
    if pq.total != T:
        raise ValueError("q_lens must add up to the number of query tokens")
    dt = tables if isinstance(tables, DecodeTables) else DecodeTables(tables, cache.keys.device, stream=stream)
    if dt.batch != lens.size:
        raise ValueError("one block table per sequence is required")
    if dt.block_size != bs:
        raise ValueError("block table block_size must equal the cache block size")
    if not isinstance(tables, DecodeTables) and any(int(n) > t.seq_len for n, t in zip(lens, tables)):
        raise ValueError("a sequence has more query tokens than cached positions (write them first)")
    if q.stride(-1) != 1:
        q = q.contiguous()
    out3 = torch.empty(T, Hq, D, dtype=q.dtype, device=q.device) if out is None else out
    if tuple(out3.shape) != (T, Hq, D) or out3.stride(-1) != 1 or out3.dtype != q.dtype:
        raise ValueError("out must be a [tokens, n_q_heads, head_dim] tensor of q's dtype, head_dim contiguous")
    if T == 0:
        return out3
    kc, vc = cache.keys[layer_idx], cache.values[layer_idx]
    if kc.stride() != vc.stride():
        raise ValueError("keys and values must share one layout")
    lib = _lib.load()
    device = kc.device
    st = stream if stream is not None else torch.cuda.current_stream(device)
    q_starts = pq.starts
    flags = _lib.ATTN_GENERIC if generic or kernel == "generic" else {
        "tcgen05": _lib.ATTN_TCGEN05, "mma_sync": _lib.ATTN_MMA_SYNC}.get(kernel, _lib.ATTN_AUTO)
    with _ops._DeviceGuard(device):
        code = lib.augur_kv_paged_prefill_attention(
            q.data_ptr(), _lib.i64_array((q.stride(0), q.stride(1))),
            kc.data_ptr(), vc.data_ptr(), _lib.i64_array((kc.stride(0), kc.stride(1), kc.stride(2))),
            NB, bs, dt.blocks.data_ptr(), dt.blocks.stride(0), dt.blocks.shape[1],
            dt.lens.data_ptr(), q_starts.data_ptr(), lens.size, pq.max_len,
            max(dt.max_seq_len, 1), Hq, Hkv, D, _ops.dtype_code(q),
            out3.data_ptr(), _lib.i64_array((out3.stride(0), out3.stride(1))), flags,
            _ops.status_word(device).data_ptr(), st.cuda_stream)
    _lib.check(code, "augur_kv_paged_prefill_attention")
    _ops.launch_count += 1
    _ops.keep_until_done(st, q, dt.blocks, dt.lens, q_starts)
    return out3


def paged_attention(
    q: Tensor,
    cache: PagedKVCache,
    layer_idx: int,
    block_table: SequenceBlockTable,
    generic: bool = False,
    kernel: str = "auto",
) -> Tensor:
    """The attention core of augur's paged branch for one sequence (augur/attention.py:72-86)
    after its write: q ``[1, n_q_heads, seq, head_dim]`` (after RoPE) attends over the
    table's seq_len cached positions with the reference's causal mask (its seq query
    tokens are the last seq positions). Returns ``[1, n_q_heads, seq, head_dim]``; the
    pool is read in place (no read_paged_kv gather, no repeated KV heads)."""
    if q.dim() != 4 or q.shape[0] != 1:
        raise ValueError("paged KV cache currently supports batch size 1")
    out = paged_prefill_attention(q[0].transpose(0, 1).contiguous(), cache, layer_idx, [block_table], [q.shape[2]],
                                  generic=generic, kernel=kernel)
    return out.transpose(0, 1).unsqueeze(0)
