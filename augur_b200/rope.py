"""Rotary position embedding fused with the KV-cache write.

augur rotates q and k (apply_rope, augur/rope.py:12-40) and then writes k and
v into its cache (augur/attention.py:53-71): three dtype elementwise ops per
rotated tensor, then a separate copy. The functions here do both in one
augur_kv_rope_scatter launch per call: q is rotated into a new tensor, k is
rotated straight into its cache slot, v is copied.

The cos/sin tables are built on the host with torch exactly as the reference
builds them (float32 angles, cos/sin in float32, cast to the dtype), for
positions 0..n-1, and kept on the device per (device, dtype, head_dim, theta).
With them the kernel's rounding matches the reference op for op, so the
rotated q and the cached k are bit-exact with apply_rope on the same CPU
table. Build the tables before a CUDA-graph capture (any call with the
largest position does it, or rope_tables()).
"""

from __future__ import annotations

from collections.abc import Sequence

import numpy as np
import torch
from torch import Tensor

from . import _lib, _ops
from .kv_cache import KVCache, keep_last_per_row, position_range
from .paged_kv_cache import PagedKVCache, SequenceBlockTable, ensure_positions, keep_last, slots_for_positions

_tables: dict[tuple, tuple[Tensor, Tensor]] = {}


def rope_tables(head_dim: int, rope_theta: float, dtype: torch.dtype, n_positions: int,
                device: torch.device) -> tuple[Tensor, Tensor]:
    """Device cos / sin tables ``[P, head_dim // 2]`` covering positions ``0..n_positions-1``.

    P is n_positions rounded up to a power of two (at least 4096); a table
    is rebuilt only when a larger position arrives. Angles follow
    augur/rope.py:29-36: inv_freq = 1 / theta^(arange(0, D, 2) / D),
    angle = position * inv_freq, all float32 on the CPU, then cos / sin cast to
    the dtype.
    """
    if head_dim % 2 != 0:
        raise ValueError(f"head_dim must be even for RoPE, got {head_dim}")
    key = (device, dtype, int(head_dim), float(rope_theta))
    entry = _tables.get(key)
    if entry is None or entry[0].shape[0] < n_positions:
        size = 4096
        while size < n_positions:
            size *= 2
        cos, sin = _host_tables(head_dim, rope_theta, size)
        entry = (cos.to(dtype).to(device), sin.to(dtype).to(device))
        _tables[key] = entry
    return entry


def _host_tables(head_dim: int, rope_theta: float, size: int, attempts: int = 4) -> tuple[Tensor, Tensor]:
    """float32 cos / sin [size, head_dim // 2] on the host, accepted only when two
    computations agree bit for bit.

    On the GPU hosts a long vectorised torch CPU loop has been seen to return, now
    and then, a contiguous run of slightly wrong values (errors growing with the
    angle, up to 1e-4; the same call repeated is exact). A table built from such
    a run would put rotated keys 1 ulp off the reference's, so the table is
    computed twice and recomputed until both agree.
    """
    def once() -> tuple[Tensor, Tensor]:
        inv_freq = 1.0 / (rope_theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
        freqs = torch.arange(size, dtype=torch.float32).unsqueeze(-1) * inv_freq
        return freqs.cos(), freqs.sin()

    first = once()
    for _ in range(attempts):
        second = once()
        if torch.equal(first[0], second[0]) and torch.equal(first[1], second[1]):
            return first
        first = second
    raise RuntimeError("rope_tables: the host's cos / sin computations disagree between attempts")


def _positions_i64(position_ids: Tensor | np.ndarray, device: torch.device) -> Tensor:
    if isinstance(position_ids, np.ndarray):
        return torch.from_numpy(np.ascontiguousarray(position_ids, dtype=np.int64)).to(device)
    if position_ids.device != device or position_ids.dtype != torch.int64:
        return position_ids.to(device=device, dtype=torch.int64)
    return position_ids


def _last_dim_contiguous(t: Tensor) -> Tensor:
    return t if t.stride(-1) == 1 else t.contiguous()


def rope_scatter(
    *,
    q: Tensor | None,
    q_strides: Sequence[int],
    q_out: Tensor | None,
    q_out_strides: Sequence[int],
    n_q_heads: int,
    key: Tensor,
    value: Tensor | None,
    key_strides: Sequence[int],
    value_strides: Sequence[int] | None,
    tokens_per_row: int,
    dst_k: Tensor,
    dst_v: Tensor | None,
    dst_strides: Sequence[int],
    rows_per_major: int,
    num_majors: int,
    index: Tensor,
    index_strides: Sequence[int],
    index_row_base: int,
    positions: Tensor,
    position_strides: Sequence[int],
    rope_theta: float,
    max_position: int,
    n_tokens: int,
    n_layers: int,
    n_heads: int,
    head_dim: int,
    stream: torch.cuda.Stream | None = None,
) -> None:
    """Launch augur_kv_rope_scatter (element strides, as the header documents)."""
    _ops.require_cuda("rope_scatter", key, value, dst_k, dst_v, index, positions, q, q_out)
    if index.dtype != torch.int64 or positions.dtype != torch.int64:
        raise ValueError("rope_scatter index and positions must be int64")
    dtypes = {t.dtype for t in (key, value, dst_k, dst_v, q, q_out) if t is not None}
    if len(dtypes) != 1:
        raise ValueError("rope_scatter needs one dtype for q, k, v and the cache")
    device = dst_k.device
    cos, sin = rope_tables(head_dim, rope_theta, key.dtype, max_position + 1, device)
    lib = _lib.load()
    st = stream if stream is not None else torch.cuda.current_stream(device)
    with _ops._DeviceGuard(device):
        code = lib.augur_kv_rope_scatter(
            key.data_ptr(), value.data_ptr() if value is not None else None,
            _lib.i64_array(key_strides), _lib.i64_array(value_strides if value is not None else key_strides),
            int(tokens_per_row), _ops.dtype_code(key),
            dst_k.data_ptr(), dst_v.data_ptr() if dst_v is not None else None, _lib.i64_array(dst_strides),
            int(rows_per_major), int(num_majors),
            index.data_ptr(), _lib.i64_array(index_strides), int(index_row_base),
            positions.data_ptr(), _lib.i64_array(position_strides),
            cos.data_ptr(), sin.data_ptr(), int(cos.shape[0]),
            q.data_ptr() if q is not None else None, _lib.i64_array(q_strides),
            q_out.data_ptr() if q_out is not None else None, _lib.i64_array(q_out_strides), int(n_q_heads),
            int(n_tokens), int(n_layers), int(n_heads), int(head_dim),
            _ops.status_word(device).data_ptr(), st.cuda_stream)
    _lib.check(code, "augur_kv_rope_scatter")
    _ops.launch_count += 1
    _ops.keep_until_done(st, key, value, index, positions, q, cos, sin)


def rope_write_paged_kv(
    cache: PagedKVCache,
    layer_idx: int,
    block_table: SequenceBlockTable,
    position_ids: Tensor,
    q: Tensor,
    key: Tensor,
    value: Tensor,
    rope_theta: float,
) -> Tensor:
    """``q, k = apply_rope(q, k, position_ids, theta)`` then ``write_paged_kv(cache, layer_idx,
    block_table, position_ids, k, value)`` in one launch; returns the rotated q.

    q ``[1, heads, seq, head_dim]``, key/value ``[1, kv_heads, seq, head_dim]``
    (augur/attention.py:53,64-71). Checks, messages, lazy block allocation and
    the partial write on a capacity error are write_paged_kv's
    (augur/paged_kv_cache.py:167-192); apply_rope's head_dim check is kept.
    """
    if key.shape != value.shape:
        raise ValueError("key and value must have the same shape")
    batch, num_heads, seq, head_dim = key.shape
    if q.dim() != 4 or q.shape[0] != batch or q.shape[2] != seq or q.shape[3] != head_dim:
        raise ValueError("q must be [batch, heads, seq, head_dim] matching key")
    if head_dim % 2 != 0:
        raise ValueError(f"head_dim must be even for RoPE, got {head_dim}")
    if batch != 1:
        raise ValueError("paged KV cache currently supports batch size 1")
    if position_ids.shape != (batch, seq):
        raise ValueError("position_ids must have shape [batch, seq]")
    if not 0 <= layer_idx < cache.keys.shape[0]:
        raise ValueError("layer_idx is outside the cache layer range")
    if (num_heads, head_dim) != (cache.keys.shape[2], cache.keys.shape[4]):
        raise ValueError("key/value shape does not match cache shape")
    _ops.require_cuda("rope_write_paged_kv", cache.keys, cache.values)
    device = cache.keys.device
    host_pos = np.asarray(position_ids[0].tolist(), dtype=np.int64)
    if seq and int(host_pos.min()) < 0:
        raise ValueError("position ids must be non-negative for RoPE")
    n_ok, err = ensure_positions(block_table, host_pos, cache.allocator)
    if block_table.block_size > cache.keys.shape[3]:
        raise IndexError("block table block_size exceeds the cache block size")
    slots = np.full(seq, -1, dtype=np.int64)
    if n_ok:
        slots[:n_ok] = keep_last(slots_for_positions(block_table, host_pos[:n_ok]))
    q, key, value = (_last_dim_contiguous(t.to(device)) for t in (q, key, value))
    q_out = torch.empty_like(q)
    kc, vc = cache.keys[layer_idx], cache.values[layer_idx]
    if seq:
        rope_scatter(
            q=q, q_strides=(0, 0, q.stride(2), q.stride(1)), q_out=q_out,
            q_out_strides=(0, 0, q_out.stride(2), q_out.stride(1)), n_q_heads=q.shape[1],
            key=key[0], value=value[0], key_strides=(0, 0, key.stride(2), key.stride(1)),
            value_strides=(0, 0, value.stride(2), value.stride(1)), tokens_per_row=seq,
            dst_k=kc, dst_v=vc, dst_strides=(0, kc.stride(0), kc.stride(2), kc.stride(1)),
            rows_per_major=block_table.block_size, num_majors=kc.shape[0],
            index=torch.from_numpy(slots).to(device), index_strides=(0, 1), index_row_base=0,
            positions=torch.from_numpy(host_pos).to(device), position_strides=(0, 1),
            rope_theta=rope_theta, max_position=int(host_pos.max()), n_tokens=seq, n_layers=1,
            n_heads=num_heads, head_dim=head_dim)
    if err is not None:
        raise err
    return q_out


def rope_write_kv(
    cache: KVCache,
    layer_idx: int,
    position_ids: Tensor,
    q: Tensor,
    key: Tensor,
    value: Tensor,
    rope_theta: float,
) -> tuple[Tensor, Tensor, Tensor]:
    """``q, k = apply_rope(q, k, position_ids, theta)`` then ``k, v = write_kv(cache,
    layer_idx, position_ids, k, value)`` in one launch (augur/attention.py:53-60).

    Returns (rotated q, cache key view, cache value view) with write_kv's
    checks, messages and return views (augur/kv_cache.py:75-112).
    """
    if key.shape != value.shape:
        raise ValueError("key and value must have the same shape")
    batch, num_heads, seq, head_dim = key.shape
    if q.dim() != 4 or q.shape[0] != batch or q.shape[2] != seq or q.shape[3] != head_dim:
        raise ValueError("q must be [batch, heads, seq, head_dim] matching key")
    if head_dim % 2 != 0:
        raise ValueError(f"head_dim must be even for RoPE, got {head_dim}")
    expected = cache.keys.shape
    if not 0 <= layer_idx < expected[0]:
        raise ValueError(f"layer_idx {layer_idx} is outside the cache layer range")
    if position_ids.shape != (batch, seq):
        raise ValueError("position_ids must have shape [batch, seq]")
    if (batch, num_heads, head_dim) != (expected[1], expected[2], expected[4]):
        raise ValueError("key/value shape does not match cache shape")
    if key.device != cache.keys.device or value.device != cache.values.device:
        raise ValueError("key/value tensors must be on the same device as the cache")
    _ops.require_cuda("rope_write_kv", cache.keys, cache.values, q)
    max_position, min_position, repeats = position_range(position_ids)
    if min_position < 0:
        raise ValueError("cache positions must be non-negative")
    if max_position >= cache.max_seq_len:
        raise ValueError("position_ids exceeds cache capacity")
    for src, dst in ((key, cache.keys), (value, cache.values)):
        if src.dtype != dst.dtype:
            raise RuntimeError("Index put requires the source and destination dtypes match, got "
                               f"{dst.dtype} for the destination and {src.dtype} for the source.")
    device = cache.keys.device
    q, key, value = (_last_dim_contiguous(t) for t in (q, key, value))
    q_out = torch.empty_like(q)
    pos = _positions_i64(position_ids, device)
    # a repeated position keeps the later token (write_kv's rule); every q is still rotated
    idx = _positions_i64(keep_last_per_row(position_ids), device) if repeats else pos
    kc, vc = cache.keys[layer_idx], cache.values[layer_idx]
    if seq and batch:
        rope_scatter(
            q=q, q_strides=(0, q.stride(0), q.stride(2), q.stride(1)), q_out=q_out,
            q_out_strides=(0, q_out.stride(0), q_out.stride(2), q_out.stride(1)), n_q_heads=q.shape[1],
            key=key, value=value, key_strides=(0, key.stride(0), key.stride(2), key.stride(1)),
            value_strides=(0, value.stride(0), value.stride(2), value.stride(1)), tokens_per_row=seq,
            dst_k=kc, dst_v=vc, dst_strides=(0, kc.stride(0), kc.stride(2), kc.stride(1)),
            rows_per_major=kc.shape[2], num_majors=kc.shape[0],
            index=idx, index_strides=(idx.stride(0), idx.stride(1)), index_row_base=kc.shape[2],
            positions=pos, position_strides=(pos.stride(0), pos.stride(1)),
            rope_theta=rope_theta, max_position=max_position, n_tokens=batch * seq, n_layers=1,
            n_heads=num_heads, head_dim=head_dim)
    cache.seq_len = max(cache.seq_len, max_position + 1)
    return (q_out, cache.keys[layer_idx, :, :, : cache.seq_len, :],
            cache.values[layer_idx, :, :, : cache.seq_len, :])


def write_paged_kv_batch_rope(
    cache: PagedKVCache,
    q: Tensor,
    key: Tensor,
    value: Tensor,
    slot_mapping: Tensor,
    positions: Tensor,
    rope_theta: float,
    layer_idx: int,
    max_position: int | None = None,
    stream: torch.cuda.Stream | None = None,
) -> Tensor:
    """Token-major batch form: rotate q ``[tokens, heads, D]`` and key ``[tokens, kv_heads, D]``
    by ``positions[t]``, write key/value to ``slot_mapping[t]`` of one layer (-1 skips the
    write, q is still rotated); returns the rotated q.

    max_position bounds the positions (sizes the cos/sin table); None reads
    it from the device (a host sync).
    """
    if key.shape != value.shape or key.dim() != 3 or q.dim() != 3 or q.shape[0] != key.shape[0]:
        raise ValueError("q [tokens, heads, D], key/value [tokens, kv_heads, D] expected")
    if not 0 <= layer_idx < cache.keys.shape[0]:
        raise ValueError("layer_idx is outside the cache layer range")
    n_tokens, num_heads, head_dim = key.shape
    if (num_heads, head_dim) != (cache.keys.shape[2], cache.keys.shape[4]) or q.shape[2] != head_dim:
        raise ValueError("key/value shape does not match cache shape")
    if tuple(slot_mapping.shape) != (n_tokens,) or tuple(positions.shape) != (n_tokens,):
        raise ValueError("slot_mapping and positions must have shape [tokens]")
    device = cache.keys.device
    q, key, value = (_last_dim_contiguous(t) for t in (q, key, value))
    q_out = torch.empty_like(q)
    if n_tokens == 0:
        return q_out
    slots = slot_mapping if slot_mapping.dtype == torch.int64 else slot_mapping.to(torch.int64)
    pos = _positions_i64(positions, device)
    if max_position is None:
        max_position = int(pos.max().item())
    kc, vc = cache.keys[layer_idx], cache.values[layer_idx]
    rope_scatter(
        q=q, q_strides=(0, 0, q.stride(0), q.stride(1)), q_out=q_out,
        q_out_strides=(0, 0, q_out.stride(0), q_out.stride(1)), n_q_heads=q.shape[1],
        key=key, value=value, key_strides=(0, 0, key.stride(0), key.stride(1)),
        value_strides=(0, 0, value.stride(0), value.stride(1)), tokens_per_row=n_tokens,
        dst_k=kc, dst_v=vc, dst_strides=(0, kc.stride(0), kc.stride(2), kc.stride(1)),
        rows_per_major=kc.shape[2], num_majors=kc.shape[0],
        index=slots, index_strides=(0, slots.stride(0)), index_row_base=0,
        positions=pos, position_strides=(0, pos.stride(0)),
        rope_theta=rope_theta, max_position=int(max_position), n_tokens=n_tokens, n_layers=1,
        n_heads=num_heads, head_dim=head_dim, stream=stream)
    return q_out
