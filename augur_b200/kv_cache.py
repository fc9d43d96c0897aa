"""Contiguous preallocated KV cache — drop-in for augur/kv_cache.py.

Layout and host semantics follow augur/kv_cache.py:9-112: K and V are
``[layers, batch, kv_heads, max_seq, head_dim]`` tensors allocated once with
torch.empty, ``seq_len`` is the high-water mark of written positions, and
write_kv returns views of the written prefix. The per-row index_put loop of
the reference (kv_cache.py:103-106) is one augur_kv_scatter launch here, with
the positions used directly as the index (no slot mapping to build).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch
from torch import Tensor

from . import _ops
from .config import QwenConfig


@dataclass
class KVCache:
    """K/V storage ``[layers, batch, kv_heads, max_seq, head_dim]`` (kv_cache.py:9-17)."""

    keys: Tensor
    values: Tensor
    seq_len: int = 0

    @property
    def max_seq_len(self) -> int:
        return self.keys.shape[3]


def new_kv_cache(
    cfg: QwenConfig,
    batch_size: int,
    max_seq_len: int,
    device: torch.device,
    dtype: torch.dtype,
) -> KVCache:
    """Allocate an uninitialised cache (kv_cache.py:20-37)."""
    shape = (
        cfg.num_hidden_layers,
        batch_size,
        cfg.num_key_value_heads,
        max_seq_len,
        cfg.head_dim,
    )
    return KVCache(
        keys=torch.empty(shape, device=device, dtype=dtype),
        values=torch.empty(shape, device=device, dtype=dtype),
    )


def kv_cache_nbytes(
    cfg: QwenConfig,
    batch_size: int,
    max_seq_len: int,
    dtype: torch.dtype,
) -> int:
    """Bytes of K plus V for a cache of this size (kv_cache.py:40-58)."""
    if batch_size <= 0:
        raise ValueError("batch_size must be positive")
    if max_seq_len <= 0:
        raise ValueError("max_seq_len must be positive")
    elements = (
        cfg.num_hidden_layers * batch_size * cfg.num_key_value_heads * max_seq_len * cfg.head_dim
    )
    return elements * torch.empty((), dtype=dtype).element_size() * 2


def format_bytes(nbytes: int) -> str:
    """Binary-unit size string with two decimals (kv_cache.py:61-72)."""
    if nbytes < 0:
        raise ValueError("nbytes must be non-negative")
    if nbytes < 1024:
        return f"{nbytes} B"
    value = float(nbytes)
    for unit in ("KiB", "MiB", "GiB", "TiB"):
        value /= 1024
        if abs(value) < 1024:
            return f"{value:.2f} {unit}"
    return f"{value:.2f} PiB"


_DTYPE_NAMES = {torch.float32: "Float", torch.float16: "Half", torch.bfloat16: "BFloat16",
                torch.float64: "Double"}


def _dtype_name(dtype: torch.dtype) -> str:
    return _DTYPE_NAMES.get(dtype, str(dtype).replace("torch.", ""))


def position_range(position_ids: Tensor) -> tuple[int, int, bool]:
    """(max, min, whether a batch row repeats a position) of ``[batch, seq]`` positions, with
    one host read of a device tensor (the reference reads max and min with two)."""
    seq = position_ids.shape[1]
    parts = [position_ids.max(), position_ids.min()]
    if seq > 1:
        srt = position_ids.sort(dim=1).values
        parts.append((srt[:, 1:] == srt[:, :-1]).any())
    vals = torch.stack([x.to(torch.int64) for x in parts]).tolist()
    return vals[0], vals[1], bool(vals[2]) if seq > 1 else False


def keep_last_per_row(position_ids: Tensor) -> Tensor:
    """Host int64 copy of ``[batch, seq]`` positions with every earlier repeat of a position
    within a row set to -1, so the last token written to a position is the one that stays
    (a negative index skips its token)."""
    rows = position_ids.detach().to("cpu", torch.int64).numpy()
    return torch.from_numpy(np.stack([_ops.keep_last(r) for r in rows]).astype(np.int64))


def _head_dim_contiguous(t: Tensor) -> Tensor:
    return t if t.stride(-1) == 1 else t.contiguous()


def write_kv(
    cache: KVCache,
    layer_idx: int,
    position_ids: Tensor,
    key: Tensor,
    value: Tensor,
) -> tuple[Tensor, Tensor]:
    """Write ``key``/``value`` ``[batch, kv_heads, seq, head_dim]`` at ``position_ids``.

    Same checks, messages and return value as augur's write_kv
    (kv_cache.py:75-112). Like the reference, reading the position range is a
    device->host sync when position_ids lives on the GPU; pass host
    position_ids to avoid it. Duplicate positions inside one batch row leave
    one of the duplicates' values (which one is unspecified, as for torch's
    CUDA index_put).
    """
    if key.shape != value.shape:
        raise ValueError("key and value must have the same shape")

    batch, num_heads, seq, head_dim = key.shape
    expected_shape = cache.keys.shape
    if not 0 <= layer_idx < expected_shape[0]:
        raise ValueError(f"layer_idx {layer_idx} is outside the cache layer range")
    if position_ids.shape != (batch, seq):
        raise ValueError("position_ids must have shape [batch, seq]")
    if (batch, num_heads, head_dim) != (expected_shape[1], expected_shape[2], expected_shape[4]):
        raise ValueError("key/value shape does not match cache shape")
    if key.device != cache.keys.device or value.device != cache.values.device:
        raise ValueError("key/value tensors must be on the same device as the cache")
    _ops.require_cuda("write_kv", cache.keys, cache.values)

    max_position, min_position, repeats = position_range(position_ids)
    if min_position < 0:
        raise ValueError("cache positions must be non-negative")
    if max_position >= cache.max_seq_len:
        raise ValueError("position_ids exceeds cache capacity")
    # The reference's index_put does not convert dtypes (kv_cache.py:105-106).
    for src, dst in ((key, cache.keys), (value, cache.values)):
        if src.dtype != dst.dtype:
            raise RuntimeError(
                "Index put requires the source and destination dtypes match, got "
                f"{_dtype_name(dst.dtype)} for the destination and {_dtype_name(src.dtype)} for the source."
            )

    scatter_rows(cache, layer_idx, keep_last_per_row(position_ids) if repeats else position_ids, key, value)

    cache.seq_len = max(cache.seq_len, max_position + 1)
    return (
        cache.keys[layer_idx, :, :, : cache.seq_len, :],
        cache.values[layer_idx, :, :, : cache.seq_len, :],
    )


def scatter_rows(
    cache: KVCache, layer_idx: int, position_ids: Tensor, key: Tensor, value: Tensor
) -> None:
    """One launch: token (b, s) of key/value goes to position position_ids[b, s] of row b.

    No validation beyond what the kernel bounds-checks; write_kv validates first.
    """
    device = cache.keys.device
    if position_ids.device.type == "cpu" and _ops.host_index_ok(position_ids.numel(), key, cache.keys):
        # few host positions (a decode step): passed to the kernel by value
        positions = np.ascontiguousarray(position_ids.numpy(), dtype=np.int64)
        index_strides = (positions.shape[1], 1)
    else:
        positions = position_ids
        if positions.device != device or positions.dtype != torch.int64:
            positions = positions.to(device=device, dtype=torch.int64)
        index_strides = (positions.stride(0), positions.stride(1))
    key = _head_dim_contiguous(key)
    value = _head_dim_contiguous(value)
    batch, num_heads, seq, head_dim = key.shape
    kc = cache.keys[layer_idx]
    vc = cache.values[layer_idx]
    if kc.stride(-1) != 1 or vc.stride(-1) != 1:
        raise ValueError("cache head_dim must be contiguous")
    # source (layer, row=batch, col=seq position, head); destination (layer,
    # major=batch, row=cache position, head); one layer per call.
    src_k_strides = (0, key.stride(0), key.stride(2), key.stride(1))
    src_v_strides = (0, value.stride(0), value.stride(2), value.stride(1))
    common = dict(
        tokens_per_row=seq,
        rows_per_major=cache.max_seq_len,
        num_majors=batch,
        index=positions,
        index_strides=index_strides,
        index_row_base=cache.max_seq_len,
        n_tokens=batch * seq,
        n_layers=1,
        n_heads=num_heads,
        head_dim=head_dim,
    )
    if kc.stride() == vc.stride() and key.dtype == value.dtype:
        _ops.scatter(
            src_k=key,
            src_v=value,
            src_k_strides=src_k_strides,
            src_v_strides=src_v_strides,
            dst_k=kc,
            dst_v=vc,
            dst_strides=(0, kc.stride(0), kc.stride(2), kc.stride(1)),
            **common,
        )
    else:
        for src, src_strides, dst in ((key, src_k_strides, kc), (value, src_v_strides, vc)):
            _ops.scatter(
                src_k=src,
                src_v=None,
                src_k_strides=src_strides,
                src_v_strides=None,
                dst_k=dst,
                dst_v=None,
                dst_strides=(0, dst.stride(0), dst.stride(2), dst.stride(1)),
                **common,
            )
