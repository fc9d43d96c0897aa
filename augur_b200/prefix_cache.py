"""Whole-prefix KV cache — drop-in for augur/prefix_cache.py.

PrefixCache / PrefixCacheEntry are host bookkeeping identical to
augur/prefix_cache.py:13-50. copy_prefix_into_cache (prefix_cache.py:53-75)
moves an entry's ``[layers, kv_heads, P, head_dim]`` K/V into one batch row
of a contiguous cache with one augur_kv_copy_runs launch covering every
layer, head, K and V (converting dtype in the kernel when they differ).
cache_prefix needs augur's model; it is resolved from the installed augur
package when first called (module attribute ``model``, patchable in tests).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch
from torch import Tensor

from . import _ops
from .kv_cache import KVCache, new_kv_cache

# augur.model.model, looked up lazily by cache_prefix (the forward pass is not
# part of this package).
model = None


@dataclass
class PrefixCacheEntry:
    token_ids: Tensor
    keys: Tensor
    values: Tensor
    logits: Tensor

    @property
    def seq_len(self) -> int:
        return self.token_ids.shape[0]


class PrefixCache:
    """FIFO list of prefix entries with longest-prefix lookup (prefix_cache.py:25-50)."""

    def __init__(self, max_entries: int | None = None) -> None:
        if max_entries is not None and max_entries <= 0:
            raise ValueError("max_entries must be positive")
        self.max_entries = max_entries
        self._entries: list[PrefixCacheEntry] = []

    def add(self, entry: PrefixCacheEntry) -> None:
        self._entries.append(entry)
        if self.max_entries is not None and len(self._entries) > self.max_entries:
            del self._entries[0]

    def longest_prefix(self, input_ids: Tensor) -> PrefixCacheEntry | None:
        if input_ids.ndim != 2 or input_ids.shape[0] != 1:
            raise ValueError("prefix cache lookup currently supports batch size 1")
        best: PrefixCacheEntry | None = None
        tokens = input_ids[0].to(device="cpu")
        for entry in self._entries:
            if entry.seq_len > tokens.shape[0]:
                continue
            if torch.equal(tokens[: entry.seq_len], entry.token_ids.to(device="cpu")):
                if best is None or entry.seq_len > best.seq_len:
                    best = entry
        return best


def prefix_runs(prefix_len: int, batch_idx: int, max_rows: int) -> np.ndarray:
    """Runs copying rows [0, prefix_len) of a [P] row range into batch row batch_idx."""
    starts = np.arange(0, prefix_len, max_rows, dtype=np.int32)
    runs = np.zeros((starts.shape[0], 5), dtype=np.int32)
    runs[:, 1] = starts
    runs[:, 2] = batch_idx
    runs[:, 3] = starts
    runs[:, 4] = np.minimum(max_rows, prefix_len - starts)
    return runs


def copy_prefix_into_cache(entry: PrefixCacheEntry, cache: KVCache, batch_idx: int = 0) -> None:
    """Copy a prefix entry into ``cache`` at batch row ``batch_idx`` (prefix_cache.py:53-75)."""
    if not 0 <= batch_idx < cache.keys.shape[1]:
        raise ValueError("batch_idx is outside the cache batch range")
    if entry.seq_len > cache.max_seq_len:
        raise ValueError("prefix length exceeds cache capacity")
    expected_shape = (cache.keys.shape[0], cache.keys.shape[2], entry.seq_len, cache.keys.shape[4])
    if entry.keys.shape != expected_shape or entry.values.shape != expected_shape:
        raise ValueError("prefix key/value tensors do not match cache shape")
    _ops.require_cuda("copy_prefix_into_cache", cache.keys, cache.values)

    prefix_len = entry.seq_len
    if prefix_len > 0:
        device = cache.keys.device
        keys, values = entry.keys, entry.values
        # An entry in pinned host memory (offload_prefix_entry) is read in
        # place by the kernel; one on another device, or in pageable host
        # memory, is transferred first. The per-row copy and any dtype
        # conversion run in the kernel.
        pinned = all(t.device.type == "cpu" and t.is_pinned() for t in (keys, values))
        if not pinned:
            if keys.device != device:
                keys = keys.to(device)
            if values.device != device:
                values = values.to(device)
        if keys.stride(-1) != 1:
            keys = keys.contiguous()
        if values.stride(-1) != 1:
            values = values.contiguous()
        num_layers, num_heads, _, head_dim = keys.shape
        max_rows = _ops.max_rows_for(head_dim, max(keys.element_size(), cache.keys.element_size()))
        runs = torch.from_numpy(prefix_runs(prefix_len, batch_idx, max_rows)).to(device)
        kc, vc = cache.keys, cache.values
        dst = lambda t: (t.stride(0), t.stride(1), t.stride(3), t.stride(2))  # noqa: E731
        src = lambda t: (t.stride(0), 0, t.stride(2), t.stride(1))  # noqa: E731
        if keys.stride() == values.stride() and keys.dtype == values.dtype and kc.stride() == vc.stride():
            pairs = [(keys, values, kc, vc)]
        else:
            pairs = [(keys, None, kc, None), (values, None, vc, None)]
        for sk, sv, dk, dv in pairs:
            _ops.copy_runs(
                src_k=sk, src_v=sv, src_strides=src(sk), src_majors=1, src_rows_per_major=prefix_len,
                dst_k=dk, dst_v=dv, dst_strides=dst(dk),
                dst_majors=dk.shape[1], dst_rows_per_major=dk.shape[3],
                runs=runs, max_rows=max_rows, n_layers=num_layers, n_heads=num_heads,
                head_dim=head_dim, allow_pinned_host=pinned,
            )
    cache.seq_len = max(cache.seq_len, entry.seq_len)


def _entry_kv(cache: KVCache) -> tuple[Tensor, Tensor]:
    """Rows [0, seq_len) of batch row 0, every layer and head, copied out of the cache into
    fresh ``[layers, kv_heads, seq_len, head_dim]`` tensors by the run-copy kernel (one launch)."""
    kc, vc = cache.keys, cache.values
    L, B, H, S, D = kc.shape
    P = cache.seq_len
    keys = torch.empty(L, H, P, D, dtype=kc.dtype, device=kc.device)
    values = torch.empty(L, H, P, D, dtype=vc.dtype, device=vc.device)
    if P > 0:
        max_rows = _ops.max_rows_for(D, kc.element_size())
        runs = torch.from_numpy(prefix_runs(P, 0, max_rows)).to(kc.device)
        src = lambda t: (t.stride(0), t.stride(1), t.stride(3), t.stride(2))  # noqa: E731
        dst = lambda t: (t.stride(0), 0, t.stride(2), t.stride(1))  # noqa: E731
        if kc.stride() == vc.stride() and kc.dtype == vc.dtype:
            pairs = [(kc, vc, keys, values)]
        else:
            pairs = [(kc, None, keys, None), (vc, None, values, None)]
        for sk, sv, dk, dv in pairs:
            _ops.copy_runs(src_k=sk, src_v=sv, src_strides=src(sk), src_majors=B, src_rows_per_major=S,
                           dst_k=dk, dst_v=dv, dst_strides=dst(dk), dst_majors=1, dst_rows_per_major=P,
                           runs=runs, max_rows=max_rows, n_layers=L, n_heads=H, head_dim=D)
    return keys, values


def cache_prefix(input_ids: Tensor, w, cfg) -> PrefixCacheEntry:
    """Prefill ``input_ids`` with augur's model and keep its K/V (prefix_cache.py:78-98).

    The model's forward pass is augur's; the cache it fills is copied into the
    entry by the library's run-copy kernel, so input_ids must be on a CUDA
    device (CPU tensors raise ValueError, as every cache entry point here does).
    """
    if input_ids.ndim != 2 or input_ids.shape[0] != 1:
        raise ValueError("prefix caching currently supports batch size 1")
    if input_ids.shape[1] == 0:
        raise ValueError("prefix must contain at least one token")
    _ops.require_cuda("cache_prefix", input_ids)
    forward = model
    if forward is None:
        try:
            from augur.model import model as forward  # the host engine's forward pass
        except ImportError as exc:
            raise RuntimeError(
                "cache_prefix runs augur's model forward; install augur or set "
                "augur_b200.prefix_cache.model"
            ) from exc
    cache = new_kv_cache(
        cfg,
        batch_size=1,
        max_seq_len=input_ids.shape[1],
        device=input_ids.device,
        dtype=w.embed_tokens.dtype,
    )
    position_ids = torch.arange(input_ids.shape[1], device=input_ids.device).unsqueeze(0)
    logits = forward(input_ids, w, cfg, cache=cache, position_ids=position_ids)
    keys, values = _entry_kv(cache)
    return PrefixCacheEntry(
        token_ids=input_ids[0].detach().clone(),
        keys=keys,
        values=values,
        logits=logits[:, -1:, :].detach().clone(),
    )
