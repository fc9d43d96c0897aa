"""Batched paged decode: the KV-cache side of augur's attention for one new token per sequence.

augur's paged branch (augur/attention.py:53-86 with paged_cache) runs for a
batch of one (paged_kv_cache.py:179-180, generation.py:35-40). Per layer it
rotates q and k (apply_rope), writes the token through the block table
(write_paged_kv), gathers the whole sequence back (read_paged_kv), repeats
the KV heads and attends. Here a whole batch does the same in two launches
per layer:
- the fused RoPE write (augur_kv_rope_scatter): q rotated, k rotated into its
  slot, v copied;
- decode attention straight from the pool (augur_kv_paged_decode_attention)
  over every sequence including its new token.

The host work of a step (growing each table by one position, the slot
mapping, the device tables) is done once per step in DecodeStep and shared
by all layers. So is everything the two launches need apart from the layer's
own tensors: the checks, the RoPE table, the attention counters and scratch,
and the argument arrays. A layer is then two foreign calls. The projections
and everything after the attention core stay the model's.
"""

from __future__ import annotations

from collections.abc import Sequence

import numpy as np
import torch
from torch import Tensor

from . import _lib, _ops
from .attention import DecodeTables, _workspace, paged_decode_attention
from .batched import decode_slot_mapping
from .paged_kv_cache import PagedKVCache, SequenceBlockTable
from .rope import rope_tables, write_paged_kv_batch_rope


class DecodeStep:
    """One decode step of a batch: each table grows by one position (allocating a block when
    it crosses a boundary, as ensure_position does), and the step's slots, positions and
    device block tables are built once for all layers."""

    def __init__(self, cache: PagedKVCache, tables: Sequence[SequenceBlockTable]) -> None:
        device = cache.keys.device
        positions = np.asarray([t.seq_len for t in tables], dtype=np.int64)
        slots = decode_slot_mapping(tables, cache.allocator)  # seq_len += 1 for every table
        self.batch = len(tables)
        self.positions = torch.from_numpy(positions).to(device)
        self.slots = torch.from_numpy(slots).to(device)
        self.max_position = int(positions.max(initial=0))
        self.tables = DecodeTables(tables, device)
        self._fast: tuple | None = None  # launch arguments shared by the layers, built on first use

    def _prepare(self, cache: PagedKVCache, q: Tensor, key: Tensor, rope_theta: float) -> tuple:
        """Checks and launch arguments that every layer of this step shares, or None when the
        inputs need the general path."""
        L, NB, Hkv, bs, D = cache.keys.shape
        B, Hq = q.shape[0], q.shape[1]
        dev, dt = cache.keys.device, cache.keys.dtype
        ok = (B > 0 and self.tables.block_size == bs and Hq % Hkv == 0 and q.dtype == dt and key.dtype == dt
              and q.device == dev and key.device == dev and cache.keys.stride() == cache.values.stride()
              and q.shape[3] == D and key.shape[1] == Hkv and key.shape[3] == D)
        if not ok:
            return None
        lib = _lib.load()
        es = cache.keys.element_size()
        cos, sin = rope_tables(D, rope_theta, dt, self.max_position + 1, dev)
        st = torch.cuda.current_stream(dev)
        dcode = _ops.dtype_code(q)
        cnt, scr = _workspace(lib, dev, st, (B, Hq, Hkv, D, self.tables.max_seq_len, dcode, _lib.ATTN_AUTO))
        q_rot = torch.empty(B, Hq, D, dtype=dt, device=dev)  # reused by every layer, stream-ordered
        kc = cache.keys
        pool_str = _lib.i64_array((kc.stride(1), kc.stride(2), kc.stride(3)))
        dst_str = _lib.i64_array((0, kc.stride(1), kc.stride(3), kc.stride(2)))
        return (lib, st, dcode, cos, sin, cnt, scr, q_rot, pool_str, dst_str, kc.stride(0) * es,
                _ops.status_word(dev), (q.stride(), key.stride()), rope_theta)

    def layer(self, cache: PagedKVCache, layer_idx: int, q: Tensor, key: Tensor, value: Tensor,
              rope_theta: float) -> Tensor | None:
        """The two launches of paged_decode_layer with the step's prepared arguments, on the
        current stream; None when the inputs need the general path."""
        if self._fast is None or self._fast[-1] != rope_theta:
            self._fast = self._prepare(cache, q, key, rope_theta)
        f = self._fast
        if (f is None or (q.stride(), key.stride()) != f[12] or value.shape != key.shape
                or value.stride() != key.stride() or value.dtype != key.dtype):
            return None
        (lib, st, dcode, cos, sin, cnt, scr, q_rot, pool_str, dst_str, layer_bytes, status, _, _) = f
        dev = cache.keys.device
        if (dev.index != torch.cuda.current_device() or st != torch.cuda.current_stream(dev)
                or not 0 <= layer_idx < cache.keys.shape[0]):
            return None
        L, NB, Hkv, bs, D = cache.keys.shape
        B, Hq = q.shape[0], q.shape[1]
        koff, sh = layer_idx * layer_bytes, st.cuda_stream
        k_layer, v_layer = cache.keys.data_ptr() + koff, cache.values.data_ptr() + koff
        qs, ks = q.stride(), key.stride()
        out = torch.empty(B, Hq, 1, D, dtype=q.dtype, device=q.device)
        code = lib.augur_kv_rope_scatter(
            key.data_ptr(), value.data_ptr(), _lib.i64_array((0, 0, ks[0], ks[1])),
            _lib.i64_array((0, 0, ks[0], ks[1])), B, dcode, k_layer, v_layer, dst_str, bs, NB,
            self.slots.data_ptr(), _lib.i64_array((0, 1)), 0, self.positions.data_ptr(), _lib.i64_array((0, 1)),
            cos.data_ptr(), sin.data_ptr(), cos.shape[0], q.data_ptr(), _lib.i64_array((0, 0, qs[0], qs[1])),
            q_rot.data_ptr(), _lib.i64_array((0, 0, Hq * D, D)), Hq, B, 1, Hkv, D, status.data_ptr(), sh)
        _lib.check(code, "augur_kv_rope_scatter")
        code = lib.augur_kv_paged_decode_attention(
            q_rot.data_ptr(), _lib.i64_array((Hq * D, D)), k_layer, v_layer, pool_str, NB, bs,
            self.tables.blocks.data_ptr(), self.tables.blocks.stride(0), self.tables.blocks.shape[1],
            self.tables.lens.data_ptr(), self.tables.max_seq_len, B, Hq, Hkv, D, dcode,
            out.data_ptr(), _lib.i64_array((Hq * D, D)), _lib.ATTN_AUTO,
            cnt.data_ptr() if cnt is not None else None, cnt.numel() * 4 if cnt is not None else 0,
            scr.data_ptr() if scr is not None else None, scr.numel() if scr is not None else 0,
            status.data_ptr(), sh)
        _lib.check(code, "augur_kv_paged_decode_attention")
        _ops.launch_count += 2
        return out


def paged_decode_layer(
    step: DecodeStep,
    cache: PagedKVCache,
    layer_idx: int,
    q: Tensor,
    key: Tensor,
    value: Tensor,
    rope_theta: float,
    stream: torch.cuda.Stream | None = None,
) -> Tensor:
    """Attention core of one layer for the step's new tokens.

    q ``[batch, heads, 1, head_dim]``, key / value ``[batch, kv_heads, 1, head_dim]``:
    the new token's projections before RoPE, as augur/attention.py:33-51 forms
    them. Returns the attention output ``[batch, heads, 1, head_dim]`` (heads not
    yet concatenated, before the o-projection). The rotated k and v are in the
    cache afterwards, bit-exact with apply_rope + write_paged_kv.
    """
    B = step.batch
    for name, t in (("q", q), ("key", key), ("value", value)):
        if t.dim() != 4 or t.shape[0] != B or t.shape[2] != 1:
            raise ValueError(f"{name} must be [batch, heads, 1, head_dim] with one token per sequence")
        if t.device.type != "cuda" or t.stride(-1) != 1:
            break
    else:
        if stream is None:
            out = step.layer(cache, layer_idx, q, key, value, rope_theta)
            if out is not None:
                return out
    q_rot = write_paged_kv_batch_rope(cache, q[:, :, 0], key[:, :, 0], value[:, :, 0], step.slots, step.positions,
                                      rope_theta, layer_idx, max_position=step.max_position, stream=stream)
    return paged_decode_attention(q_rot, cache, layer_idx, step.tables, stream=stream).unsqueeze(2)
