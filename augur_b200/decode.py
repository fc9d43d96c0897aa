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
by all layers. The projections and everything after the attention core stay
the model's.
"""

from __future__ import annotations

from collections.abc import Sequence

import numpy as np
import torch
from torch import Tensor

from .attention import DecodeTables, paged_decode_attention
from .batched import decode_slot_mapping
from .paged_kv_cache import PagedKVCache, SequenceBlockTable
from .rope import write_paged_kv_batch_rope


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
    q_rot = write_paged_kv_batch_rope(cache, q[:, :, 0], key[:, :, 0], value[:, :, 0], step.slots, step.positions,
                                      rope_theta, layer_idx, max_position=step.max_position, stream=stream)
    return paged_decode_attention(q_rot, cache, layer_idx, step.tables, stream=stream).unsqueeze(2)
