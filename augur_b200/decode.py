"""Batched paged decode: the KV-cache side of augur's attention for one new token per sequence.

augur's paged branch (augur/attention.py:53-86 with paged_cache) runs for a
batch of one (paged_kv_cache.py:179-180, generation.py:35-40). Per layer it
rotates q and k (apply_rope), writes the token through the block table
(write_paged_kv), gathers the whole sequence back (read_paged_kv), repeats
the KV heads and attends. Here a whole batch does the same in one launch per
layer: the decode attention kernel reads every sequence straight from the
pool, rotates q and the new k itself, uses the new k and v for the token's
row and writes them to its slot (bf16 / fp16, head_dim 64 or 128). Other
shapes take two launches: the RoPE write (augur_kv_rope_scatter), then the
attention (augur_kv_paged_decode_attention).

The host work of a step (growing each table by one position, the slot
mapping, the device tables) is done once per step in DecodeStep and shared
by all layers. So is everything the launch needs apart from the layer's
own tensors: the checks, the RoPE table, the attention counters and scratch,
gathered in one argument block (augur_kv_decode_args). A layer is then one
foreign call, augur_kv_decode_layer. The
projections and everything after the attention core stay the model's.
"""

from __future__ import annotations

import ctypes
from collections.abc import Sequence

import numpy as np
import torch
from torch import Tensor

from . import _lib, _ops
from .attention import DecodeTables, _table_rows, _workspace, paged_decode_attention, upload_int32, workspace_bytes
from .batched import decode_slot_mapping
from .paged_kv_cache import PagedKVCache, SequenceBlockTable
from .rope import rope_tables, write_paged_kv_batch_rope


class DecodeStep:
    """One decode step of a batch: each table grows by one position (allocating a block when
    it crosses a boundary, as ensure_position does), and the step's slots, positions and
    device block tables are built once for all layers."""

    def __init__(self, cache: PagedKVCache, tables: Sequence[SequenceBlockTable], early_reads: bool = False) -> None:
        """early_reads: the one-launch layers read the lengths, block tables and pool before the
        kernel ahead of them on the stream has finished (AUGUR_KV_ATTN_EARLY_READS). Valid
        when no kernel that may still run at a layer's launch writes them: the model's
        projections and the previous layer's launch do not; a prefill write or copy-on-write
        of the pool issued just before the first layer does."""
        device = cache.keys.device
        self.flags = _lib.ATTN_AUTO | (_lib.ATTN_EARLY_READS if early_reads else 0)
        positions = [t.seq_len for t in tables]
        slots = decode_slot_mapping(tables, cache.allocator)  # seq_len += 1 for every table
        B = self.batch = len(tables)
        self.max_position = max(positions, default=0)
        # one copy for the step: positions and slots (int64, as pairs of int32), then the
        # block tables and lengths as DecodeTables lays them out
        lens = [t.seq_len for t in tables]
        host, width = _table_rows(tables, lens, 4 * B)
        head = host[: 4 * B].view(np.int64)
        head[:B] = positions
        head[B:] = slots
        dev = upload_int32(host, device)
        pairs = dev[: 4 * B].view(torch.int64) if B else torch.empty(0, dtype=torch.int64, device=device)
        self.positions, self.slots = pairs[:B], pairs[B:]
        self.tables = DecodeTables.__new__(DecodeTables)
        self.tables._set(dev, 4 * B, tables, lens, width)
        # the copy is ordered on the current stream; a layer launched on another waits for it
        self.uploaded: torch.cuda.Event | None = None
        if device.type == "cuda":
            self.uploaded = torch.cuda.Event()
            self.uploaded.record(torch.cuda.current_stream(device))
        self._fast: tuple | None = None  # launch arguments shared by the layers, built on first use

    def _prepare(self, cache: PagedKVCache, q: Tensor, key: Tensor, value: Tensor,
                 rope_theta: float) -> tuple | None:
        """The argument block every layer of this step shares (augur_kv_decode_args) and the
        input signature it was built for, or None when the inputs need the general path."""
        if q.dim() != 4 or key.dim() != 4 or value.dim() != 4:
            return None
        L, NB, Hkv, bs, D = cache.keys.shape
        B, Hq = q.shape[0], q.shape[1]
        dev, dt = cache.keys.device, cache.keys.dtype
        ok = (B == self.batch and B > 0 and self.tables.block_size == bs and Hq % Hkv == 0
              and tuple(q.shape) == (B, Hq, 1, D) and tuple(key.shape) == (B, Hkv, 1, D)
              and value.shape == key.shape and value.stride() == key.stride()
              and q.stride(-1) == 1 and key.stride(-1) == 1
              and q.dtype == dt and key.dtype == dt and value.dtype == dt
              and q.device == dev and key.device == dev and value.device == dev
              and cache.keys.stride() == cache.values.stride())
        if not ok:
            return None
        lib = _lib.load()
        cos, sin = rope_tables(D, rope_theta, dt, self.max_position + 1, dev)
        st = torch.cuda.current_stream(dev)
        if self.uploaded is not None:
            st.wait_event(self.uploaded)  # every prepared launch is on st
        dcode = _ops.dtype_code(q)
        cnt, scr = _workspace(lib, dev, st, (B, Hq, Hkv, D, self.tables.max_seq_len, dcode, _lib.ATTN_AUTO))
        q_rot = torch.empty(B, Hq, D, dtype=dt, device=dev)  # reused by every layer, stream-ordered
        status = _ops.status_word(dev)
        kc = cache.keys
        a = _lib.DecodeArgs()
        a.k_pool, a.v_pool = kc.data_ptr(), cache.values.data_ptr()
        a.pool_strides[:] = kc.stride()[:4]  # layer, block, kv head, row
        a.num_blocks, a.block_size, a.n_layers = NB, bs, L
        a.n_q_heads, a.n_kv_heads, a.head_dim, a.dtype, a.batch, a.flags = Hq, Hkv, D, dcode, B, self.flags
        a.slots, a.positions = self.slots.data_ptr(), self.positions.data_ptr()
        a.rope_cos, a.rope_sin, a.rope_positions = cos.data_ptr(), sin.data_ptr(), cos.shape[0]
        a.q_strides[:] = q.stride()[:2]
        a.kv_strides[:] = key.stride()[:2]
        a.q_rot = q_rot.data_ptr()
        blocks = self.tables.blocks
        a.block_tables, a.tables_stride, a.max_blocks = blocks.data_ptr(), blocks.stride(0), blocks.shape[1]
        a.seq_lens, a.max_seq_len = self.tables.lens.data_ptr(), self.tables.max_seq_len
        a.counters, a.counters_bytes = (cnt.data_ptr(), cnt.numel() * 4) if cnt is not None else (None, 0)
        a.scratch, a.scratch_bytes = (scr.data_ptr(), scr.numel()) if scr is not None else (None, 0)
        a.status = status.data_ptr()
        sig = _signature(q, key, value)
        # the tensors the argument block points into stay referenced with it
        return (lib, st.cuda_stream, ctypes.addressof(a), sig, a, cache, cos, sin, q_rot, cnt, scr, status,
                rope_theta)

    def layer(self, cache: PagedKVCache, layer_idx: int, q: Tensor, key: Tensor, value: Tensor,
              rope_theta: float) -> Tensor | None:
        """paged_decode_layer's work as one augur_kv_decode_layer call with the step's
        prepared arguments, on the current stream; None when the inputs need the general path
        (anything other than the shapes, strides, dtypes, devices, cache and stream the
        arguments were prepared for, or a layer outside the cache)."""
        f = self._fast
        if f is None or f[-1] != rope_theta or f[5] is not cache:
            f = self._fast = self._prepare(cache, q, key, value, rope_theta)
            if f is None:
                return None
        if _signature(q, key, value) != f[3]:
            return None
        lib, stream = f[0], f[1]
        dev = cache.keys.device
        if not 0 <= layer_idx < f[4].n_layers or _current_raw_stream(dev) != stream:
            return None
        # q's shape, dtype and device (the signature holds them to the prepared ones), contiguous;
        # empty_like skips torch.empty's device-argument parsing, a few us of every layer's host time
        out = torch.empty_like(q, memory_format=torch.contiguous_format)
        code = lib.augur_kv_decode_layer(f[2], layer_idx, q.data_ptr(), key.data_ptr(), value.data_ptr(),
                                         out.data_ptr(), stream)
        _lib.check(code, "augur_kv_decode_layer")
        _ops.launch_count += f[4].launches
        return out


def _signature(q: Tensor, key: Tensor, value: Tensor) -> tuple:
    """What the prepared arguments of a step assume about a layer's inputs."""
    return (q.shape, q.stride(), q.dtype, q.get_device(), key.shape, key.stride(), key.dtype, key.get_device(),
            value.shape, value.stride(), value.dtype, value.get_device())


class DecodeGraphStep:
    """A decode step whose device state lives in fixed buffers, for CUDA-graph replay.

    DecodeStep uploads each step's slots, positions and block tables into new
    tensors, which a captured graph cannot follow. Here they live in buffers
    sized once for `batch` sequences of up to `max_blocks` blocks, and so does
    everything else the launches read (the RoPE table for every position the
    tables can hold, a private attention workspace, the rotated-q buffer): the
    argument block never changes. update() grows each table by one position
    and refreshes the buffers, one host-to-device copy each on the current
    stream; layer() issues augur_kv_decode_layer. A graph captured over
    layer() calls (the model's own ops between them) therefore replays
    correctly after every later update(). Rows past len(tables) are padding:
    slot -1 (nothing written), length 0 (a zero output).
    """

    def __init__(self, cache: PagedKVCache, batch: int, max_blocks: int, n_q_heads: int,
                 rope_theta: float, early_reads: bool = False) -> None:
        """early_reads: as DecodeStep's."""
        _ops.require_cuda("DecodeGraphStep", cache.keys, cache.values)
        L, NB, Hkv, bs, D = cache.keys.shape
        if batch <= 0 or max_blocks <= 0 or n_q_heads <= 0 or n_q_heads % Hkv != 0:
            raise ValueError("batch and max_blocks must be positive, n_q_heads a multiple of the KV heads")
        if cache.keys.stride() != cache.values.stride():
            raise ValueError("keys and values must share one layout")
        dev, dt = cache.keys.device, cache.keys.dtype
        self.cache, self.batch, self.max_blocks, self.rope_theta = cache, batch, max_blocks, rope_theta
        self.capacity = max_blocks * bs  # longest sequence the buffers describe
        lib = _lib.load()
        self._lib = lib
        with _ops._DeviceGuard(dev):
            self._h64 = torch.empty(2, batch, dtype=torch.int64).pin_memory()  # slots, positions
            self._h32 = torch.empty(batch * (max_blocks + 1), dtype=torch.int32).pin_memory()  # lens, tables
            self._d64 = torch.empty(2, batch, dtype=torch.int64, device=dev)
            self._d32 = torch.empty(batch * (max_blocks + 1), dtype=torch.int32, device=dev)
            self._cos, self._sin = rope_tables(D, rope_theta, dt, self.capacity, dev)
            dcode = _ops.dtype_code(cache.keys)
            need_c, need_s = workspace_bytes(lib, (batch, n_q_heads, Hkv, D, self.capacity, dcode, _lib.ATTN_AUTO))
            self._cnt = torch.zeros(max(1, -(-need_c // 4)), dtype=torch.int32, device=dev)
            self._scr = torch.empty(max(16, need_s), dtype=torch.uint8, device=dev)
            self._q_rot = torch.empty(batch, n_q_heads, D, dtype=dt, device=dev)
            self._status = _ops.status_word(dev)
        self._copied: torch.cuda.Event | None = None
        self._rows: list[list[int] | None] = [None] * batch  # block ids each staging row holds
        a = self._args = _lib.DecodeArgs()
        kc = cache.keys
        a.k_pool, a.v_pool = kc.data_ptr(), cache.values.data_ptr()
        a.pool_strides[:] = kc.stride()[:4]
        a.num_blocks, a.block_size, a.n_layers = NB, bs, L
        a.n_q_heads, a.n_kv_heads, a.head_dim, a.dtype, a.batch = n_q_heads, Hkv, D, dcode, batch
        a.flags = _lib.ATTN_AUTO | (_lib.ATTN_EARLY_READS if early_reads else 0)
        a.slots, a.positions = self._d64[0].data_ptr(), self._d64[1].data_ptr()
        a.rope_cos, a.rope_sin, a.rope_positions = self._cos.data_ptr(), self._sin.data_ptr(), self._cos.shape[0]
        a.q_strides[:] = (n_q_heads * D, D)  # dense [batch, n_q_heads, 1, head_dim]
        a.kv_strides[:] = (Hkv * D, D)
        a.q_rot = self._q_rot.data_ptr()
        a.block_tables, a.tables_stride, a.max_blocks = self._d32[batch:].data_ptr(), max_blocks, max_blocks
        a.seq_lens, a.max_seq_len = self._d32.data_ptr(), self.capacity
        a.counters, a.counters_bytes = self._cnt.data_ptr(), self._cnt.numel() * 4
        a.scratch, a.scratch_bytes = self._scr.data_ptr(), self._scr.numel()
        a.status = self._status.data_ptr()
        self._addr = ctypes.addressof(a)
        self._shapes = ((batch, n_q_heads, 1, D), (batch, Hkv, 1, D))

    def update(self, tables: Sequence[SequenceBlockTable]) -> None:
        """Grow each table by one position (allocating a block when it crosses a boundary)
        and copy the step's slots, positions, lengths and block tables to the device."""
        n, bs = len(tables), self.cache.block_size
        if n > self.batch:
            raise ValueError(f"{n} tables for a step of at most {self.batch} sequences")
        for t in tables:
            if t.block_size != bs:
                raise ValueError("block table block_size must equal the cache block size")
            if t.seq_len >= self.capacity:
                raise ValueError(f"a sequence would grow past the step's capacity of {self.capacity} positions")
        if self._copied is not None:
            self._copied.synchronize()  # the previous step's copies have left the staging buffers
        positions = [t.seq_len for t in tables]
        slots = decode_slot_mapping(tables, self.cache.allocator)
        h64 = self._h64.numpy()
        h64[0, :n], h64[0, n:] = slots, -1
        h64[1, :n], h64[1, n:] = positions, 0
        h32 = self._h32.numpy()
        lens, blocks = h32[: self.batch], h32[self.batch :].reshape(self.batch, self.max_blocks)
        lens[:n], lens[n:] = [t.seq_len for t in tables], 0
        # the staging buffer keeps the rows it was given: a row is rewritten only
        # when its table's block ids differ from what it holds (a block appended,
        # a copied last block, another sequence in the row), which spares the
        # conversion of every id on every step
        for b in range(self.batch):
            ids = tables[b].block_ids[: self.max_blocks] if b < n else []  # positions below capacity
            if self._rows[b] != ids:
                blocks[b].fill(-1)
                blocks[b, : len(ids)] = ids
                self._rows[b] = ids
        dev = self.cache.keys.device
        with _ops._DeviceGuard(dev):
            self._d64.copy_(self._h64, non_blocking=True)
            self._d32.copy_(self._h32, non_blocking=True)
            self._copied = torch.cuda.Event()
            self._copied.record(torch.cuda.current_stream(dev))

    def layer(self, layer_idx: int, q: Tensor, key: Tensor, value: Tensor) -> Tensor:
        """One layer of the step on the current stream (graph-capturable): q ``[batch,
        n_q_heads, 1, head_dim]``, key / value ``[batch, kv_heads, 1, head_dim]``, contiguous,
        before RoPE. Returns the attention output ``[batch, n_q_heads, 1, head_dim]``."""
        dev = self.cache.keys.device
        dt = self.cache.keys.dtype
        for t, shape in ((q, self._shapes[0]), (key, self._shapes[1]), (value, self._shapes[1])):
            if tuple(t.shape) != shape or not t.is_contiguous() or t.dtype != dt or t.get_device() != dev.index:
                raise ValueError(f"decode inputs must be contiguous {dt} tensors of shape {shape} on {dev}")
        if not 0 <= layer_idx < self._args.n_layers:
            raise ValueError("layer_idx is outside the cache layer range")
        with _ops._DeviceGuard(dev):
            out = torch.empty(q.shape, dtype=dt, device=dev)
            code = self._lib.augur_kv_decode_layer(self._addr, layer_idx, q.data_ptr(), key.data_ptr(),
                                                   value.data_ptr(), out.data_ptr(),
                                                   torch.cuda.current_stream(dev).cuda_stream)
        _lib.check(code, "augur_kv_decode_layer")
        _ops.launch_count += self._args.launches
        return out


# torch.cuda.current_device() without its lazy-init check: the step that asks has
# already launched on the device
_cuda_device = getattr(torch._C, "_cuda_getDevice", None) or torch.cuda.current_device
_cuda_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _current_raw_stream(dev: torch.device) -> int:
    """Handle of the current stream on dev (0 when dev is not the current device, which sends
    the caller to the general path)."""
    if dev.index != _cuda_device():
        return 0
    if _cuda_raw_stream is not None:
        return _cuda_raw_stream(dev.index)
    return torch.cuda.current_stream(dev).cuda_stream


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
    if stream is None:  # the step's prepared launch when the inputs are the ones it was prepared for
        out = step.layer(cache, layer_idx, q, key, value, rope_theta)
        if out is not None:
            return out
    if step.uploaded is not None:  # the step's slots, positions and tables, on whichever stream
        (stream if stream is not None else torch.cuda.current_stream(cache.keys.device)).wait_event(step.uploaded)
    B = step.batch
    for name, t in (("q", q), ("key", key), ("value", value)):
        if t.dim() != 4 or t.shape[0] != B or t.shape[2] != 1:
            raise ValueError(f"{name} must be [batch, heads, 1, head_dim] with one token per sequence")
    q_rot = write_paged_kv_batch_rope(cache, q[:, :, 0], key[:, :, 0], value[:, :, 0], step.slots, step.positions,
                                      rope_theta, layer_idx, max_position=step.max_position, stream=stream)
    return paged_decode_attention(q_rot, cache, layer_idx, step.tables, stream=stream).unsqueeze(2)
