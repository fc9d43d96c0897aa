"""Disaggregated prefill -> decode: push finished KV blocks to another GPU's pool.

A decode rank exports its block pool (export_pool); a prefill rank opens it
(open_pool: the pool's memory is mapped into the prefill GPU's address space
with CUDA IPC, peer access enabled as needed) and pushes blocks with
push_blocks: one augur_kv_copy_runs launch on the prefill GPU that reads its
local blocks and stores 16-byte vectors straight into the peer pool over
NVLink, every layer, K and V. Block ids on the destination come from the
decode rank's own allocator; tables travel as host data.

No reference counterpart: augur runs in one process on one device. The
result is defined as equal, byte for byte, to writing the same tokens into
the destination pool locally (tests/test_gpu_peer.py checks exactly that).
"""

from __future__ import annotations

import ctypes
from collections.abc import Sequence
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib, _ops
from .batched import split_runs
from .paged_kv_cache import PagedKVCache


@dataclass
class ExportedPool:
    """Picklable description of a pool (and its ready flags) another process can open."""

    key_handle: bytes
    key_offset: int
    value_handle: bytes
    value_offset: int
    shape: tuple[int, ...]
    stride: tuple[int, ...]
    dtype: str
    device_index: int
    block_size: int
    flags_handle: bytes | None = None
    flags_offset: int = 0
    n_flags: int = 0


def new_flags(device: torch.device, n: int = 16) -> torch.Tensor:
    """Ready flags (int32, zero) a decode rank exports with its pool."""
    return torch.zeros(n, dtype=torch.int32, device=device)


def _export(t: torch.Tensor) -> tuple[bytes, int]:
    lib = _lib.load()
    handle = ctypes.create_string_buffer(_lib.IPC_HANDLE_BYTES)
    off = ctypes.c_int64(0)
    with _ops._DeviceGuard(t.device):
        _lib.check(lib.augur_kv_ipc_export(t.data_ptr(), handle, ctypes.byref(off)), "augur_kv_ipc_export")
    return handle.raw, int(off.value)


def export_pool(cache: PagedKVCache, flags: torch.Tensor | None = None) -> ExportedPool:
    _ops.require_cuda("export_pool", cache.keys, cache.values, flags)
    if cache.keys.stride() != cache.values.stride():
        raise ValueError("keys and values must share one layout")
    kh, ko = _export(cache.keys)
    vh, vo = _export(cache.values)
    fh, fo, nf = None, 0, 0
    if flags is not None:
        if flags.dtype != torch.int32 or not flags.is_contiguous():
            raise ValueError("flags must be a contiguous int32 tensor")
        fh, fo = _export(flags)
        nf = flags.numel()
    return ExportedPool(kh, ko, vh, vo, tuple(cache.keys.shape), tuple(cache.keys.stride()),
                        str(cache.keys.dtype).replace("torch.", ""), cache.keys.device.index,
                        cache.block_size, fh, fo, nf)


class PeerPool:
    """Another process's pool, mapped into this process's current CUDA device.

    Keys and values may live in one allocation (torch's caching allocator
    packs small tensors into shared segments); each distinct allocation is
    opened once and both addresses are derived from it.
    """

    def __init__(self, exported: ExportedPool, device: torch.device) -> None:
        self.exported = exported
        self.device = device
        self.shape = exported.shape
        self.stride = exported.stride
        self.dtype = getattr(torch, exported.dtype)
        self.block_size = exported.block_size
        self._bases: dict[bytes, int] = {}
        lib = _lib.load()
        handles = {exported.key_handle, exported.value_handle}
        if exported.flags_handle is not None:
            handles.add(exported.flags_handle)
        with _ops._DeviceGuard(device):
            for h in handles:
                out = ctypes.c_void_p()
                _lib.check(lib.augur_kv_ipc_open(h, 0, ctypes.byref(out)), "augur_kv_ipc_open")
                self._bases[h] = int(out.value)
        self.keys_ptr = self._bases[exported.key_handle] + exported.key_offset
        self.values_ptr = self._bases[exported.value_handle] + exported.value_offset
        self.flags_ptr = 0
        self.n_flags = exported.n_flags
        if exported.flags_handle is not None:
            self.flags_ptr = self._bases[exported.flags_handle] + exported.flags_offset

    def close(self) -> None:
        lib = _lib.load()
        with _ops._DeviceGuard(self.device):
            for h, base in list(self._bases.items()):
                _lib.check(lib.augur_kv_ipc_close(base, 0), "augur_kv_ipc_close")
                del self._bases[h]
        self.keys_ptr = self.values_ptr = self.flags_ptr = 0


def open_pool(exported: ExportedPool, device: torch.device | None = None) -> PeerPool:
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    return PeerPool(exported, device)


@dataclass
class PreparedPush:
    """A push whose run list is already on the prefill GPU: launching it moves no host data."""

    src: PagedKVCache
    dst: PeerPool
    runs: torch.Tensor  # int32 [n_runs, 5] on the source device, each run at most max_rows rows
    max_rows: int
    payload_bytes: int


def prepare_push(src: PagedKVCache, dst: PeerPool, runs: np.ndarray) -> PreparedPush:
    """Check the two pools against each other, cut the runs {src_block, src_row, dst_block,
    dst_row, n_rows} to the copy's row limit and upload them once (for pushes repeated with the
    same blocks, or issued from inside a CUDA graph)."""
    L, NB, H, bs, D = src.keys.shape
    if dst.shape[0] != L or dst.shape[2] != H or dst.shape[4] != D or dst.dtype != src.keys.dtype:
        raise ValueError("source and destination pools have different layer/head/dim/dtype")
    max_rows = _ops.max_rows_for(D, src.keys.element_size(), cap_rows=max(bs, dst.block_size))
    runs = split_runs(np.asarray(runs, dtype=np.int64).reshape(-1, 5), max_rows)
    runs_t = torch.from_numpy(np.ascontiguousarray(runs, dtype=np.int32)).to(src.keys.device)
    payload = int(runs[:, 4].astype(np.int64).sum()) * L * 2 * H * D * src.keys.element_size()
    return PreparedPush(src, dst, runs_t, max_rows, payload)


def push_prepared(p: PreparedPush, stream: torch.cuda.Stream | None = None) -> int:
    """Launch a prepared push on the source GPU (one kernel); returns the payload bytes moved."""
    if p.runs.shape[0] == 0:
        return 0
    src, dst = p.src, p.dst
    L, NB, H, bs, D = src.keys.shape
    lib = _lib.load()
    device = src.keys.device
    st = stream if stream is not None else torch.cuda.current_stream(device)
    sk = src.keys
    s_str = (sk.stride(0), sk.stride(1), sk.stride(3), sk.stride(2))
    d = dst.stride
    d_str = (d[0], d[1], d[3], d[2])
    with _ops._DeviceGuard(device):
        code = lib.augur_kv_copy_runs(
            sk.data_ptr(), src.values.data_ptr(), _lib.i64_array(s_str), NB, bs, _ops.dtype_code(sk),
            dst.keys_ptr, dst.values_ptr, _lib.i64_array(d_str), dst.shape[1], dst.shape[3],
            _ops.dtype_code(sk), p.runs.data_ptr(), p.runs.shape[0], p.max_rows, L, H, D,
            # plain stores to peer memory (no bulk/TMA path), each thread
            # ending with a system-scope fence so a later signal() cannot
            # become visible on the peer before the data
            _lib.COPY_VECTOR | _lib.COPY_FENCE_SYSTEM,
            _ops.status_word(device).data_ptr(), st.cuda_stream)
    _lib.check(code, "augur_kv_copy_runs (peer push)")
    _ops.launch_count += 1
    return p.payload_bytes


def push_runs(src: PagedKVCache, dst: PeerPool, runs: np.ndarray, stream: torch.cuda.Stream | None = None) -> int:
    """Copy row runs {src_block, src_row, dst_block, dst_row, n_rows} from a local pool into the peer pool.

    One launch on this process's device; returns the payload bytes moved.
    """
    p = prepare_push(src, dst, runs)
    if p.runs.shape[0] == 0:
        return 0
    st = stream if stream is not None else torch.cuda.current_stream(src.keys.device)
    moved = push_prepared(p, stream=st)
    _ops.keep_until_done(st, p.runs)
    return moved


def push_blocks(src: PagedKVCache, src_blocks: Sequence[int], dst: PeerPool, dst_blocks: Sequence[int],
                n_rows: Sequence[int] | None = None, stream: torch.cuda.Stream | None = None) -> int:
    """Push whole (or the first n_rows rows of) blocks src_blocks[i] -> dst_blocks[i]."""
    if len(src_blocks) != len(dst_blocks):
        raise ValueError("src_blocks and dst_blocks must have the same length")
    n = len(src_blocks)
    runs = np.zeros((n, 5), dtype=np.int64)
    runs[:, 0] = np.asarray(src_blocks, dtype=np.int64)
    runs[:, 2] = np.asarray(dst_blocks, dtype=np.int64)
    runs[:, 4] = src.block_size if n_rows is None else np.asarray(n_rows, dtype=np.int64)
    return push_runs(src, dst, runs, stream=stream)


def signal(dst: PeerPool, value: int, index: int = 0, stream: torch.cuda.Stream | None = None) -> None:
    """Release-store `value` into the peer's ready flag `index`, after the work already on `stream`."""
    if not dst.flags_ptr:
        raise ValueError("the peer pool was exported without ready flags")
    if not 0 <= index < dst.n_flags:
        raise ValueError("flag index out of range")
    lib = _lib.load()
    st = stream if stream is not None else torch.cuda.current_stream(dst.device)
    with _ops._DeviceGuard(dst.device):
        _lib.check(lib.augur_kv_signal(dst.flags_ptr + 4 * index, int(value), st.cuda_stream), "augur_kv_signal")
    _ops.launch_count += 1


def wait(flags: torch.Tensor, value: int, timeout_s: float = 10.0, index: int = 0,
         stream: torch.cuda.Stream | None = None) -> None:
    """Order work queued after this on `stream` behind flags[index] >= value (device side).

    The wait gives up after timeout_s and records AUGUR_KV_ETIMEOUT in the
    device status word (augur_b200.check_status() raises on it); it never
    blocks the host. The signaller must run on another GPU.
    """
    _ops.require_cuda("wait", flags)
    if flags.dtype != torch.int32 or not 0 <= index < flags.numel():
        raise ValueError("flags must be int32 and index inside it")
    lib = _lib.load()
    device = flags.device
    st = stream if stream is not None else torch.cuda.current_stream(device)
    with _ops._DeviceGuard(device):
        _lib.check(lib.augur_kv_wait(flags[index:].data_ptr(), int(value), int(timeout_s * 1e9),
                                     _ops.status_word(device).data_ptr(), st.cuda_stream), "augur_kv_wait")
    _ops.launch_count += 1
