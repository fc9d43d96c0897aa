"""Tensor-level launchers for libaugur_kv.so.

These functions turn torch tensors (device memory owned by the caller) into
the raw pointers, element strides and stream the C ABI takes, and raise on a
non-zero status. They never allocate cache memory and never fall back to
torch indexing: a CPU tensor is a ValueError.
"""

from __future__ import annotations

from collections.abc import Sequence

import numpy as np
import torch
from torch import Tensor

from . import _lib

_DTYPE_CODES = {torch.float32: _lib.F32, torch.float16: _lib.F16, torch.bfloat16: _lib.BF16}

_status_words: dict[int, Tensor] = {}

# Number of launches issued through this module; bench and tests read it.
launch_count = 0


def dtype_code(t: Tensor) -> int:
    try:
        return _DTYPE_CODES[t.dtype]
    except KeyError:
        raise ValueError(
            f"unsupported KV cache dtype {t.dtype}; augur_b200 moves float32, float16 and bfloat16"
        ) from None


def require_cuda(what: str, *tensors: Tensor | None) -> None:
    for t in tensors:
        if t is not None and t.device.type != "cuda":
            raise ValueError(
                f"{what} needs CUDA tensors: augur_b200 moves KV-cache data only with its "
                f"sm_100a kernels and has no CPU fallback (got a tensor on {t.device})"
            )


def status_word(device: torch.device) -> Tensor:
    """The per-device int32 word kernels write their first error code into."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    word = _status_words.get(idx)
    if word is None:
        word = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _status_words[idx] = word
    return word


def read_status(device: torch.device | int | None = None, reset: bool = True) -> int:
    """Synchronise the device and return (and by default clear) its status word."""
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    elif isinstance(device, int):
        device = torch.device("cuda", device)
    word = status_word(device)
    torch.cuda.synchronize(device)
    code = int(word.item())
    if reset and code != 0:
        word.zero_()
    return code


def check_status(device: torch.device | int | None = None) -> None:
    """Raise KVLibraryError if a kernel on this device recorded an error."""
    code = read_status(device)
    if code != _lib.OK:
        raise _lib.KVLibraryError(
            f"a KV kernel recorded a device-side error: {_lib.STATUS_NAMES.get(code, code)}", code
        )


class _DeviceGuard:
    """Make `device` current for the duration of a launch if it is not already."""

    __slots__ = ("idx", "prev")

    def __init__(self, device: torch.device) -> None:
        self.idx = device.index if device.index is not None else torch.cuda.current_device()
        self.prev = -1

    def __enter__(self) -> None:
        cur = torch.cuda.current_device()
        if cur != self.idx:
            self.prev = cur
            torch.cuda.set_device(self.idx)

    def __exit__(self, *exc) -> None:
        if self.prev >= 0:
            torch.cuda.set_device(self.prev)


def _ptr(t: Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def keep_until_done(stream: torch.cuda.Stream, *tensors: Tensor | None) -> None:
    """Keep device tensors used by work on `stream` from being reused before it runs.

    Torch's caching allocator orders reuse on the stream a tensor was
    allocated on; for launches on another stream the tensor is recorded there.
    """
    current = None
    for t in tensors:
        if t is not None and t.device.type == "cuda":
            if current is None:
                current = torch.cuda.current_stream(t.device)
                if stream == current:
                    return  # the launch is on the stream the tensors' reuse is ordered on
            t.record_stream(stream)


def scatter(
    *,
    src_k: Tensor,
    src_v: Tensor | None,
    src_k_strides: Sequence[int],
    src_v_strides: Sequence[int] | None,
    tokens_per_row: int,
    dst_k: Tensor,
    dst_v: Tensor | None,
    dst_strides: Sequence[int],
    rows_per_major: int,
    num_majors: int,
    index: Tensor | np.ndarray,
    index_strides: Sequence[int],
    index_row_base: int,
    n_tokens: int,
    n_layers: int,
    n_heads: int,
    head_dim: int,
    stream: torch.cuda.Stream | None = None,
) -> None:
    """Launch augur_kv_scatter. Strides are element strides as the header documents.

    `index` is an int64 CUDA tensor, or an int64 numpy array in host memory
    holding at most INLINE_INDEX_MAX tokens' values (passed to the kernel by
    value; src and dst dtypes must then match).
    """
    global launch_count
    on_host = isinstance(index, np.ndarray)
    require_cuda("KV scatter", src_k, src_v, dst_k, dst_v, None if on_host else index)
    if index.dtype != (np.int64 if on_host else torch.int64):
        raise ValueError("scatter index must be int64")
    if on_host:
        index_ptr = index.ctypes.data
    else:
        index_ptr = index.data_ptr()
    lib = _lib.load()
    device = dst_k.device
    st = stream if stream is not None else torch.cuda.current_stream(device)
    with _DeviceGuard(device):
        code = lib.augur_kv_scatter(
            _ptr(src_k),
            _ptr(src_v),
            _lib.i64_array(src_k_strides),
            _lib.i64_array(src_v_strides if src_v_strides is not None else src_k_strides),
            int(tokens_per_row),
            dtype_code(src_k),
            _ptr(dst_k),
            _ptr(dst_v),
            _lib.i64_array(dst_strides),
            int(rows_per_major),
            int(num_majors),
            dtype_code(dst_k),
            index_ptr,
            _lib.i64_array(index_strides),
            int(index_row_base),
            1 if on_host else 0,
            int(n_tokens),
            int(n_layers),
            int(n_heads),
            int(head_dim),
            status_word(device).data_ptr(),
            st.cuda_stream,
        )
    _lib.check(code, "augur_kv_scatter")
    if n_tokens > 0 and n_layers > 0:
        launch_count += 1
        keep_until_done(st, None if on_host else index, src_k, src_v)


def copy_runs(
    *,
    src_k: Tensor,
    src_v: Tensor | None,
    src_strides: Sequence[int],
    src_majors: int,
    src_rows_per_major: int,
    dst_k: Tensor,
    dst_v: Tensor | None,
    dst_strides: Sequence[int],
    dst_majors: int,
    dst_rows_per_major: int,
    runs: Tensor,
    max_rows: int,
    n_layers: int,
    n_heads: int,
    head_dim: int,
    flags: int = _lib.COPY_AUTO,
    stream: torch.cuda.Stream | None = None,
    allow_pinned_host: bool = False,
) -> None:
    """Launch augur_kv_copy_runs; runs is a device int32 [n_runs, 5] tensor.

    allow_pinned_host: src or dst may be pinned host memory (the device reads
    or writes it in place over the host link, with the vector path's 16-byte
    accesses); the launch goes to the device of the CUDA-side tensor.
    """
    global launch_count
    if allow_pinned_host:
        host = [t for t in (src_k, src_v, dst_k, dst_v) if t is not None and t.device.type == "cpu"]
        if any(not t.is_pinned() for t in host):
            raise ValueError("host-side KV tensors must be in pinned memory (tensor.pin_memory())")
        require_cuda("KV block copy", runs, *[t for t in (src_k, src_v, dst_k, dst_v)
                                              if t is not None and t.device.type != "cpu"])
        if host:
            flags = (flags & ~(_lib.COPY_BULK | _lib.COPY_AUTO)) | _lib.COPY_VECTOR
    else:
        require_cuda("KV block copy", src_k, src_v, dst_k, dst_v, runs)
    if runs.dtype != torch.int32 or runs.dim() != 2 or runs.shape[1] != 5 or not runs.is_contiguous():
        raise ValueError("runs must be a contiguous int32 tensor of shape [n_runs, 5]")
    lib = _lib.load()
    device = runs.device
    st = stream if stream is not None else torch.cuda.current_stream(device)
    with _DeviceGuard(device):
        code = lib.augur_kv_copy_runs(
            _ptr(src_k),
            _ptr(src_v),
            _lib.i64_array(src_strides),
            int(src_majors),
            int(src_rows_per_major),
            dtype_code(src_k),
            _ptr(dst_k),
            _ptr(dst_v),
            _lib.i64_array(dst_strides),
            int(dst_majors),
            int(dst_rows_per_major),
            dtype_code(dst_k),
            _ptr(runs),
            int(runs.shape[0]),
            int(max_rows),
            int(n_layers),
            int(n_heads),
            int(head_dim),
            int(flags),
            status_word(device).data_ptr(),
            st.cuda_stream,
        )
    _lib.check(code, "augur_kv_copy_runs")
    if runs.shape[0] > 0 and n_layers > 0:
        launch_count += 1
        keep_until_done(st, runs, src_k, src_v)
        if allow_pinned_host:
            keep_host_until_done(st, src_k, src_v, dst_k, dst_v)


# Pinned host tensors a launch reads or writes, held until the launch is done:
# torch's host allocator does not see kernels that use host memory directly.
_host_keepalive: list[tuple[torch.cuda.Event, tuple]] = []


def keep_host_until_done(stream: torch.cuda.Stream, *tensors: Tensor | None) -> None:
    host = tuple(t for t in tensors if t is not None and t.device.type == "cpu")
    if not host or torch.cuda.is_current_stream_capturing():
        return  # a captured graph's owner keeps its buffers alive for the graph's life
    while _host_keepalive and _host_keepalive[0][0].query():
        _host_keepalive.pop(0)
    ev = torch.cuda.Event()
    ev.record(stream)
    _host_keepalive.append((ev, host))


def host_index_ok(n_tokens: int, src: Tensor, dst: Tensor) -> bool:
    """Whether a scatter of n_tokens can take its index by value from host memory."""
    return 0 < n_tokens <= _lib.INLINE_INDEX_MAX and src.dtype == dst.dtype


def max_rows_for(head_dim: int, elem_size: int, cap_rows: int = 64, cap_bytes: int = 8192) -> int:
    """Largest run length (rows) to cut copies into: at most cap_rows rows and cap_bytes bytes."""
    return max(1, min(cap_rows, cap_bytes // max(1, head_dim * elem_size)))


def keep_last(index: np.ndarray) -> np.ndarray:
    """``index`` with every earlier occurrence of a repeated value replaced by -1.

    The kernels write tokens in parallel and skip a negative index, so this
    gives duplicate destinations in one call the reference's result: its
    per-token loop (paged_kv_cache.py:188-192) writes them in order and the
    last one stays. An index without repeats is returned as is.
    """
    n = int(index.shape[0])
    if n < 2:
        return index
    uniq, first_in_reversed = np.unique(index[::-1], return_index=True)
    if uniq.size == n:
        return index
    last = n - 1 - first_in_reversed
    out = np.full(n, -1, dtype=np.int64)
    out[last] = index[last]
    return out
