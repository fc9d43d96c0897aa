"""ctypes binding of libaugur_kv.so (declared in include/augur_kv.h).

There is no fallback: if the library is missing or fails to load, every data
movement call raises KVLibraryError. Build it with
``python -m augur_b200.csrc.build``.
"""

from __future__ import annotations

import ctypes
import functools
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libaugur_kv.so")

OK = 0
EINVAL = 1
EBOUNDS = 2
ECUDA = 3
ETIMEOUT = 4

F32 = 0
F16 = 1
BF16 = 2

COPY_AUTO = 0
COPY_VECTOR = 1
COPY_BULK = 2
COPY_FENCE_SYSTEM = 4

ATTN_AUTO = 0
ATTN_GENERIC = 1
ATTN_TCGEN05 = 2  # paged prefill attention: force the tcgen05 kernel
ATTN_MMA_SYNC = 3  # paged prefill attention: force the mma.sync kernel
ATTN_EARLY_READS = 16  # decode attention: read lengths, tables and pool rows before the dependency wait

STATUS_NAMES = {
    OK: "ok",
    EINVAL: "invalid argument",
    EBOUNDS: "index out of bounds",
    ECUDA: "CUDA error",
    ETIMEOUT: "device wait timed out",
}

# Every exported symbol the header declares, with (restype, argtypes).
_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32
_I64P = ctypes.POINTER(ctypes.c_int64)

SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "augur_kv_version": (ctypes.c_int, []),
    "augur_kv_last_error": (ctypes.c_char_p, []),
    "augur_kv_scatter": (
        ctypes.c_int,
        [_P, _P, _I64P, _I64P, _I64, _I32, _P, _P, _I64P, _I64, _I64, _I32, _P, _I64P, _I64,
         _I32, _I64, _I32, _I32, _I32, _P, _P],
    ),
    "augur_kv_copy_runs": (
        ctypes.c_int,
        [_P, _P, _I64P, _I64, _I64, _I32, _P, _P, _I64P, _I64, _I64, _I32, _P, _I64, _I32,
         _I32, _I32, _I32, _I32, _P, _P],
    ),
    "augur_kv_copy_runs_noalloc": (
        ctypes.c_int,
        [_P, _P, _I64P, _I64, _I64, _I32, _P, _P, _I64P, _I64, _I64, _I32, _P, _I64, _I32,
         _I32, _I32, _I32, _I32, _P, _P],
    ),
    "augur_kv_ipc_export": (ctypes.c_int, [_P, _P, _I64P]),
    "augur_kv_ipc_open": (ctypes.c_int, [_P, _I64, ctypes.POINTER(ctypes.c_void_p)]),
    "augur_kv_ipc_close": (ctypes.c_int, [_P, _I64]),
    "augur_kv_paged_decode_attention": (
        ctypes.c_int,
        [_P, _I64P, _P, _P, _I64P, _I64, _I32, _P, _I64, _I64, _P, _I32, _I32, _I32, _I32, _I32, _I32,
         _P, _I64P, _I32, _P, _I64, _P, _I64, _P, _P],
    ),
    "augur_kv_paged_prefill_attention": (
        ctypes.c_int,
        [_P, _I64P, _P, _P, _I64P, _I64, _I32, _P, _I64, _I64, _P, _P, _I32, _I32, _I32, _I32, _I32, _I32,
         _I32, _P, _I64P, _I32, _P, _P],
    ),
    "augur_kv_paged_decode_attention_workspace": (
        ctypes.c_int, [_I32, _I32, _I32, _I32, _I32, _I32, _I32, _I64P, _I64P]),
    "augur_kv_rope_scatter": (
        ctypes.c_int,
        [_P, _P, _I64P, _I64P, _I64, _I32, _P, _P, _I64P, _I64, _I64, _P, _I64P, _I64, _P, _I64P, _P, _P, _I64,
         _P, _I64P, _P, _I64P, _I32, _I64, _I32, _I32, _I32, _P, _P],
    ),
    "augur_kv_decode_layer": (ctypes.c_int, [_P, _I32, _P, _P, _P, _P, _P]),
    "augur_kv_signal": (ctypes.c_int, [_P, _I32, _P]),
    "augur_kv_wait": (ctypes.c_int, [_P, _I32, _I64, _P, _P]),
}



class DecodeArgs(ctypes.Structure):
    """augur_kv_decode_args: what every layer of a decode step shares (field for field)."""

    _fields_ = [
        ("k_pool", ctypes.c_void_p),
        ("v_pool", ctypes.c_void_p),
        ("pool_strides", ctypes.c_int64 * 4),
        ("num_blocks", ctypes.c_int64),
        ("block_size", ctypes.c_int32),
        ("n_layers", ctypes.c_int32),
        ("n_q_heads", ctypes.c_int32),
        ("n_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("batch", ctypes.c_int32),
        ("flags", ctypes.c_int32),
        ("slots", ctypes.c_void_p),
        ("positions", ctypes.c_void_p),
        ("rope_cos", ctypes.c_void_p),
        ("rope_sin", ctypes.c_void_p),
        ("rope_positions", ctypes.c_int64),
        ("q_strides", ctypes.c_int64 * 2),
        ("kv_strides", ctypes.c_int64 * 2),
        ("q_rot", ctypes.c_void_p),
        ("block_tables", ctypes.c_void_p),
        ("tables_stride", ctypes.c_int64),
        ("max_blocks", ctypes.c_int64),
        ("seq_lens", ctypes.c_void_p),
        ("max_seq_len", ctypes.c_int32),
        ("launches", ctypes.c_int32),
        ("counters", ctypes.c_void_p),
        ("counters_bytes", ctypes.c_int64),
        ("scratch", ctypes.c_void_p),
        ("scratch_bytes", ctypes.c_int64),
        ("status", ctypes.c_void_p),
    ]


NOALLOC_MAX_RUNS = 65536
INLINE_INDEX_MAX = 32
IPC_HANDLE_BYTES = 64


class KVLibraryError(RuntimeError):
    """libaugur_kv.so is missing, failed to load, or a call returned an error."""

    def __init__(self, message: str, code: int = ECUDA) -> None:
        super().__init__(message)
        self.code = code


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load the library once and bind every declared symbol."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise KVLibraryError(
                f"{LIB_PATH} is missing: build it with `python -m augur_b200.csrc.build` "
                "(augur_b200 has no CPU or torch fallback for KV-cache data movement)",
                EINVAL,
            )
        try:
            lib = ctypes.CDLL(LIB_PATH)
        except OSError as exc:
            raise KVLibraryError(f"cannot load {LIB_PATH}: {exc}", EINVAL) from exc
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = lib
        return lib


@functools.lru_cache(maxsize=4096)
def _i64_array_cached(vals: tuple) -> ctypes.Array:
    return (ctypes.c_int64 * len(vals))(*vals)


def i64_array(values) -> ctypes.Array:
    """A C int64 array of `values`; identical tuples share one (read-only) array."""
    if type(values) is not tuple:
        values = tuple(int(v) for v in values)
    return _i64_array_cached(values)


def check(code: int, what: str) -> None:
    if code == OK:
        return
    detail = load().augur_kv_last_error().decode("utf-8", "replace")
    raise KVLibraryError(f"{what}: {STATUS_NAMES.get(code, code)}: {detail}", code)
