"""The C-ABI library loads and exports exactly what include/augur_kv.h declares (CPU only).

No kernel is launched here: the calls below fail argument validation before
any CUDA runtime call.
"""

from __future__ import annotations

import ctypes
import os
import re

import pytest

from augur_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "augur_kv.h")


def declared_functions() -> list[str]:
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(augur_kv_\w+)\s*\(", text)))


def test_header_declarations_are_exported_and_bound():
    names = declared_functions()
    assert names, "no declarations parsed"
    lib = _lib.load()
    for name in names:
        assert hasattr(lib, name), f"{name} declared but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    assert set(_lib.SIGNATURES) == set(names)


def test_status_codes_match_header():
    text = open(HEADER).read()
    for name in ("OK", "EINVAL", "EBOUNDS", "ECUDA", "ETIMEOUT", "F32", "F16", "BF16",
                 "COPY_AUTO", "COPY_VECTOR", "COPY_BULK", "COPY_FENCE_SYSTEM"):
        m = re.search(rf"#define AUGUR_KV_{name} (\d+)", text)
        assert m and int(m.group(1)) == getattr(_lib, name), name


def test_version():
    assert _lib.load().augur_kv_version() >> 16 == 0


def _i64(*v):
    return (ctypes.c_int64 * len(v))(*v)


def test_scatter_rejects_bad_arguments_without_touching_the_device():
    lib = _lib.load()
    strides = _i64(0, 0, 1, 1)
    code = lib.augur_kv_scatter(None, None, strides, strides, 1, _lib.BF16, None, None, strides,
                                16, 1, _lib.BF16, None, _i64(0, 1), 0, 0, 1, 1, 1, 8, None, None)
    assert code == _lib.EINVAL
    assert b"null pointer" in lib.augur_kv_last_error()
    fake = ctypes.c_void_p(16)
    code = lib.augur_kv_scatter(fake, None, strides, strides, 1, 7, fake, None, strides,
                                16, 1, _lib.BF16, fake, _i64(0, 1), 0, 0, 1, 1, 1, 8, None, None)
    assert code == _lib.EINVAL and b"dtype" in lib.augur_kv_last_error()
    code = lib.augur_kv_scatter(fake, None, strides, strides, 1, _lib.BF16, fake, None, strides,
                                16, 1, _lib.BF16, fake, _i64(0, 1), 3, 0, 1, 1, 1, 8, None, None)
    assert code == _lib.EINVAL and b"index_row_base" in lib.augur_kv_last_error()


def test_empty_work_is_ok_with_null_pointers():
    lib = _lib.load()
    s = _i64(0, 0, 1, 1)
    assert lib.augur_kv_scatter(None, None, s, s, 1, _lib.BF16, None, None, s, 16, 1, _lib.BF16,
                                None, _i64(0, 1), 0, 0, 0, 24, 2, 64, None, None) == _lib.OK
    assert lib.augur_kv_copy_runs(None, None, s, 1, 1, _lib.BF16, None, None, s, 1, 1, _lib.BF16,
                                  None, 0, 16, 24, 2, 64, 0, None, None) == _lib.OK
    assert lib.augur_kv_scatter(None, None, s, s, 1, _lib.BF16, None, None, s, 16, 1, _lib.BF16,
                                None, _i64(0, 1), 0, 0, -1, 24, 2, 64, None, None) == _lib.EINVAL


def test_host_index_limits():
    lib = _lib.load()
    fake = ctypes.c_void_p(16)
    s = _i64(0, 0, 1, 1)
    host = _i64(*range(40))
    code = lib.augur_kv_scatter(fake, None, s, s, 33, _lib.BF16, fake, None, s, 16, 4, _lib.BF16,
                                host, _i64(0, 1), 0, 1, 33, 1, 1, 64, None, None)
    assert code == _lib.EINVAL and b"host index" in lib.augur_kv_last_error()
    code = lib.augur_kv_scatter(fake, None, s, s, 2, _lib.F32, fake, None, s, 16, 4, _lib.BF16,
                                host, _i64(0, 1), 0, 1, 2, 1, 1, 64, None, None)
    assert code == _lib.EINVAL and b"equal dtypes" in lib.augur_kv_last_error()


def test_copy_runs_rejects_bad_arguments_without_touching_the_device():
    lib = _lib.load()
    fake = ctypes.c_void_p(16)
    s = _i64(0, 0, 1, 1)
    code = lib.augur_kv_copy_runs(fake, None, s, 1, 1, _lib.BF16, fake, None, s, 1, 1, _lib.BF16,
                                  fake, 1, 1024, 1, 1, 64, 0, None, None)
    assert code == _lib.EINVAL and b"16384" in lib.augur_kv_last_error()
    code = lib.augur_kv_copy_runs(fake, None, s, 1, 1, _lib.BF16, fake, None, s, 1, 1, _lib.BF16,
                                  fake, 1, 1, 1, 1, 64, 9, None, None)
    assert code == _lib.EINVAL and b"flags" in lib.augur_kv_last_error()
    code = lib.augur_kv_copy_runs(fake, None, s, 1, 1, _lib.F32, fake, None, s, 1, 1, _lib.BF16,
                                  fake, 1, 1, 1, 1, 64, _lib.COPY_BULK, None, None)
    assert code == _lib.EINVAL and b"equal dtypes" in lib.augur_kv_last_error()


def test_missing_library_fails_loudly(monkeypatch):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", "/nonexistent/libaugur_kv.so")
    with pytest.raises(_lib.KVLibraryError, match="no CPU or torch fallback"):
        _lib.load()


def test_decode_args_layout_matches_header(tmp_path):
    """The ctypes mirror of augur_kv_decode_args has the C struct's size and field offsets
    (compiled here with the host compiler from the header itself)."""
    import shutil
    import subprocess

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no host C compiler")
    fields = [name for name, _ in _lib.DecodeArgs._fields_]
    lines = ['#include <stddef.h>', '#include <stdio.h>', '#include "augur_kv.h"', "int main(void) {",
             '  printf("size %zu\\n", sizeof(augur_kv_decode_args));']
    lines += [f'  printf("{f} %zu\\n", offsetof(augur_kv_decode_args, {f}));' for f in fields]
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run([cc, "-I", os.path.dirname(HEADER), str(src), "-o", str(exe)], check=True)
    got = dict(line.split() for line in subprocess.run([str(exe)], check=True, capture_output=True,
                                                          text=True).stdout.splitlines())
    assert int(got["size"]) == ctypes.sizeof(_lib.DecodeArgs)
    for f in fields:
        assert int(got[f]) == getattr(_lib.DecodeArgs, f).offset, f


def test_decode_layer_rejects_bad_arguments_without_touching_the_device():
    lib = _lib.load()
    assert lib.augur_kv_decode_layer(None, 0, None, None, None, None, None) == _lib.EINVAL
    assert b"null args" in lib.augur_kv_last_error()
    args = _lib.DecodeArgs()
    args.n_layers = 24
    args.dtype = _lib.BF16
    for layer in (-1, 24):
        assert lib.augur_kv_decode_layer(ctypes.byref(args), layer, None, None, None, None, None) == _lib.EINVAL
        assert b"outside [0, 24)" in lib.augur_kv_last_error()
    assert lib.augur_kv_decode_layer(ctypes.byref(args), 0, None, None, None, None, None) == _lib.EINVAL
    assert b"null pool" in lib.augur_kv_last_error()
