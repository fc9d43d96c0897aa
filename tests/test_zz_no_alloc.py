"""augur_kv_copy_runs_noalloc: the block copy for callers that cannot allocate device memory.

An engine that owns all of its device memory as one reservation (cache blocks
carved out by its own allocator) or a C/C++ host without a device allocator
cannot hand augur_kv_copy_runs the device buffer of run descriptors it
needs. The no-allocation entry point takes the descriptors in host memory and
stages them in a fixed array inside the library. These tests call it through
the C ABI and require its results to be bit-identical to the regular entry
point's, over two calls in a row that share the library's array (the second
with fewer runs, so stale descriptors from the first are present), plus the
size limit. The second call must also leave the device's free memory as it
was: the entry point allocates nothing.

The tests here depend on no other test and pass alone or after the rest of
the suite. The file name sorts last only so that a run stopped at its first
failure (pytest -x) has already run every other test if one of these fails.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from augur_b200 import _lib, _ops, batched
from tests.conftest import assert_bits_equal, poison_

pytestmark = pytest.mark.gpu


def _i64(*v):
    return (ctypes.c_int64 * len(v))(*v)


def _strides(t: torch.Tensor):
    # (layer, major, row, head) of a [layers, major, heads, rows, dim] cache
    return _i64(t.stride(0), t.stride(1), t.stride(3), t.stride(2))


def _call(fn, src_k, src_v, dst_k, dst_v, runs_arg, n_runs, max_rows, flags, status):
    L, _, H, _, D = src_k.shape
    return fn(src_k.data_ptr(), src_v.data_ptr(), _strides(src_k), src_k.shape[1], src_k.shape[3], _lib.BF16,
              dst_k.data_ptr(), dst_v.data_ptr(), _strides(dst_k), dst_k.shape[1], dst_k.shape[3], _lib.BF16,
              runs_arg, n_runs, max_rows, L, H, D, flags, status.data_ptr(),
              torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_copy_runs_on_two_calls(cuda):
    lib = _lib.load()
    status = _ops.status_word(cuda)
    g = torch.Generator(device=cuda).manual_seed(5)
    rng = np.random.default_rng(5)
    L, B, H, S, D, bs, NB = 6, 5, 2, 100, 64, 16, 64
    src_k = torch.randn(L, B, H, S, D, generator=g, device=cuda).to(torch.bfloat16)
    src_v = torch.randn(L, B, H, S, D, generator=g, device=cuda).to(torch.bfloat16)
    lens = rng.integers(1, S + 1, size=B)
    perm = rng.permutation(NB)
    tables, cur = [], 0
    for n in lens:
        nb = -(-int(n) // bs)
        tables.append(perm[cur : cur + nb].tolist())
        cur += nb
    handoff = []
    for b, (ids, n) in enumerate(zip(tables, lens)):
        for j in range(-(-int(n) // bs)):
            handoff.append((b, j * bs, ids[j], 0, min(bs, int(n) - j * bs)))
    handoff = np.ascontiguousarray(handoff, dtype=np.int32)

    # call 1: contiguous -> paged handoff, bulk (TMA) path
    pools = [tuple(poison_(torch.empty(L, NB, H, bs, D, dtype=torch.bfloat16, device=cuda)) for _ in range(2))
             for _ in range(2)]
    dev_runs = torch.from_numpy(handoff).to(cuda)
    assert _call(lib.augur_kv_copy_runs, src_k, src_v, *pools[0], dev_runs.data_ptr(), handoff.shape[0],
                 bs, _lib.COPY_BULK, status) == _lib.OK
    assert _call(lib.augur_kv_copy_runs_noalloc, src_k, src_v, *pools[1],
                 handoff.ctypes.data_as(ctypes.c_void_p), handoff.shape[0], bs, _lib.COPY_BULK,
                 status) == _lib.OK
    torch.cuda.synchronize()
    assert_bits_equal(pools[1][0], pools[0][0], "call 1 keys")
    assert_bits_equal(pools[1][1], pools[0][1], "call 1 values")

    # call 2: fewer runs (paged -> contiguous gather of sequence 0 in 8-row
    # pieces), vector path; the shared array still holds call 1's tail
    gather = batched.split_runs(handoff[handoff[:, 0] == 0][:, [2, 3, 0, 1, 4]], 8)
    assert 0 < gather.shape[0] < handoff.shape[0]
    outs = [tuple(poison_(torch.empty(L, B, H, S, D, dtype=torch.bfloat16, device=cuda)) for _ in range(2))
            for _ in range(2)]
    gather_dev = torch.from_numpy(np.ascontiguousarray(gather)).to(cuda)
    assert _call(lib.augur_kv_copy_runs, pools[0][0], pools[0][1], *outs[0], gather_dev.data_ptr(),
                 gather.shape[0], 8, _lib.COPY_VECTOR, status) == _lib.OK
    gather_host = np.ascontiguousarray(gather, dtype=np.int32)
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info(cuda)
    assert _call(lib.augur_kv_copy_runs_noalloc, pools[0][0], pools[0][1], *outs[1],
                 gather_host.ctypes.data_as(ctypes.c_void_p), gather.shape[0], 8, _lib.COPY_VECTOR,
                 status) == _lib.OK
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info(cuda)
    assert free_after == free_before, "the no-allocation entry point changed the device's free memory"
    assert_bits_equal(outs[1][0], outs[0][0], "call 2 keys")
    assert_bits_equal(outs[1][1], outs[0][1], "call 2 values")
    # and the gather really moved data: rows [0, n_0) of batch row 0 equal the source
    assert_bits_equal(outs[1][0][:, 0, :, : int(lens[0])], src_k[:, 0, :, : int(lens[0])], "gathered rows")
    assert _ops.read_status(cuda) == _lib.OK


def test_noalloc_rejects_more_runs_than_its_scratch(cuda):
    lib = _lib.load()
    t = torch.empty(1, 1, 1, 16, 64, dtype=torch.bfloat16, device=cuda)
    runs = np.zeros((1, 5), dtype=np.int32)
    code = _call(lib.augur_kv_copy_runs_noalloc, t, t, t, t, runs.ctypes.data_as(ctypes.c_void_p),
                 _lib.NOALLOC_MAX_RUNS + 1, 16, _lib.COPY_AUTO, _ops.status_word(cuda))
    assert code == _lib.EINVAL
    assert b"exceed the fixed scratch" in lib.augur_kv_last_error()


def test_noalloc_checks_arguments_before_staging(cuda):
    # an argument the copy itself rejects (unknown flags) fails the call with
    # the copy's own message, before any descriptor is staged
    lib = _lib.load()
    t = torch.empty(1, 1, 1, 16, 64, dtype=torch.bfloat16, device=cuda)
    runs = np.zeros((1, 5), dtype=np.int32)
    code = _call(lib.augur_kv_copy_runs_noalloc, t, t, t, t, runs.ctypes.data_as(ctypes.c_void_p), 1, 16,
                 64, _ops.status_word(cuda))
    assert code == _lib.EINVAL
    assert b"copy_runs: unknown flags" in lib.augur_kv_last_error()
