"""sm_100a kernels vs the CPU oracle on seeded inputs (bit-exact).

Covers both kernel families through the public entry points: slot scatter
(all-layer, prefill, decode append) and row runs (handoff, gather, block
copies), every vector width the launchers pick (16/8/4/2/1 bytes), the TMA
bulk and vector copy paths, mixed-dtype conversion, skipped tokens, and the
device-side bounds check.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import augur_b200 as ab
from augur_b200 import _lib, _ops, batched
from tests.conftest import assert_bits_equal, poison_

pytestmark = pytest.mark.gpu


def _pool(L, NB, H, bs, D, dtype, device):
    return ab.PagedKVCache(keys=poison_(torch.empty(L, NB, H, bs, D, dtype=dtype, device=device)),
                           values=poison_(torch.empty(L, NB, H, bs, D, dtype=dtype, device=device)),
                           block_size=bs, allocator=ab.BlockAllocator(NB))


def _rand(shape, dtype, gen):
    return torch.randn(shape, generator=gen).to(dtype)


def _random_tables(rng, lens, bs, NB):
    perm = rng.permutation(NB)
    tables, cur = [], 0
    for n in lens:
        nb = -(-int(n) // bs)
        tables.append(ab.SequenceBlockTable(block_ids=perm[cur : cur + nb].tolist(), block_size=bs))
        cur += nb
    return tables


def _slots(tables, lens):
    out = []
    for t, n in zip(tables, lens):
        pos = np.arange(int(n))
        out.append(np.asarray(t.block_ids, np.int64)[pos // t.block_size] * t.block_size + pos % t.block_size)
    return np.concatenate(out) if out else np.zeros(0, np.int64)


@pytest.mark.parametrize(
    "dtype, H, D",
    [(torch.bfloat16, 2, 64), (torch.float32, 2, 64), (torch.float16, 4, 128),
     (torch.float32, 2, 2), (torch.float16, 3, 2), (torch.bfloat16, 1, 3), (torch.float16, 2, 1)],
)
def test_scatter_all_layers_vs_oracle(cuda, oracle, dtype, H, D):
    """write_paged_kv_batch == the reference's write_paged_kv per layer and token (oracle)."""
    rng = np.random.default_rng(D * 7 + H)
    g = torch.Generator().manual_seed(D + H)
    L, bs, NB = 5, 16, 96
    lens = rng.integers(1, 60, size=9)
    tables = _random_tables(rng, lens, bs, NB)
    slots = _slots(tables, lens)
    slots[rng.choice(slots.shape[0], size=5, replace=False)] = -1  # skipped tokens
    T = slots.shape[0]
    k, v = _rand((L, T, H, D), dtype, g), _rand((L, T, H, D), dtype, g)
    pool = _pool(L, NB, H, bs, D, dtype, cuda)
    batched.write_paged_kv_batch(pool, k.to(cuda), v.to(cuda), torch.from_numpy(slots).to(cuda))
    ek, ev = poison_(torch.empty(L, NB, H, bs, D, dtype=dtype)), poison_(torch.empty(L, NB, H, bs, D, dtype=dtype))
    oracle.scatter_slots(k, v, slots, ek, ev, bs, threads=4)
    assert_bits_equal(pool.keys, ek, "keys")
    assert_bits_equal(pool.values, ev, "values")
    assert _ops.read_status(cuda) == _lib.OK


def test_scatter_one_layer_and_noncontiguous_source(cuda, oracle):
    g = torch.Generator().manual_seed(3)
    L, NB, H, bs, D, T = 3, 20, 2, 8, 64, 50
    pool = _pool(L, NB, H, bs, D, torch.bfloat16, cuda)
    slots = np.random.default_rng(1).permutation(NB * bs)[:T].astype(np.int64)
    # [T, D, H] storage viewed as [T, H, D]: head stride 1 would break rows, so use [H, T, D] storage
    base = _rand((H, T, D), torch.bfloat16, g)
    k = base.permute(1, 0, 2)  # [T, H, D] with token stride D, head stride T*D
    batched.write_paged_kv_batch(pool, k.to(cuda), k.to(cuda), torch.from_numpy(slots).to(cuda), layer_idx=2)
    ek = poison_(torch.empty(L, NB, H, bs, D, dtype=torch.bfloat16))
    oracle.scatter_slots(k.contiguous().unsqueeze(0), None, slots, ek[2:3], None, bs)
    assert_bits_equal(pool.keys, ek, "keys")
    assert_bits_equal(pool.values, ek, "values")


def test_prefill_padded_vs_oracle(cuda, oracle):
    """Right-padded [L, B, S, H, D] prefill: padding (-1 slots) moves nothing."""
    rng = np.random.default_rng(5)
    g = torch.Generator().manual_seed(5)
    L, B, S, H, D, bs, NB = 4, 6, 70, 2, 64, 16, 64
    lens = rng.integers(1, S + 1, size=B)
    pool = _pool(L, NB, H, bs, D, torch.bfloat16, cuda)
    tables = [ab.SequenceBlockTable.empty(bs) for _ in range(B)]
    sm = batched.prefill_slot_mapping(tables, lens, pool.allocator, max_len=S)
    k, v = _rand((L, B, S, H, D), torch.bfloat16, g), _rand((L, B, S, H, D), torch.bfloat16, g)
    batched.write_paged_kv_prefill(pool, k.to(cuda), v.to(cuda), torch.from_numpy(sm).to(cuda))
    ek, ev = poison_(torch.empty(L, NB, H, bs, D, dtype=torch.bfloat16)), poison_(torch.empty(L, NB, H, bs, D, dtype=torch.bfloat16))
    oracle.scatter_slots(k.reshape(L, B * S, H, D), v.reshape(L, B * S, H, D), sm.reshape(-1), ek, ev, bs)
    assert_bits_equal(pool.keys, ek, "keys")
    assert_bits_equal(pool.values, ev, "values")


def test_decode_appends_vs_oracle(cuda, oracle):
    """Several decode steps, crossing block boundaries, equal the reference's per-step writes."""
    rng = np.random.default_rng(9)
    g = torch.Generator().manual_seed(9)
    L, B, H, D, bs, NB = 6, 5, 2, 64, 4, 80
    lens = rng.integers(1, 9, size=B)
    pool = _pool(L, NB, H, bs, D, torch.bfloat16, cuda)
    tables = [ab.SequenceBlockTable.empty(bs) for _ in range(B)]
    batched.prefill_slot_mapping(tables, lens, pool.allocator)
    ref_alloc = oracle.RefBlockAllocator(NB)
    ref_tables = [oracle.RefBlockTable([], bs) for _ in range(B)]
    for t, n in zip(ref_tables, lens):
        t.ensure_position(int(n) - 1, ref_alloc)
    ek, ev = poison_(torch.empty(L, NB, H, bs, D, dtype=torch.bfloat16)), poison_(torch.empty(L, NB, H, bs, D, dtype=torch.bfloat16))
    for step in range(7):
        k, v = _rand((L, B, H, D), torch.bfloat16, g), _rand((L, B, H, D), torch.bfloat16, g)
        batched.append_decode(pool, tables, k.to(cuda), v.to(cuda))
        for b, t in enumerate(ref_tables):
            pos = t.seq_len  # one new position per step, the same for every layer
            for layer in range(L):
                oracle.write_paged_kv(ek, ev, ref_alloc, layer, t, [pos],
                                      k[layer, b].unsqueeze(0).unsqueeze(2), v[layer, b].unsqueeze(0).unsqueeze(2))
    assert [t.block_ids for t in tables] == [t.block_ids for t in ref_tables]
    assert_bits_equal(pool.keys, ek, "keys")
    assert_bits_equal(pool.values, ev, "values")


@pytest.mark.parametrize("flags", [_lib.COPY_VECTOR, _lib.COPY_BULK])
@pytest.mark.parametrize("dtype, D", [(torch.bfloat16, 64), (torch.float32, 64), (torch.float16, 8)])
def test_handoff_and_gather_vs_oracle(cuda, oracle, flags, dtype, D):
    rng = np.random.default_rng(D)
    g = torch.Generator().manual_seed(D)
    L, B, H, S, bs, NB = 4, 7, 2, 100, 16, 64
    lens = rng.integers(1, S + 1, size=B)
    src = ab.KVCache(keys=_rand((L, B, H, S, D), dtype, g).to(cuda), values=_rand((L, B, H, S, D), dtype, g).to(cuda))
    pool = _pool(L, NB, H, bs, D, dtype, cuda)
    tables = _random_tables(rng, lens, bs, NB)
    for t in tables:
        t.seq_len = 0
    batched.handoff_contiguous_to_paged(src, pool, tables, lens, flags=flags)
    runs = batched.handoff_runs(tables, lens)
    ek, ev = poison_(torch.empty(L, NB, H, bs, D, dtype=dtype)), poison_(torch.empty(L, NB, H, bs, D, dtype=dtype))
    oracle.copy_runs(src.keys.cpu(), src.values.cpu(), ek, ev, runs, threads=4)
    assert_bits_equal(pool.keys, ek, "handoff keys")
    assert_bits_equal(pool.values, ev, "handoff values")
    # gather back (paged -> contiguous) and compare with the source's valid rows
    out = (poison_(torch.empty(L, B, H, S, D, dtype=dtype, device=cuda)),
           poison_(torch.empty(L, B, H, S, D, dtype=dtype, device=cuda)))
    gk, gv = batched.read_paged_kv_batch(pool, tables, out=out)
    for b, n in enumerate(lens):
        assert_bits_equal(gk[:, b, :, :n], src.keys[:, b, :, :n], f"gather k {b}")
        assert_bits_equal(gv[:, b, :, :n], src.values[:, b, :, :n], f"gather v {b}")
        assert (gk[:, b, :, n:].contiguous().view(torch.uint8) == 0xFF).all()
    assert _ops.read_status(cuda) == _lib.OK


def test_read_paged_kv_large_block_splits_runs(cuda, oracle):
    """block_size 256 at 256-byte rows needs runs cut to the 16 KiB stage limit."""
    g = torch.Generator().manual_seed(11)
    L, NB, H, bs, D = 2, 6, 2, 256, 64
    cfg = ab.QwenConfig(vocab_size=16, hidden_size=128, intermediate_size=16, num_hidden_layers=L,
                        num_attention_heads=2, num_key_value_heads=H)
    pool = ab.new_paged_kv_cache(cfg, num_blocks=NB, block_size=bs, device=cuda, dtype=torch.float32)
    table = ab.SequenceBlockTable.empty(bs)
    n = 700
    k = _rand((1, H, n, D), torch.float32, g)
    ab.write_paged_kv(pool, 1, table, torch.arange(n).unsqueeze(0), k.to(cuda), k.to(cuda))
    rk, rv = ab.read_paged_kv(pool, 1, table)
    assert_bits_equal(rk, k, "read")
    ref_t = oracle.RefBlockTable(table.block_ids, bs, n)
    ok, _ = oracle.read_paged_kv(pool.keys.cpu(), pool.values.cpu(), 1, ref_t)
    assert_bits_equal(rk, ok, "oracle read")


@pytest.mark.parametrize("flags", [_lib.COPY_VECTOR, _lib.COPY_BULK])
def test_copy_blocks_vs_oracle(cuda, oracle, flags):
    g = torch.Generator().manual_seed(2)
    L, NB, H, bs, D = 3, 40, 2, 16, 64
    pool = _pool(L, NB, H, bs, D, torch.bfloat16, cuda)
    init_k, init_v = _rand((L, NB, H, bs, D), torch.bfloat16, g), _rand((L, NB, H, bs, D), torch.bfloat16, g)
    pool.keys.copy_(init_k)
    pool.values.copy_(init_v)
    src, dst, rows = [1, 5, 9, 30], [2, 6, 20, 0], [16, 3, 1, 9]
    batched.copy_blocks(pool, src, dst, rows, flags=flags)
    ek, ev = init_k.clone(), init_v.clone()
    oracle.copy_runs(init_k, init_v, ek, ev, np.array([[s, 0, d, 0, r] for s, d, r in zip(src, dst, rows)]))
    assert_bits_equal(pool.keys, ek, "keys")
    assert_bits_equal(pool.values, ev, "values")


@pytest.mark.parametrize("L, H, D, dtype", [(3, 2, 64, torch.bfloat16), (3, 1, 64, torch.bfloat16),
                                           (5, 2, 128, torch.float32)])
def test_short_runs_take_several_planes_per_warp(cuda, oracle, L, H, D, dtype):
    """Runs of at most 1 KB per plane (copy-on-write of partly filled blocks): each warp
    copies its run for several (layer, K/V, head) planes; plane counts that do and do not
    divide by four."""
    g = torch.Generator().manual_seed(7)
    NB, bs = 48, 16
    pool = _pool(L, NB, H, bs, D, dtype, cuda)
    init_k, init_v = _rand((L, NB, H, bs, D), dtype, g), _rand((L, NB, H, bs, D), dtype, g)
    pool.keys.copy_(init_k)
    pool.values.copy_(init_v)
    max_rows = 1024 // (D * init_k.element_size())
    rng = np.random.default_rng(7)
    src = rng.choice(NB // 2, size=20, replace=False).tolist()
    dst = (NB // 2 + rng.choice(NB // 2, size=20, replace=False)).tolist()
    rows = rng.integers(1, max_rows + 1, size=20).tolist()
    batched.copy_blocks(pool, src, dst, rows)
    ek, ev = init_k.clone(), init_v.clone()
    oracle.copy_runs(init_k, init_v, ek, ev, np.array([[s, 0, d, 0, r] for s, d, r in zip(src, dst, rows)]))
    assert_bits_equal(pool.keys, ek, "keys")
    assert_bits_equal(pool.values, ev, "values")
    assert _ops.read_status(cuda) == _lib.OK


def test_conversion_special_values_vs_oracle(cuda, oracle):
    """f32 -> bf16 / f16 through write_paged_kv: RNE rounding, signed zero, inf, subnormals, ties."""
    vals = torch.tensor([0.0, -0.0, 1.0, -1.0, float("inf"), -float("inf"), 1e-40, -3e-39, 65504.0,
                         65520.0, 1e5, 1.00390625, 1.01171875, 3.14159265, 2.0**-24, 2.0**-25, 1 + 2.0**-8,
                         1 + 3 * 2.0**-9, 6e-8, 0.1, 1e38, 3.3895314e38])
    g = torch.Generator().manual_seed(4)
    D = 8
    n = 64
    data = torch.cat([vals, torch.randn(2 * n * D - vals.numel(), generator=g) * 100]).view(1, 2, n, D)
    for dst_dtype in (torch.bfloat16, torch.float16):
        cfg = ab.QwenConfig(vocab_size=16, hidden_size=16, intermediate_size=16, num_hidden_layers=1,
                            num_attention_heads=2, num_key_value_heads=2)
        pool = ab.new_paged_kv_cache(cfg, num_blocks=16, block_size=4, device=cuda, dtype=dst_dtype)
        poison_(pool.keys)
        poison_(pool.values)
        table = ab.SequenceBlockTable.empty(4)
        ab.write_paged_kv(pool, 0, table, torch.arange(n).unsqueeze(0), data.to(cuda), data.to(cuda))
        ek, ev = poison_(torch.empty_like(pool.keys, device="cpu")), poison_(torch.empty_like(pool.values, device="cpu"))
        oracle.write_paged_kv(ek, ev, oracle.RefBlockAllocator(16), 0, oracle.RefBlockTable([], 4),
                              list(range(n)), data, data)
        assert_bits_equal(pool.keys, ek, f"{dst_dtype} keys")
        # and torch's own CPU cast (what the reference's assignment does) agrees
        assert_bits_equal(data.to(dst_dtype)[0], ab.read_paged_kv(pool, 0, table)[0][0].cpu(), "torch cast")


def test_kernel_bounds_check_records_status(cuda):
    """An out-of-range slot is skipped and reported, valid tokens still land, nothing else changes."""
    lib = _lib.load()
    L, NB, H, bs, D = 1, 4, 2, 4, 64
    pool_k = poison_(torch.empty(L, NB, H, bs, D, dtype=torch.bfloat16, device=cuda))
    src = torch.randn(L, 3, H, D, device=cuda).to(torch.bfloat16)
    slots = torch.tensor([5, NB * bs, 9], dtype=torch.int64, device=cuda)  # middle one is one past the end
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    i64 = lambda *v: (ctypes.c_int64 * len(v))(*v)  # noqa: E731
    code = lib.augur_kv_scatter(
        src.data_ptr(), None, i64(0, 0, H * D, D), None, 3, _lib.BF16,
        pool_k.data_ptr(), None, i64(0, pool_k.stride(1), pool_k.stride(3), pool_k.stride(2)), bs, NB,
        _lib.BF16, slots.data_ptr(), i64(0, 1), 0, 0, 3, 1, H, D, status.data_ptr(),
        torch.cuda.current_stream().cuda_stream)
    assert code == _lib.OK
    torch.cuda.synchronize()
    assert int(status.item()) == _lib.EBOUNDS
    assert torch.equal(pool_k[0, 1, :, 1].cpu(), src[0, 0].cpu())
    assert torch.equal(pool_k[0, 2, :, 1].cpu(), src[0, 2].cpu())
    written = 2 * H * D
    assert int((pool_k.view(torch.int16) == -1).sum()) == pool_k.numel() - written
    # an out-of-range run (source block past the pool) is skipped the same way
    runs = torch.tensor([[NB, 0, 0, 0, 4], [1, 0, 3, 0, 4]], dtype=torch.int32, device=cuda)
    status.zero_()
    code = lib.augur_kv_copy_runs(
        pool_k.data_ptr(), None, i64(pool_k.stride(0), pool_k.stride(1), pool_k.stride(3), pool_k.stride(2)),
        NB, bs, _lib.BF16, pool_k.data_ptr(), None,
        i64(pool_k.stride(0), pool_k.stride(1), pool_k.stride(3), pool_k.stride(2)), NB, bs, _lib.BF16,
        runs.data_ptr(), 2, bs, L, H, D, _lib.COPY_BULK, status.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert code == _lib.OK
    torch.cuda.synchronize()
    assert int(status.item()) == _lib.EBOUNDS
    assert_bits_equal(pool_k[0, 3], pool_k[0, 1], "copied block")


def test_empty_inputs_launch_nothing(cuda):
    pool = _pool(2, 4, 2, 4, 64, torch.bfloat16, cuda)
    before = _ops.launch_count
    batched.write_paged_kv_batch(pool, torch.empty(2, 0, 2, 64, dtype=torch.bfloat16, device=cuda),
                                 torch.empty(2, 0, 2, 64, dtype=torch.bfloat16, device=cuda),
                                 torch.empty(0, dtype=torch.int64, device=cuda))
    batched.copy_blocks(pool, [], [])
    assert _ops.launch_count == before
    assert (pool.keys.view(torch.uint8) == 0xFF).all()


@pytest.mark.parametrize("flags", [_lib.COPY_BULK, _lib.COPY_VECTOR])
def test_handoff_many_runs_per_warp_vs_oracle(cuda, oracle, flags):
    """24 layers x 2 heads x 2 (K, V) planes and ~1500 runs: each bulk-pipeline warp walks
    well over 32 runs, so its descriptor windows refill several times."""
    rng = np.random.default_rng(77)
    g = torch.Generator().manual_seed(77)
    L, B, H, S, D, bs, NB = 24, 32, 2, 1024, 64, 16, 2304
    lens = rng.integers(512, S + 1, size=B)
    src = ab.KVCache(keys=_rand((L, B, H, S, D), torch.bfloat16, g).to(cuda),
                     values=_rand((L, B, H, S, D), torch.bfloat16, g).to(cuda))
    pool = _pool(L, NB, H, bs, D, torch.bfloat16, cuda)
    tables = _random_tables(rng, lens, bs, NB)
    runs_t = batched.handoff_contiguous_to_paged(src, pool, tables, lens, flags=flags)
    assert runs_t.shape[0] > 1000
    ek = poison_(torch.empty(L, NB, H, bs, D, dtype=torch.bfloat16))
    ev = poison_(torch.empty(L, NB, H, bs, D, dtype=torch.bfloat16))
    oracle.copy_runs(src.keys.cpu(), src.values.cpu(), ek, ev, batched.handoff_runs(tables, lens), threads=8)
    assert_bits_equal(pool.keys, ek, "keys")
    assert_bits_equal(pool.values, ev, "values")
    assert _ops.read_status(cuda) == _lib.OK


@pytest.mark.parametrize("dtype, H, D", [(torch.bfloat16, 2, 64), (torch.float32, 2, 64), (torch.float16, 3, 2)])
def test_host_index_path_matches_device_path(cuda, dtype, H, D):
    """Up to 32 slots/positions passed by value equal the same scatter through a device index."""
    g = torch.Generator().manual_seed(21)
    rng = np.random.default_rng(21)
    L, NB, bs = 4, 16, 8
    for n in (1, 7, 32):
        slots = rng.permutation(NB * bs)[:n].astype(np.int64)
        slots[n // 2] = -1  # one skipped token
        k = _rand((L, n, H, D), dtype, g).to(cuda)
        v = _rand((L, n, H, D), dtype, g).to(cuda)
        a, b = _pool(L, NB, H, bs, D, dtype, cuda), _pool(L, NB, H, bs, D, dtype, cuda)
        batched.write_paged_kv_batch(a, k, v, slots)  # host index, by value
        batched.write_paged_kv_batch(b, k, v, torch.from_numpy(slots).to(cuda))
        assert_bits_equal(a.keys, b.keys, f"keys n={n}")
        assert_bits_equal(a.values, b.values, f"values n={n}")
    # contiguous cache through write_kv with host positions (by value) vs device positions
    cfg = ab.QwenConfig(vocab_size=16, hidden_size=H * D, intermediate_size=16, num_hidden_layers=L,
                        num_attention_heads=H, num_key_value_heads=H)
    c1 = ab.new_kv_cache(cfg, batch_size=3, max_seq_len=20, device=cuda, dtype=dtype)
    c2 = ab.new_kv_cache(cfg, batch_size=3, max_seq_len=20, device=cuda, dtype=dtype)
    for c in (c1, c2):
        poison_(c.keys)
        poison_(c.values)
    pos = torch.tensor([[4, 9], [0, 19], [7, 3]])
    kk = _rand((3, H, 2, D), dtype, g).to(cuda)
    ab.write_kv(c1, 2, pos, kk, kk)
    ab.write_kv(c2, 2, pos.to(cuda), kk, kk)
    assert_bits_equal(c1.keys, c2.keys, "write_kv keys")
    assert _ops.read_status(cuda) == _lib.OK


def test_host_index_bounds_check(cuda):
    """An out-of-range slot passed by value is skipped and reported like a device one."""
    pool = _pool(1, 4, 2, 4, 64, torch.bfloat16, cuda)
    k = torch.randn(1, 2, 2, 64, device=cuda).to(torch.bfloat16)
    batched.write_paged_kv_batch(pool, k, k, np.array([3, 16], dtype=np.int64))
    assert _ops.read_status(cuda) == _lib.EBOUNDS
    assert_bits_equal(pool.keys[0, 0, :, 3], k[0, 0], "valid token")
    assert int((pool.keys.view(torch.int16) == -1).sum()) == pool.keys.numel() - 2 * 64


def test_wait_times_out_and_context_stays_usable(cuda):
    """A wait on a flag nothing sets gives up after its bound, reports ETIMEOUT, and the GPU carries on."""
    import time

    from augur_b200 import peer

    flags = peer.new_flags(cuda)
    t0 = time.perf_counter()
    peer.wait(flags, 1, timeout_s=0.3)
    assert _ops.read_status(cuda) == _lib.ETIMEOUT
    assert 0.25 < time.perf_counter() - t0 < 10.0
    # already satisfied: no timeout
    flags.fill_(5)
    peer.wait(flags, 3, timeout_s=0.3)
    assert _ops.read_status(cuda) == _lib.OK
    # the context still runs kernels
    pool = _pool(1, 4, 2, 4, 64, torch.bfloat16, cuda)
    k = torch.randn(1, 1, 2, 64, device=cuda).to(torch.bfloat16)
    batched.write_paged_kv_batch(pool, k, k, np.array([5], dtype=np.int64))
    assert _ops.read_status(cuda) == _lib.OK
    assert_bits_equal(pool.keys[0, 1, :, 1], k[0, 0], "write after timeout")
    with pytest.raises(_lib.KVLibraryError):
        peer.wait(flags, 1, timeout_s=0.0)
