"""Drop-in API on CUDA vs the reference's own results (bit-exact).

Every case replays, through augur_b200 on the GPU, the calls that
tests/golden/make_golden.py ran through semioz/augur on the CPU, starting
from the same 0xFF-poisoned caches, and compares every byte of the caches
(written rows and untouched rows), the host bookkeeping and the errors.
The reference's own cache tests are re-run on CUDA tensors at the end.
"""

from __future__ import annotations

import hashlib

import pytest
import torch

import augur_b200 as ab
from augur_b200 import _lib, _ops, batched
from tests.conftest import assert_bits_equal, poison_

pytestmark = pytest.mark.gpu


def _poisoned(shape, dtype, device):
    return poison_(torch.empty(shape, dtype=dtype, device=device))


def _tiny_cfg(layers, hidden, heads, kv_heads):
    return ab.QwenConfig(vocab_size=16, hidden_size=hidden, intermediate_size=16,
                         num_hidden_layers=layers, num_attention_heads=heads,
                         num_key_value_heads=kv_heads)


def _strided(t: torch.Tensor, device) -> torch.Tensor:
    """[B, H, S, D] view over token-major storage, as augur's attention hands K/V to the cache."""
    return t.permute(0, 2, 1, 3).contiguous().to(device).permute(0, 2, 1, 3)


@pytest.mark.parametrize("case", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("positions_on_host", [False, True])
def test_write_kv_golden(cuda, golden, case, positions_on_host):
    c = golden["write_kv"][case]
    L, B, H, S, D = c["cfg"]
    cache = ab.KVCache(keys=_poisoned((L, B, H, S, D), c["keys"].dtype, cuda),
                       values=_poisoned((L, B, H, S, D), c["keys"].dtype, cuda))
    kptr, vptr = cache.keys.data_ptr(), cache.values.data_ptr()
    for call in c["calls"]:
        pos = call["positions"] if positions_on_host else call["positions"].to(cuda)
        rk, rv = ab.write_kv(cache, call["layer"], pos, _strided(call["key"], cuda), _strided(call["value"], cuda))
        assert cache.seq_len == call["seq_len"]
        assert list(rk.shape) == call["view_shape"] and rv.shape == rk.shape
    assert cache.keys.data_ptr() == kptr and cache.values.data_ptr() == vptr
    assert_bits_equal(cache.keys, c["keys"], "keys")
    assert_bits_equal(cache.values, c["values"], "values")
    assert _ops.read_status(cuda) == _lib.OK


def test_write_kv_dtype_mismatch_error(cuda, golden):
    cfg = _tiny_cfg(3, 16, 2, 2)
    cache = ab.new_kv_cache(cfg, batch_size=3, max_seq_len=12, device=cuda, dtype=torch.bfloat16)
    k = torch.randn(3, 2, 1, 8, device=cuda)
    with pytest.raises(RuntimeError) as exc:
        ab.write_kv(cache, 0, torch.zeros(3, 1, dtype=torch.int64), k, k)
    assert f"RuntimeError: {exc.value}" == golden["write_kv"]["dtype_mismatch_error"]


def test_write_paged_kv_golden(cuda, golden):
    for name, c in golden["paged"].items():
        dtype = c["keys"].dtype
        cache = ab.PagedKVCache(keys=_poisoned(c["keys"].shape, dtype, cuda),
                                values=_poisoned(c["keys"].shape, dtype, cuda),
                                block_size=c["block_size"], allocator=ab.BlockAllocator(c["num_blocks"]))
        if c["initial_table"] is None:
            table = ab.SequenceBlockTable.empty(c["block_size"])
        else:
            table = ab.SequenceBlockTable(block_ids=list(c["initial_table"]), block_size=c["block_size"])
        for call in c["calls"]:
            err = None
            try:
                ab.write_paged_kv(cache, call["layer"], table, torch.tensor([call["positions"]], device=cuda),
                                  _strided(call["key"], cuda), _strided(call["value"], cuda))
            except (ValueError, RuntimeError) as exc:
                err = f"{type(exc).__name__}: {exc}"
            assert err == call["error"], name
            assert table.block_ids == call["block_ids"] and table.seq_len == call["seq_len"], name
        assert_bits_equal(cache.keys, c["keys"], f"{name} keys")
        assert_bits_equal(cache.values, c["values"], f"{name} values")
        assert list(cache.allocator._free_blocks) == c["free_after"], name
        for layer, r in c["reads"].items():
            rk, rv = ab.read_paged_kv(cache, layer, table)
            assert_bits_equal(rk, r["key"], f"{name} read key {layer}")
            assert_bits_equal(rv, r["value"], f"{name} read value {layer}")
        assert _ops.read_status(cuda) == _lib.OK, name


@pytest.mark.parametrize("case", ["bf16", "f32_to_bf16", "f32"])
@pytest.mark.parametrize("entry_on", ["device", "host", "pinned_host"])
def test_copy_prefix_golden(cuda, golden, case, entry_on):
    """Entry on the device, in pageable host memory (transferred first) or in pinned host
    memory (read in place by the kernel)."""
    c = golden["prefix"][case]
    cache = ab.KVCache(keys=_poisoned(c["keys"].shape, c["keys"].dtype, cuda),
                       values=_poisoned(c["keys"].shape, c["keys"].dtype, cuda), seq_len=2)
    dev = cuda if entry_on == "device" else torch.device("cpu")
    entry = ab.PrefixCacheEntry(token_ids=torch.arange(6), keys=c["entry_keys"].to(dev),
                                values=c["entry_values"].to(dev), logits=torch.empty(0))
    if entry_on == "pinned_host":
        from augur_b200.offload import offload_prefix_entry

        entry = offload_prefix_entry(entry)
        assert entry.keys.is_pinned()
    ab.copy_prefix_into_cache(entry, cache, batch_idx=c["batch_idx"])
    assert cache.seq_len == c["seq_len"]
    assert_bits_equal(cache.keys, c["keys"], "keys")
    assert_bits_equal(cache.values, c["values"], "values")


@pytest.mark.parametrize("flags", [_lib.COPY_AUTO, _lib.COPY_VECTOR, _lib.COPY_BULK])
def test_handoff_golden(cuda, golden, flags):
    c = golden["handoff"]
    src = ab.KVCache(keys=c["src_keys"].to(cuda), values=c["src_values"].to(cuda))
    pool = ab.PagedKVCache(keys=_poisoned(c["keys"].shape, c["keys"].dtype, cuda),
                           values=_poisoned(c["keys"].shape, c["keys"].dtype, cuda),
                           block_size=c["keys"].shape[3], allocator=ab.BlockAllocator(c["num_blocks"]))
    tables = [ab.SequenceBlockTable(block_ids=list(ids), block_size=16) for ids in c["tables"]]
    batched.handoff_contiguous_to_paged(src, pool, tables, c["lens"], flags=flags)
    assert [t.seq_len for t in tables] == c["lens"]
    assert_bits_equal(pool.keys, c["keys"], "keys")
    assert_bits_equal(pool.values, c["values"], "values")
    assert _ops.read_status(cuda) == _lib.OK


def test_fork_cow_golden(cuda, golden):
    c = golden["fork"]
    P, S = c["prefix_len"], c["suffix_len"]
    L, _, H, _, D = c["prefix_keys"].shape
    pool = ab.PagedKVCache(keys=_poisoned((L, 32, H, 4, D), torch.bfloat16, cuda),
                           values=_poisoned((L, 32, H, 4, D), torch.bfloat16, cuda),
                           block_size=4, allocator=ab.BlockAllocator(32))
    parent = ab.SequenceBlockTable.empty(4)
    for layer in range(L):
        ab.write_paged_kv(pool, layer, parent, torch.arange(P, device=cuda).unsqueeze(0),
                          c["prefix_keys"][layer].to(cuda), c["prefix_values"][layer].to(cuda))
    forks = batched.fork_prefix(pool, parent, len(c["reads"]))
    assert batched.cow_partial_blocks(pool, forks) == len(forks)
    for f, table in enumerate(forks):
        for layer in range(L):
            ab.write_paged_kv(pool, layer, table, torch.arange(P, P + S, device=cuda).unsqueeze(0),
                              c["suffix_keys"][f, layer].to(cuda), c["suffix_values"][f, layer].to(cuda))
    # the parent's own partial block was never written past the prefix
    for f, table in enumerate(forks):
        assert table.block_ids[:-2] == parent.block_ids[:-1]
        for layer in range(L):
            rk, rv = ab.read_paged_kv(pool, layer, table)
            assert_bits_equal(rk, c["reads"][f][layer]["key"], f"fork {f} layer {layer} key")
            assert_bits_equal(rv, c["reads"][f][layer]["value"], f"fork {f} layer {layer} value")
    assert _ops.read_status(cuda) == _lib.OK


def test_config1_replay_bit_exact(cuda, config1_golden):
    """Full Qwen2.5-0.5B-shaped fp32 cache: replaying the reference's 24 x 33 write_kv calls."""
    c = config1_golden
    L, T, H, D = c["keys"].shape
    cfg = ab.QwenConfig()
    cache = ab.new_kv_cache(cfg, batch_size=1, max_seq_len=c["max_seq_len"], device=cuda, dtype=torch.float32)
    poison_(cache.keys)
    poison_(cache.values)
    keys, values, positions = c["keys"].to(cuda), c["values"].to(cuda), c["positions"]
    off = 0
    for n in c["call_sizes"]:
        for layer in range(L):
            pos = positions[layer, off : off + n].unsqueeze(0)  # host positions: no device sync
            k = keys[layer, off : off + n].permute(1, 0, 2).unsqueeze(0)
            v = values[layer, off : off + n].permute(1, 0, 2).unsqueeze(0)
            ab.write_kv(cache, layer, pos, k, v)
        off += n
    assert cache.seq_len == c["seq_len"]
    assert hashlib.sha256(cache.keys.cpu().numpy().tobytes()).hexdigest() == c["sha256_keys"]
    assert hashlib.sha256(cache.values.cpu().numpy().tobytes()).hexdigest() == c["sha256_values"]


# --- the reference's own cache tests, on CUDA tensors -----------------------


def _ref_cfg():
    return _tiny_cfg(2, 4, 2, 1)


def test_ref_write_kv_without_reallocating(cuda):
    cfg = _tiny_cfg(2, 8, 2, 1)
    cache = ab.new_kv_cache(cfg, batch_size=1, max_seq_len=4, device=cuda, dtype=torch.float32)
    kptr, vptr = cache.keys.data_ptr(), cache.values.data_ptr()
    k1, v1 = torch.randn(1, 1, 3, 4, device=cuda), torch.randn(1, 1, 3, 4, device=cuda)
    k2, v2 = torch.randn(1, 1, 1, 4, device=cuda), torch.randn(1, 1, 1, 4, device=cuda)
    ab.write_kv(cache, layer_idx=1, position_ids=torch.tensor([[0, 1, 2]]), key=k1, value=v1)
    ck, cv = ab.write_kv(cache, layer_idx=1, position_ids=torch.tensor([[3]]), key=k2, value=v2)
    assert cache.keys.data_ptr() == kptr and cache.values.data_ptr() == vptr
    assert cache.seq_len == 4 and ck.shape == (1, 1, 4, 4) and cv.shape == (1, 1, 4, 4)
    assert torch.equal(ck[:, :, :3], k1) and torch.equal(ck[:, :, 3:], k2)
    assert torch.equal(cv[:, :, :3], v1) and torch.equal(cv[:, :, 3:], v2)


def test_ref_write_kv_rejects_positions_outside_capacity(cuda):
    cache = ab.new_kv_cache(_tiny_cfg(2, 8, 2, 1), batch_size=1, max_seq_len=3, device=cuda,
                            dtype=torch.float32)
    k = torch.randn(1, 1, 1, 4, device=cuda)
    with pytest.raises(ValueError, match="exceeds cache capacity"):
        ab.write_kv(cache, layer_idx=0, position_ids=torch.tensor([[3]], device=cuda), key=k, value=k)
    with pytest.raises(ValueError, match="must be non-negative"):
        ab.write_kv(cache, layer_idx=0, position_ids=torch.tensor([[-1]], device=cuda), key=k, value=k)
    with pytest.raises(ValueError, match="same device"):
        ab.write_kv(cache, layer_idx=0, position_ids=torch.tensor([[0]]), key=k.cpu(), value=k.cpu())


def test_ref_paged_scatter_and_read(cuda):
    cache = ab.new_paged_kv_cache(_ref_cfg(), num_blocks=3, block_size=4, device=cuda, dtype=torch.float32)
    table = ab.SequenceBlockTable(block_ids=[2, 0, 1], block_size=4)
    key = torch.tensor([[[[10.0, 11.0], [20.0, 21.0], [30.0, 31.0]]]], device=cuda)
    value = torch.tensor([[[[110.0, 111.0], [120.0, 121.0], [130.0, 131.0]]]], device=cuda)
    ab.write_paged_kv(cache, 1, table, torch.tensor([[3, 4, 9]], device=cuda), key, value)
    rk, rv = ab.read_paged_kv(cache, 1, table, seq_len=10)
    assert torch.equal(cache.keys[1, 2, :, 3, :], key[0, :, 0, :])
    assert torch.equal(cache.keys[1, 0, :, 0, :], key[0, :, 1, :])
    assert torch.equal(cache.keys[1, 1, :, 1, :], key[0, :, 2, :])
    assert torch.equal(rk[:, :, [3, 4, 9], :], key) and torch.equal(rv[:, :, [3, 4, 9], :], value)


def test_ref_paged_lazy_allocation_and_default_length(cuda):
    cache = ab.new_paged_kv_cache(_ref_cfg(), num_blocks=3, block_size=4, device=cuda, dtype=torch.float32)
    table = ab.SequenceBlockTable.empty(4)
    key = torch.tensor([[[[10.0, 11.0], [20.0, 21.0]]]], device=cuda)
    ab.write_paged_kv(cache, 1, table, torch.tensor([[0, 4]]), key, key + 100)
    assert table.block_ids == [0, 1]
    assert torch.equal(cache.keys[1, 0, :, 0, :], key[0, :, 0, :])
    assert torch.equal(cache.keys[1, 1, :, 0, :], key[0, :, 1, :])
    cache2 = ab.new_paged_kv_cache(_ref_cfg(), num_blocks=2, block_size=4, device=cuda, dtype=torch.float32)
    t2 = ab.SequenceBlockTable.empty(4)
    k = torch.arange(10, dtype=torch.float32, device=cuda).view(1, 1, 5, 2)
    v = torch.arange(100, 110, dtype=torch.float32, device=cuda).view(1, 1, 5, 2)
    ab.write_paged_kv(cache2, 1, t2, torch.tensor([[0, 1, 2, 3, 4]]), k, v)
    rk, rv = ab.read_paged_kv(cache2, 1, t2)
    assert t2.seq_len == 5 and torch.equal(rk, k) and torch.equal(rv, v)


def test_ref_paged_read_matches_contiguous(cuda):
    cfg = _ref_cfg()
    contiguous = ab.new_kv_cache(cfg, batch_size=1, max_seq_len=6, device=cuda, dtype=torch.float32)
    paged = ab.new_paged_kv_cache(cfg, num_blocks=2, block_size=4, device=cuda, dtype=torch.float32)
    table = ab.SequenceBlockTable(block_ids=[1, 0], block_size=4)
    key = torch.arange(12, dtype=torch.float32, device=cuda).view(1, 1, 6, 2)
    value = torch.arange(100, 112, dtype=torch.float32, device=cuda).view(1, 1, 6, 2)
    pos = torch.tensor([[0, 1, 2, 3, 4, 5]], device=cuda)
    ck, cv = ab.write_kv(contiguous, 1, pos, key, value)
    ab.write_paged_kv(paged, 1, table, pos, key, value)
    pk, pv = ab.read_paged_kv(paged, 1, table, seq_len=6)
    assert torch.equal(pk, ck) and torch.equal(pv, cv)


def test_ref_copy_prefix(cuda):
    cache = ab.new_kv_cache(_ref_cfg(), batch_size=1, max_seq_len=5, device=cuda, dtype=torch.float32)
    entry = ab.PrefixCacheEntry(token_ids=torch.tensor([1, 2, 3]),
                                keys=torch.arange(12, dtype=torch.float32).view(2, 1, 3, 2),
                                values=torch.arange(100, 112, dtype=torch.float32).view(2, 1, 3, 2),
                                logits=torch.empty(0))
    ab.copy_prefix_into_cache(entry, cache)
    assert cache.seq_len == 3
    assert torch.equal(cache.keys[:, 0, :, :3, :].cpu(), entry.keys)
    assert torch.equal(cache.values[:, 0, :, :3, :].cpu(), entry.values)


@pytest.mark.parametrize("case", ["f32", "bf16"])
@pytest.mark.parametrize("positions_on_host", [False, True])
def test_duplicate_positions_golden(cuda, golden, case, positions_on_host):
    """A position repeated in one call keeps the later token, as in the reference's
    write_kv (index_put per row) and write_paged_kv (per-token loop)."""
    c = golden["duplicates"][f"write_kv_{case}"]
    L, B, H, S, D = c["cfg"]
    cache = ab.KVCache(keys=_poisoned((L, B, H, S, D), c["keys"].dtype, cuda),
                       values=_poisoned((L, B, H, S, D), c["keys"].dtype, cuda))
    pos = c["positions"] if positions_on_host else c["positions"].to(cuda)
    ab.write_kv(cache, c["layer"], pos, _strided(c["key"], cuda), _strided(c["value"], cuda))
    assert cache.seq_len == c["seq_len"]
    assert_bits_equal(cache.keys, c["keys"], "write_kv keys")
    assert_bits_equal(cache.values, c["values"], "write_kv values")
    p = golden["duplicates"][f"write_paged_kv_{case}"]
    pool = ab.PagedKVCache(keys=_poisoned(p["keys"].shape, p["keys"].dtype, cuda),
                           values=_poisoned(p["keys"].shape, p["keys"].dtype, cuda),
                           block_size=p["block_size"], allocator=ab.BlockAllocator(p["num_blocks"]))
    table = ab.SequenceBlockTable.empty(p["block_size"])
    ppos = p["positions"] if positions_on_host else p["positions"].to(cuda)
    ab.write_paged_kv(pool, p["layer"], table, ppos, _strided(p["key"], cuda), _strided(p["value"], cuda))
    assert table.block_ids == p["block_ids"] and table.seq_len == p["seq_len"]
    assert_bits_equal(pool.keys, p["keys"], "write_paged_kv keys")
    assert_bits_equal(pool.values, p["values"], "write_paged_kv values")
    assert _ops.read_status(cuda) == _lib.OK


def test_cache_prefix_copies_the_cache_through_the_library(cuda, monkeypatch):
    """cache_prefix runs augur's forward (a stand-in here) into a fresh cache and keeps its
    K/V as [layers, kv_heads, prefix, head_dim]; the copy out of the cache is one run-copy
    launch, bit-exact with the rows the forward wrote."""
    from types import SimpleNamespace

    from augur_b200 import prefix_cache

    cfg = _tiny_cfg(3, 16, 2, 2)  # head_dim 8
    g = torch.Generator(device=cuda).manual_seed(8)
    wrote = {}

    def fake_model(input_ids, w, cfg, cache=None, position_ids=None):
        n = input_ids.shape[1]
        assert position_ids.tolist() == [list(range(n))]
        wrote["k"] = torch.randn(cache.keys[:, 0, :, :n].shape, generator=g, device=cuda).to(cache.keys.dtype)
        wrote["v"] = torch.randn(cache.keys[:, 0, :, :n].shape, generator=g, device=cuda).to(cache.keys.dtype)
        cache.keys[:, 0, :, :n] = wrote["k"]
        cache.values[:, 0, :, :n] = wrote["v"]
        cache.seq_len = n
        return torch.zeros(1, n, cfg.vocab_size, device=cuda)

    monkeypatch.setattr(prefix_cache, "model", fake_model)
    launches = _ops.launch_count
    entry = ab.cache_prefix(torch.tensor([[4, 5, 6, 7, 8]], device=cuda),
                            SimpleNamespace(embed_tokens=torch.empty(0, dtype=torch.bfloat16)), cfg)
    assert _ops.launch_count == launches + 1
    assert entry.keys.shape == (3, 2, 5, 8) and entry.keys.device == cuda
    assert_bits_equal(entry.keys, wrote["k"], "entry keys")
    assert_bits_equal(entry.values, wrote["v"], "entry values")
    assert entry.token_ids.tolist() == [4, 5, 6, 7, 8] and entry.logits.shape == (1, 1, cfg.vocab_size)
