"""Generate the golden fixtures by running the reference (semioz/augur) itself.

    python tests/golden/make_golden.py --reference <checkout of semioz/augur>

(or set AUGUR_REFERENCE to the checkout). This script needs the reference
source tree (pure Python + torch) and runs only where that tree exists; the fixtures it writes are committed and are
all that the tests read. Every case starts from caches filled with the byte
0xFF (a NaN pattern), runs the reference's own functions, and stores inputs
plus the resulting cache contents, so a comparison covers both the written
rows and every row that must stay untouched.

Outputs:
  reference_cases.pt  small seeded cases of write_kv, write_paged_kv,
                      read_paged_kv, copy_prefix_into_cache, the handoff and
                      fork compositions, duplicate positions in one call,
                      decode and prefill attention over a paged cache,
                      allocator / block table / prefix-hash scripts;
  config1_writes.pt   the full Qwen2.5-0.5B-shaped random-init model (fp32,
                      CPU): 128-token prefill into new_kv_cache(max_seq_len=512)
                      plus 32 greedy decode forwards, with every write_kv call
                      recorded (layer, positions, K, V) and the SHA-256 of the
                      reference's final K and V caches.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def poison(t: torch.Tensor) -> torch.Tensor:
    t.view(torch.uint8).fill_(0xFF)
    return t


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def strided_kv(g: torch.Generator, batch, heads, seq, dim, dtype):
    """[batch, heads, seq, dim] views over token-major storage, as attention produces them."""
    base = torch.randn(batch, seq, heads, dim, generator=g).to(dtype)
    return base.permute(0, 2, 1, 3)


def write_kv_cases(ref, g):
    cfg = ref.config.QwenConfig(vocab_size=16, hidden_size=16, intermediate_size=16,
                                num_hidden_layers=3, num_attention_heads=2, num_key_value_heads=2)
    # head_dim = 8
    cases = {}
    for name, kdtype, cdtype in (("f32", torch.float32, torch.float32),
                                 ("bf16", torch.bfloat16, torch.bfloat16),
                                 ("f16", torch.float16, torch.float16)):
        cache = ref.kv_cache.new_kv_cache(cfg, batch_size=3, max_seq_len=12,
                                          device=torch.device("cpu"), dtype=cdtype)
        poison(cache.keys)
        poison(cache.values)
        calls = []
        # prefill through an expanded (stride 0) position tensor
        pos = torch.arange(5).expand(3, -1)
        calls.append((1, pos))
        calls.append((1, torch.full((3, 1), 5)))
        calls.append((2, torch.tensor([[3, 1, 0, 2], [0, 1, 2, 3], [7, 6, 5, 4]])))
        calls.append((0, torch.tensor([[11], [0], [6]])))
        recorded = []
        for layer, p in calls:
            k = strided_kv(g, 3, 2, p.shape[1], 8, kdtype)
            v = strided_kv(g, 3, 2, p.shape[1], 8, kdtype)
            rk, rv = ref.kv_cache.write_kv(cache, layer, p, k, v)
            recorded.append({"layer": layer, "positions": p.contiguous(), "key": k.contiguous(),
                             "value": v.contiguous(), "seq_len": cache.seq_len,
                             "view_shape": list(rk.shape)})
        cases[name] = {"calls": recorded, "keys": cache.keys.clone(), "values": cache.values.clone(),
                       "seq_len": cache.seq_len, "cfg": [3, 3, 2, 12, 8]}
    # write_kv does not convert: index_put rejects a source dtype that differs from the cache's
    cache = ref.kv_cache.new_kv_cache(cfg, batch_size=3, max_seq_len=12, device=torch.device("cpu"),
                                      dtype=torch.bfloat16)
    try:
        k = strided_kv(g, 3, 2, 1, 8, torch.float32)
        ref.kv_cache.write_kv(cache, 0, torch.zeros(3, 1, dtype=torch.int64), k, k)
        mismatch = None
    except RuntimeError as exc:
        mismatch = f"{type(exc).__name__}: {exc}"
    cases["dtype_mismatch_error"] = mismatch
    return cases


def paged_cases(ref, g):
    P = ref.paged_kv_cache
    cfg = ref.config.QwenConfig(vocab_size=16, hidden_size=16, intermediate_size=16,
                                num_hidden_layers=2, num_attention_heads=2, num_key_value_heads=2)
    cases = {}
    scripts = {
        # lazy allocation from an empty table: prefill 7 tokens, then decode appends
        "lazy": dict(num_blocks=8, block_size=4, table=None,
                     calls=[(0, list(range(7))), (1, list(range(7))), (0, [7]), (1, [7]),
                            (0, [8]), (1, [8])]),
        # a pre-built permuted table and non-monotone positions
        "perm": dict(num_blocks=8, block_size=4, table=[5, 2, 7, 0],
                     calls=[(1, [9, 3, 14, 0, 6]), (0, [15, 1, 2])]),
        # pool exhaustion part-way through a call: earlier tokens stay written
        "exhaust": dict(num_blocks=3, block_size=2, table=None, calls=[(0, list(range(8)))]),
        # a negative position part-way: earlier tokens stay written
        "negative": dict(num_blocks=4, block_size=4, table=None, calls=[(1, [0, 1, 2, -1, 3])]),
    }
    # (name, source dtype, pool dtype): basic-index assignment converts dtypes
    for dname, sdtype, dtype in (("f32", torch.float32, torch.float32),
                                 ("bf16", torch.bfloat16, torch.bfloat16),
                                 ("f32_to_bf16", torch.float32, torch.bfloat16),
                                 ("bf16_to_f16", torch.bfloat16, torch.float16)):
        for sname, sc in scripts.items():
            if dname in ("f32_to_bf16", "bf16_to_f16") and sname not in ("lazy", "perm"):
                continue
            cache = P.new_paged_kv_cache(cfg, num_blocks=sc["num_blocks"], block_size=sc["block_size"],
                                         device=torch.device("cpu"), dtype=dtype)
            poison(cache.keys)
            poison(cache.values)
            if sc["table"] is None:
                table = P.SequenceBlockTable.empty(block_size=sc["block_size"])
            else:
                table = P.SequenceBlockTable(block_ids=list(sc["table"]), block_size=sc["block_size"])
            recorded = []
            for layer, positions in sc["calls"]:
                k = strided_kv(g, 1, 2, len(positions), 8, sdtype)
                v = strided_kv(g, 1, 2, len(positions), 8, sdtype)
                err = None
                try:
                    P.write_paged_kv(cache, layer, table, torch.tensor([positions]), k, v)
                except (ValueError, RuntimeError) as exc:
                    err = f"{type(exc).__name__}: {exc}"
                recorded.append({"layer": layer, "positions": list(positions), "key": k.contiguous(),
                                 "value": v.contiguous(), "error": err,
                                 "block_ids": list(table.block_ids), "seq_len": table.seq_len})
            reads = {}
            if table.seq_len > 0:
                for layer in range(2):
                    rk, rv = P.read_paged_kv(cache, layer, table)
                    reads[layer] = {"key": rk.clone(), "value": rv.clone()}
            cases[f"{sname}_{dname}"] = {
                "num_blocks": sc["num_blocks"], "block_size": sc["block_size"],
                "initial_table": sc["table"], "calls": recorded, "keys": cache.keys.clone(),
                "values": cache.values.clone(), "block_ids": list(table.block_ids),
                "seq_len": table.seq_len, "reads": reads,
                "free_after": list(cache.allocator._free_blocks),
            }
    return cases


def prefix_cases(ref, g):
    cfg = ref.config.QwenConfig(vocab_size=16, hidden_size=16, intermediate_size=16,
                                num_hidden_layers=2, num_attention_heads=2, num_key_value_heads=2)
    cases = {}
    for name, edtype, cdtype in (("bf16", torch.bfloat16, torch.bfloat16),
                                 ("f32_to_bf16", torch.float32, torch.bfloat16),
                                 ("f32", torch.float32, torch.float32)):
        cache = ref.kv_cache.new_kv_cache(cfg, batch_size=3, max_seq_len=10,
                                          device=torch.device("cpu"), dtype=cdtype)
        poison(cache.keys)
        poison(cache.values)
        cache.seq_len = 2
        entry = ref.prefix_cache.PrefixCacheEntry(
            token_ids=torch.arange(6),
            keys=torch.randn(2, 2, 6, 8, generator=g).to(edtype),
            values=torch.randn(2, 2, 6, 8, generator=g).to(edtype),
            logits=torch.empty(0),
        )
        ref.prefix_cache.copy_prefix_into_cache(entry, cache, batch_idx=2)
        cases[name] = {"entry_keys": entry.keys, "entry_values": entry.values, "batch_idx": 2,
                       "keys": cache.keys.clone(), "values": cache.values.clone(),
                       "seq_len": cache.seq_len}
    return cases


def handoff_case(ref, g):
    """Contiguous prefill cache -> paged pool, composed from the reference's write_paged_kv."""
    P = ref.paged_kv_cache
    cfg = ref.config.QwenConfig(vocab_size=16, hidden_size=32, intermediate_size=16,
                                num_hidden_layers=3, num_attention_heads=2, num_key_value_heads=2)
    # head_dim 16, block_size 16: a full block is 16 rows per (layer, head)
    contiguous = ref.kv_cache.new_kv_cache(cfg, batch_size=4, max_seq_len=40,
                                           device=torch.device("cpu"), dtype=torch.bfloat16)
    contiguous.keys.copy_(torch.randn(contiguous.keys.shape, generator=g).to(torch.bfloat16))
    contiguous.values.copy_(torch.randn(contiguous.values.shape, generator=g).to(torch.bfloat16))
    lens = [37, 16, 1, 29]
    pool = P.new_paged_kv_cache(cfg, num_blocks=40, block_size=16, device=torch.device("cpu"),
                                dtype=torch.bfloat16)
    poison(pool.keys)
    poison(pool.values)
    perm = torch.randperm(40, generator=g).tolist()
    tables, cursor = [], 0
    for n in lens:
        nb = -(-n // 16)
        tables.append(P.SequenceBlockTable(block_ids=perm[cursor : cursor + nb], block_size=16))
        cursor += nb
    for b, n in enumerate(lens):
        for layer in range(3):
            P.write_paged_kv(pool, layer, tables[b], torch.arange(n).unsqueeze(0),
                             contiguous.keys[layer, b : b + 1, :, :n, :],
                             contiguous.values[layer, b : b + 1, :, :n, :])
    return {"src_keys": contiguous.keys.clone(), "src_values": contiguous.values.clone(),
            "lens": lens, "tables": [t.block_ids for t in tables], "num_blocks": 40,
            "keys": pool.keys.clone(), "values": pool.values.clone()}


def fork_case(ref, g):
    """A 21-token prefix (bs 4: 5 full blocks + 1 row) shared by 3 forks that each append 6 tokens.

    The reference has no fork; its equivalent per fork is a private table
    written with the prefix and then the suffix. Stored: the prefix and
    suffix K/V and each fork's read_paged_kv of every layer.
    """
    P = ref.paged_kv_cache
    cfg = ref.config.QwenConfig(vocab_size=16, hidden_size=16, intermediate_size=16,
                                num_hidden_layers=2, num_attention_heads=2, num_key_value_heads=2)
    prefix_len, suffix_len, forks = 21, 6, 3
    pk = torch.randn(2, 1, 2, prefix_len, 8, generator=g).to(torch.bfloat16)
    pv = torch.randn(2, 1, 2, prefix_len, 8, generator=g).to(torch.bfloat16)
    sk = torch.randn(forks, 2, 1, 2, suffix_len, 8, generator=g).to(torch.bfloat16)
    sv = torch.randn(forks, 2, 1, 2, suffix_len, 8, generator=g).to(torch.bfloat16)
    reads = []
    for f in range(forks):
        pool = P.new_paged_kv_cache(cfg, num_blocks=16, block_size=4, device=torch.device("cpu"),
                                    dtype=torch.bfloat16)
        table = P.SequenceBlockTable.empty(block_size=4)
        for layer in range(2):
            P.write_paged_kv(pool, layer, table, torch.arange(prefix_len).unsqueeze(0), pk[layer], pv[layer])
        for layer in range(2):
            P.write_paged_kv(pool, layer, table,
                             torch.arange(prefix_len, prefix_len + suffix_len).unsqueeze(0),
                             sk[f, layer], sv[f, layer])
        per_layer = []
        for layer in range(2):
            rk, rv = P.read_paged_kv(pool, layer, table)
            per_layer.append({"key": rk.clone(), "value": rv.clone()})
        reads.append(per_layer)
    return {"prefix_len": prefix_len, "suffix_len": suffix_len, "prefix_keys": pk,
            "prefix_values": pv, "suffix_keys": sk, "suffix_values": sv, "reads": reads}


def attention_cases(ref, g):
    """Decode-step paged attention through the reference's own attention() (augur/attention.py:22-92).

    augur's GQA shape (14 query heads, 2 KV heads, head_dim 64), one layer,
    block size 16. The prompt is prefilled through attention() with a paged
    cache, then one decode token; the o-projection is the identity, so the
    output is the attention core (heads concatenated). Stored: the rotated
    decode query, the pool, the block table and the reference output.
    """
    import torch.nn.functional as F
    from einops import rearrange

    from augur.attention import attention
    from augur.rope import apply_rope

    P = ref.paged_kv_cache
    W = ref.weights
    cases = {}
    for name, dtype, seq in (("f32", torch.float32, 37), ("bf16", torch.bfloat16, 300)):
        cfg = ref.config.QwenConfig(vocab_size=16, hidden_size=896, intermediate_size=16,
                                    num_hidden_layers=1, num_attention_heads=14, num_key_value_heads=2)
        D, Hq, Hkv = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
        w = W.Attention(
            q=W.Linear((torch.randn(Hq * D, 896, generator=g) * 0.06).to(dtype),
                       (torch.randn(Hq * D, generator=g) * 0.1).to(dtype)),
            k=W.Linear((torch.randn(Hkv * D, 896, generator=g) * 0.06).to(dtype),
                       (torch.randn(Hkv * D, generator=g) * 0.1).to(dtype)),
            v=W.Linear((torch.randn(Hkv * D, 896, generator=g) * 0.06).to(dtype)),
            o=W.Linear(torch.eye(896, dtype=dtype)),
        )
        x = torch.randn(1, seq, 896, generator=g).to(dtype)
        state = P.PagedKVCacheState(
            cache=P.new_paged_kv_cache(cfg, num_blocks=-(-seq // 16) + 3, block_size=16,
                                       device=torch.device("cpu"), dtype=dtype),
            block_table=P.SequenceBlockTable.empty(block_size=16),
        )
        poison(state.cache.keys)  # rows never written stay 0xFF: deterministic fixtures
        poison(state.cache.values)
        state.cache.allocator.allocate()  # the pool already holds another block
        pos = torch.arange(seq).unsqueeze(0)
        attention(x[:, : seq - 1], w, cfg, pos[:, : seq - 1], paged_cache=state, layer_idx=0)
        out = attention(x[:, seq - 1 :], w, cfg, pos[:, seq - 1 :], paged_cache=state, layer_idx=0)
        q = rearrange(F.linear(x[:, seq - 1 :], w.q.weight, w.q.bias),
                      "batch seq (heads head_dim) -> batch heads seq head_dim", heads=Hq, head_dim=D)
        k_last = rearrange(F.linear(x[:, seq - 1 :], w.k.weight, w.k.bias),
                           "batch seq (heads head_dim) -> batch heads seq head_dim", heads=Hkv, head_dim=D)
        q, _ = apply_rope(q, k_last, pos[:, seq - 1 :], cfg.rope_theta)
        kk, vv = P.read_paged_kv(state.cache, 0, state.block_table)
        cases[name] = {"q": q.contiguous(), "keys": state.cache.keys.clone(), "values": state.cache.values.clone(),
                       "block_ids": list(state.block_table.block_ids), "seq_len": state.block_table.seq_len,
                       "k": kk.clone(), "v": vv.clone(),
                       "out": out.view(1, 1, Hq, D).permute(0, 2, 1, 3).contiguous(),
                       "n_kv_heads": Hkv}
    return cases


def prefill_attention_cases(ref, g):
    """Prefill attention over a paged cache through the reference's own attention()
    (augur/attention.py:22-92): a prefix of P tokens is prefilled first (P = 0: none),
    then a call with the n suffix tokens (seq = n > 1), whose queries attend to the
    prefix and causally to each other. augur's GQA shape, one layer, block size 16,
    o-projection the identity. Stored: the suffix's rotated queries, the pool, the
    block table and the reference output of the suffix call."""
    import torch.nn.functional as F
    from einops import rearrange

    from augur.attention import attention
    from augur.rope import apply_rope

    P = ref.paged_kv_cache
    W = ref.weights
    cases = {}
    for name, dtype, prefix, n in (("f32_prefix", torch.float32, 21, 16), ("bf16_prefix", torch.bfloat16, 200, 45),
                                   ("bf16_plain", torch.bfloat16, 0, 37)):
        cfg = ref.config.QwenConfig(vocab_size=16, hidden_size=896, intermediate_size=16,
                                    num_hidden_layers=1, num_attention_heads=14, num_key_value_heads=2)
        D, Hq, Hkv = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
        w = W.Attention(
            q=W.Linear((torch.randn(Hq * D, 896, generator=g) * 0.06).to(dtype),
                       (torch.randn(Hq * D, generator=g) * 0.1).to(dtype)),
            k=W.Linear((torch.randn(Hkv * D, 896, generator=g) * 0.06).to(dtype),
                       (torch.randn(Hkv * D, generator=g) * 0.1).to(dtype)),
            v=W.Linear((torch.randn(Hkv * D, 896, generator=g) * 0.06).to(dtype)),
            o=W.Linear(torch.eye(896, dtype=dtype)),
        )
        seq = prefix + n
        x = torch.randn(1, seq, 896, generator=g).to(dtype)
        state = P.PagedKVCacheState(
            cache=P.new_paged_kv_cache(cfg, num_blocks=-(-seq // 16) + 3, block_size=16,
                                       device=torch.device("cpu"), dtype=dtype),
            block_table=P.SequenceBlockTable.empty(block_size=16),
        )
        poison(state.cache.keys)
        poison(state.cache.values)
        state.cache.allocator.allocate()  # the pool already holds another block
        pos = torch.arange(seq).unsqueeze(0)
        if prefix:
            attention(x[:, :prefix], w, cfg, pos[:, :prefix], paged_cache=state, layer_idx=0)
        out = attention(x[:, prefix:], w, cfg, pos[:, prefix:], paged_cache=state, layer_idx=0)
        q = rearrange(F.linear(x[:, prefix:], w.q.weight, w.q.bias),
                      "batch seq (heads head_dim) -> batch heads seq head_dim", heads=Hq, head_dim=D)
        k_new = rearrange(F.linear(x[:, prefix:], w.k.weight, w.k.bias),
                          "batch seq (heads head_dim) -> batch heads seq head_dim", heads=Hkv, head_dim=D)
        q, _ = apply_rope(q, k_new, pos[:, prefix:], cfg.rope_theta)
        kk, vv = P.read_paged_kv(state.cache, 0, state.block_table)
        cases[name] = {"q": q.contiguous(), "keys": state.cache.keys.clone(), "values": state.cache.values.clone(),
                       "block_ids": list(state.block_table.block_ids), "seq_len": state.block_table.seq_len,
                       "k": kk.clone(), "v": vv.clone(), "prefix_len": prefix, "n": n,
                       "out": out.view(1, n, Hq, D).permute(0, 2, 1, 3).contiguous(), "n_kv_heads": Hkv}
    return cases


def rope_cases(ref, g):
    """apply_rope (augur/rope.py:12-40) followed by the cache write, as augur/attention.py:53-71 runs it.

    theta 1e6 (Qwen2.5's), 14 query / 2 KV heads, head_dim 64, fp32 / bf16 / fp16:
    - paged_*: write_paged_kv (block 16, one layer, a 40-block poisoned pool that
      already holds another block) of a 37-token chunk at positions 100..136, then
      one decode token at position 600 (the table grows lazily to 38 blocks).
      Stored: the inputs of each call, the rotated q, the block table and the
      pool blocks the calls touched (every other block must still be poison).
    - contig_*: write_kv of 5 tokens into two batch rows at positions 0..4 and 20..24.
    - far_*: apply_rope alone at positions 0, 1, 4095, 8191, 32767 (large angles).
    q / k / v are strided views of a token-major projection, as in the reference.
    """
    from augur.rope import apply_rope

    P, K = ref.paged_kv_cache, ref.kv_cache
    theta = 1000000.0
    cases = {}
    for name, dtype in (("f32", torch.float32), ("bf16", torch.bfloat16), ("f16", torch.float16)):
        cfg = ref.config.QwenConfig(vocab_size=16, hidden_size=896, intermediate_size=16, num_hidden_layers=1,
                                    num_attention_heads=14, num_key_value_heads=2)
        pool = P.new_paged_kv_cache(cfg, num_blocks=40, block_size=16, device=torch.device("cpu"), dtype=dtype)
        poison(pool.keys)
        poison(pool.values)
        pool.allocator.allocate()  # another sequence's block
        table = P.SequenceBlockTable.empty(block_size=16)
        calls, touched = [], set()
        for pos in (torch.arange(100, 137), torch.tensor([600])):
            S = pos.numel()
            q = strided_kv(g, 1, 14, S, 64, dtype)
            k = strided_kv(g, 1, 2, S, 64, dtype)
            v = strided_kv(g, 1, 2, S, 64, dtype)
            qe, ke = apply_rope(q, k, pos[None], theta)
            P.write_paged_kv(pool, 0, table, pos[None], ke, v)
            touched.update(int(p) // 16 for p in pos)
            calls.append({"q": q, "k": k, "v": v, "position_ids": pos[None].clone(), "q_embed": qe.contiguous()})
        blocks = [table.block_ids[j] for j in sorted(touched)]
        cases[f"paged_{name}"] = {"calls": calls, "block_ids": list(table.block_ids), "touched_blocks": blocks,
                                  "keys": pool.keys[:, blocks].clone(), "values": pool.values[:, blocks].clone(),
                                  "num_blocks": 40, "prior_allocated": 1, "theta": theta}
        cache = K.new_kv_cache(cfg, batch_size=2, max_seq_len=32, device=torch.device("cpu"), dtype=dtype)
        poison(cache.keys)
        poison(cache.values)
        pos = torch.stack([torch.arange(0, 5), torch.arange(20, 25)])
        q = strided_kv(g, 2, 14, 5, 64, dtype)
        k = strided_kv(g, 2, 2, 5, 64, dtype)
        v = strided_kv(g, 2, 2, 5, 64, dtype)
        qe, ke = apply_rope(q, k, pos, theta)
        K.write_kv(cache, 0, pos, ke, v)
        cases[f"contig_{name}"] = {"q": q, "k": k, "v": v, "position_ids": pos, "q_embed": qe.contiguous(),
                                   "keys": cache.keys.clone(), "values": cache.values.clone(),
                                   "seq_len": cache.seq_len, "theta": theta}
        pos = torch.tensor([[0, 1, 4095, 8191, 32767]])
        q = strided_kv(g, 1, 14, 5, 64, dtype)
        k = strided_kv(g, 1, 2, 5, 64, dtype)
        qe, ke = apply_rope(q, k, pos, theta)
        cases[f"far_{name}"] = {"q": q, "k": k, "position_ids": pos, "q_embed": qe.contiguous(),
                                "k_embed": ke.contiguous(), "theta": theta}
    return cases


def duplicate_cases(ref, g):
    """Duplicate positions in one call: write_kv (per-row index_put) and write_paged_kv
    (per-token loop), from poisoned caches; the reference keeps the last token written."""
    cfg = ref.config.QwenConfig(vocab_size=16, hidden_size=16, intermediate_size=16,
                                num_hidden_layers=2, num_attention_heads=2, num_key_value_heads=2)
    cases = {}
    for name, dtype in (("f32", torch.float32), ("bf16", torch.bfloat16)):
        cache = ref.kv_cache.new_kv_cache(cfg, batch_size=3, max_seq_len=12, device=torch.device("cpu"),
                                          dtype=dtype)
        poison(cache.keys)
        poison(cache.values)
        pos = torch.tensor([[2, 4, 2, 9, 4], [0, 0, 0, 1, 0], [5, 6, 7, 5, 11]])
        k = strided_kv(g, 3, 2, 5, 8, dtype)
        v = strided_kv(g, 3, 2, 5, 8, dtype)
        ref.kv_cache.write_kv(cache, 1, pos, k, v)
        cases[f"write_kv_{name}"] = {"layer": 1, "positions": pos, "key": k.contiguous(), "value": v.contiguous(),
                                     "keys": cache.keys.clone(), "values": cache.values.clone(),
                                     "seq_len": cache.seq_len, "cfg": [2, 3, 2, 12, 8]}
        pool = ref.paged_kv_cache.new_paged_kv_cache(cfg, num_blocks=6, block_size=4,
                                                     device=torch.device("cpu"), dtype=dtype)
        poison(pool.keys)
        poison(pool.values)
        table = ref.paged_kv_cache.SequenceBlockTable.empty(4)
        ppos = torch.tensor([[3, 5, 3, 7, 5, 9, 3]])
        pk = strided_kv(g, 1, 2, 7, 8, dtype)
        pv = strided_kv(g, 1, 2, 7, 8, dtype)
        ref.paged_kv_cache.write_paged_kv(pool, 0, table, ppos, pk, pv)
        cases[f"write_paged_kv_{name}"] = {"layer": 0, "positions": ppos, "key": pk.contiguous(),
                                           "value": pv.contiguous(), "keys": pool.keys.clone(),
                                           "values": pool.values.clone(), "block_ids": list(table.block_ids),
                                           "seq_len": table.seq_len, "num_blocks": 6, "block_size": 4}
    return cases


def bookkeeping_scripts(ref):
    P = ref.paged_kv_cache
    alloc = P.BlockAllocator(num_blocks=12)
    log = []
    a = [alloc.allocate() for _ in range(4)]
    log.append(("allocate4", a))
    alloc.free(a[1])
    alloc.free(a[3])
    log.append(("after_free_1_3", list(alloc._free_blocks)))
    log.append(("allocate3", [alloc.allocate() for _ in range(3)]))
    table = P.SequenceBlockTable.empty(block_size=4)
    table.ensure_position(13, alloc)
    log.append(("ensure13", list(table.block_ids), table.seq_len))
    table.free(alloc)
    log.append(("free_table", list(alloc._free_blocks)))
    t2 = P.SequenceBlockTable.allocate(alloc, max_seq_len=9, block_size=4)
    log.append(("table_allocate9", list(t2.block_ids), t2.seq_len))
    pc = P.PagedPrefixCache()
    h1 = pc.add_block(None, [1, 2, 3, 4], 7)
    h2 = pc.add_block(h1, [5, 6, 7, 8], 9)
    h3 = pc.add_block(h2, [9, 10, 11, 12], 3)
    hx = pc.add_block(None, [5, 6, 7, 8], 11)
    m = [pc.match_prefix(ids, 4) for ids in ([1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13],
                                              [1, 2, 3, 4, 5, 6, 7], [5, 6, 7, 8, 1, 2, 3, 4],
                                              [9, 9, 9, 9])]
    log.append(("hashes", [h1, h2, h3, hx]))
    log.append(("matches", [(x.block_ids, x.matched_tokens) for x in m]))
    return log


def config1(ref):
    """Full random-init Qwen2.5-0.5B shape, fp32 CPU: 128-token prefill + 32 greedy decode forwards."""
    cfg = ref.config.QwenConfig()
    g = torch.Generator().manual_seed(0)
    W = ref.weights
    D = cfg.hidden_size
    kvd = cfg.num_key_value_heads * cfg.head_dim

    def lin(out_f, in_f, bias):
        w = torch.randn(out_f, in_f, generator=g) * 0.02
        b = torch.randn(out_f, generator=g) * 0.02 if bias else None
        return W.Linear(weight=w, bias=b)

    embed = torch.randn(cfg.vocab_size, D, generator=g) * 0.02
    layers = []
    for _ in range(cfg.num_hidden_layers):
        layers.append(W.DecoderLayer(
            input_layernorm=W.RMSNorm(weight=torch.ones(D)),
            self_attn=W.Attention(q=lin(D, D, True), k=lin(kvd, D, True), v=lin(kvd, D, True),
                                  o=lin(D, D, False)),
            post_attention_layernorm=W.RMSNorm(weight=torch.ones(D)),
            mlp=W.MLP(gate=lin(cfg.intermediate_size, D, False), up=lin(cfg.intermediate_size, D, False),
                      down=lin(D, cfg.intermediate_size, False)),
        ))
    w = W.Weights(embed_tokens=embed, layers=tuple(layers), norm=W.RMSNorm(weight=torch.ones(D)),
                  lm_head=embed)
    ids = torch.randint(0, cfg.vocab_size, (1, 128), generator=torch.Generator().manual_seed(0))

    import augur.attention as attn_mod

    recorded = []
    orig = attn_mod.write_kv

    def recording(cache, layer_idx, position_ids, key, value):
        recorded.append((layer_idx, position_ids.clone(), key.clone(), value.clone()))
        return orig(cache, layer_idx, position_ids, key, value)

    attn_mod.write_kv = recording
    try:
        cache = ref.kv_cache.new_kv_cache(cfg, batch_size=1, max_seq_len=512,
                                          device=torch.device("cpu"), dtype=torch.float32)
        poison(cache.keys)
        poison(cache.values)
        with torch.no_grad():
            logits = ref.model.model(ids, w, cfg, cache=cache, position_ids=torch.arange(128).unsqueeze(0))
            for step in range(32):
                nxt = logits[:, -1, :].argmax(dim=-1, keepdim=True)
                logits = ref.model.model(nxt, w, cfg, cache=cache,
                                         position_ids=torch.tensor([[128 + step]]))
    finally:
        attn_mod.write_kv = orig
    L = cfg.num_hidden_layers
    assert len(recorded) == L * 33
    # K/V of every written token, per layer in write order: [L, 160, H, D]
    keys = torch.zeros(L, 160, cfg.num_key_value_heads, cfg.head_dim)
    values = torch.zeros_like(keys)
    positions = torch.zeros(L, 160, dtype=torch.int64)
    fill = [0] * L
    for layer, pos, k, v in recorded:
        n = pos.shape[1]
        keys[layer, fill[layer] : fill[layer] + n] = k[0].permute(1, 0, 2)
        values[layer, fill[layer] : fill[layer] + n] = v[0].permute(1, 0, 2)
        positions[layer, fill[layer] : fill[layer] + n] = pos[0]
        fill[layer] += n
    return {"keys": keys, "values": values, "positions": positions, "seq_len": cache.seq_len,
            "max_seq_len": 512, "call_sizes": [128] + [1] * 32,
            "sha256_keys": sha(cache.keys), "sha256_values": sha(cache.values)}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("AUGUR_REFERENCE"),
                    help="root of a semioz/augur checkout (its src/ holds the augur package); "
                         "defaults to $AUGUR_REFERENCE")
    ap.add_argument("--skip-config1", action="store_true")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference <augur checkout> or set AUGUR_REFERENCE")
    sys.path.insert(0, os.path.join(args.reference, "src"))
    import augur.attention  # noqa: F401
    import augur.config
    import augur.kv_cache
    import augur.model
    import augur.paged_kv_cache
    import augur.prefix_cache
    import augur.weights

    class Ref:
        config = augur.config
        kv_cache = augur.kv_cache
        paged_kv_cache = augur.paged_kv_cache
        prefix_cache = augur.prefix_cache
        model = augur.model
        weights = augur.weights

    g = torch.Generator().manual_seed(1234)
    cases = {
        "write_kv": write_kv_cases(Ref, g),
        "paged": paged_cases(Ref, g),
        "prefix": prefix_cases(Ref, g),
        "handoff": handoff_case(Ref, g),
        "fork": fork_case(Ref, g),
        "bookkeeping": bookkeeping_scripts(Ref),
    }
    cases["attention"] = attention_cases(Ref, torch.Generator().manual_seed(4321))
    cases["rope"] = rope_cases(Ref, torch.Generator().manual_seed(777))
    cases["duplicates"] = duplicate_cases(Ref, torch.Generator().manual_seed(99))
    cases["prefill_attention"] = prefill_attention_cases(Ref, torch.Generator().manual_seed(2024))
    torch.save(cases, os.path.join(HERE, "reference_cases.pt"))
    if not args.skip_config1:
        torch.save(config1(Ref), os.path.join(HERE, "config1_writes.pt"))
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    main()
