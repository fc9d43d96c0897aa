"""A batch of sequences in one paged pool: shared prefixes, forks and decode steps.

augur's generate keeps a paged cache for one sequence and no prefix cache
(augur/generation.py:35-40 refuses a batch above 1 and a prefix cache with
the paged backend). PagedSequences is the KV-side bookkeeping that a batched
paged generate needs, built on augur's own hash-chained index of full blocks
(PagedPrefixCache, augur/paged_kv_cache.py:45-85), its block tables and its
allocator, plus the batched kernels here:

- admit: a prompt takes the longest chain of cached full blocks as its own
  (shared, no data moves) and gets the pool slots of its remaining tokens,
  which the caller's prefill writes (write_paged_kv_batch);
- publish_prefix: a prefilled prompt's full blocks join the prefix cache,
  which holds each of them until evict_prefixes drops it;
- fork: new sequences share a parent's blocks (several samples of one
  prompt);
- decode_step: shared, partially filled last blocks are copied before they
  are appended to (one launch for the batch), then every table grows by one
  position (DecodeStep, or DecodeGraphStep.update for a captured step);
- release: a finished sequence's blocks go back to the pool once no other
  sequence and no prefix-cache entry holds them.

The model (projections, MLP, sampling) stays augur's. At least one prompt
token is always left to prefill, so the model produces the logits of the
prompt's last token even when every full block was cached.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass

import numpy as np

from .batched import cow_partial_blocks
from .decode import DecodeGraphStep, DecodeStep
from .paged_kv_cache import PagedKVCache, PagedPrefixCache, SequenceBlockTable, slots_for_positions


@dataclass
class Admission:
    """A prompt's place in the pool: its sequence id, how many of its tokens came from the
    prefix cache, and the int64 pool slots of the remaining ones (prompt positions
    cached_tokens, cached_tokens + 1, ...)."""

    seq_id: int
    cached_tokens: int
    slots: np.ndarray


class PagedSequences:
    """The sequences of one paged pool, with prefix sharing through a PagedPrefixCache."""

    def __init__(self, cache: PagedKVCache, prefix_cache: PagedPrefixCache | None = None) -> None:
        self.cache = cache
        self.prefix_cache = prefix_cache if prefix_cache is not None else PagedPrefixCache()
        self.tables: dict[int, SequenceBlockTable] = {}
        self.prompts: dict[int, list[int]] = {}
        self._published: list[tuple[int | None, tuple[int, ...], int]] = []  # (parent hash, tokens, block)
        self._next_id = 0
        self.last_cow_blocks = 0  # blocks the latest decode step copied before appending

    # -- admission and prefill ------------------------------------------------

    def admit(self, token_ids: Sequence[int]) -> Admission:
        """A new sequence for a prompt. Its leading full blocks that the prefix cache holds
        are shared; blocks for the rest are allocated (all or nothing: on an exhausted pool
        nothing is kept and augur's "no free KV cache blocks" error is raised)."""
        ids = [int(t) for t in token_ids]
        if not ids:
            raise ValueError("a prompt needs at least one token")
        bs, alloc = self.cache.block_size, self.cache.allocator
        match = self.prefix_cache.match_prefix(ids, bs)
        n_shared = min(len(match.block_ids), (len(ids) - 1) // bs)  # one token is always prefilled
        shared = match.block_ids[:n_shared]
        need = -(-len(ids) // bs) - n_shared
        fresh = alloc.allocate_many(need)  # raises before anything is held
        for b in shared:
            alloc.incref(b)
        table = SequenceBlockTable(block_ids=list(shared) + fresh, block_size=bs, seq_len=len(ids))
        sid = self._next_id
        self._next_id += 1
        self.tables[sid] = table
        self.prompts[sid] = ids
        positions = np.arange(n_shared * bs, len(ids), dtype=np.int64)
        return Admission(seq_id=sid, cached_tokens=n_shared * bs, slots=slots_for_positions(table, positions))

    def publish_prefix(self, seq_id: int) -> int:
        """Register the full blocks of a prefilled prompt in the prefix cache, which then
        holds each newly registered block. Returns how many blocks were registered (blocks
        whose tokens are already registered keep their existing entry)."""
        table, ids = self.tables[seq_id], self.prompts[seq_id]
        bs, alloc = self.cache.block_size, self.cache.allocator
        parent: int | None = None
        added = 0
        for j in range(len(ids) // bs):
            tokens = ids[j * bs : (j + 1) * bs]
            entry = self.prefix_cache.lookup(parent, tokens)
            if entry is None:
                block = table.block_ids[j]
                h = self.prefix_cache.add_block(parent, tokens, block)
                alloc.incref(block)
                self._published.append((parent, tuple(tokens), block))
                added += 1
            else:
                h = entry[0]
            parent = h
        return added

    # -- forks and decode -----------------------------------------------------

    def fork(self, seq_id: int, n: int) -> list[int]:
        """n new sequences sharing every block of seq_id (no data moves). A shared block is
        copied before any of them appends to it (decode_step)."""
        if n < 0:
            raise ValueError("n must be non-negative")
        parent = self.tables[seq_id]
        out = []
        for _ in range(n):
            sid = self._next_id
            self._next_id += 1
            self.tables[sid] = parent.fork(self.cache.allocator)
            self.prompts[sid] = list(self.prompts[seq_id])
            out.append(sid)
        return out

    def _prepare_append(self, seq_ids: Sequence[int]) -> list[SequenceBlockTable]:
        tables = [self.tables[s] for s in seq_ids]
        if len(set(map(id, tables))) != len(tables):
            raise ValueError("a sequence appears twice in one step")
        self.last_cow_blocks = cow_partial_blocks(self.cache, tables)  # one launch; none when nothing is shared
        return tables

    def decode_step(self, seq_ids: Sequence[int], early_reads: bool = False) -> DecodeStep:
        """The next decode step of these sequences: shared partial last blocks are copied,
        then each table grows by one position (see DecodeStep, and its early_reads: the
        copy-on-write launch here is followed by the step's uploads, so it has finished
        before the first layer's launch)."""
        return DecodeStep(self.cache, self._prepare_append(seq_ids), early_reads=early_reads)

    def update_graph_step(self, step: DecodeGraphStep, seq_ids: Sequence[int]) -> None:
        """decode_step for a captured step: copy shared partial blocks, then step.update."""
        step.update(self._prepare_append(seq_ids))

    # -- release ---------------------------------------------------------------

    def release(self, seq_id: int) -> None:
        """Drop a finished sequence; blocks nobody else holds return to the pool."""
        table = self.tables.pop(seq_id)
        self.prompts.pop(seq_id, None)
        table.free(self.cache.allocator)

    def evict_prefixes(self) -> int:
        """Unregister every prefix-cache block that only the cache still holds (latest
        first, so a chain's later blocks go before the ones they follow) and return them to
        the pool. Returns the number of blocks freed."""
        alloc = self.cache.allocator
        kept, freed = [], 0
        for parent, tokens, block in reversed(self._published):
            if alloc.refcount(block) == 1:
                self.prefix_cache.remove_block(parent, list(tokens))
                alloc.free(block)
                freed += 1
            else:
                kept.append((parent, tokens, block))
        self._published = kept[::-1]
        return freed
