"""Block manager for the paged pool: the reference's API (engine/block_manager.py: allocate / acquire / free /
clear_cache / check and the num_free / num_cached / blocks_for / is_cached_unheld queries) over this
package's own bookkeeping, plus the planners that feed the block-copy kernel, which the reference lacks.

The invariant the reference calls R3 (engine/block_manager.py:1-10): every block is in exactly one of three
states, and a held block's refcount equals the number of block tables that list it.
- free: nothing worth keeping in it;
- held: refcount >= 1;
- cached: refcount 0 but named by the prefix cache, so a later request may reuse its KV; such blocks are
  handed out (their names dropped) only when no free block is left, least recently released first.

Bookkeeping here: refcounts in one numpy array (so `check` is a bincount, not a Python loop); free blocks
in a min-heap, so allocation always takes the lowest free id and the used part of the pool stays dense,
which keeps later compactions short; cached blocks in an insertion-ordered dict used as the LRU queue.

Planners:
- `cow` / `cow_for_append`: copy-on-write.  Before a table writes into a block that other tables also hold
  (refcount > 1, e.g. the partly filled last block of a shared prefix), it gets a private copy: one new
  block, one (src, dst) pair for the device copy, and its table points at the copy.
- `compact`: after evictions, move every live block (held, or cached for a later prefix hit) into the lowest
  ids so the used part of the pool is one dense range; tables, refcounts, the LRU order and the prefix
  cache's names follow the moved blocks.
"""

from __future__ import annotations

import heapq
import itertools

import numpy as np

from .prefix import PrefixCache


class BlockManager:
    def __init__(self, num_blocks: int, block_size: int, prefix: PrefixCache | None = None) -> None:
        if num_blocks <= 0 or block_size <= 0:
            raise ValueError(f"a pool needs a positive block count and block size, got {num_blocks}, {block_size}")
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.prefix = prefix
        self._refs = np.zeros(num_blocks, dtype=np.int64)
        self._free_heap: list[int] = list(range(num_blocks))  # ascending: already a valid heap
        self._lru: dict[int, None] = {}  # cached blocks, oldest release first

    # ------------------------------------------------------------------ queries
    @property
    def num_free(self) -> int:
        """Blocks that `allocate` can hand out: the free ones and the cached ones it would evict."""
        return len(self._free_heap) + len(self._lru)

    @property
    def num_cached(self) -> int:
        return len(self._lru)

    def blocks_for(self, num_tokens: int) -> int:
        return -(-num_tokens // self.block_size)

    def is_cached_unheld(self, block: int) -> bool:
        return block in self._lru

    def refcount(self, block: int) -> int:
        return int(self._refs[block])

    def cached_blocks(self) -> list[int]:
        """The cached (unheld, named) blocks, the next to be evicted first."""
        return list(self._lru)

    # ------------------------------------------------------------------ hand out and take back
    def _take(self) -> int:
        if self._free_heap:
            return heapq.heappop(self._free_heap)
        victim = next(iter(self._lru))  # nothing free: evict the least recently released cached block
        del self._lru[victim]
        self.prefix.forget(victim)
        return victim

    def allocate(self, n: int) -> list[int]:
        available = self.num_free
        if n > available:
            raise RuntimeError(f"cannot allocate {n} KV blocks: only {available} are free or evictable")
        got = [self._take() for _ in range(n)]
        self._refs[got] = 1
        return got

    def acquire(self, blocks: list[int]) -> None:
        """One more reference on each block: a prefix-cache hit, or a table that shares another's prefix."""
        for b in blocks:
            if self._refs[b] == 0:
                if b not in self._lru:
                    raise ValueError(f"block {b} is free: only held or cached blocks can be acquired")
                del self._lru[b]
            self._refs[b] += 1

    def _release(self, b: int) -> None:
        left = self._refs[b] - 1
        if left < 0:
            raise ValueError(f"block {b} released more often than it was held")
        self._refs[b] = left
        if left:
            return
        if self.prefix is not None and self.prefix.is_cached(b):
            self._lru[b] = None  # most recently released: evicted last
        else:
            heapq.heappush(self._free_heap, b)

    def free(self, blocks: list[int]) -> None:
        """Drop one reference on each block of a table and empty the list.  The table is released from its
        end, so its first blocks become the most recently released: a prefix lookup stops at the first miss,
        and evicting a table's first block would strand every block after it."""
        for b in reversed(blocks):
            self._release(b)
        blocks.clear()

    def clear_cache(self) -> None:
        """Drop every cached block's name and free it (an idle engine then has every block free)."""
        for b in self._lru:
            self.prefix.forget(b)
            heapq.heappush(self._free_heap, b)
        self._lru.clear()

    def check(self, held: list[list[int]]) -> None:
        """R3, with `held` = every live block table: refcounts equal how often the tables list each block,
        and every block is in exactly one of the states free / held / cached."""
        listed = np.fromiter(itertools.chain.from_iterable(held), dtype=np.int64)
        uses = np.bincount(listed, minlength=self.num_blocks) if listed.size else np.zeros(self.num_blocks, np.int64)
        wrong = np.nonzero(uses[:self.num_blocks] != self._refs)[0]
        if wrong.size or uses.size > self.num_blocks:
            raise AssertionError(f"R3: refcounts disagree with the block tables at blocks {wrong[:10].tolist()}")
        states = (self._refs > 0).astype(np.int64)
        for group in (self._free_heap, list(self._lru)):
            if group:
                np.add.at(states, np.asarray(group, dtype=np.int64), 1)
        if (states != 1).any():
            odd = np.nonzero(states != 1)[0]
            raise AssertionError(f"R3: blocks {odd[:10].tolist()} are in no state or in several (held "
                                 f"{int((self._refs > 0).sum())}, free {len(self._free_heap)}, cached "
                                 f"{len(self._lru)}, pool {self.num_blocks})")

    # ------------------------------------------------------------------ copy-on-write
    def cow(self, block_ids: list[int], index: int) -> tuple[int, int] | None:
        """Make block_ids[index] private before it is written.  Returns (src, dst) to copy, or None when the
        table already owns the block alone."""
        b = block_ids[index]
        if self._refs[b] <= 1:
            return None
        (dst,) = self.allocate(1)
        self._refs[b] -= 1  # still held by the other tables
        block_ids[index] = dst
        return b, dst

    def cow_for_append(self, block_ids: list[int], num_cached: int, num_new: int) -> list[tuple[int, int]]:
        """COW every block that positions [num_cached, num_cached + num_new) will write into."""
        if num_new <= 0:
            return []
        first, last = num_cached // self.block_size, (num_cached + num_new - 1) // self.block_size
        pairs = [self.cow(block_ids, i) for i in range(first, min(last, len(block_ids) - 1) + 1)]
        return [p for p in pairs if p is not None]

    # ------------------------------------------------------------------ compaction
    def compact(self, tables: list[list[int]]) -> tuple[list[int], list[int]]:
        """Pack live blocks (held by `tables`, or cached) into ids [0, n_live).  `tables` must list every held
        block table; they are rewritten in place.  Returns (src, dst) for the device block copy: live blocks
        at ids >= n_live, ascending, paired with the free ids below n_live, ascending."""
        self.check(tables)
        live = self._refs > 0
        if self._lru:
            live[np.fromiter(self._lru, dtype=np.int64)] = True
        n_live = int(live.sum())
        src = np.nonzero(live[n_live:])[0] + n_live
        dst = np.nonzero(~live[:n_live])[0]
        if src.size == 0:
            return [], []
        remap = np.arange(self.num_blocks)
        remap[src] = dst
        for t in tables:
            t[:] = remap[np.asarray(t, dtype=np.int64)].tolist()
        self._refs[dst] = self._refs[src]
        self._refs[src] = 0
        if self.prefix is not None:
            for s, d in zip(src.tolist(), dst.tolist()):
                self.prefix.move(s, d)
        self._lru = {int(remap[b]): None for b in self._lru}
        self._free_heap = list(range(n_live, self.num_blocks))
        return src.tolist(), dst.tolist()
