"""Block manager: hands out and takes back the paged pool's blocks (the reference's engine/block_manager.py
API: allocate / acquire / free / clear_cache / check), plus the two planners that feed the block-copy
kernel, which the reference does not have:

- `cow`: copy-on-write.  Before a sequence writes into a block that another block table also holds
  (refcount > 1, e.g. the partly filled last block of a shared prefix), the sequence gets a private
  copy: one new block, one (src, dst) pair for the device copy, and its table points at the copy.
- `compact`: move every live block (held, or cached for a later prefix hit) into the lowest ids so the
  used part of the pool is one dense range after evictions; tables, refcounts, the LRU order and the
  prefix-cache names follow the moved blocks.

Every block is in exactly one state: free, held (refcount >= 1) or cached (refcount 0, named in the prefix
cache, kept in LRU order).  `check` verifies that ("R3" in the reference).
"""

from __future__ import annotations

import math
from collections import Counter, OrderedDict, deque

from .prefix import PrefixCache


class BlockManager:
    def __init__(self, num_blocks: int, block_size: int, prefix: PrefixCache | None = None) -> None:
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.prefix = prefix
        self._free: deque[int] = deque(range(num_blocks))
        self._cached: OrderedDict[int, None] = OrderedDict()  # oldest first
        self._ref = [0] * num_blocks

    # ------------------------------------------------------------------ the reference's API
    @property
    def num_free(self) -> int:
        """Blocks that can be handed out: free ones plus cached ones that would be evicted."""
        return len(self._free) + len(self._cached)

    @property
    def num_cached(self) -> int:
        return len(self._cached)

    def blocks_for(self, num_tokens: int) -> int:
        return math.ceil(num_tokens / self.block_size)

    def is_cached_unheld(self, block: int) -> bool:
        return block in self._cached

    def refcount(self, block: int) -> int:
        return self._ref[block]

    def allocate(self, n: int) -> list[int]:
        if n > self.num_free:
            raise RuntimeError(f"asked for {n} blocks, {self.num_free} free")
        out = []
        for _ in range(n):
            if self._free:
                b = self._free.popleft()
            else:  # evict the least recently used cached block
                b, _ = self._cached.popitem(last=False)
                self.prefix.forget(b)
            self._ref[b] = 1
            out.append(b)
        return out

    def acquire(self, blocks: list[int]) -> None:
        """Take a reference on blocks (a prefix-cache hit, or a table sharing another's prefix)."""
        for b in blocks:
            if self._ref[b] == 0:
                del self._cached[b]
            self._ref[b] += 1

    def free(self, blocks: list[int]) -> None:
        """Drop one reference on each block, tail first; an unheld block becomes cached (if named) or free."""
        for b in reversed(blocks):
            self._ref[b] -= 1
            if self._ref[b] == 0:
                if self.prefix is not None and self.prefix.is_cached(b):
                    self._cached[b] = None
                else:
                    self._free.append(b)
        blocks.clear()

    def clear_cache(self) -> None:
        while self._cached:
            b, _ = self._cached.popitem(last=False)
            self.prefix.forget(b)
            self._free.append(b)

    def check(self, held: list[list[int]]) -> None:
        """Every block is free, cached or held exactly once, and held refcounts match the block tables."""
        owners = Counter(b for table in held for b in table)
        bad = [b for b in range(self.num_blocks) if self._ref[b] != owners.get(b, 0)]
        if bad:
            raise AssertionError(f"refcounts don't match block tables for blocks {bad[:10]}")
        states = list(owners) + list(self._free) + list(self._cached)
        if len(states) != self.num_blocks or len(set(states)) != self.num_blocks:
            raise AssertionError(f"block accounting broken: {len(owners)} held + {len(self._free)} free + "
                                 f"{len(self._cached)} cached != {self.num_blocks} total, or a block is listed twice")

    # ------------------------------------------------------------------ copy-on-write
    def cow(self, block_ids: list[int], index: int) -> tuple[int, int] | None:
        """Make block_ids[index] private before it is written.  Returns (src, dst) to copy, or None when the
        table already owns the block alone."""
        b = block_ids[index]
        if self._ref[b] <= 1:
            return None
        (dst,) = self.allocate(1)
        self._ref[b] -= 1  # still held by the other tables
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
        live = sorted({b for t in tables for b in t} | set(self._cached))
        n_live = len(live)
        live_set = set(live)
        dst = [b for b in range(n_live) if b not in live_set]
        src = [b for b in live if b >= n_live]
        remap = dict(zip(src, dst))
        if not remap:
            return [], []
        for t in tables:
            t[:] = [remap.get(b, b) for b in t]
        for s, d in remap.items():
            self._ref[d], self._ref[s] = self._ref[s], 0
            if self.prefix is not None:
                self.prefix.move(s, d)
        self._cached = OrderedDict((remap.get(b, b), None) for b in self._cached)
        self._free = deque(range(n_live, self.num_blocks))
        return src, dst
