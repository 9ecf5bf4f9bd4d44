"""Paged KV pool with the reference's interface (cache/paged.py:21-69: `PagedKVCache(config, num_blocks,
device, dtype, block_size)`, per-layer `.k` / `.v` lists of [num_blocks, block_size, Hkv, Dh] tensors in NHD
layout, `bytes_per_block`, `blocks_for_bytes`, `step(meta)`).  Token p of a request lives at
block_ids[p // block_size], offset p % block_size, in every layer.

Storage: ONE device allocation `[2, layers, num_blocks, block_size, Hkv, Dh]` (K pools, then V pools),
zero-filled, of which `.k[l]` / `.v[l]` are contiguous views.  A single range keeps the pool out of the
caching allocator's per-tensor blocks (the engine sizes it to nearly all free memory at start-up), and the
block-copy kernel's address table is the 2 x layers view bases, made once.

Added for copy-on-write and compaction: `copy_blocks(src, dst)` copies whole blocks in every layer's K and
V with ONE launch of the block-copy kernel.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import ops

BLOCK_SIZE = 16


@dataclass
class KVShape:
    """The three numbers of a model config the pool needs (LlamaConfig's field names, so either fits)."""

    num_hidden_layers: int
    num_key_value_heads: int
    head_dim: int


class PagedKVCache:
    def __init__(self, config, num_blocks: int, device: torch.device | str, dtype: torch.dtype,
                 block_size: int = BLOCK_SIZE) -> None:
        layers = config.num_hidden_layers
        block = (block_size, config.num_key_value_heads, config.head_dim)
        self.storage = torch.zeros((2, layers, num_blocks, *block), device=device, dtype=dtype)
        self.k = list(self.storage[0].unbind(0))
        self.v = list(self.storage[1].unbind(0))
        self.num_blocks = num_blocks
        self.block_size = block_size
        self._ptrs: torch.Tensor | None = None

    @staticmethod
    def bytes_per_block(config, dtype: torch.dtype, block_size: int = BLOCK_SIZE) -> int:
        """Device bytes one block id stands for: its K and V rows in every layer."""
        row = config.num_key_value_heads * config.head_dim * dtype.itemsize
        return 2 * config.num_hidden_layers * block_size * row

    @classmethod
    def blocks_for_bytes(cls, config, dtype: torch.dtype, num_bytes: int, block_size: int = BLOCK_SIZE) -> int:
        """How many blocks a budget of `num_bytes` pays for (whole blocks only)."""
        return num_bytes // cls.bytes_per_block(config, dtype, block_size)

    def step(self, meta) -> PagedStep:
        return PagedStep(self, meta)

    def copy_blocks(self, src, dst, err: torch.Tensor | None = None) -> None:
        """pool[dst[i]] = pool[src[i]] in every layer's K and V (bit-exact).  src/dst: lists or int32 tensors;
        the destination set must be disjoint from the source set (as `BlockManager.cow/compact` plan it)."""
        dev = self.storage.device
        s = torch.as_tensor(src, dtype=torch.int32).to(dev, non_blocking=True)
        d = torch.as_tensor(dst, dtype=torch.int32).to(dev, non_blocking=True)
        if self._ptrs is None:
            self._ptrs = ops.pool_pointer_table(self.k + self.v)
        ops.block_copy(self._ptrs, self.k[0], s, d, err)


class PagedStep:
    """What the reference's model asks of a KV cache during one ragged step (cache/paged.py:48-69).  The
    backend's `forward` writes and reads the pool itself and the engine counts each request's cached tokens,
    so a step only supplies positions and refuses padding."""

    ragged = True

    def __init__(self, cache: PagedKVCache, meta) -> None:
        self.cache, self.meta = cache, meta

    def positions(self, input_ids: torch.Tensor, attention_mask: torch.Tensor | None = None) -> torch.Tensor:
        return self.meta.positions.unsqueeze(0)  # the step's tokens form one row [1, N]

    def mark(self, attention_mask: torch.Tensor | None, num_tokens: int) -> None:
        if attention_mask is not None:
            raise ValueError("paged steps are ragged (no padding): attention_mask must be None")

    def key_valid(self, num_new: int) -> None:
        return None

    def advance(self, num_tokens: int) -> None:
        return None
