"""Paged KV pool: per layer, K and V tensors [num_blocks, block_size, Hkv, Dh] (NHD, token-major inside a
block), allocated once by torch (the reference's cache/paged.py:21-69, same constructor and layout).
Token p of a request lives at block_ids[p // block_size], offset p % block_size, in every layer.

Added for copy-on-write and compaction: `copy_blocks(src, dst)` copies whole blocks in every layer's K
and V with ONE launch of the block-copy kernel (a device table of the 2 x layers pool addresses is built
once, here).
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
        shape = (num_blocks, block_size, config.num_key_value_heads, config.head_dim)
        self.k = [torch.zeros(shape, device=device, dtype=dtype) for _ in range(config.num_hidden_layers)]
        self.v = [torch.zeros(shape, device=device, dtype=dtype) for _ in range(config.num_hidden_layers)]
        self.num_blocks = num_blocks
        self.block_size = block_size
        self._ptrs: torch.Tensor | None = None

    @staticmethod
    def bytes_per_block(config, dtype: torch.dtype, block_size: int = BLOCK_SIZE) -> int:
        """K and V, every layer: 2 x layers x block_size x KV heads x head_dim x bytes per element."""
        elem = torch.tensor([], dtype=dtype).element_size()
        return 2 * config.num_hidden_layers * block_size * config.num_key_value_heads * config.head_dim * elem

    @classmethod
    def blocks_for_bytes(cls, config, dtype: torch.dtype, num_bytes: int, block_size: int = BLOCK_SIZE) -> int:
        return num_bytes // cls.bytes_per_block(config, dtype, block_size)

    def step(self, meta) -> PagedStep:
        return PagedStep(self, meta)

    def copy_blocks(self, src, dst, err: torch.Tensor | None = None) -> None:
        """pool[dst[i]] = pool[src[i]] in every layer's K and V (bit-exact).  src/dst: lists or int32 tensors;
        the destination set must be disjoint from the source set (as `BlockManager.cow/compact` plan it)."""
        dev = self.k[0].device
        s = torch.as_tensor(src, dtype=torch.int32).to(dev, non_blocking=True)
        d = torch.as_tensor(dst, dtype=torch.int32).to(dev, non_blocking=True)
        if self._ptrs is None:
            self._ptrs = ops.pool_pointer_table(self.k + self.v)
        ops.block_copy(self._ptrs, self.k[0], s, d, err)


class PagedStep:
    """The cache as one forward pass sees it (cache/paged.py:48-69): attention reads and writes the pool
    through the backend's `forward`, so there is nothing to mark or advance."""

    ragged = True

    def __init__(self, cache: PagedKVCache, meta) -> None:
        self.cache, self.meta = cache, meta

    def positions(self, input_ids: torch.Tensor, attention_mask: torch.Tensor | None = None) -> torch.Tensor:
        return self.meta.positions[None, :]

    def mark(self, attention_mask: torch.Tensor | None, num_tokens: int) -> None:
        if attention_mask is not None:
            raise ValueError("a ragged step has no padding, so no attention mask")

    def key_valid(self, num_new: int) -> None:
        return None

    def advance(self, num_tokens: int) -> None:
        pass
