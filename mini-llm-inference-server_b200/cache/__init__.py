"""Paged KV pool, prefix-cache index and block manager (host side of the paged path)."""

from .block_manager import BlockManager
from .paged import BLOCK_SIZE, KVShape, PagedKVCache, PagedStep
from .prefix import PrefixCache, block_hash, extend_chain, root_hash

__all__ = ["BLOCK_SIZE", "BlockManager", "KVShape", "PagedKVCache", "PagedStep", "PrefixCache", "block_hash",
           "extend_chain", "root_hash"]
