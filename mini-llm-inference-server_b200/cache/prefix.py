"""Prefix-cache index: which full blocks hold KV for which token prefix (the reference's cache/prefix.py,
decision docs/decisions/08-block-hash-spec.md).  Host-side; it names the shared blocks that the paged
kernels read and that copy-on-write protects.

Hash spec (byte-for-byte the reference's, so a router computes the same names):
    root    = SHA-256("minillm-kv-v1" || 0x00 || canonical JSON of the extra keys)
    hash[i] = SHA-256(hash[i-1] || the block's tokens as uint32 little-endian)
"""

from __future__ import annotations

import hashlib
import json

import numpy as np

HASH_VERSION = b"minillm-kv-v1"


def root_hash(extra_keys: dict) -> bytes:
    canonical = json.dumps(extra_keys, sort_keys=True, separators=(",", ":"), ensure_ascii=False).encode("utf-8")
    return hashlib.sha256(HASH_VERSION + b"\x00" + canonical).digest()


def block_hash(parent: bytes, tokens: list[int]) -> bytes:
    return hashlib.sha256(parent + np.asarray(tokens, dtype="<u4").tobytes()).digest()


def extend_chain(chain: list[bytes], root: bytes, tokens: list[int], num_blocks: int, block_size: int) -> None:
    """Grow `chain` (hashes of a sequence's first full blocks) to `num_blocks` entries."""
    for i in range(len(chain), num_blocks):
        chain.append(block_hash(chain[-1] if chain else root, tokens[i * block_size:(i + 1) * block_size]))


class PrefixCache:
    """hash -> block id and back.  The first block to hold a prefix stays its cached copy."""

    def __init__(self) -> None:
        self._block_of: dict[bytes, int] = {}
        self._hash_of: dict[int, bytes] = {}
        self.queries = 0  # prompt tokens looked up
        self.hits = 0  # of those, tokens served from cached blocks

    def __len__(self) -> int:
        return len(self._block_of)

    def lookup(self, hashes: list[bytes]) -> list[int]:
        """Blocks of the longest cached prefix of `hashes`."""
        out = []
        for h in hashes:
            b = self._block_of.get(h)
            if b is None:
                break
            out.append(b)
        return out

    def insert(self, h: bytes, block: int) -> None:
        if h in self._block_of or block in self._hash_of:
            return
        self._block_of[h] = block
        self._hash_of[block] = h

    def is_cached(self, block: int) -> bool:
        return block in self._hash_of

    def forget(self, block: int) -> None:
        h = self._hash_of.pop(block, None)
        if h is not None:
            del self._block_of[h]

    def move(self, src: int, dst: int) -> None:
        """The block's contents moved from `src` to `dst` (compaction): its name follows it."""
        h = self._hash_of.pop(src, None)
        if h is not None:
            self._block_of[h] = dst
            self._hash_of[dst] = h

    def clear(self) -> None:
        self._block_of.clear()
        self._hash_of.clear()
