"""CPU restatement of the reference's prefix-cache hash chain.  TEST INFRASTRUCTURE ONLY.

Restates `src/minillm/cache/prefix.py:21-35` (decision `docs/decisions/08-block-hash-spec.md`):
    root    = SHA-256("minillm-kv-v1" || 0x00 || canonical JSON of the extra keys)
    hash[i] = SHA-256(hash[i-1] || the block's 16 token ids as uint32 little-endian)
Canonical JSON: keys sorted, separators "," and ":", UTF-8 kept as is.
"""

from __future__ import annotations

import hashlib
import json
import struct


def root_hash(extra_keys: dict) -> bytes:
    text = json.dumps(extra_keys, sort_keys=True, separators=(",", ":"), ensure_ascii=False)
    return hashlib.sha256(b"minillm-kv-v1" + b"\x00" + text.encode("utf-8")).digest()


def block_hash(parent: bytes, tokens: list[int]) -> bytes:
    return hashlib.sha256(parent + b"".join(struct.pack("<I", t) for t in tokens)).digest()


def extend_chain(chain: list[bytes], root: bytes, tokens: list[int], num_blocks: int, block_size: int) -> None:
    while len(chain) < num_blocks:
        i = len(chain)
        chain.append(block_hash(chain[-1] if chain else root, tokens[i * block_size:(i + 1) * block_size]))
