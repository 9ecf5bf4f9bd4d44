"""Seeded input builders shared by the golden generator (`make_golden.py`) and the tests.

Inputs are drawn with numpy's PCG64 generator (`np.random.default_rng(seed)`), whose streams are stable
across machines and numpy releases, so the fixtures only store each case's outputs plus a SHA-256 of its
inputs: a test rebuilds the inputs, checks the digest, and compares.  Shapes follow BASELINE.json's
configs (config 1 exactly; the Llama-3.1-8B head shape at reduced batch for the others) and the reference's
own kernel tests (`tests/test_kernels.py:29-72`, `tests/test_paged.py:63-93`).
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass, field

import numpy as np
import torch

BS = 16


@dataclass
class PagedCase:
    """One ragged step on one layer's pools (fp32 values; tests cast to bf16/fp16 where they need to)."""

    name: str
    h: int
    hkv: int
    dh: int
    bs: int
    steps: list[tuple[int, int]]  # (num_cached, num_new) per sequence
    blocks: list[list[int]]  # each sequence's block ids, covering cached + new tokens
    q: torch.Tensor  # [N, H, Dh]
    k: torch.Tensor  # [N, Hkv, Dh] this step's new rows
    v: torch.Tensor
    k_pool: torch.Tensor  # [num_blocks, bs, Hkv, Dh] before the step's write
    v_pool: torch.Tensor
    extra: dict = field(default_factory=dict)

    @property
    def seqs(self) -> list[tuple[int, int, list[int]]]:
        return [(c, n, b) for (c, n), b in zip(self.steps, self.blocks)]

    def digest(self) -> str:
        h = hashlib.sha256()
        for t in (self.q, self.k, self.v, self.k_pool, self.v_pool):
            h.update(t.numpy().tobytes())
        h.update(repr((self.steps, self.blocks)).encode())
        return h.hexdigest()


def _normal(r: np.random.Generator, shape, scale: float = 1.0) -> torch.Tensor:
    x = r.standard_normal(shape, dtype=np.float32)
    if scale != 1.0:
        x = x * np.float32(scale)
    return torch.from_numpy(x)


def _take_blocks(perm: list[int], steps) -> list[list[int]]:
    out = []
    for cached, new in steps:
        need = -(-(cached + new) // BS)
        out.append([perm.pop() for _ in range(need)])
    return out


def make_case(name, seed, h, hkv, dh, steps, num_blocks, kv_scale=1.0, pool_fill="normal") -> PagedCase:
    r = np.random.default_rng(seed)
    perm = [int(b) for b in r.permutation(num_blocks)]
    blocks = _take_blocks(perm, steps)
    n = sum(new for _, new in steps)
    shape = (num_blocks, BS, hkv, dh)
    if pool_fill == "normal":  # junk everywhere a sequence doesn't own (tests/test_kernels.py:34)
        k_pool, v_pool = _normal(r, shape, kv_scale), _normal(r, shape, kv_scale)
    else:  # poisoned: any stray read changes the output (tests/test_paged.py:99-107)
        k_pool = torch.full(shape, float(pool_fill))
        v_pool = torch.full(shape, float(pool_fill))
        for (cached, _), b in zip(steps, blocks):
            for p in range(cached):
                k_pool[b[p // BS], p % BS] = _normal(r, (hkv, dh), kv_scale)
                v_pool[b[p // BS], p % BS] = _normal(r, (hkv, dh), kv_scale)
    q = _normal(r, (n, h, dh))
    k = _normal(r, (n, hkv, dh), kv_scale)
    v = _normal(r, (n, hkv, dh), kv_scale)
    return PagedCase(name, h, hkv, dh, BS, list(steps), blocks, q, k, v, k_pool, v_pool)


def tiny_config1(seed: int = 1) -> PagedCase:
    """fp32, H 8, Hkv 2, Dh 64, bs 16, pool 128 blocks, batch 4, context ~ U[1, 256]
    (context after the append), tables a seeded permutation, Q/K/V ~ N(0, 1); 1 new token per sequence."""
    r = np.random.default_rng(seed)
    ctx = [int(c) for c in r.integers(1, 257, size=4)]
    return make_case("cfg1_tiny", seed + 1000, 8, 2, 64, [(c - 1, 1) for c in ctx], 128)


def llama_decode(seed: int, batch: int, lo: int, hi: int, kv_scale: float = 0.5) -> PagedCase:
    """BASELINE config 2's distribution at a small batch: H 32, Hkv 8, Dh 128, context ~ U[lo, hi],
    pool = 1.25x the blocks needed, K/V ~ 0.5 N(0, 1), Q ~ N(0, 1)."""
    r = np.random.default_rng(seed)
    ctx = [int(c) for c in r.integers(lo, hi + 1, size=batch)]
    need = sum(-(-c // BS) for c in ctx)
    return make_case(f"llama_decode_b{batch}", seed + 1000, 32, 8, 128, [(c - 1, 1) for c in ctx],
                     int(need * 1.25) + 1, kv_scale=kv_scale)


MIXED_STEPS = [(0, 37), (90, 1), (40, 25), (0, 1), (300, 1)]  # tests/test_kernels.py:33


def mixed_step(seed: int = 3, h: int = 8, hkv: int = 2, dh: int = 128) -> PagedCase:
    """Every row kind in one ragged step: fresh prompt, decode, prompt on top of cache, 1-token prompt,
    decode at 300 (tests/test_kernels.py:29-48)."""
    return make_case(f"mixed_h{h}_kv{hkv}_d{dh}", seed, h, hkv, dh, MIXED_STEPS, 64)


def boundaries(seed: int = 5, h: int = 8, hkv: int = 2, dh: int = 64) -> PagedCase:
    """Decode rows whose contexts sit on and around page boundaries (1, 15, 16, 17, 32, 33, 255, 256, 257)."""
    ctx = [1, 15, 16, 17, 32, 33, 255, 256, 257]
    return make_case(f"bounds_h{h}_kv{hkv}_d{dh}", seed, h, hkv, dh, [(c - 1, 1) for c in ctx], 160)


def poisoned(seed: int = 7) -> PagedCase:
    """Unused slots hold 1e4, so any read outside a sequence's own tokens shows in the output."""
    steps = [(16, 1), (0, 5), (33, 1), (7, 9), (0, 1)]
    return make_case("poisoned", seed, 8, 2, 64, steps, 48, pool_fill=1e4)


def gqa_variants() -> list[PagedCase]:
    """MHA, GQA and MQA groupings (tests/test_attention.py:21-22) with ragged decode and multi-token rows."""
    steps = [(20, 1), (0, 3), (50, 1), (17, 6), (64, 1)]
    return [make_case(f"gqa_h{h}_kv{hkv}_d{dh}", 11 + i, h, hkv, dh, steps, 48)
            for i, (h, hkv, dh) in enumerate([(4, 4, 64), (4, 2, 64), (8, 1, 128), (16, 2, 128), (8, 8, 128)])]


def attention_cases() -> list[PagedCase]:
    """The cases whose reference outputs are stored in attention.npz (kept small: outputs only)."""
    return [tiny_config1(), llama_decode(21, 4, 512, 4096), mixed_step(), boundaries(),
            boundaries(6, 32, 8, 128), poisoned(), *gqa_variants()]


# ---------- append: casts into a 16-bit pool ----------


def cast_rows(seed: int = 31, n: int = 24, hkv: int = 2, dh: int = 64) -> torch.Tensor:
    """fp32 rows [n, hkv, dh] that exercise round-to-nearest-even: exact ties, values one ulp either side
    of a tie, signed zeros, subnormals, the largest finite values, infinities and NaN."""
    r = np.random.default_rng(seed)
    x = r.standard_normal((n, hkv, dh), dtype=np.float32)
    bits = x.view(np.uint32).reshape(-1)
    m = bits.size
    # bf16 ties: low 16 bits exactly 0x8000 (even and odd upper halves), and 0x7fff / 0x8001 around them
    bits[0:m:7] = (bits[0:m:7] & 0xFFFF0000) | 0x8000
    bits[1:m:11] = (bits[1:m:11] & 0xFFFF0000) | 0x7FFF
    bits[2:m:13] = (bits[2:m:13] & 0xFFFF0000) | 0x8001
    bits[3:m:17] = (bits[3:m:17] & 0xFFFE0000) | 0x18000  # odd upper half, tie: rounds up
    # fp16 ties: 13 dropped mantissa bits exactly half
    bits[4:m:19] = (bits[4:m:19] & 0xFFFFE000) | 0x1000
    special = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 3.3895314e38, -3.3895314e38, 1e-40, -1e-40,
                        65504.0, 65520.0, 65519.996, 6.1e-5, 5.96e-8, 2.98e-8, 1e-45], dtype=np.float32)
    x = bits.view(np.float32).reshape(n, hkv, dh).copy()
    x.reshape(-1)[5:5 + special.size] = special
    return torch.from_numpy(x)
