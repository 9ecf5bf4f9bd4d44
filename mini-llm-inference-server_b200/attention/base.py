"""The attention-backend interface of the reference (src/minillm/attention/base.py:16-45), restated so the
B200 backend is usable where the reference package is not installed.

When `minillm` (the reference) is importable, its own `AttentionBackend` is used as the base class, so
the B200 backend passes the reference engine's isinstance checks and can be assigned to
`layer.self_attn.backend` exactly like the backends S5 part C swaps in (benchmarks/s5_kv_pressure.py:201-219).
"""

from __future__ import annotations

from abc import ABC, abstractmethod

import torch

try:  # the reference's own interface, when the reference is installed beside this package
    from minillm.attention.base import AttentionBackend as _ReferenceBase
except ImportError:  # pragma: no cover - depends on the environment
    _ReferenceBase = None


class _Interface(ABC):
    name: str = "base"

    @abstractmethod
    def prefill(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                key_valid: torch.Tensor | None = None, **kwargs) -> torch.Tensor:
        """Causal attention of q [B, H, Tq, Dh] over contiguous k, v [B, Hkv, Tk, Dh] (Tk >= Tq): query i sits
        at position Tk - Tq + i.  `key_valid` [B, Tk] marks real keys.  Returns [B, H, Tq, Dh]."""

    @abstractmethod
    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor,
                v_cache: torch.Tensor, meta) -> torch.Tensor:
        """One layer of one engine step on paged KV: write k, v [N, Hkv, Dh] into the pools
        [num_blocks, block_size, Hkv, Dh] at meta.slot_mapping, then return each new token's causal attention
        over its sequence's pages, [N, H, Dh]."""


AttentionBackend = _ReferenceBase if _ReferenceBase is not None else _Interface

__all__ = ["AttentionBackend"]
