"""Attention backends on paged KV.

- `b200`: this package's sm_100a kernels (`B200Backend`): append, paged attention with split-K, and the
  per-step plan cached on the metadata object.
- any other name is looked up in the reference's registry (src/minillm/attention/__init__.py:15-28) when
  the reference is installed, so `get_backend` is a superset of the reference's.
- `metadata.py`: the per-step description of a ragged batch (AttentionMetadata, SeqStep), built once
  per step as device tensors.
"""

from __future__ import annotations

from .backend import B200Backend, DeviceFault
from .base import AttentionBackend
from .metadata import AttentionMetadata, SeqStep


def get_backend(name: str, **kwargs) -> AttentionBackend:
    if name == "b200":
        return B200Backend(**kwargs)
    try:
        from minillm.attention import get_backend as reference_get_backend
    except ImportError:
        raise ValueError(f"unknown attention backend: {name!r} (this package provides 'b200'; the reference's "
                         "backends need the minillm package)") from None
    return reference_get_backend(name)


__all__ = ["AttentionBackend", "AttentionMetadata", "B200Backend", "DeviceFault", "SeqStep", "get_backend"]
