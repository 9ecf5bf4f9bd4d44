"""`B200Backend`: the reference's `AttentionBackend` (attention/base.py:16-45) on sm_100a kernels.

`forward` per layer (the engine calls it 32 times per step for Llama-3.1-8B):
1. the step's split plan, built on the first layer that sees a new `meta` and reused by the rest, as the
   FlashInfer backend caches its plan() (flashinfer_backend.py:44-45);
2. K1 `kv_append`: this step's k/v rows into the pools through `meta.slot_mapping` (replaces write_kv,
   paged_torch_ref.py:23-28, which all three reference backends share) -- or, when every written block is
   private to its sequence (`meta.append_private`) and the plan allows it, no separate launch: the
   attention launch stores the rows and uses them for the pages that hold them;
3. K2a paged attention over `meta.block_tables_i32` + K2b split-K reduction (replaces paged_attention,
   paged_torch_ref.py:40-74, and FlashInfer's run(), flashinfer_backend.py:46).
No host synchronisation happens inside `forward` with this package's `AttentionMetadata`; every launch goes
on torch's current stream.  With the reference's own metadata object (only the reference's fields), the
first layer of a step copies its block tables and slot_mapping back to the host once (`host_view`), so the
plan still gets shared-prefix units and query tiles and the append can still ride in the attention launch.

`prefill` (the contiguous, non-paged path of generate.py and the correctness tests) is not part of the
paged hot path; like the reference's CUDA backends (flashinfer_backend.py:39-40) it is plain SDPA.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from .. import _lib
from ..ops import (AttentionPlan, Workspace, attention_partials, can_fuse_append, kv_append, paged_attention,
                   plan_attention, splitk_reduce_exchange, splitk_reduce_gather)
from .base import AttentionBackend
from .metadata import host_view


class DeviceFault(RuntimeError):
    """A kernel met an out-of-range slot / block id (skipped) or gave up a bounded wait."""


class B200Backend(AttentionBackend):
    name = "b200"

    def __init__(self, pages_per_unit: int = 0, num_sms: int | None = None, check_errors: bool = False,
                 fuse_append: bool = True, derive_host_tables: bool = True) -> None:
        """pages_per_unit: split-K size in pages (0 = chosen per step from the work and the SM count).
        check_errors: after every forward, synchronise and raise `DeviceFault` if a kernel flagged a range
        fault (debugging aid; it costs a host sync per layer).
        fuse_append: let the attention launch do the append when that is exact (one launch fewer per layer);
        False always launches kv_append first.  Same results either way.
        derive_host_tables: for a metadata object without this package's host fields (the reference's
        AttentionMetadata), copy its tables and slots back once per step to plan shared prefixes / query
        tiles and the fused append; False plans every row on 8-column units and launches kv_append first.
        Same results either way."""
        _lib.lib()  # the CUDA library is required: fail here, not on the first step
        self.pages_per_unit = pages_per_unit
        self.num_sms = num_sms
        self.check_errors = check_errors
        self.fuse_append = fuse_append
        self.derive_host_tables = derive_host_tables
        self.last_append_fused = False  # whether the latest forward let the attention launch do the append
        self._host_for = None  # the foreign metadata object _host is derived from
        self._host: tuple[np.ndarray | None, bool] = (None, False)
        self._planned = None  # the AttentionMetadata the plan was built for
        self._plan_key: tuple | None = None
        self._plan: AttentionPlan | None = None
        self._workspace = Workspace()
        self._err: torch.Tensor | None = None

    # ------------------------------------------------------------------ contiguous path
    def prefill(self, q, k, v, key_valid=None, **kwargs):
        tq, tk = q.shape[2], k.shape[2]
        if key_valid is None and tq in (1, tk):  # decode step sees every key; a fresh prompt is plain causal
            return F.scaled_dot_product_attention(q, k, v, is_causal=tq > 1, enable_gqa=True)
        # query i (position tk - tq + i) sees keys 0 .. tk - tq + i
        mask = torch.ones(tq, tk, dtype=torch.bool, device=q.device).tril(diagonal=tk - tq)
        if key_valid is not None:
            mask = mask & key_valid[:, None, None, :]
            # a query with no real key may see its own position (softmax over nothing would be NaN)
            own = torch.zeros(tq, tk, dtype=torch.bool, device=q.device)
            own[torch.arange(tq), torch.arange(tq) + tk - tq] = True
            mask = mask | (own & ~mask.any(dim=-1, keepdim=True))
        return F.scaled_dot_product_attention(q, k, v, attn_mask=mask, enable_gqa=True)

    # ------------------------------------------------------------------ paged path
    def host_fields(self, meta) -> tuple[np.ndarray | None, bool]:
        """(host int32 block tables, append_private) of the step: this package's AttentionMetadata carries
        them; for another object with the reference's fields they are derived once per metadata object
        (`host_view`, one device-to-host copy) unless derive_host_tables is off."""
        if hasattr(meta, "block_tables_host"):
            return meta.block_tables_host, bool(getattr(meta, "append_private", False))
        if not self.derive_host_tables:
            return None, False
        if self._host_for is not meta:
            self._host = host_view(meta)
            self._host_for = meta
        return self._host

    def plan(self, meta, num_heads: int, num_kv_heads: int, device: torch.device,
             dtype: torch.dtype = torch.bfloat16) -> AttentionPlan:
        """The step's plan, built on the first call with a new `meta` and reused after.  Shared-prefix units
        and query tiles are planned from the host block tables (`host_fields`) when the pools are 16-bit."""
        key = (num_heads, num_kv_heads, device, dtype)
        if self._planned is not meta or self._plan_key != key:
            tables = self.host_fields(meta)[0] if dtype != torch.float32 else None
            self._plan = plan_attention(meta.query_start_loc, meta.seq_lens, meta.block_tables_i32.shape[1],
                                        num_heads, num_kv_heads, device, meta.block_size, self.num_sms,
                                        self.pages_per_unit, block_tables_host=tables)
            self._planned, self._plan_key = meta, key
        return self._plan

    def forward(self, q, k, v, k_cache, v_cache, meta, out_targets=None, peer_gather=None):
        """out_targets (optional, `ops.out_targets`): store the output rows there and return None.
        peer_gather (optional, `(PeerOutputs, slot, head_offset)`, used by KV-head sharding): put every row
        in every rank's gathered buffer of that slot (the reduction carries the all-gather: as flagged
        packets, or plain stores followed by the peers' barrier, as the PeerOutputs was built)."""
        if k_cache.shape[1] != meta.block_size:
            raise ValueError(f"pool block size {k_cache.shape[1]} != metadata block size {meta.block_size}")
        err = self._error_word(q.device) if self.check_errors else None
        plan = self.plan(meta, q.shape[1], k_cache.shape[2], q.device, k_cache.dtype)
        append = None
        if self.fuse_append and can_fuse_append(plan, k_cache, k, v) and self.host_fields(meta)[1]:
            append = (k, v, meta.slot_mapping)
        else:
            kv_append(k_cache, v_cache, meta.slot_mapping, k, v, err)
        self.last_append_fused = append is not None
        if peer_gather is not None:
            peers, slot, head_offset = peer_gather
            attention_partials(q, k_cache, v_cache, meta.block_tables_i32, meta.seq_lens_i32, meta.qo_indptr, plan,
                               self._workspace, err=err, targets=peers.local_targets(slot, head_offset),
                               append=append)
            if peers.use_packets(q.shape[0]):
                splitk_reduce_exchange(plan, self._workspace, peers, slot, q.dtype, q.shape[2], q.device)
            else:
                splitk_reduce_gather(plan, self._workspace, peers.targets(slot, head_offset), peers.self_dest,
                                     q.dtype, q.shape[2], q.device)
                peers.barrier()
            out = None
        else:
            out = paged_attention(q, k_cache, v_cache, meta.block_tables_i32, meta.seq_lens_i32, meta.qo_indptr,
                                  plan, self._workspace, err=err, targets=out_targets, append=append)
        if self.check_errors:
            self.raise_device_errors()
        return out

    # ------------------------------------------------------------------ device error word
    def _error_word(self, device: torch.device) -> torch.Tensor:
        if self._err is None or self._err.device != device:
            self._err = torch.zeros(1, dtype=torch.int32, device=device)
        return self._err

    def raise_device_errors(self) -> None:
        if self._err is None:
            return
        bits = int(self._err.item())
        if bits:
            self._err.zero_()
            names = [n for b, n in ((_lib.DEV_SLOT_RANGE, "slot out of range"),
                                    (_lib.DEV_BLOCK_RANGE, "block id out of range"),
                                    (_lib.DEV_WAIT_TIMEOUT, "page copy wait timed out"),
                                    (_lib.DEV_COPY_RANGE, "block-copy pair out of range")) if bits & b]
            raise DeviceFault("device fault flags: " + ", ".join(names))
