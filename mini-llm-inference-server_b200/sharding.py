"""KV-head sharding of the paged path across the GPUs of one node (one process per GPU).

Rank r of n owns KV heads [r * Hkv / n, (r + 1) * Hkv / n) and their query heads
[r * H / n, (r + 1) * H / n) (grouped-query attention keeps each KV head with its query group), so its
pools are [num_blocks, block_size, Hkv / n, Dh].  Block ids, block tables, slot_mapping and seq_lens are
the same on every rank: append, copy-on-write, compaction and attention are purely local.  The one
exchange is the attention output: each rank holds [N, H / n, Dh] and an all-gather over NCCL (NVLink /
NVSwitch) reassembles [N, H, Dh].  The reference has no parallelism (its roadmap names NCCL tensor
parallelism, docs/distributed_inference_plan.md:325).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .attention.base import AttentionBackend


def head_range(rank: int, world: int, num_heads: int) -> slice:
    if num_heads % world:
        raise ValueError(f"{num_heads} heads do not split over {world} ranks")
    per = num_heads // world
    return slice(rank * per, (rank + 1) * per)


class KVHeadShardedBackend(AttentionBackend):
    """Wraps a single-GPU backend (default: B200Backend) so that `forward` takes the FULL q / k / v of the
    step, keeps this rank's heads, runs on this rank's pools and returns the full [N, H, Dh] output."""

    name = "b200_kv_sharded"

    def __init__(self, inner: AttentionBackend | None = None, group: dist.ProcessGroup | None = None) -> None:
        if inner is None:
            from .attention.backend import B200Backend

            inner = B200Backend()
        self.inner = inner
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)

    def prefill(self, q, k, v, key_valid=None, **kwargs):
        qs = head_range(self.rank, self.world, q.shape[1])
        ks = head_range(self.rank, self.world, k.shape[1])
        local = self.inner.prefill(q[:, qs], k[:, ks], v[:, ks], key_valid=key_valid, **kwargs)  # [B, H/n, T, Dh]
        return self._gather(local.transpose(0, 1).contiguous(), dim_heads=1).transpose(0, 1)

    def forward(self, q, k, v, k_cache, v_cache, meta):
        qs = head_range(self.rank, self.world, q.shape[1])
        ks = head_range(self.rank, self.world, k.shape[1])
        if k_cache.shape[2] != ks.stop - ks.start:
            raise ValueError(f"rank {self.rank}: pools hold {k_cache.shape[2]} KV heads, expected {ks.stop - ks.start}")
        local = self.inner.forward(q[:, qs], k[:, ks], v[:, ks], k_cache, v_cache, meta)  # [N, H/n, Dh]
        return self._gather(local, dim_heads=1)

    def _gather(self, local: torch.Tensor, dim_heads: int) -> torch.Tensor:
        """[A, H/n, ...] on every rank -> [A, H, ...] with rank r's heads at [r*H/n, (r+1)*H/n)."""
        if self.world == 1:
            return local
        local = local.contiguous()
        out = torch.empty((self.world * local.shape[0], *local.shape[1:]), dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(out, local, group=self.group)  # rank-major concatenation along dim 0
        out = out.view(self.world, *local.shape).movedim(0, dim_heads)  # [A, n, H/n, ...]
        return out.reshape(*local.shape[:dim_heads], -1, *local.shape[dim_heads + 1:])
