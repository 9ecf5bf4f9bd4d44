"""KV-head sharding of the paged path across the GPUs of one node (one process per GPU).

Rank r of n owns KV heads [r * Hkv / n, (r + 1) * Hkv / n) and their query heads
[r * H / n, (r + 1) * H / n) (grouped-query attention keeps each KV head with its query group), so its
pools are [num_blocks, block_size, Hkv / n, Dh].  Block ids, block tables, slot_mapping and seq_lens are
the same on every rank: append, copy-on-write, compaction and attention are purely local.  The one
exchange is the attention output: each rank computes [N, H / n, Dh] and every rank needs [N, H, Dh].
Two transports:
- "p2p": `PeerOutputs` maps every rank's gathered-output buffer into every process (CUDA IPC).  The
  attention kernel leaves unsplit rows in this rank's own buffer; the split-K reduction kernel then
  finishes the split rows and stores every row of this rank into every peer's buffer over NVLink
  (mlb_splitk_reduce_gather), and a one-warp flag barrier kernel says that every peer's rows have landed.
  No NCCL launch on the data path.
- "nccl": the rank's [N, H / n, Dh] rows, then `all_gather_into_tensor` (also the path for gloo / CPU).
The reference has no parallelism (its roadmap names NCCL tensor parallelism,
docs/distributed_inference_plan.md:325).
"""

from __future__ import annotations

import ctypes
import math

import torch
import torch.distributed as dist

from . import _lib
from .attention.base import AttentionBackend
from .ops import _stream, out_targets


def head_range(rank: int, world: int, num_heads: int) -> slice:
    if num_heads % world:
        raise ValueError(f"{num_heads} heads do not split over {world} ranks")
    per = num_heads // world
    return slice(rank * per, (rank + 1) * per)


class _DeviceBytes:
    """A raw device allocation seen by torch as a uint8 tensor (CUDA array interface, no copy)."""

    def __init__(self, ptr: int, nbytes: int) -> None:
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3, "strides": None}


PACKET_BYTES_PER_PEER = 384 << 10  # exchange="auto": the largest step (bytes of rows per peer) sent as packets


class PeerOutputs:
    """Gathered attention-output buffers shared by the ranks of one node, written by the kernels' stores.

    Collective: every rank of `group` constructs it with the same arguments.  Each rank allocates
    `slots` buffers of [capacity, num_heads, head_dim] plus flag words (mlb_ipc_alloc), the handles are
    exchanged over the process group, and every rank opens its peers' (mlb_ipc_open).  `targets(slot,
    head_offset)` gives the kernels every rank's slot buffer; `barrier()` launches the flag barrier
    (mlb_peer_barrier) on the current stream; `output(slot, n)` is this rank's slot as [n, H, Dh].

    exchange "auto" (default): "packets" for a step whose rows are at most PACKET_BYTES_PER_PEER bytes per
    peer, "barrier" for a larger one (measured on two B200s: packets 2.9% faster per step at 64 decode rows
    of 16 heads, 256 KB per peer; 2-2.5% slower at 128 rows, 512 KB per peer, where the doubled NVLink bytes
    cost more than the second launch, fence and flag round trip they save).
    exchange "packets": the rows travel as flagged packets (`ops.splitk_reduce_exchange`: one
    launch sends this rank's rows and waits for the peers', no barrier; twice the NVLink bytes, no fence or
    flag round trip); each rank also holds two packet areas of [capacity, H, Dh] x 2 element bytes, which
    the calls take in turn whatever slot they write.
    exchange "barrier": plain stores into every rank's buffer (`ops.splitk_reduce_gather`), then
    `barrier()`.

    A slot is rewritten by the peers' next use of it, so rotate through the slots (forward after forward)
    and consume each output before the forward that reuses its slot: with 2 slots that is guaranteed
    when the output is read on the stream before the next forward's barrier completes.
    """

    def __init__(self, capacity: int, num_heads: int, head_dim: int, dtype: torch.dtype, device: torch.device,
                 slots: int = 2, group: dist.ProcessGroup | None = None, timeout_s: float = 2.0,
                 exchange: str = "auto") -> None:
        if exchange not in ("auto", "packets", "barrier"):
            raise ValueError(f"exchange must be 'auto', 'packets' or 'barrier', got {exchange!r}")
        self.exchange = exchange
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        if self.world > _lib.MAX_OUT_DESTS:
            raise ValueError(f"PeerOutputs: at most {_lib.MAX_OUT_DESTS} ranks, got {self.world}")
        self.capacity, self.num_heads, self.head_dim, self.dtype = capacity, num_heads, head_dim, dtype
        self.device, self.slots, self.group = torch.device(device), slots, group
        elt = torch.empty(0, dtype=dtype).element_size()
        self.slot_bytes = -(-capacity * num_heads * head_dim * elt // 256) * 256
        self._flags_off = slots * self.slot_bytes  # world uint32 flag words, then the epoch counter
        self._epoch_off = self._flags_off + 128
        self._state_off = self._epoch_off + 128  # the packet exchange's {epoch, arrivals}
        self._packets_off = self._state_off + 128
        # per packet area (two): [capacity][world][H / world][Dh x elt / 4] packets of 8 bytes
        self.packet_bytes = (-(-capacity * num_heads * head_dim * elt * 2 // 256) * 256) if exchange != "barrier" else 0
        self._row_bytes = num_heads // self.world * head_dim * elt  # one token's rows of this rank's heads
        total = self._packets_off + 2 * self.packet_bytes
        lib = _lib.lib()
        with torch.cuda.device(self.device):
            ptr, handle = ctypes.c_void_p(), ctypes.create_string_buffer(_lib.IPC_HANDLE_BYTES)
            _lib.check(lib.mlb_ipc_alloc(total, ctypes.byref(ptr), handle), "ipc_alloc")
            self._own = ptr.value
            handles: list[bytes | None] = [None] * self.world
            dist.all_gather_object(handles, handle.raw, group=group)
            self._opened: list[int] = []
            self.bases: list[int] = []
            for r, h in enumerate(handles):
                if r == self.rank:
                    self.bases.append(self._own)
                    continue
                p = ctypes.c_void_p()
                _lib.check(lib.mlb_ipc_open(h, ctypes.byref(p)), f"ipc_open (rank {r})")
                self._opened.append(p.value)
                self.bases.append(p.value)
        self._bytes = torch.as_tensor(_DeviceBytes(self._own, total), device=self.device)
        self._flags = (ctypes.c_void_p * self.world)(*[b + self._flags_off for b in self.bases])
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.timeout_ns = int(timeout_s * 1e9)
        self._targets: dict[tuple[int, int, bool], _lib.OutTargets] = {}
        self._areas = (ctypes.c_void_p * (2 * self.world))(*[b + self._packets_off + a * self.packet_bytes
                                                             for a in range(2) for b in self.bases])

    def use_packets(self, num_tokens: int) -> bool:
        """Whether a step of `num_tokens` rows goes as flagged packets (else plain stores + barrier()).  Every
        rank decides the same way (same step shape)."""
        if self.exchange != "auto":
            return self.exchange == "packets"
        return num_tokens * self._row_bytes <= PACKET_BYTES_PER_PEER

    def packet_areas(self):
        """Both packet areas of every rank: a ctypes array of 2 x world device addresses, area a of rank p
        at a * world + p."""
        if not self.packet_bytes:
            raise RuntimeError("PeerOutputs: built with exchange='barrier' (no packet areas)")
        return self._areas

    def slot_address(self, slot: int) -> int:
        """Device address of this rank's gathered buffer of `slot`."""
        return self._own + slot * self.slot_bytes

    @property
    def state_address(self) -> int:
        return self._own + self._state_off

    def targets(self, slot: int, head_offset: int) -> _lib.OutTargets:
        """Every rank's buffer of `slot` (in rank order: this rank's is `self_dest` = rank)."""
        key = (slot, head_offset, True)
        if key not in self._targets:
            off = slot * self.slot_bytes
            self._targets[key] = out_targets([b + off for b in self.bases], head_offset,
                                             self.num_heads * self.head_dim, self.head_dim)
        return self._targets[key]

    def local_targets(self, slot: int, head_offset: int) -> _lib.OutTargets:
        """This rank's own buffer of `slot` only (where the attention kernel leaves unsplit rows)."""
        key = (slot, head_offset, False)
        if key not in self._targets:
            self._targets[key] = out_targets([self._own + slot * self.slot_bytes], head_offset,
                                             self.num_heads * self.head_dim, self.head_dim)
        return self._targets[key]

    @property
    def self_dest(self) -> int:
        return self.rank

    def slot_bytes_view(self, lo: int, hi: int) -> torch.Tensor:
        """This rank's slots [lo, hi) as one contiguous uint8 tensor (slot s at (s - lo) * slot_bytes): a
        run of outputs can be read back with one copy."""
        if not 0 <= lo <= hi <= self.slots:
            raise ValueError(f"PeerOutputs: slots [{lo}, {hi}) outside [0, {self.slots})")
        return self._bytes[lo * self.slot_bytes: hi * self.slot_bytes]

    def output(self, slot: int, num_tokens: int) -> torch.Tensor:
        if num_tokens > self.capacity:
            raise ValueError(f"PeerOutputs: {num_tokens} tokens > capacity {self.capacity}")
        elt = torch.empty(0, dtype=self.dtype).element_size()
        n = num_tokens * self.num_heads * self.head_dim * elt
        raw = self._bytes[slot * self.slot_bytes: slot * self.slot_bytes + n]
        return raw.view(self.dtype).view(num_tokens, self.num_heads, self.head_dim)

    def barrier(self) -> None:
        rc = _lib.lib().mlb_peer_barrier(self._flags, self.rank, self.world, self._own + self._epoch_off,
                                         self.timeout_ns, self.err.data_ptr(),
                                         _stream(self.device))
        _lib.check(rc, "peer_barrier")

    def raise_errors(self) -> None:
        """Synchronise and raise if a barrier wait ran out of time (a peer never arrived)."""
        bits = int(self.err.item())
        if bits:
            raise RuntimeError(f"rank {self.rank}: a peer barrier timed out (device error bits {bits:#x})")

    def close(self) -> None:
        """Collective: unmap the peers' buffers, then free this rank's once every rank has unmapped it."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        lib = _lib.lib()
        for p in self._opened:
            lib.mlb_ipc_close(p)
        self._opened = []
        dist.barrier(group=self.group)
        self._bytes = None
        lib.mlb_ipc_free(self._own)
        self._own = None


class KVHeadShardedBackend(AttentionBackend):
    """Wraps a single-GPU backend (default: B200Backend) so that `forward` takes the FULL q / k / v of the
    step, keeps this rank's heads, runs on this rank's pools and returns the full [N, H, Dh] output.

    transport "p2p" (B200Backend inner, CUDA tensors): the output rows go straight into every rank's
    `PeerOutputs` slot; the returned tensor is a view of that slot, valid until `slots` - 1 more forwards
    have run (forwards rotate through the slots; 2 by default).
    transport "nccl": a fresh tensor from an NCCL (or gloo) all-gather.
    exchange (p2p only): "auto", "packets" or "barrier", how the rows reach the peers (see PeerOutputs)."""

    name = "b200_kv_sharded"

    def __init__(self, inner: AttentionBackend | None = None, group: dist.ProcessGroup | None = None,
                 transport: str = "nccl", slots: int = 2, exchange: str = "auto") -> None:
        if inner is None:
            from .attention.backend import B200Backend

            inner = B200Backend()
        if transport not in ("nccl", "p2p"):
            raise ValueError(f"transport must be 'nccl' or 'p2p', got {transport!r}")
        self.inner = inner
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.transport = transport
        if slots < 2:
            raise ValueError(f"slots must be >= 2, got {slots}")
        self.slots = slots
        if exchange not in ("auto", "packets", "barrier"):
            raise ValueError(f"exchange must be 'auto', 'packets' or 'barrier', got {exchange!r}")
        self.exchange = exchange
        self.peers: PeerOutputs | None = None
        self._slot = 0

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
        if self.transport == "p2p" and self.world > 1:
            return self._forward_p2p(q, k, v, k_cache, v_cache, meta, qs, ks)
        local = self.inner.forward(q[:, qs], k[:, ks], v[:, ks], k_cache, v_cache, meta)  # [N, H/n, Dh]
        return self._gather(local, dim_heads=1)

    def forward_local(self, q_l, k_l, v_l, k_cache, v_cache, meta):
        """`forward` for a rank that holds only its own heads of the step's rows, as a column-parallel QKV
        projection leaves them: q_l [N, H/n, Dh] (query heads [r H/n, (r+1) H/n)), k_l / v_l [N, Hkv/n, Dh].
        Returns the same full [N, H, Dh] output as `forward` on the full tensors, without any rank holding
        (or uploading) the other ranks' heads."""
        h = q_l.shape[1] * self.world
        qs = head_range(self.rank, self.world, h)
        ks = head_range(self.rank, self.world, k_l.shape[1] * self.world)
        if k_cache.shape[2] != k_l.shape[1]:
            raise ValueError(f"rank {self.rank}: pools hold {k_cache.shape[2]} KV heads, k_l {k_l.shape[1]}")
        if self.transport == "p2p" and self.world > 1:
            return self._forward_p2p(q_l, k_l, v_l, k_cache, v_cache, meta, qs, ks, local=True)
        local = self.inner.forward(q_l, k_l, v_l, k_cache, v_cache, meta)
        return self._gather(local, dim_heads=1)

    def _forward_p2p(self, q, k, v, k_cache, v_cache, meta, qs, ks, local=False):
        n, dh = q.shape[0], q.shape[2]
        h = q.shape[1] * self.world if local else q.shape[1]
        if not local:
            q, k, v = q[:, qs], k[:, ks], v[:, ks]
        p = self.peers
        if p is None or n > p.capacity or (p.num_heads, p.head_dim, p.dtype) != (h, dh, q.dtype):
            # collective (every rank sees the same step shape): grow to a power of two of tokens
            if p is not None:
                p.close()
            self.peers = p = PeerOutputs(1 << max(6, math.ceil(math.log2(max(n, 1)))), h, dh, q.dtype, q.device,
                                         slots=self.slots, group=self.group, exchange=self.exchange)
            self._slot = 0
        slot, self._slot = self._slot, (self._slot + 1) % p.slots
        self.inner.forward(q, k, v, k_cache, v_cache, meta, peer_gather=(p, slot, qs.start))
        return p.output(slot, n)

    def close(self) -> None:
        """Collective: release the p2p output buffers."""
        if self.peers is not None:
            self.peers.close()
            self.peers = None

    def _gather(self, local: torch.Tensor, dim_heads: int) -> torch.Tensor:
        """[A, H/n, ...] on every rank -> [A, H, ...] with rank r's heads at [r*H/n, (r+1)*H/n)."""
        if self.world == 1:
            return local
        local = local.contiguous()
        out = torch.empty((self.world * local.shape[0], *local.shape[1:]), dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(out, local, group=self.group)  # rank-major concatenation along dim 0
        out = out.view(self.world, *local.shape).movedim(0, dim_heads)  # [A, n, H/n, ...]
        return out.reshape(*local.shape[:dim_heads], -1, *local.shape[dim_heads + 1:])
