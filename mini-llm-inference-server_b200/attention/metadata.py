"""Per-step attention metadata for paged KV, the reference's `AttentionMetadata` (metadata.py:27-103) with
the same fields, built without a per-token Python loop.

The reference's `build` walks every new token in Python (metadata.py:72-81) and makes eleven separate
host-to-device tensors.  Here the step is described with numpy array arithmetic and all device tensors
are views into two buffers (int64 and int32) that cross to the device in two copies from pinned
memory, once per step; every layer reuses them.

Example (block size 16): sequence 0 has 3 tokens cached and adds 1; sequence 1 is a fresh 5-token prompt.
    query_start_loc = [0, 1, 6]; seq_lens = [4, 5]; positions = [3, 0, 1, 2, 3, 4]
    slot_mapping    = [b0*16 + 3, b1*16 + 0, ..., b1*16 + 4]
"""

from __future__ import annotations

import itertools
from dataclasses import dataclass

import numpy as np
import torch


# The fields of the reference's AttentionMetadata (metadata.py:36-52), in its order: the object an unmodified
# reference engine hands a backend.  Every one is kept here with the same meaning.
REFERENCE_FIELDS = ("block_size", "query_start_loc", "seq_lens", "positions", "slot_mapping", "block_tables",
                    "logits_index", "qo_indptr", "seq_lens_i32", "block_tables_i32", "kv_indptr", "kv_indices",
                    "kv_last_page_len")


@dataclass
class SeqStep:
    """One sequence in a step: `num_cached` tokens already in the pool, `num_new` added now (metadata.py:27-33)."""

    num_cached: int
    num_new: int
    block_ids: list[int]  # covers num_cached + num_new tokens


@dataclass
class AttentionMetadata:
    block_size: int
    query_start_loc: list[int]  # host, len S + 1
    seq_lens: list[int]  # host: context length per sequence, this step's tokens included
    positions: torch.Tensor  # [N] int64
    slot_mapping: torch.Tensor  # [N] int64 flat pool slot of each new token
    block_tables: torch.Tensor  # [S, max_blocks] int64, padded with block 0
    logits_index: torch.Tensor  # [S] int64 index of each sequence's last new token
    qo_indptr: torch.Tensor  # [S + 1] int32
    seq_lens_i32: torch.Tensor  # [S] int32
    block_tables_i32: torch.Tensor  # [S, max_blocks] int32
    kv_indptr: torch.Tensor  # [S + 1] int32 offsets into kv_indices
    kv_indices: torch.Tensor  # int32: the pages each sequence uses, concatenated
    kv_last_page_len: torch.Tensor  # [S] int32
    # Not in the reference's metadata: the int32 block tables on the host, which let the planner find decode
    # rows that share prefix blocks without a device round trip.
    block_tables_host: np.ndarray | None = None
    # Not in the reference's metadata either: True when every block that receives one of this step's rows is
    # among the context pages of one sequence, once.  No other sequence (or position) then reads a written
    # block, and the append may ride in the attention launch (ops.attention_partials(append=...)).
    append_private: bool = False

    @property
    def max_query_len(self) -> int:
        return max(self.num_new)

    @property
    def max_seq_len(self) -> int:
        return max(self.seq_lens)

    @property
    def num_seqs(self) -> int:
        return len(self.seq_lens)

    @property
    def num_new(self) -> list[int]:
        q = self.query_start_loc
        return [q[i + 1] - q[i] for i in range(len(q) - 1)]

    @classmethod
    def build(cls, seqs: list[SeqStep], block_size: int, device: torch.device | str) -> AttentionMetadata:
        """The step's metadata (metadata.py:71-103).  On a CUDA device the host sends the block ids and
        O(S) prefix arrays in one upload and `mlb_build_metadata` expands the per-token / per-page arrays
        and both padded tables on the GPU; elsewhere numpy computes them.  Same values either way."""
        s = len(seqs)
        cached = np.fromiter((q.num_cached for q in seqs), dtype=np.int64, count=s)
        new = np.fromiter((q.num_new for q in seqs), dtype=np.int64, count=s)
        nblk = np.fromiter((len(q.block_ids) for q in seqs), dtype=np.int64, count=s)
        ids = np.fromiter(itertools.chain.from_iterable(q.block_ids for q in seqs), dtype=np.int64,
                          count=int(nblk.sum()))
        return cls.build_arrays(cached, new, ids, nblk, block_size, device)

    @classmethod
    def build_arrays(cls, num_cached: np.ndarray, num_new: np.ndarray, block_ids: np.ndarray,
                     num_blocks: np.ndarray, block_size: int, device: torch.device | str,
                     expand_on: torch.cuda.Stream | None = None) -> AttentionMetadata:
        """`build` for an engine that keeps its block tables in arrays: num_cached / num_new / num_blocks are
        per sequence, block_ids every sequence's ids back to back (num_blocks[i] of them for sequence i).
        Skips turning Python lists of ids into an array, the bulk of `build`'s host time at large batches
        (512 sequences, 75K ids: ~2 ms of the ~5 ms).
        expand_on (CUDA): the upload stays on the current stream, the expansion kernel runs on this stream
        once the upload is in (an engine that uploads a step ahead on a side stream can expand on its compute
        stream just before the step's first layer, instead of beside whatever that stream is running)."""
        device = torch.device(device)
        cached = np.ascontiguousarray(num_cached, dtype=np.int64)
        new = np.ascontiguousarray(num_new, dtype=np.int64)
        nblk = np.ascontiguousarray(num_blocks, dtype=np.int64)
        ids = np.ascontiguousarray(block_ids, dtype=np.int64)
        s = cached.size
        if new.size != s or nblk.size != s or ids.size != int(nblk.sum()):
            raise ValueError(f"build_arrays: {s} sequences, {new.size} num_new, {nblk.size} num_blocks, "
                             f"{ids.size} ids for {int(nblk.sum())} table entries")
        ends = cached + new
        short = np.nonzero(nblk * block_size < ends)[0]
        if short.size:
            i = int(short[0])
            raise ValueError(f"{int(nblk[i])} blocks can't hold {int(ends[i])} tokens")
        width = int(nblk.max()) if s else 0
        starts = np.zeros(s + 1, dtype=np.int64)
        np.cumsum(new, out=starts[1:])
        n = int(starts[-1])
        used = -(-ends // block_size)  # pages holding context
        kv_indptr = np.zeros(s + 1, dtype=np.int64)
        np.cumsum(used, out=kv_indptr[1:])
        last_len = ends - (used - 1) * block_size
        ids_indptr = np.zeros(s + 1, dtype=np.int64)
        np.cumsum(nblk, out=ids_indptr[1:])
        owner = np.repeat(np.arange(s), new)  # sequence of each new token
        positions = np.arange(n, dtype=np.int64) - starts[owner] + cached[owner]
        written = ids[ids_indptr[owner] + positions // block_size]  # block of every new row
        if bool((nblk == used).all()):
            used_ids = ids
        else:  # the ids beyond each context's last page are not read
            col = np.arange(ids.size) - np.repeat(ids_indptr[:-1], nblk)
            used_ids = ids[col < np.repeat(used, nblk)]
        mask = np.arange(width)[None, :] < nblk[:, None]  # row-major order is the ids' order
        table32 = np.zeros((s, width), dtype=np.int32)
        table32[mask] = ids  # truncated to int32 like Tensor.to(torch.int32)

        if device.type == "cuda" and s:
            from .. import ops

            upload = _to_device(np.concatenate([ids, ids_indptr, starts, ends, kv_indptr, last_len]), device)
            d64 = torch.empty(2 * n + s * width + s, dtype=torch.int64, device=device)
            d32 = torch.empty(s * width + 4 * s + 2 + int(kv_indptr[-1]), dtype=torch.int32, device=device)
            if expand_on is None:
                ops.build_metadata(upload, ids.size, s, n, int(kv_indptr[-1]), width, block_size, d64, d32)
            else:
                expand_on.wait_stream(torch.cuda.current_stream(device))
                for t in (upload, d64, d32):  # used on that stream too: not reused before it is done
                    t.record_stream(expand_on)
                with torch.cuda.stream(expand_on):
                    ops.build_metadata(upload, ids.size, s, n, int(kv_indptr[-1]), width, block_size, d64, d32)
        else:
            table = np.zeros((s, width), dtype=np.int64)
            table[mask] = ids
            slots = written * block_size + positions % block_size
            kv_indices = table[np.arange(width)[None, :] < used[:, None]]  # row-major: sequence by sequence
            # two transfers: every int64 tensor in one buffer, every int32 tensor in another
            i64 = np.concatenate([positions, slots, table.reshape(-1), starts[1:] - 1])
            i32 = np.concatenate([starts, ends, table.reshape(-1), kv_indptr, kv_indices, last_len]).astype(np.int32)
            d64, d32 = _to_device(i64, device), _to_device(i32, device)
        o64 = np.cumsum([0, n, n, s * width, s])
        o32 = np.cumsum([0, s + 1, s, s * width, s + 1, int(kv_indptr[-1]), s])
        return cls(
            block_size=block_size,
            query_start_loc=starts.tolist(),
            seq_lens=ends.tolist(),
            positions=d64[o64[0]:o64[1]],
            slot_mapping=d64[o64[1]:o64[2]],
            block_tables=d64[o64[2]:o64[3]].view(s, width),
            logits_index=d64[o64[3]:o64[4]],
            qo_indptr=d32[o32[0]:o32[1]],
            seq_lens_i32=d32[o32[1]:o32[2]],
            block_tables_i32=d32[o32[2]:o32[3]].view(s, width),
            kv_indptr=d32[o32[3]:o32[4]],
            kv_indices=d32[o32[4]:o32[5]],
            kv_last_page_len=d32[o32[5]:o32[6]],
            block_tables_host=table32,
            append_private=_written_private(written, used_ids),
        )


def host_view(meta) -> tuple[np.ndarray, bool]:
    """(int32 block tables on the host, append_private) for a metadata object that carries only the
    reference's fields (minillm.attention.metadata.AttentionMetadata, metadata.py:36-52): its device
    `block_tables_i32` and `slot_mapping` are copied back (one synchronisation), and `append_private` holds
    only if every slot is the one the tables give (block_ids[p // bs] * bs + p % bs, as the reference's build
    makes it) and every written block is read by its own row alone.  This package's AttentionMetadata
    carries both already and needs no copy."""
    bs = int(meta.block_size)
    qo = np.asarray(meta.query_start_loc, dtype=np.int64)
    lens = np.asarray(meta.seq_lens, dtype=np.int64)
    tables_t = meta.block_tables_i32
    slots_t = meta.slot_mapping
    if tables_t.is_cuda:  # both copies queued, then one wait
        t_host = torch.empty(tables_t.shape, dtype=torch.int32, pin_memory=True)
        s_host = torch.empty(slots_t.shape, dtype=torch.int64, pin_memory=True)
        t_host.copy_(tables_t, non_blocking=True)
        s_host.copy_(slots_t, non_blocking=True)
        torch.cuda.current_stream(tables_t.device).synchronize()
    else:
        t_host, s_host = tables_t.to(torch.int32), slots_t.to(torch.int64)
    tables = t_host.numpy().copy()
    slots = s_host.numpy()
    s = lens.size
    new = np.diff(qo)
    n = int(qo[-1]) if s else 0
    if s == 0 or n == 0 or slots.shape != (n,):
        return tables, n == 0
    owner = np.repeat(np.arange(s), new)
    positions = np.arange(n, dtype=np.int64) - qo[owner] + (lens - new)[owner]
    page = positions // bs
    if tables.ndim != 2 or tables.shape[0] != s or (page >= tables.shape[1]).any() or (positions < 0).any():
        return tables, False
    written = tables[owner, page].astype(np.int64)
    if not np.array_equal(written * bs + positions % bs, slots):
        return tables, False
    used = -(-lens // bs)
    used_ids = tables[np.arange(tables.shape[1])[None, :] < used[:, None]].astype(np.int64)
    return tables, _written_private(written, used_ids)


def _written_private(written: np.ndarray, used_ids: np.ndarray) -> bool:
    """Every written block occurs once among all sequences' context pages (`written` is a subset of them)."""
    if written.size == 0:
        return True
    lo, hi = int(used_ids.min()), int(used_ids.max())
    if lo < 0:  # an invalid id: keep the separate append (it flags the slot)
        return False
    if hi < 4 * used_ids.size + (1 << 16):  # dense counters stay small next to the ids themselves
        return bool((np.bincount(used_ids)[written] == 1).all())
    ids, counts = np.unique(used_ids, return_counts=True)  # sparse ids: count by sorting
    return bool((counts[np.searchsorted(ids, written)] == 1).all())


def _to_device(a: np.ndarray, device: torch.device) -> torch.Tensor:
    host = torch.from_numpy(np.ascontiguousarray(a))
    if device.type == "cuda":
        return host.pin_memory().to(device, non_blocking=True)
    return host.clone() if device.type == "cpu" else host.to(device)
