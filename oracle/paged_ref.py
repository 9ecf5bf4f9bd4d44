"""CPU restatement of the reference's paged KV path.  TEST INFRASTRUCTURE ONLY (see `oracle/__init__.py`).

Reference files restated here (paths inside prakhar-iit/mini-llm-inference-server):
- `src/minillm/attention/metadata.py:71-103`   AttentionMetadata.build   -> `build_metadata`
- `src/minillm/attention/paged_torch_ref.py:23-28`  write_kv           -> `write_kv`
- `src/minillm/attention/paged_torch_ref.py:31-37`  gather             -> `gather`
- `src/minillm/attention/paged_torch_ref.py:40-74`  paged_attention    -> `paged_attention`
- `src/minillm/attention/torch_ref.py:46-48`        TorchRefBackend.forward -> `forward`
- `src/minillm/cache/slot.py:41-46` SlotKVCache.move (the reference's only compaction-by-copy) is the
  model for `copy_blocks`; the reference has no block copy-on-write or block compaction, so
  `copy_blocks` / `compact_plan` state the definition this build's kernels are checked against.

Tensors are torch CPU tensors: the reference's arithmetic is torch's (`Tensor.to` casts with
round-to-nearest-even, SDPA in the pool dtype), so the restatement keeps torch as its maths library and
restates the algorithm around it.  Attention is run in float32 on up-cast inputs, which is the oracle
the CUDA kernels are measured against (2e-2 max-abs in bf16/fp16, 1e-5 in fp32).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F


@dataclass
class OracleMeta:
    """The host-side facts of one ragged step, as `AttentionMetadata` holds them (metadata.py:36-51)."""

    block_size: int
    query_start_loc: list[int]
    seq_lens: list[int]
    positions: list[int]
    slot_mapping: list[int]
    block_tables: list[list[int]]
    logits_index: list[int]
    kv_indptr: list[int]
    kv_indices: list[int]
    kv_last_page_len: list[int]

    @property
    def num_new(self) -> list[int]:
        q = self.query_start_loc
        return [q[i + 1] - q[i] for i in range(len(q) - 1)]


def build_metadata(seqs: list[tuple[int, int, list[int]]], block_size: int) -> OracleMeta:
    """seqs = [(num_cached, num_new, block_ids), ...] -> the step's metadata (metadata.py:71-103).

    Token p of a sequence lives at flat slot block_ids[p // bs] * bs + p % bs.  Tables are padded with
    block 0 to the widest table.  The CSR page list keeps only pages that hold context.
    """
    starts, lens, positions, slots = [0], [], [], []
    for cached, new, blocks in seqs:
        end = cached + new
        if len(blocks) * block_size < end:
            raise ValueError(f"{len(blocks)} blocks can't hold {end} tokens")
        starts.append(starts[-1] + new)
        lens.append(end)
        for p in range(cached, end):
            positions.append(p)
            slots.append(blocks[p // block_size] * block_size + p % block_size)
    width = max(len(b) for _, _, b in seqs)
    tables = [list(b) + [0] * (width - len(b)) for _, _, b in seqs]
    indptr, indices, last = [0], [], []
    for (_, _, blocks), n in zip(seqs, lens):
        used = (n + block_size - 1) // block_size
        indices.extend(blocks[:used])
        indptr.append(indptr[-1] + used)
        last.append(n - (used - 1) * block_size)
    return OracleMeta(block_size, starts, lens, positions, slots, tables, [s - 1 for s in starts[1:]],
                      indptr, indices, last)


def write_kv(k_cache: torch.Tensor, v_cache: torch.Tensor, slot_mapping, k: torch.Tensor,
             v: torch.Tensor) -> None:
    """Scatter k, v [N, Hkv, Dh] into the pools [num_blocks, bs, Hkv, Dh] at flat slots (in place).

    paged_torch_ref.py:23-28: the rows are cast to the pool dtype with `Tensor.to` (round to nearest
    even) and written through the pool's flat [num_blocks * bs, Hkv, Dh] view.
    """
    slots = torch.as_tensor(slot_mapping, dtype=torch.long)
    for pool, rows in ((k_cache, k), (v_cache, v)):
        flat = pool.view(-1, pool.shape[-2], pool.shape[-1])
        flat[slots] = rows.to(pool.dtype)


def gather(cache: torch.Tensor, block_tables: torch.Tensor, length: int) -> torch.Tensor:
    """cache [num_blocks, bs, Hkv, Dh], tables [B, >= ceil(length / bs)] -> [B, Hkv, length, Dh].

    paged_torch_ref.py:31-37: whole pages are fetched through the table, then cut to `length` tokens.
    """
    bs = cache.shape[1]
    pages = -(-length // bs)
    picked = cache[block_tables[:, :pages].long()]  # [B, pages, bs, Hkv, Dh]
    b = picked.shape[0]
    return picked.reshape(b, pages * bs, *cache.shape[2:])[:, :length].permute(0, 2, 1, 3)


def paged_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, meta: OracleMeta,
                    compute_dtype: torch.dtype | None = torch.float32) -> torch.Tensor:
    """q [N, H, Dh] -> [N, H, Dh] in q's dtype; attention of each new token over its sequence's pages.

    paged_torch_ref.py:40-74.  Decode rows (one new token) are gathered together up to the longest
    context and masked past each row's own length; a row with several new tokens attends causally with
    the mask aligned to the end of its context (query i of n sees keys 0 .. length - n + i).
    Scale 1/sqrt(Dh); each KV head serves H / Hkv query heads.  `compute_dtype` up-casts q and the
    pools first (None keeps the pool dtype, as the reference itself does).
    """
    dt = compute_dtype or q.dtype
    qc = q.to(dt)
    tables = torch.as_tensor(meta.block_tables, dtype=torch.long)
    starts, lens, news = meta.query_start_loc, meta.seq_lens, meta.num_new
    out = torch.empty(q.shape, dtype=dt)

    rows = [i for i, n in enumerate(news) if n == 1]
    if rows:
        longest = max(lens[i] for i in rows)
        sel = torch.tensor(rows)
        k = gather(k_cache, tables[sel], longest).to(dt)  # gathered first, then up-cast: same values
        v = gather(v_cache, tables[sel], longest).to(dt)
        tok = torch.tensor([starts[i] for i in rows])
        ends = torch.tensor([lens[i] for i in rows])
        mask = (torch.arange(longest)[None, :] < ends[:, None])[:, None, None, :]
        o = F.scaled_dot_product_attention(qc[tok][:, :, None], k, v, attn_mask=mask, enable_gqa=True)
        out[tok] = o[:, :, 0]

    for i, n in enumerate(news):
        if n == 1:
            continue
        s, length = starts[i], lens[i]
        k = gather(k_cache, tables[i:i + 1], length).to(dt)
        v = gather(v_cache, tables[i:i + 1], length).to(dt)
        mask = torch.ones(n, length, dtype=torch.bool).tril(diagonal=length - n)
        o = F.scaled_dot_product_attention(qc[s:s + n].transpose(0, 1)[None], k, v, attn_mask=mask,
                                           enable_gqa=True)
        out[s:s + n] = o[0].transpose(0, 1)
    return out.to(q.dtype) if compute_dtype is None else out


def forward(q, k, v, k_cache, v_cache, meta: OracleMeta, compute_dtype=torch.float32) -> torch.Tensor:
    """torch_ref.py:46-48: write this step's k, v first (a new token attends to itself), then attend."""
    write_kv(k_cache, v_cache, meta.slot_mapping, k, v)
    return paged_attention(q, k_cache, v_cache, meta, compute_dtype)


def copy_blocks(pools: list[torch.Tensor], src, dst) -> None:
    """pool[dst[i]] = pool[src[i]] for every pool (every layer's K and V), bit for bit, in place.

    All reads happen before any write (the source blocks are materialised first), the definition the
    CUDA block copy is held to when the destination set is disjoint from the source set.
    """
    s = torch.as_tensor(src, dtype=torch.long)
    d = torch.as_tensor(dst, dtype=torch.long)
    for pool in pools:
        pool[d] = pool[s].clone()


def compact_plan(tables: list[list[int]], num_blocks: int) -> tuple[list[int], list[int], list[list[int]]]:
    """Move every live block whose id is >= the number of live blocks into the lowest free ids.

    Returns (src, dst, new_tables).  Live blocks are taken in ascending id order and paired with free
    ids in ascending order, so after the copy the live blocks occupy exactly [0, n_live).  A block
    listed by several tables (a shared prefix) moves once and every table is rewritten.
    """
    live = sorted({b for t in tables for b in t})
    n_live = len(live)
    if n_live > num_blocks:
        raise ValueError("more live blocks than the pool holds")
    live_set = set(live)
    holes = [b for b in range(n_live) if b not in live_set]
    movers = [b for b in live if b >= n_live]
    assert len(holes) == len(movers)
    remap = dict(zip(movers, holes))
    new_tables = [[remap.get(b, b) for b in t] for t in tables]
    return movers, holes, new_tables


def ceil_div(a: int, b: int) -> int:
    return -(-a // b)


def kv_read_bytes(seq_lens: list[int], num_kv_heads: int, head_dim: int, elt: int) -> int:
    """Algorithmic K+V bytes one decode pass reads: every context token, K and V, every KV head."""
    return sum(seq_lens) * 2 * num_kv_heads * head_dim * elt


__all__ = ["OracleMeta", "build_metadata", "write_kv", "gather", "paged_attention", "forward",
           "copy_blocks", "compact_plan", "ceil_div", "kv_read_bytes"]
