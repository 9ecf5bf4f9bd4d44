"""K3 block copy on the GPU: bit-exact against the oracle's copy_blocks, the copy-on-write flow of BASELINE
config 4 (shared prefix whose last block is partly filled), and the evict + compact flow of config 5
(attention after compaction is bit-identical to attention before it)."""

from __future__ import annotations

import random

import pytest
import torch

import oracle
from paged_helpers import assert_close, bits

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16], ids=str)
def test_copy_blocks_bit_exact_all_layers(mlb, cuda, dtype):
    cfg = mlb.KVShape(num_hidden_layers=4, num_key_value_heads=8, head_dim=128)
    cache = mlb.PagedKVCache(cfg, 64, cuda, dtype)
    g = torch.Generator(device=cuda).manual_seed(1)
    for p in cache.k + cache.v:
        p.copy_(torch.randn(p.shape, device=cuda, generator=g).to(dtype))
    ids = list(range(64))
    random.Random(2).shuffle(ids)
    src, dst = ids[:20], ids[20:40]
    ref = [p.cpu() for p in cache.k + cache.v]
    oracle.copy_blocks(ref, src, dst)
    cache.copy_blocks(src, dst)
    for got, exp in zip(cache.k + cache.v, ref):
        assert torch.equal(bits(got.cpu()), bits(exp))


def test_copy_blocks_flags_out_of_range_pairs(mlb, cuda):
    cfg = mlb.KVShape(2, 2, 64)
    cache = mlb.PagedKVCache(cfg, 8, cuda, torch.bfloat16)
    for p in cache.k + cache.v:
        p.normal_()
    before = [p.clone() for p in cache.k + cache.v]
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    cache.copy_blocks([1, 2], [8, 3], err=err)  # 8 is outside the pool: skipped, flagged
    assert int(err.item()) & 8
    for got, b in zip(cache.k + cache.v, before):
        assert torch.equal(got[3], b[2]) and torch.equal(got[:3], b[:3]) and torch.equal(got[4:], b[4:])


def test_prefix_sharing_with_copy_on_write(mlb, cuda):
    """Config-4 shape at small scale: 6 sequences share a 40-token prefix (blocks 0-2, the last one partly
    filled, refcount 6).  Each sequence's first append lands in the shared partial block, so it is COW-copied
    first; the shared blocks must stay untouched and every output must match the oracle."""
    h, hkv, dh, nb = 32, 8, 128, 64
    cfg = mlb.KVShape(1, hkv, dh)
    cache = mlb.PagedKVCache(cfg, nb, cuda, torch.bfloat16)
    bm = mlb.BlockManager(nb, 16)
    g = torch.Generator(device=cuda).manual_seed(4)
    prefix_len, n_seq = 40, 6
    prefix_blocks = bm.allocate(3)
    pre_k = torch.randn(prefix_len, hkv, dh, device=cuda, generator=g).to(torch.bfloat16)
    pre_v = torch.randn(prefix_len, hkv, dh, device=cuda, generator=g).to(torch.bfloat16)
    slots = torch.tensor([prefix_blocks[p // 16] * 16 + p % 16 for p in range(prefix_len)], device=cuda)
    mlb.kv_append(cache.k[0], cache.v[0], slots, pre_k, pre_v)
    tables = []
    for _ in range(n_seq):
        bm.acquire(prefix_blocks)
        tables.append(list(prefix_blocks))
    bm.free(list(prefix_blocks))  # the prefix's creator leaves; each sequence holds one reference
    bm.check(tables)
    shared_before = cache.k[0][prefix_blocks].clone()
    # each sequence appends 3 tokens at positions 40..42: they land in the shared partial block 2
    pairs = [p for t in tables for p in bm.cow_for_append(t, prefix_len, 3)]
    assert len(pairs) == n_seq - 1  # the last holder writes in place
    cache.copy_blocks([s for s, _ in pairs], [d for _, d in pairs])
    bm.check(tables)
    n_tok = 3 * n_seq
    q = torch.randn(n_tok, h, dh, device=cuda, generator=g).to(torch.bfloat16)
    k = torch.randn(n_tok, hkv, dh, device=cuda, generator=g).to(torch.bfloat16)
    v = torch.randn(n_tok, hkv, dh, device=cuda, generator=g).to(torch.bfloat16)
    steps = [mlb.SeqStep(prefix_len, 3, t) for t in tables]
    meta = mlb.AttentionMetadata.build(steps, 16, cuda)
    ref_k, ref_v = cache.k[0].cpu(), cache.v[0].cpu()
    out = mlb.B200Backend().forward(q, k, v, cache.k[0], cache.v[0], meta)
    om = oracle.build_metadata([(s.num_cached, s.num_new, s.block_ids) for s in steps], 16)
    expected = oracle.forward(q.cpu(), k.cpu(), v.cpu(), ref_k, ref_v, om)
    assert_close(out, expected, torch.bfloat16)
    assert torch.equal(cache.k[0].cpu(), ref_k)
    # only the last holder wrote into the original partial block; the full shared blocks never change
    assert torch.equal(cache.k[0][prefix_blocks[:2]], shared_before[:2])


def test_evict_compact_then_attend_is_bit_identical(mlb, cuda):
    """Config-5 shape at small scale: evict ~10% of the sequences, compact the pool, and the attention over the
    moved blocks is bit-identical to the attention before the move (same values, same split)."""
    h, hkv, dh = 32, 8, 128
    n_seq, ctx = 20, 300
    pages = -(-(ctx + 1) // 16)
    nb = n_seq * pages + 10
    cfg = mlb.KVShape(2, hkv, dh)
    cache = mlb.PagedKVCache(cfg, nb, cuda, torch.bfloat16)
    g = torch.Generator(device=cuda).manual_seed(7)
    for p in cache.k + cache.v:
        p.copy_(torch.randn(p.shape, device=cuda, generator=g).to(torch.bfloat16))
    bm = mlb.BlockManager(nb, 16)
    junk = bm.allocate(10)  # scatter the allocation so compaction has work
    tables = [bm.allocate(pages) for _ in range(n_seq)]
    bm.free(junk)
    evict = sorted(random.Random(3).sample(range(n_seq), 2))
    for i in reversed(evict):
        bm.free(tables.pop(i))
    q = torch.randn(len(tables), h, dh, device=cuda, generator=g).to(torch.bfloat16)
    k = torch.randn(len(tables), hkv, dh, device=cuda, generator=g).to(torch.bfloat16)
    v = torch.randn(len(tables), hkv, dh, device=cuda, generator=g).to(torch.bfloat16)

    def attend(layer):
        meta = mlb.AttentionMetadata.build([mlb.SeqStep(ctx, 1, t) for t in tables], 16, cuda)
        return mlb.B200Backend().forward(q, k, v, cache.k[layer], cache.v[layer], meta)

    before = [attend(0), attend(1)]
    src, dst = bm.compact(tables)
    assert src and len(src) == len(dst)
    cache.copy_blocks(src, dst)
    bm.check(tables)
    after = [attend(0), attend(1)]
    for a, b in zip(before, after):
        assert torch.equal(a, b)
