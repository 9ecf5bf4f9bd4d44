"""Host-side logic of the paged path, on the CPU: the vectorised metadata build, the block manager (the
reference's accounting tests plus copy-on-write and compaction planning), and the prefix-cache index."""

from __future__ import annotations

import json
import random

import pytest
import torch

import oracle
from conftest import GOLDEN

FIELDS = ("positions", "slot_mapping", "block_tables", "logits_index", "kv_indptr", "kv_indices", "kv_last_page_len")


def test_metadata_matches_reference_golden(mlb):
    for g in json.loads((GOLDEN / "metadata.json").read_text()):
        seqs = [mlb.SeqStep(c, n, b) for c, n, b in g["seqs"]]
        if "error" in g:
            with pytest.raises(ValueError, match="can't hold"):
                mlb.AttentionMetadata.build(seqs, g["block_size"], "cpu")
            continue
        m = mlb.AttentionMetadata.build(seqs, g["block_size"], "cpu")
        assert m.query_start_loc == g["query_start_loc"] and m.seq_lens == g["seq_lens"]
        for f in FIELDS:
            assert getattr(m, f).tolist() == g[f], f
        assert m.qo_indptr.tolist() == g["query_start_loc"] and m.seq_lens_i32.tolist() == g["seq_lens"]
        assert m.block_tables_i32.tolist() == g["block_tables"]
        assert m.slot_mapping.dtype == torch.long and m.block_tables_i32.dtype == torch.int32


@pytest.mark.parametrize("seed", range(5))
def test_metadata_matches_oracle_on_random_steps(mlb, seed):
    r = random.Random(seed)
    seqs = []
    for _ in range(r.randint(1, 30)):
        cached, new = r.randint(0, 500), r.randint(1, 70)
        seqs.append((cached, new, [r.randrange(10_000) for _ in range(-(-(cached + new) // 16) + r.randint(0, 3))]))
    m = mlb.AttentionMetadata.build([mlb.SeqStep(*s) for s in seqs], 16, "cpu")
    o = oracle.build_metadata(seqs, 16)
    assert m.query_start_loc == o.query_start_loc and m.seq_lens == o.seq_lens and m.num_new == o.num_new
    for f in FIELDS:
        assert getattr(m, f).tolist() == getattr(o, f), f
    assert m.max_query_len == max(o.num_new) and m.num_seqs == len(seqs)


def test_metadata_known_answer():  # tests/test_paged.py:41-50 of the reference, block size 4
    from importlib import import_module

    mlb = import_module("mini-llm-inference-server_b200")
    meta = mlb.AttentionMetadata.build([mlb.SeqStep(3, 1, [7]), mlb.SeqStep(0, 5, [2, 9])], 4, "cpu")
    assert meta.query_start_loc == [0, 1, 6] and meta.seq_lens == [4, 5] and meta.num_new == [1, 5]
    assert meta.positions.tolist() == [3, 0, 1, 2, 3, 4]
    assert meta.slot_mapping.tolist() == [7 * 4 + 3, 8, 9, 10, 11, 9 * 4]
    assert meta.block_tables.tolist() == [[7, 0], [2, 9]] and meta.logits_index.tolist() == [0, 5]


def test_append_private_flag(mlb):
    """append_private: every block that receives a row is among all sequences' context pages once."""
    S = mlb.SeqStep
    build = lambda seqs: mlb.AttentionMetadata.build(seqs, 4, "cpu").append_private
    assert build([S(3, 1, [7]), S(0, 5, [2, 9])])
    assert build([S(4, 1, [7, 3]), S(4, 1, [7, 5])])  # a shared prefix block, but the writes go to 3 and 5
    assert not build([S(2, 1, [7]), S(3, 1, [7])])  # both rows write block 7
    assert not build([S(2, 1, [7]), S(4, 0, [7])])  # another sequence reads the written block
    assert not build([S(5, 1, [4, 4])])  # the same block twice in one table
    assert not build([S(1, 1, [-1])])  # an invalid id: no fusion, the separate append flags it
    assert build([S(3, 0, [7])])  # nothing written
    big = 1 << 40  # sparse ids far past the dense-count range
    assert build([S(2, 1, [big]), S(3, 1, [big + 1])]) and not build([S(2, 1, [big]), S(3, 1, [big])])
    # a block beyond a sequence's context pages is not read by it
    assert build([S(2, 1, [7]), S(4, 0, [6, 1, 7])])


# ---------- block manager: the reference's accounting (tests/test_paged.py:152-163, test_prefix_cache.py:69-93)


def test_block_manager_accounting(mlb):
    bm = mlb.BlockManager(8, 16)
    assert bm.blocks_for(1) == 1 and bm.blocks_for(16) == 1 and bm.blocks_for(17) == 2
    a, b = bm.allocate(3), bm.allocate(5)
    assert bm.num_free == 0 and len(set(a + b)) == 8
    bm.check([a, b])
    with pytest.raises(RuntimeError, match="free"):
        bm.allocate(1)
    with pytest.raises(AssertionError):
        bm.check([a, b, a[:1]])
    bm.free(a)
    assert a == [] and bm.num_free == 3
    bm.check([b])


def test_refcounts_cached_blocks_and_lru_eviction(mlb):
    pc = mlb.PrefixCache()
    bm = mlb.BlockManager(4, 16, pc)
    a, b = bm.allocate(2), bm.allocate(2)
    pc.insert(b"a0", a[0])
    pc.insert(b"b0", b[0])
    a_ids, b_ids = list(a), list(b)
    bm.free(a)
    bm.free(b)
    assert bm.num_free == 4 and bm.num_cached == 2
    bm.check([])
    shared = pc.lookup([b"b0"])
    bm.acquire(shared)
    bm.acquire(shared)
    bm.check([shared, shared])
    got = bm.allocate(3)
    assert a_ids[0] in got and pc.lookup([b"a0"]) == [] and pc.lookup([b"b0"]) == [b_ids[0]]
    with pytest.raises(AssertionError, match="refcounts"):
        bm.check([shared, got])
    bm.free(got)
    bm.free(list(shared))
    bm.free(shared)
    bm.check([])
    bm.clear_cache()
    assert bm.num_cached == 0 and len(pc) == 0 and bm.num_free == 4


# ---------- copy-on-write and compaction planning


def test_cow_gives_the_writer_a_private_block(mlb):
    bm = mlb.BlockManager(16, 16)
    prefix = bm.allocate(3)  # a shared prefix ending in a partly filled block
    tables = [list(prefix)]
    for _ in range(3):
        bm.acquire(prefix)
        tables.append(list(prefix))
    bm.check(tables)
    pairs = bm.cow_for_append(tables[1], num_cached=40, num_new=1)  # writes into block 2 (tokens 32..47)
    assert len(pairs) == 1 and pairs[0][0] == prefix[2] and tables[1][2] == pairs[0][1]
    assert tables[1][:2] == prefix[:2] and bm.refcount(prefix[2]) == 3
    bm.check(tables)
    # the last holder writes in place: nothing to copy
    for t in tables[2:]:
        bm.cow_for_append(t, 40, 1)
    assert bm.cow_for_append(tables[0], 40, 1) == [] and bm.refcount(prefix[2]) == 1
    bm.check(tables)


@pytest.mark.parametrize("seed", range(4))
def test_compaction_matches_oracle_plan_and_keeps_accounting(mlb, seed):
    r = random.Random(seed)
    pc = mlb.PrefixCache()
    bm = mlb.BlockManager(200, 16, pc)
    tables = [bm.allocate(r.randint(1, 12)) for _ in range(14)]
    shared = tables[0][:3]
    for t in tables[1:4]:
        bm.acquire(shared)
        t[:0] = shared
    named = tables[5][:2]
    for i, b in enumerate(named):
        pc.insert(bytes([seed, i]), b)
    evicted = [tables.pop(r.randrange(len(tables))) for _ in range(3)]  # 10%-style eviction
    for t in evicted:
        bm.free(t)
    bm.check(tables)
    before = [list(t) for t in tables]
    cached = bm.cached_blocks()
    src, dst, expect = oracle.compact_plan(before + [cached], 200)
    got_src, got_dst = bm.compact(tables)
    assert (got_src, got_dst) == (src, dst)
    assert tables == expect[:-1]
    bm.check(tables)
    live = {b for t in tables for b in t} | set(bm.cached_blocks())
    assert live == set(range(len(live)))
    for b_old, b_new in zip(src, dst):  # prefix names follow the moved blocks
        assert not pc.is_cached(b_old) or b_old in live
    assert all(pc.is_cached(b) for b in bm.cached_blocks())


# ---------- prefix-cache index


def test_prefix_hashes_match_reference_golden(mlb):
    from importlib import import_module

    prefix = import_module(mlb.__name__ + ".cache.prefix")
    g = json.loads((GOLDEN / "prefix.json").read_text())
    assert [prefix.root_hash(k).hex() for k in g["keys"]] == g["roots"]
    for c in g["chains"]:
        chain: list[bytes] = []
        prefix.extend_chain(chain, prefix.root_hash(g["keys"][c["key"]]), c["tokens"], 5, 16)
        assert [h.hex() for h in chain] == c["chain"]


def test_prefix_cache_index(mlb):
    pc = mlb.PrefixCache()
    pc.insert(b"h0", 4)
    pc.insert(b"h1", 9)
    pc.insert(b"h1", 2)
    assert pc.lookup([b"h0", b"h1", b"h2"]) == [4, 9] and pc.lookup([b"h1"]) == [9]
    assert not pc.is_cached(2)
    pc.move(9, 1)
    assert pc.lookup([b"h0", b"h1"]) == [4, 1] and not pc.is_cached(9)
    pc.forget(4)
    assert pc.lookup([b"h0", b"h1"]) == []
