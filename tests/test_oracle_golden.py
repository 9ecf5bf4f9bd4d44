"""The CPU oracle against golden vectors produced by running the reference itself
(`tests/golden/make_golden.py`).  This is what pins the oracle before the CUDA path is held to it."""

from __future__ import annotations

import hashlib
import json

import numpy as np
import pytest
import torch

import cases
import oracle
from conftest import GOLDEN

ATTN = np.load(GOLDEN / "attention.npz")


@pytest.mark.parametrize("case", cases.attention_cases(), ids=lambda c: c.name)
def test_attention_matches_reference(case):
    assert str(ATTN[f"{case.name}.digest"]) == case.digest(), "seeded inputs changed: regenerate the fixtures"
    meta = oracle.build_metadata(case.seqs, case.bs)
    k_pool, v_pool = case.k_pool.clone(), case.v_pool.clone()
    out = oracle.forward(case.q, case.k, case.v, k_pool, v_pool, meta)
    expected = torch.from_numpy(ATTN[f"{case.name}.out"])
    torch.testing.assert_close(out, expected, atol=1e-6, rtol=1e-6)
    # the rows landed where slot_mapping says, nothing else changed
    flat_k = k_pool.view(-1, case.hkv, case.dh)
    assert torch.equal(flat_k[meta.slot_mapping], case.k)
    untouched = torch.ones(flat_k.shape[0], dtype=torch.bool)
    untouched[meta.slot_mapping] = False
    assert torch.equal(flat_k[untouched], case.k_pool.view(-1, case.hkv, case.dh)[untouched])


def test_append_cast_bits_match_reference():
    g = np.load(GOLDEN / "append_cast.npz")
    x = cases.cast_rows()
    assert str(g["rows.digest"]) == hashlib.sha256(x.numpy().tobytes()).hexdigest()
    slots = torch.from_numpy(g["slots"])
    n, hkv, dh = x.shape
    for name, dt in (("bf16", torch.bfloat16), ("f16", torch.float16)):
        k_pool = torch.zeros(8, cases.BS, hkv, dh, dtype=dt)
        v_pool = torch.zeros_like(k_pool)
        oracle.write_kv(k_pool, v_pool, slots, x, -x)
        for pool, key in ((k_pool, "k_bits"), (v_pool, "v_bits")):
            bits = pool.view(-1, hkv, dh)[slots].view(torch.int16).numpy().view(np.uint16)
            np.testing.assert_array_equal(bits, g[f"{name}.{key}"])


def test_metadata_matches_reference():
    for g in json.loads((GOLDEN / "metadata.json").read_text()):
        seqs = [(c, n, b) for c, n, b in g["seqs"]]
        if "error" in g:
            with pytest.raises(ValueError, match="can't hold"):
                oracle.build_metadata(seqs, g["block_size"])
            continue
        m = oracle.build_metadata(seqs, g["block_size"])
        for key in ("query_start_loc", "seq_lens", "positions", "slot_mapping", "block_tables", "logits_index",
                    "kv_indptr", "kv_indices", "kv_last_page_len"):
            assert getattr(m, key) == g[key], key


def test_prefix_hash_chain_matches_reference():
    g = json.loads((GOLDEN / "prefix.json").read_text())
    assert [oracle.root_hash(k).hex() for k in g["keys"]] == g["roots"]
    for c in g["chains"]:
        chain: list[bytes] = []
        oracle.extend_chain(chain, oracle.root_hash(g["keys"][c["key"]]), c["tokens"], 5, 16)
        assert [h.hex() for h in chain] == c["chain"]
    assert oracle.block_hash(oracle.root_hash(g["keys"][0]), list(range(100, 116))).hex() == g["block_100_115"]


def test_copy_blocks_definition():
    pools = [torch.randn(10, 16, 2, 8) for _ in range(3)]
    before = [p.clone() for p in pools]
    oracle.copy_blocks(pools, [1, 5, 7], [2, 0, 9])
    for p, b in zip(pools, before):
        assert torch.equal(p[[2, 0, 9]], b[[1, 5, 7]])
        keep = [i for i in range(10) if i not in (2, 0, 9)]
        assert torch.equal(p[keep], b[keep])


def test_compact_plan_packs_live_blocks_low():
    tables = [[9, 3, 7], [1, 8], [9, 3, 4]]  # a shared prefix [9, 3]
    src, dst, new = oracle.compact_plan(tables, 12)
    live = {b for t in new for b in t}
    assert live == set(range(len(live)))  # live blocks now occupy [0, n_live)
    assert sorted(src) == src and all(s >= len(live) for s in src) and all(d < len(live) for d in dst)
    assert new[0][:2] == new[2][:2]  # the shared prefix moved once and stays shared
