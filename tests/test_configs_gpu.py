"""BASELINE configs 3 and 4 at full size on the GPU (the workloads bench.py measures), checked against the
oracle on a sample of sequences: config 3's varlen append of 8 prefill chunks into a fragmented pool must
land bit-exactly and its lognormal decode rows must attend within tolerance; config 4's copy-on-write of the
shared partial block must leave the shared blocks intact, and the 128 sequences attending over the shared
prefix must match the oracle."""

from __future__ import annotations

import random

import pytest
import torch

import bench
import oracle
from paged_helpers import assert_close

pytestmark = pytest.mark.gpu


def _pools(nb, dev, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    k = torch.empty(nb, 16, 8, 128, device=dev, dtype=torch.bfloat16).normal_(generator=g)
    v = torch.empty(nb, 16, 8, 128, device=dev, dtype=torch.bfloat16).normal_(generator=g)
    return k, v, g


def _check_rows(mlb, dev, wl, k_pool, v_pool, q, out, sample):
    """The sampled decode rows against the oracle over their own pages (copied after the step's write)."""
    for s in sample:
        c, n, blocks = wl.attend_rows[s]
        used = blocks[:-(-(c + n) // 16)]
        ids = torch.tensor(used, device=dev)
        om = oracle.build_metadata([(c, n, list(range(len(used))))], 16)
        exp = oracle.paged_attention(q[s:s + 1].cpu(), k_pool[ids].cpu(), v_pool[ids].cpu(), om)
        assert_close(out[s:s + 1], exp, torch.bfloat16)


def test_config3_mixed_step_full_size(mlb, cuda):
    wl = bench.config3()
    k_pool, v_pool, g = _pools(wl.num_blocks, cuda, 3)
    n_app = sum(n for _, n, _ in wl.append_rows)
    k = torch.randn(n_app, 8, 128, device=cuda, generator=g).to(torch.bfloat16)
    v = torch.randn(n_app, 8, 128, device=cuda, generator=g).to(torch.bfloat16)
    q = torch.randn(len(wl.attend_rows), 32, 128, device=cuda, generator=g).to(torch.bfloat16)
    meta_app = mlb.AttentionMetadata.build([mlb.SeqStep(*r) for r in wl.append_rows], 16, cuda)
    meta_att = mlb.AttentionMetadata.build([mlb.SeqStep(*r) for r in wl.attend_rows], 16, cuda)
    mlb.kv_append(k_pool, v_pool, meta_app.slot_mapping, k, v)
    # every appended row (decode tokens and the ~8.7K prefill-chunk tokens) landed at its slot
    flat = k_pool.view(-1, 8, 128)
    assert torch.equal(flat[meta_app.slot_mapping], k)
    assert torch.equal(v_pool.view(-1, 8, 128)[meta_app.slot_mapping], v)
    plan = mlb.plan_attention(meta_att.query_start_loc, meta_att.seq_lens, meta_att.block_tables_i32.shape[1], 32, 8,
                              cuda)
    out = mlb.paged_attention(q, k_pool, v_pool, meta_att.block_tables_i32, meta_att.seq_lens_i32, meta_att.qo_indptr,
                              plan, mlb.Workspace())
    torch.cuda.synchronize()
    longest = max(range(256), key=lambda i: wl.attend_rows[i][0])
    sample = sorted(set(random.Random(3).sample(range(256), 6)) | {longest})
    _check_rows(mlb, cuda, wl, k_pool, v_pool, q, out, sample)


def test_config4_prefix_sharing_with_cow_full_size(mlb, cuda):
    wl = bench.config4()
    k_pool, v_pool, g = _pools(wl.num_blocks, cuda, 4)
    shared = wl.attend_rows[0][2][:bench.CONFIG4_PREFIX // 16]
    before_k = k_pool[torch.tensor(shared, device=cuda)].clone()
    partial = wl.copy_src[0]
    src = torch.tensor(wl.copy_src, dtype=torch.int32, device=cuda)
    dst = torch.tensor(wl.copy_dst, dtype=torch.int32, device=cuda)
    mlb.ops.block_copy(mlb.ops.pool_pointer_table([k_pool, v_pool]), k_pool, src, dst)
    for d in wl.copy_dst[:5]:
        assert torch.equal(k_pool[d], k_pool[partial]) and torch.equal(v_pool[d], v_pool[partial])
    n = len(wl.attend_rows)
    q = torch.randn(n, 32, 128, device=cuda, generator=g).to(torch.bfloat16)
    k = torch.randn(n, 8, 128, device=cuda, generator=g).to(torch.bfloat16)
    v = torch.randn(n, 8, 128, device=cuda, generator=g).to(torch.bfloat16)
    meta = mlb.AttentionMetadata.build([mlb.SeqStep(*r) for r in wl.attend_rows], 16, cuda)
    out = mlb.B200Backend().forward(q, k, v, k_pool, v_pool, meta)
    torch.cuda.synchronize()
    # the shared full blocks were read by 128 sequences and written by none
    assert torch.equal(k_pool[torch.tensor(shared, device=cuda)], before_k)
    _check_rows(mlb, cuda, wl, k_pool, v_pool, q, out, random.Random(4).sample(range(n), 5))
