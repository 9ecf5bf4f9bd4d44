"""mlb_paged_attention_noalloc: paged attention for callers that cannot allocate device memory when they
attend (an engine that gave nearly all free memory to the KV pool at start-up, or a serving loop outside
PyTorch with no device allocator).  Its split-K scratch is a static device array inside the library, so the
call allocates nothing.  Checked through the C ABI against the allocating entry point on two calls in a row
(the shared array keeps the first call's contents, which must not leak into the second), and a plan too big
for the array must be refused before anything runs.

Collected last on purpose (file name), so a run that stops at the first failure has run everything else."""

from __future__ import annotations

import math
from importlib import import_module

import pytest
import torch

import cases
from paged_helpers import TOL, device_case

pytestmark = pytest.mark.gpu


def _noalloc(L, q, k_pool, v_pool, meta, plan, out, err):
    nb, bs, hkv, dh = k_pool.shape
    return L.lib().mlb_paged_attention_noalloc(
        q.data_ptr(), q.stride(0), q.stride(1), k_pool.data_ptr(), v_pool.data_ptr(), L.MLB_BF16, nb, bs, q.shape[1],
        hkv, dh, 1.0 / math.sqrt(dh), meta.block_tables_i32.data_ptr(), meta.block_tables_i32.stride(0),
        meta.seq_lens_i32.data_ptr(), meta.qo_indptr.data_ptr(), len(meta.seq_lens), plan.units.data_ptr(),
        plan.num_units, plan.shared_units.data_ptr(), plan.num_shared_units, plan.members.data_ptr(),
        plan.num_partial_rows, plan.reduce_rows.data_ptr(), plan.reduce_chunks.data_ptr(),
        q.shape[0], out.data_ptr(), out.stride(0), out.stride(1), err.data_ptr(),
        torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_the_allocating_entry_point_twice(mlb, cuda):
    L = import_module(mlb.__name__ + "._lib")
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    for call, case in enumerate((cases.llama_decode(21, 4, 512, 4096), cases.mixed_step(4, 32, 8, 128))):
        t = device_case(case, torch.bfloat16, cuda)
        meta = mlb.AttentionMetadata.build([mlb.SeqStep(c, n, list(b)) for c, n, b in case.seqs], 16, cuda)
        mlb.kv_append(t["k_pool"], t["v_pool"], meta.slot_mapping, t["k"], t["v"])
        plan = mlb.plan_attention(meta.query_start_loc, meta.seq_lens, meta.block_tables_i32.shape[1], case.h,
                                  case.hkv, cuda, pages_per_unit=3)
        assert 0 < plan.num_partial_rows
        expected = mlb.paged_attention(t["q"], t["k_pool"], t["v_pool"], meta.block_tables_i32, meta.seq_lens_i32,
                                       meta.qo_indptr, plan, mlb.Workspace())
        got = torch.full_like(t["q"], float("nan"))
        rc = _noalloc(L, t["q"], t["k_pool"], t["v_pool"], meta, plan, got, err)
        assert rc == L.MLB_OK, L.last_error()
        torch.cuda.synchronize()
        torch.testing.assert_close(got.float(), expected.float(), atol=TOL[torch.bfloat16], rtol=TOL[torch.bfloat16])
        assert int(err.item()) == 0, f"call {call}: device fault flags {int(err.item())}"


def test_noalloc_refuses_a_plan_larger_than_its_scratch(mlb, cuda):
    L = import_module(mlb.__name__ + "._lib")
    case = cases.llama_decode(21, 4, 512, 4096)
    t = device_case(case, torch.bfloat16, cuda)
    meta = mlb.AttentionMetadata.build([mlb.SeqStep(c, n, list(b)) for c, n, b in case.seqs], 16, cuda)
    plan = mlb.plan_attention(meta.query_start_loc, meta.seq_lens, meta.block_tables_i32.shape[1], case.h, case.hkv,
                              cuda, pages_per_unit=1)
    need = plan.num_partial_rows * case.h * (case.dh + 1) * 4
    assert need > L.NOALLOC_SCRATCH_BYTES
    out = torch.zeros_like(t["q"])
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    rc = _noalloc(L, t["q"], t["k_pool"], t["v_pool"], meta, plan, out, err)
    assert rc == L.MLB_ENOSPACE and "static array" in L.last_error()
    torch.cuda.synchronize()
    assert int(torch.count_nonzero(out).item()) == 0  # refused before anything ran
