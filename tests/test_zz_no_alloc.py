"""mlb_paged_attention_noalloc: paged attention for callers that cannot allocate device memory when they
attend (an engine that gave nearly all free memory to the KV pool at start-up, or a serving loop outside
PyTorch with no device allocator).  Its split-K scratch is a static device array inside the library, so the
call allocates nothing.

Checked through the C ABI, call after call on the one shared array: every output must equal the allocating
entry point's bit for bit (same kernels, same plan) and the fp32 oracle within the north star's max-abs
bar.  The plans cover split decode rows, a mixed ragged step, and shared-prefix plus query-tile units (the
tensor-core kernel's partial rows in the static array too).  A plan too big for the array must be refused
before anything runs.

Collected last on purpose (file name), so a run that stops at the first failure has run everything else."""

from __future__ import annotations

import math
import random
from importlib import import_module

import numpy as np
import pytest
import torch

import cases
from paged_helpers import assert_close, device_case, oracle_forward

pytestmark = pytest.mark.gpu


def _noalloc(L, q, k_pool, v_pool, meta, plan, out, err):
    nb, bs, hkv, dh = k_pool.shape
    code = {torch.bfloat16: L.MLB_BF16, torch.float16: L.MLB_F16}[q.dtype]
    return L.lib().mlb_paged_attention_noalloc(
        q.data_ptr(), q.stride(0), q.stride(1), k_pool.data_ptr(), v_pool.data_ptr(), code, nb, bs, q.shape[1],
        hkv, dh, 1.0 / math.sqrt(dh), meta.block_tables_i32.data_ptr(), meta.block_tables_i32.stride(0),
        meta.seq_lens_i32.data_ptr(), meta.qo_indptr.data_ptr(), len(meta.seq_lens), plan.units.data_ptr(),
        plan.num_units, plan.shared_units.data_ptr(), plan.num_shared_units, plan.members.data_ptr(),
        plan.num_partial_rows, plan.reduce_rows.data_ptr(), plan.reduce_chunks.data_ptr(),
        q.shape[0], out.data_ptr(), out.stride(0), out.stride(1), err.data_ptr(),
        torch.cuda.current_stream().cuda_stream)


def _shared_and_prefill_case(h=32, hkv=8, dh=128):
    """Decode rows behind a 24-page shared prefix (shared-prefix units) plus two multi-token rows (query
    tiles; the 3000-token context splits into pieces)."""
    r = random.Random(17)
    nb = 900
    ids = list(range(nb))
    r.shuffle(ids)
    prefix, nxt = ids[:24], 24
    steps, blocks = [], []
    for _ in range(20):
        ctx = len(prefix) * 16 + r.randint(1, 60)
        own = -(-ctx // 16) - len(prefix)
        steps.append((ctx - 1, 1))
        blocks.append(prefix + ids[nxt:nxt + own])
        nxt += own
    for c, n in ((3000, 40), (200, 17)):
        need = -(-(c + n) // 16)
        steps.append((c, n))
        blocks.append(ids[nxt:nxt + need])
        nxt += need
    ntok = sum(n for _, n in steps)
    gen = np.random.default_rng(23)
    return cases.PagedCase("shared_prefill", h, hkv, dh, 16, steps, blocks, *(
        torch.from_numpy(gen.standard_normal(shape, dtype=np.float32))
        for shape in ((ntok, h, dh), (ntok, hkv, dh), (ntok, hkv, dh), (nb, 16, hkv, dh), (nb, 16, hkv, dh))))


def _step(mlb, L, case, dtype, cuda, err, host_tables, pages_per_unit=0):
    t = device_case(case, dtype, cuda)
    meta = mlb.AttentionMetadata.build([mlb.SeqStep(c, n, list(b)) for c, n, b in case.seqs], 16, cuda)
    mlb.kv_append(t["k_pool"], t["v_pool"], meta.slot_mapping, t["k"], t["v"])
    plan = mlb.plan_attention(meta.query_start_loc, meta.seq_lens, meta.block_tables_i32.shape[1], case.h, case.hkv,
                              cuda, pages_per_unit=pages_per_unit,
                              block_tables_host=meta.block_tables_host if host_tables else None)
    assert plan.num_partial_rows > 0  # the static array is used
    expected = mlb.paged_attention(t["q"], t["k_pool"], t["v_pool"], meta.block_tables_i32, meta.seq_lens_i32,
                                   meta.qo_indptr, plan, mlb.Workspace())
    got = torch.full_like(t["q"], float("nan"))
    rc = _noalloc(L, t["q"], t["k_pool"], t["v_pool"], meta, plan, got, err)
    assert rc == L.MLB_OK, L.last_error()
    torch.cuda.synchronize()
    assert int(err.item()) == 0, f"{case.name}: device fault flags {int(err.item())}"
    return got, expected, plan


def test_noalloc_equals_the_allocating_entry_point_call_after_call(mlb, cuda):
    L = import_module(mlb.__name__ + "._lib")
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    steps = [(cases.llama_decode(21, 4, 512, 4096), torch.bfloat16, False, 3),
             (cases.mixed_step(4, 32, 8, 128), torch.bfloat16, False, 2),
             (_shared_and_prefill_case(), torch.bfloat16, True, 0),
             (_shared_and_prefill_case(), torch.float16, True, 0),
             (cases.llama_decode(21, 4, 512, 4096), torch.bfloat16, False, 3)]  # after the array held others
    kinds = set()
    for case, dtype, host_tables, ppu in steps:
        got, expected, plan = _step(mlb, L, case, dtype, cuda, err, host_tables, ppu)
        assert torch.equal(got, expected), f"{case.name} {dtype}: differs from the allocating entry point"
        assert_close(got, oracle_forward(case, dtype)[0], dtype)
        kinds |= {int(k) & 0xFF for k in plan.shared_host[:, 6]}
    assert kinds == {0, 1}  # shared-prefix units and query tiles both ran through the static array


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
