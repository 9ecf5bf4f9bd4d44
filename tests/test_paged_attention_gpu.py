"""K2a/K2b paged attention on the GPU against the fp32 oracle (paged_torch_ref.py:40-74): every golden case
in fp32 / bf16 / fp16, forced split-K, head dims 64 / 128 / 256, poisoned and NaN-filled junk, range
faults, and BASELINE configs 2 and 5 at full size checked on a sample of their sequences."""

from __future__ import annotations

import random

import numpy as np
import pytest
import torch

import cases
import oracle
from conftest import GOLDEN
from paged_helpers import TOL, assert_close, device_case, oracle_forward

pytestmark = pytest.mark.gpu

DTYPES = [torch.float32, torch.bfloat16, torch.float16]
ATTN = np.load(GOLDEN / "attention.npz")


def run_backend(mlb, case, dtype, dev, ppu=0, err=None):
    t = device_case(case, dtype, dev)
    meta = mlb.AttentionMetadata.build([mlb.SeqStep(c, n, list(b)) for c, n, b in case.seqs], case.bs, dev)
    backend = mlb.B200Backend(pages_per_unit=ppu)
    out = backend.forward(t["q"], t["k"], t["v"], t["k_pool"], t["v_pool"], meta)
    return out, t, backend


@pytest.mark.parametrize("dtype", DTYPES, ids=str)
@pytest.mark.parametrize("case", cases.attention_cases(), ids=lambda c: c.name)
def test_golden_cases(mlb, cuda, case, dtype):
    out, t, _ = run_backend(mlb, case, dtype, cuda)
    expected, k_after, v_after = oracle_forward(case, dtype)
    assert_close(out, expected, dtype)
    assert torch.equal(t["k_pool"].cpu(), k_after) and torch.equal(t["v_pool"].cpu(), v_after)
    if dtype == torch.float32:  # straight against the reference's own output
        assert_close(out, torch.from_numpy(ATTN[f"{case.name}.out"]), dtype)


@pytest.mark.parametrize("dtype", DTYPES, ids=str)
@pytest.mark.parametrize("ppu", [1, 2, 5])
def test_forced_split_k_matches(mlb, cuda, dtype, ppu):
    ws = mlb.Workspace()  # shared across cases and calls
    for case in (cases.llama_decode(21, 4, 512, 4096), cases.mixed_step(), cases.boundaries(6, 32, 8, 128)):
        t = device_case(case, dtype, cuda)
        meta = mlb.AttentionMetadata.build([mlb.SeqStep(c, n, list(b)) for c, n, b in case.seqs], case.bs, cuda)
        mlb.kv_append(t["k_pool"], t["v_pool"], meta.slot_mapping, t["k"], t["v"])
        plan = mlb.plan_attention(meta.query_start_loc, meta.seq_lens, meta.block_tables_i32.shape[1], case.h,
                                  case.hkv, cuda, pages_per_unit=ppu)
        assert plan.num_partial_rows > 0
        expected = oracle_forward(case, dtype)[0]
        for _ in range(2):
            out = mlb.paged_attention(t["q"], t["k_pool"], t["v_pool"], meta.block_tables_i32, meta.seq_lens_i32,
                                      meta.qo_indptr, plan, ws)
            assert_close(out, expected, dtype)


@pytest.mark.parametrize("dtype", DTYPES, ids=str)
@pytest.mark.parametrize("h,hkv,dh", [(8, 2, 256), (16, 16, 64), (24, 8, 128), (7, 7, 128)])
def test_head_shapes(mlb, cuda, dtype, h, hkv, dh):
    case = cases.make_case(f"shape_{h}_{hkv}_{dh}", 99, h, hkv, dh, [(70, 1), (0, 9), (200, 3), (31, 1)], 40)
    for ppu in (0, 2):
        out, _, _ = run_backend(mlb, case, dtype, cuda, ppu=ppu)
        assert_close(out, oracle_forward(case, dtype)[0], dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32], ids=str)
def test_nan_junk_past_the_context_does_not_leak(mlb, cuda, dtype):
    case = cases.make_case("nan_junk", 5, 8, 2, 128, [(20, 1), (40, 1), (5, 3)], 24)
    meta = oracle.build_metadata(case.seqs, case.bs)
    used = torch.zeros(24 * 16, dtype=torch.bool)
    used[meta.slot_mapping] = True
    for (cached, _), blocks in zip(case.steps, case.blocks):
        for p in range(cached):
            used[blocks[p // 16] * 16 + p % 16] = True
    # The reference's batched decode gathers every row to the longest context and lets SDPA weight the
    # masked tail by 0, and 0 * NaN = NaN: with non-finite junk it returns NaN for the shorter rows.  The
    # kernels read only each sequence's own tokens, so the answer is the oracle's on zeroed junk.
    expected = oracle_forward(case, dtype)[0]
    for pool in (case.k_pool, case.v_pool):
        pool.view(-1, case.hkv, case.dh)[~used] = float("nan")
    out, _, _ = run_backend(mlb, case, dtype, cuda, ppu=1)
    assert torch.isfinite(out).all()
    assert_close(out, expected, dtype)


def test_out_of_range_block_ids_are_flagged_not_read(mlb, cuda):
    case = cases.make_case("bad_ids", 8, 8, 2, 128, [(40, 1), (10, 1)], 16)
    t = device_case(case, torch.bfloat16, cuda)
    meta = mlb.AttentionMetadata.build([mlb.SeqStep(c, n, list(b)) for c, n, b in case.seqs], 16, cuda)
    meta.block_tables_i32[0, 1] = 1 << 20  # far outside the 16-block pool
    backend = mlb.B200Backend(check_errors=True)
    with pytest.raises(Exception, match="block id out of range"):
        backend.forward(t["q"], t["k"], t["v"], t["k_pool"], t["v_pool"], meta)
    # the other sequence is unaffected
    out = mlb.B200Backend().forward(t["q"], t["k"], t["v"], t["k_pool"], t["v_pool"], meta)
    torch.cuda.synchronize()
    assert_close(out[1:], oracle_forward(case, torch.bfloat16)[0][1:], torch.bfloat16)


def _subset_check(mlb, dev, steps, blocks, q, k, v, k_pool, v_pool, sample, dtype):
    """Run the full step on the GPU, then check `sample` sequences against the oracle on the CPU.  Sequences
    are independent, so the oracle needs only the sampled sequence's pages (copied out after the step's
    write, which the append tests check bit for bit) to attend over."""
    meta = mlb.AttentionMetadata.build([mlb.SeqStep(c, n, b) for (c, n), b in zip(steps, blocks)], 16, dev)
    out = mlb.B200Backend().forward(q, k, v, k_pool, v_pool, meta)
    torch.cuda.synchronize()
    starts = meta.query_start_loc
    for s in sample:
        ids = torch.tensor(blocks[s], device=dev)
        kp, vp = k_pool[ids].cpu(), v_pool[ids].cpu()
        om = oracle.build_metadata([(steps[s][0], steps[s][1], list(range(len(blocks[s]))))], 16)
        rows = slice(starts[s], starts[s + 1])
        flat = kp.view(-1, kp.shape[2], kp.shape[3])
        assert torch.equal(flat[om.slot_mapping], k[rows].cpu())  # the new rows landed
        exp = oracle.paged_attention(q[rows].cpu(), kp, vp, om)
        assert_close(out[rows], exp, dtype)


def test_config2_full_size_sampled(mlb, cuda):
    """bf16, H 32 / Hkv 8 / Dh 128, batch 64, context U[512, 4096], pool 1.25x."""
    r = np.random.default_rng(2)
    ctx = r.integers(512, 4097, size=64)
    need = int(sum(-(-int(c) // 16) for c in ctx))
    nb = int(need * 1.25)
    perm = r.permutation(nb).tolist()
    blocks = [[perm.pop() for _ in range(-(-int(c) // 16))] for c in ctx]
    steps = [(int(c) - 1, 1) for c in ctx]
    g = torch.Generator(device=cuda).manual_seed(0)
    k_pool = (torch.randn(nb, 16, 8, 128, device=cuda, generator=g) * 0.5).to(torch.bfloat16)
    v_pool = (torch.randn(nb, 16, 8, 128, device=cuda, generator=g) * 0.5).to(torch.bfloat16)
    q = torch.randn(64, 32, 128, device=cuda, generator=g).to(torch.bfloat16)
    k = (torch.randn(64, 8, 128, device=cuda, generator=g) * 0.5).to(torch.bfloat16)
    v = (torch.randn(64, 8, 128, device=cuda, generator=g) * 0.5).to(torch.bfloat16)
    _subset_check(mlb, cuda, steps, blocks, q, k, v, k_pool, v_pool, random.Random(0).sample(range(64), 6),
                  torch.bfloat16)


def test_config5_full_size_sampled(mlb, cuda):
    """BASELINE config 5 at one GPU: 32 sequences x 131072 tokens, bf16, H 32 / Hkv 8 / Dh 128 (17 GB of
    pool per K and V); two sequences are checked against the oracle."""
    ctx, b = 131072, 32
    pages = ctx // 16
    nb = b * pages + 64
    perm = torch.randperm(nb, generator=torch.Generator().manual_seed(5)).tolist()
    blocks = [perm[i * pages:(i + 1) * pages] for i in range(b)]
    steps = [(ctx - 1, 1)] * b
    g = torch.Generator(device=cuda).manual_seed(1)
    k_pool = torch.empty(nb, 16, 8, 128, device=cuda, dtype=torch.bfloat16).normal_(generator=g)
    v_pool = torch.empty(nb, 16, 8, 128, device=cuda, dtype=torch.bfloat16).normal_(generator=g)
    q = torch.randn(b, 32, 128, device=cuda, generator=g).to(torch.bfloat16)
    k = torch.randn(b, 8, 128, device=cuda, generator=g).to(torch.bfloat16)
    v = torch.randn(b, 8, 128, device=cuda, generator=g).to(torch.bfloat16)
    _subset_check(mlb, cuda, steps, blocks, q, k, v, k_pool, v_pool, [3, 30], torch.bfloat16)
    del k_pool, v_pool
    torch.cuda.empty_cache()


def test_tolerances_are_the_north_star():
    assert TOL[torch.bfloat16] == 2e-2 and TOL[torch.float32] == 1e-5


@pytest.mark.parametrize("tc", [1, 0], ids=["tcgen05", "mma_sync"])
@pytest.mark.parametrize("rows_a", [18, 45])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=str)
@pytest.mark.parametrize("h,hkv,dh", [(32, 8, 128), (8, 8, 64), (16, 2, 128), (8, 1, 256), (12, 4, 64)])
def test_shared_prefix_units_match_oracle(mlb, cuda, dtype, h, hkv, dh, rows_a, tc):
    """Rows whose tables share leading blocks (prefix-cache hits) are attended through shared-prefix units
    (one page load per block of rows) plus their own pages; results must equal the oracle's.  Both kernels
    of the shared units: tcgen05 (128-column tiles; head_dim 64 / 128) and mma.sync (every head_dim); 45
    rows need two units of 128 columns at GQA 4, and the 9-page prefix ends in a partial 128-key tile."""
    lib = mlb._lib.lib()
    prev = lib.mlb_set_tensor_core_prefix(tc)
    try:
        _shared_prefix_case(mlb, cuda, dtype, h, hkv, dh, rows_a)
    finally:
        lib.mlb_set_tensor_core_prefix(prev)


def _shared_prefix_case(mlb, cuda, dtype, h, hkv, dh, rows_a):
    r = random.Random(h * 100 + dh)
    nb = 1200
    ids = list(range(nb))
    r.shuffle(ids)
    shared_a, shared_b = ids[:24], ids[24:33]  # two prefixes: 24 and 9 full pages
    nxt = 33
    steps, blocks = [], []
    for i in range(rows_a + 9):
        prefix = shared_a if i < rows_a else shared_b
        ctx = len(prefix) * 16 + r.randint(1, 70)
        own = -(-ctx // 16) - len(prefix)
        steps.append((ctx - 1, 1))
        blocks.append(prefix + ids[nxt:nxt + own])
        nxt += own
    steps.append((40, 3))  # a multi-token row that starts with the same blocks: planned on its own
    blocks.append(shared_a[:3])
    case = cases.PagedCase("shared", h, hkv, dh, 16, steps, blocks, *(
        torch.from_numpy(np.random.default_rng(9).standard_normal(shape, dtype=np.float32))
        for shape in ((sum(n for _, n in steps), h, dh), (sum(n for _, n in steps), hkv, dh),
                      (sum(n for _, n in steps), hkv, dh), (nb, 16, hkv, dh), (nb, 16, hkv, dh))))
    t = device_case(case, dtype, cuda)
    meta = mlb.AttentionMetadata.build([mlb.SeqStep(c, n, list(b)) for c, n, b in case.seqs], 16, cuda)
    backend = mlb.B200Backend()
    out = backend.forward(t["q"], t["k"], t["v"], t["k_pool"], t["v_pool"], meta)
    assert backend._plan.num_shared_units > 0 and len(backend._plan.members_host) == rows_a + 9
    assert_close(out, oracle_forward(case, dtype)[0], dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=str)
def test_shared_prefix_multi_tile_units_repeatable(mlb, cuda, dtype):
    """tcgen05 shared units of 2 and 3 key tiles (prefixes of 9, 10, 17 and 24 pages): five runs give
    bit-identical outputs, equal to the oracle's.  The output rows may only be read once the last tile's
    P . V is done; a wait that an earlier tile's MMA could satisfy shows here as run-to-run differences."""
    lib = mlb._lib.lib()
    prev = lib.mlb_set_tensor_core_prefix(1)
    try:
        h, hkv, dh = 32, 8, 128
        r = random.Random(5)
        nb = 900
        ids = list(range(nb))
        r.shuffle(ids)
        steps, blocks, nxt = [], [], 0
        for plen in (9, 10, 17, 24):
            prefix = ids[nxt:nxt + plen]
            nxt += plen
            for _ in range(6):
                ctx = plen * 16 + r.randint(1, 40)
                own = -(-ctx // 16) - plen
                steps.append((ctx - 1, 1))
                blocks.append(prefix + ids[nxt:nxt + own])
                nxt += own
        ntok = len(steps)
        gen = np.random.default_rng(21)
        case = cases.PagedCase("multi_tile", h, hkv, dh, 16, steps, blocks, *(
            torch.from_numpy(gen.standard_normal(shape, dtype=np.float32))
            for shape in ((ntok, h, dh), (ntok, hkv, dh), (ntok, hkv, dh), (nb, 16, hkv, dh), (nb, 16, hkv, dh))))
        t = device_case(case, dtype, cuda)
        meta = mlb.AttentionMetadata.build([mlb.SeqStep(c, n, list(b)) for c, n, b in case.seqs], 16, cuda)
        backend = mlb.B200Backend()
        outs = []
        for _ in range(5):
            k_pool, v_pool = t["k_pool"].clone(), t["v_pool"].clone()  # each run appends its own k / v
            outs.append(backend.forward(t["q"], t["k"], t["v"], k_pool, v_pool, meta).clone())
        assert backend._plan.num_shared_units >= 4
        assert max(int(u[3]) - int(u[2]) for u in backend._plan.shared_host) > 8  # a unit of several tiles
        for o in outs[1:]:
            assert torch.equal(o, outs[0])
        assert_close(outs[0], oracle_forward(case, dtype)[0], dtype)
    finally:
        lib.mlb_set_tensor_core_prefix(prev)


@pytest.mark.parametrize("tc", [1, 0], ids=["tcgen05", "mma_sync"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=str)
@pytest.mark.parametrize("h,hkv,dh", [(32, 8, 128), (8, 8, 64), (16, 2, 128), (8, 1, 256), (12, 4, 64)])
def test_prefill_query_tiles_match_oracle(mlb, cuda, dtype, h, hkv, dh, tc):
    """Multi-token rows of >= 16 tokens (prefill chunks on cache) run as 128-column query tiles with a causal
    mask per column (paged_torch_ref.py:61-73), on fresh and cached contexts, split in pieces on a long
    context, next to short rows and decode rows.  The slots past every sequence's end in its last page hold
    NaN on the device: they must not reach the output (the oracle sees finite values there)."""
    lib = mlb._lib.lib()
    prev = lib.mlb_set_tensor_core_prefix(tc)
    try:
        steps = [(0, 40), (300, 70), (3000, 33), (500, 1), (100, 15), (2400, 16), (37, 129)]
        r = random.Random(h * 7 + dh)
        nb = 700
        ids = list(range(nb))
        r.shuffle(ids)
        blocks, nxt = [], 0
        for c, n in steps:
            need = -(-(c + n) // 16)
            blocks.append(ids[nxt:nxt + need])
            nxt += need
        ntok = sum(n for _, n in steps)
        gen = np.random.default_rng(11)
        case = cases.PagedCase("prefill", h, hkv, dh, 16, steps, blocks, *(
            torch.from_numpy(gen.standard_normal(shape, dtype=np.float32))
            for shape in ((ntok, h, dh), (ntok, hkv, dh), (ntok, hkv, dh), (nb, 16, hkv, dh), (nb, 16, hkv, dh))))
        t = device_case(case, dtype, cuda)
        for (c, n), b in zip(steps, blocks):  # junk past the end of each context
            rest = (c + n) % 16
            if rest:
                t["k_pool"][b[-1], rest:] = float("nan")
                t["v_pool"][b[-1], rest:] = float("nan")
        meta = mlb.AttentionMetadata.build([mlb.SeqStep(c, n, list(b)) for c, n, b in case.seqs], 16, cuda)
        backend = mlb.B200Backend(check_errors=True)
        out = backend.forward(t["q"], t["k"], t["v"], t["k_pool"], t["v_pool"], meta)
        kinds = backend._plan.shared_host[:, 6] & 0xFF
        assert (kinds == 1).sum() > 0, "prefill rows must run as query tiles"
        assert ((backend._plan.shared_host[:, 6] >> 8) > 1).any(), "the long context must split in pieces"
        assert torch.isfinite(out).all()
        assert_close(out, oracle_forward(case, dtype)[0], dtype)
    finally:
        lib.mlb_set_tensor_core_prefix(prev)
