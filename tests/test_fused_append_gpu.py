"""The append fused into the attention launch (mlb_paged_attention_append): the reference's forward writes
the step's k/v rows, then attends (attention/torch_ref.py:46-48); the fused launch must give the same pools
bit for bit, the same outputs bit for bit as kv_append + attention, and the oracle's outputs within the
tolerance.  Covers decode rows (new token first / last in its page), short multi-token rows split over
several query tiles, split-K pieces, shared-prefix members, NaN junk past every context end, and an
out-of-range block id."""

from __future__ import annotations

import importlib
import random

import numpy as np
import pytest
import torch

import cases
from paged_helpers import assert_close, bits, device_case, oracle_forward

pytestmark = pytest.mark.gpu

STEPS = [(15, 1), (16, 1), (100, 5), (31, 2), (0, 7), (47, 15), (0, 15), (3000, 1), (1200, 3), (255, 1)]


def _case(h, hkv, dh, steps, nb, seed, prefix_pages=0, sharers=0):
    """A PagedCase whose blocks are a seeded shuffle; the first `sharers` rows start with the same
    `prefix_pages` blocks (a prefix-cache hit) and append into their own pages."""
    r = random.Random(seed)
    ids = list(range(nb))
    r.shuffle(ids)
    prefix, nxt = ids[:prefix_pages], prefix_pages
    blocks = []
    for i, (c, n) in enumerate(steps):
        need = -(-(c + n) // 16)
        head = prefix if i < sharers else []
        blocks.append(head + ids[nxt:nxt + need - len(head)])
        nxt += need - len(head)
    ntok = sum(n for _, n in steps)
    gen = np.random.default_rng(seed)
    return cases.PagedCase("fused", h, hkv, dh, 16, steps, blocks, *(
        torch.from_numpy(gen.standard_normal(shape, dtype=np.float32))
        for shape in ((ntok, h, dh), (ntok, hkv, dh), (ntok, hkv, dh), (nb, 16, hkv, dh), (nb, 16, hkv, dh))))


def _junk_past_ends(case, t):
    """NaN in every slot past a context's end in its last page (the oracle keeps the finite values)."""
    for (c, n), b in zip(case.steps, case.blocks):
        rest = (c + n) % 16
        if rest:
            t["k_pool"][b[-1], rest:] = float("nan")
            t["v_pool"][b[-1], rest:] = float("nan")


def _both(mlb, monkeypatch, t, meta, **kw):
    """(output, k pool, v pool, backend) with the separate append and with the fused launch; the fused run
    fails if it launches kv_append."""
    runs = []
    for fuse in (False, True):
        kp, vp = t["k_pool"].clone(), t["v_pool"].clone()
        backend = mlb.B200Backend(fuse_append=fuse, **kw)
        if fuse:
            mod = importlib.import_module(mlb.__name__ + ".attention.backend")

            def no_separate_append(*a, **k):
                raise AssertionError("the fused path launched kv_append")

            monkeypatch.setattr(mod, "kv_append", no_separate_append)
        out = backend.forward(t["q"], t["k"], t["v"], kp, vp, meta)
        monkeypatch.undo()
        runs.append((out, kp, vp, backend))
    return runs


def _check(runs, case, dtype):
    (out_s, kp_s, vp_s, _), (out_f, kp_f, vp_f, _) = runs
    assert torch.equal(bits(kp_f), bits(kp_s)) and torch.equal(bits(vp_f), bits(vp_s))
    assert torch.equal(out_f, out_s)
    expected, ref_k, ref_v = oracle_forward(case, dtype)
    assert_close(out_f, expected, dtype)
    # every written slot holds the row (the rest of the pool is the input's, junk included)
    new_k = torch.cat([torch.as_tensor(case.k)]).to(dtype)
    meta_slots = [b[p // 16] * 16 + p % 16 for (c, n), b in zip(case.steps, case.blocks) for p in range(c, c + n)]
    flat = kp_f.view(-1, *kp_f.shape[2:]).cpu()
    assert torch.equal(bits(flat[meta_slots]), bits(new_k))


@pytest.mark.parametrize("ppu", [0, 3], ids=["auto_split", "split_3"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=str)
@pytest.mark.parametrize("h,hkv,dh", [(32, 8, 128), (8, 2, 64), (16, 2, 128), (12, 4, 64), (8, 8, 64)])
def test_fused_append_equals_append_then_attend(mlb, cuda, monkeypatch, h, hkv, dh, dtype, ppu):
    case = _case(h, hkv, dh, STEPS, 420, seed=h + dh)
    t = device_case(case, dtype, cuda)
    _junk_past_ends(case, t)
    meta = mlb.AttentionMetadata.build([mlb.SeqStep(c, n, list(b)) for c, n, b in case.seqs], 16, cuda)
    assert meta.append_private
    runs = _both(mlb, monkeypatch, t, meta, pages_per_unit=ppu)
    plan = runs[1][3]._plan
    assert plan.num_units > len(STEPS)  # split-K pieces and several query tiles per row
    _check(runs, case, dtype)


@pytest.mark.parametrize("tc", [1, 0], ids=["tcgen05", "mma_sync"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=str)
def test_fused_append_with_shared_prefix_units(mlb, cuda, monkeypatch, dtype, tc):
    """Decode rows that share 20 prefix blocks (planned as shared-prefix units) each append into a page
    of their own: the fused launch writes from the rows' own units."""
    lib = mlb._lib.lib()
    prev = lib.mlb_set_tensor_core_prefix(tc)
    try:
        r = random.Random(7)
        steps = [(20 * 16 + r.randint(0, 90), 1) for _ in range(40)] + [(500, 1), (33, 4)]
        case = _case(32, 8, 128, steps, 900, seed=17, prefix_pages=20, sharers=40)
        t = device_case(case, dtype, cuda)
        _junk_past_ends(case, t)
        meta = mlb.AttentionMetadata.build([mlb.SeqStep(c, n, list(b)) for c, n, b in case.seqs], 16, cuda)
        assert meta.append_private
        runs = _both(mlb, monkeypatch, t, meta)
        assert runs[1][3]._plan.num_shared_units > 0
        _check(runs, case, dtype)
    finally:
        lib.mlb_set_tensor_core_prefix(prev)


def test_written_block_read_by_another_row_is_not_fused(mlb, cuda, monkeypatch):
    """A row appends into a block that another row's context also holds: the other row must see the new
    values (write, then attend), so the backend keeps the separate append launch."""
    steps = [(40, 3), (60, 1)]
    blocks = [[5, 9, 11], [5, 9, 11, 2]]  # row 0 writes block 11 (positions 40-42), row 1 reads it
    gen = np.random.default_rng(3)
    case = cases.PagedCase("shared_write", 8, 2, 64, 16, steps, blocks, *(
        torch.from_numpy(gen.standard_normal(shape, dtype=np.float32))
        for shape in ((4, 8, 64), (4, 2, 64), (4, 2, 64), (16, 16, 2, 64), (16, 16, 2, 64))))
    t = device_case(case, torch.bfloat16, cuda)
    meta = mlb.AttentionMetadata.build([mlb.SeqStep(c, n, list(b)) for c, n, b in case.seqs], 16, cuda)
    assert not meta.append_private
    backend = mlb.B200Backend()
    calls = []
    mod = importlib.import_module(mlb.__name__ + ".attention.backend")
    real = mod.kv_append
    monkeypatch.setattr(mod, "kv_append", lambda *a, **k: (calls.append(1), real(*a, **k))[1])
    out = backend.forward(t["q"], t["k"], t["v"], t["k_pool"], t["v_pool"], meta)
    assert calls == [1]
    assert_close(out, oracle_forward(case, torch.bfloat16)[0], torch.bfloat16)


def test_fused_append_flags_an_out_of_range_block_like_the_separate_append(mlb, cuda, monkeypatch):
    """A block id past the pool's end in a row's last page: the separate append skips the write and flags
    the slot, the attention treats the page as empty and flags the id; the fused launch does both."""
    steps = [(20, 1), (70, 1)]
    blocks = [[3, 1], [4, 7, 6, 9, 16 + 5]]  # the second row's last page is past the pool (16 blocks)
    gen = np.random.default_rng(4)
    case = cases.PagedCase("bad_id", 8, 2, 64, 16, steps, blocks, *(
        torch.from_numpy(gen.standard_normal(shape, dtype=np.float32))
        for shape in ((2, 8, 64), (2, 2, 64), (2, 2, 64), (16, 16, 2, 64), (16, 16, 2, 64))))
    t = device_case(case, torch.bfloat16, cuda)
    meta = mlb.AttentionMetadata.build([mlb.SeqStep(c, n, list(b)) for c, n, b in case.seqs], 16, cuda)
    assert meta.append_private
    faults, pools = [], []
    for fuse in (False, True):
        kp, vp = t["k_pool"].clone(), t["v_pool"].clone()
        backend = mlb.B200Backend(check_errors=True, fuse_append=fuse)
        with pytest.raises(mlb.DeviceFault) as e:
            backend.forward(t["q"], t["k"], t["v"], kp, vp, meta)
        faults.append(str(e.value))
        pools.append((kp, vp))
    assert faults[0] == faults[1] and "slot out of range" in faults[0] and "block id out of range" in faults[0]
    for a, b in zip(pools[0], pools[1]):
        assert torch.equal(bits(a), bits(b))


def test_fused_append_in_a_cuda_graph(mlb, cuda):
    """The fused launch replays inside a CUDA graph (the decode step engines capture), step after step."""
    case = _case(32, 8, 128, [(c, 1) for c in (30, 400, 1000, 64, 2047)], 300, seed=5)
    t = device_case(case, torch.bfloat16, cuda)
    meta = mlb.AttentionMetadata.build([mlb.SeqStep(c, n, list(b)) for c, n, b in case.seqs], 16, cuda)
    backend = mlb.B200Backend()
    kp, vp = t["k_pool"].clone(), t["v_pool"].clone()
    out = backend.forward(t["q"], t["k"], t["v"], kp, vp, meta)  # warm-up: plan, workspace
    torch.cuda.synchronize()
    kp2, vp2 = t["k_pool"].clone(), t["v_pool"].clone()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out_g = backend.forward(t["q"], t["k"], t["v"], kp2, vp2, meta)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out_g, out) and torch.equal(bits(kp2), bits(kp)) and torch.equal(bits(vp2), bits(vp))
