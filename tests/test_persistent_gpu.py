"""mlb_set_persistent_attention: the per-sequence units on resident CTAs that take (unit, KV head) items from a
device work queue must give the one-shot kernel's results bit for bit (same plan, same per-warp arithmetic),
launch after launch (the last CTA resets the queue) and replayed from a CUDA graph; and the oracle's
within the tolerance."""

from __future__ import annotations

import importlib
import random

import numpy as np
import pytest
import torch

import cases
from paged_helpers import assert_close, bits, device_case, oracle_forward

pytestmark = pytest.mark.gpu

STEPS = [(15, 1), (16, 1), (100, 5), (31, 2), (0, 7), (47, 15), (3000, 1), (1200, 3), (255, 1), (37, 129),
         (2000, 40), (5, 1)]


def _case(h, hkv, dh, steps, nb, seed, prefix_pages=0, sharers=0):
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
    return cases.PagedCase("persistent", h, hkv, dh, 16, steps, blocks, *(
        torch.from_numpy(gen.standard_normal(shape, dtype=np.float32))
        for shape in ((ntok, h, dh), (ntok, hkv, dh), (ntok, hkv, dh), (nb, 16, hkv, dh), (nb, 16, hkv, dh))))


def _junk(case, t):
    for (c, n), b in zip(case.steps, case.blocks):
        rest = (c + n) % 16
        if rest:
            t["k_pool"][b[-1], rest:] = float("nan")
            t["v_pool"][b[-1], rest:] = float("nan")


def _run(mlb, t, meta, persistent, repeats=1, **kw):
    lib = mlb._lib.lib()
    prev = lib.mlb_set_persistent_attention(persistent)
    try:
        outs, pools = [], []
        backend = mlb.B200Backend(**kw)
        for _ in range(repeats):
            kp, vp = t["k_pool"].clone(), t["v_pool"].clone()
            outs.append(backend.forward(t["q"], t["k"], t["v"], kp, vp, meta).clone())
            pools.append((kp, vp))
        torch.cuda.synchronize()
        return outs, pools, backend
    finally:
        lib.mlb_set_persistent_attention(prev)


@pytest.mark.parametrize("ppu", [0, 3], ids=["auto_split", "split_3"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=str)
@pytest.mark.parametrize("h,hkv,dh", [(32, 8, 128), (8, 2, 64), (16, 2, 128), (12, 4, 64), (8, 1, 256)])
def test_persistent_equals_one_shot(mlb, cuda, h, hkv, dh, dtype, ppu):
    case = _case(h, hkv, dh, STEPS, 600, seed=h * 3 + dh)
    t = device_case(case, dtype, cuda)
    _junk(case, t)
    meta = mlb.AttentionMetadata.build([mlb.SeqStep(c, n, list(b)) for c, n, b in case.seqs], 16, cuda)
    want, want_pools, _ = _run(mlb, t, meta, 0, pages_per_unit=ppu)
    got, got_pools, backend = _run(mlb, t, meta, 1, repeats=3, pages_per_unit=ppu)
    for o, (kp, vp) in zip(got, got_pools):  # launch after launch: the queue starts empty every time
        assert torch.equal(o, want[0])
        assert torch.equal(bits(kp), bits(want_pools[0][0])) and torch.equal(bits(vp), bits(want_pools[0][1]))
    assert_close(got[0], oracle_forward(case, dtype)[0], dtype)


@pytest.mark.parametrize("tc", [1, 0], ids=["tcgen05", "mma_sync"])
def test_persistent_with_shared_prefix_units_and_fused_append(mlb, cuda, tc):
    lib = mlb._lib.lib()
    prev = lib.mlb_set_tensor_core_prefix(tc)
    try:
        r = random.Random(9)
        steps = [(20 * 16 + r.randint(0, 90), 1) for _ in range(40)] + [(500, 1), (33, 4), (4000, 1)]
        case = _case(32, 8, 128, steps, 1200, seed=23, prefix_pages=20, sharers=40)
        t = device_case(case, torch.bfloat16, cuda)
        _junk(case, t)
        meta = mlb.AttentionMetadata.build([mlb.SeqStep(c, n, list(b)) for c, n, b in case.seqs], 16, cuda)
        assert meta.append_private
        want, want_pools, _ = _run(mlb, t, meta, 0)
        got, got_pools, backend = _run(mlb, t, meta, 1, repeats=2)
        assert backend._plan.num_shared_units > 0
        for o, (kp, vp) in zip(got, got_pools):
            assert torch.equal(o, want[0])
            assert torch.equal(bits(kp), bits(want_pools[0][0])) and torch.equal(bits(vp), bits(want_pools[0][1]))
        assert_close(got[0], oracle_forward(case, torch.bfloat16)[0], torch.bfloat16)
    finally:
        lib.mlb_set_tensor_core_prefix(prev)


def test_persistent_flags_an_out_of_range_block(mlb, cuda):
    steps = [(20, 1), (70, 1), (300, 1)]
    # a 16-block pool; ids 21 and 25 lie past it (the second row's last page, a middle page of the third)
    blocks = [[3, 1], [4, 7, 6, 9, 21], [0, 10, 11, 12, 13, 14, 15, 2, 8, 5, 25, 0, 10, 11, 12, 13, 14, 15, 2]]
    gen = np.random.default_rng(4)
    case = cases.PagedCase("bad_id", 8, 2, 64, 16, steps, blocks, *(
        torch.from_numpy(gen.standard_normal(shape, dtype=np.float32))
        for shape in ((3, 8, 64), (3, 2, 64), (3, 2, 64), (16, 16, 2, 64), (16, 16, 2, 64))))
    t = device_case(case, torch.bfloat16, cuda)
    meta = mlb.AttentionMetadata.build([mlb.SeqStep(c, n, list(b)) for c, n, b in case.seqs], 16, cuda)
    lib = mlb._lib.lib()
    faults, outs = [], []
    for persistent in (0, 1):
        prev = lib.mlb_set_persistent_attention(persistent)
        try:
            backend = mlb.B200Backend(check_errors=True, fuse_append=False)
            kp, vp = t["k_pool"].clone(), t["v_pool"].clone()
            with pytest.raises(mlb.DeviceFault) as e:
                backend.forward(t["q"], t["k"], t["v"], kp, vp, meta)
            faults.append(str(e.value))
        finally:
            lib.mlb_set_persistent_attention(prev)
    assert faults[0] == faults[1] and "block id out of range" in faults[0]


def test_persistent_in_a_cuda_graph(mlb, cuda):
    case = _case(32, 8, 128, [(c, 1) for c in (30, 400, 1000, 64, 2047, 3000, 90, 2500, 1800)], 900, seed=5)
    t = device_case(case, torch.bfloat16, cuda)
    meta = mlb.AttentionMetadata.build([mlb.SeqStep(c, n, list(b)) for c, n, b in case.seqs], 16, cuda)
    want, _, _ = _run(mlb, t, meta, 0, pages_per_unit=4)
    lib = mlb._lib.lib()
    prev = lib.mlb_set_persistent_attention(1)
    try:
        backend = mlb.B200Backend(pages_per_unit=4)
        kp, vp = t["k_pool"].clone(), t["v_pool"].clone()
        backend.forward(t["q"], t["k"], t["v"], kp, vp, meta)  # warm-up: plan, workspace, queue address
        # more items than 2 x the resident CTAs (148 SMs x 3): CTAs move from item to item with prefetch
        assert backend._plan.num_units * 8 > 2 * 148 * 3
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            out = backend.forward(t["q"], t["k"], t["v"], kp, vp, meta)
        for _ in range(4):
            g.replay()
            torch.cuda.synchronize()
            assert torch.equal(out, want[0])
    finally:
        lib.mlb_set_persistent_attention(prev)
