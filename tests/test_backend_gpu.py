"""B200Backend as a drop-in AttentionBackend, in the shape of the reference's own kernel tests
(tests/test_kernels.py:29-72: a mixed ragged step and a decode-only step, pool writes bit-identical,
outputs within 2e-2), plus plan reuse across layers and a multi-step decode loop."""

from __future__ import annotations

import random

import pytest
import torch

import oracle
from paged_helpers import assert_close

pytestmark = pytest.mark.gpu


def mixed_step(mlb, dev, h=8, hkv=2, dh=128, bs=16, dtype=torch.bfloat16):
    """tests/test_kernels.py:29-48: fresh prompt, decode, prompt on top of cache, 1-token prompt, decode."""
    torch.manual_seed(0)
    steps = [(0, 37), (90, 1), (40, 25), (0, 1), (300, 1)]
    k_pool = torch.randn(64, bs, hkv, dh, device=dev, dtype=dtype)
    v_pool = torch.randn_like(k_pool)
    free = list(range(64))
    random.Random(3).shuffle(free)
    seqs = []
    for cached, new in steps:
        n = cached + new
        seqs.append(mlb.SeqStep(cached, new, [free.pop() for _ in range(-(-n // bs))]))
    meta = mlb.AttentionMetadata.build(seqs, bs, dev)
    n = meta.query_start_loc[-1]
    q = torch.randn(n, h, dh, device=dev, dtype=dtype)
    k = torch.randn(n, hkv, dh, device=dev, dtype=dtype)
    v = torch.randn(n, hkv, dh, device=dev, dtype=dtype)
    return q, k, v, k_pool, v_pool, meta, seqs


def reference(q, k, v, k_pool, v_pool, seqs):
    om = oracle.build_metadata([(s.num_cached, s.num_new, s.block_ids) for s in seqs], 16)
    kp, vp = k_pool.cpu(), v_pool.cpu()
    out = oracle.forward(q.cpu(), k.cpu(), v.cpu(), kp, vp, om)
    return out, kp, vp


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=str)
def test_backend_matches_reference_on_a_mixed_step(mlb, cuda, dtype):
    q, k, v, k_pool, v_pool, meta, seqs = mixed_step(mlb, cuda, dtype=dtype)
    expected, ref_k, ref_v = reference(q, k, v, k_pool, v_pool, seqs)
    backend = mlb.get_backend("b200")
    got = backend.forward(q, k, v, k_pool, v_pool, meta)
    assert torch.equal(k_pool.cpu(), ref_k) and torch.equal(v_pool.cpu(), ref_v)  # identical writes
    assert got.dtype == q.dtype and got.shape == q.shape
    assert_close(got, expected, dtype)


def test_backend_on_a_decode_only_step(mlb, cuda):
    q, k, v, k_pool, v_pool, _, _ = mixed_step(mlb, cuda)
    seqs = [mlb.SeqStep(c, 1, list(range(i * 4, i * 4 + 4))) for i, c in enumerate([5, 63, 17])]
    meta = mlb.AttentionMetadata.build(seqs, 16, cuda)
    q, k, v = q[:3], k[:3], v[:3]
    expected, _, _ = reference(q, k, v, k_pool, v_pool, seqs)
    got = mlb.B200Backend().forward(q, k, v, k_pool, v_pool, meta)
    assert_close(got, expected, torch.bfloat16)


def test_plan_is_built_once_per_step_and_reused_by_every_layer(mlb, cuda):
    q, k, v, k_pool, v_pool, meta, seqs = mixed_step(mlb, cuda, h=32, hkv=8)
    layers = [(k_pool.clone(), v_pool.clone()) for _ in range(4)]
    backend = mlb.B200Backend()
    outs, plans = [], []
    for kp, vp in layers:
        outs.append(backend.forward(q, k, v, kp, vp, meta))
        plans.append(backend._plan)
    assert all(p is plans[0] for p in plans)
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    meta2 = mlb.AttentionMetadata.build(seqs, 16, cuda)  # a new step gets a new plan
    backend.forward(q, k, v, *layers[0], meta2)
    assert backend._plan is not plans[0]


def test_decode_loop_matches_reference_every_step(mlb, cuda):
    """Several engine steps: sequences grow one token per step, taking a new block at each boundary."""
    h, hkv, dh, nb = 32, 8, 128, 128
    g = torch.Generator(device=cuda).manual_seed(11)
    k_pool = torch.randn(nb, 16, hkv, dh, device=cuda, generator=g).to(torch.bfloat16)
    v_pool = torch.randn(nb, 16, hkv, dh, device=cuda, generator=g).to(torch.bfloat16)
    bm = mlb.BlockManager(nb, 16)
    cached = [14, 31, 1, 47, 100]
    tables = [bm.allocate(-(-c // 16)) for c in cached]
    backend = mlb.B200Backend()
    for _ in range(5):
        for i, c in enumerate(cached):
            if c + 1 > len(tables[i]) * 16:
                tables[i] += bm.allocate(1)
        seqs = [mlb.SeqStep(c, 1, list(t)) for c, t in zip(cached, tables)]
        meta = mlb.AttentionMetadata.build(seqs, 16, cuda)
        n = len(seqs)
        q = torch.randn(n, h, dh, device=cuda, generator=g).to(torch.bfloat16)
        k = torch.randn(n, hkv, dh, device=cuda, generator=g).to(torch.bfloat16)
        v = torch.randn(n, hkv, dh, device=cuda, generator=g).to(torch.bfloat16)
        expected, ref_k, _ = reference(q, k, v, k_pool, v_pool, seqs)
        got = backend.forward(q, k, v, k_pool, v_pool, meta)
        assert torch.equal(k_pool.cpu(), ref_k)
        assert_close(got, expected, torch.bfloat16)
        cached = [c + 1 for c in cached]
    bm.check(tables)


def test_forward_is_stream_ordered_without_host_syncs(mlb, cuda):
    """Everything goes on torch's current stream: running on a side stream gives the same answer."""
    q, k, v, k_pool, v_pool, meta, _ = mixed_step(mlb, cuda, h=32, hkv=8)
    kp2, vp2 = k_pool.clone(), v_pool.clone()
    base = mlb.B200Backend().forward(q, k, v, k_pool, v_pool, meta)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        got = mlb.B200Backend().forward(q, k, v, kp2, vp2, meta)
    torch.cuda.current_stream().wait_stream(side)
    assert torch.equal(got, base)


def test_programmatic_launch_changes_no_bit(mlb, cuda):
    """Every kernel with and without programmatic dependent launch: pools and outputs bit-identical over a
    4-layer chain (append -> attention -> split-K reduction, layer after layer, no host sync between)."""
    lib = mlb._lib.lib()
    results = []
    for enable in (1, 0):
        prev = lib.mlb_set_programmatic_launch(enable)
        try:
            q, k, v, k_pool, v_pool, meta, _ = mixed_step(mlb, cuda)
            pools = [(k_pool.clone(), v_pool.clone()) for _ in range(4)]
            backend = mlb.B200Backend(pages_per_unit=1)
            outs = [backend.forward(q, k, v, kp, vp, meta) for kp, vp in pools]
            torch.cuda.synchronize()
            results.append((outs, pools))
        finally:
            lib.mlb_set_programmatic_launch(prev)
    for (o1, p1), (o2, p2) in zip(zip(*results[0]), zip(*results[1])):
        assert torch.equal(o1.view(torch.int16), o2.view(torch.int16))
        assert torch.equal(p1[0], p2[0]) and torch.equal(p1[1], p2[1])


@pytest.mark.parametrize("tc", [1, 0], ids=["tcgen05", "mma_sync"])
def test_concurrent_prefix_kernel_changes_no_bit(mlb, cuda, tc):
    """mlb_set_concurrent_prefix: the shared-prefix / query-tile kernel on the library's side stream beside the
    per-sequence kernel (forked from and joined into the caller's stream) gives the same bits as the two
    launches in a row, eagerly and replayed from a CUDA graph, layer after layer."""
    lib = mlb._lib.lib()
    prev_tc, prev_cc = lib.mlb_set_tensor_core_prefix(tc), lib.mlb_set_concurrent_prefix(1)
    try:
        r = random.Random(11)
        ids = list(range(1500))
        r.shuffle(ids)
        prefix, nxt, seqs = ids[:20], 20, []
        steps = [(20 * 16 + r.randint(0, 60), 1) for _ in range(40)] + [(0, 40), (700, 33), (90, 1), (3000, 1)]
        for i, (c, n) in enumerate(steps):
            need = -(-(c + n) // 16)
            head = prefix if i < 40 else []
            seqs.append(mlb.SeqStep(c, n, head + ids[nxt:nxt + need - len(head)]))
            nxt += need - len(head)
        meta = mlb.AttentionMetadata.build(seqs, 16, cuda)
        ntok = meta.query_start_loc[-1]
        g = torch.Generator(device=cuda).manual_seed(2)
        pools = [(torch.randn(1500, 16, 8, 128, device=cuda, generator=g).to(torch.bfloat16),
                  torch.randn(1500, 16, 8, 128, device=cuda, generator=g).to(torch.bfloat16)) for _ in range(3)]
        q = torch.randn(ntok, 32, 128, device=cuda, generator=g).to(torch.bfloat16)
        k = torch.randn(ntok, 8, 128, device=cuda, generator=g).to(torch.bfloat16)
        v = torch.randn(ntok, 8, 128, device=cuda, generator=g).to(torch.bfloat16)

        def run(concurrent, graph=False):
            lib.mlb_set_concurrent_prefix(concurrent)
            backend = mlb.B200Backend()
            layers = [(kp.clone(), vp.clone()) for kp, vp in pools]
            outs = [backend.forward(q, k, v, kp, vp, meta) for kp, vp in layers]  # eager (and warm-up)
            if not graph:
                return outs
            layers = [(kp.clone(), vp.clone()) for kp, vp in pools]
            torch.cuda.synchronize()
            cg = torch.cuda.CUDAGraph()
            with torch.cuda.graph(cg):
                outs = [backend.forward(q, k, v, kp, vp, meta) for kp, vp in layers]
            cg.replay()
            cg.replay()
            torch.cuda.synchronize()
            return [o.clone() for o in outs]

        serial = run(0)
        plan = mlb.B200Backend().plan(meta, 32, 8, cuda)
        assert plan.num_shared_units > 0 and plan.num_units > 0 and plan.has_query_tiles
        for got in (run(1), run(1, graph=True)):
            for a, b in zip(got, serial):
                assert torch.equal(a, b)
    finally:
        lib.mlb_set_tensor_core_prefix(prev_tc)
        lib.mlb_set_concurrent_prefix(prev_cc)


def _reference_shaped(meta):
    """An object with exactly the reference's AttentionMetadata fields (tests/golden/interface.json, made by
    running the reference): what an unmodified reference engine hands the backend."""
    import json
    import types

    from conftest import GOLDEN

    fields = json.loads((GOLDEN / "interface.json").read_text())["metadata_fields"]
    return types.SimpleNamespace(**{f: getattr(meta, f) for f in fields})


@pytest.mark.parametrize("kind", ["decode", "shared_prefix", "mixed"])
def test_reference_metadata_object_keeps_every_fast_path(mlb, cuda, kind):
    """The reference's metadata object (no host tables, no append_private): the backend derives them once per
    step, so the plan, the fused append and therefore every bit of the pools and outputs equal the run with
    this package's metadata, over 3 layers; both within the north star's bar of the oracle.  With
    derive_host_tables off, every row runs on 8-column units and the append launches first: pools still
    bit-identical, outputs within the bar."""
    r = random.Random(5)
    ids = list(range(1200))
    r.shuffle(ids)
    if kind == "decode":
        steps = [(c, 1) for c in (17, 300, 2047, 64, 999, 5)]
        prefix = []
    elif kind == "shared_prefix":
        steps = [(30 * 16 + r.randint(0, 50), 1) for _ in range(12)]
        prefix = ids[:30]
    else:
        steps = [(0, 37), (90, 1), (40, 25), (0, 1), (300, 1), (1000, 70)]
        prefix = []
    nxt, seqs = len(prefix), []
    for c, n in steps:
        need = -(-(c + n) // 16)
        own = need - len(prefix)
        seqs.append(mlb.SeqStep(c, n, prefix + ids[nxt:nxt + own]))
        nxt += own
    meta = mlb.AttentionMetadata.build(seqs, 16, cuda)
    ntok = meta.query_start_loc[-1]
    g = torch.Generator(device=cuda).manual_seed(8)
    pools = [(torch.randn(1200, 16, 8, 128, device=cuda, generator=g).to(torch.bfloat16),
              torch.randn(1200, 16, 8, 128, device=cuda, generator=g).to(torch.bfloat16)) for _ in range(3)]
    q = torch.randn(ntok, 32, 128, device=cuda, generator=g).to(torch.bfloat16)
    k = torch.randn(ntok, 8, 128, device=cuda, generator=g).to(torch.bfloat16)
    v = torch.randn(ntok, 8, 128, device=cuda, generator=g).to(torch.bfloat16)

    def run(m, **kw):
        backend = mlb.B200Backend(**kw)
        layers = [(kp.clone(), vp.clone()) for kp, vp in pools]
        outs = [backend.forward(q, k, v, kp, vp, m) for kp, vp in layers]
        torch.cuda.synchronize()
        return backend, outs, layers

    b_own, o_own, p_own = run(meta)
    ref_meta = _reference_shaped(meta)
    b_ref, o_ref, p_ref = run(ref_meta)
    assert b_ref._plan.num_shared_units == b_own._plan.num_shared_units
    assert b_ref.last_append_fused == b_own.last_append_fused == (kind != "mixed")
    if kind == "shared_prefix":
        assert b_ref._plan.num_shared_units > 0
    for a, b in zip(o_ref, o_own):
        assert torch.equal(a, b)
    for (ka, va), (kb, vb) in zip(p_ref, p_own):
        assert torch.equal(ka, kb) and torch.equal(va, vb)
    expected, ref_k, ref_v = reference(q, k, v, pools[0][0], pools[0][1], seqs)
    assert torch.equal(p_ref[0][0].cpu(), ref_k) and torch.equal(p_ref[0][1].cpu(), ref_v)
    assert_close(o_ref[0], expected, torch.bfloat16)
    b_off, o_off, p_off = run(_reference_shaped(meta), derive_host_tables=False)
    assert b_off._plan.num_shared_units == 0 and not b_off.last_append_fused
    for (ka, va), (kb, vb) in zip(p_off, p_own):
        assert torch.equal(ka, kb) and torch.equal(va, vb)
    assert_close(o_off[0], expected, torch.bfloat16)
