"""The C-ABI library without a GPU: it loads, exports exactly what include/*.h declares, and its host-side
entry points (the planner, argument validation) behave.  No call here launches a kernel."""

from __future__ import annotations

import ctypes
import random
import re

import numpy as np
import pytest
import torch

from conftest import REPO

HEADERS = sorted((REPO / "include").glob("*.h"))


def declared_symbols() -> set[str]:
    names = set()
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"MLB_API\s+[\w\s\*]+?\b(mlb_\w+)\s*\(", text))
    return names


@pytest.fixture(scope="module")
def L(mlb):
    from importlib import import_module

    return import_module(mlb.__name__ + "._lib")


def test_library_exports_every_declared_symbol(L):
    declared = declared_symbols()
    assert declared, "no MLB_API declarations found"
    lib = L.lib()
    for name in declared:
        assert hasattr(lib, name), name
    assert declared == set(L.EXPORTS)
    assert lib.mlb_abi_version() == L.ABI_VERSION == 10


def test_plan_record_layouts_match_header(L):
    assert ctypes.sizeof(L.WorkUnit) == 32 and ctypes.sizeof(L.SharedUnit) == 32 and ctypes.sizeof(L.ShareMember) == 16
    assert ctypes.sizeof(L.OutTargets) == 24 + 8 * L.MAX_OUT_DESTS


def test_output_targets_and_peer_calls_validate_on_the_host(L, mlb):
    lib = L.lib()
    fake = 1 << 20  # never dereferenced: every call below is refused before a launch
    for n, dests in ((0, []), (9, [fake] * 8), (2, [fake, None])):
        t = L.OutTargets()
        t.num_dests = n
        for i, d in enumerate(dests):
            t.dests[i] = d
        rc = lib.mlb_splitk_reduce(fake, fake, 4, fake, fake, 2, 4, 8, 64, None, 0, 0, 2, ctypes.byref(t), None)
        assert rc == L.MLB_EINVAL and "out_targets" in L.last_error()
    rc = lib.mlb_splitk_reduce(fake, fake, 4, fake, fake, 2, 4, 8, 64, None, 0, 0, 2, None, None)
    assert rc == L.MLB_EINVAL and "null out" in L.last_error()
    with pytest.raises(ValueError, match="destinations"):
        mlb.ops.out_targets([fake] * 9, 0, 1, 1)
    flags = (ctypes.c_void_p * 8)(*([fake] * 8))
    for rank, world in ((0, 0), (0, 9), (2, 2), (-1, 2)):
        rc = lib.mlb_peer_barrier(flags, rank, world, fake, 0, None, None)
        assert rc == L.MLB_EINVAL and "rank" in L.last_error()
    assert lib.mlb_peer_barrier(flags, 0, 2, None, 0, None, None) == L.MLB_EINVAL
    assert lib.mlb_peer_barrier(flags, 0, 2, fake, -1, None, None) == L.MLB_EINVAL
    flags[1] = None
    rc = lib.mlb_peer_barrier(flags, 0, 2, fake, 0, None, None)
    assert rc == L.MLB_EINVAL and "null" in L.last_error()
    t = mlb.ops.out_targets([fake, fake], 0, 8, 1)
    red = lambda tg, self_dest: lib.mlb_splitk_reduce_gather(fake, fake, 4, fake, fake, 2, 4, 8, 64, 2, tg,
                                                             self_dest, None)
    assert red(None, 0) == L.MLB_EINVAL and "null out_targets" in L.last_error()
    assert red(ctypes.byref(t), 2) == L.MLB_EINVAL and "self_dest" in L.last_error()
    assert red(ctypes.byref(t), -1) == L.MLB_EINVAL
    p = ctypes.c_void_p()
    assert lib.mlb_ipc_alloc(0, ctypes.byref(p), ctypes.create_string_buffer(64)) == L.MLB_EINVAL
    assert lib.mlb_ipc_open(None, ctypes.byref(p)) == L.MLB_EINVAL
    assert lib.mlb_ipc_close(None) == L.MLB_OK and lib.mlb_ipc_free(None) == L.MLB_OK


def test_invalid_arguments_return_status_without_launching(L):
    lib = L.lib()
    # unknown dtype, null pointers: rejected on the host with a message
    rc = lib.mlb_kv_append(None, None, 7, 10, 16, None, None, 0, 0, None, 0, 0, 2, 1, 2, 64, None, None)
    assert rc == L.MLB_EINVAL and "dtype" in L.last_error()
    rc = lib.mlb_kv_append(None, None, 2, 10, 16, None, None, 0, 0, None, 0, 0, 2, 1, 2, 64, None, None)
    assert rc == L.MLB_EINVAL and "null" in L.last_error()
    rc = lib.mlb_paged_attention(None, 0, 0, None, None, 2, 10, 32, 8, 2, 64, 0.1, None, 0, None, None, 1, None, 1,
                                 None, 0, None, None, None, 0, None, 0, 0, None, None, None)
    assert rc == L.MLB_EUNSUPPORTED and "block_size" in L.last_error()
    rc = lib.mlb_paged_attention(None, 0, 0, None, None, 2, 10, 16, 32, 2, 64, 0.1, None, 0, None, None, 1, None, 1,
                                 None, 0, None, None, None, 0, None, 0, 0, None, None, None)
    assert rc == L.MLB_EUNSUPPORTED and "query heads per KV head" in L.last_error()
    rc = lib.mlb_block_copy(None, 2, 10, 100, None, None, 3, None, None)
    assert rc == L.MLB_EUNSUPPORTED
    rc = lib.mlb_paged_attention(None, 0, 0, None, None, 2, 10, 8, 8, 2, 64, 0.1, None, 0, None, None, 1, None, 1,
                                 None, 0, None, None, None, 0, None, 0, 0, None, None, None)
    with pytest.raises(ValueError, match="block_size"):  # status codes become the reference's ValueError
        L.check(rc, "paged_attention")
    # zero work is a successful no-op
    assert lib.mlb_block_copy(None, 0, 10, 64, None, None, 0, None, None) == L.MLB_OK


def test_noalloc_rejects_row_counts_that_would_wrap_the_size_check(L):
    """A huge split-K row count must be refused before its byte total is computed: rows x 32 heads x 129
    floats x 4 B for rows = 2^60 wraps a 64-bit size to a small number.  Refused on the host, no launch."""
    lib = L.lib()
    for rows in (1 << 60, (1 << 63) - 1, L.NOALLOC_SCRATCH_BYTES):
        rc = lib.mlb_paged_attention_noalloc(None, 0, 0, None, None, 2, 10, 16, 32, 8, 128, 0.1, None, 0, None,
                                             None, 1, None, 1, None, 0, None, rows, None, None, 1, None, 0, 0,
                                             None, None)
        assert rc == L.MLB_ENOSPACE and "static array" in L.last_error(), rows
    rc = lib.mlb_paged_attention_noalloc(None, 0, 0, None, None, 2, 10, 16, 30, 8, 128, 0.1, None, 0, None, None, 1,
                                         None, 1, None, 0, None, 4, None, None, 1, None, 0, 0, None, None)
    assert rc == L.MLB_EINVAL  # 30 query heads do not group over 8 KV heads


def test_fused_append_validates_on_the_host(L, mlb):
    lib = L.lib()
    fake = 1 << 20  # never dereferenced: every call below is refused before a launch
    assert ctypes.sizeof(L.AppendRows) == 64

    def call(rows, dtype=2, dh=128):
        return lib.mlb_paged_attention_append(fake, 0, 0, fake, fake, dtype, 10, 16, 32, 8, dh, 0.1, fake, 0, fake,
                                              fake, 1, fake, 1, None, 0, None, None, None, 0, fake, 0, 0, None,
                                              rows, None, None)

    def rows(**kw):
        r = L.AppendRows()
        r.k, r.v, r.slot_mapping, r.num_tokens = fake, fake, fake, 1
        r.k_stride_tok, r.k_stride_head, r.v_stride_tok, r.v_stride_head = 1024, 128, 1024, 128
        for name, val in kw.items():
            setattr(r, name, val)
        return ctypes.byref(r)

    assert call(None) == L.MLB_EINVAL and "null append" in L.last_error()
    assert call(rows(slot_mapping=None)) == L.MLB_EINVAL
    assert call(rows(num_tokens=-1)) == L.MLB_EINVAL
    assert call(rows(), dtype=0) == L.MLB_EUNSUPPORTED and "16-bit" in L.last_error()
    assert call(rows(), dh=256) == L.MLB_EUNSUPPORTED
    for bad in (dict(k=fake + 2), dict(v_stride_head=129), dict(k_stride_tok=1028)):
        assert call(rows(**bad)) == L.MLB_EINVAL and "16-byte" in L.last_error()


def test_build_metadata_validates_on_the_host(L):
    lib = L.lib()
    fake = 1 << 20  # never dereferenced: every call below is refused before a launch (or does nothing)
    call = lambda *a: lib.mlb_build_metadata(*a, None)
    assert call(fake, 10, 2, 3, 4, 8, 0, fake, fake) == L.MLB_EINVAL and "bad sizes" in L.last_error()
    assert call(fake, -1, 2, 3, 4, 8, 16, fake, fake) == L.MLB_EINVAL
    assert call(fake, 10, 2, 1 << 31, 4, 8, 16, fake, fake) == L.MLB_EINVAL and "2^31" in L.last_error()
    assert call(None, 10, 2, 3, 4, 8, 16, fake, fake) == L.MLB_EINVAL and "null" in L.last_error()
    assert call(None, 0, 0, 0, 0, 0, 16, None, None) == L.MLB_OK  # no sequences: nothing to do


def test_can_fuse_append_conditions(mlb):
    """The plan / tensor half of the fused-append condition (the metadata half is append_private)."""
    ops = mlb.ops
    pool = torch.zeros(64, 16, 8, 128, dtype=torch.bfloat16)
    plan_dec = mlb.plan_attention([0, 1, 2], [40, 70], 8, 32, 8, "cpu")
    k = torch.zeros(2, 8, 128, dtype=torch.bfloat16)
    assert ops.can_fuse_append(plan_dec, pool, k, k)
    assert ops.can_fuse_append(plan_dec, pool, torch.zeros(2, 24, 128, dtype=torch.bfloat16)[:, 8:16], k)  # a view
    assert not ops.can_fuse_append(plan_dec, pool, k.float(), k)  # k / v must be in the pools' dtype
    assert not ops.can_fuse_append(plan_dec, pool.float(), k.float(), k.float())  # f32 pools
    assert not ops.can_fuse_append(plan_dec, pool, k[:1], k[:1])  # not the plan's token count
    assert not ops.can_fuse_append(plan_dec, pool, torch.zeros(2, 8, 132, dtype=torch.bfloat16)[..., :128], k)
    # a row of >= 16 new tokens becomes query-tile units with host tables: those launches need the append first
    tables = np.arange(16, dtype=np.int32).reshape(2, 8)
    plan_pre = mlb.plan_attention([0, 1, 21], [40, 70], 8, 32, 8, "cpu", block_tables_host=tables)
    k21 = torch.zeros(21, 8, 128, dtype=torch.bfloat16)
    assert not ops.can_fuse_append(plan_pre, pool, k21, k21)
    plan_pre_nt = mlb.plan_attention([0, 1, 21], [40, 70], 8, 32, 8, "cpu")  # no tables: 8-column tiles
    assert ops.can_fuse_append(plan_pre_nt, pool, k21, k21)


def plan(mlb, steps, h=32, hkv=8, ppu=0, sms=148, width=None):
    qo = [0]
    lens = []
    for cached, new in steps:
        qo.append(qo[-1] + new)
        lens.append(cached + new)
    width = width or max(-(-n // 16) for n in lens)
    return mlb.plan_attention(qo, lens, width, h, hkv, "cpu", num_sms=sms, pages_per_unit=ppu), qo, lens


@pytest.mark.parametrize("seed", range(6))
@pytest.mark.parametrize("h,hkv,ppu", [(32, 8, 0), (32, 8, 3), (8, 2, 1), (8, 8, 0), (16, 2, 2), (12, 4, 5)])
def test_planner_covers_every_page_once(mlb, seed, h, hkv, ppu):
    r = random.Random(seed)
    steps = [(r.randint(0, 3000), r.choice([1, 1, 1, r.randint(1, 40)])) for _ in range(r.randint(1, 20))]
    p, qo, lens = plan(mlb, steps, h, hkv, ppu)
    g = h // hkv
    tpt = max(1, 8 // g)
    assert p.tokens_per_tile == tpt
    u = p.units_host
    sizes = u[:, 3] - u[:, 2]
    assert (np.diff(sizes) <= 0).all(), "largest units first"
    # per (seq, tile) the units tile the pages the tile's last query can see, exactly once
    cover: dict[tuple[int, int], list[tuple[int, int, int]]] = {}
    for seq, tile, pb, pe, prow, *_ in u.tolist():
        cover.setdefault((seq, tile), []).append((pb, pe, prow))
    for s, (cached, new) in enumerate(steps):
        for t in range(-(-new // tpt)):
            last = min((t + 1) * tpt, new) - 1
            pages = -(-(cached + last + 1) // 16)
            got = sorted(cover.pop((s, t)))
            assert got[0][0] == 0 and got[-1][1] == pages
            assert all(a[1] == b[0] for a, b in zip(got, got[1:]))
            if len(got) == 1:
                assert got[0][2] == -1
            else:
                rows = [x[2] for x in got]
                assert rows == [rows[0] + c * tpt for c in range(len(got))]
                for i in range(min(tpt, new - t * tpt)):
                    tok = qo[s] + t * tpt + i
                    assert p.reduce_chunks_host[tok] == len(got)
    assert not cover


def test_planner_rejects_a_table_that_cannot_hold_the_context(mlb):
    with pytest.raises(ValueError, match="can't hold"):
        plan(mlb, [(40, 1)], width=2)
    with pytest.raises(ValueError, match="multiple"):
        plan(mlb, [(4, 1)], h=6, hkv=4)


def test_planner_auto_split_targets_waves_of_ctas(mlb):
    # 64 decode rows, context U[512, 4096]: enough units for several waves on 148 SMs
    r = random.Random(0)
    steps = [(r.randint(512, 4096) - 1, 1) for _ in range(64)]
    p, _, _ = plan(mlb, steps)
    ctas = p.num_units * 8
    assert 148 * 3 <= ctas <= 148 * 3 * 4
    assert p.num_partial_rows > 0


@pytest.mark.parametrize("hkv", [1, 2, 4, 8])
def test_planner_fills_about_one_and_a_half_waves_with_equal_rows(mlb, hkv):
    """Rows of one length (29 x 8192 pages, one rank of KV-head sharding at 8 / 4 / 2 / 1
    heads): every row gets the same number of units and the CTAs fill ~1.55 waves of 3 per SM, so the last
    wave is more than half full (a thin last wave measured up to 20% slower)."""
    steps = [(131071, 1)] * 29
    p, _, _ = plan(mlb, steps, h=4 * hkv, hkv=hkv)
    per_row = np.bincount(p.units_host[:, 0], minlength=29)
    assert len(set(per_row.tolist())) == 1
    waves = p.num_units * hkv / (148 * 3)
    assert 1.5 <= waves <= 1.7


def test_planner_uses_fewer_longer_units_when_the_step_is_small(mlb):
    """Under 64 page-heads per CTA slot (config 2's 64 rows at one or two KV heads per GPU) the split aims at
    ~0.55 waves: per-CTA start-up and split-K rows cost more than the parallelism buys."""
    r = random.Random(0)
    steps = [(r.randint(512, 4096) - 1, 1) for _ in range(64)]
    for hkv in (1, 2):
        p, _, _ = plan(mlb, steps, h=4 * hkv, hkv=hkv)
        assert 0.45 <= p.num_units * hkv / (148 * 3) <= 0.8
    p8, _, _ = plan(mlb, steps, h=32, hkv=8)
    assert p8.num_units * 8 / (148 * 3) >= 1.3  # a large step keeps >= 1.3 waves


def test_planner_finds_shared_prefixes(mlb):
    """Decode rows whose tables start with the same blocks get shared-prefix units over those pages; their
    own units start after the prefix, and the pieces line up with the partial rows."""
    r = random.Random(1)
    shared = list(range(1000, 1040))  # 40 shared full blocks
    steps, tables = [], []
    for i in range(20):  # 20 rows share the prefix; suffixes differ
        ctx = 40 * 16 + r.randint(1, 300)
        steps.append((ctx - 1, 1))
        tables.append(shared + [5000 + 100 * i + j for j in range(-(-ctx // 16) - 40)])
    for i in range(3):  # 3 rows share only their first block with them: not enough to count
        steps.append((700, 1))
        tables.append([1000] + [8000 + 100 * i + j for j in range(-(-701 // 16) - 1)])
    steps.append((500, 7))  # a multi-token row is never a member
    tables.append(shared + [9000 + j for j in range(-(-507 // 16) - 40)])
    width = max(len(t) for t in tables)
    host = np.zeros((len(tables), width), dtype=np.int32)
    for i, t in enumerate(tables):
        host[i, :len(t)] = t
    qo = [0]
    for _, n in steps:
        qo.append(qo[-1] + n)
    lens = [c + n for c, n in steps]
    p = mlb.plan_attention(qo, lens, width, 32, 8, "cpu", num_sms=148, block_tables_host=host)
    assert p.num_shared_units > 0
    members = p.members_host
    assert sorted(members[:, 0].tolist()) == list(range(20))
    su = p.shared_host
    pieces = sorted({(int(x[2]), int(x[3]), int(x[4])) for x in su})
    assert pieces[0][0] == 0 and pieces[-1][1] == 40 and all(a[1] == b[0] for a, b in zip(pieces, pieces[1:]))
    npieces = len(pieces)
    assert_pairs(su)
    for mb, mc, pb, pe, piece, tseq, *_ in su.tolist():
        assert 0 <= mc <= 128 // 4 and tseq in range(20)  # one unit: at most 128 query columns (0: empty partner)
        assert (pe - pb) % 8 == 0 or pe == 40  # pieces are whole 8-page (128-key) tiles but the last
    per_member = {m: 0 for m in range(len(members))}
    for mb, mc, *_ in su.tolist():
        for m in range(mb, mb + mc):
            per_member[m] += 1
    assert set(per_member.values()) == {npieces}  # each member: every shared piece exactly once
    units = p.units_host
    for s in range(20):
        own = [u for u in units.tolist() if u[0] == s]
        assert min(u[2] for u in own) == 40 and max(u[3] for u in own) == -(-lens[s] // 16)
        tok = qo[s]
        assert p.reduce_chunks_host[tok] == npieces + len(own)
        base = int(members[list(members[:, 0]).index(s), 2])
        assert p.reduce_rows_host[tok] == base
        assert sorted(u[4] for u in own) == [base + (npieces + c) * 2 for c in range(len(own))]
    for s in range(20, len(steps)):  # the rest plan as usual, from page 0
        assert min(u[2] for u in units.tolist() if u[0] == s) == 0
    plain = mlb.plan_attention(qo, lens, width, 32, 8, "cpu", num_sms=148)
    assert plain.num_shared_units == 0


def assert_pairs(su: np.ndarray) -> None:
    """Shared units come in pairs (2i, 2i + 1) over the same pages, table row, piece and kind, ordered largest
    first as whole pairs; a pair's second unit may be empty, its first never is."""
    assert su.shape[0] % 2 == 0
    a, b = su[0::2], su[1::2]
    assert (a[:, 2:6] == b[:, 2:6]).all() and ((a[:, 6] & 0xFF) == (b[:, 6] & 0xFF)).all()
    assert (a[:, 1] > 0).all() and (b[:, 1] >= 0).all()
    sizes = a[:, 3] - a[:, 2]
    assert (np.diff(sizes) <= 0).all()


def _prefix_step(suffix_lo: int, suffix_hi: int, rows: int = 128, prefix_pages: int = 512, seed: int = 0):
    """BASELINE config 4's shape: `rows` decode rows sharing `prefix_pages` full pages, own suffixes."""
    r = random.Random(seed)
    prefix = list(range(prefix_pages))
    nxt, lens, tables = prefix_pages + 1, [], []
    for _ in range(rows):
        ctx = prefix_pages * 16 + r.randint(suffix_lo, suffix_hi) + 1
        own = -(-ctx // 16) - prefix_pages
        tables.append(prefix + list(range(nxt, nxt + own)))
        nxt += own
        lens.append(ctx)
    host = np.zeros((rows, max(len(t) for t in tables)), dtype=np.int32)
    for i, t in enumerate(tables):
        host[i, :len(t)] = t
    return list(range(rows + 1)), lens, host


EXPECTED_SHARED_CTAS = {"config4": 96, "tiny": 128, "long": 32}  # CTAs = blocks x KV heads x pieces


def test_planner_balances_shared_ctas_against_private_work(mlb):
    """The shared-prefix kernel runs beside the per-sequence kernel, one CTA per SM: the planner gives it the
    share of the SMs that balances the two (config 4: 3 pieces x 4 row blocks x 8 KV heads = 96 CTAs, the
    measured best of 64 / 96 / 128), every SM when the rows have almost no pages of their own, and fewer as
    their own pages grow.  Every shared page stays covered once per member whatever the piece count."""
    ctas = {}
    for name, lo, hi in (("config4", 64, 512), ("tiny", 0, 15), ("long", 512, 2048)):
        qo, lens, host = _prefix_step(lo, hi)
        p = mlb.plan_attention(qo, lens, host.shape[1], 32, 8, "cpu", num_sms=148, block_tables_host=host)
        su = p.shared_host
        assert_pairs(su)
        ctas[name] = p.num_shared_units // 2 * 8  # one CTA per pair of units and KV head
        pieces = sorted({(int(x[2]), int(x[3])) for x in su})
        assert pieces[0][0] == 0 and pieces[-1][1] == 512 and all(a[1] == b[0] for a, b in zip(pieces, pieces[1:]))
        assert ctas[name] <= 148
    assert ctas == EXPECTED_SHARED_CTAS


@pytest.mark.parametrize("h,hkv", [(32, 8), (8, 8), (16, 2), (12, 4)])
def test_planner_makes_query_tiles_for_prefill_rows(mlb, h, hkv):
    """With host tables, rows of >= 16 new tokens become kind-1 query tiles of 128 / group tokens over the
    keys their last token sees, split in pieces of <= 128 pages with token-major partial rows; shorter rows
    keep 8-column work units."""
    g = h // hkv
    tpt = max(1, 8 // g)
    tile = 128 // g
    steps = [(0, 40), (300, 70), (3000, 33), (500, 1), (100, 15), (2400, 16)]
    qo, lens = [0], []
    for c, n in steps:
        qo.append(qo[-1] + n)
        lens.append(c + n)
    width = max(-(-n // 16) for n in lens)
    host = np.arange(len(steps) * width, dtype=np.int32).reshape(len(steps), width)
    p = mlb.plan_attention(qo, lens, width, h, hkv, "cpu", block_tables_host=host)
    su = p.shared_host
    assert_pairs(su)
    kind1 = [u for u in su.tolist() if (u[6] & 0xFF) == 1]
    prefill = {s for s, (c, n) in enumerate(steps) if n >= 16}
    assert {u[5] for u in kind1} == prefill
    assert not any(u[0] in prefill for u in p.units_host.tolist()), "prefill rows get no 8-column units"
    covered = {}
    pair_pages = {}
    for i in range(0, len(kind1), 2):  # a pair covers the keys its later tile's last token sees
        (fa, na, *_), (fb, nb, _, _, _, seq, *_) = kind1[i], kind1[i + 1]
        c = steps[seq][0]
        pair_pages[(seq, fa - qo[seq])] = -(-(c + fa - qo[seq] + na + nb) // 16)
    for first, ntok, pb, pe, piece, seq, kp, base in kind1:
        if ntok == 0:
            continue  # an empty partner
        c, n = steps[seq]
        assert 1 <= ntok <= tile and qo[seq] <= first and first + ntok <= qo[seq + 1]
        t0 = first - qo[seq]
        lead = t0 - t0 % (2 * tile)
        pages = pair_pages[(seq, lead)]
        pieces = kp >> 8
        covered.setdefault((seq, t0), []).append((pb, pe, piece, pieces, base, ntok, pages))
        assert 0 <= pb < pe <= pages
        if pieces == 1:
            assert piece == -1 and (pb, pe) == (0, pages)
        else:
            assert 0 <= piece < pieces and pe - pb <= 128
            for i in range(ntok):
                tok = first + i
                assert p.reduce_chunks_host[tok] == pieces
                assert p.reduce_rows_host[tok] == base + i * pieces * tpt
                assert base + ((i * pieces) + pieces - 1) * tpt < p.num_partial_rows
    for (seq, t0), parts in covered.items():
        parts.sort()
        c, n = steps[seq]
        assert parts[0][0] == 0 and parts[-1][1] == parts[0][6]
        assert parts[-1][1] >= -(-(c + t0 + parts[0][5]) // 16)  # at least the keys the tile's last token sees
        assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
    for s in prefill:  # every token of a prefill row is in exactly one tile
        n = steps[s][1]
        starts = sorted(t0 for (seq, t0) in covered if seq == s)
        assert starts == list(range(0, n, tile))
    plain = mlb.plan_attention(qo, lens, width, h, hkv, "cpu")
    assert plain.num_shared_units == 0  # without host tables: 8-column units for every row
