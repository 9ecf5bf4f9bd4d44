"""AttentionMetadata.build on a CUDA device expands the per-token / per-page arrays and both padded block
tables on the GPU (mlb_build_metadata) from a compact upload; every field must equal the numpy build's
(which the CPU tests pin to the reference's own outputs, metadata.py:71-103) exactly."""

from __future__ import annotations

import json
import random

import numpy as np
import pytest
import torch

from conftest import GOLDEN

pytestmark = pytest.mark.gpu

TENSORS = ("positions", "slot_mapping", "block_tables", "logits_index", "qo_indptr", "seq_lens_i32",
           "block_tables_i32", "kv_indptr", "kv_indices", "kv_last_page_len")


def _same(mlb, seqs, bs, cuda):
    dev = mlb.AttentionMetadata.build(seqs, bs, cuda)
    ref = mlb.AttentionMetadata.build(seqs, bs, "cpu")
    for f in TENSORS:
        a, b = getattr(dev, f), getattr(ref, f)
        assert a.device.type == "cuda" and a.dtype == b.dtype and a.shape == b.shape, f
        assert torch.equal(a.cpu(), b), f
    assert dev.query_start_loc == ref.query_start_loc and dev.seq_lens == ref.seq_lens
    assert np.array_equal(dev.block_tables_host, ref.block_tables_host)
    assert dev.append_private == ref.append_private
    return dev


def test_device_build_matches_reference_golden(mlb, cuda):
    for g in json.loads((GOLDEN / "metadata.json").read_text()):
        if "error" in g:
            continue
        seqs = [mlb.SeqStep(c, n, b) for c, n, b in g["seqs"]]
        m = _same(mlb, seqs, g["block_size"], cuda)
        assert m.slot_mapping.tolist() == g["slot_mapping"] and m.kv_indices.tolist() == g["kv_indices"]


@pytest.mark.parametrize("seed", range(8))
def test_device_build_matches_numpy_on_random_steps(mlb, cuda, seed):
    r = random.Random(seed)
    bs = r.choice([16, 16, 4, 32])
    seqs = []
    for _ in range(r.randint(1, 60)):
        cached, new = r.randint(0, 600), r.choice([0, 1, 1, 1, r.randint(1, 90)])
        need = -(-(cached + new) // bs)
        ids = [r.randrange(-2, 20_000) for _ in range(need + r.randint(0, 4))]  # spare ids, a few invalid
        seqs.append(mlb.SeqStep(cached, new, ids))
    _same(mlb, seqs, bs, cuda)


def test_device_build_edge_cases(mlb, cuda):
    S = mlb.SeqStep
    _same(mlb, [], 16, cuda)  # no rows
    _same(mlb, [S(0, 0, [])], 16, cuda)  # an empty row
    _same(mlb, [S(3, 1, [7]), S(0, 0, []), S(0, 5, [2, 9])], 4, cuda)
    big = [(1 << 31) + 5, (1 << 33) + 1, 3]  # ids past int32: the int32 views truncate as Tensor.to does
    m = _same(mlb, [S(40, 1, big)], 16, cuda)
    assert m.block_tables.tolist() == [big] and m.append_private  # block 3, written, occurs once
    assert m.slot_mapping.tolist() == [3 * 16 + 8]
    seqs = [S(c, 1, list(range(i * 600, i * 600 + -(-(c + 1) // 16)))) for i, c in enumerate(range(0, 9000, 37))]
    _same(mlb, seqs, 16, cuda)  # 244 rows, ragged tables up to 563 wide


def test_device_build_at_config_sizes(mlb, cuda):
    import bench

    for wl in (bench.config2(), bench.config3()):
        for rows in {id(wl.attend_rows): wl.attend_rows, id(wl.append_rows): wl.append_rows}.values():
            _same(mlb, [mlb.SeqStep(c, n, b) for c, n, b in rows], 16, cuda)


def test_build_arrays_expands_on_another_stream(mlb, cuda):
    """build_arrays(expand_on=s): the upload on the current stream, the expansion kernel on s after it; every
    field equals the build without it (config 3's rows: ragged tables, multi-token rows)."""
    import bench

    rows = bench.config3(attend_chunks=True).attend_rows
    arrays = (np.array([c for c, _, _ in rows], dtype=np.int64), np.array([n for _, n, _ in rows], dtype=np.int64),
              np.concatenate([np.asarray(b, dtype=np.int64) for _, _, b in rows]),
              np.array([len(b) for _, _, b in rows], dtype=np.int64))
    plain = mlb.AttentionMetadata.build_arrays(*arrays, 16, cuda)
    side = torch.cuda.Stream(cuda)
    loader = torch.cuda.Stream(cuda)
    with torch.cuda.stream(loader):
        other = mlb.AttentionMetadata.build_arrays(*arrays, 16, cuda, expand_on=side)
    side.synchronize()
    for f in TENSORS:
        assert torch.equal(getattr(plain, f).cpu(), getattr(other, f).cpu()), f
