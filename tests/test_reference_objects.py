"""The drop-in boundary against the reference's own objects, on the CPU.

An unmodified reference engine hands a backend `minillm.attention.metadata.AttentionMetadata`, which has
only the reference's fields (metadata.py:36-52): no host block tables and no `append_private`.  The
backend then derives both with `host_view` (one device-to-host copy per step), so the shared-prefix units,
query tiles and fused append stay on.  Checked here:
- `tests/golden/interface.json` (made by running the reference) is the reference's current interface;
- `host_view` of the reference's live metadata object equals what this package's build records;
- the same on an object that carries exactly the reference's fields and nothing else (no reference
  needed), and the backend's plan from it equals the plan from this package's metadata.
The GPU half (outputs and pools through such an object) is in test_backend_gpu.py.
"""

from __future__ import annotations

import importlib
import json
import sys
import types

import numpy as np
import pytest
import torch

from conftest import GOLDEN, reference_src

REF = reference_src()
needs_reference = pytest.mark.skipif(REF is None, reason="the reference's source tree is not at hand")
FIELDS = json.loads((GOLDEN / "interface.json").read_text())


def _reference(module: str):
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    return importlib.import_module(module)


def _steps():
    """(name, [(num_cached, num_new, block_ids)]) steps of block size 16."""
    r = np.random.default_rng(4)
    ids = r.permutation(4000).tolist()
    take = lambda n: [ids.pop() for _ in range(n)]  # noqa: E731
    decode = [(c - 1, 1, take(-(-c // 16))) for c in r.integers(20, 900, size=12).tolist()]
    prefix = take(12)
    shared = [(12 * 16 + e - 1, 1, prefix + take(-(-e // 16))) for e in r.integers(1, 60, size=9).tolist()]
    mixed = decode[:3] + [(0, 37, take(3)), (300, 40, take(22)), (5, 1, take(1) + take(2))]  # spare blocks
    # two rows hold the same last block and one of them writes into it: the append is not private
    tail = take(1)
    clash = [(40, 1, prefix[:2] + tail), (39, 1, prefix[2:4] + tail)]  # slots 8 and 7 of the shared block
    return [("decode", decode), ("shared_prefix", shared), ("mixed", mixed), ("clash", clash)]


STEPS = _steps()


@needs_reference
def test_interface_fixture_is_the_reference_interface():
    import dataclasses
    import inspect

    meta = _reference("minillm.attention.metadata")
    base = _reference("minillm.attention.base")
    assert [f.name for f in dataclasses.fields(meta.AttentionMetadata)] == FIELDS["metadata_fields"]
    assert sorted(base.AttentionBackend.__abstractmethods__) == FIELDS["backend_abstract_methods"]
    assert list(inspect.signature(base.AttentionBackend.forward).parameters) == FIELDS["forward_parameters"]


@needs_reference
@pytest.mark.parametrize("name,seqs", STEPS, ids=[s[0] for s in STEPS])
def test_host_view_of_the_reference_metadata(mlb, name, seqs):
    M = _reference("minillm.attention.metadata")
    host_view = importlib.import_module(mlb.__name__ + ".attention.metadata").host_view
    ref_meta = M.AttentionMetadata.build([M.SeqStep(c, n, list(b)) for c, n, b in seqs], 16, "cpu")
    ours = mlb.AttentionMetadata.build([mlb.SeqStep(c, n, list(b)) for c, n, b in seqs], 16, "cpu")
    tables, private = host_view(ref_meta)
    assert np.array_equal(tables, ours.block_tables_host)
    assert private == ours.append_private == (name != "clash")


def test_package_field_list_is_the_reference_interface(mlb):
    md = importlib.import_module(mlb.__name__ + ".attention.metadata")
    assert list(md.REFERENCE_FIELDS) == FIELDS["metadata_fields"]
    assert all(hasattr(mlb.AttentionMetadata, f) or f in mlb.AttentionMetadata.__dataclass_fields__
               for f in md.REFERENCE_FIELDS)


def reference_shaped(meta) -> types.SimpleNamespace:
    """An object with exactly the reference's AttentionMetadata fields, taken from this package's build."""
    return types.SimpleNamespace(**{f: getattr(meta, f) for f in FIELDS["metadata_fields"]})


@pytest.mark.parametrize("name,seqs", STEPS, ids=[s[0] for s in STEPS])
def test_host_view_of_reference_shaped_metadata(mlb, name, seqs):
    host_view = importlib.import_module(mlb.__name__ + ".attention.metadata").host_view
    ours = mlb.AttentionMetadata.build([mlb.SeqStep(c, n, list(b)) for c, n, b in seqs], 16, "cpu")
    ns = reference_shaped(ours)
    assert not hasattr(ns, "block_tables_host") and not hasattr(ns, "append_private")
    tables, private = host_view(ns)
    assert np.array_equal(tables, ours.block_tables_host) and private == ours.append_private
    # a slot that is not the table's: the append may not ride in the attention launch
    ns.slot_mapping = ours.slot_mapping.clone()
    ns.slot_mapping[-1] += 1
    assert host_view(ns)[1] is False


@pytest.mark.parametrize("name,seqs", STEPS, ids=[s[0] for s in STEPS])
def test_backend_plans_the_same_from_reference_shaped_metadata(mlb, name, seqs):
    ours = mlb.AttentionMetadata.build([mlb.SeqStep(c, n, list(b)) for c, n, b in seqs], 16, "cpu")
    cpu = torch.device("cpu")
    want = mlb.B200Backend(num_sms=148).plan(ours, 32, 8, cpu, torch.bfloat16)
    backend = mlb.B200Backend(num_sms=148)
    got = backend.plan(reference_shaped(ours), 32, 8, cpu, torch.bfloat16)
    for f in ("units_host", "shared_host", "members_host", "reduce_rows_host", "reduce_chunks_host"):
        assert np.array_equal(getattr(got, f), getattr(want, f)), f
    if name == "shared_prefix":
        assert got.num_shared_units > 0  # the cascade stays on with the reference's object
    if name == "mixed":
        assert got.has_query_tiles
    off = mlb.B200Backend(num_sms=148, derive_host_tables=False).plan(reference_shaped(ours), 32, 8, cpu,
                                                                      torch.bfloat16)
    assert off.num_shared_units == 0  # without host tables every row is on 8-column units
