"""K1 kv_append on the GPU: bit-exact against the oracle's write_kv (paged_torch_ref.py:23-28) for every
dtype pair, strided inputs, the reference's own cast bit patterns, and range faults."""

from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

import cases
import oracle
from conftest import GOLDEN
from paged_helpers import bits

pytestmark = pytest.mark.gpu

DTYPES = [torch.float32, torch.bfloat16, torch.float16]


def _pools(nb, hkv, dh, dtype, dev, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    k = torch.randn(nb, 16, hkv, dh, generator=g).to(dtype)
    v = torch.randn(nb, 16, hkv, dh, generator=g).to(dtype)
    return k.to(dev), v.to(dev)


@pytest.mark.parametrize("in_dtype", DTYPES)
@pytest.mark.parametrize("cache_dtype", DTYPES)
@pytest.mark.parametrize("hkv,dh", [(2, 64), (8, 128), (1, 256)])
def test_append_bit_exact(mlb, cuda, in_dtype, cache_dtype, hkv, dh):
    n, nb = 37, 40
    g = torch.Generator().manual_seed(hkv * 1000 + dh)
    slots = torch.randperm(nb * 16, generator=g)[:n]
    # a llama-style strided view: [1, Hkv, N, Dh] transposed to [N, Hkv, Dh] (model/llama.py:114-116)
    k = torch.randn(1, hkv, n, dh, generator=g).to(in_dtype)[0].transpose(0, 1)
    v = (torch.randn(1, n, hkv * 2, dh, generator=g).to(in_dtype) * 3)[0][:, ::2]  # every other head
    k_pool, v_pool = _pools(nb, hkv, dh, cache_dtype, cuda)
    ref_k, ref_v = k_pool.cpu(), v_pool.cpu()
    oracle.write_kv(ref_k, ref_v, slots, k, v)
    mlb.kv_append(k_pool, v_pool, slots.to(cuda), k.to(cuda), v.to(cuda))
    assert torch.equal(bits(k_pool.cpu()), bits(ref_k))
    assert torch.equal(bits(v_pool.cpu()), bits(ref_v))


def test_append_cast_bits_match_reference_golden(mlb, cuda):
    g = np.load(GOLDEN / "append_cast.npz")
    x = cases.cast_rows()
    assert str(g["rows.digest"]) == hashlib.sha256(x.numpy().tobytes()).hexdigest()
    slots = torch.from_numpy(g["slots"]).to(cuda)
    n, hkv, dh = x.shape
    for name, dt in (("bf16", torch.bfloat16), ("f16", torch.float16)):
        k_pool = torch.zeros(8, 16, hkv, dh, dtype=dt, device=cuda)
        v_pool = torch.zeros_like(k_pool)
        mlb.kv_append(k_pool, v_pool, slots, x.to(cuda), (-x).to(cuda))
        for pool, key in ((k_pool, "k_bits"), (v_pool, "v_bits")):
            got = pool.view(-1, hkv, dh)[slots].view(torch.int16).cpu().numpy().view(np.uint16)
            np.testing.assert_array_equal(got, g[f"{name}.{key}"])


def test_append_skips_and_flags_out_of_range_slots(mlb, cuda):
    hkv, dh, nb = 2, 64, 4
    k_pool, v_pool = _pools(nb, hkv, dh, torch.bfloat16, cuda)
    before_k = k_pool.clone()
    rows = torch.randn(3, hkv, dh, device=cuda).to(torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    slots = torch.tensor([5, nb * 16, -1], device=cuda)  # one good slot, two outside the pool
    mlb.kv_append(k_pool, v_pool, slots, rows, rows, err=err)
    assert int(err.item()) & 1  # MLB_DEV_SLOT_RANGE
    flat, flat_before = k_pool.view(-1, hkv, dh), before_k.view(-1, hkv, dh)
    assert torch.equal(flat[5], rows[0])
    keep = torch.ones(nb * 16, dtype=torch.bool)
    keep[5] = False
    assert torch.equal(flat[keep.to(cuda)], flat_before[keep.to(cuda)])


def test_append_empty_and_validation(mlb, cuda):
    k_pool, v_pool = _pools(4, 2, 64, torch.bfloat16, cuda)
    empty = torch.empty(0, 2, 64, dtype=torch.bfloat16, device=cuda)
    mlb.kv_append(k_pool, v_pool, torch.empty(0, dtype=torch.long, device=cuda), empty, empty)
    with pytest.raises(ValueError, match="slot_mapping"):
        rows = torch.zeros(2, 2, 64, dtype=torch.bfloat16, device=cuda)
        mlb.kv_append(k_pool, v_pool, torch.zeros(2, dtype=torch.int32, device=cuda), rows, rows)
    with pytest.raises(ValueError, match="rows must be"):
        rows = torch.zeros(2, 3, 64, dtype=torch.bfloat16, device=cuda)
        mlb.kv_append(k_pool, v_pool, torch.zeros(2, dtype=torch.long, device=cuda), rows, rows)
