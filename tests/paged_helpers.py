"""Helpers shared by the GPU parity tests: move a seeded case to the device in a given dtype, and compute
the oracle's answer on exactly the values the device sees (16-bit values up-cast to fp32)."""

from __future__ import annotations

import torch

import oracle

TOL = {torch.float32: 1e-5, torch.bfloat16: 2e-2, torch.float16: 2e-2}  # north star: max-abs vs fp32 oracle


def cast_case(case, dtype):
    """The case's tensors rounded to `dtype` (still on the CPU)."""
    return {name: getattr(case, name).to(dtype) for name in ("q", "k", "v", "k_pool", "v_pool")}


def device_case(case, dtype, device):
    t = cast_case(case, dtype)
    return {name: x.to(device) for name, x in t.items()}


def oracle_forward(case, dtype):
    """fp32 oracle on the dtype-rounded inputs; returns (out fp32, k_pool after write, v_pool after write)."""
    t = cast_case(case, dtype)
    meta = oracle.build_metadata(case.seqs, case.bs)
    k_pool, v_pool = t["k_pool"].clone(), t["v_pool"].clone()
    out = oracle.forward(t["q"], t["k"], t["v"], k_pool, v_pool, meta, compute_dtype=torch.float32)
    return out, k_pool, v_pool


def bits(x: torch.Tensor) -> torch.Tensor:
    """Bit pattern view (NaN-safe exact comparison)."""
    return x.view(torch.int32) if x.element_size() == 4 else x.view(torch.int16)


def max_abs(got: torch.Tensor, expected: torch.Tensor) -> float:
    """Largest elementwise |got - expected| (NaN if either holds a NaN where the other does not agree)."""
    g, e = got.float().cpu(), expected.float().cpu()
    if g.shape != e.shape:
        raise AssertionError(f"shapes differ: {tuple(g.shape)} vs {tuple(e.shape)}")
    return (g - e).abs().max().item() if g.numel() else 0.0


def assert_close(got: torch.Tensor, expected: torch.Tensor, dtype) -> None:
    """The north star's bar, max-abs <= 2e-2 (16-bit) or 1e-5 (fp32) against the fp32 oracle with no relative
    term, and beside it the reference's own form of the check (tests/test_kernels.py:59: atol = rtol)."""
    tol = TOL[dtype]
    torch.testing.assert_close(got.float().cpu(), expected.float().cpu(), atol=tol, rtol=tol)
    err = max_abs(got, expected)
    assert err <= tol, f"max |diff| {err:.3g} > {tol} ({dtype})"
