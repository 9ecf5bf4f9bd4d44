"""Torch-facing wrappers of the C ABI: tensors in, raw pointers + strides + the current CUDA stream out.

Every function validates what the kernels rely on (shapes, dtypes, devices, contiguity of the pools)
and raises `ValueError` like the reference does for malformed input (metadata.py:75-76); device-side
range faults (a bad slot or block id) are skipped by the kernels and recorded in an optional int32
error word instead of faulting the GPU.
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import (MAX_OUT_DESTS, MEMBER_INT32S, SHARED_UNIT_INT32S, WORK_UNIT_INT32S, AppendRows, OutTargets, check,
                   lib)

DTYPE_CODE = {torch.float32: _lib.MLB_F32, torch.float16: _lib.MLB_F16, torch.bfloat16: _lib.MLB_BF16}
BLOCK_SIZE = 16


def _code(t: torch.Tensor, what: str) -> int:
    try:
        return DTYPE_CODE[t.dtype]
    except KeyError:
        raise ValueError(f"{what}: dtype {t.dtype} not supported (float32, float16, bfloat16)") from None


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(device: torch.device) -> int:
    """Handle of torch's current stream on `device` (the raw query: a decode step makes ~100 of these)."""
    if _raw_stream is not None and device.index is not None:
        return _raw_stream(device.index)
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _check_pool(pool: torch.Tensor, what: str) -> None:
    if pool.dim() != 4 or not pool.is_contiguous():
        raise ValueError(f"{what}: pools are contiguous [num_blocks, block_size, Hkv, Dh], got {tuple(pool.shape)}")
    if not pool.is_cuda:
        raise ValueError(f"{what}: pools must be CUDA tensors")


def _check_rows(x: torch.Tensor, hkv: int, dh: int, what: str) -> None:
    if x.dim() != 3 or x.shape[1:] != (hkv, dh) or (x.shape[0] and x.stride(2) != 1):
        raise ValueError(f"{what}: rows must be [N, {hkv}, {dh}] with unit stride on the last dim, "
                         f"got {tuple(x.shape)} strides {x.stride()}")


# ---------------------------------------------------------------- K1: append


def kv_append(k_cache: torch.Tensor, v_cache: torch.Tensor, slot_mapping: torch.Tensor, k: torch.Tensor,
              v: torch.Tensor, err: torch.Tensor | None = None) -> None:
    """write_kv (paged_torch_ref.py:23-28) on the GPU: pools[slot_mapping[i]] = k[i] / v[i], cast to the
    pool dtype (round to nearest even).  k, v may be strided views [N, Hkv, Dh]."""
    _check_pool(k_cache, "kv_append")
    _check_pool(v_cache, "kv_append")
    nb, bs, hkv, dh = k_cache.shape
    if v_cache.shape != k_cache.shape or v_cache.dtype != k_cache.dtype:
        raise ValueError("kv_append: k_cache and v_cache differ")
    _check_rows(k, hkv, dh, "kv_append k")
    _check_rows(v, hkv, dh, "kv_append v")
    n = k.shape[0]
    if v.shape[0] != n or slot_mapping.shape != (n,):
        raise ValueError(f"kv_append: {n} k rows, {v.shape[0]} v rows, slot_mapping {tuple(slot_mapping.shape)}")
    if slot_mapping.dtype != torch.long or not slot_mapping.is_contiguous():
        raise ValueError("kv_append: slot_mapping must be a contiguous int64 tensor")
    if k.dtype != v.dtype:
        raise ValueError("kv_append: k and v dtypes differ")
    for t in (v_cache, slot_mapping, k, v):
        if t.device != k_cache.device:
            raise ValueError("kv_append: all tensors must be on the pools' device")
    if n == 0:
        return
    rc = lib().mlb_kv_append(k_cache.data_ptr(), v_cache.data_ptr(), _code(k_cache, "kv_append"), nb, bs,
                             slot_mapping.data_ptr(), k.data_ptr(), k.stride(0), k.stride(1), v.data_ptr(),
                             v.stride(0), v.stride(1), _code(k, "kv_append"), n, hkv, dh, _ptr(err),
                             _stream(k_cache.device))
    check(rc, "kv_append")


# ---------------------------------------------------------------- K2: plan, attention, reduction


@dataclass
class AttentionPlan:
    """A step's split of paged-attention work (built once per AttentionMetadata, reused by every layer)."""

    units: torch.Tensor  # device int32 [num_units, 8]: mlb_work_unit records
    num_units: int
    shared_units: torch.Tensor  # device int32 [num_shared_units, 8]: mlb_shared_unit records (may be empty)
    num_shared_units: int
    members: torch.Tensor  # device int32 [num_members, 4]: mlb_share_member records
    reduce_rows: torch.Tensor  # device int32 [N]
    reduce_chunks: torch.Tensor  # device int32 [N]
    num_partial_rows: int
    tokens_per_tile: int
    num_heads: int
    num_kv_heads: int
    num_tokens: int
    units_host: np.ndarray  # the same records on the host (inspection and tests)
    shared_host: np.ndarray
    members_host: np.ndarray
    reduce_rows_host: np.ndarray
    reduce_chunks_host: np.ndarray  # [N] pieces per token on the host
    has_query_tiles: bool = False  # kind-1 shared units (rows of >= 16 new tokens) in the plan


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32))


def plan_attention(qo_indptr: list[int], seq_lens: list[int], max_blocks: int, num_heads: int, num_kv_heads: int,
                   device: torch.device | str, block_size: int = BLOCK_SIZE, num_sms: int | None = None,
                   pages_per_unit: int = 0, block_tables_host: np.ndarray | None = None) -> AttentionPlan:
    """Split the step into units (host work, like FlashInfer's plan(); flashinfer_backend.py:48-64).

    qo_indptr / seq_lens are the host lists AttentionMetadata keeps (metadata.py:39-40), so planning
    needs no device round trip.  With `block_tables_host` (int32 [S, W]) decode rows that share leading
    blocks (prefix-cache hits) are planned as shared-prefix units (16-bit pools only).  The plan is copied
    to the device in one transfer.
    """
    device = torch.device(device)
    qo, lens = _i32(qo_indptr), _i32(seq_lens)
    s = len(lens)
    if qo.shape != (s + 1,):
        raise ValueError(f"plan: qo_indptr has {qo.shape[0]} entries for {s} sequences")
    n_tok = int(qo[-1]) if s else 0
    if num_sms is None:
        num_sms = torch.cuda.get_device_properties(device).multi_processor_count if device.type == "cuda" else 148
    tables = None if block_tables_host is None else _i32(block_tables_host)
    if tables is not None and (tables.ndim != 2 or tables.shape[0] != s):
        raise ValueError(f"plan: block_tables_host must be [{s}, W], got {tables.shape}")
    L = lib()
    nu, ns, nm, npart = (ctypes.c_int64(0) for _ in range(4))
    head = (qo.ctypes.data, lens.ctypes.data, s, max_blocks, None if tables is None else tables.ctypes.data,
            0 if tables is None else tables.shape[1], num_heads, num_kv_heads, block_size, num_sms, pages_per_unit)
    check(L.mlb_plan_attention(*head, None, 0, ctypes.byref(nu), None, 0, ctypes.byref(ns), None, 0,
                               ctypes.byref(nm), None, None, n_tok, ctypes.byref(npart)), "plan_attention")
    units = np.zeros((max(nu.value, 1), WORK_UNIT_INT32S), dtype=np.int32)
    shared = np.zeros((max(ns.value, 1), SHARED_UNIT_INT32S), dtype=np.int32)
    members = np.zeros((max(nm.value, 1), MEMBER_INT32S), dtype=np.int32)
    rows = np.empty(max(n_tok, 1), dtype=np.int32)
    chunks = np.empty(max(n_tok, 1), dtype=np.int32)
    check(L.mlb_plan_attention(*head, units.ctypes.data, units.shape[0], ctypes.byref(nu), shared.ctypes.data,
                               shared.shape[0], ctypes.byref(ns), members.ctypes.data, members.shape[0],
                               ctypes.byref(nm), rows.ctypes.data, chunks.ctypes.data, n_tok, ctypes.byref(npart)),
          "plan_attention")
    u, sh, m = nu.value, ns.value, nm.value
    # one host -> device copy for the whole plan
    parts = [units[:u].reshape(-1), shared[:sh].reshape(-1), members[:m].reshape(-1), rows[:n_tok], chunks[:n_tok]]
    offs = np.cumsum([0] + [p.size for p in parts])
    host = torch.from_numpy(np.concatenate(parts))
    dev = host.pin_memory().to(device, non_blocking=True) if device.type == "cuda" else host.clone()
    seg = [dev[offs[i]:offs[i + 1]] for i in range(len(parts))]
    return AttentionPlan(seg[0].view(u, WORK_UNIT_INT32S), u, seg[1].view(sh, SHARED_UNIT_INT32S), sh,
                         seg[2].view(m, MEMBER_INT32S), seg[3], seg[4], npart.value,
                         max(1, 8 // (num_heads // num_kv_heads)), num_heads, num_kv_heads, n_tok,
                         units[:u].copy(), shared[:sh].copy(), members[:m].copy(), rows[:n_tok].copy(),
                         chunks[:n_tok].copy(), bool(sh and ((shared[:sh, 6] & 0xFF) == 1).any()))


class Workspace:
    """Split-K scratch (fp32 partial rows + their log-sum-exp), grown on demand and reused across calls."""

    def __init__(self) -> None:
        self._o: torch.Tensor | None = None
        self._lse: torch.Tensor | None = None

    def get(self, rows: int, heads: int, dh: int, device: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
        need_o, need_l = rows * heads * dh, rows * heads
        if self._o is None or self._o.device != device or self._o.numel() < need_o:
            self._o = torch.empty(max(need_o, 1), dtype=torch.float32, device=device)
        if self._lse is None or self._lse.device != device or self._lse.numel() < need_l:
            self._lse = torch.empty(max(need_l, 1), dtype=torch.float32, device=device)
        return self._o, self._lse


def paged_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_tables: torch.Tensor,
                    seq_lens: torch.Tensor, qo_indptr: torch.Tensor, plan: AttentionPlan,
                    workspace: Workspace | None = None, out: torch.Tensor | None = None, scale: float | None = None,
                    err: torch.Tensor | None = None, targets: OutTargets | None = None,
                    append: tuple[torch.Tensor, torch.Tensor, torch.Tensor] | None = None) -> torch.Tensor | None:
    """paged_attention (paged_torch_ref.py:40-74) on the GPU: q [N, H, Dh] -> [N, H, Dh] in q's dtype.

    block_tables int32 [S, W], seq_lens int32 [S], qo_indptr int32 [S + 1] are AttentionMetadata's
    device tensors (block_tables_i32, seq_lens_i32, qo_indptr).  The pools must already hold this
    step's k/v (kv_append first), unless `append` = (k, v, slot_mapping) asks the attention launch to do
    the append itself (see `attention_partials`).  Launches the shared-prefix and per-sequence attention
    kernels, then the split-K reduction when the plan split any sequence.  With `targets` (see
    `out_targets`) the rows go to those destinations instead and nothing is returned.
    """
    workspace = workspace or Workspace()
    out = attention_partials(q, k_cache, v_cache, block_tables, seq_lens, qo_indptr, plan, workspace, out, scale,
                             err, targets, append)
    splitk_reduce(plan, workspace, out, targets, q.dtype, q.shape[2], q.device)
    return out


def out_targets(dests: list[int], head_offset: int, stride_tok: int, stride_head: int) -> OutTargets:
    """mlb_out_targets: store every final row (token t, local head h) at element offset
    t * stride_tok + (head_offset + h) * stride_head of each destination address in `dests`."""
    if not 1 <= len(dests) <= MAX_OUT_DESTS:
        raise ValueError(f"out_targets: 1..{MAX_OUT_DESTS} destinations, got {len(dests)}")
    t = OutTargets()
    t.num_dests, t.head_offset, t.stride_tok, t.stride_head = len(dests), head_offset, stride_tok, stride_head
    for i, d in enumerate(dests):
        t.dests[i] = d
    return t


def attention_partials(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_tables: torch.Tensor,
                       seq_lens: torch.Tensor, qo_indptr: torch.Tensor, plan: AttentionPlan, workspace: Workspace,
                       out: torch.Tensor | None = None, scale: float | None = None,
                       err: torch.Tensor | None = None, targets: OutTargets | None = None,
                       append: tuple[torch.Tensor, torch.Tensor, torch.Tensor] | None = None) -> torch.Tensor | None:
    """The attention kernels (K2s, K2a): unsplit sequences are final in `out` (or `targets`); split ones
    leave fp32 partial rows in `workspace` for `splitk_reduce`.

    append = (k, v, slot_mapping): kv_append fused into the attention launch (mlb_paged_attention_append;
    torch_ref.py:46-48 writes, then attends).  The caller guarantees what that entry point needs:
    slot_mapping is the one the block tables give, and every written block is in one sequence's context
    pages only (AttentionMetadata.append_private); `can_fuse_append` checks the rest."""
    _check_pool(k_cache, "paged_attention")
    _check_pool(v_cache, "paged_attention")
    nb, bs, hkv, dh = k_cache.shape
    if q.dim() != 3 or q.shape[2] != dh or (q.shape[0] and q.stride(2) != 1):
        raise ValueError(f"paged_attention: q must be [N, H, {dh}] with unit last stride, got {tuple(q.shape)}")
    n, h = q.shape[0], q.shape[1]
    if q.dtype != k_cache.dtype or v_cache.dtype != k_cache.dtype or v_cache.shape != k_cache.shape:
        raise ValueError(f"paged_attention: q {q.dtype} and pools {k_cache.dtype}/{v_cache.dtype} must agree")
    if (plan.num_heads, plan.num_kv_heads, plan.num_tokens) != (h, hkv, n):
        raise ValueError("paged_attention: the plan was built for another shape")
    for t, name in ((block_tables, "block_tables"), (seq_lens, "seq_lens"), (qo_indptr, "qo_indptr")):
        if t.dtype != torch.int32 or not t.is_contiguous() or t.device != q.device:
            raise ValueError(f"paged_attention: {name} must be a contiguous int32 tensor on {q.device}")
    if targets is not None:
        out = None
    elif out is None:
        out = torch.empty_like(q)
    elif out.shape != q.shape or out.dtype != q.dtype or out.stride(2) != 1:
        raise ValueError("paged_attention: out must match q")
    if n == 0 or plan.num_units + plan.num_shared_units == 0:
        return out
    scale = 1.0 / math.sqrt(dh) if scale is None else float(scale)
    po = plse = None
    if plan.num_partial_rows:
        po, plse = workspace.get(plan.num_partial_rows, h, dh, q.device)
    args = (q.data_ptr(), q.stride(0), q.stride(1), k_cache.data_ptr(), v_cache.data_ptr(),
            _code(q, "paged_attention"), nb, bs, h, hkv, dh, scale, block_tables.data_ptr(), block_tables.stride(0),
            seq_lens.data_ptr(), qo_indptr.data_ptr(), seq_lens.shape[0], plan.units.data_ptr(), plan.num_units,
            plan.shared_units.data_ptr(), plan.num_shared_units, plan.members.data_ptr(), _ptr(po), _ptr(plse),
            plan.num_partial_rows, _ptr(out), *_strides(out), _targets(targets))
    if append is None:
        rc = lib().mlb_paged_attention(*args, _ptr(err), _stream(q.device))
        check(rc, "paged_attention")
        return out
    k, v, slots = append
    if not can_fuse_append(plan, k_cache, k, v):
        raise ValueError("paged_attention: this append cannot ride in the attention launch (see can_fuse_append)")
    if slots.dtype != torch.long or not slots.is_contiguous() or slots.shape != (n,) or slots.device != q.device:
        raise ValueError(f"paged_attention: slot_mapping must be a contiguous int64 [{n}] tensor on {q.device}")
    rows = AppendRows()
    rows.k, rows.v, rows.slot_mapping, rows.num_tokens = k.data_ptr(), v.data_ptr(), slots.data_ptr(), n
    rows.k_stride_tok, rows.k_stride_head, rows.v_stride_tok, rows.v_stride_head = (k.stride(0), k.stride(1),
                                                                                    v.stride(0), v.stride(1))
    rc = lib().mlb_paged_attention_append(*args, ctypes.byref(rows), _ptr(err), _stream(q.device))
    check(rc, "paged_attention_append")
    return out


def can_fuse_append(plan: AttentionPlan, k_cache: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> bool:
    """Whether kv_append can ride in the attention launch, as far as the plan and tensors go: 16-bit pools
    with head_dim 64 / 128, k / v [N, Hkv, Dh] in the pools' dtype on their device with 16-byte aligned
    rows, N the plan's token count, and no query-tile units (rows of >= 16 new tokens).  The metadata's
    half of the condition is AttentionMetadata.append_private."""
    dt = k_cache.dtype
    if plan.has_query_tiles or (dt is not torch.bfloat16 and dt is not torch.float16) or k_cache.shape[3] not in (64, 128):
        return False
    shape = (plan.num_tokens, k_cache.shape[2], k_cache.shape[3])
    for t in (k, v):
        if t.dtype is not dt or t.shape != shape or t.device != k_cache.device:
            return False
        if shape[0]:
            s0, s1, s2 = t.stride()
            if s2 != 1 or (s0 | s1) & 7 or t.data_ptr() & 15:  # 16-byte rows: strides x 2 B multiples of 16
                return False
    return True


def splitk_reduce(plan: AttentionPlan, workspace: Workspace, out: torch.Tensor | None,
                  targets: OutTargets | None = None, dtype: torch.dtype | None = None, head_dim: int | None = None,
                  device: torch.device | None = None) -> None:
    """K2b: combine the split sequences' partial rows into `out` (no-op when the plan split nothing).
    With `targets`, the rows go there instead; dtype / head_dim / device then describe them."""
    if not plan.num_partial_rows or plan.num_tokens == 0:
        return
    if targets is None:
        if out is None:
            raise ValueError("splitk_reduce: no out and no targets")
        dtype, head_dim, device = out.dtype, out.shape[2], out.device
    n, h = plan.num_tokens, plan.num_heads
    po, plse = workspace.get(plan.num_partial_rows, h, head_dim, device)
    rc = lib().mlb_splitk_reduce(po.data_ptr(), plse.data_ptr(), plan.num_partial_rows, plan.reduce_rows.data_ptr(),
                                 plan.reduce_chunks.data_ptr(), plan.tokens_per_tile, n, h, head_dim, _ptr(out),
                                 *_strides(out), DTYPE_CODE[dtype], _targets(targets), _stream(device))
    check(rc, "splitk_reduce")


def splitk_reduce_gather(plan: AttentionPlan, workspace: Workspace, targets: OutTargets, self_dest: int,
                         dtype: torch.dtype, head_dim: int, device: torch.device) -> None:
    """The split-K reduction carrying the output all-gather (mlb_splitk_reduce_gather): after
    `attention_partials` wrote the unsplit rows into destination `self_dest` only, every row of the step
    is stored into every destination.  Follow it with the peers' barrier (`PeerOutputs.barrier`)."""
    po = plse = None
    if plan.num_partial_rows:
        po, plse = workspace.get(plan.num_partial_rows, plan.num_heads, head_dim, device)
    rc = lib().mlb_splitk_reduce_gather(_ptr(po), _ptr(plse), plan.num_partial_rows, plan.reduce_rows.data_ptr(),
                                        plan.reduce_chunks.data_ptr(), plan.tokens_per_tile, plan.num_tokens,
                                        plan.num_heads, head_dim, DTYPE_CODE[dtype], ctypes.byref(targets), self_dest,
                                        _stream(device))
    check(rc, "splitk_reduce_gather")


def splitk_reduce_exchange(plan: AttentionPlan, workspace: Workspace, peers, slot: int, dtype: torch.dtype,
                           head_dim: int, device: torch.device, err: torch.Tensor | None = None) -> None:
    """The output all-gather as flagged packets (mlb_splitk_reduce_exchange): after `attention_partials` left
    this rank's unsplit rows in its own buffer of `slot` (`peers.local_targets`), one launch finishes this
    rank's rows, sends them to every peer and waits for theirs; no barrier follows.  `peers` is the
    `sharding.PeerOutputs` of the step (its packet areas and state words)."""
    po = plse = None
    if plan.num_partial_rows:
        po, plse = workspace.get(plan.num_partial_rows, plan.num_heads, head_dim, device)
    rc = lib().mlb_splitk_reduce_exchange(_ptr(po), _ptr(plse), plan.num_partial_rows, plan.reduce_rows.data_ptr(),
                                          plan.reduce_chunks.data_ptr(), plan.tokens_per_tile, plan.num_tokens,
                                          plan.num_heads, head_dim, DTYPE_CODE[dtype], peers.slot_address(slot),
                                          peers.num_heads * head_dim, head_dim, peers.packet_areas(),
                                          peers.capacity, peers.rank, peers.world, peers.state_address,
                                          peers.timeout_ns, peers.err.data_ptr() if err is None else err.data_ptr(),
                                          _stream(device))
    check(rc, "splitk_reduce_exchange")


def _strides(out: torch.Tensor | None) -> tuple[int, int]:
    return (out.stride(0), out.stride(1)) if out is not None else (0, 0)


def _targets(t: OutTargets | None):
    return ctypes.byref(t) if t is not None else None


# ---------------------------------------------------------------- metadata expansion on the device


def build_metadata(upload: torch.Tensor, num_ids: int, num_seqs: int, num_tokens: int, num_pages: int, width: int,
                   block_size: int, out64: torch.Tensor, out32: torch.Tensor) -> None:
    """mlb_build_metadata: expand a step's compact int64 upload (block ids, ids_indptr, qo_indptr, seq_lens,
    kv_indptr, kv_last_page_len) into the two buffers AttentionMetadata's device tensors view
    (metadata.py:71-103's arrays, computed on the GPU)."""
    s = num_seqs
    need = {"upload": (upload, torch.long, num_ids + 5 * s + 3),
            "out64": (out64, torch.long, 2 * num_tokens + s * width + s),
            "out32": (out32, torch.int32, s * width + 4 * s + 2 + num_pages)}
    for name, (t, dt, n) in need.items():
        if t.dtype != dt or not t.is_contiguous() or not t.is_cuda or t.device != upload.device or t.numel() < n:
            raise ValueError(f"build_metadata: {name} must be a contiguous {dt} CUDA tensor of >= {n} elements")
    rc = lib().mlb_build_metadata(upload.data_ptr(), num_ids, s, num_tokens, num_pages, width, block_size,
                                  out64.data_ptr(), out32.data_ptr(), _stream(upload.device))
    check(rc, "build_metadata")


# ---------------------------------------------------------------- K3: block copy


def pool_pointer_table(pools: list[torch.Tensor]) -> torch.Tensor:
    """Device int64 array of pool base addresses (every layer's K and V), the block copy's `pools`."""
    if not pools:
        raise ValueError("block_copy: no pools")
    first = pools[0]
    for p in pools:
        _check_pool(p, "block_copy")
        if p.shape != first.shape or p.dtype != first.dtype or p.device != first.device:
            raise ValueError("block_copy: every pool must have the same shape, dtype and device")
    ptrs = torch.tensor([p.data_ptr() for p in pools], dtype=torch.int64)
    return ptrs.to(first.device)


def block_copy(pool_ptrs: torch.Tensor, template: torch.Tensor, src: torch.Tensor, dst: torch.Tensor,
               err: torch.Tensor | None = None) -> None:
    """pool[dst[i]] = pool[src[i]] for every pool in `pool_ptrs` (see `pool_pointer_table`); `template` is
    any one of the pools (it fixes num_blocks and the block size in bytes).  src / dst: device int32."""
    if src.shape != dst.shape or src.dim() != 1:
        raise ValueError("block_copy: src and dst must be 1-D and of equal length")
    for t, name in ((src, "src"), (dst, "dst")):
        if t.dtype != torch.int32 or not t.is_contiguous() or t.device != template.device:
            raise ValueError(f"block_copy: {name} must be a contiguous int32 tensor on {template.device}")
    if src.numel() == 0:
        return
    nb = template.shape[0]
    block_bytes = template[0].numel() * template.element_size()
    rc = lib().mlb_block_copy(pool_ptrs.data_ptr(), pool_ptrs.numel(), nb, block_bytes, src.data_ptr(),
                              dst.data_ptr(), src.numel(), _ptr(err), _stream(template.device))
    check(rc, "block_copy")
