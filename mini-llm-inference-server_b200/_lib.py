"""ctypes binding of the C ABI in `include/mlb_paged_kv.h` (the in-tree `_mlb_paged_kv.so`).

The library is required: there is no fallback.  If it is missing, `lib()` raises with the command that
builds it.  Argument and result types are declared once so ctypes converts Python ints exactly.
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_int64, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).with_name("_mlb_paged_kv.so")

# dtype codes and status codes (mlb_paged_kv.h)
MLB_F32, MLB_F16, MLB_BF16 = 0, 1, 2
MLB_OK, MLB_EINVAL, MLB_EUNSUPPORTED, MLB_ECUDA, MLB_ENOSPACE = 0, 1, 2, 3, 4
# bits kernels OR into the device error word
DEV_SLOT_RANGE, DEV_BLOCK_RANGE, DEV_WAIT_TIMEOUT, DEV_COPY_RANGE = 1, 2, 4, 8

EXPORTS = ("mlb_last_error", "mlb_abi_version", "mlb_kv_append", "mlb_plan_attention", "mlb_paged_attention",
           "mlb_splitk_reduce", "mlb_block_copy", "mlb_paged_attention_noalloc", "mlb_ipc_alloc", "mlb_ipc_open",
           "mlb_ipc_close", "mlb_ipc_free", "mlb_peer_barrier", "mlb_set_programmatic_launch",
           "mlb_splitk_reduce_gather", "mlb_set_tensor_core_prefix", "mlb_paged_attention_append",
           "mlb_build_metadata", "mlb_set_concurrent_prefix", "mlb_splitk_reduce_exchange")
ABI_VERSION = 10
NOALLOC_SCRATCH_BYTES = 8 << 20  # MLB_NOALLOC_SCRATCH_BYTES
MAX_OUT_DESTS = 8  # MLB_MAX_OUT_DESTS
IPC_HANDLE_BYTES = 64  # MLB_IPC_HANDLE_BYTES


class WorkUnit(ctypes.Structure):
    """mlb_work_unit: one (sequence, query tile, page range) of paged-attention work."""

    _fields_ = [("seq", c_int32), ("tile_splits", c_int32), ("page_begin", c_int32), ("page_end", c_int32),
                ("part_row", c_int32), ("q0", c_int32), ("num_new", c_int32), ("seq_len", c_int32)]


class SharedUnit(ctypes.Structure):
    """mlb_shared_unit: query-tile work for the tensor-core kernel: a page range of a shared prefix attended
    once for a block of member rows (kind 0), or a tile of a multi-token row's tokens (kind 1)."""

    _fields_ = [("member_begin", c_int32), ("member_count", c_int32), ("page_begin", c_int32),
                ("page_end", c_int32), ("piece", c_int32), ("table_seq", c_int32), ("reserved", c_int32 * 2)]


class ShareMember(ctypes.Structure):
    """mlb_share_member: a decode row that reads a shared prefix."""

    _fields_ = [("seq", c_int32), ("q0", c_int32), ("part_base", c_int32), ("reserved", c_int32)]


class OutTargets(ctypes.Structure):
    """mlb_out_targets: the destinations of the final attention rows (every rank's gathered output)."""

    _fields_ = [("num_dests", c_int32), ("head_offset", c_int32), ("stride_tok", c_int64),
                ("stride_head", c_int64), ("dests", c_void_p * MAX_OUT_DESTS)]


class AppendRows(ctypes.Structure):
    """mlb_append_rows: the step's new k / v rows and their slots, for the fused append + attention."""

    _fields_ = [("k", c_void_p), ("v", c_void_p), ("k_stride_tok", c_int64), ("k_stride_head", c_int64),
                ("v_stride_tok", c_int64), ("v_stride_head", c_int64), ("slot_mapping", c_void_p),
                ("num_tokens", c_int64)]


WORK_UNIT_INT32S = ctypes.sizeof(WorkUnit) // 4
SHARED_UNIT_INT32S = ctypes.sizeof(SharedUnit) // 4
MEMBER_INT32S = ctypes.sizeof(ShareMember) // 4

_I32P, _I64P = POINTER(c_int32), POINTER(c_int64)
_SIGNATURES = {
    "mlb_last_error": (c_char_p, []),
    "mlb_abi_version": (c_int, []),
    "mlb_set_programmatic_launch": (c_int, [c_int]),
    "mlb_set_tensor_core_prefix": (c_int, [c_int]),
    "mlb_set_concurrent_prefix": (c_int, [c_int]),
    "mlb_kv_append": (c_int, [c_void_p, c_void_p, c_int, c_int64, c_int, c_void_p, c_void_p, c_int64, c_int64,
                              c_void_p, c_int64, c_int64, c_int, c_int64, c_int, c_int, c_void_p, c_void_p]),
    "mlb_plan_attention": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_int64, c_int, c_int, c_int, c_int,
                                   c_int, c_void_p, c_int64, _I64P, c_void_p, c_int64, _I64P, c_void_p, c_int64,
                                   _I64P, c_void_p, c_void_p, c_int64, _I64P]),
    "mlb_paged_attention": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int, c_int64, c_int, c_int,
                                    c_int, c_int, c_float, c_void_p, c_int64, c_void_p, c_void_p, c_int, c_void_p,
                                    c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_int64, c_void_p,
                                    c_int64, c_int64, POINTER(OutTargets), c_void_p, c_void_p]),
    "mlb_paged_attention_append": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int, c_int64, c_int,
                                           c_int, c_int, c_int, c_float, c_void_p, c_int64, c_void_p, c_void_p,
                                           c_int, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p,
                                           c_void_p, c_int64, c_void_p, c_int64, c_int64, POINTER(OutTargets),
                                           POINTER(AppendRows), c_void_p, c_void_p]),
    "mlb_splitk_reduce": (c_int, [c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_int, c_int64, c_int, c_int,
                                  c_void_p, c_int64, c_int64, c_int, POINTER(OutTargets), c_void_p]),
    "mlb_block_copy": (c_int, [c_void_p, c_int, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_void_p,
                               c_void_p]),
    "mlb_build_metadata": (c_int, [c_void_p, c_int64, c_int, c_int64, c_int64, c_int, c_int, c_void_p, c_void_p,
                                   c_void_p]),
    "mlb_paged_attention_noalloc": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int, c_int64, c_int,
                                            c_int, c_int, c_int, c_float, c_void_p, c_int64, c_void_p, c_void_p,
                                            c_int, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64,
                                            c_void_p, c_void_p, c_int64, c_void_p, c_int64, c_int64, c_void_p,
                                            c_void_p]),
    "mlb_ipc_alloc": (c_int, [c_int64, POINTER(c_void_p), c_void_p]),
    "mlb_ipc_open": (c_int, [c_void_p, POINTER(c_void_p)]),
    "mlb_ipc_close": (c_int, [c_void_p]),
    "mlb_ipc_free": (c_int, [c_void_p]),
    "mlb_peer_barrier": (c_int, [POINTER(c_void_p), c_int, c_int, c_void_p, c_int64, c_void_p, c_void_p]),
    "mlb_splitk_reduce_gather": (c_int, [c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_int, c_int64, c_int,
                                         c_int, c_int, POINTER(OutTargets), c_int, c_void_p]),
    "mlb_splitk_reduce_exchange": (c_int, [c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_int, c_int64, c_int,
                                           c_int, c_int, c_void_p, c_int64, c_int64, POINTER(c_void_p), c_int64,
                                           c_int, c_int, c_void_p, c_int64, c_void_p, c_void_p]),
}

_lib: ctypes.CDLL | None = None


class MlbError(RuntimeError):
    """A CUDA-side failure reported by the library (MLB_ECUDA / MLB_ENOSPACE)."""


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH.name} is not built: run `python {LIB_PATH.parent.name}/build.py` "
                              "(nvcc, sm_100a); the paged-KV ops have no fallback")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def last_error() -> str:
    return lib().mlb_last_error().decode(errors="replace")


def check(rc: int, what: str) -> None:
    """Turn a status code into the exception the reference raises for the same fault."""
    if rc == MLB_OK:
        return
    msg = f"{what}: {last_error()}"
    if rc in (MLB_EINVAL, MLB_EUNSUPPORTED):
        raise ValueError(msg)
    raise MlbError(msg)
