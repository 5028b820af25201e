"""ctypes binding of libabkv.so (the C ABI declared in include/abkv.h).

The shared library is the product: there is no CPU or PyTorch fallback.  If
the library is missing, every entry point raises at import of the op.
"""
from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

_LIB_PATH = Path(__file__).resolve().parent / "libabkv.so"
_lock = threading.Lock()
_lib: C.CDLL | None = None

c_int = C.c_int
c_i32p = C.POINTER(C.c_int32)
c_i64p = C.POINTER(C.c_int64)
c_i64 = C.c_int64
c_vp = C.c_void_p
c_vpp = C.POINTER(C.c_void_p)
c_size = C.c_size_t

GATHER_FLAG_BYTES = 256   # ABKV_GATHER_FLAG_BYTES
MAX_PEERS = 8             # ABKV_MAX_PEERS
PEER_HANDLE_BYTES = 64    # ABKV_PEER_HANDLE_BYTES


class GatherT(C.Structure):
    """abkv_gather_t."""
    _fields_ = [("rank_buffers", C.c_void_p * MAX_PEERS), ("buffer_bytes", C.c_size_t), ("world", C.c_int),
                ("rank", C.c_int), ("hq_total", C.c_int), ("epoch", C.c_uint32), ("timeout_us", C.c_uint32)]


class SidecarT(C.Structure):
    """abkv_sidecar_t."""
    _fields_ = [("pages", C.c_void_p), ("page_table", C.c_void_p), ("page_count", C.c_void_p),
                ("page_table_stride", C.c_int64), ("num_pages", C.c_int64), ("slots", C.c_int),
                ("quotas", C.c_int * 8)]


# name -> (restype, argtypes); must mirror include/abkv.h exactly.
SIGNATURES: dict[str, tuple] = {
    "abkv_status_string": (C.c_char_p, [c_int]),
    "abkv_version": (C.c_char_p, []),
    "abkv_workspace_error": (c_int, [c_vp, c_vp, c_i32p]),
    "abkv_decode_workspace_size": (c_size, [c_int, c_int, c_int, c_int, c_int, c_int, c_int]),
    "abkv_decode": (
        c_int,
        [c_vpp, c_vpp, c_vpp, c_i64p, c_vpp, c_i64p, c_vpp, c_int, c_int, c_int, c_int, c_int,
         c_int, c_int, C.c_float, c_int, c_vp, c_size, c_vp],
    ),
    "abkv_decode_noalloc": (
        c_int,
        [c_vpp, c_vpp, c_vpp, c_i64p, c_vpp, c_i64p, c_vpp, c_int, c_int, c_int, c_int, c_int,
         c_int, c_int, C.c_float, c_int, c_vp, c_vp],
    ),
    "abkv_decode_gather": (
        c_int,
        [c_vpp, c_vpp, c_vpp, c_i64p, c_vpp, c_i64p, c_vpp, c_int, c_int, c_int, c_int, c_int,
         c_int, c_int, C.c_float, c_int, c_vp, c_vp, c_size, c_vp],
    ),
    "abkv_decode_packed_workspace_size": (c_size, [c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_i64]),
    "abkv_decode_packed": (
        c_int,
        [c_vpp, c_vpp, c_vpp, c_i64p, c_vpp, c_i64p, c_vpp, c_int, c_int, c_int, c_int, c_int,
         c_int, c_int, C.c_float, c_int, c_vp, c_vp, c_size, c_vp],
    ),
    "abkv_peer_alloc": (c_int, [c_size, c_vpp, c_vp]),
    "abkv_peer_open": (c_int, [c_vp, c_vpp]),
    "abkv_peer_close": (c_int, [c_vp]),
    "abkv_peer_free": (c_int, [c_vp]),
    "abkv_planner_create": (c_vp, [c_int, c_int, c_int]),
    "abkv_planner_destroy": (None, [c_vp]),
    "abkv_planner_add_request": (c_int, [c_vp, C.c_int64]),
    "abkv_planner_set_num_computed": (c_int, [c_vp, C.c_int64, C.c_int64]),
    "abkv_planner_allocate_slots": (c_int, [c_vp, C.c_int64, C.c_int64]),
    "abkv_planner_free_request": (c_int, [c_vp, C.c_int64]),
    "abkv_planner_mask_token_span": (c_int, [c_vp, C.c_int64, C.c_int64, C.c_int64, c_i32p, c_int, c_vp]),
    "abkv_planner_finish_block": (
        c_int, [c_vp, C.c_int64, C.c_int64, C.c_int64, C.c_int64, C.c_int64, c_i32p, c_int, c_int, c_vp]),
    "abkv_planner_block_table": (c_int, [c_vp, C.c_int64, c_int, c_i32p, c_int, C.POINTER(c_int)]),
    "abkv_planner_free_queue": (c_int, [c_vp, c_i32p, c_int, C.POINTER(c_int)]),
    "abkv_planner_num_free": (c_int, [c_vp]),
    "abkv_planner_span_map": (c_int, [c_vp, C.c_int64, c_int, C.c_int64, c_int, c_i64p]),
    "abkv_planner_compacted_spans": (c_int, [c_vp, C.c_int64, c_int, c_i64p, c_int, C.POINTER(c_int)]),
    "abkv_planner_pending_requests": (c_int, [c_vp, c_i64p, c_int, C.POINTER(c_int)]),
    "abkv_planner_pending_num_batches": (c_int, [c_vp, C.c_int64, c_int]),
    "abkv_planner_pending_batch": (c_int, [c_vp, C.c_int64, c_int, c_int, c_i32p, c_int, C.POINTER(c_int)]),
    "abkv_planner_pending_truncation": (c_int, [c_vp, C.c_int64, c_i32p, c_int, C.POINTER(c_int)]),
    "abkv_planner_pending_export": (c_int, [c_vp, c_i64p, c_i32p, c_i32p, c_i32p, c_int, c_int, c_int,
                                            C.POINTER(c_int), C.POINTER(c_int), C.POINTER(c_int)]),
    "abkv_planner_pending_trunc_export": (c_int, [c_vp, c_i64p, c_i32p, c_int, C.POINTER(c_int)]),
    "abkv_planner_clear_pending": (c_int, [c_vp]),
    "abkv_compact_workspace_size": (c_size, [c_int, c_int, c_int, c_int, C.c_int64]),
    "abkv_compact": (c_int, [c_vpp, c_int, c_int, C.c_int64, c_int, c_int, c_int, c_i32p, c_i64p, c_int,
                             c_vp, c_size, c_vp]),
    "abkv_gather_rows": (c_int, [c_vpp, c_vpp, c_int, C.c_int64, C.c_int64, C.c_int64, C.c_int64, c_vp,
                                 c_vp, c_size, c_vp]),
    "abkv_store_kv": (c_int, [c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_int, c_i64, c_int, c_int, c_int,
                              c_vp, c_int, c_vp, c_size, c_vp]),
    "abkv_prefill_masked": (c_int, [c_vp, c_i64p, c_vp, c_i64p, c_vp, c_i64p, c_vp, c_i64p, c_vp, c_i32p, c_vp,
                                    c_int, c_int, c_int, c_int, c_int, c_int, c_int, C.c_float, c_vp, c_size,
                                    c_vp]),
    "abkv_prefill_masked_backward_workspace_size": (c_size, [c_int, c_int, c_int, c_int]),
    "abkv_prefill_masked_backward": (c_int, [c_vp, c_i64p, c_vp, c_i64p, c_vp, c_i64p, c_vp, c_i64p, c_vp,
                                             c_i64p, c_vp, c_vp, c_i64p, c_vp, c_i64p, c_vp, c_i64p, c_i32p,
                                             c_vp, c_int, c_int, c_int, c_int, c_int, c_int, c_int, C.c_float,
                                             c_vp, c_size, c_vp]),
    "abkv_code_step_attention": (c_int, [c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_vp, c_int, c_i64, c_int,
                                         c_vp, c_i64, c_vp, c_vp, c_i32p, c_int, c_int, c_int, c_int, c_int,
                                         c_int, C.c_float, c_vp, c_size, c_vp]),
    "abkv_paged_prefill": (c_int, [c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_vp, c_int, c_i64, c_int, c_vp,
                                   c_i64, c_vp, c_int, c_int, c_int, c_int, c_int, c_int, C.c_float, c_vp, c_size,
                                   c_vp]),
    "abkv_code_step_attention_packed": (c_int, [c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_vp, c_int, c_i64,
                                                c_int, c_vp, c_i64, c_vp, c_vp, c_i32p, c_int, c_int, c_int, c_int,
                                                c_int, c_int, C.c_float, c_vp, c_vp, c_size, c_vp]),
    "abkv_paged_prefill_packed": (c_int, [c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_vp, c_int, c_i64, c_int,
                                          c_vp, c_i64, c_vp, c_int, c_int, c_int, c_int, c_int, c_int, C.c_float,
                                          c_vp, c_vp, c_size, c_vp]),
    "abkv_code_step_compact_workspace_size": (c_size, [c_int, c_i64]),
    "abkv_code_step_attention_compact": (c_int, [c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_vp, c_int, c_i64,
                                                 c_int, c_vp, c_i64, c_vp, c_vp, c_i32p, c_int, c_int, c_int, c_int,
                                                 c_int, c_int, C.c_float, c_i32p, c_i64p, c_i64, c_vp, c_size,
                                                 c_vp]),
}


class AbkvError(RuntimeError):
    """A libabkv entry point returned a non-zero status."""

    def __init__(self, fn: str, status: int, detail: str = ""):
        self.status = status
        msg = f"{fn} failed: {status_string(status)} (status {status})"
        if detail:
            msg += f": {detail}"
        super().__init__(msg)


def lib() -> C.CDLL:
    """Load libabkv.so once (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not _LIB_PATH.exists():
                raise RuntimeError(
                    f"{_LIB_PATH} is missing: build it with `python -m abridgekv_b200.build` "
                    "(the sm_100a kernels have no fallback)"
                )
            handle = C.CDLL(str(_LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def status_string(status: int) -> str:
    return lib().abkv_status_string(status).decode()


def check(fn: str, status: int, detail: str = "") -> None:
    if status != 0:
        raise AbkvError(fn, status, detail)


def ptr_array(values) -> C.Array:
    arr = (C.c_void_p * len(values))()
    for i, v in enumerate(values):
        arr[i] = int(v)
    return arr


def i64_array(values) -> C.Array:
    arr = (C.c_int64 * len(values))()
    for i, v in enumerate(values):
        arr[i] = int(v)
    return arr


def i32_array(values) -> C.Array:
    arr = (C.c_int32 * len(values))()
    for i, v in enumerate(values):
        arr[i] = int(v)
    return arr
