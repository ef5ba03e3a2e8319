"""ctypes binding of the C ABI declared in include/heterocache_b200.h.

The shared library is built in-tree (``heterocache_b200/libhcb200.so``) by
``heterocache_b200.build``.  There is no fallback: importing an op without the
library raises, so a missing build can never silently route work elsewhere.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import c_double, c_float, c_int, c_int64, c_longlong, c_size_t, c_void_p

LIB_NAME = "libhcb200.so"
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), LIB_NAME)

# Every entry point the header declares, with its ctypes signature.
SIGNATURES = {
    "hc_abi_version": (c_int, []),
    "hc_status_string": (ctypes.c_char_p, [c_int]),
    "hc_last_cuda_error": (ctypes.c_char_p, []),
    "hc_set_wait_limits": (c_int, [ctypes.c_ulonglong, c_int]),
    "hc_prefill_keep": (c_int, [c_int, c_int, c_int, c_int, c_int, c_void_p, c_int, c_void_p, c_void_p,
                                c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_int,
                                c_void_p, c_int, c_void_p, c_void_p, c_void_p]),
    "hc_prefill_select_workspace_size": (c_size_t, [c_int, c_int, c_int, c_int, c_int, c_int]),
    "hc_prefill_select": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                                  c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_int64,
                                  c_int64, c_int64, c_int64, c_int64,
                                  c_void_p, c_int, c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p,
                                  c_void_p, c_void_p, c_void_p, c_size_t, c_void_p, c_void_p]),
    "hc_snapkv_update_kv_workspace_size": (c_size_t, [c_int, c_int, c_int, c_int, c_int]),
    "hc_snapkv_update_kv": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                                    c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_int64,
                                    c_int64, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p,
                                    c_void_p, c_size_t, c_void_p, c_void_p]),
    "hc_pivot_init_workspace_size": (c_size_t, [c_int, c_int, c_int, c_int, c_int]),
    "hc_pivot_init": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                              c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int64, c_int64,
                              c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p, c_void_p]),
    "hc_decode_append": (c_int, [c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                                 c_int64, c_void_p,
                                 c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p, c_int, c_void_p,
                                 c_void_p, c_int64, c_int, c_void_p, c_void_p, c_void_p]),
    "hc_flash_decode_workspace_size": (c_size_t, [c_int, c_int, c_int, c_int]),
    "hc_flash_decode": (c_int, [c_int, c_int, c_int, c_int, c_int, c_void_p, c_int64, c_int64, c_void_p,
                                c_void_p, c_int, c_void_p, c_int, c_void_p, c_float, c_void_p, c_longlong,
                                c_void_p, c_size_t, c_void_p, c_void_p]),
    "hc_flash_decode_with_new": (c_int, [c_int, c_int, c_int, c_int, c_int, c_void_p, c_int64, c_int64, c_void_p,
                                         c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_int64,
                                         c_int64, c_int64, c_int64, c_float, c_void_p, c_void_p, c_void_p, c_size_t,
                                         c_void_p, c_void_p]),
    "hc_flash_decode_noalloc": (c_int, [c_int, c_int, c_int, c_int, c_int, c_void_p, c_int64, c_int64, c_void_p,
                                        c_void_p, c_int, c_void_p, c_int, c_void_p, c_float, c_void_p, c_void_p,
                                        c_void_p]),
    "hc_drift_check_workspace_size": (c_size_t, [c_int, c_int, c_int, c_int, c_int]),
    "hc_drift_check": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_double,
                               c_void_p, c_int64, c_int64, c_void_p, c_int, c_void_p, c_int, c_int, c_void_p,
                               c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                               c_void_p, c_void_p, c_void_p, c_size_t, c_void_p, c_void_p]),
    "hc_drift_check_batch_per_launch": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int]),
    "hc_drift_check_batch_workspace_size": (c_size_t, [c_int, c_int, c_int, c_int, c_int, c_int]),
    "hc_drift_check_batch": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_double,
                                     c_void_p, c_int, c_int, c_void_p, c_size_t, c_void_p, c_void_p]),
    "hc_prefill_attention": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, c_void_p, c_int64, c_int64, c_int64,
                                     c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int64, c_int64,
                                     c_float, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p]),
    "hc_retrieve": (c_int, [c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_int, c_void_p,
                            c_void_p, c_int, c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p,
                            c_int, c_void_p, c_int, c_void_p, c_void_p]),
    "hc_retrieve_delta": (c_int, [c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                  c_int, c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p, c_int64,
                                  c_int64, c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p,
                                  c_void_p, c_int64, c_void_p, c_void_p]),
    "hc_flash_decode_peer": (c_int, [c_int, c_int, c_int, c_int, c_int, c_void_p, c_int64, c_int64, c_void_p,
                                     c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_int64,
                                     c_int64, c_int64, c_int64, c_float, c_void_p, c_void_p, c_int, c_void_p,
                                     c_int64, c_void_p, c_size_t, c_void_p, c_void_p]),
    "hc_peer_barrier": (c_int, [c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p]),
    "hc_peer_put": (c_int, [c_int, c_void_p, c_void_p, c_int, c_void_p, c_void_p]),
    "hc_enable_peer_access": (c_int, [c_int]),
    "hc_ipc_export": (c_int, [c_void_p, c_void_p, c_void_p]),
    "hc_ipc_open": (c_int, [c_void_p, c_void_p]),
    "hc_ipc_close": (c_int, [c_void_p]),
    "hc_profile_topk_workspace_size": (c_size_t, [c_int, c_int, c_int]),
    "hc_profile_topk": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, c_void_p, c_int64, c_int64, c_int64,
                                c_int64, c_int, c_int, c_void_p, c_int64, c_void_p, c_size_t, c_void_p]),
    "hc_profile_overlap": (c_int, [c_void_p, c_int64, c_int, c_void_p, c_int64, c_int, c_int64, c_int, c_void_p,
                                   c_void_p]),
}



class DriftJob(ctypes.Structure):
    """``hc_drift_job``: one drift check of a batch (device pointers)."""
    _fields_ = [("qbuf", c_void_p), ("qss", c_int64), ("qsh", c_int64), ("k_pool", c_void_p),
                ("block_table", c_void_p), ("n_pool_blocks", c_int), ("max_blocks", c_int),
                ("pivot_head", c_int), ("max_len", c_int), ("ref_bitmap", c_void_p),
                ("ref_positions", c_void_p), ("trigger", c_void_p), ("retrieve_positions", c_void_p),
                ("coeffs", c_void_p), ("median", c_void_p), ("out_scores", c_void_p)]


_LIB = None


def library_path() -> str:
    return LIB_PATH


def lib() -> ctypes.CDLL:
    """Load the CUDA library (once) or raise if it has not been built."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"heterocache_b200: the sm_100a library {LIB_PATH} is not built; run "
                "`python -c 'import heterocache_b200.build as b; b.build()'` first")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        if handle.hc_abi_version() != 1:
            raise RuntimeError("heterocache_b200: library ABI version mismatch")
        _LIB = handle
    return _LIB


class HCError(RuntimeError):
    """A status code returned by the C ABI."""

    def __init__(self, op: str, code: int):
        l = lib()
        msg = l.hc_status_string(code).decode()
        cuda = l.hc_last_cuda_error().decode()
        super().__init__(f"{op}: {msg} (status {code})" + (f" [{cuda}]" if code == 5 and cuda else ""))
        self.code = code


def check(op: str, code: int) -> None:
    if code != 0:
        raise HCError(op, code)
