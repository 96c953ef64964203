"""ctypes binding of libstk_b200.so (C ABI: include/stk_b200.h).

The library is the only compute path: if it is missing, every op raises.
There is no CPU or PyTorch fallback.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libstk_b200.so")

STK_OK, STK_EINVAL, STK_ECUDA, STK_EDEVICE, STK_ENOSPACE = 0, 1, 2, 3, 4
STK_F32, STK_F16, STK_BF16, STK_E4M3 = 0, 1, 2, 3
STK_FLAG_ANY_K, STK_FLAG_ANY_D, STK_FLAG_SIMT, STK_FLAG_NO_PILOT, STK_FLAG_TF32 = 1, 2, 4, 8, 16
STK_FLAG_SEPARATE_FINISH, STK_FLAG_NO_PAIR = 32, 64

EXPORTS = (
    "stk_version", "stk_last_error", "stk_list_len", "stk_workspace_bytes",
    "stk_exact_forward", "stk_approx_forward", "stk_approx_candidates",
    "stk_shard_forward", "stk_merge_keys", "stk_device_error",
    "stk_profile_begin", "stk_profile_end", "stk_exact_forward_noalloc", "stk_candidates_workspace_bytes",
    "stk_exchange_bytes", "stk_exchange_create", "stk_exchange_ipc_handle", "stk_exchange_connect",
    "stk_exchange_forward", "stk_exchange_destroy",
    "stk_workspace_bytes_fp8", "stk_exact_forward_fp8", "stk_quantize_rows_fp8",
    "stk_approx_cand_workspace_bytes", "stk_approx_forward_cand", "stk_decode_forward",
    "stk_pipeline_workspace_bytes", "stk_pipeline_create", "stk_pipeline_submit", "stk_pipeline_flush",
    "stk_pipeline_pipelined", "stk_pipeline_destroy", "stk_pipeline_create_sharded",
)
IPC_HANDLE_BYTES = 64

_lib = None
_lock = threading.Lock()


class NativeLibraryMissing(RuntimeError):
    pass


def load():
    """Load and type the library (once)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.isfile(LIB_PATH):
            raise NativeLibraryMissing(
                f"streamtopk_sae native library not built ({LIB_PATH} missing). "
                "Run: make -C streamtopk-sae_b200")
        L = ctypes.CDLL(LIB_PATH)
        i64, i32, vp, sz = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t
        L.stk_version.restype = i32
        L.stk_version.argtypes = []
        L.stk_last_error.restype = ctypes.c_char_p
        L.stk_last_error.argtypes = []
        L.stk_list_len.restype = i32
        L.stk_list_len.argtypes = [i64]
        L.stk_workspace_bytes.restype = i32
        L.stk_workspace_bytes.argtypes = [i64, i64, i64, i64, i32, ctypes.POINTER(sz)]
        L.stk_exact_forward.restype = i32
        L.stk_exact_forward.argtypes = [vp, vp, vp, vp, vp, i64, i64, i64, i64, i32, i32, vp, sz, vp]
        L.stk_approx_forward.restype = i32
        L.stk_approx_forward.argtypes = [vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, i32, i32, vp, sz, vp]
        L.stk_approx_candidates.restype = i32
        L.stk_approx_candidates.argtypes = [vp, vp, vp, vp, vp, i64, i64, i64, i64, i32, vp, sz, vp]
        L.stk_candidates_workspace_bytes.restype = i32
        L.stk_candidates_workspace_bytes.argtypes = [i64, i64, i64, i64, i32, ctypes.POINTER(sz)]
        L.stk_shard_forward.restype = i32
        L.stk_shard_forward.argtypes = [vp, vp, vp, vp, i64, i64, i64, i64, i64, i32, i32, vp, sz, vp]
        L.stk_merge_keys.restype = i32
        L.stk_merge_keys.argtypes = [vp, i64, i64, i64, vp, vp, vp]
        L.stk_exact_forward_noalloc.restype = i32
        L.stk_exact_forward_noalloc.argtypes = [vp, vp, vp, vp, vp, i64, i64, i64, i64, i32, i32, vp]
        L.stk_profile_begin.restype = i32
        L.stk_profile_begin.argtypes = [i64]
        L.stk_profile_end.restype = i32
        L.stk_profile_end.argtypes = [ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_int64)]
        L.stk_device_error.restype = i32
        L.stk_device_error.argtypes = [vp, ctypes.POINTER(ctypes.c_uint)]
        L.stk_exchange_bytes.restype = i32
        L.stk_exchange_bytes.argtypes = [i32, i64, i64, ctypes.POINTER(sz)]
        L.stk_exchange_create.restype = i32
        L.stk_exchange_create.argtypes = [i32, i32, i64, i64, vp, sz, ctypes.c_double, ctypes.POINTER(vp)]
        L.stk_exchange_ipc_handle.restype = i32
        L.stk_exchange_ipc_handle.argtypes = [vp, vp, ctypes.POINTER(i64)]
        L.stk_exchange_connect.restype = i32
        L.stk_exchange_connect.argtypes = [vp, vp, vp]
        L.stk_exchange_forward.restype = i32
        L.stk_exchange_forward.argtypes = [vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, i32, i32, vp, sz, vp]
        L.stk_exchange_destroy.restype = i32
        L.stk_exchange_destroy.argtypes = [vp]
        L.stk_workspace_bytes_fp8.restype = i32
        L.stk_workspace_bytes_fp8.argtypes = [i64, i64, i64, i64, ctypes.POINTER(sz)]
        L.stk_exact_forward_fp8.restype = i32
        L.stk_exact_forward_fp8.argtypes = [vp, i32, vp, vp, vp, vp, vp, i64, i64, i64, i64, i32, vp, sz, vp]
        L.stk_quantize_rows_fp8.restype = i32
        L.stk_quantize_rows_fp8.argtypes = [vp, i32, vp, vp, i64, i64, vp]
        L.stk_approx_cand_workspace_bytes.restype = i32
        L.stk_approx_cand_workspace_bytes.argtypes = [i64, i64, i64, i64, i64, i32, ctypes.POINTER(sz)]
        L.stk_decode_forward.restype = i32
        L.stk_decode_forward.argtypes = [vp, vp, vp, vp, vp, i64, i64, i64, i64, i32, vp]
        L.stk_approx_forward_cand.restype = i32
        L.stk_approx_forward_cand.argtypes = [vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, i32, i32, vp, sz,
                                              vp]
        L.stk_pipeline_workspace_bytes.restype = i32
        L.stk_pipeline_workspace_bytes.argtypes = [i64, i64, i64, i64, i32, i32, ctypes.POINTER(sz)]
        L.stk_pipeline_create.restype = i32
        L.stk_pipeline_create.argtypes = [ctypes.POINTER(vp), i64, i64, i64, i64, i32, i32, vp, sz]
        L.stk_pipeline_submit.restype = i32
        L.stk_pipeline_submit.argtypes = [vp, vp, vp, vp, vp, vp, vp]
        L.stk_pipeline_flush.restype = i32
        L.stk_pipeline_flush.argtypes = [vp, vp]
        L.stk_pipeline_pipelined.restype = i32
        L.stk_pipeline_pipelined.argtypes = [vp]
        L.stk_pipeline_create_sharded.restype = i32
        L.stk_pipeline_create_sharded.argtypes = [ctypes.POINTER(vp), vp, i64, i64, i64, i64, i64, i32, i32, vp, sz]
        L.stk_pipeline_destroy.restype = i32
        L.stk_pipeline_destroy.argtypes = [vp]
        _lib = L
    return _lib


def check(rc: int) -> None:
    """Raise RuntimeError with the library's message for a non-zero status."""
    if rc != STK_OK:
        msg = load().stk_last_error().decode(errors="replace")
        raise RuntimeError(msg)


def workspace_bytes(B: int, d: int, F: int, k: int, dtype_code: int) -> int:
    out = ctypes.c_size_t(0)
    check(load().stk_workspace_bytes(B, d, F, k, dtype_code, ctypes.byref(out)))
    return int(out.value)


def workspace_bytes_fp8(B: int, d: int, F: int, k: int) -> int:
    out = ctypes.c_size_t(0)
    check(load().stk_workspace_bytes_fp8(B, d, F, k, ctypes.byref(out)))
    return int(out.value)


def approx_cand_workspace_bytes(B: int, d: int, F: int, k: int, c: int, dtype_code: int) -> int:
    out = ctypes.c_size_t(0)
    check(load().stk_approx_cand_workspace_bytes(B, d, F, k, c, dtype_code, ctypes.byref(out)))
    return int(out.value)


def candidates_workspace_bytes(B: int, d: int, F: int, c: int, dtype_code: int) -> int:
    out = ctypes.c_size_t(0)
    check(load().stk_candidates_workspace_bytes(B, d, F, c, dtype_code, ctypes.byref(out)))
    return int(out.value)


def list_len(k: int) -> int:
    return int(load().stk_list_len(k))


def device_error(stream_handle: int) -> int:
    """Synchronise the stream; raise if a kernel reported a device-side error."""
    code = ctypes.c_uint(0)
    check(load().stk_device_error(stream_handle, ctypes.byref(code)))
    return int(code.value)


PROFILE_KINDS = ("fused_topk_kernel", "simt_topk_kernel", "finish_kernel", "finish_kernel_exchange")


class KernelTimer:
    """CUDA-event timing of every library kernel launched inside the block.

    >>> with KernelTimer(max_launches=10000) as kt: ...
    >>> kt.ms["fused_topk_kernel"], kt.launches["fused_topk_kernel"]
    """

    def __init__(self, max_launches=100000):
        self.max_launches = max_launches
        self.ms = {}
        self.launches = {}

    def __enter__(self):
        check(load().stk_profile_begin(self.max_launches))
        return self

    def __exit__(self, *exc):
        ms = (ctypes.c_double * 4)()
        n = (ctypes.c_int64 * 4)()
        check(load().stk_profile_end(ms, n))
        self.ms = {k: float(ms[i]) for i, k in enumerate(PROFILE_KINDS)}
        self.launches = {k: int(n[i]) for i, k in enumerate(PROFILE_KINDS)}
        return False
