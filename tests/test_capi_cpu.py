"""The C-ABI library loads without a GPU, exports every symbol of
include/stk_b200.h, and validates arguments before touching the device.
No kernel is launched here."""
import ctypes
import os
import re

import pytest

from streamtopk_sae import _capi

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _header_symbols():
    txt = open(os.path.join(REPO, "include", "stk_b200.h")).read()
    return sorted(set(re.findall(r"STK_API\s+[\w\s\*]+?\b(stk_\w+)\s*\(", txt)))


def test_library_exports_every_header_symbol():
    lib = _capi.load()
    syms = _header_symbols()
    assert len(syms) >= 10
    for s in syms:
        assert hasattr(lib, s), s
    assert set(syms) == set(_capi.EXPORTS)


def test_version_and_list_len():
    lib = _capi.load()
    assert lib.stk_version() >= 100
    assert [lib.stk_list_len(k) for k in (1, 16, 32, 33, 64, 65, 128, 129)] == [32, 32, 32, 64, 64, 128, 128, 0]


def _exact(lib, B=4, d=64, F=128, k=8, dtype=_capi.STK_BF16, flags=0):
    return lib.stk_exact_forward(None, None, None, None, None, B, d, F, k, dtype, flags, None, 0, None)


@pytest.mark.parametrize("k,msg", [(3, "unsupported k=3. Supported: 1,2,4,8,16,32,64,128."),
                                   (0, "k out of range"), (129, "k out of range")])
def test_exact_argument_messages(k, msg):
    lib = _capi.load()
    assert _exact(lib, k=k) == _capi.STK_EINVAL
    assert msg in lib.stk_last_error().decode()


def test_exact_d_and_dtype_checks():
    lib = _capi.load()
    assert _exact(lib, d=4104) == _capi.STK_EINVAL
    assert "d exceeds D_MAX=4096" in lib.stk_last_error().decode()
    assert _exact(lib, dtype=7) == _capi.STK_EINVAL
    assert "X dtype must be fp32, fp16, or bf16" in lib.stk_last_error().decode()


def test_approx_argument_messages():
    lib = _capi.load()
    rc = lib.stk_approx_forward(None, None, None, None, None, 4, 64, 128, 32, 16, _capi.STK_BF16, 0, None, 0, None)
    assert rc == _capi.STK_EINVAL and "k must be <= c" in lib.stk_last_error().decode()
    rc = lib.stk_approx_forward(None, None, None, None, None, 4, 64, 128, 8, 24, _capi.STK_BF16, 0, None, 0, None)
    assert rc == _capi.STK_EINVAL and "unsupported c=24" in lib.stk_last_error().decode()


def test_ops_fail_loudly_without_library(monkeypatch, tmp_path):
    """The product has no fallback: a missing library raises on use."""
    monkeypatch.setattr(_capi, "_lib", None)
    monkeypatch.setattr(_capi, "LIB_PATH", str(tmp_path / "missing.so"))
    with pytest.raises(_capi.NativeLibraryMissing):
        _capi.load()


def test_exchange_sizes_and_argument_checks():
    """stk_exchange_*: sizes and argument errors that need no GPU."""
    import ctypes
    lib = _capi.load()
    n = ctypes.c_size_t(0)
    assert lib.stk_exchange_bytes(2, 128, 64, ctypes.byref(n)) == _capi.STK_OK
    # receive slots [2][world][rows][L] of int64 keys, counters, step state
    assert n.value >= 2 * 2 * 128 * 64 * 8 + 2 * 2 * 8 + 16
    m = ctypes.c_size_t(0)
    assert lib.stk_exchange_bytes(8, 128, 128, ctypes.byref(m)) == _capi.STK_OK and m.value > n.value
    assert lib.stk_exchange_bytes(9, 128, 64, ctypes.byref(n)) == _capi.STK_EINVAL
    assert "world must be in [1, 8]" in lib.stk_last_error().decode()
    assert lib.stk_exchange_bytes(2, 128, 129, ctypes.byref(n)) == _capi.STK_EINVAL
    h = ctypes.c_void_p()
    assert lib.stk_exchange_create(2, 2, 128, 64, None, 0, 1.0, ctypes.byref(h)) == _capi.STK_EINVAL
    assert "rank out of range" in lib.stk_last_error().decode()
    assert lib.stk_exchange_create(0, 2, 128, 64, None, 0, 0.0, ctypes.byref(h)) == _capi.STK_EINVAL
    assert lib.stk_exchange_create(0, 2, 128, 64, None, 0, 1.0, ctypes.byref(h)) == _capi.STK_ENOSPACE
    assert "exchange buffer too small" in lib.stk_last_error().decode()
    assert not h.value
    assert lib.stk_exchange_forward(None, None, None, None, None, None, 4, 64, 128, 8, 0, _capi.STK_BF16, 0,
                                    None, 0, None) == _capi.STK_EINVAL
    assert lib.stk_exchange_destroy(None) == _capi.STK_OK


def test_p2p_transport_rejects_custom_kernels():
    import torch
    from streamtopk_sae import shard
    W = torch.zeros(128, 16)
    b = torch.zeros(128)
    with pytest.raises(RuntimeError, match="transport 'p2p' runs the library kernels only"):
        shard.ShardedEncoder(W, b, 128, 0, 8, transport="p2p", shard_fn=lambda *a: None)
    with pytest.raises(RuntimeError, match="transport must be"):
        shard.ShardedEncoder(W, b, 128, 0, 8, transport="mpi")


def test_pipeline_argument_checks():
    """The pipelined encode validates its arguments before touching the device."""
    lib = _capi.load()
    n = ctypes.c_size_t(0)
    assert lib.stk_pipeline_workspace_bytes(128, 64, 1000, 0, _capi.STK_BF16, 0, ctypes.byref(n)) == _capi.STK_EINVAL
    assert "k out of range" in lib.stk_last_error().decode()
    assert lib.stk_pipeline_workspace_bytes(128, 64, 1000, 3, _capi.STK_BF16, 0, ctypes.byref(n)) == _capi.STK_EINVAL
    assert "unsupported k=3" in lib.stk_last_error().decode()
    assert lib.stk_pipeline_workspace_bytes(0, 64, 1000, 8, _capi.STK_BF16, 0, ctypes.byref(n)) == _capi.STK_EINVAL
    assert "B must be >= 1" in lib.stk_last_error().decode()
    h = ctypes.c_void_p()
    assert lib.stk_pipeline_create(ctypes.byref(h), 128, 64, 1000, 256, _capi.STK_BF16, _capi.STK_FLAG_ANY_K,
                                   None, 0) == _capi.STK_EINVAL
    assert lib.stk_pipeline_submit(None, None, None, None, None, None, None) == _capi.STK_EINVAL
    assert "pipeline is NULL" in lib.stk_last_error().decode()
    assert lib.stk_pipeline_flush(None, None) == _capi.STK_EINVAL
    assert lib.stk_pipeline_pipelined(None) == 0
    assert lib.stk_pipeline_destroy(None) == _capi.STK_OK
    assert lib.stk_pipeline_create_sharded(ctypes.byref(h), None, 128, 64, 1000, 8, 0, _capi.STK_BF16, 0,
                                           None, 0) == _capi.STK_EINVAL
    assert "exchange is NULL" in lib.stk_last_error().decode()
