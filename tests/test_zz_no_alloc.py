"""The allocation-free exact encode (stk_exact_forward_noalloc) on a GPU.

Some callers cannot allocate device memory at all (code running inside an
allocator's hooks, plugins whose host application owns every allocation,
fixed-memory embedded or real-time code), so the library offers an entry point
that needs no workspace: its scratch is an array built into the library.  These
tests call it through the C ABI and check, on two calls in a row with different
inputs (the shared scratch keeps the previous call's contents), that it returns
what the workspace-based entry point returns.  This file is named so that
pytest collects it last.
"""
import ctypes

import numpy as np
import pytest
import torch

from gpu_util import RTOL, device_inputs
from oracle import oracle

pytestmark = pytest.mark.gpu

BF16 = 2


def _noalloc(lib, Xt, Wt, bt, k):
    B, d = Xt.shape
    F = Wt.shape[0]
    V = torch.empty((B, k), dtype=torch.float32, device=Xt.device)
    I = torch.empty((B, k), dtype=torch.int32, device=Xt.device)
    rc = lib.stk_exact_forward_noalloc(Xt.data_ptr(), Wt.data_ptr(), bt.data_ptr(), V.data_ptr(), I.data_ptr(),
                                       B, d, F, k, BF16, 0, torch.cuda.current_stream().cuda_stream)
    return rc, V, I


def test_noalloc_matches_workspace_entry_point_twice():
    import streamtopk_sae as stk
    from streamtopk_sae import _capi
    lib = _capi.load()
    k = 64
    for call, (B, d, F) in enumerate([(128, 512, 60000), (100, 256, 33000)]):
        X, W, b = oracle.gaussian_inputs(B, d, F, seed=100 + call)
        Xt, Wt, bt, *_ = device_inputs(X, W, b, "bf16")
        V0, I0 = stk.topk_sae_cuda_exact(Xt, Wt, bt, k)
        rc, V, I = _noalloc(lib, Xt, Wt, bt, k)
        _capi.check(rc)
        torch.cuda.synchronize()
        assert _capi.device_error(torch.cuda.current_stream().cuda_stream) == 0
        tol = RTOL["bf16"] * V0.abs().amax(dim=1, keepdim=True)
        assert torch.all((V - V0).abs() <= tol), f"call {call}: values differ"
        assert torch.equal(I, I0), f"call {call}: indices differ"


def test_noalloc_rejects_shapes_beyond_its_scratch():
    from streamtopk_sae import _capi
    lib = _capi.load()
    B, d, F, k = 4096, 64, 1 << 20, 128   # needs far more than the built-in 24 MiB
    Xt = torch.zeros((1, d), dtype=torch.bfloat16, device="cuda")
    rc = lib.stk_exact_forward_noalloc(Xt.data_ptr(), Xt.data_ptr(), Xt.data_ptr(), Xt.data_ptr(), Xt.data_ptr(),
                                       B, d, F, k, BF16, 0, torch.cuda.current_stream().cuda_stream)
    assert rc == _capi.STK_ENOSPACE
    msg = lib.stk_last_error().decode()
    assert "built-in scratch holds" in msg and "stk_exact_forward" in msg
