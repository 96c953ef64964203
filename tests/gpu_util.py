"""Shared helpers of the GPU parity tests (test infrastructure)."""
import numpy as np
import torch

from oracle import oracle

DT = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}
# Parity tolerance on values (relative to the row's largest top-k magnitude).
# BASELINE.json's contract is 1e-2 for bf16/fp16 and 1e-5 for fp32; the tests
# use 1e-3 for the 16-bit types (products are exact in fp32, only the fp32
# accumulation order differs from the float64 oracle).
RTOL = {"fp32": 1e-5, "fp16": 1e-3, "bf16": 1e-3}


def device_inputs(X, W, b, dtype_name, device="cuda"):
    """Move float32 numpy inputs to the GPU in the given dtype.

    Returns the device tensors and float32 numpy copies of exactly the values
    the GPU sees (rounded to the dtype), which is what the oracle must score.
    """
    dt = DT[dtype_name]
    Xt = torch.from_numpy(np.ascontiguousarray(X)).to(dt)
    Wt = torch.from_numpy(np.ascontiguousarray(W)).to(dt)
    bt = torch.from_numpy(np.ascontiguousarray(b)).float()
    Xr, Wr = Xt.float().numpy(), Wt.float().numpy()
    return Xt.to(device), Wt.to(device), bt.to(device), Xr, Wr, bt.numpy()


def check(V, I, Xr, Wr, br, k, rtol, oracle_res=None):
    V = V.cpu().numpy()
    I = I.cpu().numpy()
    assert V.dtype == np.float32 and I.dtype == np.int32
    assert np.all(np.diff(V, axis=1) <= 0), "rows must be descending"
    chk = oracle.check_topk(V, I, Xr, Wr, br, k, rtol=rtol, oracle=oracle_res)
    chk.raise_if_bad()
    assert chk.tie_recall == 1.0
    return chk


def no_device_error():
    from streamtopk_sae import _capi
    assert _capi.device_error(torch.cuda.current_stream().cuda_stream) == 0
