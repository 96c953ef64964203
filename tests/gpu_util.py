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


class HostRows:
    """Row access to a (F, d) matrix held on the host in a 16-bit torch dtype.

    The float64 oracle (oracle.exact_topk_f64 / check_topk) slices W by row
    ranges and by index arrays; this returns those rows as float32 numpy arrays
    (exactly the values the GPU read), so matrices of several GB need not be
    expanded to float32 all at once.
    """

    def __init__(self, t):
        self.t = t.detach().cpu().contiguous()
        self.shape = tuple(self.t.shape)

    def __getitem__(self, key):
        if isinstance(key, np.ndarray):
            key = torch.from_numpy(key.astype(np.int64))
        return self.t[key].float().numpy()


def sample_rows(n_rows, B, seed=0):
    """Sorted row sample (always includes the first and last row)."""
    rng = np.random.default_rng(seed)
    rows = set(rng.choice(B, size=min(n_rows, B), replace=False).tolist()) | {0, B - 1}
    return np.array(sorted(rows), dtype=np.int64)
