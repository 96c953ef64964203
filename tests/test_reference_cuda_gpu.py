"""The reference's own CUDA op on the same B200, beside this build.

oracle/build_ref.py --cuda compiles the reference's four sources (its
setup.py:15-38 flags, sm_100a instead of sm_80/86/89) into
oracle/_ref/cuda/streamtopk_sae_native_cuda*.so; test infrastructure only.
Both ops run on the same seeded inputs at BASELINE.json's configs[1] and
configs[2] shapes: each result is checked against the float64 oracle
(tie-aware) and both are timed with CUDA events, so the reference's GPU
speed on this hardware is measured, not assumed.  Skipped when the module
was not built.
"""
import glob
import importlib.util
import os

import numpy as np
import pytest
import torch

from gpu_util import RTOL, HostRows, check, no_device_error, sample_rows
from oracle import oracle

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DT = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}


def _reference_cuda():
    found = glob.glob(os.path.join(REPO, "oracle", "_ref", "cuda", "streamtopk_sae_native_cuda*.so"))
    if not found:
        pytest.skip("reference CUDA op not built (python oracle/build_ref.py --ref <tree> --cuda)")
    spec = importlib.util.spec_from_file_location("streamtopk_sae_native_cuda", found[0])
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _time_ms(fn, n):
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(n):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / n


def _sorted(V, I):
    order = torch.argsort(V, dim=1, descending=True)
    return torch.gather(V, 1, order), torch.gather(I, 1, order)


@pytest.mark.parametrize("cfg", ["cfg2_bf16", "cfg2_fp32", "cfg3_bf16"])
def test_reference_cuda_beside_b200(cfg):
    import streamtopk_sae as stk
    ref = _reference_cuda()
    if cfg.startswith("cfg2"):
        B, d, F, k, w_init, n = 128, 768, 65536, 32, "normal_1_over_d", 20
    else:
        B, d, F, k, w_init, n = 128, 2048, 262144, 64, "unit_rows", 5
    dtype_name = cfg.split("_")[1]
    X, W, b = stk.make_inputs(B, d, F, dtype=DT[dtype_name], seed=5, device="cuda", w_init=w_init)
    # The reference launches on the legacy default stream: run it there.
    torch.cuda.synchronize()
    Vr, Ir = ref.streamtopk_cuda_exact_forward(X, W, b, k)
    torch.cuda.synchronize()
    V, I = stk.topk_sae_cuda_exact(X, W, b, k)
    torch.cuda.synchronize()
    no_device_error()
    Vr, Ir = _sorted(Vr.float(), Ir.int())
    Xr, Wh, br = X.float().cpu().numpy(), HostRows(W), b.cpu().numpy()
    rows = sample_rows(8, B, seed=1)
    rt = torch.from_numpy(rows).to(V.device)
    ok = check(V[rt], I[rt], Xr[rows], Wh, br, k, RTOL[dtype_name])
    # The reference's result against the same float64 oracle (its fp32 FMA
    # accumulation order differs; the tolerance is the contract's).
    rchk = oracle.check_topk(Vr[rt].cpu().numpy(), Ir[rt].cpu().numpy(), Xr[rows], Wh, br, k,
                             rtol=1e-2 if dtype_name != "fp32" else 1e-5)
    ms_ref = _time_ms(lambda: ref.streamtopk_cuda_exact_forward(X, W, b, k), n)
    ms_b200 = _time_ms(lambda: stk.topk_sae_cuda_exact(X, W, b, k), n)
    print(f"\n[{cfg}] B={B} d={d} F={F} k={k}: reference CUDA (sm_100a rebuild) {ms_ref:.3f} ms "
          f"= {B / ms_ref * 1e3:,.0f} rows/s; this build {ms_b200:.3f} ms = {B / ms_b200 * 1e3:,.0f} rows/s; "
          f"{ms_ref / ms_b200:.1f}x; reference tie-recall {rchk.tie_recall:.4f}, this build {ok.tie_recall:.4f}")
    assert ms_b200 < ms_ref
