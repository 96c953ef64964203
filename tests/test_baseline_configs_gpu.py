"""Parity at BASELINE.json's own configurations, at their full sizes.

Each configuration runs through the public op (streamtopk_sae.topk_sae_cuda_*)
on seeded inputs with the configuration's distributions (generated on the GPU
by streamtopk_sae.make_inputs) and is checked against the float64 oracle
(oracle.exact_topk_f64 / oracle.check_topk, tie-aware, in F-chunks on the
host):

  configs[1]  B=128 d=768  F=65536    k=32   fp32 / fp16 / bf16, plus its edge set
  configs[2]  B=128 d=2048 F=262144   k=64   bf16 (unit-norm W_enc rows), all rows
  configs[3]  B=128 d=2048 F=1048576  k=32   approx bf16, c in {32, 64, 128}: tie-aware recall@k
  configs[4]  B=4096 d=4096 F=262144  k=128  fp16, a fixed sample of rows

The reference's own tests use the same structure at small sizes
(tests/test_correctness.py:159-284 and tests/test_recall.py:22-95 in the
reference); these are the sizes its benchmark reports.
"""
import numpy as np
import pytest
import torch

from gpu_util import RTOL, HostRows, check, no_device_error, sample_rows
from oracle import oracle

pytestmark = pytest.mark.gpu

DT = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}


def _inputs(B, d, F, dtype_name, seed, w_init):
    import streamtopk_sae as stk
    return stk.make_inputs(B, d, F, dtype=DT[dtype_name], seed=seed, device="cuda", w_init=w_init)


def _host(X, W, b):
    return X.float().cpu().numpy(), HostRows(W), b.cpu().numpy()


@pytest.mark.parametrize("dtype_name", ["fp32", "fp16", "bf16"])
def test_config2_exact_shape(dtype_name):
    import streamtopk_sae as stk
    B, d, F, k = 128, 768, 65536, 32
    X, W, b = _inputs(B, d, F, dtype_name, 2, "normal_1_over_d")
    V, I = stk.topk_sae_cuda_exact(X, W, b, k)
    torch.cuda.synchronize()
    no_device_error()
    Xr, Wr, br = _host(X, W, b)
    check(V, I, Xr, Wr, br, k, RTOL[dtype_name])


@pytest.mark.parametrize("case", ["F_tail", "k1", "zero_x", "outliers"])
@pytest.mark.parametrize("dtype_name", ["fp32", "bf16"])
def test_config2_edge_set(case, dtype_name):
    """configs[1]'s edge set at its shape: F not a multiple of any tile, k = 1,
    all-zero X, +-100 bias on 1% of the features."""
    import streamtopk_sae as stk
    B, d, F, k = 128, 768, 65536, 32
    if case == "F_tail":
        F += 37
    if case == "k1":
        k = 1
    X, W, b = _inputs(B, d, F, dtype_name, 3, "normal_1_over_d")
    if case == "zero_x":
        X.zero_()
    if case == "outliers":
        g = torch.Generator(device="cuda")
        g.manual_seed(7)
        pos = torch.randperm(F, generator=g, device="cuda")[: F // 100]
        sign = torch.where(torch.rand(pos.numel(), generator=g, device="cuda") < 0.5, -100.0, 100.0)
        b[pos] = sign
    V, I = stk.topk_sae_cuda_exact(X, W, b, k)
    torch.cuda.synchronize()
    no_device_error()
    Xr, Wr, br = _host(X, W, b)
    check(V, I, Xr, Wr, br, k, RTOL[dtype_name])


@pytest.mark.parametrize("dtype_name", ["fp32", "fp16", "bf16"])
def test_config2_k_equals_F_4096(dtype_name):
    """configs[1]'s edge case k = F for F = 4096 (the reference rejects it:
    streamtopk_exact.cu:818-830; allowed here under allow_any_k by sorting
    whole rows)."""
    import streamtopk_sae as stk
    B, d, F = 128, 768, 4096
    X, W, b = _inputs(B, d, F, dtype_name, 6, "normal_1_over_d")
    with pytest.raises(RuntimeError, match="unsupported k=4096"):
        stk.topk_sae_cuda_exact(X, W, b, F)
    V, I = stk.topk_sae_cuda_exact(X, W, b, F, allow_any_k=True)
    torch.cuda.synchronize()
    no_device_error()
    Xr, Wr, br = _host(X, W, b)
    check(V, I, Xr, Wr, br, F, RTOL[dtype_name])
    assert torch.equal(torch.sort(I.long(), dim=1).values.cpu(), torch.arange(F).expand(B, F))
    V2, I2 = stk.topk_sae_cuda_exact(X, W, b, 300, allow_any_k=True)   # k > 128 below F
    assert torch.equal(I2, I[:, :300]) and torch.equal(V2, V[:, :300])


def test_config3_full_F():
    """The north-star workload on one GPU, every row checked."""
    import streamtopk_sae as stk
    B, d, F, k = 128, 2048, 262144, 64
    X, W, b = _inputs(B, d, F, "bf16", 0, "unit_rows")
    V, I = stk.topk_sae_cuda_exact(X, W, b, k)
    torch.cuda.synchronize()
    no_device_error()
    Xr, Wr, br = _host(X, W, b)
    check(V, I, Xr, Wr, br, k, RTOL["bf16"])


@pytest.fixture(scope="module")
def config4():
    """configs[3] inputs and the float64 exact top-k of every row (computed once)."""
    B, d, F, k = 128, 2048, 1 << 20, 32
    X, W, b = _inputs(B, d, F, "bf16", 4, "unit_rows")
    Xr, Wr, br = _host(X, W, b)
    ref = oracle.exact_topk_f64(Xr, Wr, br, k, chunk=65536)
    return X, W, b, k, Xr, Wr, br, ref


@pytest.mark.parametrize("c", [32, 64, 128])
def test_config4_approx_recall(config4, c):
    """Approx encode at F = 1M: tie-aware recall@k = 1 at every c (the reference
    reports recall below 1 for its approximate mode, tests/test_recall.py)."""
    import streamtopk_sae as stk
    X, W, b, k, Xr, Wr, br, ref = config4
    V, I = stk.topk_sae_cuda_approx(X, W, b, k, c)
    torch.cuda.synchronize()
    no_device_error()
    In = I.cpu().numpy()
    assert oracle.tie_aware_recall(In, Xr, Wr, br, k, RTOL["bf16"], oracle=ref) == 1.0
    assert oracle.recall_at_k(In, ref[1]) >= 0.999
    check(V, I, Xr, Wr, br, k, RTOL["bf16"], oracle_res=ref)


def test_config5_row_sample():
    """Large batch (B = 4096, compute-bound): a fixed sample of 64 rows checked
    against float64 scores over all F."""
    import streamtopk_sae as stk
    B, d, F, k = 4096, 4096, 262144, 128
    X, W, b = _inputs(B, d, F, "fp16", 5, "normal_1_over_d")
    V, I = stk.topk_sae_cuda_exact(X, W, b, k)
    torch.cuda.synchronize()
    no_device_error()
    rows = sample_rows(62, B, seed=5)
    Xs = X[torch.from_numpy(rows).cuda()].float().cpu().numpy()
    Vs, Is = V.cpu()[torch.from_numpy(rows)], I.cpu()[torch.from_numpy(rows)]
    check(Vs, Is, Xs, HostRows(W), b.cpu().numpy(), k, RTOL["fp16"])
