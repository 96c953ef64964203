"""The approximate encoder and its per-tile candidates on the GPU.

Mirrors the reference's approx tests (tests/test_recall.py:22-95 and
tests/test_smoke.py:74 in the reference) with stronger checks: the per-tile
top-c candidates of streamtopk_cuda_approx_forward against float64 per-tile
top-c (values within tolerance, indices tie-aware, (-FLT_MAX, -1) padding of
short tiles), the approximate result against the exact one (equal for k <= c),
the reference's Python-side final step (torch.topk over the flat candidates),
and tie-aware recall@k = 1 at every c.
"""
import numpy as np
import pytest
import torch

from gpu_util import RTOL, check, device_inputs, no_device_error
from oracle import oracle

pytestmark = pytest.mark.gpu
NEG = float(np.finfo(np.float32).min)  # -FLT_MAX, as float64


def _tile_topc_f64(Xr, Wr, br, c):
    S = oracle.scores_f64(Xr, Wr, br)
    B, F = S.shape
    T = (F + 127) // 128
    out_v = np.full((B, T, c), NEG)
    out_i = np.full((B, T, c), -1, np.int64)
    for t in range(T):
        f0, f1 = 128 * t, min(F, 128 * t + 128)
        sub = S[:, f0:f1]
        n = min(c, f1 - f0)
        idx = np.argsort(-sub, axis=1, kind="stable")[:, :n]
        out_v[:, t, :n] = np.take_along_axis(sub, idx, axis=1)
        out_i[:, t, :n] = idx + f0
    return S, out_v, out_i


@pytest.mark.parametrize("c", [16, 32, 64, 128])
@pytest.mark.parametrize("dtype_name", ["bf16", "fp32"])
@pytest.mark.parametrize("B,d,F", [(8, 64, 300), (32, 256, 2048), (130, 128, 1000)])
def test_candidates_match_tile_topc(B, d, F, c, dtype_name):
    from streamtopk_sae import native
    X, W, b = oracle.gaussian_inputs(B, d, F, seed=F + c)
    Xt, Wt, bt, Xr, Wr, br = device_inputs(X, W, b, dtype_name)
    fv, fi, cv, ci = native.streamtopk_cuda_approx_forward(Xt, Wt, bt, min(c, 16), c)
    torch.cuda.synchronize()
    no_device_error()
    T = (F + 127) // 128
    assert cv.shape == (B, T, c) and ci.shape == (B, T, c)
    assert fv.shape == (B, T * c) and fv.data_ptr() == cv.data_ptr()
    S, ov, oi = _tile_topc_f64(Xr, Wr, br, c)
    cvn, cin = cv.cpu().numpy().astype(np.float64), ci.cpu().numpy().astype(np.int64)
    pad = oi < 0
    assert np.array_equal(cin < 0, pad), "padding positions differ"
    assert np.all(cvn[pad] == NEG)
    tau = RTOL[dtype_name] * np.maximum(np.abs(np.where(pad, 0, ov)).max(axis=2, keepdims=True), 1e-30)
    real = ~pad
    assert np.all(np.abs(cvn - np.where(pad, NEG, ov))[real] <= np.broadcast_to(tau, ov.shape)[real])
    # each index carries its own score and ranks within the tile's top-c up to ties
    for r in range(B):
        for t in range(T):
            n = int(real[r, t].sum())
            idx = cin[r, t, :n]
            assert len(set(idx.tolist())) == n
            assert np.all((idx >= 128 * t) & (idx < min(F, 128 * t + 128)))
            sc = S[r, idx]
            assert np.all(np.abs(sc - cvn[r, t, :n]) <= tau[r, t, 0])
            assert np.all(sc >= ov[r, t, n - 1] - tau[r, t, 0])


@pytest.mark.parametrize("k,c", [(8, 16), (16, 16), (32, 64), (64, 128), (128, 128)])
def test_approx_equals_exact_when_k_le_c(k, c):
    import streamtopk_sae as stk
    X, W, b = oracle.gaussian_inputs(64, 256, 9000, seed=k + c)
    Xt, Wt, bt, Xr, Wr, br = device_inputs(X, W, b, "bf16")
    Va, Ia = stk.topk_sae_cuda_approx(Xt, Wt, bt, k, c)
    Ve, Ie = stk.topk_sae_cuda_exact(Xt, Wt, bt, k)
    torch.cuda.synchronize()
    assert torch.equal(Va, Ve) and torch.equal(Ia, Ie)
    check(Va, Ia, Xr, Wr, br, k, RTOL["bf16"])


def test_reference_final_step_over_candidates():
    """torch.topk over the flat candidates (reference ops.py:80-81) gives the exact top-k."""
    from streamtopk_sae import native
    X, W, b = oracle.gaussian_inputs(16, 128, 5000, seed=3)
    Xt, Wt, bt, Xr, Wr, br = device_inputs(X, W, b, "bf16")
    fv, fi, _, _ = native.streamtopk_cuda_approx_forward(Xt, Wt, bt, 32, 32)
    V, pos = torch.topk(fv, 32, dim=-1)
    I = fi.gather(1, pos).to(torch.int32)
    check(V, I, Xr, Wr, br, 32, RTOL["bf16"])


def test_candidate_buffer_is_filled():
    import streamtopk_sae as stk
    from streamtopk_sae import native
    X, W, b = oracle.gaussian_inputs(8, 64, 700, seed=4)
    Xt, Wt, bt, *_ = device_inputs(X, W, b, "bf16")
    cb = torch.full((8, 6, 32), 7.0, device="cuda")
    V, I = stk.topk_sae_cuda_approx(Xt, Wt, bt, 16, 32, candidate_buffer=cb)
    _, _, cv, _ = native.streamtopk_cuda_approx_forward(Xt, Wt, bt, 16, 32)
    torch.cuda.synchronize()
    assert torch.equal(cb, cv)
    with pytest.raises(RuntimeError, match="candidate_buffer shape mismatch"):
        stk.topk_sae_cuda_approx(Xt, Wt, bt, 16, 32, candidate_buffer=torch.zeros(8, 5, 32, device="cuda"))


@pytest.mark.parametrize("c", [32, 64, 128])
def test_tie_aware_recall_is_one_at_every_c(c):
    """BASELINE.json config 4 scaled down: recall@k against an exact fp32-input top-k."""
    import streamtopk_sae as stk
    B, d, F, k = 128, 2048, 65536, 32
    X, W, b = oracle.gaussian_inputs(B, d, F, seed=c, w_scale="unit")
    Xt, Wt, bt, Xr, Wr, br = device_inputs(X, W, b, "bf16")
    V, I = stk.topk_sae_cuda_approx(Xt, Wt, bt, k, c)
    ov = oracle.exact_topk_f64(Xr, Wr, br, k)
    assert oracle.tie_aware_recall(I.cpu().numpy(), Xr, Wr, br, k, 1e-3, oracle=ov) == 1.0
    assert oracle.recall_at_k(I.cpu().numpy(), ov[1]) >= 0.999


def test_approx_argument_errors():
    import streamtopk_sae as stk
    X = torch.randn(4, 64, device="cuda", dtype=torch.bfloat16)
    W = torch.randn(128, 64, device="cuda", dtype=torch.bfloat16)
    b = torch.zeros(128, device="cuda")
    with pytest.raises(RuntimeError, match="k must be <= c"):
        stk.topk_sae_cuda_approx(X, W, b, 32, 16)
    with pytest.raises(RuntimeError, match="unsupported c=24"):
        stk.topk_sae_cuda_approx(X, W, b, 8, 24)


@pytest.mark.parametrize("B,d,F,k,c", [(128, 512, 100000, 32, 32), (128, 256, 60037, 16, 16),
                                       (300, 256, 40000, 8, 32), (64, 128, 20000, 32, 32)])
def test_candidates_single_pass_equals_two_pass(B, d, F, k, c):
    """With fp16 / bf16 and c <= 32 the approximate op with a candidate buffer
    is one W_enc pass (the fused kernel also writes each tile's top c): its
    candidates equal the separate candidates pass bit for bit, and its top-k
    the exact op's (k <= c)."""
    import streamtopk_sae as stk
    from streamtopk_sae import native
    X, W, b = oracle.gaussian_inputs(B, d, F, seed=F + c)
    Xt, Wt, bt, *_ = device_inputs(X, W, b, "bf16")
    T = (F + 127) // 128
    cv = torch.empty(B, T, c, device="cuda")
    ci = torch.empty(B, T, c, dtype=torch.int32, device="cuda")
    V1, I1 = native.approx_forward_with_candidates(Xt, Wt, bt, k, c, cv, ci)
    _, _, cv2, ci2 = native.streamtopk_cuda_approx_forward(Xt, Wt, bt, k, c)
    Ve, Ie = stk.topk_sae_cuda_exact(Xt, Wt, bt, k)
    torch.cuda.synchronize()
    no_device_error()
    assert torch.equal(cv, cv2) and torch.equal(ci, ci2)
    assert torch.equal(V1, Ve) and torch.equal(I1, Ie)
