"""Pin the CPU oracle against the reference's own outputs (golden fixtures).

The fixtures in tests/golden/golden_cpu.npz were produced by the reference's
CPU op compiled from its sources (tests/golden/make_golden.py).  These tests
need no GPU.
"""
import numpy as np
import pytest

from make_golden import GAUSS_CASES, SYN_CASES, digest, gauss_case_inputs
from oracle import oracle


def _syn_inputs(g, name):
    dt = str(g[f"{name}/dtype"])
    if dt == "bf16":
        import torch
        X = torch.from_numpy(g[f"{name}/X_bf16"]).view(torch.bfloat16).float().numpy()
        W = torch.from_numpy(g[f"{name}/W_bf16"]).view(torch.bfloat16).float().numpy()
    else:
        X, W = g[f"{name}/X"], g[f"{name}/W"]
    return X, W, g[f"{name}/b"]


def _same_up_to_fp32_ties(V, I, Vr, Ir, rtol=1e-5):
    """Outputs agree position by position, except where two scores are fp32 ties."""
    assert V.shape == Vr.shape
    tol = rtol * np.maximum(np.abs(Vr).max(axis=1, keepdims=True), 1e-30)
    assert np.all(np.abs(V - Vr) <= tol)
    for r in range(V.shape[0]):
        if not np.array_equal(I[r], Ir[r]):
            # only allowed where the swapped entries carry (near-)equal values
            assert set(I[r].tolist()) == set(Ir[r].tolist()) or np.any(
                np.abs(np.diff(np.sort(Vr[r]))) <= tol[r])


@pytest.mark.parametrize("name", sorted(GAUSS_CASES))
def test_gauss_inputs_reproduce(golden, name):
    B, d, F, k, seed, kind = GAUSS_CASES[name]
    X, W, b = gauss_case_inputs(B, d, F, seed, kind)
    assert str(golden[f"{name}/digest"]) == digest(X, W, b)


@pytest.mark.parametrize("name", sorted(GAUSS_CASES))
def test_c_oracle_matches_reference_gauss(golden, name):
    B, d, F, k, seed, kind = GAUSS_CASES[name]
    X, W, b = gauss_case_inputs(B, d, F, seed, kind)
    V, I = oracle.stream_topk(X, W, b, k)
    _same_up_to_fp32_ties(V, I, golden[f"{name}/V"], golden[f"{name}/I"])


@pytest.mark.parametrize("name", sorted(SYN_CASES))
def test_c_oracle_matches_reference_synthetic(golden, name):
    X, W, b = _syn_inputs(golden, name)
    k = int(golden[f"{name}/meta"][3])
    V, I = oracle.stream_topk(X, W, b, k)
    _same_up_to_fp32_ties(V, I, golden[f"{name}/V"], golden[f"{name}/I"])


@pytest.mark.parametrize("name", sorted(GAUSS_CASES))
def test_f64_oracle_accepts_reference(golden, name):
    """The float64 exact oracle and the reference agree tie-aware at fp32 tolerance."""
    B, d, F, k, seed, kind = GAUSS_CASES[name]
    X, W, b = gauss_case_inputs(B, d, F, seed, kind)
    chk = oracle.check_topk(golden[f"{name}/V"], golden[f"{name}/I"], X, W, b, k, rtol=1e-5)
    chk.raise_if_bad()
    assert chk.tie_recall == 1.0


@pytest.mark.parametrize("name", sorted(SYN_CASES))
def test_f64_oracle_accepts_reference_synthetic(golden, name):
    X, W, b = _syn_inputs(golden, name)
    k = int(golden[f"{name}/meta"][3])
    chk = oracle.check_topk(golden[f"{name}/V"], golden[f"{name}/I"], X, W, b, k, rtol=1e-5)
    chk.raise_if_bad()


def test_heap_order_for_k128(golden):
    """k > 64 returns the reference's min-heap order, not descending order."""
    Vr = golden["gauss_k128/V"]
    assert np.all(Vr[:, 0] <= Vr.min(axis=1) + 0)  # heap root is the row minimum
    assert not np.all(np.diff(Vr, axis=1) <= 0)


def test_big_bias_feature_always_selected(golden):
    assert np.all((golden["gauss_bigbias/I"] == 0).any(axis=1))


def test_check_topk_rejects_a_planted_mistake():
    """The checker catches a wrong index planted in an oracle result (CPU only)."""
    X, W, b = oracle.gaussian_inputs(4, 32, 200, seed=11)
    V, I = oracle.stream_topk(X, W, b, 8)
    assert oracle.check_topk(V, I, X, W, b, 8, rtol=1e-5).ok
    I2 = I.copy()
    ov, oi = oracle.exact_topk_f64(X, W, b, 8, margin=40)
    I2[0, 0] = oi[0, -1]  # a feature ranked ~48th, far below the boundary
    bad = oracle.check_topk(V, I2, X, W, b, 8, rtol=1e-5)
    assert not bad.ok and 0 in bad.bad_rows
    V2 = V.copy()
    V2[1, 3] += 1e-2
    assert not oracle.check_topk(V2, I, X, W, b, 8, rtol=1e-5).ok


def test_exact_topk_chunking_is_consistent():
    X, W, b = oracle.gaussian_inputs(3, 16, 1000, seed=5)
    a = oracle.exact_topk_f64(X, W, b, 10, chunk=1000)
    c = oracle.exact_topk_f64(X, W, b, 10, chunk=97)
    assert np.array_equal(a[1], c[1])
    S = oracle.scores_f64_c(X, W, b, (0, 3), 0, 1000)
    assert np.allclose(S, oracle.scores_f64(X, W, b), rtol=1e-12, atol=1e-12)


def test_recall_helpers():
    X, W, b = oracle.gaussian_inputs(4, 32, 300, seed=3)
    ov, oi = oracle.exact_topk_f64(X, W, b, 16)
    assert oracle.recall_at_k(oi, oi) == 1.0
    assert oracle.tie_aware_recall(oi, X, W, b, 16, 1e-5) == 1.0
    bad = oi.copy()
    bad[:, :4] = (oi[:, :4] + 150) % 300
    assert oracle.tie_aware_recall(bad, X, W, b, 16, 1e-5) < 1.0
