"""Host-side pieces that need no GPU: input generation, recall, dtype names,
and the op layer's argument checks that run before any device work."""
import pytest
import torch

import streamtopk_sae as stk
from streamtopk_sae import utils


def test_make_inputs_seeded_and_shaped():
    X, W, b = stk.make_inputs(4, 16, 40, dtype=torch.float32, seed=3, device="cpu")
    X2, W2, b2 = stk.make_inputs(4, 16, 40, dtype=torch.float32, seed=3, device="cpu")
    assert X.shape == (4, 16) and W.shape == (40, 16) and b.shape == (40,)
    assert b.dtype == torch.float32
    assert torch.equal(X, X2) and torch.equal(W, W2) and torch.equal(b, b2)
    X3, _, _ = stk.make_inputs(4, 16, 40, dtype=torch.float32, seed=4, device="cpu")
    assert not torch.equal(X, X3)


def test_make_inputs_unit_rows_and_dtypes():
    _, W, _ = stk.make_inputs(2, 64, 30, dtype=torch.float32, seed=0, device="cpu", w_init="unit_rows")
    assert torch.allclose(W.norm(dim=1), torch.ones(30), atol=1e-5)
    X, W16, b = stk.make_inputs(2, 64, 30, dtype=torch.bfloat16, seed=0, device="cpu")
    assert X.dtype == torch.bfloat16 and W16.dtype == torch.bfloat16 and b.dtype == torch.float32
    # W ~ N(0, 1/d): row norms near 1
    assert 0.5 < float(W16.float().norm(dim=1).mean()) < 1.5


def test_recall_at_k():
    t = torch.tensor([[1, 2, 3, 4], [5, 6, 7, 8]])
    assert utils.recall_at_k(t, t) == 1.0
    p = torch.tensor([[4, 3, 9, 9], [8, 0, 0, 0]])
    assert utils.recall_at_k(p, t) == pytest.approx((2 / 4 + 1 / 4) / 2)


def test_str_to_dtype():
    assert utils.str_to_dtype("bf16") is torch.bfloat16
    with pytest.raises(ValueError, match="Unknown dtype"):
        utils.str_to_dtype("fp8")


def test_ops_reject_host_tensors_and_bad_dtypes():
    X = torch.zeros(4, 64, dtype=torch.bfloat16)
    W = torch.zeros(128, 64, dtype=torch.bfloat16)
    b = torch.zeros(128)
    with pytest.raises(RuntimeError, match="X must be on CUDA"):
        stk.topk_sae_cuda_exact(X, W, b, 8)
    with pytest.raises(RuntimeError, match="X must be on CUDA"):
        stk.topk_sae_cuda_approx(X, W, b, 8, 16)
    with pytest.raises(RuntimeError, match="not provided by the B200 build"):
        stk.topk_sae_cpu(X, W, b, 8)
