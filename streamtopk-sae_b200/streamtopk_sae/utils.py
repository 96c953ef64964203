"""Helpers kept from the reference API: recall and seeded inputs.

``recall_at_k`` follows streamtopk_sae/utils.py:23-36 (mean set overlap / k).
``make_inputs`` produces BASELINE.json-style Gaussian inputs with a seeded
torch.Generator: X ~ N(0, 1); W_enc ~ N(0, 1/d) or rows N(0, 1) scaled to unit
L2 norm; b_enc ~ N(0, bias_std^2) in fp32.  (The reference's default
synthetic generator is test data only and is not part of this package.)
"""
from __future__ import annotations

import torch

DTYPE_MAP = {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32}


def str_to_dtype(s):
    if s not in DTYPE_MAP:
        raise ValueError(f"Unknown dtype '{s}'. Choose from: {list(DTYPE_MAP)}")
    return DTYPE_MAP[s]


def recall_at_k(pred_idxs, true_idxs):
    """Mean over rows of |pred & true| / k (indices as (B, k) tensors)."""
    B, k = true_idxs.shape
    p = pred_idxs.detach().cpu().tolist()
    t = true_idxs.detach().cpu().tolist()
    return sum(len(set(a) & set(b)) / k for a, b in zip(p, t)) / B


def make_inputs(B, d, F, dtype=torch.bfloat16, seed=0, device="cuda", w_init="normal_1_over_d", bias_std=0.1):
    """Seeded Gaussian SAE inputs, generated on `device` with a torch.Generator."""
    dev = torch.device(device)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    X = torch.randn(B, d, generator=g, device=dev, dtype=torch.float32)
    W = torch.empty(F, d, device=dev, dtype=dtype)
    chunk = max(1, (1 << 26) // max(d, 1))
    for f0 in range(0, F, chunk):
        f1 = min(F, f0 + chunk)
        w = torch.randn(f1 - f0, d, generator=g, device=dev, dtype=torch.float32)
        if w_init == "unit_rows":
            w = w / w.norm(dim=1, keepdim=True).clamp_min(1e-8)
        else:
            w = w * (1.0 / d ** 0.5)
        W[f0:f1] = w.to(dtype)
    b = torch.randn(F, generator=g, device=dev, dtype=torch.float32) * bias_std
    return X.to(dtype), W, b
