"""FP8 (E4M3) W_enc streaming: half the HBM bytes of bf16 per encode.

An extension beyond the reference (whose dtype set is fp32 / fp16 / bf16,
streamtopk_sae/csrc/cuda/streamtopk_exact.cu:803-804).  W_enc is stored once as
E4M3 with one fp32 scale per feature; every encode quantizes X per row to E4M3
on the GPU and runs the fused kernel on the tensor cores' kind::f8f6f4 path
with fp32 accumulation:

    score[r][f] = x_scale[r] * w_scale[f] * (X8[r] . W8[f]) + b_enc[f]

``topk_sae_cuda_exact_fp8`` returns the exact top-k of these scores (sorted,
ties by smaller index, like ``topk_sae_cuda_exact``); against the unquantized
scores it is an approximation (E4M3 keeps 3 mantissa bits), so compare it by
recall, not by parity.

    W8, w_scale = quantize_weights(W_enc)                    # once
    vals, idxs = topk_sae_cuda_exact_fp8(X, W8, w_scale, b_enc, k)
"""
from __future__ import annotations

import torch

from . import _capi
from .native import _DTYPE_CODE, _require

E4M3 = torch.float8_e4m3fn


def quantize_rows(X: torch.Tensor):
    """Per-row E4M3 quantization on the GPU (stk_quantize_rows_fp8):
    scale[r] = max_j |x[r][j]| / 448 (1 for an all-zero row) and
    Q[r][j] = E4M3(x[r][j] * 448 / max_j |x[r][j]|), round to nearest even,
    saturating; X ~= scale[:, None] * Q.  Returns (Q as float8_e4m3fn, scale)."""
    _require(X.is_cuda and X.dim() == 2 and X.is_contiguous(), "X must be a contiguous 2-D CUDA tensor")
    _require(X.dtype in _DTYPE_CODE, "X dtype must be fp32, fp16, or bf16")
    rows, d = X.shape
    _require(d % 16 == 0, "d must be a multiple of 16")
    Q = torch.empty((rows, d), dtype=E4M3, device=X.device)
    scale = torch.empty((rows,), dtype=torch.float32, device=X.device)
    with torch.cuda.device(X.device):
        stream = torch.cuda.current_stream(X.device).cuda_stream
        _capi.check(_capi.load().stk_quantize_rows_fp8(X.data_ptr(), _DTYPE_CODE[X.dtype], Q.data_ptr(),
                                                       scale.data_ptr(), rows, d, stream))
    return Q, scale


def quantize_weights(W_enc: torch.Tensor):
    """W_enc (F, d) -> (W8 E4M3 (F, d), w_scale fp32 (F,)), one scale per feature."""
    return quantize_rows(W_enc.contiguous())


def topk_sae_cuda_exact_fp8(X, W8, w_scale, b_enc, k, flags=0):
    """Top-k of x_scale * w_scale * (X8 . W8) + b_enc per row of X (see module doc)."""
    _require(X.is_cuda and W8.is_cuda and w_scale.is_cuda and b_enc.is_cuda, "inputs must be on CUDA")
    _require(X.dim() == 2 and W8.dim() == 2, "X and W8 must be 2-D")
    X = X.contiguous()
    W8 = W8.contiguous()
    b_enc = b_enc.float().contiguous()
    w_scale = w_scale.float().contiguous()
    _require(X.dtype in _DTYPE_CODE, "X dtype must be fp32, fp16, or bf16")
    _require(W8.dtype == E4M3, "W8 must be float8_e4m3fn")
    B, d = X.shape
    F = W8.shape[0]
    _require(W8.shape[1] == d, "W_enc d-dim mismatch")
    _require(b_enc.shape == (F,) and w_scale.shape == (F,), "b_enc / w_scale F-dim mismatch")
    k = int(k)
    _require(1 <= k <= F, "k out of range")
    V = torch.empty((B, k), dtype=torch.float32, device=X.device)
    I = torch.empty((B, k), dtype=torch.int32, device=X.device)
    with torch.cuda.device(X.device):
        nbytes = _capi.workspace_bytes_fp8(B, d, F, k)
        ws = torch.empty(max(nbytes, 8), dtype=torch.uint8, device=X.device)
        stream = torch.cuda.current_stream(X.device).cuda_stream
        _capi.check(_capi.load().stk_exact_forward_fp8(
            X.data_ptr(), _DTYPE_CODE[X.dtype], W8.data_ptr(), w_scale.data_ptr(), b_enc.data_ptr(),
            V.data_ptr(), I.data_ptr(), B, d, F, k, flags, ws.data_ptr(), nbytes, stream))
    return V, I
