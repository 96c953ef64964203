"""SAE decoder over the encoder's sparse codes (an extension: the reference
stops at the encoder, README.md:9-14).

    x_hat = b_dec + sum_j vals[:, j, None] * W_dec[idxs[:, j]]

computed by the library's gather kernel (stk_decode_forward): each row reads
its k rows of W_dec once, fp32 accumulation, without forming the dense (B, F)
codes.  ``topk_sae_forward`` is the whole SAE forward: encode (exact top-k)
then decode.
"""
from __future__ import annotations

import torch

from . import _capi
from .native import _DTYPE_CODE, _require


def topk_sae_decode(vals, idxs, W_dec, b_dec=None):
    """x_hat (B, d) fp32 from vals (B, k) fp32 / idxs (B, k) int32 and W_dec (F, d)
    in fp32 / fp16 / bf16; b_dec (d,) optional.  Indices < 0 are skipped."""
    _require(vals.is_cuda and idxs.is_cuda and W_dec.is_cuda, "inputs must be on CUDA")
    _require(vals.dim() == 2 and vals.shape == idxs.shape, "vals and idxs must be (B, k)")
    _require(W_dec.dim() == 2 and W_dec.dtype in _DTYPE_CODE, "W_dec must be (F, d) fp32, fp16 or bf16")
    vals = vals.float().contiguous()
    idxs = idxs.to(torch.int32).contiguous()
    W_dec = W_dec.contiguous()
    B, k = vals.shape
    F, d = W_dec.shape
    if b_dec is not None:
        b_dec = b_dec.float().contiguous()
        _require(b_dec.shape == (d,) and b_dec.device == W_dec.device, "b_dec must be (d,) on W_dec's device")
    out = torch.empty((B, d), dtype=torch.float32, device=W_dec.device)
    with torch.cuda.device(W_dec.device):
        stream = torch.cuda.current_stream(W_dec.device).cuda_stream
        _capi.check(_capi.load().stk_decode_forward(
            vals.data_ptr(), idxs.data_ptr(), W_dec.data_ptr(), b_dec.data_ptr() if b_dec is not None else None,
            out.data_ptr(), B, k, F, d, _DTYPE_CODE[W_dec.dtype], stream))
    return out


def topk_sae_forward(X, W_enc, b_enc, W_dec, b_dec, k):
    """SAE forward: (x_hat (B, d) fp32, vals (B, k), idxs (B, k))."""
    from .ops import topk_sae_cuda_exact
    vals, idxs = topk_sae_cuda_exact(X, W_enc, b_enc, k)
    return topk_sae_decode(vals, idxs, W_dec, b_dec), vals, idxs
