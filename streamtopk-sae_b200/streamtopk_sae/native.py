"""Drop-in for the reference's native module ``streamtopk_sae_native``.

Same function names, arguments, return values and error texts as the
reference's pybind module (streamtopk_sae/csrc/bindings.cpp:28-51), implemented
as torch-level argument checks plus one call into the C ABI of libstk_b200.so.
Outputs and the workspace are allocated here with torch (the C ABI never
allocates); kernels run on the current stream of X's device.
"""
from __future__ import annotations

import torch

from . import _capi

_DTYPE_CODE = {torch.float32: _capi.STK_F32, torch.float16: _capi.STK_F16, torch.bfloat16: _capi.STK_BF16}
T_APPROX = 128  # feature tile of the approximate candidates (streamtopk_approx.cu:31)


def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _common_checks(X, W_enc, b_enc, check_w_b_cuda=True):
    # streamtopk_exact.cu:794-811 / streamtopk_approx.cu:243-259
    _require(X.is_contiguous(), "X must be contiguous")
    _require(W_enc.is_contiguous(), "W_enc must be contiguous")
    _require(b_enc.is_contiguous(), "b_enc must be contiguous")
    _require(X.is_cuda, "X must be on CUDA")
    if check_w_b_cuda:
        _require(W_enc.is_cuda, "W_enc must be on CUDA")
        _require(b_enc.is_cuda, "b_enc must be on CUDA")
    _require(b_enc.dtype == torch.float32, "b_enc must be fp32")
    _require(X.dtype in _DTYPE_CODE, "X dtype must be fp32, fp16, or bf16")
    _require(W_enc.dtype == X.dtype, "W_enc dtype must match X")
    _require(X.dim() == 2 and W_enc.dim() == 2 and b_enc.dim() == 1, "X, W_enc must be 2-D and b_enc 1-D")
    B, d = X.shape
    F = W_enc.shape[0]
    _require(W_enc.shape[1] == d, "W_enc d-dim mismatch")
    _require(b_enc.shape[0] == F, "b_enc F-dim mismatch")
    _require(W_enc.device == X.device and b_enc.device == X.device,
             "X, W_enc and b_enc must be on the same device")
    return B, d, F


def _workspace(X, B, d, F, k):
    nbytes = _capi.workspace_bytes(B, d, F, k, _DTYPE_CODE[X.dtype])
    return torch.empty(max(nbytes, 8), dtype=torch.uint8, device=X.device), nbytes


def streamtopk_cuda_exact_forward(X, W_enc, b_enc, k, flags=0):
    """Reference: streamtopk_sae/csrc/cuda/streamtopk_exact.cu:788-833."""
    B, d, F = _common_checks(X, W_enc, b_enc)
    k = int(k)
    _require(1 <= k <= F, "k out of range")
    _require(d <= 4096 or (flags & _capi.STK_FLAG_ANY_D), "d exceeds D_MAX=4096")
    _require(k in (1, 2, 4, 8, 16, 32, 64, 128) or ((flags & _capi.STK_FLAG_ANY_K) and (k <= 128 or F <= 4096)),
             f"streamtopk_cuda_exact: unsupported k={k}. Supported: 1,2,4,8,16,32,64,128.")
    V = torch.empty((B, k), dtype=torch.float32, device=X.device)
    I = torch.empty((B, k), dtype=torch.int32, device=X.device)
    lib = _capi.load()
    with torch.cuda.device(X.device):
        ws, nbytes = _workspace(X, B, d, F, k)
        stream = torch.cuda.current_stream(X.device).cuda_stream
        _capi.check(lib.stk_exact_forward(X.data_ptr(), W_enc.data_ptr(), b_enc.data_ptr(), V.data_ptr(),
                                          I.data_ptr(), B, d, F, k, _DTYPE_CODE[X.dtype], flags, ws.data_ptr(),
                                          nbytes, stream))
    return V, I


def approx_topk_forward(X, W_enc, b_enc, k, c, flags=0):
    """Final (B, k) result of the approximate path (stk_approx_forward)."""
    B, d, F = _common_checks(X, W_enc, b_enc, check_w_b_cuda=False)
    k, c = int(k), int(c)
    _require(1 <= k <= c, "k must be <= c")
    _require(c in (16, 32, 64, 128), f"streamtopk_cuda_approx: unsupported c={c}. Supported: 16,32,64,128.")
    _require(W_enc.is_cuda and b_enc.is_cuda, "W_enc and b_enc must be on CUDA")
    V = torch.empty((B, k), dtype=torch.float32, device=X.device)
    I = torch.empty((B, k), dtype=torch.int32, device=X.device)
    lib = _capi.load()
    with torch.cuda.device(X.device):
        ws, nbytes = _workspace(X, B, d, F, k)
        stream = torch.cuda.current_stream(X.device).cuda_stream
        _capi.check(lib.stk_approx_forward(X.data_ptr(), W_enc.data_ptr(), b_enc.data_ptr(), V.data_ptr(),
                                           I.data_ptr(), B, d, F, k, c, _DTYPE_CODE[X.dtype], flags,
                                           ws.data_ptr(), nbytes, stream))
    return V, I


def approx_forward_with_candidates(X, W_enc, b_enc, k, c, cand_vals, cand_idxs, flags=0):
    """Final (B, k) result of the approximate path and, into cand_vals /
    cand_idxs (B, ceil(F/128), c), each 128-feature tile's top c
    (stk_approx_forward_cand: one W_enc pass for fp16 / bf16 with c <= 32)."""
    B, d, F = _common_checks(X, W_enc, b_enc, check_w_b_cuda=False)
    k, c = int(k), int(c)
    _require(1 <= k <= c, "k must be <= c")
    _require(c in (16, 32, 64, 128), f"streamtopk_cuda_approx: unsupported c={c}. Supported: 16,32,64,128.")
    _require(W_enc.is_cuda and b_enc.is_cuda, "W_enc and b_enc must be on CUDA")
    V = torch.empty((B, k), dtype=torch.float32, device=X.device)
    I = torch.empty((B, k), dtype=torch.int32, device=X.device)
    lib = _capi.load()
    with torch.cuda.device(X.device):
        nbytes = _capi.approx_cand_workspace_bytes(B, d, F, k, c, _DTYPE_CODE[X.dtype])
        ws = torch.empty(max(nbytes, 8), dtype=torch.uint8, device=X.device)
        stream = torch.cuda.current_stream(X.device).cuda_stream
        _capi.check(lib.stk_approx_forward_cand(X.data_ptr(), W_enc.data_ptr(), b_enc.data_ptr(), V.data_ptr(),
                                                I.data_ptr(), cand_vals.data_ptr(), cand_idxs.data_ptr(), B, d, F, k,
                                                c, _DTYPE_CODE[X.dtype], flags, ws.data_ptr(), nbytes, stream))
    return V, I


def streamtopk_cuda_approx_forward(X, W_enc, b_enc, k, c, candidate_buffer=None):
    """Reference: streamtopk_sae/csrc/cuda/streamtopk_approx.cu:234-291.

    Returns (flat_vals, flat_idxs, cand_vals, cand_idxs): the per-128-feature
    tile top-c candidates (B, ceil(F/128), c) and their (B, tiles*c) views.
    """
    B, d, F = _common_checks(X, W_enc, b_enc, check_w_b_cuda=False)
    k, c = int(k), int(c)
    _require(1 <= k <= c, "k must be <= c")
    _require(W_enc.is_cuda and b_enc.is_cuda, "W_enc and b_enc must be on CUDA")
    tiles = (F + T_APPROX - 1) // T_APPROX
    if candidate_buffer is not None:
        cb = candidate_buffer
        _require(cb.dim() == 3 and cb.shape[0] == B and cb.shape[1] == tiles and cb.shape[2] == c,
                 "candidate_buffer shape mismatch")
        _require(cb.dtype == torch.float32 and cb.is_contiguous() and cb.device == X.device,
                 "candidate_buffer must be a contiguous fp32 tensor on X's device")
        cand_vals = cb
    else:
        cand_vals = torch.empty((B, tiles, c), dtype=torch.float32, device=X.device)
    cand_idxs = torch.empty((B, tiles, c), dtype=torch.int32, device=X.device)
    _require(c in (16, 32, 64, 128), f"streamtopk_cuda_approx: unsupported c={c}. Supported: 16,32,64,128.")
    lib = _capi.load()
    with torch.cuda.device(X.device):
        nbytes = _capi.candidates_workspace_bytes(B, d, F, c, _DTYPE_CODE[X.dtype])
        ws = torch.empty(max(nbytes, 8), dtype=torch.uint8, device=X.device)
        stream = torch.cuda.current_stream(X.device).cuda_stream
        _capi.check(lib.stk_approx_candidates(X.data_ptr(), W_enc.data_ptr(), b_enc.data_ptr(),
                                              cand_vals.data_ptr(), cand_idxs.data_ptr(), B, d, F, c,
                                              _DTYPE_CODE[X.dtype], ws.data_ptr(), nbytes, stream))
    return cand_vals.view(B, tiles * c), cand_idxs.view(B, tiles * c), cand_vals, cand_idxs


def streamtopk_cpu_forward(X, W_enc, b_enc, k):
    """The reference's CPU op is not part of this B200 build."""
    raise RuntimeError("streamtopk_cpu_forward is not provided by the B200 build "
                       "(the CPU path is the reference's; use topk_sae_cuda_exact)")
