"""Python op API: drop-in for the reference's ``streamtopk_sae.ops``.

``topk_sae_cuda_exact`` and ``topk_sae_cuda_approx`` keep the reference's
signatures, argument preparation (b_enc cast to fp32, inputs made contiguous)
and return types (values fp32 (B, k), indices int32 (B, k)); see
streamtopk_sae/ops.py:43-83 in the reference.  Both run the sm_100a kernels of
libstk_b200.so through its C ABI; there is no other compute path.

Extensions (keyword-only, off by default so behaviour matches the reference):
  allow_any_k  accept any 1 <= k <= 128 instead of {1,2,4,8,16,32,64,128}, and
               any k <= F when F <= 4096 (whole-row sort; e.g. k = F = 4096)
  allow_any_d  lift the exact path's d <= 4096 limit

Device-side errors.  The kernels bound every wait (pipeline barriers: 4 s; the
sampled-threshold barrier: 200 us, after which the kernel simply runs without
the threshold).  A pipeline wait that runs out -- in practice only when the GPU
is time-sliced away for seconds -- ends the kernel early and sets a device
error word; the op itself cannot see it without synchronising.  Callers that
need the guarantee call ``check_device_errors()`` at a synchronisation point
they already have (it synchronises the current stream, reads and clears the
word, and raises RuntimeError if a kernel reported an error).
"""
from __future__ import annotations

import torch

from . import _capi, native


def _check_native():
    # Fails loudly when the sm_100a library is missing (no fallback).
    _capi.load()


def _flags(allow_any_k: bool, allow_any_d: bool) -> int:
    return (_capi.STK_FLAG_ANY_K if allow_any_k else 0) | (_capi.STK_FLAG_ANY_D if allow_any_d else 0)


def _prepare(X, W_enc, b_enc):
    if b_enc.dtype != torch.float32:
        b_enc = b_enc.float()
    return X.contiguous(), W_enc.contiguous(), b_enc.contiguous()


def topk_sae_cuda_exact(X, W_enc, b_enc, k, *, allow_any_k=False, allow_any_d=False):
    """Exact streaming top-k SAE forward on B200.

    scores = X @ W_enc.T + b_enc is never materialised.  X, W_enc in fp32,
    fp16 or bf16 (same dtype); b_enc is cast to fp32.
    Returns: values (B, k) fp32 (each row descending), indices (B, k) int32.
    """
    _check_native()
    X, W_enc, b_enc = _prepare(X, W_enc, b_enc)
    return native.streamtopk_cuda_exact_forward(X, W_enc, b_enc, k, flags=_flags(allow_any_k, allow_any_d))


def topk_sae_cuda_approx(X, W_enc, b_enc, k, c, candidate_buffer=None, *, allow_any_k=False):
    """Approximate streaming top-k SAE forward (per-128-feature-tile top-c).

    c must be in {16, 32, 64, 128} and >= k.  With k <= c the tile filter keeps
    every feature of the exact top-k, so the result equals the exact op's; the
    final top-k runs on the GPU inside the library instead of a torch.topk over
    (B, ceil(F/128)*c) candidates.  If ``candidate_buffer`` (B, ceil(F/128), c)
    fp32 is given, it is filled with the per-tile candidate values, as the
    reference does -- for fp16 / bf16 with c <= 32 in the same W_enc pass as
    the top-k (one kernel), otherwise by a candidates pass first.
    Returns: values (B, k) fp32 (descending), indices (B, k) int32.
    """
    _check_native()
    X, W_enc, b_enc = _prepare(X, W_enc, b_enc)
    if candidate_buffer is not None:
        B, F = X.shape[0], W_enc.shape[0]
        tiles = (F + native.T_APPROX - 1) // native.T_APPROX
        cb = candidate_buffer
        if not (cb.dim() == 3 and tuple(cb.shape) == (B, tiles, int(c))):
            raise RuntimeError("candidate_buffer shape mismatch")
        if not (cb.dtype == torch.float32 and cb.is_contiguous() and cb.device == X.device):
            raise RuntimeError("candidate_buffer must be a contiguous fp32 tensor on X's device")
        idxs = torch.empty(cb.shape, dtype=torch.int32, device=X.device)
        return native.approx_forward_with_candidates(X, W_enc, b_enc, k, c, cb, idxs,
                                                     flags=_flags(allow_any_k, True))
    return native.approx_topk_forward(X, W_enc, b_enc, k, c, flags=_flags(allow_any_k, True))


def check_device_errors(device=None):
    """Synchronise the current stream of `device` and raise RuntimeError if a
    library kernel reported a device-side error (a bounded wait that ran out)
    since the last check; the error word is cleared."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        _capi.device_error(torch.cuda.current_stream(dev).cuda_stream)


def topk_sae_cpu(X, W_enc, b_enc, k):
    """The reference's CPU op is not part of the B200 build (raises)."""
    return native.streamtopk_cpu_forward(X, W_enc, b_enc, k)
