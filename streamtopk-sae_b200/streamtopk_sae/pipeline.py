"""Pipelined exact encode: batch after batch of one shape (stk_pipeline_*).

Each batch gets exactly ``topk_sae_cuda_exact``'s result for its inputs (the
reference op, streamtopk_sae/ops.py:43-57 / streamtopk_exact.cu:788-833).
What changes is the work per batch on the GPU: one launch, whose score kernel
also finishes the previous batch (selects and writes its rows while the first
W_enc tile streams in), so the finish step leaves the critical path.  A
batch's (V, I) are complete, in stream order, once the next batch has been
submitted or after ``flush()``:

    pipe = EncodePipeline(B, d, F, k, torch.bfloat16)
    outs = [pipe.submit(X, W_enc, b_enc) for X in batches]
    pipe.flush()                      # outs[-1] complete from here on

Submit and flush on one stream.  Shapes that do not pipeline (k > 64, or
several rounds of work units per CTA, e.g. B > 256) run each batch as one
``topk_sae_cuda_exact`` call, complete at once (``pipelined`` False).
"""
from __future__ import annotations

import ctypes

import torch

from streamtopk_sae import _capi
from streamtopk_sae.native import _DTYPE_CODE, _common_checks, _require


class EncodePipeline:
    def __init__(self, B: int, d: int, F: int, k: int, dtype=torch.bfloat16, device=None, flags: int = 0):
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        _require(dtype in _DTYPE_CODE, "X dtype must be fp32, fp16, or bf16")
        self.B, self.d, self.F, self.k, self.dtype, self.flags = int(B), int(d), int(F), int(k), dtype, int(flags)
        lib = _capi.load()
        nbytes = ctypes.c_size_t(0)
        code = _DTYPE_CODE[dtype]
        _capi.check(lib.stk_pipeline_workspace_bytes(self.B, self.d, self.F, self.k, code, self.flags,
                                                     ctypes.byref(nbytes)))
        self._handle = None
        with torch.cuda.device(self.device):
            self.workspace = torch.empty(int(nbytes.value), dtype=torch.uint8, device=self.device)
            h = ctypes.c_void_p()
            _capi.check(lib.stk_pipeline_create(ctypes.byref(h), self.B, self.d, self.F, self.k, code, self.flags,
                                                self.workspace.data_ptr(), int(nbytes.value)))
        self._handle = h
        self._keep = []  # the pending batch's V / I (written by the next launch), alive until then

    @property
    def pipelined(self) -> bool:
        """True when this shape runs pipelined (else each batch runs as one call)."""
        return bool(_capi.load().stk_pipeline_pipelined(self._handle))

    def submit(self, X, W_enc, b_enc, out=None):
        """Enqueue one batch; returns its (V, I), complete after the next submit() or flush()."""
        _require(self._handle is not None, "pipeline is closed")
        B, d, F = _common_checks(X, W_enc, b_enc)
        _require((B, d, F) == (self.B, self.d, self.F) and X.dtype == self.dtype,
                 "EncodePipeline: X / W_enc shape or dtype differs from the pipeline's")
        _require(X.device == self.device, "EncodePipeline: tensors are not on the pipeline's device")
        if out is None:
            V = torch.empty((B, self.k), dtype=torch.float32, device=X.device)
            I = torch.empty((B, self.k), dtype=torch.int32, device=X.device)
        else:
            V, I = out
        b = b_enc if b_enc.dtype == torch.float32 else b_enc.float()
        X, W, b = X.contiguous(), W_enc.contiguous(), b.contiguous()
        with torch.cuda.device(X.device):
            stream = torch.cuda.current_stream(X.device).cuda_stream
            _capi.check(_capi.load().stk_pipeline_submit(self._handle, X.data_ptr(), W.data_ptr(), b.data_ptr(),
                                                         V.data_ptr(), I.data_ptr(), stream))
        self._keep = [V, I]
        return V, I

    def flush(self):
        """Enqueue the finish of the last submitted batch (no-op if none is pending)."""
        _require(self._handle is not None, "pipeline is closed")
        with torch.cuda.device(self.device):
            stream = torch.cuda.current_stream(self.device).cuda_stream
            _capi.check(_capi.load().stk_pipeline_flush(self._handle, stream))
        self._keep = []

    def encode(self, batches, W_enc, b_enc):
        """All batches, pipelined; returns their (V, I) (complete in stream order)."""
        outs = [self.submit(X, W_enc, b_enc) for X in batches]
        self.flush()
        return outs

    def close(self):
        """Flush, wait for the GPU, and destroy the pipeline."""
        if self._handle is not None:
            self.flush()
            torch.cuda.synchronize(self.device)
            _capi.load().stk_pipeline_destroy(self._handle)
            self._handle = None
            self.workspace = None

    def __del__(self):
        try:
            if self._handle is not None:
                _capi.load().stk_pipeline_destroy(self._handle)
        except Exception:
            pass
