"""StreamTopK-SAE for B200: streaming fused top-k SAE encoder on sm_100a.

Drop-in for the reference package's op API (streamtopk_sae/__init__.py in
ayushimehrotra/streamtopk-sae): ``topk_sae_cuda_exact`` and
``topk_sae_cuda_approx`` compute top_k(X @ W_enc.T + b_enc, k) without
materialising the (B, F) score matrix, on tcgen05 tensor cores with the top-k
selection fused into the GEMM epilogue.  ``shard`` adds the multi-GPU
F-sharded encoder (one process per GPU; the per-rank key lists are exchanged
by direct peer stores between the GPUs, or by an NCCL all-gather, then merged).
``fp8`` adds an E4M3 W_enc path (half the HBM bytes; lossy, an extension);
``decode`` the SAE decoder over the sparse codes (gather-GEMM, an extension);
``EncodePipeline`` the same exact encode for loops over batches of one shape,
consecutive steps overlapped on the GPU.
"""
from streamtopk_sae.decode import topk_sae_decode, topk_sae_forward
from streamtopk_sae.fp8 import quantize_weights, topk_sae_cuda_exact_fp8
from streamtopk_sae.ops import check_device_errors, topk_sae_cpu, topk_sae_cuda_approx, topk_sae_cuda_exact
from streamtopk_sae.pipeline import EncodePipeline
from streamtopk_sae.utils import make_inputs, recall_at_k

__all__ = [
    "topk_sae_cpu",
    "topk_sae_cuda_exact",
    "topk_sae_cuda_approx",
    "check_device_errors",
    "recall_at_k",
    "make_inputs",
    "quantize_weights",
    "topk_sae_cuda_exact_fp8",
    "topk_sae_decode",
    "topk_sae_forward",
    "EncodePipeline",
]
