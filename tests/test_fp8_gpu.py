"""FP8 (E4M3) W_enc streaming (streamtopk_sae.fp8, stk_exact_forward_fp8).

The fp8 encode is exact for the quantized operands: its top-k must equal, up
to ties within the fp32 tolerance, the float64 top-k of
x_scale * w_scale * (X8 . W8) + b computed on the host from the GPU's own
quantized X8 / W8 and scales.  Against the unquantized (bf16) scores it is an
approximation, measured as recall.  The row quantizer is checked bit for bit
against torch's E4M3 conversion of the same scaled values.
"""
import numpy as np
import pytest
import torch

from gpu_util import HostRows, no_device_error, sample_rows
from oracle import oracle

pytestmark = pytest.mark.gpu


def _quantized_host(X, W8, w_scale):
    from streamtopk_sae import fp8
    Q, sx = fp8.quantize_rows(X)
    torch.cuda.synchronize()
    Xq = (Q.float() * sx[:, None]).cpu().numpy()
    Wq = W8.float() * w_scale[:, None]
    return Xq, Wq


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_quantize_rows_matches_torch(dtype):
    from streamtopk_sae import fp8
    g = torch.Generator(device="cuda").manual_seed(3)
    X = (torch.randn(67, 320, generator=g, device="cuda") * 3).to(dtype)
    X[5] = 0                                  # an all-zero row: scale 1, zeros
    X[6, 7] = 1e4                             # one large element: the rest underflows toward 0
    Q, s = fp8.quantize_rows(X)
    torch.cuda.synchronize()
    Xf = X.float()
    amax = Xf.abs().amax(dim=1)
    c448 = torch.full_like(amax, 448.0)  # tensor / tensor: IEEE division, like the kernel's
    ref_s = torch.where(amax > 0, amax / c448, torch.ones_like(amax))
    inv = torch.where(amax > 0, c448 / amax, torch.ones_like(amax))
    ref_q = (Xf * inv[:, None]).to(fp8.E4M3)
    assert torch.equal(s, ref_s)
    assert torch.equal(Q.view(torch.uint8), ref_q.view(torch.uint8))


@pytest.mark.parametrize("B,d,F,k", [(128, 768, 65536, 32), (128, 2048, 100000, 64), (300, 256, 30000, 128),
                                     (7, 64, 1000, 16), (128, 512, 20000, 1), (1024, 256, 30000, 128)])
def test_fp8_encode_exact_on_quantized_operands(B, d, F, k):
    import streamtopk_sae as stk
    from streamtopk_sae import fp8
    X, W, b = stk.make_inputs(B, d, F, dtype=torch.bfloat16, seed=B + F, device="cuda", w_init="unit_rows")
    W8, ws = fp8.quantize_weights(W)
    V, I = fp8.topk_sae_cuda_exact_fp8(X, W8, ws, b, k)
    torch.cuda.synchronize()
    no_device_error()
    assert V.shape == (B, k) and I.dtype == torch.int32
    assert bool((V[:, 1:] <= V[:, :-1]).all())
    Xq, Wq = _quantized_host(X, W8, ws)
    rows = sample_rows(16, B, seed=2)
    rt = torch.from_numpy(rows).to(V.device)
    chk = oracle.check_topk(V[rt].cpu().numpy(), I[rt].cpu().numpy(), Xq[rows], HostRows(Wq), b.cpu().numpy(), k,
                            rtol=1e-4)
    chk.raise_if_bad()
    assert chk.tie_recall == 1.0


def test_fp8_deterministic_and_graph_stable():
    import streamtopk_sae as stk
    from streamtopk_sae import fp8
    X, W, b = stk.make_inputs(128, 1024, 50000, dtype=torch.bfloat16, seed=9, device="cuda")
    W8, ws = fp8.quantize_weights(W)
    V1, I1 = fp8.topk_sae_cuda_exact_fp8(X, W8, ws, b, 64)
    V2, I2 = fp8.topk_sae_cuda_exact_fp8(X, W8, ws, b, 64)
    torch.cuda.synchronize()
    assert torch.equal(V1, V2) and torch.equal(I1, I2)


def test_fp8_recall_against_bf16_config3():
    """BASELINE.json configs[2]'s shape with W_enc and X in E4M3: recall of the
    fp8 top-k against the bf16 exact top-k (the quantization's effect)."""
    import streamtopk_sae as stk
    from streamtopk_sae import fp8
    B, d, F, k = 128, 2048, 262144, 64
    X, W, b = stk.make_inputs(B, d, F, dtype=torch.bfloat16, seed=0, device="cuda", w_init="unit_rows")
    W8, ws = fp8.quantize_weights(W)
    Vq, Iq = fp8.topk_sae_cuda_exact_fp8(X, W8, ws, b, k)
    Ve, Ie = stk.topk_sae_cuda_exact(X, W, b, k)
    torch.cuda.synchronize()
    no_device_error()
    rec = stk.recall_at_k(Iq.long(), Ie.long())
    print(f"\nfp8 (E4M3 X and W_enc) recall@{k} vs bf16 exact at B={B} d={d} F={F}: {rec:.4f}")
    assert rec >= 0.90   # measured 0.942


def test_fp8_argument_errors():
    from streamtopk_sae import fp8
    X = torch.randn(4, 40, device="cuda", dtype=torch.bfloat16)
    W8 = torch.zeros(100, 40, device="cuda", dtype=fp8.E4M3)
    s = torch.ones(100, device="cuda")
    b = torch.zeros(100, device="cuda")
    with pytest.raises(RuntimeError, match="multiple of 16"):
        fp8.topk_sae_cuda_exact_fp8(X, W8, s, b, 8)
    with pytest.raises(RuntimeError, match="float8_e4m3fn"):
        fp8.topk_sae_cuda_exact_fp8(X[:, :32].contiguous(), torch.zeros(100, 32, device="cuda"), s, b, 8)
