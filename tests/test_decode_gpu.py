"""SAE decoder over the sparse codes (stk_decode_forward): the gather-GEMM
x_hat = b_dec + sum_j vals[:, j] * W_dec[idxs[:, j]] against a float64 torch
reference of the same gather, and the whole SAE forward (encode then decode)
against the dense float64 computation on the encoder's own top-k."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(vals, idxs, W_dec, b_dec):
    v = vals.double()
    ok = idxs >= 0
    rows = W_dec[idxs.clamp_min(0).long()].double() * ok[..., None]
    out = (v[..., None] * rows).sum(1)
    return out + (b_dec.double() if b_dec is not None else 0.0)


def _close(out, ref, vals, W_dec):
    # fp32 accumulation of k products: error well below 1e-5 of the row's scale
    scale = (vals.abs().sum(1, keepdim=True).double() * W_dec.float().abs().max().double()).clamp_min(1e-30)
    assert float(((out.double() - ref).abs() / scale).max()) < 1e-5


@pytest.mark.parametrize("B,k,F,d,dt", [(128, 64, 65536, 768, torch.bfloat16), (128, 32, 262144, 2048, torch.float16),
                                        (7, 33, 1000, 40, torch.float32), (300, 128, 20000, 1032, torch.bfloat16),
                                        (1, 1, 10, 8, torch.bfloat16)])
def test_decode_matches_float64(B, k, F, d, dt):
    from streamtopk_sae import decode
    g = torch.Generator(device="cuda").manual_seed(B + k + d)
    W_dec = torch.randn(F, d, generator=g, device="cuda").to(dt)
    b_dec = torch.randn(d, generator=g, device="cuda")
    idxs = torch.randint(0, F, (B, k), generator=g, device="cuda", dtype=torch.int32)
    vals = torch.randn(B, k, generator=g, device="cuda").abs()
    if B > 2:
        idxs[2, : k // 2] = -1                      # padding entries are skipped
    out = decode.topk_sae_decode(vals, idxs, W_dec, b_dec)
    out_nb = decode.topk_sae_decode(vals, idxs, W_dec)
    torch.cuda.synchronize()
    _close(out, _ref(vals, idxs, W_dec, b_dec), vals, W_dec)
    _close(out_nb, _ref(vals, idxs, W_dec, None), vals, W_dec)


def test_sae_forward_encode_then_decode():
    import streamtopk_sae as stk
    B, d, F, k = 64, 512, 30000, 32
    X, W_enc, b_enc = stk.make_inputs(B, d, F, dtype=torch.bfloat16, seed=3, device="cuda")
    W_dec = W_enc.clone()
    b_dec = torch.zeros(d, device="cuda")
    x_hat, vals, idxs = stk.topk_sae_forward(X, W_enc, b_enc, W_dec, b_dec, k)
    torch.cuda.synchronize()
    codes = torch.zeros(B, F, dtype=torch.float64, device="cuda")
    codes.scatter_(1, idxs.long(), vals.double())
    dense = codes @ W_dec.double() + b_dec.double()
    _close(x_hat, dense, vals, W_dec)


def test_decode_argument_errors():
    from streamtopk_sae import decode
    W = torch.zeros(10, 12, device="cuda", dtype=torch.bfloat16)
    v = torch.ones(2, 3, device="cuda")
    i = torch.zeros(2, 3, device="cuda", dtype=torch.int32)
    with pytest.raises(RuntimeError, match="multiple of 8"):
        decode.topk_sae_decode(v, i, W)
