"""Pipelined exact encode (EncodePipeline / stk_pipeline_*) against the one-call op.

Every batch of a pipeline must give exactly topk_sae_cuda_exact's result for
its inputs (same keys: bit-identical V and I), whether its rows are finished
by the next batch's score kernel, by flush(), inside a replayed multi-batch
graph, or on a shape that does not pipeline.  Different X per batch catch a
batch finished from the wrong half of the workspace.
"""
import pytest
import torch

import streamtopk_sae as stk
from gpu_util import no_device_error

pytestmark = pytest.mark.gpu

# (B, d, F, k, dtype, pipelined)
SHAPES = [
    (128, 768, 65536, 32, torch.bfloat16, True),    # BASELINE cfg2 shape
    (128, 2048, 32768, 64, torch.bfloat16, True),   # one rank's shard of cfg3 at N = 8
    (64, 256, 4096, 32, torch.float16, True),
    (1, 128, 1000, 8, torch.bfloat16, True),
    (100, 512, 16384, 128, torch.bfloat16, False),  # k > 64: one call per batch
    (128, 512, 16384, 16, torch.float32, True),     # fp32 on tensor cores (3-pass TF32)
    (384, 96, 50000, 32, torch.bfloat16, False),    # several rounds of units per CTA: one call per step
]


def _batches(B, d, dtype, n, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return [torch.randn(B, d, generator=g, device="cuda").to(dtype) for _ in range(n)]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: f"B{s[0]}_d{s[1]}_F{s[2]}_k{s[3]}_{str(s[4])[6:]}")
def test_pipeline_steps_equal_one_call(shape):
    B, d, F, k, dtype, piped = shape
    _, W, b = stk.make_inputs(B, d, F, dtype=dtype, seed=3, device="cuda")
    Xs = _batches(B, d, dtype, 6, seed=11)
    torch.cuda.synchronize()
    pipe = stk.EncodePipeline(B, d, F, k, dtype)
    assert pipe.pipelined == piped
    outs = pipe.encode(Xs, W, b)
    torch.cuda.synchronize()
    no_device_error()
    for X, (V, I) in zip(Xs, outs):
        Vr, Ir = stk.topk_sae_cuda_exact(X, W, b, k)
        assert torch.equal(V, Vr) and torch.equal(I, Ir)
    pipe.close()
    no_device_error()


def test_pipeline_captured_graph_replays():
    B, d, F, k, dtype = 128, 2048, 32768, 64, torch.bfloat16
    _, W, b = stk.make_inputs(B, d, F, dtype=dtype, seed=4, device="cuda")
    pipe = stk.EncodePipeline(B, d, F, k, dtype)
    G = 3
    Xs = [torch.zeros(B, d, dtype=dtype, device="cuda") for _ in range(G)]
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):  # warm-up outside the capture
        pipe.encode(Xs, W, b)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        outs = pipe.encode(Xs, W, b)
    for rep in range(3):
        new = _batches(B, d, dtype, G, seed=20 + rep)
        for X, Xn in zip(Xs, new):
            X.copy_(Xn)
        graph.replay()
        torch.cuda.synchronize()
        no_device_error()
        for Xn, (V, I) in zip(new, outs):
            Vr, Ir = stk.topk_sae_cuda_exact(Xn, W, b, k)
            assert torch.equal(V, Vr) and torch.equal(I, Ir)
    graph.reset()
    pipe.close()


def test_pipeline_rejects_other_shapes():
    B, d, F, k = 64, 256, 4096, 32
    _, W, b = stk.make_inputs(B, d, F, dtype=torch.bfloat16, seed=5, device="cuda")
    pipe = stk.EncodePipeline(B, d, F, k, torch.bfloat16)
    X = torch.randn(B + 1, d, device="cuda").to(torch.bfloat16)
    with pytest.raises(RuntimeError, match="differs from the pipeline"):
        pipe.submit(X, W, b)
    pipe.close()


def test_pipeline_results_complete_after_next_submit():
    """Batch s is readable once batch s + 1 is enqueued (before any flush)."""
    B, d, F, k, dtype = 128, 768, 65536, 32, torch.bfloat16
    _, W, b = stk.make_inputs(B, d, F, dtype=dtype, seed=6, device="cuda")
    Xs = _batches(B, d, dtype, 3, seed=30)
    pipe = stk.EncodePipeline(B, d, F, k, dtype)
    V0, I0 = pipe.submit(Xs[0], W, b)
    V1, I1 = pipe.submit(Xs[1], W, b)
    got0 = (V0.clone(), I0.clone())  # stream-ordered after batch 1's launch
    pipe.submit(Xs[2], W, b)
    pipe.flush()
    torch.cuda.synchronize()
    no_device_error()
    for X, (V, I) in zip(Xs[:2], (got0, (V1, I1))):
        Vr, Ir = stk.topk_sae_cuda_exact(X, W, b, k)
        assert torch.equal(V, Vr) and torch.equal(I, Ir)
    pipe.close()
