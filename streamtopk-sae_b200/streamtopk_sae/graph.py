"""CUDA-graph capture of a fixed-shape encode step.

Serving loops call the encoder with a new batch of the same shape many times;
the library's kernels are asynchronous, so at small per-step GPU times (F
sharded over 8 GPUs: tens of microseconds) the host-side launch work (argument
checks, workspace allocation, ctypes calls, the NCCL enqueue) becomes the
bottleneck.  ``CapturedEncode`` records `steps` back-to-back calls of an encode
function on a static input buffer into one CUDA graph (the library's memset,
kernels with their programmatic-dependent launches, and NCCL collectives are
all capturable) and replays it.

    step = CapturedEncode(lambda x: topk_sae_cuda_exact(x, W, b, k), X_example)
    V, I = step(X_new)        # copies X_new into the static buffer, replays

Outputs are the graph's own tensors (overwritten by the next replay).

A pipelined encode (``EncodePipeline.submit`` / ``ShardedEncoder.submit``)
finishes each batch in the next batch's launch: pass its ``flush`` as
``finish``, called once after the captured steps, so every replay is complete.
"""
from __future__ import annotations

import torch


class CapturedEncode:
    def __init__(self, fn, X_example, steps: int = 1, warmup: int = 3, finish=None):
        if steps < 1:
            raise ValueError("steps must be >= 1")
        self.fn = fn
        self.steps = steps
        self.X = X_example.detach().clone().contiguous()
        if warmup > 0:  # first calls outside the graph (lazy init, allocator pools)
            side = torch.cuda.Stream(device=self.X.device)
            side.wait_stream(torch.cuda.current_stream(self.X.device))
            with torch.cuda.stream(side):
                for _ in range(warmup):
                    fn(self.X)
                if finish is not None:
                    finish()
            torch.cuda.current_stream(self.X.device).wait_stream(side)
        torch.cuda.synchronize(self.X.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            for _ in range(steps):
                out = fn(self.X)
            if finish is not None:
                finish()
        self.V, self.I = out

    def replay(self):
        self.graph.replay()
        return self.V, self.I

    def close(self):
        """Release the graph (and any NCCL work captured in it).

        Graphs that hold NCCL collectives must be released before the process
        group is destroyed, or the teardown waits for them forever.
        """
        if self.graph is not None:
            torch.cuda.synchronize(self.X.device)
            self.graph.reset()
            self.graph = None
        self.V = self.I = None

    def __call__(self, X=None):
        if X is not None:
            self.X.copy_(X, non_blocking=True)
        return self.replay()
