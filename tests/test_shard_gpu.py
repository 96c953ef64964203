"""F-sharded encode over NCCL on 2 GPUs equals the single-GPU encode.

Two processes (one per GPU) each hold a shard of W_enc / b_enc, run
stk_shard_forward, all-gather the key lists over NCCL and merge.  Skipped when
fewer than 2 GPUs are visible.  NCCL's NVLS is off for the child processes.
"""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, cases, q):
    import datetime
    import sys
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        import streamtopk_sae as stk
        from streamtopk_sae import shard
        out = []
        for (B, d, F, k, seed) in cases:
            X, W, b = stk.make_inputs(B, d, F, dtype=torch.bfloat16, seed=seed, device=dev, w_init="unit_rows")
            f0, f1 = shard.shard_bounds(F, world, rank)
            enc = shard.ShardedEncoder(W[f0:f1].clone(), b[f0:f1].clone(), F, f0, k)
            V, I = enc.encode(X)
            V1, I1 = stk.topk_sae_cuda_exact(X, W, b, k)
            torch.cuda.synchronize()
            out.append((bool(torch.equal(I, I1)), bool(torch.equal(V, V1))))
        q.put((rank, out))
    except Exception as e:
        q.put((rank, repr(e)))
        raise
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_two_gpu_shards_equal_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    world = 2
    cases = [(128, 2048, 262144, 64, 0), (64, 512, 50000, 32, 1), (128, 256, 30001, 128, 2)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, cases, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert not isinstance(res[r], str), res[r]
        for ci, (idx_eq, val_eq) in enumerate(res[r]):
            assert idx_eq and val_eq, f"rank {r} case {cases[ci]}"
    assert all(p.exitcode == 0 for p in procs)
