"""F-shard plumbing of streamtopk_sae.shard on CPU ranks (gloo, world size 2 and 3).

The GPU kernels are replaced by a CPU stand-in built on the oracle (float64
scores, keys ordered by (score desc, index asc)), so this checks the host
logic: shard bounds, global index offsets, the all-gather of key lists and
the final merge, against the unsharded oracle.  The real kernels are covered
by the GPU tests.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from streamtopk_sae import shard


def _order32(v):
    u = np.asarray(v, np.float32).view(np.uint32).astype(np.uint64)
    u = np.where((u << np.uint64(1)) & np.uint64(0xFFFFFFFF) == 0, np.uint64(0), u)
    neg = (u & np.uint64(0x80000000)) != 0
    return np.where(neg, (~u) & np.uint64(0xFFFFFFFF), u | np.uint64(0x80000000))


def _keys(vals, idx):
    return ((_order32(vals) << np.uint64(32)) | ((~idx.astype(np.uint64)) & np.uint64(0xFFFFFFFF)))


def cpu_shard_fn(X, W, b, k, f_offset, out_keys):
    S = (X.double() @ W.double().T + b.double()).float().numpy()
    L = out_keys.shape[1]
    idx = np.arange(W.shape[0], dtype=np.int64) + f_offset
    kk = _keys(S, np.broadcast_to(idx, S.shape))
    top = np.sort(kk, axis=1)[:, ::-1][:, :L]
    if top.shape[1] < L:
        top = np.concatenate([top, np.zeros((top.shape[0], L - top.shape[1]), np.uint64)], axis=1)
    out_keys.copy_(torch.from_numpy(top.view(np.int64).copy()))
    return out_keys


def cpu_merge_fn(gathered, k):
    P, B, L = gathered.shape
    allk = gathered.numpy().view(np.uint64).transpose(1, 0, 2).reshape(B, P * L)
    top = np.sort(allk, axis=1)[:, ::-1][:, :k]
    hi = (top >> np.uint64(32)).astype(np.uint32)
    neg = (hi & np.uint32(0x80000000)) == 0
    u = np.where(neg, ~hi, hi & np.uint32(0x7FFFFFFF)).astype(np.uint32)
    V = u.view(np.float32).copy()
    I = (~(top & np.uint64(0xFFFFFFFF)).astype(np.uint32)).view(np.int32).copy()
    empty = top == 0
    V[empty] = -3.402823466e38
    I[empty] = -1
    return torch.from_numpy(V), torch.from_numpy(I)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, F, k, out_q, transport="nccl"):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(0)
        X = torch.from_numpy(rng.standard_normal((6, 32)).astype(np.float32))
        W = torch.from_numpy(rng.standard_normal((F, 32)).astype(np.float32))
        b = torch.from_numpy(rng.standard_normal(F).astype(np.float32) * 0.1)
        f0, f1 = shard.shard_bounds(F, world, rank)
        if transport == "auto":
            # The peer exchange cannot be set up without GPUs: every rank must
            # reach the same verdict and fall back to the process-group path
            # (here with the CPU stand-ins).
            enc = shard.ShardedEncoder(W[f0:f1], b[f0:f1], F, f0, k, transport="auto")
            enc.shard_fn, enc.merge_fn = cpu_shard_fn, cpu_merge_fn
        else:
            enc = shard.ShardedEncoder(W[f0:f1], b[f0:f1], F, f0, k, shard_fn=cpu_shard_fn, merge_fn=cpu_merge_fn)
        V, I = enc.encode(X)
        # The pipelined submit / flush falls back to encode without the p2p
        # exchange: same result, complete at once.
        Vs, Is = enc.submit(X)
        enc.flush()
        assert torch.equal(V, Vs) and torch.equal(I, Is)
        if transport == "auto":
            assert enc.transport == "nccl" and enc.fallback_reason, (enc.transport, enc.fallback_reason)
            V2, I2 = enc.encode(X)     # later steps stay on the fallback path
            assert torch.equal(V, V2) and torch.equal(I, I2)
        out_q.put((rank, V.numpy(), I.numpy()))
    except Exception as e:  # report instead of leaving the parent waiting
        out_q.put((rank, repr(e), None))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,F,k,transport", [(2, 1000, 16, "nccl"), (3, 700, 64, "nccl"), (2, 200, 128, "nccl"),
                                                 (2, 1000, 16, "auto"), (3, 700, 64, "auto")])
def test_sharded_matches_unsharded(world, F, k, transport):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, F, k, q, transport)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=60) for _ in range(world)]
    for rank, V, I in res:
        assert I is not None, f"rank {rank}: {V}"
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    rng = np.random.default_rng(0)
    X = rng.standard_normal((6, 32)).astype(np.float32)
    W = rng.standard_normal((F, 32)).astype(np.float32)
    b = rng.standard_normal(F).astype(np.float32) * 0.1
    S = (X.astype(np.float64) @ W.astype(np.float64).T + b).astype(np.float32)
    want_i = np.argsort(-S, axis=1, kind="stable")[:, :k]
    want_v = np.take_along_axis(S, want_i, axis=1)
    for rank, V, I in res:
        assert np.array_equal(I, want_i.astype(np.int32)), rank
        assert np.array_equal(V, want_v), rank


def test_shard_bounds_cover_F():
    for F in (1, 127, 128, 1000, 262144, 1048576):
        for world in (1, 2, 3, 4, 8):
            bounds = [shard.shard_bounds(F, world, r) for r in range(world)]
            assert bounds[0][0] == 0 and bounds[-1][1] == F
            for (a0, a1), (b0, b1) in zip(bounds, bounds[1:]):
                assert a1 == b0 and a0 <= a1
            assert all(f0 % shard.ALIGN == 0 or f0 == F for f0, _ in bounds)
