"""F-sharded encode on 2 GPUs equals the single-GPU encode.

Two processes (one per GPU) each hold a shard of W_enc / b_enc.  Two
transports of the per-rank key lists are checked:
  * "nccl": stk_shard_forward, all-gather over NCCL, stk_merge_keys;
  * "p2p":  stk_exchange_forward (publish kernel with peer stores into the
    other rank's receive buffer over CUDA IPC, bounded wait, final merge),
    eagerly and replayed from a CUDA graph (both receive slots), with an empty
    shard, and with a batch larger than the exchange was sized for;
  * "p2p" pipelined (ShardedEncoder.submit / flush): each batch finished by
    the next batch's score kernel, eagerly, mixed with encode, and in a graph.
A failure test makes one rank skip a step: the other rank's final merge gives
up after its (short) wait limit and reports device error 3.  Skipped when
fewer than 2 GPUs are visible.  NCCL's NVLS is off for the child processes.
"""
import os
import socket

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    return dist, dev


def _same(a, b):
    return bool(torch.equal(a[0], b[0]) and torch.equal(a[1], b[1]))


def _worker_cases(rank, world, port, transport, cases, q):
    dist, dev = _init(rank, world, port)
    try:
        import streamtopk_sae as stk
        from streamtopk_sae import shard
        out = []
        for (B, d, F, k, seed) in cases:
            X, W, b = stk.make_inputs(B, d, F, dtype=torch.bfloat16, seed=seed, device=dev, w_init="unit_rows")
            f0, f1 = shard.shard_bounds(F, world, rank)
            enc = shard.ShardedEncoder(W[f0:f1].clone(), b[f0:f1].clone(), F, f0, k, transport=transport)
            got = enc.encode(X)
            got2 = enc.encode(X)          # second step: the other receive slot
            ref = stk.topk_sae_cuda_exact(X, W, b, k)
            torch.cuda.synchronize()
            out.append(_same(got, ref) and _same(got2, ref))
            enc.close()
        q.put((rank, out))
    except Exception as e:
        q.put((rank, repr(e)))
        raise
    finally:
        dist.barrier()
        dist.destroy_process_group()


def _worker_p2p_graph(rank, world, port, q):
    dist, dev = _init(rank, world, port)
    try:
        import streamtopk_sae as stk
        from streamtopk_sae import _capi, shard
        from streamtopk_sae.graph import CapturedEncode
        B, d, F, k = 128, 1024, 100000, 64
        X, W, b = stk.make_inputs(B, d, F, dtype=torch.bfloat16, seed=7, device=dev, w_init="unit_rows")
        f0, f1 = shard.shard_bounds(F, world, rank)
        enc = shard.ShardedEncoder(W[f0:f1].clone(), b[f0:f1].clone(), F, f0, k, transport="p2p")
        g = CapturedEncode(enc.encode, X, steps=3, warmup=2)   # odd number of steps per replay
        ok = []
        for seed in (11, 12, 13):
            Xn = stk.make_inputs(B, d, 8, dtype=torch.bfloat16, seed=seed, device=dev)[0]
            V, I = g(Xn)
            ref = stk.topk_sae_cuda_exact(Xn, W, b, k)
            torch.cuda.synchronize()
            ok.append(_same((V, I), ref))
        ok.append(_capi.device_error(torch.cuda.current_stream().cuda_stream) == 0)
        g.close()
        # empty shard on the last rank (F < 128 * world) and a batch beyond max_rows
        F2 = 100
        X2, W2, b2 = stk.make_inputs(200, 256, F2, dtype=torch.bfloat16, seed=3, device=dev, w_init="unit_rows")
        g0, g1 = shard.shard_bounds(F2, world, rank)
        enc2 = shard.ShardedEncoder(W2[g0:g1].clone(), b2[g0:g1].clone(), F2, g0, 16, transport="p2p")
        ok.append(_same(enc2.encode(X2[:64].contiguous()), stk.topk_sae_cuda_exact(X2[:64].contiguous(), W2, b2, 16)))
        ok.append(_same(enc2.encode(X2), stk.topk_sae_cuda_exact(X2, W2, b2, 16)))
        enc2.close()
        enc.close()
        q.put((rank, ok))
    except Exception as e:
        q.put((rank, repr(e)))
        raise
    finally:
        dist.barrier()
        dist.destroy_process_group()


def _worker_p2p_timeout(rank, world, port, q):
    """Rank 1 never joins step 0: rank 0's final merge gives up after 0.5 s."""
    dist, dev = _init(rank, world, port)
    try:
        import streamtopk_sae as stk
        from streamtopk_sae import _capi, shard
        B, d, F, k = 32, 256, 4096, 16
        X, W, b = stk.make_inputs(B, d, F, dtype=torch.bfloat16, seed=1, device=dev)
        f0, f1 = shard.shard_bounds(F, world, rank)
        ex = shard.PeerExchange(B, k, dev, wait_seconds=0.5)
        res = None
        if rank == 0:
            V = torch.empty((B, k), dtype=torch.float32, device=dev)
            I = torch.empty((B, k), dtype=torch.int32, device=dev)
            ex.forward(X, W[f0:f1].contiguous(), b[f0:f1].contiguous(), f0, V, I)
            try:
                _capi.device_error(torch.cuda.current_stream().cuda_stream)
                res = "no error reported"
            except RuntimeError as e:
                res = "device error code 3" in str(e)
        else:
            res = True
        ex.close()
        q.put((rank, [res]))
    except Exception as e:
        q.put((rank, repr(e)))
        raise
    finally:
        dist.barrier()
        dist.destroy_process_group()


def _worker_p2p_pipeline(rank, world, port, q):
    """Pipelined submit / flush over the exchange: each batch is finished by the
    next batch's score kernel (cross-GPU publish, wait and merge included)."""
    dist, dev = _init(rank, world, port)
    try:
        import streamtopk_sae as stk
        from streamtopk_sae import _capi, shard
        from streamtopk_sae.graph import CapturedEncode
        ok = []
        for (B, d, F, k) in ((128, 2048, 65536, 64), (100, 768, 50000, 32)):
            X, W, b = stk.make_inputs(B, d, F, dtype=torch.bfloat16, seed=9, device=dev, w_init="unit_rows")
            f0, f1 = shard.shard_bounds(F, world, rank)
            enc = shard.ShardedEncoder(W[f0:f1].clone(), b[f0:f1].clone(), F, f0, k, transport="p2p", max_rows=B)
            Xs = [stk.make_inputs(B, d, 8, dtype=torch.bfloat16, seed=40 + i, device=dev)[0] for i in range(5)]
            outs = [enc.submit(x) for x in Xs[:4]]
            enc.flush()
            mixed = enc.submit(Xs[4])
            after = enc.encode(Xs[0])   # flushes the pending batch first
            torch.cuda.synchronize()
            for x, got in zip(Xs[:4] + [Xs[4], Xs[0]], outs + [mixed, after]):
                ok.append(_same(got, stk.topk_sae_cuda_exact(x, W, b, k)))
            g = CapturedEncode(enc.submit, Xs[0], steps=3, warmup=2, finish=enc.flush)
            for seed in (21, 22):
                Xn = stk.make_inputs(B, d, 8, dtype=torch.bfloat16, seed=seed, device=dev)[0]
                V, I = g(Xn)
                torch.cuda.synchronize()
                ok.append(_same((V, I), stk.topk_sae_cuda_exact(Xn, W, b, k)))
            g.close()
            ok.append(_capi.device_error(torch.cuda.current_stream().cuda_stream) == 0)
            enc.close()
        q.put((rank, ok))
    except Exception as e:
        q.put((rank, repr(e)))
        raise
    finally:
        dist.barrier()
        dist.destroy_process_group()


def _run(target, extra):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=target, args=(r, world, port, *extra, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = dict(q.get(timeout=240) for _ in range(world))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in range(world):
        assert not isinstance(res[r], str), res[r]
        assert all(v is True for v in res[r]), f"rank {r}: {res[r]}"
    assert all(p.exitcode == 0 for p in procs)


CASES = [(128, 2048, 262144, 64, 0), (64, 512, 50000, 32, 1), (128, 256, 30001, 128, 2), (300, 256, 20000, 8, 3)]


@pytest.mark.parametrize("transport", ["nccl", "p2p"])
def test_two_gpu_shards_equal_single_gpu(transport):
    _run(_worker_cases, (transport, CASES))


def test_two_gpu_p2p_graph_empty_shard_and_growth():
    _run(_worker_p2p_graph, ())


def test_two_gpu_p2p_missing_rank_times_out():
    _run(_worker_p2p_timeout, ())


def test_two_gpu_p2p_pipelined_submit_flush():
    _run(_worker_p2p_pipeline, ())
