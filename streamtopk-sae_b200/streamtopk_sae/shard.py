"""Multi-GPU encoder: W_enc sharded along F, one process per GPU.

Each rank holds the contiguous feature range [f0, f1) of W_enc / b_enc
(``shard_bounds``).  One encode:

  1. ``stk_shard_forward`` on the local shard: fused tcgen05 scores + top-k,
     then the local merge of the CTA lists; writes this rank's best L keys per
     row (L = 32/64/128 for k <= 32/64/128) with global feature indices
     (local index + f0).
  2. ``all_gather_into_tensor`` of the (B, L) int64 key lists over the process
     group (NCCL over NVLink on B200; gloo works for host-side tests).
  3. ``stk_merge_keys`` on every rank: top-k of world * L keys per row.

With ``transport="p2p"`` steps 2-3 run inside the library instead
(``PeerExchange``, C ABI stk_exchange_*): the score kernel finishes its rows
in its own tail and stores each row's best keys straight into every rank's
receive buffer (CUDA IPC mappings, peer stores over NVLink) with a per-row flag
set to the step number, then waits (bounded) for all ranks' rows and merges
them -- one kernel launch per step, no NCCL call and no host involvement.

Device-side errors: a wait for another rank's rows that runs out (default
10 s) sets device error 3 and that step's rows are finished over the ranks
whose rows had arrived.  The kernels cannot raise; ``check_device_errors()``
(at a synchronisation point the caller already has) reads the error word and
raises.  Steps are tagged with their absolute number, so rows that arrive late
are never taken for a later step's rows.

Keys order by (score desc, feature index asc), so the result is identical to
the single-GPU encode for any world size.  The reference has no multi-GPU
path; the shard / all-gather / merge scheme follows BASELINE.json's north
star.  The kernels are pluggable (``shard_fn`` / ``merge_fn``) so that the
collective plumbing can be tested on CPU ranks with gloo.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _capi
from .native import _DTYPE_CODE, _require

ALIGN = 128  # shard bounds are multiples of 128 features


def shard_bounds(F: int, world: int, rank: int):
    """Contiguous, 128-aligned feature range [f0, f1) of `rank` (last rank takes the tail)."""
    per = -(-F // world)
    per = -(-per // ALIGN) * ALIGN
    f0 = min(F, rank * per)
    f1 = min(F, (rank + 1) * per)
    return f0, f1


def _cuda_shard_fn(X, W_shard, b_shard, k, f_offset, out_keys):
    B, d = X.shape
    Fs = W_shard.shape[0]
    lib = _capi.load()
    with torch.cuda.device(X.device):
        nbytes = _capi.workspace_bytes(B, d, Fs, k, _DTYPE_CODE[X.dtype])
        ws = torch.empty(max(nbytes, 8), dtype=torch.uint8, device=X.device)
        stream = torch.cuda.current_stream(X.device).cuda_stream
        _capi.check(lib.stk_shard_forward(X.data_ptr(), W_shard.data_ptr(), b_shard.data_ptr(),
                                          out_keys.data_ptr(), B, d, Fs, k, f_offset, _DTYPE_CODE[X.dtype],
                                          _capi.STK_FLAG_ANY_K | _capi.STK_FLAG_ANY_D, ws.data_ptr(), nbytes,
                                          stream))
    return out_keys


def _cuda_merge_fn(gathered, k):
    P, B, L = gathered.shape
    V = torch.empty((B, k), dtype=torch.float32, device=gathered.device)
    I = torch.empty((B, k), dtype=torch.int32, device=gathered.device)
    with torch.cuda.device(gathered.device):
        stream = torch.cuda.current_stream(gathered.device).cuda_stream
        _capi.check(_capi.load().stk_merge_keys(gathered.data_ptr(), P, B, k, V.data_ptr(), I.data_ptr(), stream))
    return V, I


class PeerExchangeUnavailable(RuntimeError):
    """Raised on every rank when some rank could not map its peers' buffers."""


class PeerExchange:
    """One rank's receive buffer of the direct GPU-to-GPU exchange.

    Collective: every rank of `group` constructs it with the same max_rows and
    k (the IPC handles are all-gathered over the group).  ``forward`` runs the
    shard's scores + top-k, the publish kernel and the final merge on the
    current stream.  ``close()`` (collective) unmaps the peers' buffers.
    """

    def __init__(self, max_rows, k, device, group=None, wait_seconds=10.0):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.max_rows, self.k, self.device = int(max_rows), int(k), torch.device(device)
        self.handle = None
        self.buf = None
        # Each step may fail on some ranks only; the ranks always run the same
        # collectives and decide together, so either every rank is connected
        # or every rank raises PeerExchangeUnavailable.
        mine, why = None, ""
        try:
            lib = _capi.load()
            nbytes = ctypes.c_size_t(0)
            _capi.check(lib.stk_exchange_bytes(self.world, self.max_rows, self.k, ctypes.byref(nbytes)))
            handle = ctypes.c_void_p()
            with torch.cuda.device(self.device):
                self.buf = torch.empty(int(nbytes.value), dtype=torch.uint8, device=self.device)
                _capi.check(lib.stk_exchange_create(self.rank, self.world, self.max_rows, self.k,
                                                    self.buf.data_ptr(), int(nbytes.value), float(wait_seconds),
                                                    ctypes.byref(handle)))
                self.handle = handle
                ipc = (ctypes.c_char * _capi.IPC_HANDLE_BYTES)()
                off = ctypes.c_int64(0)
                _capi.check(lib.stk_exchange_ipc_handle(self.handle, ipc, ctypes.byref(off)))
            mine = (bytes(ipc), int(off.value))
        except Exception as e:  # noqa: BLE001 - reported to every rank below
            why = f"rank {self.rank}: {e}"
        every = [None] * self.world
        dist.all_gather_object(every, (mine, why), group=group)
        if any(m is None for m, _ in every):
            self._release()
            raise PeerExchangeUnavailable(next(w for m, w in every if m is None))
        ok = 1
        try:
            handles = b"".join(m[0] for m, _ in every)
            offsets = (ctypes.c_int64 * self.world)(*[m[1] for m, _ in every])
            with torch.cuda.device(self.device):
                _capi.check(lib.stk_exchange_connect(self.handle, handles, offsets))
        except Exception as e:  # noqa: BLE001
            ok, why = 0, f"rank {self.rank}: {e}"
        verdict = [None] * self.world
        dist.all_gather_object(verdict, (ok, why), group=group)
        if not all(v for v, _ in verdict):
            self._release()
            raise PeerExchangeUnavailable(next(w for v, w in verdict if not v))

    def _release(self):
        if self.handle is not None:
            _capi.load().stk_exchange_destroy(self.handle)
            self.handle = None
        self.buf = None

    def forward(self, X, W_shard, b_shard, f_offset, V, I):
        B, d = X.shape
        Fs = W_shard.shape[0]
        lib = _capi.load()
        with torch.cuda.device(self.device):
            nbytes = _capi.workspace_bytes(B, d, Fs, self.k, _DTYPE_CODE[X.dtype]) if Fs > 0 else 0
            ws = torch.empty(max(nbytes, 8), dtype=torch.uint8, device=self.device)
            stream = torch.cuda.current_stream(self.device).cuda_stream
            _capi.check(lib.stk_exchange_forward(self.handle, X.data_ptr(), W_shard.data_ptr(), b_shard.data_ptr(),
                                                 V.data_ptr(), I.data_ptr(), B, d, Fs, self.k, f_offset,
                                                 _DTYPE_CODE[X.dtype], _capi.STK_FLAG_ANY_K | _capi.STK_FLAG_ANY_D,
                                                 ws.data_ptr(), nbytes, stream))
        return V, I

    def check_device_errors(self):
        """Synchronise this rank's stream and raise RuntimeError if a library
        kernel reported a device-side error since the last check (code 3: a wait
        for another rank's rows ran out)."""
        with torch.cuda.device(self.device):
            _capi.device_error(torch.cuda.current_stream(self.device).cuda_stream)

    def close(self):
        if self.handle is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        rc = _capi.load().stk_exchange_destroy(self.handle)
        self.handle = None
        dist.barrier(group=self.group)   # no rank frees its buffer while a peer still maps it
        self.buf = None
        _capi.check(rc)


class ShardedEncoder:
    """F-sharded exact (or approx, c >= k) top-k encoder for one rank.

    W_shard / b_shard: this rank's rows [f_offset, f_offset + F_shard) of
    W_enc / b_enc; F_total: the full F; k: top-k.  ``encode(X)`` takes the
    replicated (B, d) batch and returns (values fp32 (B, k), indices int32
    (B, k)), identical on every rank.

    ``encode`` is asynchronous and does not read the device error word (that
    would synchronise every step).  With the p2p transport a rank that stalls
    for longer than the exchange's wait limit makes the other ranks finish that
    step without its rows and set device error 3; call ``check_device_errors()``
    at a synchronisation point to turn that into an exception.  After a rank has
    skipped a step entirely the ranks stay a step apart: ``close()`` on every
    rank and encode again (a fresh exchange is set up collectively).
    """

    def __init__(self, W_shard, b_shard, F_total, f_offset, k, group=None, mode="exact", c=None,
                 shard_fn=None, merge_fn=None, transport="nccl", max_rows=128):
        k = int(k)
        _require(transport in ("nccl", "p2p", "auto"), "transport must be 'nccl', 'p2p' or 'auto'")
        _require(transport != "p2p" or (shard_fn is None and merge_fn is None),
                 "transport 'p2p' runs the library kernels only")
        _require(1 <= k <= 128, "k out of range")
        _require(mode in ("exact", "approx"), "mode must be 'exact' or 'approx'")
        if mode == "approx":
            _require(c in (16, 32, 64, 128), f"streamtopk_cuda_approx: unsupported c={c}. Supported: 16,32,64,128.")
            _require(k <= c, "k must be <= c")
        _require(k <= F_total, "k out of range")
        _require(W_shard.dim() == 2 and b_shard.dim() == 1 and b_shard.shape[0] == W_shard.shape[0],
                 "b_enc F-dim mismatch")
        self.W = W_shard.contiguous()
        self.b = b_shard.float().contiguous()
        self.F_total = int(F_total)
        self.f_offset = int(f_offset)
        self.k = k
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.L = _capi.list_len(k) if shard_fn is None else (32 if k <= 32 else 64 if k <= 64 else 128)
        self.shard_fn = shard_fn or _cuda_shard_fn
        self.merge_fn = merge_fn or _cuda_merge_fn
        self.transport = transport if self.world > 1 else "nccl"
        self.max_rows = int(max_rows)
        self.exchange = None
        self.fallback_reason = None
        self._pipe = None       # (handle, key, workspace) of the pipelined encode (submit / flush)
        self._pending = None    # the pending batch's (V, I): written by the next launch, kept alive until then

    def _peer_exchange(self, B, device):
        if self.exchange is not None and self.exchange.max_rows < B:
            self.flush()
            self._drop_pipeline()  # it holds the exchange being replaced
            self.exchange.close()
            self.exchange = None
        if self.exchange is None:
            try:
                self.exchange = PeerExchange(max(B, self.max_rows), self.k, device, group=self.group)
            except PeerExchangeUnavailable as e:
                if self.transport != "auto":
                    raise
                self.transport = "nccl"        # same decision on every rank (collective check)
                self.fallback_reason = str(e)
                return None
        return self.exchange

    def check_device_errors(self):
        """Synchronise the current stream of this rank's device and raise
        RuntimeError if a library kernel reported a device-side error."""
        dev = self.W.device
        with torch.cuda.device(dev):
            _capi.device_error(torch.cuda.current_stream(dev).cuda_stream)

    def close(self):
        """Release the pipeline and the p2p exchange (collective); a no-op for the NCCL transport."""
        self._drop_pipeline()
        if self.exchange is not None:
            self.exchange.close()
            self.exchange = None

    # ------------------------------------------------------------ pipelined encode
    def _drop_pipeline(self):
        if self._pipe is not None:
            torch.cuda.synchronize(self.W.device)
            _capi.load().stk_pipeline_destroy(self._pipe[0])
            self._pipe = None

    def _pipeline(self, X):
        B, d = X.shape
        key = (B, d, X.dtype)
        if self._pipe is not None and self._pipe[1] == key:
            return self._pipe[0]
        if self.transport not in ("p2p", "auto") or self.W.shape[0] == 0 or self.world == 1:
            return None
        if self._pipe is not None:  # another shape: finish its last batch first
            self.flush()
            self._drop_pipeline()
        ex = self._peer_exchange(B, X.device)
        if ex is None:
            return None
        lib = _capi.load()
        code = _DTYPE_CODE[X.dtype]
        flags = _capi.STK_FLAG_ANY_K | _capi.STK_FLAG_ANY_D
        nbytes = ctypes.c_size_t(0)
        _capi.check(lib.stk_pipeline_workspace_bytes(B, d, self.W.shape[0], self.k, code, flags,
                                                     ctypes.byref(nbytes)))
        with torch.cuda.device(X.device):
            ws = torch.empty(int(nbytes.value), dtype=torch.uint8, device=X.device)
            h = ctypes.c_void_p()
            _capi.check(lib.stk_pipeline_create_sharded(ctypes.byref(h), ex.handle, B, d, self.W.shape[0], self.k,
                                                        self.f_offset, code, flags, ws.data_ptr(),
                                                        int(nbytes.value)))
        self._pipe = (h, key, ws)
        return h

    def submit(self, X):
        """Pipelined encode of one batch (p2p transport): returns its (V, I),
        complete in stream order once the next batch is submitted or after
        ``flush()``.  Every rank submits the same batches in the same order.
        Without the p2p exchange this is ``encode`` (complete at once)."""
        X = X.contiguous()
        _require(X.dim() == 2 and X.shape[1] == self.W.shape[1], "W_enc d-dim mismatch")
        _require(X.dtype == self.W.dtype, "W_enc dtype must match X")
        B = X.shape[0]
        h = self._pipeline(X) if B > 0 else None
        if h is None:
            return self.encode(X)
        V = torch.empty((B, self.k), dtype=torch.float32, device=X.device)
        I = torch.empty((B, self.k), dtype=torch.int32, device=X.device)
        with torch.cuda.device(X.device):
            stream = torch.cuda.current_stream(X.device).cuda_stream
            _capi.check(_capi.load().stk_pipeline_submit(h, X.data_ptr(), self.W.data_ptr(), self.b.data_ptr(),
                                                         V.data_ptr(), I.data_ptr(), stream))
        self._pending = (V, I)
        return V, I

    def flush(self):
        """Finish the last submitted batch (no-op if none is pending)."""
        if self._pipe is None:
            return
        dev = self.W.device
        with torch.cuda.device(dev):
            _capi.check(_capi.load().stk_pipeline_flush(self._pipe[0], torch.cuda.current_stream(dev).cuda_stream))
        self._pending = None

    def encode(self, X):
        self.flush()  # a pending pipelined batch uses the exchange first
        X = X.contiguous()
        _require(X.dim() == 2 and X.shape[1] == self.W.shape[1], "W_enc d-dim mismatch")
        _require(X.dtype == self.W.dtype, "W_enc dtype must match X")
        B = X.shape[0]
        if self.transport in ("p2p", "auto"):
            V = torch.empty((B, self.k), dtype=torch.float32, device=X.device)
            I = torch.empty((B, self.k), dtype=torch.int32, device=X.device)
            if B == 0:
                return V, I
            ex = self._peer_exchange(B, X.device)
            if ex is not None:
                return ex.forward(X, self.W, self.b, self.f_offset, V, I)
        keys = torch.empty((B, self.L), dtype=torch.int64, device=X.device)
        if self.W.shape[0] > 0:
            self.shard_fn(X, self.W, self.b, self.k, self.f_offset, keys)
        else:
            keys.zero_()
        if self.world > 1:
            flat = torch.empty((self.world * B, self.L), dtype=torch.int64, device=X.device)
            dist.all_gather_into_tensor(flat, keys, group=self.group)
            gathered = flat.view(self.world, B, self.L)
        else:
            gathered = keys.unsqueeze(0)
        return self.merge_fn(gathered, self.k)


def topk_sae_cuda_exact_sharded(X, W_shard, b_shard, k, F_total, f_offset, group=None):
    """One-shot sharded exact encode over NCCL (see ShardedEncoder)."""
    return ShardedEncoder(W_shard, b_shard, F_total, f_offset, k, group=group).encode(X)
