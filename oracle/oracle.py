"""TEST INFRASTRUCTURE ONLY -- CPU oracle and parity checker.

Only tests/, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference leg may import this module, and only to check or to time the
reference.  The product (``streamtopk-sae_b200/``) never imports it.

Contents
  stream_topk      ctypes call into oracle/_build/libstk_oracle.so, a plain-C
                   restatement of the reference CPU op
                   (streamtopk_sae/csrc/cpu/streamtopk_cpu.cpp:15-79).
  ref_cpu_topk     the reference's own CPU op, compiled from its sources into
                   oracle/_ref/ by oracle/build_ref.py; called with the same
                   argument preparation as streamtopk_sae/ops.py:23-40.
  exact_topk_f64   exact top-k under the total order (score desc, index asc)
                   from float64 scores computed in F-chunks.
  check_topk       tie-aware parity check (values, distinctness, boundary
                   ties, value/index consistency) against float64 scores.
  gaussian_inputs  seeded numpy inputs with BASELINE.json's distributions.
"""
from __future__ import annotations

import ctypes
import glob
import importlib.util
import os
import subprocess
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None
_REF = None

# The reference accepts only these k (streamtopk_cpu.cpp:110-122,
# streamtopk_exact.cu:818-830); other k abort the reference process.
REF_K_SET = (1, 2, 4, 8, 16, 32, 64, 128)


def _lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(HERE, "_build", "libstk_oracle.so")
        if not os.path.isfile(path):
            subprocess.run(["make", "-C", HERE], check=True,
                           stdout=subprocess.DEVNULL)
        lib = ctypes.CDLL(path)
        i64 = ctypes.c_int64
        vp = ctypes.c_void_p
        lib.stk_oracle_stream_topk.argtypes = [vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, i64]
        lib.stk_oracle_stream_topk.restype = ctypes.c_int
        lib.stk_oracle_scores_f64.argtypes = [vp, vp, vp, vp, i64, i64, i64, i64, i64]
        lib.stk_oracle_scores_f64.restype = ctypes.c_int
        _LIB = lib
    return _LIB


def _f32(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def stream_topk(X, W, b, k, row_begin=0, row_end=None):
    """C restatement of the reference CPU streaming top-k (fp32, bias first).

    Returns (V, I) with V float32 (B,k), I int32 (B,k) in the reference's
    buffer order (descending for k <= 64, min-heap order for k > 64).
    """
    X, W, b = _f32(X), _f32(W), _f32(b)
    B, d = X.shape
    F = W.shape[0]
    if row_end is None:
        row_end = B
    V = np.empty((B, k), np.float32)
    I = np.empty((B, k), np.int32)
    rc = _lib().stk_oracle_stream_topk(
        X.ctypes.data, W.ctypes.data, b.ctypes.data, V.ctypes.data, I.ctypes.data,
        B, d, F, k, row_begin, row_end)
    if rc != 0:
        raise ValueError(f"stk_oracle_stream_topk rc={rc}")
    return V, I


def scores_f64_c(X, W, b, rows, f_begin, f_end):
    """float64 scores via the C loop (small sizes; independent of BLAS)."""
    X, W, b = _f32(X), _f32(W), _f32(b)
    r0, r1 = rows
    S = np.empty((r1 - r0, f_end - f_begin), np.float64)
    rc = _lib().stk_oracle_scores_f64(X.ctypes.data, W.ctypes.data, b.ctypes.data,
                                      S.ctypes.data, X.shape[1], r0, r1, f_begin, f_end)
    if rc != 0:
        raise ValueError(f"stk_oracle_scores_f64 rc={rc}")
    return S


def scores_f64(X, W, b, f_begin=0, f_end=None):
    """float64 scores X @ W[f_begin:f_end].T + b[f_begin:f_end] (numpy BLAS)."""
    X = np.asarray(X, dtype=np.float64)
    if f_end is None:
        f_end = W.shape[0]
    Wc = np.asarray(W[f_begin:f_end], dtype=np.float64)
    return X @ Wc.T + np.asarray(b[f_begin:f_end], dtype=np.float64)[None, :]


def _topk_total_order(S, k, f_offset=0):
    """Top-k of each row of S under (score desc, index asc). Returns (vals, idx)."""
    B, n = S.shape
    kk = min(k, n)
    idx = np.broadcast_to(np.arange(n, dtype=np.int64), S.shape)
    order = np.lexsort((idx, -S), axis=1)[:, :kk]
    return np.take_along_axis(S, order, axis=1), order + f_offset


def exact_topk_f64(X, W, b, k, chunk=16384, margin=0):
    """Exact top-(k+margin) under (score desc, index asc) with float64 scores.

    Ties at the boundary are resolved by the smaller index, which is the order
    the CUDA path uses; tie-aware checks do not depend on it.
    """
    X = np.asarray(X)
    F = W.shape[0]
    kk = min(k + margin, F)
    best_v = None
    best_i = None
    for f0 in range(0, F, chunk):
        f1 = min(F, f0 + chunk)
        S = scores_f64(X, W, b, f0, f1)
        v, i = _topk_total_order(S, kk, f0)
        if best_v is None:
            best_v, best_i = v, i
        else:
            cv = np.concatenate([best_v, v], axis=1)
            ci = np.concatenate([best_i, i], axis=1)
            o = np.lexsort((ci, -cv), axis=1)[:, :kk]
            best_v = np.take_along_axis(cv, o, axis=1)
            best_i = np.take_along_axis(ci, o, axis=1)
    return best_v, best_i


def gather_scores_f64(X, W, b, idx):
    """float64 score of (row r, feature idx[r, j]) for every entry of idx."""
    X = np.asarray(X, dtype=np.float64)
    idx = np.asarray(idx, dtype=np.int64)
    B, k = idx.shape
    out = np.empty((B, k), np.float64)
    for r in range(B):
        Wr = np.asarray(W[idx[r]], dtype=np.float64)
        out[r] = Wr @ X[r] + np.asarray(b, dtype=np.float64)[idx[r]]
    return out


@dataclass
class TopkCheck:
    ok: bool
    bad_rows: list
    messages: list
    tie_recall: float

    def raise_if_bad(self):
        if not self.ok:
            raise AssertionError("; ".join(self.messages[:8]))


def check_topk(pred_v, pred_i, X, W, b, k, rtol, oracle=None, F=None):
    """Tie-aware parity of a (values, indices) prediction against float64 scores.

    Per row, with v_1..v_k the oracle's top-k scores and tau = rtol*max|v_j|:
      (i)   sorted predicted values match the sorted oracle values within tau;
      (ii)  predicted indices are distinct and in [0, F);
      (iii) every predicted index has oracle score >= v_k - tau;
      (iv)  every oracle index with score > v_k + tau is predicted;
      (v)   each predicted value matches the oracle score at its index within tau.
    tie_recall = fraction of rows satisfying (ii)-(iv).
    """
    pred_v = np.asarray(pred_v, dtype=np.float64)
    pred_i = np.asarray(pred_i, dtype=np.int64)
    B = pred_v.shape[0]
    if F is None:
        F = W.shape[0]
    if oracle is None:
        oracle = exact_topk_f64(X, W, b, k)
    ov, oi = oracle
    ov = ov[:, :k]
    oi = oi[:, :k]
    bad, msgs, tie_ok = [], [], 0
    if pred_v.shape != (B, k) or pred_i.shape != (B, k):
        return TopkCheck(False, list(range(B)), [f"shape {pred_v.shape}/{pred_i.shape} != {(B, k)}"], 0.0)
    in_range = (pred_i >= 0) & (pred_i < F)
    safe_i = np.where(in_range, pred_i, 0)
    ps = gather_scores_f64(X, W, b, safe_i)
    for r in range(B):
        tau = rtol * max(np.max(np.abs(ov[r])), 1e-30)
        vk = ov[r, -1]
        row_msgs = []
        pv = np.sort(pred_v[r])[::-1]
        if not np.all(np.abs(pv - ov[r]) <= tau):
            j = int(np.argmax(np.abs(pv - ov[r])))
            row_msgs.append(f"row {r}: sorted value {j} pred={pv[j]:.8g} oracle={ov[r, j]:.8g} tau={tau:.3g}")
        tie_row = True
        if not np.all(in_range[r]):
            row_msgs.append(f"row {r}: index out of range {pred_i[r][~in_range[r]][:4]}")
            tie_row = False
        if len(set(pred_i[r].tolist())) != k:
            row_msgs.append(f"row {r}: duplicate indices")
            tie_row = False
        if np.any(ps[r] < vk - tau):
            j = int(np.argmin(ps[r]))
            row_msgs.append(f"row {r}: predicted idx {pred_i[r, j]} score {ps[r, j]:.8g} < v_k-tau {vk - tau:.8g}")
            tie_row = False
        must = set(oi[r][ov[r] > vk + tau].tolist())
        missing = must - set(pred_i[r].tolist())
        if missing:
            row_msgs.append(f"row {r}: missing certain indices {sorted(missing)[:4]}")
            tie_row = False
        if np.any(np.abs(pred_v[r] - ps[r]) > tau):
            j = int(np.argmax(np.abs(pred_v[r] - ps[r])))
            row_msgs.append(f"row {r}: value/index mismatch at {j}: val={pred_v[r, j]:.8g} score={ps[r, j]:.8g}")
        tie_ok += int(tie_row)
        if row_msgs:
            bad.append(r)
            msgs.extend(row_msgs)
    return TopkCheck(not bad, bad, msgs, tie_ok / max(B, 1))


def recall_at_k(pred_i, true_i):
    """The reference's recall (streamtopk_sae/utils.py:23-36): mean |pred & true| / k."""
    pred_i = np.asarray(pred_i)
    true_i = np.asarray(true_i)
    B, k = true_i.shape
    return float(np.mean([len(set(pred_i[r].tolist()) & set(true_i[r].tolist())) / k
                          for r in range(B)]))


def tie_aware_recall(pred_i, X, W, b, k, rtol, oracle=None):
    """Fraction of predicted indices whose score is within tau of the true top-k.

    A predicted index counts as a hit if its float64 score is >= v_k - tau; the
    per-row hit count is capped at k and duplicates count once.
    """
    if oracle is None:
        oracle = exact_topk_f64(X, W, b, k)
    ov = oracle[0][:, :k]
    pred_i = np.asarray(pred_i, dtype=np.int64)
    ps = gather_scores_f64(X, W, b, np.clip(pred_i, 0, W.shape[0] - 1))
    tot = 0.0
    for r in range(pred_i.shape[0]):
        tau = rtol * max(np.max(np.abs(ov[r])), 1e-30)
        seen = set()
        hits = 0
        for j in range(k):
            t = int(pred_i[r, j])
            if t in seen or t < 0 or t >= W.shape[0]:
                continue
            seen.add(t)
            hits += int(ps[r, j] >= ov[r, -1] - tau)
        tot += min(hits, k) / k
    return tot / pred_i.shape[0]


def gaussian_inputs(B, d, F, seed=0, w_scale="1/d", bias_std=0.1):
    """Seeded numpy inputs with BASELINE.json's distributions (float32).

    X ~ N(0,1); W ~ N(0, 1/d) (w_scale="1/d") or rows N(0,1) L2-normalised
    (w_scale="unit"); b ~ N(0, bias_std^2).  BASELINE.json writes b ~ N(0,0.01),
    read here as variance 0.01 (std 0.1).
    """
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((B, d), dtype=np.float32)
    W = rng.standard_normal((F, d), dtype=np.float32)
    if w_scale == "unit":
        W /= np.maximum(np.linalg.norm(W, axis=1, keepdims=True), 1e-8)
    else:
        W *= np.float32(1.0 / np.sqrt(d))
    b = (rng.standard_normal(F, dtype=np.float32) * np.float32(bias_std)).astype(np.float32)
    return X, W, b


# ---------------------------------------------------------------------------
# The reference's own CPU op (compiled from its sources into oracle/_ref/).
# ---------------------------------------------------------------------------

def ref_available() -> bool:
    return bool(glob.glob(os.path.join(HERE, "_ref", "streamtopk_sae_native*.so")))


def _ref_mod():
    global _REF
    if _REF is None:
        import torch  # noqa: F401  (the module links against libtorch)
        paths = glob.glob(os.path.join(HERE, "_ref", "streamtopk_sae_native*.so"))
        if not paths:
            raise FileNotFoundError("oracle/_ref/streamtopk_sae_native*.so not built "
                                    "(python oracle/build_ref.py)")
        spec = importlib.util.spec_from_file_location("streamtopk_sae_native", paths[0])
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        _REF = mod
    return _REF


def ref_cpu_topk(X, W, b, k):
    """Reference ``topk_sae_cpu`` (streamtopk_sae/ops.py:23-40) on torch CPU tensors.

    Only k in REF_K_SET is passed through: other k abort the reference process.
    """
    import torch
    if k not in REF_K_SET:
        raise ValueError(f"reference CPU op does not support k={k}")
    X = torch.as_tensor(X)
    W = torch.as_tensor(W)
    b = torch.as_tensor(b)
    if X.dtype != torch.float32:
        X = X.float()
        W = W.float()
    if b.dtype != torch.float32:
        b = b.float()
    return _ref_mod().streamtopk_cpu_forward(X.contiguous(), W.contiguous(), b.contiguous(), k)
