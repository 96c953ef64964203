"""Generate the golden fixtures in tests/golden/ from the reference itself.

Run in a container where the reference tree exists (it is not needed at test
time):

    python oracle/build_ref.py --ref <reference tree>          # reference CPU op -> oracle/_ref/
    python tests/golden/make_golden.py --ref <reference tree>  # writes tests/golden/golden_cpu.npz

(or set STK_REFERENCE_ROOT instead of passing --ref)

Every output in the fixture is produced by the reference's own code:
  * ``streamtopk_cpu_forward`` compiled from the reference sources
    (oracle/_ref/, called with the argument preparation of
    streamtopk_sae/ops.py:23-40), and
  * for the "syn_*" cases, inputs from the reference's synthetic generator
    ``generate_realistic_preacts`` (streamtopk_sae/synthetic.py:20-100),
    imported from the reference tree with the shapes/seeds of
    tests/test_correctness.py:16-33,137-143.
Gaussian cases regenerate their inputs from a numpy PCG64 seed
(``oracle.gaussian_inputs`` and the per-case edits below), so only the seed,
an input digest and the outputs are stored.
"""
import argparse
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle import oracle  # noqa: E402


def digest(*arrs):
    h = hashlib.sha256()
    for a in arrs:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()[:16]


# name -> (B, d, F, k, seed, kind)
GAUSS_CASES = {
    "gauss_cfg1": (32, 768, 16384, 32, 0, "plain"),
    "gauss_k128": (8, 64, 1024, 128, 1, "plain"),        # heap-order output (k > 64)
    "gauss_k64": (8, 96, 2048, 64, 2, "plain"),
    "gauss_F300": (8, 128, 300, 16, 3, "plain"),         # F not a multiple of any tile
    "gauss_k1": (8, 64, 256, 1, 4, "plain"),
    "gauss_kF16": (4, 64, 16, 16, 5, "plain"),           # k == F
    "gauss_zeroX": (4, 64, 128, 8, 6, "zero_x"),         # all-zero X
    "gauss_bigbias": (4, 64, 128, 8, 7, "big_bias"),     # b[0] = 1e6
    "gauss_outliers": (16, 128, 4096, 32, 8, "outliers"),  # +-100 bias on 1% of features
    "gauss_k2_d100": (8, 100, 700, 2, 9, "plain"),       # d not a multiple of 8
}


def gauss_case_inputs(B, d, F, seed, kind):
    """Inputs of a Gaussian golden case (shared with the tests)."""
    X, W, b = oracle.gaussian_inputs(B, d, F, seed=seed)
    if kind == "zero_x":
        X[:] = 0.0
        b = np.random.default_rng(seed + 1000).standard_normal(F).astype(np.float32)
    elif kind == "big_bias":
        b[:] = 0.0
        b[0] = 1e6
    elif kind == "outliers":
        rng = np.random.default_rng(seed + 2000)
        n = max(1, F // 100)
        pos = rng.choice(F, size=n, replace=False)
        b[pos] = np.where(rng.random(n) < 0.5, -100.0, 100.0).astype(np.float32)
    return X, W, b


SYN_CASES = {
    # name -> (B, d, F, k, seed, dtype)   shapes of tests/test_correctness.py
    "syn_small": (4, 64, 256, 8, 42, "fp32"),
    "syn_k16": (16, 128, 512, 16, 42, "fp32"),
    "syn_k32": (16, 128, 512, 32, 42, "fp32"),
    "syn_k64": (16, 128, 512, 64, 42, "fp32"),
    "syn_small_bf16": (4, 64, 256, 8, 42, "bf16"),
}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("STK_REFERENCE_ROOT"), required="STK_REFERENCE_ROOT" not in os.environ,
                    help="root of the reference tree (default: $STK_REFERENCE_ROOT)")
    ap.add_argument("--out", default=os.path.join(HERE, "golden_cpu.npz"))
    a = ap.parse_args()
    import torch
    if not oracle.ref_available():
        from oracle.build_ref import build
        build(a.ref)
    out = {}
    for name, (B, d, F, k, seed, kind) in GAUSS_CASES.items():
        X, W, b = gauss_case_inputs(B, d, F, seed, kind)
        V, I = oracle.ref_cpu_topk(torch.from_numpy(X), torch.from_numpy(W), torch.from_numpy(b), k)
        out[f"{name}/meta"] = np.array([B, d, F, k, seed], np.int64)
        out[f"{name}/kind"] = np.array(kind)
        out[f"{name}/digest"] = np.array(digest(X, W, b))
        out[f"{name}/V"] = V.numpy()
        out[f"{name}/I"] = I.numpy()
        print(name, V.shape)
    sys.path.insert(0, a.ref)
    from streamtopk_sae.synthetic import generate_realistic_preacts
    tdt = {"fp32": torch.float32, "bf16": torch.bfloat16}
    for name, (B, d, F, k, seed, dt) in SYN_CASES.items():
        X, W, b = generate_realistic_preacts(B, F, d, k_effective=k, seed=seed, dtype=tdt[dt])
        V, I = oracle.ref_cpu_topk(X, W, b, k)
        out[f"{name}/meta"] = np.array([B, d, F, k, seed], np.int64)
        out[f"{name}/dtype"] = np.array(dt)
        if dt == "bf16":
            out[f"{name}/X_bf16"] = X.view(torch.int16).numpy()
            out[f"{name}/W_bf16"] = W.view(torch.int16).numpy()
        else:
            out[f"{name}/X"] = X.numpy()
            out[f"{name}/W"] = W.numpy()
        out[f"{name}/b"] = b.numpy()
        out[f"{name}/V"] = V.numpy()
        out[f"{name}/I"] = I.numpy()
        print(name, V.shape)
    np.savez_compressed(a.out, **out)
    print("wrote", a.out, os.path.getsize(a.out), "bytes")


if __name__ == "__main__":
    main()
