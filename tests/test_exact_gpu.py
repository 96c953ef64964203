"""Parity of the exact encoder (sm_100a kernels via the C ABI) with the oracle.

Mirrors the reference's CUDA tests (tests/test_correctness.py:159-284 in the
reference: shapes x dtypes, k sweep, k = F, k = 1, F not a multiple of the
tile, all-zero X, huge bias) with tie-aware checks of values AND indices
against float64 scores, plus BASELINE.json's edge set (+-100 bias outliers on
1% of features) and shapes that exercise the tile/range/M-tile boundaries.
"""
import numpy as np
import pytest
import torch

from gpu_util import RTOL, check, device_inputs, no_device_error
from make_golden import GAUSS_CASES, gauss_case_inputs
from oracle import oracle

pytestmark = pytest.mark.gpu

SHAPES = {
    "small": dict(B=4, d=64, F=256, k=8),
    "medium": dict(B=32, d=512, F=4096, k=32),
    "large": dict(B=128, d=2048, F=131072, k=64),
}


def _run(X, W, b, k, dtype_name, **kw):
    import streamtopk_sae as stk
    Xt, Wt, bt, Xr, Wr, br = device_inputs(X, W, b, dtype_name)
    V, I = stk.topk_sae_cuda_exact(Xt, Wt, bt, k, **kw)
    torch.cuda.synchronize()
    no_device_error()
    return V, I, Xr, Wr, br


@pytest.mark.parametrize("shape", ["small", "medium", "large"])
@pytest.mark.parametrize("dtype_name", ["fp32", "fp16", "bf16"])
def test_exact_shapes(shape, dtype_name):
    s = SHAPES[shape]
    X, W, b = oracle.gaussian_inputs(s["B"], s["d"], s["F"], seed=42)
    V, I, Xr, Wr, br = _run(X, W, b, s["k"], dtype_name)
    check(V, I, Xr, Wr, br, s["k"], RTOL[dtype_name])


@pytest.mark.parametrize("k", [1, 2, 4, 8, 16, 32, 64, 128])
@pytest.mark.parametrize("dtype_name", ["bf16", "fp32"])
def test_exact_k_sweep(k, dtype_name):
    X, W, b = oracle.gaussian_inputs(16, 128, 2048, seed=k)
    V, I, Xr, Wr, br = _run(X, W, b, k, dtype_name)
    check(V, I, Xr, Wr, br, k, RTOL[dtype_name])


@pytest.mark.parametrize("dtype_name", ["bf16", "fp16", "fp32"])
@pytest.mark.parametrize("B,d,F,k", [
    (8, 128, 300, 16),       # F not a multiple of 32 / 128 / 256 (reference F=300 case)
    (4, 64, 16, 16),         # k == F
    (8, 64, 256, 1),         # k == 1
    (1, 64, 1000, 8),        # single row
    (129, 64, 700, 32),      # two M tiles, the second with one row
    (300, 96, 5000, 64),     # three M tiles
    (5, 64, 33, 32),         # one full chunk plus one feature
    (16, 72, 4100, 32),      # d not a multiple of 64 (TMA K tail)
    (64, 100, 2000, 16),     # d not a multiple of 8 (SIMT path for 16-bit types)
    (8, 4096, 3000, 64),     # d at the reference's D_MAX
])
def test_exact_edge_shapes(B, d, F, k, dtype_name):
    X, W, b = oracle.gaussian_inputs(B, d, F, seed=B * 7 + F)
    V, I, Xr, Wr, br = _run(X, W, b, k, dtype_name)
    check(V, I, Xr, Wr, br, k, RTOL[dtype_name])


@pytest.mark.parametrize("dtype_name", ["bf16", "fp32"])
def test_exact_all_zero_x(dtype_name):
    """All scores equal the bias (reference test_edge_all_zero_X)."""
    X, W, b = oracle.gaussian_inputs(4, 64, 128, seed=3)
    X[:] = 0
    b = np.random.default_rng(1).standard_normal(128).astype(np.float32)
    V, I, Xr, Wr, br = _run(X, W, b, 8, dtype_name)
    check(V, I, Xr, Wr, br, 8, RTOL[dtype_name])


def test_exact_zero_x_zero_bias_ties():
    """Every score is 0: the smallest feature indices win (deterministic ties)."""
    X = np.zeros((3, 64), np.float32)
    W = np.random.default_rng(0).standard_normal((500, 64)).astype(np.float32)
    b = np.zeros(500, np.float32)
    V, I, *_ = _run(X, W, b, 16, "bf16")
    assert torch.all(V == 0)
    assert torch.equal(I.cpu(), torch.arange(16, dtype=torch.int32).expand(3, 16))


@pytest.mark.parametrize("dtype_name", ["bf16", "fp32"])
def test_exact_huge_bias(dtype_name):
    """b[0] = 1e6 must be in every row (reference test_edge_large_bias)."""
    X, W, b = oracle.gaussian_inputs(4, 64, 128, seed=4)
    b[:] = 0
    b[0] = 1e6
    V, I, Xr, Wr, br = _run(X, W, b, 8, dtype_name)
    assert torch.all(I[:, 0] == 0)
    check(V, I, Xr, Wr, br, 8, RTOL[dtype_name])


@pytest.mark.parametrize("dtype_name", ["bf16", "fp16", "fp32"])
def test_exact_bias_outliers(dtype_name):
    """BASELINE.json edge set: +-100 bias on 1% of features."""
    B, d, F, k, seed, kind = GAUSS_CASES["gauss_outliers"]
    X, W, b = gauss_case_inputs(B, d, F, seed, kind)
    V, I, Xr, Wr, br = _run(X, W, b, k, dtype_name)
    check(V, I, Xr, Wr, br, k, RTOL[dtype_name])


def test_increasing_scores_stress_merges():
    """Scores rise with the feature index, so every feature beats the running
    threshold: the worst case for the per-row merge machinery."""
    F, d, k = 6000, 64, 128
    X = np.ones((8, d), np.float32)
    W = np.zeros((F, d), np.float32)
    b = (np.arange(F, dtype=np.float32) * 1e-3)
    V, I, Xr, Wr, br = _run(X, W, b, k, "bf16")
    expect = torch.arange(F - 1, F - 1 - k, -1, dtype=torch.int32).expand(8, k)
    assert torch.equal(I.cpu(), expect)
    check(V, I, Xr, Wr, br, k, RTOL["bf16"])


@pytest.mark.parametrize("name", sorted(GAUSS_CASES))
def test_exact_matches_reference_golden(golden, name):
    """fp32 inputs of the golden cases: agree with the reference's own outputs."""
    B, d, F, k, seed, kind = GAUSS_CASES[name]
    X, W, b = gauss_case_inputs(B, d, F, seed, kind)
    V, I, Xr, Wr, br = _run(X, W, b, k, "fp32")
    Vr, Ir = golden[f"{name}/V"], golden[f"{name}/I"]
    Vs = np.sort(Vr, axis=1)[:, ::-1]
    tol = RTOL["fp32"] * np.maximum(np.abs(Vr).max(axis=1, keepdims=True), 1e-30)
    assert np.all(np.abs(V.cpu().numpy() - Vs) <= tol)
    ov = oracle.exact_topk_f64(Xr, Wr, br, k)
    for r in range(B):
        if set(I[r].tolist()) != set(Ir[r].tolist()):
            # only boundary ties may differ
            vk = ov[0][r, -1]
            diff = set(I[r].tolist()) ^ set(Ir[r].tolist())
            for f in diff:
                s = float(np.dot(Wr[f].astype(np.float64), Xr[r].astype(np.float64)) + br[f])
                assert abs(s - vk) <= 1e-5 * max(abs(vk), 1e-30), (r, f, s, vk)


@pytest.mark.parametrize("dtype_name", ["bf16", "fp16"])
def test_tensor_core_and_simt_paths_agree(dtype_name):
    """The tcgen05 path and the SIMT path select the same features."""
    import streamtopk_sae as stk
    from streamtopk_sae import _capi, native
    X, W, b = oracle.gaussian_inputs(96, 256, 9000, seed=5)
    Xt, Wt, bt, Xr, Wr, br = device_inputs(X, W, b, dtype_name)
    V1, I1 = stk.topk_sae_cuda_exact(Xt, Wt, bt, 32)
    V2, I2 = native.streamtopk_cuda_exact_forward(Xt, Wt, bt, 32, flags=_capi.STK_FLAG_SIMT)
    torch.cuda.synchronize()
    no_device_error()
    check(V1, I1, Xr, Wr, br, 32, RTOL[dtype_name])
    check(V2, I2, Xr, Wr, br, 32, RTOL[dtype_name])
    assert torch.allclose(V1, V2, rtol=1e-4, atol=1e-5)


def test_deterministic_across_calls():
    import streamtopk_sae as stk
    X, W, b = oracle.gaussian_inputs(64, 512, 20000, seed=9)
    Xt, Wt, bt, *_ = device_inputs(X, W, b, "bf16")
    V1, I1 = stk.topk_sae_cuda_exact(Xt, Wt, bt, 64)
    V2, I2 = stk.topk_sae_cuda_exact(Xt, Wt, bt, 64)
    assert torch.equal(V1, V2) and torch.equal(I1, I2)


def test_argument_errors_match_reference():
    import streamtopk_sae as stk
    X = torch.randn(4, 64, device="cuda", dtype=torch.bfloat16)
    W = torch.randn(128, 64, device="cuda", dtype=torch.bfloat16)
    b = torch.zeros(128, device="cuda")
    with pytest.raises(RuntimeError, match="unsupported k=3"):
        stk.topk_sae_cuda_exact(X, W, b, 3)
    with pytest.raises(RuntimeError, match="k out of range"):
        stk.topk_sae_cuda_exact(X, W, b, 129)
    with pytest.raises(RuntimeError, match="W_enc dtype must match X"):
        stk.topk_sae_cuda_exact(X, W.float(), b, 8)
    with pytest.raises(RuntimeError, match="W_enc d-dim mismatch"):
        stk.topk_sae_cuda_exact(X, W[:, :32].contiguous(), b, 8)
    with pytest.raises(RuntimeError, match="b_enc F-dim mismatch"):
        stk.topk_sae_cuda_exact(X, W, b[:64], 8)
    with pytest.raises(RuntimeError, match="d exceeds D_MAX=4096"):
        Xb = torch.randn(2, 4104, device="cuda", dtype=torch.bfloat16)
        Wb = torch.randn(64, 4104, device="cuda", dtype=torch.bfloat16)
        stk.topk_sae_cuda_exact(Xb, Wb, torch.zeros(64, device="cuda"), 8)
    # the extension flags lift the two limits
    V, I = stk.topk_sae_cuda_exact(X, W, b, 3, allow_any_k=True)
    assert V.shape == (4, 3)


def test_bias_cast_and_noncontiguous_inputs():
    """ops casts b_enc to fp32 and makes inputs contiguous (reference ops.py:50-55)."""
    import streamtopk_sae as stk
    X, W, b = oracle.gaussian_inputs(8, 128, 1024, seed=12)
    Xt, Wt, bt, Xr, Wr, br = device_inputs(X, W, b, "bf16")
    Wnc = Wt.t().contiguous().t()
    V, I = stk.topk_sae_cuda_exact(Xt, Wnc, bt.double(), 16)
    check(V, I, Xr, Wr, br, 16, RTOL["bf16"])


@pytest.mark.parametrize("B,d,F,k", [(128, 256, 65536, 64), (96, 512, 40000, 32), (200, 128, 30000, 128),
                                     (128, 64, 300000, 16), (384, 256, 60000, 32), (640, 128, 40000, 128)])
def test_sampled_floor_changes_nothing(B, d, F, k):
    """The sampled threshold floor (B <= 256) and the floor the units of an M
    tile share (B > 256, several units per CTA) only skip work: results are
    bitwise equal with and without them (keys are unique, so the top-k is
    unique)."""
    from streamtopk_sae import _capi, native
    X, W, b = oracle.gaussian_inputs(B, d, F, seed=F % 1000)
    Xt, Wt, bt, Xr, Wr, br = device_inputs(X, W, b, "bf16")
    V1, I1 = native.streamtopk_cuda_exact_forward(Xt, Wt, bt, k)
    V2, I2 = native.streamtopk_cuda_exact_forward(Xt, Wt, bt, k, flags=_capi.STK_FLAG_NO_PILOT)
    torch.cuda.synchronize()
    no_device_error()
    assert torch.equal(V1, V2) and torch.equal(I1, I2)
    if F <= 70000:
        check(V1, I1, Xr, Wr, br, k, RTOL["bf16"])


@pytest.mark.parametrize("B,d,F,k,dt", [(1024, 256, 30000, 128, "bf16"), (2048, 512, 20000, 128, "fp16"),
                                        (1024, 128, 50000, 100, "bf16"), (768, 64, 9000, 128, "bf16")])
def test_cta_pairs_equal_single_cta(B, d, F, k, dt):
    """k > 64 with an even number of 128-row M tiles and several units per CTA
    runs as CTA pairs (tcgen05 cta_group::2, M = 256, each CTA loading half of
    the W tile): bit-identical to the one-CTA kernel, and right against float64."""
    from streamtopk_sae import _capi, native
    X, W, b = oracle.gaussian_inputs(B, d, F, seed=B + d)
    Xt, Wt, bt, Xr, Wr, br = device_inputs(X, W, b, dt)
    flags = _capi.STK_FLAG_ANY_K
    V1, I1 = native.streamtopk_cuda_exact_forward(Xt, Wt, bt, k, flags=flags)
    V2, I2 = native.streamtopk_cuda_exact_forward(Xt, Wt, bt, k, flags=flags | _capi.STK_FLAG_NO_PAIR)
    torch.cuda.synchronize()
    no_device_error()
    assert torch.equal(V1, V2) and torch.equal(I1, I2)
    rows = np.array(sorted({0, 1, B // 2, B - 2, B - 1}))
    rt = torch.from_numpy(rows).cuda()
    check(V1[rt], I1[rt], Xr[rows], Wr, br, k, RTOL[dt])


@pytest.mark.parametrize("B,d,F,k", [(128, 512, 60000, 64), (256, 256, 40000, 32), (200, 128, 30000, 128),
                                     (7, 64, 300, 16), (128, 64, 6000, 128), (1, 64, 100000, 1)])
def test_fused_finish_equals_separate_finish(B, d, F, k):
    """The finish step in the fused kernel's tail (grid barrier, per-row select in
    the same launch) and the standalone finish kernel give bit-identical rows."""
    from streamtopk_sae import _capi, native
    X, W, b = oracle.gaussian_inputs(B, d, F, seed=B + F)
    if F == 6000:   # scores rise with the index: every list is full, the fold path runs
        X[:] = 1.0
        W[:] = 0.0
        b = np.arange(F, dtype=np.float32) * 1e-3
    Xt, Wt, bt, Xr, Wr, br = device_inputs(X, W, b, "bf16")
    V1, I1 = native.streamtopk_cuda_exact_forward(Xt, Wt, bt, k)
    V2, I2 = native.streamtopk_cuda_exact_forward(Xt, Wt, bt, k, flags=_capi.STK_FLAG_SEPARATE_FINISH)
    torch.cuda.synchronize()
    no_device_error()
    assert torch.equal(V1, V2) and torch.equal(I1, I2)
    check(V1, I1, Xr, Wr, br, k, RTOL["bf16"])


@pytest.mark.parametrize("k", [16, 64, 128])
def test_exchange_single_rank_equals_exact(k):
    """A one-rank peer exchange (publish kernel into its own receive buffer, arrival
    counters, final merge) over several steps equals the exact encode."""
    import ctypes
    import streamtopk_sae as stk
    from streamtopk_sae import _capi
    lib = _capi.load()
    B, d, F = 128, 1024, 50000
    X, W, b = stk.make_inputs(B, d, F, dtype=torch.bfloat16, seed=5, device="cuda", w_init="unit_rows")
    nbytes = ctypes.c_size_t(0)
    _capi.check(lib.stk_exchange_bytes(1, B, k, ctypes.byref(nbytes)))
    buf = torch.empty(nbytes.value, dtype=torch.uint8, device="cuda")
    h = ctypes.c_void_p()
    _capi.check(lib.stk_exchange_create(0, 1, B, k, buf.data_ptr(), nbytes.value, 5.0, ctypes.byref(h)))
    try:
        _capi.check(lib.stk_exchange_connect(h, b"\0" * _capi.IPC_HANDLE_BYTES, (ctypes.c_int64 * 1)(0)))
        wsb = _capi.workspace_bytes(B, d, F, k, _capi.STK_BF16)
        ws = torch.empty(max(wsb, 8), dtype=torch.uint8, device="cuda")
        stream = torch.cuda.current_stream().cuda_stream
        Ve, Ie = stk.topk_sae_cuda_exact(X, W, b, k)
        # both receive slots and the step counter; the finish in the score
        # kernel's tail and in the standalone finish kernel, alternately
        for step in range(4):
            V = torch.empty((B, k), dtype=torch.float32, device="cuda")
            I = torch.empty((B, k), dtype=torch.int32, device="cuda")
            flags = _capi.STK_FLAG_SEPARATE_FINISH if step % 2 else 0
            _capi.check(lib.stk_exchange_forward(h, X.data_ptr(), W.data_ptr(), b.data_ptr(), V.data_ptr(),
                                                 I.data_ptr(), B, d, F, k, 0, _capi.STK_BF16, flags, ws.data_ptr(),
                                                 wsb, stream))
            torch.cuda.synchronize()
            assert torch.equal(V, Ve) and torch.equal(I, Ie)
        assert _capi.device_error(stream) == 0
    finally:
        lib.stk_exchange_destroy(h)


@pytest.mark.parametrize("B,d,F,k", [(128, 768, 65536, 32), (64, 256, 30001, 64), (130, 100, 5000, 16),
                                     (1, 64, 300, 8), (32, 2048, 20000, 128), (128, 2048, 262144, 64)])
def test_tf32_path_matches_oracle(B, d, F, k):
    """fp32 inputs on tensor cores (STK_FLAG_TF32: round_tf32 split, 3 passes) within the fp32 tolerance."""
    from streamtopk_sae import _capi, native
    X, W, b = oracle.gaussian_inputs(B, d, F, seed=B + d + k)
    Xt, Wt, bt, Xr, Wr, br = device_inputs(X, W, b, "fp32")
    V, I = native.streamtopk_cuda_exact_forward(Xt, Wt, bt, k, flags=_capi.STK_FLAG_TF32)
    torch.cuda.synchronize()
    no_device_error()
    check(V, I, Xr, Wr, br, k, RTOL["fp32"])


def test_tf32_path_ties_and_zero_x():
    """All-equal scores rank by feature index on the TF32 path too."""
    from streamtopk_sae import _capi, native
    B, d, F, k = 16, 128, 3000, 32
    X = torch.zeros(B, d, device="cuda")
    W = torch.randn(F, d, device="cuda")
    b = torch.zeros(F, device="cuda")
    V, I = native.streamtopk_cuda_exact_forward(X, W, b, k, flags=_capi.STK_FLAG_TF32)
    torch.cuda.synchronize()
    assert torch.equal(I.cpu(), torch.arange(k, dtype=torch.int32).expand(B, k))
    assert torch.all(V == 0)


@pytest.mark.parametrize("B,d,F,k", [(128, 2048, 262144, 64), (128, 768, 65536, 32), (300, 256, 50000, 128)])
def test_working_memory_is_the_workspace(B, d, F, k):
    """Peak device memory of a call = inputs + V/I + the workspace the C ABI reports
    (the reference's run_memory.py 'working memory'); no F-sized scratch."""
    import streamtopk_sae as stk
    from streamtopk_sae import _capi
    X, W, b = stk.make_inputs(B, d, F, dtype=torch.bfloat16, seed=1, device="cuda")
    stk.topk_sae_cuda_exact(X, W, b, k)          # first call: library and module setup
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    base = torch.cuda.memory_allocated()
    stk.topk_sae_cuda_exact(X, W, b, k)
    torch.cuda.synchronize()
    working = torch.cuda.max_memory_allocated() - base - B * k * 8
    ws = _capi.workspace_bytes(B, d, F, k, _capi.STK_BF16)
    assert ws - 4096 <= working <= ws + 4096, (working, ws)
    assert ws < 64 << 20 or B > 256


@pytest.mark.parametrize("cfg", ["32,256,3,32,1", "32,128,5,32,1", "64,256,3,16,1", "64,128,4,16,1",
                                 "128,256,2,32,0", "128,128,3,32,0", "128,128,3,32,1,1", "128,256,4,32,1,1"])
def test_tile_configurations_agree(cfg, monkeypatch):
    """Every instantiated tile configuration (128- or 256-feature tiles,
    pipeline depth, append slots in shared or global memory, top lists in
    shared or tensor memory) gives the default configuration's rows bit for bit."""
    from streamtopk_sae import native
    L = int(cfg.split(",")[0])
    k = {32: 32, 64: 64, 128: 128}[L]
    X, W, b = oracle.gaussian_inputs(200, 320, 50000, seed=L)
    Xt, Wt, bt, Xr, Wr, br = device_inputs(X, W, b, "bf16")
    V0, I0 = native.streamtopk_cuda_exact_forward(Xt, Wt, bt, k)
    monkeypatch.setenv("STK_FUSED_CFG", cfg)
    V1, I1 = native.streamtopk_cuda_exact_forward(Xt, Wt, bt, k)
    torch.cuda.synchronize()
    no_device_error()
    assert torch.equal(V0, V1) and torch.equal(I0, I1)
    check(V1, I1, Xr, Wr, br, k, RTOL["bf16"])
