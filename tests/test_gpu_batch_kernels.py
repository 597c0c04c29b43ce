"""GPU parity of the batched GEMM (bmo_k_batch_gemm_q4_0): every session's
output row against the CPU oracle's single-session GEMV on the same Q4_0
weights and input.

Bars: the CUDA-core path (tensor_cores=0) and the exact tensor-core path
(1) keep the batch-1 GEMV's rounding (near exact: 1-2 ULP, see
tests/parity.py); the fast tensor-core path (2) sums full-block terms in
fp32 and agrees to fp32 rounding (relative L2 below 1e-6).
"""
import numpy as np
import pytest

from bmo_jetson_b200 import engine
from oracle import oracle as orc
from tests.parity import assert_near_exact, rel_l2
from tests.test_gpu_kernels import DEV, PERM_ID, PERM_SWIGLU, ptr, stream, tiled, to_dev, torch, weights

pytestmark = pytest.mark.gpu

TC_TOL = 1e-6


def run_batch(T, rows, cols, X, perm=PERM_ID, F=0, gamma=None, resid=None, tensor_cores=1, eps=1e-8):
    L = engine.lib()
    n = X.shape[0]
    xd = to_dev(X)
    gd = to_dev(gamma) if gamma is not None else None
    rd = to_dev(resid) if resid is not None else None
    out_w = F if perm == PERM_SWIGLU else rows
    y = torch.full((n, out_w), float("nan"), device=DEV)
    nbytes = L.bmo_k_batch_gemm_scratch_bytes(rows, cols, perm, F, n)
    assert nbytes > 0
    scratch = torch.zeros(nbytes, dtype=torch.uint8, device=DEV)
    rc = L.bmo_k_batch_gemm_q4_0(T.data_ptr(), rows, cols, perm, F, xd.data_ptr(), ptr(gd), eps, ptr(rd),
                                 y.data_ptr(), n, tensor_cores, scratch.data_ptr(), nbytes, stream())
    torch.cuda.synchronize()
    assert rc == 0
    return y.cpu().numpy(), scratch


SHAPES = [(4096, 4096), (12288, 4096), (4096, 11264), (1024, 2816), (3072, 1024), (2048, 1024), (1024, 4096),
          (96, 256), (40, 96), (1000, 4096)]


@pytest.mark.parametrize("tensor_cores", [1, 0, 2])
@pytest.mark.parametrize("n_sess", [1, 7, 33, 64])
@pytest.mark.parametrize("rows,cols", SHAPES)
def test_batch_gemm_matches_oracle_per_session(rows, cols, n_sess, tensor_cores):
    if tensor_cores != 1 and n_sess in (7, 33) and rows * cols > 4096 * 4096:
        pytest.skip("CUDA-core and fast paths: large shapes covered at 1 and 64 sessions")
    W = weights(rows, cols, rows * 3 + cols)
    X = np.random.default_rng(n_sess + rows).normal(0, 1, (n_sess, cols)).astype(np.float32)
    y, _ = run_batch(tiled(W, rows, cols), rows, cols, X, tensor_cores=tensor_cores)
    for s in range(n_sess):
        want = orc.gemv_q4_0(W, X[s], rows, cols)
        if tensor_cores == 2:
            assert rel_l2(y[s], want) < TC_TOL, (s, rel_l2(y[s], want))
        else:
            assert_near_exact(y[s], want, what=f"session {s}")


@pytest.mark.parametrize("tensor_cores", [1, 0, 2])
def test_batch_gemm_fused_epilogues(tensor_cores):
    rng = np.random.default_rng(5)
    n = 64
    # RMSNorm prologue + residual epilogue
    rows, cols = 4096, 4096
    W = weights(rows, cols, 21)
    X = rng.normal(0, 2, (n, cols)).astype(np.float32)
    g = (1 + 0.1 * rng.normal(0, 1, cols)).astype(np.float32)
    R = rng.normal(0, 1, (n, rows)).astype(np.float32)
    y, _ = run_batch(tiled(W, rows, cols), rows, cols, X, gamma=g, resid=R, tensor_cores=tensor_cores)
    for s in (0, 31, 32, 63):
        want = R[s] + orc.gemv_q4_0(W, orc.rmsnorm(X[s], g, 1e-8), rows, cols)
        assert rel_l2(y[s], want) < (TC_TOL if tensor_cores == 2 else 1e-6), s
    # SwiGLU epilogue
    F, cols = 2816, 1024
    W = weights(2 * F, cols, 22)
    X = rng.normal(0, 1, (n, cols)).astype(np.float32)
    y, _ = run_batch(tiled(W, 2 * F, cols, PERM_SWIGLU, F), 2 * F, cols, X, perm=PERM_SWIGLU, F=F,
                     tensor_cores=tensor_cores)
    for s in (0, 17, 63):
        want = orc.swiglu(orc.gemv_q4_0(W, X[s], 2 * F, cols))
        assert rel_l2(y[s], want) < (2 * TC_TOL if tensor_cores == 2 else 1e-6), s


def test_batch_gemm_deterministic_and_scratch_reusable():
    rows, cols, n = 12288, 4096, 64
    W = weights(rows, cols, 31)
    T = tiled(W, rows, cols)
    X = np.random.default_rng(32).normal(0, 1, (n, cols)).astype(np.float32)
    y1, sc = run_batch(T, rows, cols, X)
    y2, _ = run_batch(T, rows, cols, X)
    np.testing.assert_array_equal(y1, y2)
    # the split-combine counters are back at zero after the call
    L = engine.lib()
    assert sc.numel() == L.bmo_k_batch_gemm_scratch_bytes(rows, cols, PERM_ID, 0, n)
    # a row's result does not depend on the other rows of the batch
    y1s, _ = run_batch(T, rows, cols, X[5:6])
    np.testing.assert_array_equal(y1s[0], y1[5])
