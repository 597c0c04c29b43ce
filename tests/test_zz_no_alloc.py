"""The allocation-free GEMV entry point (bmo_k_gemv_q4_0_static).

Callers that cannot allocate device memory when they run a kernel -- a
real-time audio callback that must not block in cudaMalloc, a framework that
owns every allocation, a process under a device-memory cap -- use this entry
point; its split-K scratch is a fixed buffer inside libbmo.  Here it is
called through the C ABI and compared with the allocating entry point
(bmo_k_gemv_q4_0, caller scratch) on the same inputs, twice in a row so that
state the shared buffer keeps from one call cannot leak into the next.  The
file is named to be collected last.
"""
import numpy as np
import pytest
from gguf import GGMLQuantizationType, quants

from bmo_jetson_b200 import engine

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

SCRATCH_TOO_SMALL = -2


def _tiled(L, W, rows, cols, perm, F, dev, stream):
    src = torch.from_numpy(W.reshape(-1)).to(dev)
    dst = torch.empty(L.bmo_k_q4_0_tiled_bytes(rows, cols, perm, F), dtype=torch.uint8, device=dev)
    assert L.bmo_k_repack_q4_0(src.data_ptr(), dst.data_ptr(), rows, cols, perm, F, stream) == 0
    torch.cuda.synchronize(dev)
    return dst


@pytest.mark.parametrize("rows,cols,perm,F,norm,resid", [
    (22528, 4096, 1, 11264, True, False),   # FFN-in: fused RMSNorm + SwiGLU
    (4096, 11264, 0, 0, False, True),        # FFN-out: residual epilogue, split tiles
    (3072, 1024, 0, 0, True, False),         # depformer QKV shape
])
def test_static_scratch_gemv_matches_allocating_entry_point(rows, cols, perm, F, norm, resid):
    L = engine.lib()
    dev = torch.device("cuda:0")
    stream = torch.cuda.current_stream(dev).cuda_stream
    rng = np.random.default_rng(rows + cols)
    W = np.ascontiguousarray(quants.quantize(rng.normal(0, 0.02, (rows, cols)).astype(np.float32),
                                             GGMLQuantizationType.Q4_0))
    T = _tiled(L, W, rows, cols, perm, F, dev, stream)
    n_out = F if perm == 1 else rows
    gamma = torch.from_numpy((1 + 0.1 * rng.normal(0, 1, cols)).astype(np.float32)).to(dev) if norm else None
    r = torch.from_numpy(rng.normal(0, 1, rows).astype(np.float32)).to(dev) if resid else None
    nbytes = L.bmo_k_gemv_scratch_bytes(rows, cols, perm, F)
    scratch = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    for call in range(2):
        x = torch.from_numpy(rng.normal(0, 1 + call, cols).astype(np.float32)).to(dev)
        y_ref = torch.full((n_out,), float("nan"), device=dev)
        y_static = torch.full((n_out,), float("nan"), device=dev)
        rc = L.bmo_k_gemv_q4_0(T.data_ptr(), rows, cols, perm, F, x.data_ptr(),
                               gamma.data_ptr() if norm else None, 1e-8, r.data_ptr() if resid else None,
                               y_ref.data_ptr(), None, None, scratch.data_ptr(), nbytes, 0, stream)
        assert rc == 0
        rc = L.bmo_k_gemv_q4_0_static(T.data_ptr(), rows, cols, perm, F, x.data_ptr(),
                                      gamma.data_ptr() if norm else None, 1e-8, r.data_ptr() if resid else None,
                                      y_static.data_ptr(), None, None, 0, stream)
        assert rc == 0
        torch.cuda.synchronize(dev)
        got, want = y_static.cpu().numpy(), y_ref.cpu().numpy()
        assert not np.isnan(got).any()
        # the same kernel, grid and summation order: bit-identical results
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32), err_msg=f"call {call}")


def test_static_scratch_rejects_oversized_matrix():
    L = engine.lib()
    dev = torch.device("cuda:0")
    x = torch.zeros(4096, device=dev)
    y = torch.zeros(32000, device=dev)
    t = torch.zeros(16, dtype=torch.uint8, device=dev)
    # the 32000-row text head needs more than the 4 MiB fixed buffer
    assert L.bmo_k_gemv_scratch_bytes(32000, 4096, 0, 0) > (4 << 20)
    rc = L.bmo_k_gemv_q4_0_static(t.data_ptr(), 32000, 4096, 0, 0, x.data_ptr(), None, 1e-8, None, y.data_ptr(),
                                  None, None, 0, torch.cuda.current_stream(dev).cuda_stream)
    assert rc == SCRATCH_TOO_SMALL
