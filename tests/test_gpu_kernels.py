"""GPU parity of the sm_100a kernels, called through the C-ABI kernel layer
(include/bmo_kernels.h), against the CPU oracle.

Bars: Q8_1 activation blocks and Q4_0 KV packing bit-exact; dot products and
attention within 1e-5 relative L2 (only the fp32 reduction order differs).
"""
import ctypes

import numpy as np
import pytest
from gguf import GGMLQuantizationType, quants

from bmo_jetson_b200 import engine
from oracle import oracle as orc
from tests.parity import assert_near_exact

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
DEV = torch.device("cuda:0")
PERM_ID, PERM_SWIGLU = 0, 1


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def stream():
    return torch.cuda.current_stream().cuda_stream


def to_dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def ptr(t):
    return None if t is None else t.data_ptr()


def tiled(W, rows, cols, perm=PERM_ID, F=0):
    L = engine.lib()
    n = L.bmo_k_q4_0_tiled_bytes(rows, cols, perm, F)
    assert n > 0
    src = to_dev(W.reshape(-1))
    dst = torch.empty(n, dtype=torch.uint8, device=DEV)
    assert L.bmo_k_repack_q4_0(src.data_ptr(), dst.data_ptr(), rows, cols, perm, F, stream()) == 0
    return dst


def run_gemv(T, rows, cols, x, perm=PERM_ID, F=0, gamma=None, resid=None, grid=0, eps=1e-8):
    L = engine.lib()
    xd = to_dev(x)
    gd = to_dev(gamma) if gamma is not None else None
    rd = to_dev(resid) if resid is not None else None
    y = torch.full((F if perm == PERM_SWIGLU else rows,), float("nan"), device=DEV)
    q8 = torch.zeros(cols // 32 * 36, dtype=torch.uint8, device=DEV)
    xn = torch.zeros(cols, device=DEV)
    nbytes = L.bmo_k_gemv_scratch_bytes(rows, cols, perm, F)
    scratch = torch.zeros(nbytes, dtype=torch.uint8, device=DEV)
    rc = L.bmo_k_gemv_q4_0(T.data_ptr(), rows, cols, perm, F, xd.data_ptr(), ptr(gd), eps, ptr(rd), y.data_ptr(),
                           q8.data_ptr(), xn.data_ptr(), scratch.data_ptr(), nbytes, grid, stream())
    torch.cuda.synchronize()
    assert rc == 0
    assert int(scratch.count_nonzero()) == 0 or _only_partials_used(scratch, rows, cols, perm, F)
    return y.cpu().numpy(), q8.cpu().numpy().reshape(-1, 36), xn.cpu().numpy()


def _only_partials_used(scratch, rows, cols, perm, F):
    # counters (after the partial area) must be back at zero
    n_tiles = F // 16 if perm == PERM_SWIGLU else (rows + 31) // 32
    cpt = ((cols // 32) + 7) // 8
    part = (n_tiles * (cpt + 1) * 32 * 8 + 255) // 256 * 256
    return int(scratch[part:].count_nonzero()) == 0


def weights(rows, cols, seed, sigma=0.02):
    rng = np.random.default_rng(seed)
    w = rng.normal(0, sigma, (rows, cols)).astype(np.float32)
    return np.ascontiguousarray(quants.quantize(w, GGMLQuantizationType.Q4_0))


def test_quantize_q8_1_bit_exact():
    from tests.golden.make_ref_golden import q8_input
    x = q8_input()
    out = torch.zeros(x.size // 32 * 36, dtype=torch.uint8, device=DEV)
    assert engine.lib().bmo_k_quantize_q8_1(to_dev(x).data_ptr(), out.data_ptr(), x.size, stream()) == 0
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), orc.quantize_q8_1(x).reshape(-1))


SHAPES = [(64, 4096), (4096, 4096), (12288, 4096), (4096, 11264), (32000, 4096), (1000, 4096), (3072, 1024),
          (1024, 2816), (2048, 1024), (1024, 4096), (40, 96), (33, 256)]


@pytest.mark.parametrize("rows,cols", SHAPES)
def test_gemv_plain_matches_oracle(rows, cols):
    W = weights(rows, cols, rows + cols)
    x = np.random.default_rng(cols).normal(0, 1, cols).astype(np.float32)
    y, q8, _ = run_gemv(tiled(W, rows, cols), rows, cols, x)
    np.testing.assert_array_equal(q8, orc.quantize_q8_1(x))
    assert_near_exact(y, orc.gemv_q4_0(W, x, rows, cols), what=f"gemv {rows}x{cols}")


@pytest.mark.parametrize("rows,cols", [(12288, 4096), (3072, 1024), (96, 256)])
def test_gemv_rmsnorm_prologue(rows, cols):
    W = weights(rows, cols, 7)
    rng = np.random.default_rng(8)
    x = rng.normal(0, 3, cols).astype(np.float32)
    g = (1 + 0.1 * rng.normal(0, 1, cols)).astype(np.float32)
    y, q8, xn = run_gemv(tiled(W, rows, cols), rows, cols, x, gamma=g)
    assert_near_exact(xn, orc.rmsnorm(x, g, 1e-8), what="rmsnorm")
    # the activation blocks are bit-exact given the normalised vector the kernel used
    np.testing.assert_array_equal(q8, orc.quantize_q8_1(xn))
    assert_near_exact(y, orc.gemv_q4_0(W, xn, rows, cols), what="gemv after norm")


def test_gemv_rmsnorm_unaligned_gamma_and_limits():
    """A norm weight off a 16-byte boundary is read with plain loads (the bulk
    copy needs alignment) and gives the same bits; norm widths beyond the
    kernel's staging buffer and unaligned activations are rejected."""
    L = engine.lib()
    rows, cols = 3072, 1024
    W = weights(rows, cols, 17)
    rng = np.random.default_rng(18)
    x = rng.normal(0, 2, cols).astype(np.float32)
    g = (1 + 0.1 * rng.normal(0, 1, cols)).astype(np.float32)
    T = tiled(W, rows, cols)
    y_al, _, xn_al = run_gemv(T, rows, cols, x, gamma=g)
    xd = to_dev(x)
    gbuf = torch.zeros(cols + 1, device=DEV)
    gbuf[1:] = torch.from_numpy(g).to(DEV)
    y = torch.empty(rows, device=DEV)
    xn = torch.zeros(cols, device=DEV)
    nbytes = L.bmo_k_gemv_scratch_bytes(rows, cols, PERM_ID, 0)
    scratch = torch.zeros(nbytes, dtype=torch.uint8, device=DEV)
    assert gbuf[1:].data_ptr() % 16 != 0
    rc = L.bmo_k_gemv_q4_0(T.data_ptr(), rows, cols, PERM_ID, 0, xd.data_ptr(), gbuf[1:].data_ptr(), 1e-8, None,
                           y.data_ptr(), None, xn.data_ptr(), scratch.data_ptr(), nbytes, 0, stream())
    torch.cuda.synchronize()
    assert rc == 0
    np.testing.assert_array_equal(xn.cpu().numpy(), xn_al)
    np.testing.assert_array_equal(y.cpu().numpy(), y_al)
    # unaligned activation
    xb = torch.zeros(cols + 1, device=DEV)
    rc = L.bmo_k_gemv_q4_0(T.data_ptr(), rows, cols, PERM_ID, 0, xb[1:].data_ptr(), None, 1e-8, None,
                           y.data_ptr(), None, None, scratch.data_ptr(), nbytes, 0, stream())
    assert rc != 0
    # RMSNorm prologue wider than the staging buffer
    wide = 8192
    Tw = torch.zeros(L.bmo_k_q4_0_tiled_bytes(64, wide, PERM_ID, 0), dtype=torch.uint8, device=DEV)
    xw = torch.zeros(wide, device=DEV)
    gw = torch.ones(wide, device=DEV)
    nb2 = L.bmo_k_gemv_scratch_bytes(64, wide, PERM_ID, 0)
    s2 = torch.zeros(nb2, dtype=torch.uint8, device=DEV)
    rc = L.bmo_k_gemv_q4_0(Tw.data_ptr(), 64, wide, PERM_ID, 0, xw.data_ptr(), gw.data_ptr(), 1e-8, None,
                           y.data_ptr(), None, None, s2.data_ptr(), nb2, 0, stream())
    assert rc != 0
    torch.cuda.synchronize()


def test_gemv_residual_epilogue():
    rows, cols = 4096, 4096
    W = weights(rows, cols, 9)
    rng = np.random.default_rng(10)
    x = rng.normal(0, 1, cols).astype(np.float32)
    r = rng.normal(0, 1, rows).astype(np.float32)
    y, _, _ = run_gemv(tiled(W, rows, cols), rows, cols, x, resid=r)
    assert_near_exact(y, r + orc.gemv_q4_0(W, x, rows, cols), what="residual")


@pytest.mark.parametrize("F,cols", [(11264, 4096), (2816, 1024), (704, 256)])
def test_gemv_swiglu_epilogue(F, cols):
    W = weights(2 * F, cols, F)
    rng = np.random.default_rng(F + 1)
    x = rng.normal(0, 1, cols).astype(np.float32)
    g = (1 + 0.1 * rng.normal(0, 1, cols)).astype(np.float32)
    y, _, xn = run_gemv(tiled(W, 2 * F, cols, PERM_SWIGLU, F), 2 * F, cols, x, perm=PERM_SWIGLU, F=F, gamma=g)
    h = orc.gemv_q4_0(W, xn, 2 * F, cols)
    assert_near_exact(y, orc.swiglu(h), max_ulp=4, what="swiglu")


def test_gemv_grids_and_determinism():
    rows, cols = 12288, 4096
    W = weights(rows, cols, 11)
    x = np.random.default_rng(12).normal(0, 1, cols).astype(np.float32)
    T = tiled(W, rows, cols)
    ref = orc.gemv_q4_0(W, x, rows, cols)
    for grid in (1, 7, 148, 300, 999):
        y1, _, _ = run_gemv(T, rows, cols, x, grid=grid)
        y2, _, _ = run_gemv(T, rows, cols, x, grid=grid)
        np.testing.assert_array_equal(y1, y2)
        assert_near_exact(y1, ref, what=f"grid {grid}")


def q4_planes_to_blocks(plane, scales, hd):
    """GPU Q4_0 ring planes -> ggml 18-byte blocks."""
    nb = plane.size // 16
    blocks = np.zeros((nb, 18), np.uint8)
    blocks[:, :2] = scales.reshape(nb, 2)
    blocks[:, 2:] = plane.reshape(nb, 16)
    return blocks


ATTN = [(128, 4, 512, 2, 1, p) for p in (0, 1, 5, 511, 512, 700, 1500)] + \
       [(128, 32, 512, 1, 0, 700), (64, 16, 8, 6, 2, 0), (64, 16, 8, 6, 2, 3), (64, 16, 8, 6, 5, 7),
        (128, 8, 2048, 1, 0, 3000), (64, 4, 100, 3, 2, 250)]


@pytest.mark.parametrize("kv_type", [0, 1])
@pytest.mark.parametrize("hd,nh,n_ctx,n_layers,layer,pos", ATTN)
def test_attention_matches_oracle(kv_type, hd, nh, n_ctx, n_layers, layer, pos):
    L = engine.lib()
    rng = np.random.default_rng(pos * 7 + nh)
    q, k, v = (rng.normal(0, 1, nh * hd).astype(np.float32) for _ in range(3))
    n = n_layers * nh * n_ctx * hd
    hist_k = rng.normal(0, 1, n).astype(np.float32)
    hist_v = rng.normal(0, 1, n).astype(np.float32)
    pos_d = torch.tensor([pos], dtype=torch.int32, device=DEV)
    out = torch.zeros(nh * hd, device=DEV)
    if kv_type == 0:
        kc = hist_k.astype(np.float16).view(np.uint16)
        vc = hist_v.astype(np.float16).view(np.uint16)
        kd, vd = to_dev(kc.copy()), to_dev(vc.copy())
        ksd = vsd = None
    else:
        kb = orc.quantize_q4_0(hist_k.reshape(-1, 32)).reshape(-1, 18)
        vb = orc.quantize_q4_0(hist_v.reshape(-1, 32)).reshape(-1, 18)
        kd, vd = to_dev(kb[:, 2:].copy().reshape(-1)), to_dev(vb[:, 2:].copy().reshape(-1))
        ksd, vsd = to_dev(kb[:, :2].copy().reshape(-1)), to_dev(vb[:, :2].copy().reshape(-1))
    qd, kdev, vdev = to_dev(q), to_dev(k), to_dev(v)  # keep alive until the kernels ran
    rc = L.bmo_k_decode_attention(qd.data_ptr(), kdev.data_ptr(), vdev.data_ptr(), kd.data_ptr(),
                                  vd.data_ptr(), ptr(ksd), ptr(vsd), out.data_ptr(), hd, nh, nh, n_ctx,
                                  pos_d.data_ptr(), layer, kv_type, stream())
    torch.cuda.synchronize()
    assert rc == 0
    if kv_type == 0:
        kc_o, vc_o = kc.copy(), vc.copy()
        ref = orc.attention_f16(q, k, v, kc_o, vc_o, hd, nh, nh, n_ctx, pos, layer)
        np.testing.assert_array_equal(kd.cpu().numpy(), kc_o)
        np.testing.assert_array_equal(vd.cpu().numpy(), vc_o)
    else:
        kb_o, vb_o = kb.copy().reshape(-1), vb.copy().reshape(-1)
        ref = orc.attention_q4(q, k, v, kb_o, vb_o, hd, nh, nh, n_ctx, pos, layer)
        # Q4_0 KV packing bit-exact (ggml blocks of the appended rows)
        gk = q4_planes_to_blocks(kd.cpu().numpy(), ksd.cpu().numpy(), hd)
        gv = q4_planes_to_blocks(vd.cpu().numpy(), vsd.cpu().numpy(), hd)
        np.testing.assert_array_equal(gk.reshape(-1), kb_o)
        np.testing.assert_array_equal(gv.reshape(-1), vb_o)
        slot = pos % n_ctx
        rows = [(layer * nh + hh) * n_ctx + slot for hh in range(nh)]
        blocks_k = gk.reshape(-1, hd // 32, 18)[rows].reshape(-1, 18)
        np.testing.assert_array_equal(blocks_k, quants.quantize(k.reshape(-1, 32), GGMLQuantizationType.Q4_0))
    # exact-reduction semantics: the oracle's value up to rare double-rounding ties
    assert_near_exact(out.cpu().numpy(), ref, what="attention")
