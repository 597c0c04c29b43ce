"""Kernel-level parity of the reference-order kernels (bmo_k_gemv_q4_0_ref,
bmo_k_decode_attention_ref, through the C-ABI kernel layer) with the
REFERENCE's own CUDA kernels: bit for bit, against the golden outputs those
kernels produced on a B200 (tests/golden/ref_kernels.npz) and, where the
reference kernels are built (oracle/_ref), against them live on random inputs
with the fused RMSNorm, SwiGLU and residual forms."""
import numpy as np
import pytest

from bmo_jetson_b200 import engine
from oracle import oracle as orc
from tests.golden import make_ref_golden as RG

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
DEV = torch.device("cuda:0")
PERM_ID, PERM_SWIGLU = 0, 1
GOLDEN = RG.os.path.join(RG.HERE, "ref_kernels.npz")


def stream():
    return torch.cuda.current_stream().cuda_stream


def to_dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def ptr(t):
    return None if t is None else t.data_ptr()


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def tiled(W, rows, cols, perm=PERM_ID, F=0):
    L = engine.lib()
    n = L.bmo_k_q4_0_tiled_bytes(rows, cols, perm, F)
    src = to_dev(np.ascontiguousarray(W, np.uint8).reshape(-1))
    dst = torch.empty(n, dtype=torch.uint8, device=DEV)
    assert L.bmo_k_repack_q4_0(src.data_ptr(), dst.data_ptr(), rows, cols, perm, F, stream()) == 0
    return dst


def gemv_ref(W, rows, cols, x, perm=PERM_ID, F=0, gamma=None, resid=None):
    L = engine.lib()
    T = tiled(W, rows, cols, perm, F)
    xd, gd, rd = to_dev(x), (to_dev(gamma) if gamma is not None else None), (to_dev(resid) if resid is not None else None)
    y = torch.full((F if perm == PERM_SWIGLU else rows,), float("nan"), device=DEV)
    q8 = torch.zeros(cols // 32 * 36, dtype=torch.uint8, device=DEV)
    xn = torch.zeros(cols, device=DEV)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    rc = L.bmo_k_gemv_q4_0_ref(T.data_ptr(), rows, cols, perm, F, xd.data_ptr(), ptr(gd), 1e-8, ptr(rd), y.data_ptr(),
                               q8.data_ptr(), xn.data_ptr(), st.data_ptr(), stream())
    torch.cuda.synchronize()
    assert rc == 0 and int(st.item()) == 0
    return y.cpu().numpy(), q8.cpu().numpy(), xn.cpu().numpy()


def attention_ref(q, k, v, kc, vc, hd, nh, nkv, n_ctx, pos, layer):
    L = engine.lib()
    kcd, vcd = to_dev(kc.view(np.float16)), to_dev(vc.view(np.float16))
    out = torch.full((nh * hd,), float("nan"), device=DEV)
    posd = torch.tensor([pos], dtype=torch.int32, device=DEV)
    qd, kd, vd = to_dev(q), to_dev(k), to_dev(v)  # held until the kernels are done
    rc = L.bmo_k_decode_attention_ref(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), kcd.data_ptr(), vcd.data_ptr(),
                                      out.data_ptr(), hd, nh, nkv, n_ctx, posd.data_ptr(), layer, stream())
    torch.cuda.synchronize()
    assert rc == 0
    return out.cpu().numpy(), kcd.cpu().numpy().view(np.uint16), vcd.cpu().numpy().view(np.uint16)


# ---- against the reference kernels' golden outputs --------------------------

def test_gemv_ref_bit_exact_vs_golden():
    g = np.load(GOLDEN)
    for i, (r, c) in enumerate(RG.GEMV_SHAPES):
        W, x = RG.gemv_inputs(r, c, 200 + i)
        y, q8, _ = gemv_ref(W, r, c, x)
        np.testing.assert_array_equal(q8, g[f"gemv{i}_q8"], err_msg=f"Q8_1 blocks {r}x{c}")
        np.testing.assert_array_equal(bits(y), bits(g[f"gemv{i}_y"]), err_msg=f"GEMV {r}x{c}")


def test_rmsnorm_prologue_bit_exact_vs_golden():
    """The fused RMSNorm (normalised vector the GEMV quantised) equals rmsnorm_kernel's output."""
    g = np.load(GOLDEN)
    for i, n in enumerate((4096, 1024)):
        rng = np.random.default_rng(300 + i)
        x = rng.normal(0, 1, n).astype(np.float32)
        w = (1 + 0.1 * rng.normal(0, 1, n)).astype(np.float32)
        W = orc.quantize_q4_0(np.random.default_rng(9).normal(0, 0.02, (32, n)).astype(np.float32))
        _, q8, xn = gemv_ref(W, 32, n, x, gamma=w)
        np.testing.assert_array_equal(bits(xn), bits(g[f"rms{i}_y"]), err_msg=f"rmsnorm n={n}")
        np.testing.assert_array_equal(q8.reshape(-1, 36), orc.quantize_q8_1(g[f"rms{i}_y"]))


def test_attention_ref_bit_exact_vs_golden():
    g = np.load(GOLDEN)
    for i, (hd, nh, n_ctx, n_layers, layer, pos) in enumerate(RG.ATTN_CASES):
        q, k, v, kc, vc = RG.attn_inputs(hd, nh, n_ctx, n_layers, 600 + i)
        out, kc2, vc2 = attention_ref(q, k, v, kc, vc, hd, nh, nh, n_ctx, pos, layer)
        np.testing.assert_array_equal(bits(out), bits(g[f"attn{i}_out"]), err_msg=f"case {i} pos {pos}")
        slot = pos % n_ctx
        base = layer * nh * n_ctx * hd
        idx = np.array([base + (hh * n_ctx + slot) * hd + d for hh in range(nh) for d in range(hd)])
        np.testing.assert_array_equal(kc2[idx], g[f"attn{i}_kslot"])
        np.testing.assert_array_equal(vc2[idx], g[f"attn{i}_vslot"])


# ---- against the reference kernels, live ------------------------------------

def _ref():
    from oracle import ref_chain
    if not ref_chain.available():
        pytest.skip("reference kernels not built (make -C oracle ref)")
    return orc.ref_lib()


@pytest.mark.parametrize("rows,cols", [(96, 4096), (64, 11264), (96, 1024), (32, 2816), (48, 704), (32, 256)])
def test_gemv_ref_live(rows, cols):
    R = _ref()
    rng = np.random.default_rng(rows * 7 + cols)
    W = orc.quantize_q4_0(rng.normal(0, 0.02, (rows, cols)).astype(np.float32))
    x = (rng.normal(0, 1, cols) * rng.choice([1e-3, 1.0, 40.0])).astype(np.float32)
    want = np.zeros(rows, np.float32)
    assert R.ref_gemv_q4_0_q8_1(W.reshape(-1), x, want, np.zeros(cols // 32 * 36, np.uint8), rows, cols) == 0
    y, _, _ = gemv_ref(W, rows, cols, x)
    np.testing.assert_array_equal(bits(y), bits(want))


@pytest.mark.parametrize("cols,F", [(4096, 64), (1024, 48), (256, 16)])
def test_gemv_ref_norm_swiglu_residual_live(cols, F):
    """rmsnorm -> GEMV -> swiglu_split, and GEMV -> residual_add, of the
    reference's kernels equal the fused forms."""
    R = _ref()
    rng = np.random.default_rng(cols + F)
    x = rng.normal(0, 3, cols).astype(np.float32)
    gam = (1 + 0.1 * rng.normal(0, 1, cols)).astype(np.float32)
    W = orc.quantize_q4_0(rng.normal(0, 0.02, (2 * F, cols)).astype(np.float32))
    xn = np.zeros(cols, np.float32)
    assert R.ref_rmsnorm(x, gam, 1e-8, cols, xn) == 0
    h = np.zeros(2 * F, np.float32)
    assert R.ref_gemv_q4_0_q8_1(W.reshape(-1), xn, h, np.zeros(cols // 32 * 36, np.uint8), 2 * F, cols) == 0
    want = np.zeros(F, np.float32)
    assert R.ref_swiglu(h, F, want) == 0
    y, _, _ = gemv_ref(W, 2 * F, cols, x, PERM_SWIGLU, F, gamma=gam)
    np.testing.assert_array_equal(bits(y), bits(want))
    # residual: y = resid + W x
    Wr = orc.quantize_q4_0(rng.normal(0, 0.02, (64, cols)).astype(np.float32))
    resid = rng.normal(0, 1, 64).astype(np.float32)
    yr = np.zeros(64, np.float32)
    assert R.ref_gemv_q4_0_q8_1(Wr.reshape(-1), x, yr, np.zeros(cols // 32 * 36, np.uint8), 64, cols) == 0
    want_r = (resid + yr).astype(np.float32)
    y2, _, _ = gemv_ref(Wr, 64, cols, x, resid=resid)
    np.testing.assert_array_equal(bits(y2), bits(want_r))


@pytest.mark.parametrize("hd,nh,nkv,n_ctx", [(128, 4, 4, 512), (128, 8, 8, 1024), (64, 16, 16, 8), (64, 4, 4, 100)])
def test_attention_ref_live(hd, nh, nkv, n_ctx):
    R = _ref()
    rng = np.random.default_rng(hd + nh + n_ctx)
    for pos in sorted({0, 1, 2, 7, n_ctx - 1, n_ctx, n_ctx + 1, 3 * n_ctx // 2 + 3, 2999}):
        q = (rng.normal(0, 1, nh * hd) * 3).astype(np.float32)
        k = rng.normal(0, 1, nkv * hd).astype(np.float32)
        v = rng.normal(0, 1, nkv * hd).astype(np.float32)
        nl, layer = 2, 1
        kc = rng.normal(0, 1, nl * nkv * n_ctx * hd).astype(np.float16).view(np.uint16)
        vc = rng.normal(0, 1, nl * nkv * n_ctx * hd).astype(np.float16).view(np.uint16)
        # the reference kernel sizes its ring by n_heads: give it full-size caches
        kf = np.zeros(nl * nh * n_ctx * hd, np.uint16)
        vf = np.zeros_like(kf)
        kf.reshape(nl, nh, n_ctx, hd)[:, :nkv] = kc.reshape(nl, nkv, n_ctx, hd)
        vf.reshape(nl, nh, n_ctx, hd)[:, :nkv] = vc.reshape(nl, nkv, n_ctx, hd)
        want = np.zeros(nh * hd, np.float32)
        assert R.ref_attention(q, k, v, kf, vf, want, hd, nh, nkv, n_ctx, pos, layer, nl) == 0
        out, kc2, vc2 = attention_ref(q, k, v, kc, vc, hd, nh, nkv, n_ctx, pos, layer)
        np.testing.assert_array_equal(bits(out), bits(want), err_msg=f"pos {pos}")
        np.testing.assert_array_equal(kc2.reshape(nl, nkv, n_ctx, hd), kf.reshape(nl, nh, n_ctx, hd)[:, :nkv])
        np.testing.assert_array_equal(vc2.reshape(nl, nkv, n_ctx, hd), vf.reshape(nl, nh, n_ctx, hd)[:, :nkv])
