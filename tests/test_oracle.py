"""CPU checks of the oracle: the checker itself must be pinned before it is trusted.

Pins:
  * Q4_0 quantiser bit-exact against gguf-py's quants.Q4_0 (the upstream numpy
    restatement of ggml's quantize_row_q4_0_ref);
  * Q8_1 quantiser bit-exact against an independent numpy statement of the
    reference rule (bmo_cuda_kernels.cu:529-558) and against the reference
    kernel's own output (tests/golden/ref_kernels.npz, made on a B200);
  * GEMV, RMSNorm, RoPE, SwiGLU and ring attention against the reference
    kernels' golden outputs.
"""
import os

import numpy as np
import pytest
from gguf import GGMLQuantizationType, quants

from oracle import oracle as orc

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "ref_kernels.npz")


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def np_q8_1(x: np.ndarray) -> np.ndarray:
    """Numpy statement of the reference Q8_1 rule (independent of the C oracle)."""
    x = x.astype(np.float32).reshape(-1, 32)
    amax = np.abs(x).max(axis=1)
    d = (amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        idv = np.where(d != 0, np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
    v = (x * idv[:, None]).astype(np.float32)
    t = np.trunc(v)
    frac = np.abs(v - t)
    q = t + np.sign(v) * (frac >= 0.5)  # roundf: halves away from zero
    q = np.clip(q, -128, 127).astype(np.int8)
    s = np.zeros(x.shape[0], np.float32)
    for j in range(32):  # sequential fp32 sum, as the kernel
        s = (s + x[:, j]).astype(np.float32)
    out = np.zeros((x.shape[0], 36), np.uint8)
    out[:, 0:2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:4] = s.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 4:] = q.view(np.uint8)
    return out


def q8_edge_input():
    from tests.golden.make_ref_golden import q8_input
    return q8_input()


def test_fp16_round_trip_matches_numpy():
    L = orc.lib()
    rng = np.random.default_rng(0)
    vals = np.concatenate([
        rng.normal(0, 1, 2000), rng.normal(0, 1e-5, 500), rng.normal(0, 3e4, 500),
        [0.0, -0.0, 65504.0, 65519.0, 65520.0, 1e9, -1e9, 2.0 ** -25, 2.0 ** -24, 3 * 2.0 ** -26, 6.1e-5,
         np.inf, -np.inf],
    ]).astype(np.float32)
    ours = np.array([L.orc_fp32_to_fp16(float(v)) for v in vals], np.uint16)
    np.testing.assert_array_equal(ours, vals.astype(np.float16).view(np.uint16))
    halves = np.arange(0, 65536, 7, dtype=np.uint32).astype(np.uint16)
    halves = halves[(halves & 0x7C00) != 0x7C00]  # finite
    back = np.array([L.orc_fp16_to_fp32(int(h)) for h in halves], np.float32)
    np.testing.assert_array_equal(back, halves.view(np.float16).astype(np.float32))


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_q4_0_bit_exact_vs_gguf(seed):
    rng = np.random.default_rng(seed)
    x = rng.normal(0, 0.02, (64, 256)).astype(np.float32)
    x[0, :32] = 0.0                                  # all-zero block
    x[1, :32] = 1.0                                  # ties on |max|
    x[2, :32] = -np.linspace(0, 1, 32)               # negative max
    x[3, 5] = 1e30                                   # huge outlier
    x[4, :32] = rng.normal(0, 1e-8, 32)              # tiny scale (subnormal fp16 d)
    ref = quants.quantize(x, GGMLQuantizationType.Q4_0)
    np.testing.assert_array_equal(orc.quantize_q4_0(x), ref)


def test_q4_0_dequant_matches_gguf():
    rng = np.random.default_rng(5)
    x = rng.normal(0, 0.02, (8, 128)).astype(np.float32)
    blocks = quants.quantize(x, GGMLQuantizationType.Q4_0)
    ref = quants.dequantize(blocks, GGMLQuantizationType.Q4_0).reshape(-1)
    np.testing.assert_array_equal(orc.dequantize_q4_0(blocks, x.size), ref)


def test_q8_1_matches_numpy_statement():
    x = q8_edge_input()
    np.testing.assert_array_equal(orc.quantize_q8_1(x), np_q8_1(x))


def test_q8_1_known_answers():
    # amax 127 -> d = 1, id = 1: halves round away from zero (roundf)
    x = np.zeros(32, np.float32)
    x[:6] = [127.0, 2.5, -2.5, 0.5, -0.5, 1.49999994]
    b = orc.quantize_q8_1(x)[0]
    q = b[4:].view(np.int8)
    assert list(q[:6]) == [127, 3, -3, 1, -1, 1]
    assert b[0:2].view(np.float16)[0] == np.float16(1.0)
    # all-zero block: d = 0, id = 0, q = 0, sum = 0
    z = orc.quantize_q8_1(np.zeros(32, np.float32))[0]
    assert not z.any()


def test_gemv_oracle_matches_float_reference():
    """The integer dot equals sum(dequant(W) * dequant(x)) up to the s8 term."""
    rng = np.random.default_rng(7)
    rows, cols = 48, 512
    w = rng.normal(0, 0.02, (rows, cols)).astype(np.float32)
    W = quants.quantize(w, GGMLQuantizationType.Q4_0)
    x = rng.normal(0, 1, cols).astype(np.float32)
    y = orc.gemv_q4_0(W, x, rows, cols)
    # reconstruct: W deq * (q8 * d8), with the -8*s8 term using half(sum x) per block
    q8 = orc.quantize_q8_1(x)
    d8 = q8[:, 0:2].copy().view(np.float16).astype(np.float64).ravel()
    s8 = q8[:, 2:4].copy().view(np.float16).astype(np.float64).ravel()
    qv = q8[:, 4:].view(np.int8).astype(np.float64)
    blocks = W.reshape(rows, cols // 32, 18)
    d4 = blocks[:, :, 0:2].copy().view(np.float16).astype(np.float64)[..., 0]
    lo = (blocks[:, :, 2:] & 0x0F).astype(np.float64)
    hi = (blocks[:, :, 2:] >> 4).astype(np.float64)
    nib = np.concatenate([lo, hi], axis=2)  # [rows, nb, 32]
    sumi = (nib * qv[None]).sum(axis=2)
    expect = (d4 * (sumi * d8[None] - 8 * s8[None])).sum(axis=1)
    assert rel_l2(y, expect) < 1e-6


def test_rmsnorm_rope_swiglu_against_numpy():
    rng = np.random.default_rng(9)
    x = rng.normal(0, 1, 256).astype(np.float32)
    w = (1 + 0.1 * rng.normal(0, 1, 256)).astype(np.float32)
    y = orc.rmsnorm(x, w, 1e-8)
    ref = x.astype(np.float64) / np.sqrt(np.mean(x.astype(np.float64) ** 2) + 1e-8) * w
    assert rel_l2(y, ref) < 1e-6
    r = orc.rope(x, 2, 128, 700)
    xr = x.reshape(2, 64, 2).astype(np.float64)
    i = np.arange(64)
    ang = np.float32(700) * (np.float32(10000.0) ** (-(2 * i).astype(np.float32) / np.float32(128)))
    c, s = np.cos(ang.astype(np.float64)), np.sin(ang.astype(np.float64))
    ref = np.stack([xr[..., 0] * c - xr[..., 1] * s, xr[..., 0] * s + xr[..., 1] * c], -1).reshape(-1)
    assert rel_l2(r, ref) < 1e-5
    h = rng.normal(0, 1, 512).astype(np.float32)
    g, u = h[:256].astype(np.float64), h[256:].astype(np.float64)
    assert rel_l2(orc.swiglu(h), g / (1 + np.exp(-g)) * u) < 1e-6


def test_attention_oracle_matches_dense_softmax():
    rng = np.random.default_rng(11)
    hd, nh, n_ctx, layers = 64, 4, 16, 2
    kc = rng.normal(0, 1, layers * nh * n_ctx * hd).astype(np.float16).view(np.uint16)
    vc = rng.normal(0, 1, layers * nh * n_ctx * hd).astype(np.float16).view(np.uint16)
    q, k, v = (rng.normal(0, 1, nh * hd).astype(np.float32) for _ in range(3))
    pos, layer = 20, 1  # wrapped: window 16 = positions 5..20
    out = orc.attention_f16(q, k, v, kc.copy(), vc.copy(), hd, nh, nh, n_ctx, pos, layer)
    K = kc.view(np.float16).astype(np.float64).reshape(layers, nh, n_ctx, hd)[layer].copy()
    V = vc.view(np.float16).astype(np.float64).reshape(layers, nh, n_ctx, hd)[layer].copy()
    K[:, pos % n_ctx] = k.reshape(nh, hd).astype(np.float16)
    V[:, pos % n_ctx] = v.reshape(nh, hd).astype(np.float16)
    slots = [(t % n_ctx) for t in range(pos - n_ctx + 1, pos + 1)]
    qh = q.reshape(nh, hd).astype(np.float64)
    sc = np.einsum("hd,hsd->hs", qh, K[:, slots]) / np.sqrt(hd)
    p = np.exp(sc - sc.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    ref = np.einsum("hs,hsd->hd", p, V[:, slots]).reshape(-1)
    assert rel_l2(out, ref) < 1e-6
    # window of one returns v itself
    out0 = orc.attention_f16(q, k, v, kc.copy(), vc.copy(), hd, nh, nh, n_ctx, 0, 0)
    np.testing.assert_array_equal(out0, v)


# ---- golden vectors from the reference's own kernels on a B200 -------------

golden = pytest.mark.skipif(not os.path.exists(GOLDEN), reason="reference golden vectors not generated yet")


@golden
def test_golden_q8_1_bit_exact():
    g = np.load(GOLDEN)
    from tests.golden.make_ref_golden import digest
    x = q8_edge_input()
    assert str(g["q8_x_digest"]) == digest(x)
    np.testing.assert_array_equal(orc.quantize_q8_1(x).reshape(-1), g["q8_blocks"])


@golden
def test_golden_gemv():
    g = np.load(GOLDEN)
    from tests.golden.make_ref_golden import GEMV_SHAPES, digest, gemv_inputs
    for i, (r, c) in enumerate(GEMV_SHAPES):
        W, x = gemv_inputs(r, c, 200 + i)
        assert str(g[f"gemv{i}_digest"]) == digest(W, x)
        np.testing.assert_array_equal(orc.quantize_q8_1(x).reshape(-1), g[f"gemv{i}_q8"])
        assert rel_l2(orc.gemv_q4_0(W, x, r, c), g[f"gemv{i}_y"]) < 1e-5


@golden
def test_golden_elementwise():
    g = np.load(GOLDEN)
    from tests.golden.make_ref_golden import ROPE_CASES
    for i, n in enumerate((4096, 1024)):
        rng = np.random.default_rng(300 + i)
        x = rng.normal(0, 1, n).astype(np.float32)
        w = (1 + 0.1 * rng.normal(0, 1, n)).astype(np.float32)
        assert rel_l2(orc.rmsnorm(x, w, 1e-8), g[f"rms{i}_y"]) < 1e-6
    for i, (nh, hd, pos) in enumerate(ROPE_CASES):
        rng = np.random.default_rng(400 + i)
        x = rng.normal(0, 1, nh * hd).astype(np.float32)
        # the reference uses __powf/__sincosf; the oracle evaluates the trig accurately
        assert rel_l2(orc.rope(x, nh, hd, pos), g[f"rope{i}_y"]) < 1e-3
    rng = np.random.default_rng(500)
    h = rng.normal(0, 1, 2 * 11264).astype(np.float32)
    assert rel_l2(orc.swiglu(h), g["swiglu_y"]) < 1e-5


@golden
def test_golden_attention():
    g = np.load(GOLDEN)
    from tests.golden.make_ref_golden import ATTN_CASES, attn_inputs
    for i, (hd, nh, n_ctx, n_layers, layer, pos) in enumerate(ATTN_CASES):
        q, k, v, kc, vc = attn_inputs(hd, nh, n_ctx, n_layers, 600 + i)
        out = orc.attention_f16(q, k, v, kc, vc, hd, nh, nh, n_ctx, pos, layer)
        assert rel_l2(out, g[f"attn{i}_out"]) < 1e-5, (i, pos)
        slot = pos % n_ctx
        base = layer * nh * n_ctx * hd
        idx = np.array([base + (hh * n_ctx + slot) * hd + d for hh in range(nh) for d in range(hd)])
        np.testing.assert_array_equal(kc[idx], g[f"attn{i}_kslot"])
        np.testing.assert_array_equal(vc[idx], g[f"attn{i}_vslot"])


# ---- the reference kernels' own fp32 order ---------------------------------

def ulps(a, b):
    """Distance in units in the last place between two float32 arrays."""
    ia = np.asarray(a, np.float32).view(np.int32).astype(np.int64)
    ib = np.asarray(b, np.float32).view(np.int32).astype(np.int64)
    ia = np.where(ia < 0, -(ia & 0x7FFFFFFF), ia)
    ib = np.where(ib < 0, -(ib & 0x7FFFFFFF), ib)
    return np.abs(ia - ib)


@golden
def test_golden_gemv_reforder_bit_exact():
    """The reference-order restatement reproduces the reference GEMV kernel's
    output bit for bit on all five shapes (main-loop only, tail only, both,
    and a padded 2816-column case)."""
    g = np.load(GOLDEN)
    from tests.golden.make_ref_golden import GEMV_SHAPES, gemv_inputs
    for i, (r, c) in enumerate(GEMV_SHAPES):
        W, _ = gemv_inputs(r, c, 200 + i)
        y = orc.gemv_q4_0_reforder(W, g[f"gemv{i}_q8"], r, c)
        np.testing.assert_array_equal(y.view(np.uint32), g[f"gemv{i}_y"].view(np.uint32), err_msg=f"shape {r}x{c}")


@golden
def test_golden_rmsnorm_reforder():
    """Reference order up to rsqrtf: within 4 ulp of the kernel's output."""
    g = np.load(GOLDEN)
    for i, n in enumerate((4096, 1024)):
        rng = np.random.default_rng(300 + i)
        x = rng.normal(0, 1, n).astype(np.float32)
        w = (1 + 0.1 * rng.normal(0, 1, n)).astype(np.float32)
        assert int(ulps(orc.rmsnorm_reforder(x, w, 1e-8), g[f"rms{i}_y"]).max()) <= 4


@golden
def test_golden_attention_reforder():
    """Reference order up to CUDA's expf: within 1e-6 relative L2 of the
    kernel's output, appended fp16 slots bit-exact."""
    g = np.load(GOLDEN)
    from tests.golden.make_ref_golden import ATTN_CASES, attn_inputs
    for i, (hd, nh, n_ctx, n_layers, layer, pos) in enumerate(ATTN_CASES):
        q, k, v, kc, vc = attn_inputs(hd, nh, n_ctx, n_layers, 600 + i)
        out = orc.attention_f16_reforder(q, k, v, kc, vc, hd, nh, nh, n_ctx, pos, layer)
        assert rel_l2(out, g[f"attn{i}_out"]) < 1e-6, (i, pos)
        if pos == 0:
            np.testing.assert_array_equal(out, g[f"attn{i}_out"])
