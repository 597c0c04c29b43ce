"""Generates golden vectors from the REFERENCE's own CUDA kernels on a B200.

utkarshyadav009/bmo_jetson has no fixtures or known-answer tests for the
decode step, so its kernels themselves (src/bmo_cuda_kernels.cu, compiled
unmodified for sm_100a into oracle/_ref/libbmo_refkernels.so by
``make -C oracle ref``) are run on seeded inputs and their outputs are kept
here.  Inputs are regenerated from the seeds in `cases()` (numpy PCG64 and
gguf-py's Q4_0 quantiser), with a digest stored to catch drift.

    python tests/golden/make_ref_golden.py OUT.npz      # on a GPU box
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

GEMV_SHAPES = [(64, 4096), (32, 11264), (96, 1024), (32, 2816), (40, 4096)]
ROPE_CASES = [(32, 128, 0), (32, 128, 1), (32, 128, 5), (32, 128, 700), (32, 128, 2999), (16, 64, 3)]
ATTN_CASES = [  # head_dim, n_heads, n_ctx, n_layers, layer, pos
    (128, 4, 512, 2, 1, 0), (128, 4, 512, 2, 1, 1), (128, 4, 512, 2, 1, 5), (128, 4, 512, 2, 1, 511),
    (128, 4, 512, 2, 1, 512), (128, 4, 512, 2, 1, 700), (64, 16, 8, 6, 2, 0), (64, 16, 8, 6, 2, 3),
    (64, 16, 8, 6, 2, 7),
]


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()[:16]


def q8_input() -> np.ndarray:
    """4096 N(0,1) values followed by edge-case blocks for the Q8_1 rounding rule."""
    rng = np.random.default_rng(101)
    x = rng.normal(0, 1, 4096).astype(np.float32)
    zero = np.zeros(32, np.float32)
    halves = np.array([127.0, 2.5, -2.5, 0.5, -0.5, 1.5, -1.5, 126.5, -126.5] + [0.25] * 23, np.float32)
    tiny = np.full(32, 1e-30, np.float32) * rng.normal(0, 1, 32).astype(np.float32)
    big = (rng.normal(0, 1, 32) * 6e4).astype(np.float32)
    negz = np.array([-0.0] * 31 + [3.0], np.float32)
    one_hot = np.zeros(32, np.float32)
    one_hot[17] = -7.0
    return np.concatenate([x, zero, halves, tiny, big, negz, one_hot])


def gemv_inputs(rows: int, cols: int, seed: int):
    from gguf import GGMLQuantizationType, quants
    rng = np.random.default_rng(seed)
    w = rng.normal(0, 0.02, (rows, cols)).astype(np.float32)
    W = quants.quantize(w, GGMLQuantizationType.Q4_0)
    x = rng.normal(0, 1, cols).astype(np.float32)
    return np.ascontiguousarray(W), x


def attn_inputs(hd, nh, n_ctx, n_layers, seed):
    rng = np.random.default_rng(seed)
    q = rng.normal(0, 1, nh * hd).astype(np.float32)
    k = rng.normal(0, 1, nh * hd).astype(np.float32)
    v = rng.normal(0, 1, nh * hd).astype(np.float32)
    kc = rng.normal(0, 1, n_layers * nh * n_ctx * hd).astype(np.float16).view(np.uint16)
    vc = rng.normal(0, 1, n_layers * nh * n_ctx * hd).astype(np.float16).view(np.uint16)
    return q, k, v, kc, vc


def main(out_path: str) -> None:
    from oracle import oracle as orc
    R = orc.ref_lib()
    res = {}
    # Q8_1 through the reference launcher (its q8 scratch is the quantised x)
    x = q8_input()
    W = np.zeros((1, x.size // 32 * 18), np.uint8)
    y = np.zeros(1, np.float32)
    q8 = np.zeros(x.size // 32 * 36, np.uint8)
    assert R.ref_gemv_q4_0_q8_1(W.reshape(-1), x, y, q8, 1, x.size) == 0
    res["q8_x_digest"] = np.array(digest(x))
    res["q8_blocks"] = q8
    for i, (r, c) in enumerate(GEMV_SHAPES):
        W, xv = gemv_inputs(r, c, 200 + i)
        y = np.zeros(r, np.float32)
        q8 = np.zeros(c // 32 * 36, np.uint8)
        assert R.ref_gemv_q4_0_q8_1(W.reshape(-1), xv, y, q8, r, c) == 0
        res[f"gemv{i}_digest"] = np.array(digest(W, xv))
        res[f"gemv{i}_y"] = y
        res[f"gemv{i}_q8"] = q8
    for i, n in enumerate((4096, 1024)):
        rng = np.random.default_rng(300 + i)
        xv = rng.normal(0, 1, n).astype(np.float32)
        wv = (1 + 0.1 * rng.normal(0, 1, n)).astype(np.float32)
        y = np.zeros(n, np.float32)
        assert R.ref_rmsnorm(xv, wv, 1e-8, n, y) == 0
        res[f"rms{i}_y"] = y
    for i, (nh, hd, pos) in enumerate(ROPE_CASES):
        rng = np.random.default_rng(400 + i)
        xv = rng.normal(0, 1, nh * hd).astype(np.float32)
        y = np.zeros_like(xv)
        assert R.ref_rope(xv, nh, hd, pos, 10000.0, y) == 0
        res[f"rope{i}_y"] = y
    rng = np.random.default_rng(500)
    h = rng.normal(0, 1, 2 * 11264).astype(np.float32)
    y = np.zeros(11264, np.float32)
    assert R.ref_swiglu(h, 11264, y) == 0
    res["swiglu_y"] = y
    for i, (hd, nh, n_ctx, n_layers, layer, pos) in enumerate(ATTN_CASES):
        q, k, v, kc, vc = attn_inputs(hd, nh, n_ctx, n_layers, 600 + i)
        out = np.zeros(nh * hd, np.float32)
        assert R.ref_attention(q, k, v, kc, vc, out, hd, nh, nh, n_ctx, pos, layer, n_layers) == 0
        res[f"attn{i}_out"] = out
        slot = pos % n_ctx
        base = layer * nh * n_ctx * hd
        idx = np.array([base + (hh * n_ctx + slot) * hd + d for hh in range(nh) for d in range(hd)])
        res[f"attn{i}_kslot"] = kc[idx]
        res[f"attn{i}_vslot"] = vc[idx]
    np.savez_compressed(out_path, **res)
    print(f"wrote {out_path} ({len(res)} arrays)")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.join(HERE, "ref_kernels.npz"))
