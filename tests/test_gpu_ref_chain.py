"""End-to-end parity with the REFERENCE's own decode step.

The reference (utkarshyadav009/bmo_jetson) decodes with its own CUDA kernels
chained eagerly in src/bmo_compute.cpp order; oracle/ref_chain.py runs that
chain with those kernels compiled unmodified.  The engine, in its default
reference-order semantics, must reproduce it BIT FOR BIT: the normed hidden
state z, the text logits, every depformer step's audio logits, the greedy
text and audio tokens, and the K/V ring after the frames -- on small models,
on one full-width temporal block at a wrapped position (config 1), and on
the full 32-layer model with its depformer (configs 2 + 3).  Where the
reference kernels are not built, the same cases are checked against the
chain's outputs kept in tests/golden/ref_chain.npz.
"""
import os

import numpy as np
import pytest

from bmo_jetson_b200 import engine
from tests.golden import make_ref_chain_golden as G

pytestmark = pytest.mark.gpu


def _live() -> bool:
    from oracle import ref_chain
    return ref_chain.available() and os.environ.get("BMO_REF_CHAIN_FIXTURES", "0") != "1"


def _fixture(prefix):
    if not os.path.exists(G.OUT):
        pytest.skip("reference kernels not built and no reference-chain fixtures")
    g = np.load(G.OUT)
    return {k[len(prefix) + 1:]: g[k] for k in g.files if k.startswith(prefix + "_")}


def _same(ours, ref, what):
    ours = np.asarray(ours, np.float32)
    ref = np.asarray(ref, np.float32)
    assert ours.shape == ref.shape, what
    bad = np.flatnonzero(ours.view(np.uint32) != ref.view(np.uint32))
    if bad.size:
        rel = float(np.linalg.norm(ours.astype(np.float64) - ref) / max(np.linalg.norm(ref), 1e-30))
        raise AssertionError(f"{what}: {bad.size}/{ref.size} values differ (first {bad[:5].tolist()}), rel L2 {rel:.3e}")


def _same_or_digest(ours, exp, key, what):
    if key in exp:
        _same(ours, exp[key], what)
    else:
        assert G.digest(np.asarray(ours, np.float32)) == str(exp[key + "_digest"]), what
        top = exp[key + "_top"]
        flat = np.asarray(ours, np.float32).reshape(-1)
        np.testing.assert_array_equal(flat[top[0].astype(np.int64)], top[1], err_msg=what)


def _engine_ring_digest(e):
    ks = [e.kv_raw(0, 0, l) for l in range(e.n_layers)]
    vs = [e.kv_raw(1, 0, l) for l in range(e.n_layers)]
    return G.digest(np.concatenate(ks), np.concatenate(vs))


@pytest.mark.parametrize("name", ["tiny", "tiny17", "config2"])
def test_frames_bit_identical_to_reference_chain(name, model_dir):
    preset, n_ctx, pos0, n_frames, hseed, tseed = G.FRAME_CASES[name]
    exp = G.run_chain_frames(name, model_dir) if _live() else _fixture(name)
    path = G.model_path(preset, model_dir)
    e = engine.BMOEngine(path, n_ctx=n_ctx, device=0, kv_type=engine.KV_F16, flags=engine.FLAG_REF_ORDER)
    try:
        assert e.ref_order
        for layer, (k, v) in enumerate(G.history(e.n_layers, n_ctx, e.n_kv_heads * e.head_dim, hseed)):
            e.kv_import(layer, 0, k, v)
        toks = exp["tokens"]
        assert toks.shape == (n_frames, e.n_codebooks)
        e.pos = pos0
        for f in range(n_frames):
            z, lg = e.forward_temporal(toks[f], copy=True)
            _same(z, exp[f"z{f}"], f"{name} frame {f} z")
            _same_or_digest(lg, exp, f"logits{f}", f"{name} frame {f} text logits")
            text = int(np.argmax(lg))
            assert text == int(exp[f"text{f}"])
            audio = e.forward_depth_cascade(text, z, temp=0.0, top_k=0)
            np.testing.assert_array_equal(audio, exp[f"audio{f}"], err_msg=f"{name} frame {f} audio tokens")
            # the greedy cascade's own logits (one cluster launch where the model allows it)
            _same_or_digest(e.debug_tap("dlogits").reshape(e.dep_q, -1), exp, f"dlogits{f}",
                            f"{name} frame {f} cascade logits")
            prev, dl = text, []
            for cb in range(e.dep_q):
                dl.append(e.forward_depth(cb, prev, z, copy=True))
                prev = int(audio[cb])
            _same_or_digest(np.stack(dl), exp, f"dlogits{f}", f"{name} frame {f} depformer logits")
        assert _engine_ring_digest(e) == str(exp["ring_digest"]), f"{name}: K/V ring after the frames"
    finally:
        del e


def test_block_bit_identical_to_reference_chain(model_dir):
    """Config 1: one 4096-wide temporal block (32 heads x 128, FFN 11264) at
    position 700 of a 512-slot ring that has wrapped."""
    preset, n_ctx, pos, hseed, xseed = G.BLOCK_CASE
    exp = G.run_chain_block(model_dir) if _live() else _fixture("block")
    e = engine.BMOEngine(G.model_path(preset, model_dir), n_ctx=n_ctx, device=0, kv_type=engine.KV_F16,
                         flags=engine.FLAG_REF_ORDER)
    (k, v), = G.history(1, n_ctx, e.n_kv_heads * e.head_dim, hseed)
    e.kv_import(0, 0, k, v)
    x = np.random.default_rng(xseed).standard_normal(e.n_embd, dtype=np.float32)
    _same(x, exp["x"], "block input")
    y = e.forward_layers(x, pos, 0, 1)
    _same(y, exp["y"], "block output")
    slot = pos % n_ctx
    kr = e.kv_raw(0, 0, 0).view(np.float16).reshape(e.n_kv_heads, n_ctx, e.head_dim)[:, slot]
    vr = e.kv_raw(1, 0, 0).view(np.float16).reshape(e.n_kv_heads, n_ctx, e.head_dim)[:, slot]
    np.testing.assert_array_equal(kr.view(np.uint16), exp["kslot"].view(np.uint16))
    np.testing.assert_array_equal(vr.view(np.uint16), exp["vslot"].view(np.uint16))
