"""The greedy depformer cascade as one launch -- on a thread-block cluster
(kernels/dep_cascade.cu, BMO_FLAG_DEP_CLUSTER) or as a cooperative launch
over every SM (kernels/dep_cascade_ll.cu, BMO_DEP_GRID=1) -- against the same
cascade run one kernel per op: all compute the reference kernels' fp32
operations in the reference's order, so the tokens and every step's audio
logits must be identical bit for bit -- through bmo_forward_depth_cascade (host z and
text token), through the whole-frame graph (text token from the device text
head), and with the per-step entry point afterwards (bmo_forward_depth keeps
using the depformer K/V ring the cascade wrote)."""
import os

import numpy as np
import pytest

from bmo_jetson_b200 import engine, synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model_dir(tmp_path_factory):
    return str(tmp_path_factory.mktemp("models"))


def _pair(path, n_ctx, mode):
    """(engine running the cascade in `mode`, engine running it per op)."""
    os.environ["BMO_DEP_GRID"] = "1" if mode == 2 else "0"
    try:
        a = engine.BMOEngine(path, n_ctx=n_ctx, device=0, kv_type=engine.KV_F16,
                             flags=engine.FLAG_DEP_CLUSTER if mode == 1 else 0)
        os.environ["BMO_DEP_GRID"] = "0"
        b = engine.BMOEngine(path, n_ctx=n_ctx, device=0, kv_type=engine.KV_F16)
    finally:
        os.environ.pop("BMO_DEP_GRID", None)
    return a, b


def _bits(x):
    return np.ascontiguousarray(x, np.float32).view(np.uint32)


@pytest.mark.parametrize("mode", [1, 2])
@pytest.mark.parametrize("preset", ["tiny", "tiny17", "config2"])
def test_one_launch_cascade_equals_per_op_cascade(preset, mode, model_dir):
    path = synth.ensure_model(preset, model_dir)
    a, b = _pair(path, 64, mode)
    try:
        assert a.ref_order and b.ref_order
        assert a.dep_mode == mode, "the cascade kernel should run this depformer"
        assert b.dep_mode == 0
        rng = np.random.default_rng(5)
        for trial in range(3):
            z = rng.standard_normal(a.n_embd).astype(np.float32) * (1.0 + trial)
            text = int(rng.integers(0, a.text_vocab))
            ta = a.forward_depth_cascade(text, z, temp=0.0, top_k=0)
            tb = b.forward_depth_cascade(text, z, temp=0.0, top_k=0)
            np.testing.assert_array_equal(ta, tb, err_msg=f"{preset} trial {trial} tokens")
            la, lb = a.debug_tap("dlogits"), b.debug_tap("dlogits")
            assert la.size == a.dep_q * a.audio_vocab
            np.testing.assert_array_equal(_bits(la), _bits(lb), err_msg=f"{preset} trial {trial} logits")
        # a single step after a cascade reads the depformer ring the cascade left
        z = rng.standard_normal(a.n_embd).astype(np.float32)
        text = int(rng.integers(0, a.text_vocab))
        ta = a.forward_depth_cascade(text, z, temp=0.0, top_k=0)
        tb = b.forward_depth_cascade(text, z, temp=0.0, top_k=0)
        np.testing.assert_array_equal(ta, tb)
        cb = a.dep_q - 1
        da = a.forward_depth(cb, int(ta[cb - 1]), z, copy=True)
        db = b.forward_depth(cb, int(tb[cb - 1]), z, copy=True)
        np.testing.assert_array_equal(_bits(da), _bits(db), err_msg=f"{preset} step {cb} after a cascade")
    finally:
        del a, b


@pytest.mark.parametrize("mode", [1, 2])
@pytest.mark.parametrize("preset", ["tiny", "config2"])
def test_one_launch_cascade_in_the_frame_graph(preset, mode, model_dir):
    path = synth.ensure_model(preset, model_dir)
    a, b = _pair(path, 64, mode)
    try:
        rng = np.random.default_rng(9)
        w = a.n_kv_heads * a.head_dim
        for layer in range(a.n_layers):
            k = rng.standard_normal((40, w), dtype=np.float32)
            v = rng.standard_normal((40, w), dtype=np.float32)
            a.kv_import(layer, 0, k, v)
            b.kv_import(layer, 0, k, v)
        a.pos = b.pos = 40
        for f in range(3):
            toks = np.concatenate([[rng.integers(0, a.text_vocab)],
                                   rng.integers(0, a.audio_vocab, a.n_codebooks - 1)]).astype(np.int32)
            za, _, text_a, audio_a = a.forward_frame_greedy(toks)
            zb, _, text_b, audio_b = b.forward_frame_greedy(toks)
            np.testing.assert_array_equal(_bits(za), _bits(zb), err_msg=f"{preset} frame {f} z")
            assert text_a == text_b, f"{preset} frame {f} text token"
            np.testing.assert_array_equal(audio_a, audio_b, err_msg=f"{preset} frame {f} audio tokens")
            np.testing.assert_array_equal(_bits(a.debug_tap("dlogits")), _bits(b.debug_tap("dlogits")),
                                          err_msg=f"{preset} frame {f} logits")
    finally:
        del a, b
