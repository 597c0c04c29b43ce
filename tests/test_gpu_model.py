"""Full-size parity: the config-2/3 model (32-layer d4096 temporal
transformer, 32000 text head, 8-step depformer) on a 512-slot ring of seeded
history, decoding frames at positions 700.. (wrapped ring), through the
reference C ABI and the fused frame graph, in the exact-reduction order
(FLAG_EXACT) against the CPU oracle, with fp16 and Q4_0 rings.  The default
reference order is checked bit for bit against the reference's own kernels
on the same model in test_gpu_ref_chain.py."""
import numpy as np
import pytest

from bmo_jetson_b200 import engine, synth
from oracle import oracle as orc
from tests.parity import rel_l2

pytestmark = pytest.mark.gpu

N_CTX = 512


def fill(e, o, seed):
    rng = np.random.default_rng(seed)
    width = e.n_kv_heads * e.head_dim
    for layer in range(e.n_layers):
        k = rng.standard_normal((N_CTX, width), dtype=np.float32)
        v = rng.standard_normal((N_CTX, width), dtype=np.float32)
        e.kv_import(layer, 0, k, v)
        o.kv_import(layer, 0, k, v)


@pytest.fixture(scope="module")
def model(model_dir):
    return synth.ensure_model("config2", model_dir)


@pytest.mark.parametrize("kv_type", [0, 1])
def test_full_model_frames_match_oracle(model, kv_type):
    e = engine.BMOEngine(model, n_ctx=N_CTX, kv_type=kv_type, flags=engine.FLAG_EXACT)
    assert not e.ref_order
    o = orc.OracleModel(model, n_ctx=N_CTX, kv_type=kv_type)
    assert (e.n_layers, e.n_embd, e.text_vocab, e.audio_vocab, e.dep_q) == (32, 4096, 32000, 2048, 8)
    fill(e, o, 11 + kv_type)
    rng = np.random.default_rng(5)
    for step in range(3):
        pos = 700 + step
        t = np.concatenate([[rng.integers(0, 32000)], rng.integers(0, 2048, e.n_codebooks - 1)]).astype(np.int32)
        e.pos = pos
        z, logits = e.forward_temporal(t, copy=True)
        zo, lo, _ = o.forward_temporal(t, pos)
        assert rel_l2(z, zo) < 1e-5, (step, rel_l2(z, zo))
        assert rel_l2(logits, lo) < 1e-5, (step, rel_l2(logits, lo))
        text = int(np.argmax(logits))
        assert text == int(np.argmax(lo))
        audio = e.forward_depth_cascade(text, z, 0.0, 0)
        np.testing.assert_array_equal(audio, o.depth_cascade_greedy(text, zo))
    # the fused one-graph frame gives the same tokens as the ABI calls
    t = np.concatenate([[7], np.arange(1, e.n_codebooks)]).astype(np.int32)
    e.pos = 703
    z, logits, text, audio = e.forward_frame_greedy(t)
    zo, lo, _ = o.forward_temporal(t, 703)
    assert rel_l2(z, zo) < 1e-5 and text == int(np.argmax(lo))
    np.testing.assert_array_equal(audio, o.depth_cascade_greedy(text, zo))
    e.close()
    o.close()
