"""Full-size parity: the BASELINE config-2/3 model (32-layer d4096 temporal
transformer, 32000 text head, 8-step depformer) on a 512-slot ring of seeded
history, decoding frames at positions 700.. (wrapped ring), through the
reference C ABI and the fused frame graph, against the CPU oracle -- once
with one kernel per op and once through the persistent frame kernel."""
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


@pytest.mark.parametrize("kv_type,persistent", [(0, False), (1, False), (0, True)])
def test_full_model_frames_match_oracle(model, kv_type, persistent):
    flags = engine.FLAG_PERSISTENT if persistent else 0
    e = engine.BMOEngine(model, n_ctx=N_CTX, kv_type=kv_type, flags=flags)
    assert e.persistent == persistent
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
