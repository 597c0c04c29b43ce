"""The reference's own caller sequence against this library: the flow of
utkarshyadav009/bmo_jetson test_cabi_roundtrip.py (its geometry invariants,
an eager warm-up frame with the 8-step depformer chained by argmax, reset,
CUDA-graph capture with has_cuda_graphs, then frames of random 17-channel
tokens with no NaN anywhere), driven through bmo_jetson_b200.engine.BMOEngine,
whose methods and arguments are those of the reference's bmo_engine.py, on a
17-channel synthetic model."""
import numpy as np
import pytest

from bmo_jetson_b200 import engine

pytestmark = pytest.mark.gpu


def test_cabi_roundtrip_flow(tiny17_model):
    e = engine.BMOEngine(tiny17_model, n_ctx=1024)
    # the reference caller's invariants (its model: 17 channels, dep_q 8, 2048-way audio heads)
    assert e.n_codebooks == 17 and e.dep_q == 8 and e.audio_vocab == 2048
    assert e.text_vocab > 0 and e.n_embd > 0 and e.n_attn_heads * e.head_dim == e.n_embd

    warm = np.zeros(17, dtype=np.int32)
    warm[0] = 3
    z, text_logits = e.forward_temporal(warm)
    assert z.shape == (e.n_embd,) and text_logits.shape == (e.text_vocab,)
    assert not np.isnan(z).any() and not np.isnan(text_logits).any()
    prev = int(np.argmax(text_logits))
    for s in range(e.dep_q):
        a = e.forward_depth(s, prev, z)
        assert a.shape == (2048,) and not np.isnan(a).any()
        prev = int(np.argmax(a))
    e.reset()

    assert e.capture_graphs() == 0
    assert e.has_cuda_graphs()
    e.reset()
    rng = np.random.RandomState(42)
    for _ in range(20):
        tokens = np.concatenate([[rng.randint(0, e.text_vocab)], rng.randint(0, e.audio_vocab, size=16)]).astype(np.int32)
        z, text_logits = e.forward_temporal(tokens)
        assert not np.isnan(z).any() and not np.isnan(text_logits).any()
        prev = int(np.argmax(text_logits))
        for s in range(e.dep_q):
            a = e.forward_depth(s, prev, z)
            assert not np.isnan(a).any()
            prev = int(np.argmax(a))
    assert e.pos == 20
    e.close()
