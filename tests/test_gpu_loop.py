"""The caller's frame loop on the device (kernels/loop.cu, bmo_loop_reset /
bmo_loop_run) against the daemon's own loop restated on the host
(utkarshyadav009/bmo_jetson src/bmo_daemon.cpp:641-816): the 17-channel
interleave with its one-frame delay, bmo_forward_temporal at position =
frame, the text token (first argmax; a pause token 3 or 0 or greedy mode keeps
it, else sample_token_cpp), eight bmo_forward_depth steps each followed by its
audio draw from the same std::mt19937, the codec input [last frame's cb0,
cb1..7] and the delay-line update.  The restatement drives the library's
per-step entry points, whose logits are the same kernels' outputs, and draws
with tests/sampler.py (pinned to libstdc++ in test_sampler.py), so the
device loop must reproduce every token.  The device sampler alone
(bmo_k_sample_token) is checked draw for draw first, generator state
included."""
import numpy as np
import pytest

from bmo_jetson_b200 import engine, synth
from tests import sampler
from tests.daemon import daemon_restated, fresh_state
from tests.test_sampler import restated_draws, sampler_cases

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _rng_words(g):
    return np.array(list(g.mt) + [g.idx], dtype=np.uint32)


def _device_draws(cases, seed):
    L = engine.lib()
    dev = torch.device("cuda:0")
    rng = torch.from_numpy(_rng_words(sampler.MT19937(seed)).view(np.int32).copy()).to(dev)
    out = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    toks = []
    for n, temp, k, rule, x in cases:
        xd = torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(dev)
        rc = L.bmo_k_sample_token(xd.data_ptr(), n, float(temp), k, rule, rng.data_ptr(), out.data_ptr(), stream)
        assert rc == 0
        toks.append(int(out.item()))
    return toks, rng.cpu().numpy().view(np.uint32)


def _tie_cases(seed=11):
    """Logits with many equal values across the top-k boundary: both sides
    take equal logits in index order."""
    r = np.random.default_rng(seed)
    out = []
    for n, k in [(2048, 250), (2048, 1024), (2048, 2048), (32000, 25), (32000, 2048), (777, 777)]:
        x = (np.round(r.normal(0, 2, n) * 2) / 2).astype(np.float32)
        out.append((n, 0.8, k, 0, x))
    # more equal logits than the text sampler's candidate buffer holds: the full radix path
    x = np.zeros(32000, np.float32)
    x[r.choice(32000, 10, replace=False)] = r.normal(1, 0.5, 10).astype(np.float32) + 1
    out.append((32000, 0.7, 25, 0, x))
    out.append((32000, 0.7, 25, 0, np.full(32000, 0.25, np.float32)))
    out.append((2048, 0.8, 250, 0, np.full(2048, -3.0, np.float32)))
    out.append((32000, 0.7, 1024, 0, (np.round(r.normal(0, 2, 32000) * 4) / 4).astype(np.float32)))
    return out


def test_device_sampler_matches_restatement():
    cases = sampler_cases() + _tie_cases()
    toks, words = _device_draws(cases, 1337)
    g = sampler.MT19937(1337)
    exp = []
    for n, temp, k, rule, x in cases:
        exp.append(sampler.daemon_text(x, True, temp, k, g) if rule else sampler.sample(x, temp, k, g))
    assert toks == exp
    assert toks[:len(sampler_cases())] == restated_draws(sampler_cases(), 1337)
    np.testing.assert_array_equal(words, _rng_words(g), err_msg="generator state after the draws")


def test_device_sampler_generator_wraps():
    """Enough draws to run the generator through several state refreshes
    (624 words, two per draw)."""
    r = np.random.default_rng(5)
    x = ((r.permutation(2048) / 2048.0 * 2.0 - 1.0) * 6.0).astype(np.float32)
    cases = [(2048, 0.8, 250, 0, x)] * 700
    toks, words = _device_draws(cases, 99)
    g = sampler.MT19937(99)
    assert toks == [sampler.sample(x, 0.8, 250, g) for _ in range(700)]
    np.testing.assert_array_equal(words, _rng_words(g))


CASES = {"tiny": 256, "tiny17": 256, "config2": 512}


@pytest.mark.parametrize("name", ["tiny", "tiny17", "config2"])
@pytest.mark.parametrize("sampling", [False, True])
def test_loop_matches_daemon(name, sampling, model_dir):
    e = engine.BMOEngine(synth.ensure_model(name, model_dir), n_ctx=CASES[name], device=0, kv_type=engine.KV_F16)
    try:
        assert e.loop_frame == -1
        r = np.random.default_rng(3)
        calls = [(3, None), (4, r.integers(0, 2048, (4, 8)))] if name == "config2" else \
            [(5, None), (30, r.integers(0, 2048, (30, 8))), (40, None), (3, r.integers(0, 2048, (3, 8)))]
        params = (0.7, 25, 0.8, 250)
        st = fresh_state(e)
        rng = sampler.MT19937(1337)
        exp = [daemon_restated(e, st, n, u, sampling, *params, rng) for n, u in calls]
        e.loop_reset(1337)
        assert e.loop_frame == 0
        got = []
        for n, u in calls:
            got.append(e.loop_run(n, u, sampling, *params))
        assert e.loop_frame == sum(n for n, _ in calls)
        for c, (a, b) in enumerate(zip(got, exp)):
            np.testing.assert_array_equal(a, b, err_msg=f"{name} call {c} (sampling={sampling})")
        if name == "config2":  # 32000 text logits: a text top-k above the sampler's 2048 is refused
            out = np.zeros((1, 17), np.int32)
            assert engine.lib().bmo_loop_run(e._h, 1, None, 1, 0.7, 2049, 0.8, 250,
                                             out.ctypes.data_as(engine._c_i32p)) == 2
    finally:
        del e


def test_loop_top_k_2048_and_restart(model_dir):
    """The largest top-k the device sampler takes (every audio logit), then a restart with
    another seed: the second conversation repeats the restated one."""
    e = engine.BMOEngine(synth.ensure_model("tiny", model_dir), n_ctx=256, device=0, kv_type=engine.KV_F16)
    try:
        for seed in (7, 8):
            exp = daemon_restated(e, fresh_state(e), 6, None, True, 1.1, 2048, 1.2, 2048, sampler.MT19937(seed))
            e.loop_reset(seed)
            got = e.loop_run(6, None, True, 1.1, 2048, 1.2, 2048)
            np.testing.assert_array_equal(got, exp, err_msg=f"seed {seed}")
    finally:
        del e


def test_loop_argument_errors(model_dir):
    e = engine.BMOEngine(synth.ensure_model("tiny", model_dir), n_ctx=256, device=0, kv_type=engine.KV_F16)
    L = engine.lib()
    try:
        out = np.zeros((2, 17), np.int32)
        op = out.ctypes.data_as(engine._c_i32p)
        assert L.bmo_loop_run(e._h, 1, None, 0, 0.7, 25, 0.8, 250, op) == 4      # not reset
        e.loop_reset(1337)
        assert L.bmo_loop_run(e._h, 0, None, 0, 0.7, 25, 0.8, 250, op) == 2      # no frames
        assert L.bmo_loop_run(e._h, 65, None, 0, 0.7, 25, 0.8, 250, op) == 2     # above the ring
        assert L.bmo_loop_run(e._h, 1, None, 1, 0.7, 5000, 0.8, 5000, op) == 0   # k = min(top_k, 1000 | 2048)
        assert L.bmo_loop_run(e._h, 1, None, 0, 0.7, 25, 0.8, 250, None) == 1
        assert e.loop_frame == 1
        assert L.bmo_loop_run(e._h, 2, None, 0, 0.7, 25, 0.8, 250, op) == 0
        assert e.loop_frame == 3
    finally:
        del e
