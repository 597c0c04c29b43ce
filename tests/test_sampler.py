"""The restatement of the reference's depformer sampler (tests/sampler.py),
pinned on the CPU: the C++ standard's known answer for std::mt19937, and the
greedy and degenerate branches of sample_token_internal
(src/bmo_api.cpp:638-666)."""
import numpy as np

from tests import sampler


def test_mt19937_standard_known_answer():
    # [rand.predef]: the 10000th output of a default-constructed mt19937 is 4123659995
    g = sampler.MT19937()
    for _ in range(9999):
        g()
    assert g() == 4123659995


def test_generate_canonical_in_unit_interval():
    g = sampler.MT19937(42)
    us = [sampler.generate_canonical(g) for _ in range(1000)]
    assert min(us) >= 0.0 and max(us) < 1.0


def test_greedy_branches_take_the_first_maximum():
    x = np.array([0.5, 2.0, 2.0, -1.0], np.float32)
    g = sampler.MT19937(42)
    assert sampler.sample(x, 0.8, 0, g) == 1      # top_k <= 0
    assert sampler.sample(x, 1e-5, 50, g) == 1    # temp <= 1e-4
    assert g() == sampler.MT19937(42)()           # greedy draws nothing


def test_top1_always_takes_the_maximum():
    x = np.random.default_rng(3).normal(0, 1, 2048).astype(np.float32)
    g = sampler.MT19937(42)
    assert all(sampler.sample(x, 0.8, 1, g) == int(np.argmax(x)) for _ in range(5))
