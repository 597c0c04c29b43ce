"""The restatement of the reference's depformer sampler (tests/sampler.py),
pinned on the CPU: the C++ standard's known answer for std::mt19937, the
greedy and degenerate branches of sample_token_internal
(src/bmo_api.cpp:638-666), and token for token against the same draw written
with libstdc++'s own partial_sort, discrete_distribution and mt19937
(tests/sampler_std.cpp, built with the host compiler)."""
import os

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


def sampler_cases(seed=7):
    """(n, temp, top_k, rule, logits) draws covering the sampler's branches:
    greedy (top_k <= 0, temp <= 1e-4), one weight (no draw), k above n,
    k up to 1024, underflowing weights, -1e9 masks, and the daemon's text
    rule with a pause token on top.  Values are distinct (ties are ordered
    differently by std::partial_sort and by the restatement).  top_k stays
    within the device sampler's 2048."""
    r = np.random.default_rng(seed)
    out = []
    for n, temp, k, rule in [(1, 0.7, 25, 0), (5, 0.8, 250, 0), (64, 0.8, 1, 0), (64, 0.8, 2, 0),
                             (2048, 0.8, 250, 0), (2048, 0.8, 1024, 0), (2048, 0.8, 2048, 0), (2048, 1e-5, 250, 0), (2048, 0.8, 0, 0),
                             (2048, 1.3, 4096, 0), (32000, 0.7, 25, 1), (32000, 0.7, 25, 0), (1000, 0.7, 25, 1),
                             (300, 0.5, 300, 0), (2048, 0.8, 250, 0), (2048, 0.8, 250, 0)]:
        x = ((r.permutation(n) / max(n, 1) * 2.0 - 1.0) * 8.0 + r.normal(0, 1)).astype(np.float32)
        assert np.unique(x).size == n
        out.append((n, temp, k, rule, x))
    x = np.arange(2048, dtype=np.float32) * np.float32(-0.37)   # weights underflow to 0 past a few hundred
    out.append((2048, 0.7, 1024, 0, r.permutation(x)))
    x = (r.permutation(2048).astype(np.float32) * np.float32(0.01)).astype(np.float32)
    x[2048 - 1000:] = np.float32(-1e9)
    out.append((2048, 0.8, 1024, 0, x))
    x = ((r.permutation(2048) / 2048.0 * 2.0 - 1.0) * 8.0).astype(np.float32)
    x[17] = np.float32(np.inf)                                 # an infinite logit: NaN weights, first entry kept
    out.append((2048, 0.8, 250, 0, x))
    for pause in (3, 0):                                        # text rule: a pause token keeps the argmax
        x = (r.permutation(1000).astype(np.float32) * np.float32(0.01)).astype(np.float32)
        x[pause] = np.float32(50.0)
        out.append((1000, 0.7, 25, 1, x))
    return out


def restated_draws(cases, seed):
    g = sampler.MT19937(seed)
    toks = []
    for n, temp, k, rule, x in cases:
        toks.append(sampler.daemon_text(x, True, temp, k, g) if rule else sampler.sample(x, temp, k, g))
    return toks


def test_restatement_matches_libstdcxx(tmp_path):
    import shutil
    import subprocess
    cxx = shutil.which("g++")
    if cxx is None:
        import pytest
        pytest.skip("no host C++ compiler")
    src = os.path.join(os.path.dirname(os.path.abspath(__file__)), "sampler_std.cpp")
    exe = str(tmp_path / "sampler_std")
    subprocess.run([cxx, "-O2", "-std=c++17", src, "-o", exe], check=True)
    cases = sampler_cases()
    lines = [f"1337 {len(cases)}"]
    for n, temp, k, rule, x in cases:
        lines.append(f"{n} {float(np.float32(temp)).hex()} {k} {rule}")
        lines.append(" ".join(float(v).hex() for v in x))
    res = subprocess.run([exe], input="\n".join(lines) + "\n", capture_output=True, text=True, check=True)
    std = [int(t) for t in res.stdout.split()]
    assert std == restated_draws(cases, 1337)
