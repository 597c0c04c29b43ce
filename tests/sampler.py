"""An independent restatement of the reference's depformer token sampler
(utkarshyadav009/bmo_jetson src/bmo_api.cpp:638-666, sample_token_internal,
called by bmo_forward_depth_cascade :668-743 with a per-thread
``std::mt19937 rng(42)`` that lives as long as the thread; the daemon's
sample_token_cpp, src/bmo_daemon.cpp:147-175, is the same arithmetic), for
checking the library's samplers token for token.  TEST INFRASTRUCTURE.

Greedy (first maximum) when top_k <= 0 or temp <= 1e-4.  Otherwise the top_k
logits in descending order, probs_i = expf(l_i / temp - l_0 / temp) in
float, and one draw of ``std::discrete_distribution<int>`` over them:
the probabilities widened to double, divided by their sequential double sum,
their running sums as the cumulative table with its last entry set to 1;
u = ``std::generate_canonical<double, 53>`` = (g1 + g2 * 2^32) / 2^64 from
two 32-bit engine outputs (the C++ standard's [rand.util.canonical]); the
token is the first index whose cumulative value is >= u.
"""
from __future__ import annotations

import ctypes
import ctypes.util

import numpy as np

_libm = ctypes.CDLL(ctypes.util.find_library("m") or "libm.so.6")
_libm.expf.argtypes = [ctypes.c_float]
_libm.expf.restype = ctypes.c_float


class MT19937:
    """The 32-bit Mersenne Twister of the C++ standard (std::mt19937)."""

    def __init__(self, seed: int = 5489):
        self.mt = [0] * 624
        self.mt[0] = seed & 0xFFFFFFFF
        for i in range(1, 624):
            self.mt[i] = (1812433253 * (self.mt[i - 1] ^ (self.mt[i - 1] >> 30)) + i) & 0xFFFFFFFF
        self.idx = 624

    def _twist(self):
        mt = self.mt
        for i in range(624):
            y = (mt[i] & 0x80000000) | (mt[(i + 1) % 624] & 0x7FFFFFFF)
            mt[i] = mt[(i + 397) % 624] ^ (y >> 1) ^ (0x9908B0DF if y & 1 else 0)
        self.idx = 0

    def __call__(self) -> int:
        if self.idx >= 624:
            self._twist()
        y = self.mt[self.idx]
        self.idx += 1
        y ^= y >> 11
        y ^= (y << 7) & 0x9D2C5680
        y ^= (y << 15) & 0xEFC60000
        y ^= y >> 18
        return y & 0xFFFFFFFF


def generate_canonical(rng: MT19937) -> float:
    s = float(rng()) + float(rng()) * 4294967296.0
    u = s / 18446744073709551616.0
    return u if u < 1.0 else float(np.nextafter(1.0, 0.0))


def sample(logits: np.ndarray, temp: float, top_k: int, rng: MT19937) -> int:
    logits = np.asarray(logits, np.float32)
    if top_k <= 0 or temp <= 1e-4:
        return int(np.argmax(logits))
    order = np.argsort(-logits, kind="stable")
    k = min(top_k, logits.size)
    top = order[:k]
    t = np.float32(temp)
    max_l = np.float32(logits[top[0]] / t)
    probs = [_libm.expf(float(np.float32(np.float32(logits[i] / t) - max_l))) for i in top]
    sum_p = np.float32(0.0)
    for p in probs:
        sum_p = np.float32(sum_p + np.float32(p))
    if sum_p <= 0.0 or np.isnan(sum_p):
        return int(top[0])
    if k < 2:  # libstdc++'s discrete_distribution keeps no table for one weight and draws nothing
        return int(top[0])
    total = 0.0
    for p in probs:
        total += float(p)
    cum, run = [], 0.0
    for p in probs:
        run += float(p) / total
        cum.append(run)
    cum[-1] = 1.0
    u = generate_canonical(rng)
    return int(top[int(np.searchsorted(np.array(cum), u, side="left"))])


def daemon_text(logits: np.ndarray, sampling: bool, temp: float, top_k: int, rng: MT19937) -> int:
    """The daemon's text token (bmo_daemon.cpp:755-762): the first argmax,
    kept when it is a pause token (3 or 0) or sampling is off, else one
    draw of the sampler."""
    top1 = int(np.argmax(np.asarray(logits, np.float32)))
    if top1 in (3, 0) or not sampling:
        return top1
    return sample(logits, temp, top_k, rng)
