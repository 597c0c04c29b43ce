"""The tensor-parallel peer-memory exchange kernel (bmo_k_tp_exchange) on one
GPU: the ranks' partial buffers and arrival words are local buffers that the
test fills as the peers would, so the protocol and the arithmetic are checked
without a second GPU; and the bounded wait is made to run out (a word that
nothing sets) to check the error status and that the kernel leaves its
output alone.
"""
import ctypes
import time

import numpy as np
import pytest

from bmo_jetson_b200 import engine

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
PEER_TIMEOUT_BIT = 1 << 4


def ptr_array(ts):
    return (ctypes.c_void_p * len(ts))(*[t.data_ptr() if t is not None else None for t in ts])


def call(parts, flag_out, flag_in, seq, resid, y, status, rank, size):
    L = engine.lib()
    rc = L.bmo_k_tp_exchange(ptr_array(parts), ptr_array(flag_out), flag_in.data_ptr(), seq.data_ptr(),
                             resid.data_ptr(), y.data_ptr(), status.data_ptr(), rank, size, resid.numel(),
                             torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return rc


@pytest.mark.parametrize("size,rank,n", [(2, 0, 4096), (3, 1, 1024), (8, 5, 4096)])
def test_exchange_sums_in_rank_order_and_publishes(size, rank, n):
    rng = np.random.default_rng(size * 10 + rank)
    seq = torch.zeros(1, dtype=torch.int64, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    flag_in = torch.zeros(8, dtype=torch.int64, device=DEV)
    peer_words = [torch.zeros(1, dtype=torch.int64, device=DEV) for _ in range(size)]
    for e in (1, 2):  # two exchanges: the number advances
        parts_h = [rng.standard_normal(n) * 10.0 ** rng.integers(-3, 3) for _ in range(size)]
        resid_h = rng.standard_normal(n).astype(np.float32)
        parts = [torch.from_numpy(p).to(DEV) for p in parts_h]
        resid = torch.from_numpy(resid_h).to(DEV)
        y = torch.full((n,), float("nan"), device=DEV)
        flag_in[:size] = e  # every peer has published exchange e
        assert call(parts, peer_words, flag_in, seq, resid, y, status, rank, size) == 0
        assert int(status.item()) == 0
        acc = np.zeros(n)
        for p in parts_h:
            acc = acc + p
        want = (resid_h + acc.astype(np.float32)).astype(np.float32)
        np.testing.assert_array_equal(y.cpu().numpy(), want)
        for r in range(size):  # published into every peer's word, not its own
            assert int(peer_words[r].item()) == (0 if r == rank else e)


def test_exchange_wait_runs_out_and_reports():
    size, rank, n = 2, 0, 512
    seq = torch.zeros(1, dtype=torch.int64, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    flag_in = torch.zeros(8, dtype=torch.int64, device=DEV)  # the peer never publishes
    peer_words = [torch.zeros(1, dtype=torch.int64, device=DEV) for _ in range(size)]
    parts = [torch.ones(n, dtype=torch.float64, device=DEV) for _ in range(size)]
    resid = torch.zeros(n, device=DEV)
    y = torch.full((n,), -7.0, device=DEV)
    t0 = time.perf_counter()
    assert call(parts, peer_words, flag_in, seq, resid, y, status, rank, size) == 0
    first = time.perf_counter() - t0
    assert int(status.item()) & PEER_TIMEOUT_BIT
    assert 1.0 < first < 30.0, first
    assert (y.cpu().numpy() == -7.0).all()
    # with the bit set, the next exchange returns at once and writes nothing
    t0 = time.perf_counter()
    assert call(parts, peer_words, flag_in, seq, resid, y, status, rank, size) == 0
    assert time.perf_counter() - t0 < 0.5
    assert (y.cpu().numpy() == -7.0).all()


def test_exchange_argument_errors():
    L = engine.lib()
    one = torch.zeros(8, dtype=torch.int64, device=DEV)
    d = torch.zeros(16, dtype=torch.float64, device=DEV)
    f = torch.zeros(16, device=DEV)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    s = torch.cuda.current_stream().cuda_stream
    for rank, size, n in [(0, 1, 16), (2, 2, 16), (0, 9, 16), (0, 2, 0), (0, 2, 8193)]:
        rc = L.bmo_k_tp_exchange(ptr_array([d] * max(size, 1)), ptr_array([one] * max(size, 1)), one.data_ptr(),
                                 one.data_ptr(), f.data_ptr(), f.data_ptr(), st.data_ptr(), rank, size, n, s)
        assert rc != 0, (rank, size, n)
