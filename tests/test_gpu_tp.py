"""Tensor-parallel batch-1 mode (bmo_init_tp): attention heads and FFN
columns split over ranks, partial sums of the O-projection and FFN-out summed
over the ranks in double and rounded once -- over NVLink peer memory (one
exchange kernel reading every rank's partial buffer through CUDA IPC
mappings; the default) or an NCCL all-reduce (BMO_TP_P2P=0).

Bars: with one rank the frames are bit-identical to the single-GPU handle;
with two ranks (two GPUs) both ranks hold the same hidden state and the
tokens equal the single-GPU run, hidden states and logits within 1e-5 of the
oracle (the sums over ranks reorder the double sums, which may move a rare
rounding tie by one ULP).
"""
import multiprocessing as mp

import numpy as np
import pytest

from bmo_jetson_b200 import engine
from oracle import oracle as orc
from tests.parity import rel_l2

pytestmark = pytest.mark.gpu

N_CTX = 16


def history(e_full, seed=3):
    rng = np.random.default_rng(seed)
    w = e_full.n_kv_heads * e_full.head_dim
    return [(rng.standard_normal((N_CTX, w), dtype=np.float32), rng.standard_normal((N_CTX, w), dtype=np.float32))
            for _ in range(e_full.n_layers)]


def frame_tokens(K, text_vocab, audio_vocab, n=3, seed=9):
    rng = np.random.default_rng(seed)
    return [np.concatenate([[rng.integers(0, text_vocab)], rng.integers(0, audio_vocab, K - 1)]).astype(np.int32)
            for _ in range(n)]


def run_frames(e, hist, toks, kv_slice=None):
    for layer, (k, v) in enumerate(hist):
        if kv_slice is not None:
            k, v = k[:, kv_slice], v[:, kv_slice]
        e.kv_import(layer, 0, k, v)
    out = []
    for i, t in enumerate(toks):
        e.pos = 20 + i  # ring of 16 already wrapped
        z, lg, text, audio = e.forward_frame_greedy(t)
        out.append((z, lg, text, audio))
    return out


def test_tp_one_rank_is_bit_identical_to_single_gpu(tiny_model):
    e1 = engine.BMOEngine(tiny_model, n_ctx=N_CTX, flags=engine.FLAG_EXACT)  # tensor parallel runs the exact order
    et = engine.BMOEngine(tiny_model, n_ctx=N_CTX, tp=(0, 1, engine.tp_unique_id()))
    assert et.tp_size == 1 and e1.tp_size == 1
    hist = history(e1)
    toks = frame_tokens(e1.n_codebooks, e1.text_vocab, e1.audio_vocab)
    a, b = run_frames(e1, hist, toks), run_frames(et, hist, toks)
    for (z1, l1, t1, a1), (z2, l2, t2, a2) in zip(a, b):
        np.testing.assert_array_equal(z1, z2)
        np.testing.assert_array_equal(l1, l2)
        assert t1 == t2
        np.testing.assert_array_equal(a1, a2)
    e1.close()
    et.close()


def _tp_rank(rank, size, gid, path, q, exchange):
    import os
    os.environ["BMO_TP_P2P"] = "1" if exchange == "p2p" else "0"
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch
    torch.cuda.set_device(rank)
    try:
        e = engine.BMOEngine(path, n_ctx=N_CTX, device=rank, tp=(rank, size, gid))
        if e.tp_peer_exchange != (exchange == "p2p"):
            raise RuntimeError(f"exchange path: peer memory {e.tp_peer_exchange}, wanted {exchange}")
        # the full model's KV width, for slicing this rank's heads out of the shared history
        w = e.n_kv_heads * e.head_dim
        full = type("G", (), {"n_kv_heads": e.n_kv_heads * size, "head_dim": e.head_dim, "n_layers": e.n_layers})
        hist = history(full)
        toks = frame_tokens(e.n_codebooks, e.text_vocab, e.audio_vocab)
        out = run_frames(e, hist, toks, kv_slice=slice(rank * w, (rank + 1) * w))
        q.put((rank, [(z, lg, int(t), a) for z, lg, t, a in out], e.n_attn_heads))
        e.close()
    except Exception as ex:  # reported to the parent
        q.put((rank, repr(ex), 0))


@pytest.mark.parametrize("exchange", ["p2p", "nccl"])
def test_tp_two_ranks_match_single_gpu_and_oracle(tiny_model, exchange):
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    size = 2
    gid = engine.tp_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_tp_rank, args=(r, size, gid, tiny_model, q, exchange)) for r in range(size)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(size):
        rank, out, heads = q.get(timeout=600)
        assert not isinstance(out, str), f"rank {rank}: {out}"
        res[rank] = (out, heads)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    # both ranks hold the same state
    for (z0, l0, t0, a0), (z1, l1, t1, a1) in zip(res[0][0], res[1][0]):
        np.testing.assert_array_equal(z0, z1)
        np.testing.assert_array_equal(l0, l1)
        assert t0 == t1
        np.testing.assert_array_equal(a0, a1)
    # against the oracle on the full model
    o = orc.OracleModel(tiny_model, n_ctx=N_CTX)
    full = type("G", (), {"n_kv_heads": o.n_kv_heads, "head_dim": o.head_dim, "n_layers": o.n_layers})
    hist = history(full)
    for layer, (k, v) in enumerate(hist):
        o.kv_import(layer, 0, k, v)
    toks = frame_tokens(o.n_codebooks, o.text_vocab, o.audio_vocab)
    assert res[0][1] * size == o.geom.get("n_heads", res[0][1] * size)
    for i, t in enumerate(toks):
        zo, lo, to, ao = o.frame_greedy(t, 20 + i)
        z, lg, text, audio = res[0][0][i]
        assert rel_l2(z, zo) < 1e-5 and rel_l2(lg, lo) < 1e-5, (i, rel_l2(z, zo), rel_l2(lg, lo))
        assert text == to
        np.testing.assert_array_equal(audio, ao)
    o.close()
