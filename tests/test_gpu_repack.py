"""Repacked GGUFs on the GPU: the host tiling (bmo_q4_0_tile_host) is the
load-time device repack (bmo_k_repack_q4_0) byte for byte, and an engine
loaded from a repacked file -- tiles only, or tiles beside the raw rows --
computes bit for bit what the engine loaded from the original file computes
(hidden state, text logits, depformer logits and tokens over several
frames), with every GEMV weight copied from the file's tiles.  The load time
of both files is printed.  A real Moshi GGUF (BMO_REAL_GGUF) is loaded both
ways when one is present."""
import os
import time

import numpy as np
import pytest

from bmo_jetson_b200 import engine, repack, synth
from tests.test_repack import SHAPES

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.mark.parametrize("rows,cols,perm,F", SHAPES + [(22528, 4096, 1, 11264), (32000, 4096, 0, 0)])
def test_host_tiling_is_the_device_repack(rows, cols, perm, F):
    L = engine.lib()
    dev = torch.device("cuda:0")
    raw = np.random.default_rng(rows + cols).integers(0, 256, rows * cols // 32 * 18, dtype=np.uint8)
    want_rows = 2 * F if perm == 1 else rows
    n = L.bmo_k_q4_0_tiled_bytes(want_rows, cols, perm, F)
    src = torch.from_numpy(raw).to(dev)
    dst = torch.zeros(n, dtype=torch.uint8, device=dev)
    assert L.bmo_k_repack_q4_0(src.data_ptr(), dst.data_ptr(), want_rows, cols, perm, F, None) == 0
    torch.cuda.synchronize(dev)
    np.testing.assert_array_equal(repack.tile_q4_0(raw, rows, cols, perm, F), dst.cpu().numpy())


def _frames(e, n_frames, seed=4):
    r = np.random.default_rng(seed)
    K = e.n_codebooks
    out = []
    for f in range(n_frames):
        toks = np.concatenate([[r.integers(0, e.text_vocab)], r.integers(0, e.audio_vocab, K - 1)]).astype(np.int32)
        z, lg = e.forward_temporal(toks, copy=True)
        text = int(np.argmax(lg))
        audio = e.forward_depth_cascade(text, z, 0.0, 0)
        dl = [e.forward_depth(cb, int(text if cb == 0 else audio[cb - 1]), z, copy=True) for cb in range(e.dep_q)]
        out.append((z, lg, np.array(audio), np.stack(dl)))
    return out


def _load(path, n_ctx):
    t0 = time.perf_counter()
    e = engine.BMOEngine(path, n_ctx=n_ctx, device=0, kv_type=engine.KV_F16)
    return e, time.perf_counter() - t0


@pytest.mark.parametrize("name,keep_raw", [("tiny", False), ("tiny17", False), ("tiny17", True), ("config2", False)])
def test_repacked_model_is_bit_identical(name, keep_raw, model_dir, tmp_path):
    src = synth.ensure_model(name, model_dir)
    dst = str(tmp_path / f"{name}-tiled.gguf")
    repack.repack(src, dst, keep_raw=keep_raw)
    n_ctx = 512 if name == "config2" else 256
    n_frames = 3 if name == "config2" else 5
    a, ta = _load(src, n_ctx)
    try:
        assert a.tiled_weights == 0
        ref = _frames(a, n_frames)
    finally:
        a.close()
    b, tb = _load(dst, n_ctx)
    try:
        n_tiled = b.tiled_weights
        got = _frames(b, n_frames)
    finally:
        b.close()
    print(f"{name}: load {ta:.2f} s from the original file, {tb:.2f} s from the repacked one; {n_tiled} tiled weights")
    # every GEMV weight came from the tiles: 4 per temporal layer, the text head, and per depformer
    # step its input projection, head and 4 per layer
    info = synth.PRESETS[name]
    expect = 4 * info.n_layers + (1 if info.text_vocab else 0) + info.dep_q * (2 + 4 * 6)
    assert n_tiled == expect
    for f, (x, y) in enumerate(zip(ref, got)):
        for what, u, v in zip(("z", "text logits", "audio tokens", "depformer logits"), x, y):
            np.testing.assert_array_equal(u, v, err_msg=f"{name} frame {f} {what}")


@pytest.mark.skipif(not os.environ.get("BMO_REAL_GGUF"), reason="BMO_REAL_GGUF names no real Moshi GGUF here")
def test_real_model_repacked(tmp_path):
    src = os.environ["BMO_REAL_GGUF"]
    dst = str(tmp_path / "real-tiled.gguf")
    repack.repack(src, dst)
    a, ta = _load(src, 1024)
    try:
        ref = _frames(a, 2)
    finally:
        a.close()
    b, tb = _load(dst, 1024)
    try:
        assert b.tiled_weights > 0
        got = _frames(b, 2)
    finally:
        b.close()
    print(f"real model: load {ta:.2f} s original, {tb:.2f} s repacked")
    for x, y in zip(ref, got):
        for u, v in zip(x, y):
            np.testing.assert_array_equal(u, v)
