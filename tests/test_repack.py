"""Offline repacking (bmo_jetson_b200/repack.py, bmo_q4_0_tile_host) on the
CPU: the host tiling against an independent numpy statement of the row-tile
layout, and repacked files read back with gguf-py -- every GEMV matrix
present as tiles equal to the tiling of its raw rows, with the descriptor of
its form; embedding tables, norms and biases unchanged; raw rows dropped or
kept as asked; a repacked file refused as input."""
import os

import numpy as np
import pytest

from bmo_jetson_b200 import repack, synth


def tile_np(raw: np.ndarray, rows: int, cols: int, perm: int, F: int) -> np.ndarray:
    """Row tiles by array indexing: tile t, lane l holds row 32 t + l
    (perm 0) or gate row 16 t + l / up row F + 16 t + l - 16 (perm 1); chunk
    c holds blocks 8c..8c+7 as [8][32][16 B] nibbles then [8][32] fp16 d;
    missing rows and blocks are zero scales with nibbles 8."""
    nb = cols // 32
    nbx = (nb + 7) // 8 * 8
    n_tiles = F // 16 if perm == 1 else (rows + 31) // 32
    t = np.arange(n_tiles)[:, None]
    lane = np.arange(32)[None, :]
    if perm == 1:
        r = np.where(lane < 16, t * 16 + lane, F + t * 16 + lane - 16)
        live = (t * 16 + (lane & 15)) < F
    else:
        r = t * 32 + lane
        live = np.ones_like(r, bool)
    live &= r < rows
    full = np.zeros((n_tiles, 32, nbx, 18), np.uint8)
    full[..., 2:] = 0x88
    blocks = raw.reshape(rows, nb, 18)
    full[np.nonzero(live)[0], np.nonzero(live)[1], :nb] = blocks[r[live]]
    f = full.reshape(n_tiles, 32, nbx // 8, 8, 18)
    qs = f[..., 2:].transpose(0, 2, 3, 1, 4).reshape(n_tiles, nbx // 8, 4096)
    d = f[..., :2].transpose(0, 2, 3, 1, 4).reshape(n_tiles, nbx // 8, 512)
    return np.concatenate([qs, d], axis=2).reshape(-1)


SHAPES = [(70, 96, 0, 0), (64, 256, 0, 0), (32, 4096, 0, 0), (64, 320, 1, 32), (96, 544, 1, 48), (7, 32, 0, 0)]


@pytest.mark.parametrize("rows,cols,perm,F", SHAPES)
def test_host_tiling_matches_layout(rows, cols, perm, F):
    raw = np.random.default_rng(rows * 7 + cols).integers(0, 256, rows * cols // 32 * 18, dtype=np.uint8)
    got = repack.tile_q4_0(raw, rows, cols, perm, F)
    np.testing.assert_array_equal(got, tile_np(raw, rows, cols, perm, F))
    assert got.size == repack.tiled_bytes(rows, cols, perm, F)


@pytest.mark.parametrize("rows,cols,perm,F", [(64, 48, 0, 0), (60, 64, 1, 30), (64, 64, 1, 16), (0, 64, 0, 0),
                                              (64, 64, 2, 0)])
def test_host_tiling_refuses_other_shapes(rows, cols, perm, F):
    with pytest.raises(ValueError):
        repack.tiled_bytes(rows, cols, perm, F)


def _read(path):
    from gguf import GGUFReader
    rd = GGUFReader(path)
    return rd, {t.name: t for t in rd.tensors}


def _raw_bytes(t):
    return np.asarray(t.data).view(np.uint8).reshape(-1)


@pytest.mark.parametrize("name", ["tiny", "tiny17"])
@pytest.mark.parametrize("keep_raw", [False, True])
def test_repacked_file(name, keep_raw, tmp_path, model_dir):
    src = synth.ensure_model(name, model_dir)
    dst = str(tmp_path / f"{name}-tiled.gguf")
    info = repack.repack(src, dst, keep_raw=keep_raw)
    rd_in, tin = _read(src)
    rd_out, tout = _read(dst)
    assert int(rd_out.fields["bmo.tiled.version"].parts[-1][0]) == 1
    assert bytes(rd_out.fields["bmo.tiled.layout"].parts[-1]).decode().startswith("q4_0 row tiles")
    n_tiled = 0
    for tname, t in tin.items():
        ne = [int(x) for x in t.shape]  # gguf-py lists the dims ne0 first
        form = repack.tile_form(repack.Tensor(tname, ne, int(t.tensor_type), 0))
        if form is None:
            assert tname in tout, tname
            np.testing.assert_array_equal(_raw_bytes(tout[tname]), _raw_bytes(t), err_msg=tname)
            continue
        n_tiled += 1
        perm, F = form
        cols, rows = ne[0], ne[1]
        if "gating" in tname and "linear_in" in tname:
            assert perm == 1 and F == rows // 2
        desc = np.asarray(tout[f"bmo.tiled_desc:{tname}"].data).reshape(-1)
        assert desc.tolist() == [cols, rows, perm, F]
        np.testing.assert_array_equal(_raw_bytes(tout[f"bmo.tiled:{tname}"]),
                                      tile_np(_raw_bytes(t), rows, cols, perm, F), err_msg=tname)
        assert (tname in tout) == keep_raw
        if keep_raw:
            np.testing.assert_array_equal(_raw_bytes(tout[tname]), _raw_bytes(t))
    assert n_tiled == info["tiled"] > 0
    # embedding tables stay raw rows (tiny17 stores them as Q4_0)
    assert "text_emb.weight" in tout and "bmo.tiled:text_emb.weight" not in tout
    with pytest.raises(ValueError, match="already repacked"):
        repack.repack(dst, str(tmp_path / "again.gguf"))
    assert not os.path.exists(str(tmp_path / "again.gguf"))
