"""Offline repacking of a Moshi GGUF into the engine's row-tile layout.

    python -m bmo_jetson_b200.repack IN.gguf OUT.gguf [--keep-raw]

The engine multiplies Q4_0 weights stored as "row tiles" (32 rows by 8
blocks per 4608-byte chunk, tile-major; the layout is described in
csrc/layout.h) and normally converts ggml's row-major blocks into that form
on the GPU while it loads.  This tool does the conversion once, on the host
(libbmo's bmo_q4_0_tile_host, byte for byte the load-time result), and
writes a GGUF that carries it:

* key ``bmo.tiled.version`` = 1 and a one-line ``bmo.tiled.layout`` note;
* for each Q4_0 GEMV matrix N: the I8 tensor ``bmo.tiled:N`` (the tiles) and
  the I32 tensor ``bmo.tiled_desc:N`` = [cols, rows, perm, swiglu_f];
* N itself only with ``--keep-raw`` (then the file still serves the
  reference's loader and tensor-parallel shards);
* every other key and tensor unchanged.

The SwiGLU input matrices (``*_gating[_S]_linear_in[_weight]``, the names the
reference loader gives them, src/bmo.cpp:285-508) are stored in the
gate/up-paired form the engine multiplies them in; embedding tables stay raw
(they are gathered by row, not multiplied).  The engine checks each tiled
tensor's form against the one it asks for and falls back to raw rows, or
fails with a message, when they differ.
"""
from __future__ import annotations

import argparse
import ctypes
import mmap
import os
import re
import struct
import sys
from typing import List, Tuple

import numpy as np

GGUF_MAGIC = 0x46554747
TILED_VERSION = 1
LAYOUT_NOTE = "q4_0 row tiles: 32 rows x 8 blocks per 4608-byte chunk ([8][32][16 B] nibbles, [8][32] fp16 d), tile-major"
T_U32, T_STRING, T_ARRAY = 4, 8, 9
_SCALAR_SIZE = {0: 1, 1: 1, 2: 2, 3: 2, 4: 4, 5: 4, 6: 4, 7: 1, 10: 8, 11: 8, 12: 8}
GGML_Q4_0, GGML_I8, GGML_I32 = 2, 24, 26
PERM_IDENTITY, PERM_SWIGLU = 0, 1
_SWIGLU = re.compile(r"_gating(_\d+)?_linear_in(_weight)?$")


def _row_bytes(gtype: int, ne0: int) -> int:
    per = {0: 4 * ne0, 1: 2 * ne0, 30: 2 * ne0, 2: ne0 // 32 * 18, 8: ne0 // 32 * 34, 24: ne0, 25: 2 * ne0,
           26: 4 * ne0, 27: 8 * ne0, 28: 8 * ne0}
    if gtype not in per:
        raise ValueError(f"tensor type {gtype} is not one this tool copies")
    return per[gtype]


class Tensor:
    def __init__(self, name: str, ne: List[int], gtype: int, offset: int):
        self.name, self.ne, self.gtype, self.offset = name, ne, gtype, offset

    @property
    def rows(self) -> int:
        return int(np.prod(self.ne[1:])) if len(self.ne) > 1 else 1

    @property
    def nbytes(self) -> int:
        return _row_bytes(self.gtype, self.ne[0]) * self.rows


class GgufIn:
    """The parts of a GGUF this tool needs: each key/value entry as raw
    bytes, the tensor infos and the data section (memory-mapped)."""

    def __init__(self, path: str):
        self._f = open(path, "rb")
        self.buf = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        b = self.buf
        magic, self.version, n_t, n_kv = struct.unpack_from("<IIQQ", b, 0)
        if magic != GGUF_MAGIC or self.version not in (2, 3):
            raise ValueError(f"{path}: not a GGUF v2/v3 file")
        off = 24
        self.kv: List[Tuple[str, bytes]] = []
        self.alignment = 32
        for _ in range(n_kv):
            start = off
            key, off = self._str(off)
            vtype = struct.unpack_from("<I", b, off)[0]
            off += 4
            if key == "general.alignment" and vtype == T_U32:
                self.alignment = struct.unpack_from("<I", b, off)[0]
            off = self._skip(off, vtype)
            self.kv.append((key, bytes(b[start:off])))
        self.tensors: List[Tensor] = []
        for _ in range(n_t):
            name, off = self._str(off)
            nd = struct.unpack_from("<I", b, off)[0]
            ne = list(struct.unpack_from(f"<{nd}Q", b, off + 4))
            gtype, toff = struct.unpack_from("<IQ", b, off + 4 + 8 * nd)
            off += 4 + 8 * nd + 12
            self.tensors.append(Tensor(name, ne, gtype, toff))
        self.data0 = (off + self.alignment - 1) // self.alignment * self.alignment

    def _str(self, off: int) -> Tuple[str, int]:
        n = struct.unpack_from("<Q", self.buf, off)[0]
        return self.buf[off + 8:off + 8 + n].decode("utf-8"), off + 8 + n

    def _skip(self, off: int, vtype: int) -> int:
        if vtype == T_STRING:
            return off + 8 + struct.unpack_from("<Q", self.buf, off)[0]
        if vtype == T_ARRAY:
            et, n = struct.unpack_from("<IQ", self.buf, off)
            off += 12
            if et in _SCALAR_SIZE:
                return off + n * _SCALAR_SIZE[et]
            for _ in range(n):
                off = self._skip(off, et)
            return off
        return off + _SCALAR_SIZE[vtype]

    def data(self, t: Tensor) -> memoryview:
        a = self.data0 + t.offset
        return memoryview(self.buf)[a:a + t.nbytes]

    def close(self) -> None:
        self.buf.close()
        self._f.close()


def _gstr(s: str) -> bytes:
    b = s.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def tile_form(t: Tensor) -> Tuple[int, int] | None:
    """(perm, swiglu_f) the engine multiplies tensor `t` in, or None when
    it is not a tiled GEMV matrix (not Q4_0, not a matrix, an embedding)."""
    if t.gtype != GGML_Q4_0 or len(t.ne) != 2 or t.ne[0] % 32:
        return None
    if "emb" in t.name.split(".")[0]:
        return None
    if _SWIGLU.search(t.name) and t.rows % 32 == 0:
        return PERM_SWIGLU, t.rows // 2
    return PERM_IDENTITY, 0


def _tile_fn():
    from . import engine
    fn = engine.lib().bmo_q4_0_tile_host
    fn.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_longlong, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    fn.restype = ctypes.c_longlong
    return fn


def tiled_bytes(rows: int, cols: int, perm: int, swiglu_f: int) -> int:
    """Bytes of the row-tile form of a rows x cols Q4_0 matrix."""
    n = _tile_fn()(None, rows, cols, perm, swiglu_f, None)
    if n < 0:
        raise ValueError(f"Q4_0 {rows}x{cols} perm {perm} F {swiglu_f}: not a shape the GEMV takes")
    return int(n)


def tile_q4_0(raw, rows: int, cols: int, perm: int, swiglu_f: int) -> np.ndarray:
    """The row-tile form of a Q4_0 matrix (libbmo's host tiling)."""
    fn = _tile_fn()
    n = tiled_bytes(rows, cols, perm, swiglu_f)
    src = np.frombuffer(raw, np.uint8)
    out = np.empty(n, np.uint8)
    if fn(src.ctypes.data, rows, cols, perm, swiglu_f, out.ctypes.data) != n:
        raise RuntimeError("tiling failed")
    return out


def repack(src: str, dst: str, keep_raw: bool = False, log=None) -> dict:
    """Writes the repacked form of `src` to `dst` (atomically); returns
    counts of the tensors written."""
    g = GgufIn(src)
    try:
        if any(k.startswith("bmo.tiled") for k, _ in g.kv):
            raise ValueError(f"{src} is already repacked")
        kv = [raw for _, raw in g.kv]
        kv.append(_gstr("bmo.tiled.version") + struct.pack("<II", T_U32, TILED_VERSION))
        kv.append(_gstr("bmo.tiled.layout") + struct.pack("<I", T_STRING) + _gstr(LAYOUT_NOTE))
        # output tensors: (name, ne, type, producer of the bytes)
        outs = []
        n_tiled = 0
        for t in g.tensors:
            form = tile_form(t)
            if form is None or keep_raw:
                outs.append((t.name, t.ne, t.gtype, (lambda t=t: g.data(t))))
            if form is not None:
                perm, f = form
                cols, rows = t.ne[0], t.rows
                tb = tiled_bytes(rows, cols, perm, f)
                outs.append((f"bmo.tiled:{t.name}", [tb], GGML_I8,
                             (lambda t=t, rows=rows, cols=cols, perm=perm, f=f: tile_q4_0(g.data(t), rows, cols, perm, f))))
                outs.append((f"bmo.tiled_desc:{t.name}", [4], GGML_I32,
                             (lambda cols=cols, rows=rows, perm=perm, f=f: np.array([cols, rows, perm, f], np.int32))))
                n_tiled += 1
        al = g.alignment
        header = bytearray(struct.pack("<IIQQ", GGUF_MAGIC, 3, len(outs), len(kv)))
        for raw in kv:
            header += raw
        off, sizes = 0, []
        for name, ne, gtype, _ in outs:
            size = _row_bytes(gtype, ne[0]) * (int(np.prod(ne[1:])) if len(ne) > 1 else 1)
            sizes.append(size)
            header += _gstr(name) + struct.pack("<I", len(ne)) + b"".join(struct.pack("<Q", int(n)) for n in ne)
            header += struct.pack("<IQ", gtype, off)
            off += (size + al - 1) // al * al
        header += b"\0" * ((-len(header)) % al)
        tmp = dst + ".tmp"
        with open(tmp, "wb") as f:
            f.write(header)
            for (name, _, _, make), size in zip(outs, sizes):
                data = make()
                if isinstance(data, np.ndarray):
                    data = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
                mv = memoryview(data).cast("B")
                if mv.nbytes != size:
                    raise RuntimeError(f"{name}: {mv.nbytes} bytes, expected {size}")
                f.write(mv)
                f.write(b"\0" * ((-size) % al))
                if log:
                    log(name)
        os.replace(tmp, dst)
        return {"tensors": len(outs), "tiled": n_tiled, "kept_raw": keep_raw}
    finally:
        g.close()


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("src")
    ap.add_argument("dst")
    ap.add_argument("--keep-raw", action="store_true", help="keep the raw Q4_0 matrices beside their tiles")
    a = ap.parse_args(argv)
    r = repack(a.src, a.dst, a.keep_raw)
    print(f"{a.dst}: {r['tensors']} tensors, {r['tiled']} tiled" + (" (raw rows kept)" if a.keep_raw else ""))
    return 0


if __name__ == "__main__":
    sys.exit(main())
