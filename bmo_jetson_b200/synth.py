"""Synthetic Moshi-shaped GGUF models for tests and benchmarks.

Writes the reference's tensor-name contract (utkarshyadav009/bmo_jetson
src/bmo.cpp:285-508): temporal layers ``transformer_layers_{i}_*``, the
depformer (``depformer.layers.{i}.*`` stacked per-step projections and
``depformer_layers_{i}_gating_{s}_*``), embeddings, heads and the 1-element
hyperparameter tensors.  GEMV weights are N(0, sigma) quantised to Q4_0 with
ggml's reference rule, embeddings N(0, 1) (f16 by default), norms ~1.
Values come from libbmo's counter-based generator, so a (config, seed) pair
names one file.

    python -m bmo_jetson_b200.synth config2 /tmp/model.gguf
"""
from __future__ import annotations

import argparse
import ctypes
import dataclasses
import hashlib
import json
import os
import struct
import zlib

import numpy as np

from . import engine as _eng

GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q8_0, GGML_I32 = 0, 1, 2, 8, 26
_ALIGN = 32


@dataclasses.dataclass
class SynthConfig:
    n_layers: int = 2
    n_embd: int = 256
    n_heads: int = 2
    head_dim: int = 128
    n_kv_heads: int = 0          # 0: same as n_heads
    ffn_hidden: int = 704
    text_vocab: int = 1000       # rows of text_linear (text_emb has one more)
    audio_vocab: int = 2048      # rows of linears.{k} (emb tables have one more)
    n_q: int = 8                 # temporal audio codebooks; K = n_q + 1
    dep_q: int = 8
    dep_dim: int = 256
    dep_heads: int = 4
    dep_ffn: int = 704
    text_bias: bool = True
    emb_type: str = "f16"        # f16 | f32 | q4_0
    weight_sigma: float = 0.02
    seed: int = 0
    rope_theta: float = 10000.0
    norm_eps: float = 1e-8

    def key(self) -> str:
        blob = json.dumps(dataclasses.asdict(self), sort_keys=True).encode()
        return hashlib.sha1(blob).hexdigest()[:12]


PRESETS = {
    # small model for parity tests (runs through the CPU oracle in seconds)
    "tiny": SynthConfig(),
    # tiny with the reference's 17-channel input (n_q = 16) and Q4_0 embeddings
    "tiny17": SynthConfig(n_q=16, emb_type="q4_0", text_bias=False, seed=3),
    # one full-width temporal block (no heads, no depformer), the benchmark's config 1
    "config1": SynthConfig(n_layers=1, n_embd=4096, n_heads=32, head_dim=128, ffn_hidden=11264,
                           text_vocab=0, n_q=8, dep_q=0, seed=1),
    # configs 2 + 3: 32-layer 7B-class temporal transformer, 32000 text head,
    # 8 audio codebook inputs, depformer 6 x 1024 with 16 heads, FFN 2816, dep_q 8
    "config2": SynthConfig(n_layers=32, n_embd=4096, n_heads=32, head_dim=128, ffn_hidden=11264,
                           text_vocab=32000, audio_vocab=2048, n_q=8, dep_q=8, dep_dim=1024, dep_heads=16,
                           dep_ffn=2816, seed=2),
}


_GEN = None  # (library, symbol prefix) of the tensor generator


def use_generator(cdll, prefix: str) -> None:
    """Generates tensors with `cdll`'s <prefix>normal_f32, <prefix>f16 and
    <prefix>q4_0 (the same counter-based generator, bit for bit) instead of
    libbmo's bmo_synth_* -- for processes that must not load the engine."""
    global _GEN
    for name in ("normal_f32", "f16"):
        getattr(cdll, prefix + name).argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_longlong, ctypes.c_float,
                                                 ctypes.c_float, ctypes.c_void_p]
    getattr(cdll, prefix + "q4_0").argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_longlong,
                                               ctypes.c_longlong, ctypes.c_float, ctypes.c_void_p]
    _GEN = (cdll, prefix)


def _gen(name: str):
    if _GEN is None:
        use_generator(_eng.lib(), "bmo_synth_")
    return getattr(_GEN[0], _GEN[1] + name)


def normal_f32(seed: int, stream: int, n: int, mean: float = 0.0, sigma: float = 1.0) -> np.ndarray:
    out = np.empty(n, np.float32)
    _gen("normal_f32")(seed, stream, n, mean, sigma, out.ctypes.data)
    return out


def f16_normal(seed: int, stream: int, n: int, mean: float = 0.0, sigma: float = 1.0) -> np.ndarray:
    out = np.empty(n, np.uint16)
    _gen("f16")(seed, stream, n, mean, sigma, out.ctypes.data)
    return out


def q4_0_normal(seed: int, stream: int, rows: int, cols: int, sigma: float) -> np.ndarray:
    out = np.empty((rows, cols // 32 * 18), np.uint8)
    _gen("q4_0")(seed, stream, rows, cols, sigma, out.ctypes.data)
    return out


def quantize_q4_0(x: np.ndarray) -> np.ndarray:
    L = _eng.lib()
    L.bmo_quantize_q4_0_ref.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p]
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(x.shape[:-1] + (x.shape[-1] // 32 * 18,), np.uint8)
    L.bmo_quantize_q4_0_ref(x.ctypes.data, x.size, out.ctypes.data)
    return out


class _Spec:
    """One tensor: GGUF dims (ne order), type and a generator."""

    def __init__(self, name, ne, gtype, make):
        self.name, self.ne, self.gtype, self.make = name, list(ne), gtype, make

    def nbytes(self) -> int:
        ne0 = self.ne[0]
        rows = int(np.prod(self.ne[1:])) if len(self.ne) > 1 else 1
        per = {GGML_F32: 4 * ne0, GGML_F16: 2 * ne0, GGML_I32: 4 * ne0, GGML_Q4_0: ne0 // 32 * 18,
               GGML_Q8_0: ne0 // 32 * 34}[self.gtype]
        return per * rows


def _stream_id(name: str) -> int:
    return zlib.crc32(name.encode())


def tensor_specs(cfg: SynthConfig):
    """The ordered tensor list of a synthetic model."""
    s = cfg.seed
    specs = []

    def q4(name, rows, cols):
        specs.append(_Spec(name, [cols, rows], GGML_Q4_0,
                           lambda n=name, r=rows, c=cols: q4_0_normal(s, _stream_id(n), r, c, cfg.weight_sigma)))

    def f32(name, n, mean, sigma):
        specs.append(_Spec(name, [n], GGML_F32, lambda nm=name: normal_f32(s, _stream_id(nm), n, mean, sigma)))

    def emb(name, rows, dim):
        if cfg.emb_type == "f16":
            def make(nm=name):
                return f16_normal(s, _stream_id(nm), rows * dim)
            specs.append(_Spec(name, [dim, rows], GGML_F16, make))
        elif cfg.emb_type == "f32":
            specs.append(_Spec(name, [dim, rows], GGML_F32, lambda nm=name: normal_f32(s, _stream_id(nm), rows * dim)))
        elif cfg.emb_type == "q4_0":
            specs.append(_Spec(name, [dim, rows], GGML_Q4_0, lambda nm=name: q4_0_normal(s, _stream_id(nm), rows, dim, 1.0)))
        else:
            raise ValueError(cfg.emb_type)

    def scalar_i32(name, v):
        specs.append(_Spec(name, [1], GGML_I32, lambda v=v: np.array([v], np.int32)))

    def scalar_f32(name, v):
        specs.append(_Spec(name, [1], GGML_F32, lambda v=v: np.array([v], np.float32)))

    scalar_i32("n_layers", cfg.n_layers)
    scalar_i32("n_heads", cfg.n_heads)
    scalar_i32("n_embd", cfg.n_embd)
    scalar_i32("head_dim", cfg.head_dim)
    scalar_i32("n_ctx", 3000)
    scalar_f32("rope_theta", cfg.rope_theta)
    scalar_f32("norm_eps", cfg.norm_eps)
    if cfg.dep_q and cfg.dep_heads != 16:
        scalar_i32("depformer_num_heads", cfg.dep_heads)

    d, hd = cfg.n_embd, cfg.head_dim
    nkv = cfg.n_kv_heads or cfg.n_heads
    q_dim, kv_dim = cfg.n_heads * hd, nkv * hd
    for i in range(cfg.n_layers):
        b = f"transformer_layers_{i}"
        q4(f"{b}_self_attn_in_proj_weight", q_dim + 2 * kv_dim, d)
        q4(f"{b}_self_attn_out_proj_weight", d, q_dim)
        q4(f"{b}_gating_linear_in_weight", 2 * cfg.ffn_hidden, d)
        q4(f"{b}_gating_linear_out_weight", d, cfg.ffn_hidden)
        f32(f"{b}_norm1_weight", d, 1.0, 0.1)
        f32(f"{b}_norm2_weight", d, 1.0, 0.1)
    f32("out_norm_weight", d, 1.0, 0.1)
    if cfg.text_vocab:
        q4("text_linear.weight", cfg.text_vocab, d)
        if cfg.text_bias:
            f32("text_linear.bias", cfg.text_vocab, 0.0, 0.02)
        emb("text_emb.weight", cfg.text_vocab + 1, d)
    for k in range(cfg.n_q):
        emb(f"emb.{k}.weight", cfg.audio_vocab + 1, d)
    if cfg.dep_q:
        D = cfg.dep_dim
        for k in range(cfg.dep_q):
            q4(f"depformer_in.{k}.weight", D, d)
            emb(f"depformer_emb.{k}.weight", cfg.audio_vocab + 1, D)
            q4(f"linears.{k}.weight", cfg.audio_vocab, D)
        emb("depformer_text_emb.weight", (cfg.text_vocab or 1000) + 1, D)
        for i in range(6):
            p = f"depformer.layers.{i}"
            q4(f"{p}.self_attn.in_proj_weight", cfg.dep_q * 3 * D, D)
            q4(f"{p}.self_attn.out_proj.weight", cfg.dep_q * D, D)
            f32(f"{p}.norm1.weight", D, 1.0, 0.1)
            f32(f"{p}.norm2.weight", D, 1.0, 0.1)
            for st in range(cfg.dep_q):
                q4(f"depformer_layers_{i}_gating_{st}_linear_in_weight", 2 * cfg.dep_ffn, D)
                q4(f"depformer_layers_{i}_gating_{st}_linear_out_weight", D, cfg.dep_ffn)
    return specs


def _gguf_str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def write_gguf(cfg: SynthConfig, path: str) -> str:
    """Writes the model to `path` (atomically) and returns the path."""
    specs = tensor_specs(cfg)
    kv = [("general.architecture", 8, _gguf_str("bmo")), ("general.alignment", 4, struct.pack("<I", _ALIGN))]
    header = bytearray()
    header += struct.pack("<IIQQ", 0x46554747, 3, len(specs), len(kv))
    for k, t, v in kv:
        header += _gguf_str(k) + struct.pack("<I", t) + v
    off = 0
    offsets = []
    for sp in specs:
        offsets.append(off)
        off += (sp.nbytes() + _ALIGN - 1) // _ALIGN * _ALIGN
    for sp, o in zip(specs, offsets):
        header += _gguf_str(sp.name) + struct.pack("<I", len(sp.ne))
        header += b"".join(struct.pack("<Q", int(n)) for n in sp.ne)
        header += struct.pack("<IQ", sp.gtype, o)
    pad = (-len(header)) % _ALIGN
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(header + b"\0" * pad)
        for sp in specs:
            data = np.ascontiguousarray(sp.make()).view(np.uint8).reshape(-1)
            if data.size != sp.nbytes():
                raise RuntimeError(f"{sp.name}: generated {data.size} bytes, expected {sp.nbytes()}")
            f.write(data.tobytes())
            f.write(b"\0" * ((-data.size) % _ALIGN))
    os.replace(tmp, path)
    return path


def ensure_model(preset_or_cfg, directory: str | None = None) -> str:
    """Path of a cached synthetic model, generating it if needed."""
    cfg = PRESETS[preset_or_cfg] if isinstance(preset_or_cfg, str) else preset_or_cfg
    directory = directory or os.environ.get("BMO_MODEL_DIR") or os.path.join(os.environ.get("TMPDIR", "/tmp"), "bmo_models")
    os.makedirs(directory, exist_ok=True)
    name = preset_or_cfg if isinstance(preset_or_cfg, str) else "custom"
    path = os.path.join(directory, f"{name}-{cfg.key()}.gguf")
    if not os.path.exists(path):
        write_gguf(cfg, path)
    return path


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("preset", choices=sorted(PRESETS))
    ap.add_argument("out")
    a = ap.parse_args()
    print(write_gguf(PRESETS[a.preset], a.out))


if __name__ == "__main__":
    main()
