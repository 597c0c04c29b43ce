"""Golden outputs of the REFERENCE's own decode step on a B200, for the
engine's end-to-end parity tests.

utkarshyadav009/bmo_jetson has no fixtures for its decode step, so its own
CUDA kernels (src/bmo_cuda_kernels.cu, compiled unmodified by
``make -C oracle ref``) are chained in its own order by oracle/ref_chain.py on
seeded synthetic models, and the outputs kept here, so the parity tests can
run where that library is not built.  The cases (models, rings, positions,
tokens) are defined below and regenerated from their seeds; the tokens and
the block's input vector are stored with the outputs, and logit vectors as a
digest of their bytes plus their largest entries.

    python tests/golden/make_ref_chain_golden.py OUT.npz     # on a GPU box
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

OUT = os.path.join(HERE, "ref_chain.npz")


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()[:16]


def history(n_layers: int, n_ctx: int, width: int, seed: int):
    """Seeded N(0,1) K/V rows [slot][width] for every layer's ring."""
    rng = np.random.default_rng(seed)
    for _ in range(n_layers):
        yield (rng.standard_normal((n_ctx, width), dtype=np.float32),
               rng.standard_normal((n_ctx, width), dtype=np.float32))


def ring_f16(rows: np.ndarray, n_kv: int, hd: int) -> np.ndarray:
    """fp32 rows [slot][n_kv * hd] -> fp16 ring [n_kv][slot][hd] (round to nearest even)."""
    n_ctx = rows.shape[0]
    return rows.reshape(n_ctx, n_kv, hd).transpose(1, 0, 2).astype(np.float16)


def frame_tokens(n: int, K: int, text_vocab: int, audio_vocab: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    t = np.empty((n, K), np.int32)
    t[:, 0] = rng.integers(0, text_vocab, n)
    t[:, 1:] = rng.integers(0, audio_vocab, (n, K - 1))
    return t


# Model-level cases: (synthetic preset, ring slots, first position, frames, history seed, token seed)
FRAME_CASES = {
    "tiny": ("tiny", 16, 37, 3, 11, 12),
    "tiny17": ("tiny17", 64, 70, 2, 13, 14),
    "config2": ("config2", 512, 700, 3, 7, 1),
}
# One full-width temporal block at a wrapped position (config 1).
BLOCK_CASE = ("config1", 512, 700, 5, 6)   # preset, ring slots, pos, history seed, input seed


def model_path(preset: str, model_dir: str | None = None) -> str:
    from bmo_jetson_b200 import synth
    return synth.ensure_model(preset, model_dir or os.environ.get("BMO_MODEL_DIR"))


def run_chain_frames(name: str, model_dir: str | None = None) -> dict:
    """The reference chain's outputs for one FRAME_CASES entry."""
    from oracle.ref_chain import RefChain
    preset, n_ctx, pos0, n_frames, hseed, tseed = FRAME_CASES[name]
    ch = RefChain(model_path(preset, model_dir), n_ctx)
    w = ch.n_kv * ch.head_dim
    ks, vs = [], []
    for k, v in history(ch.n_layers, n_ctx, w, hseed):
        ks.append(ring_f16(k, ch.n_kv, ch.head_dim))
        vs.append(ring_f16(v, ch.n_kv, ch.head_dim))
    ch.set_ring(np.stack(ks), np.stack(vs))
    K = 1 + sum(1 for i in range(64) if f"emb.{i}.weight" in ch._t)
    toks = frame_tokens(n_frames, K, ch.text_vocab, ch.audio_vocab or 2048, tseed)
    out = {"tokens": toks}
    for f in range(n_frames):
        z, lg = ch.forward_temporal(toks[f], pos0 + f)
        text = int(np.argmax(lg))
        audio, dl = ch.cascade_greedy(text, z)
        out[f"z{f}"] = z
        out[f"logits{f}"] = lg
        out[f"text{f}"] = np.int32(text)
        out[f"audio{f}"] = audio
        out[f"dlogits{f}"] = np.stack(dl)
    kr, vr = ch.ring()
    out["ring_digest"] = np.array(digest(kr, vr))
    return out


def run_chain_block(model_dir: str | None = None) -> dict:
    from oracle.ref_chain import RefChain
    preset, n_ctx, pos, hseed, xseed = BLOCK_CASE
    ch = RefChain(model_path(preset, model_dir), n_ctx)
    (k, v), = history(1, n_ctx, ch.n_kv * ch.head_dim, hseed)
    ch.set_ring(ring_f16(k, ch.n_kv, ch.head_dim)[None], ring_f16(v, ch.n_kv, ch.head_dim)[None])
    x = np.random.default_rng(xseed).standard_normal(ch.n_embd, dtype=np.float32)
    y = ch.forward_layers(x, pos, 0, 1)
    kr, vr = ch.ring()
    slot = pos % n_ctx
    kslot = kr.reshape(ch.n_kv, n_ctx, ch.head_dim)[:, slot]
    vslot = vr.reshape(ch.n_kv, n_ctx, ch.head_dim)[:, slot]
    return {"x": x, "y": y, "kslot": kslot, "vslot": vslot}


def compact(raw: dict) -> dict:
    """Logit vectors become a digest of their bytes plus their 8 largest
    entries (index, value); everything else is kept as it is."""
    res = {}
    for key, val in raw.items():
        tail = key.split("_", 1)[1] if "_" in key else key
        if tail.startswith(("logits", "dlogits")) and not tail.endswith(("_digest", "_top")):
            res[f"{key}_digest"] = np.array(digest(val))
            flat = np.asarray(val, np.float32).reshape(-1)
            top = np.argsort(-flat, kind="stable")[:8]
            res[f"{key}_top"] = np.stack([top.astype(np.float32), flat[top]])
        else:
            res[key] = val
    return res


def main(out_path: str) -> None:
    raw = {}
    for name in FRAME_CASES:
        for key, val in run_chain_frames(name).items():
            raw[f"{name}_{key}"] = val
    for key, val in run_chain_block().items():
        raw[f"block_{key}"] = val
    res = compact(raw)
    np.savez_compressed(out_path, **res)
    print(f"wrote {out_path} ({len(res)} arrays)")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else OUT)
