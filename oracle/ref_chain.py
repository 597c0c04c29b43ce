"""The reference's decode step, run as its own CUDA kernels chained in its own
order on a B200 (TEST INFRASTRUCTURE ONLY: the parity oracle of the engine).

utkarshyadav009/bmo_jetson runs its Jetson decode step as a chain of eager
kernel launches (``apply_*_gpu`` interceptors in src/bmo_compute.cpp): per
temporal layer (:2188-2640) ``launch_rmsnorm`` -> ``launch_gemv_q4_0_q8_1``
(QKV) -> ``launch_rope_interleaved`` on q and on k -> ``launch_decode_attention``
-> GEMV (O) -> ``launch_residual_add`` -> ``launch_rmsnorm`` -> GEMV (FFN in)
-> ``launch_swiglu_split`` -> GEMV (FFN out) -> ``launch_residual_add``; then
the output norm and the text head plus its bias (:2660-2735).  A depformer
step (:2741-3340) is GEMV (``depformer_in.{cb}``) -> residual add of the
previous token's embedding row -> six layers of the same chain without RoPE
on the step's row slices of the stacked projections and its own FFN, with a
linear 8-slot ring -> GEMV (``linears.{cb}``).  The input embedding is summed
on the host in channel order (:1867-1912) and the greedy tokens are the first
maximum (src/bmo_api.cpp:638-666, logit 2048 excluded).

This module drives exactly that chain with the reference's kernels compiled
unmodified from its sources (``oracle/_ref/libbmo_refkernels.so``, made by
``make -C oracle ref``), on weights read straight from the GGUF through
gguf-py, so it needs none of the engine's code.  It runs where that library
and a GPU exist.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import oracle as _orc

_vp, _i, _f = ctypes.c_void_p, ctypes.c_int, ctypes.c_float


def ref_dev_lib() -> ctypes.CDLL:
    """The device-pointer launchers of the reference's kernels (refd_*)."""
    L = ctypes.CDLL(_orc.REF_SO)
    L.refd_rmsnorm.argtypes = [_vp, _vp, _f, _i, _vp]
    L.refd_residual.argtypes = [_vp, _vp, _i, _vp]
    L.refd_rope.argtypes = [_vp, _i, _i, _vp, _f, _vp]
    L.refd_swiglu.argtypes = [_vp, _i, _vp]
    L.refd_gemv.argtypes = [_vp, _vp, _vp, _i, _i, _vp]
    L.refd_attention.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp] + [_i] * 6 + [_vp]
    L.refd_rvq_decode.argtypes = [_vp, _vp, _vp]
    L.refd_rvq_encode.argtypes = [_vp] * 9
    for n in ("refd_rmsnorm", "refd_residual", "refd_rope", "refd_swiglu", "refd_gemv", "refd_attention",
              "refd_rvq_decode", "refd_rvq_encode", "refd_sync"):
        getattr(L, n).restype = _i
    return L


def available() -> bool:
    return os.path.isfile(_orc.REF_SO)


def _f16_to_f32(raw: np.ndarray) -> np.ndarray:
    return raw.view(np.float16).astype(np.float32)


def _q4_0_rows_to_f32(raw: np.ndarray, dim: int) -> np.ndarray:
    """ggml dequantize_row_q4_0: element j of a block is (low nibble of byte j
    - 8) * d, element j + 16 (high nibble - 8) * d."""
    b = raw.reshape(-1, 18)
    d = b[:, :2].copy().view(np.float16).astype(np.float32)
    q = b[:, 2:]
    lo = (q & 0x0F).astype(np.float32) - 8.0
    hi = (q >> 4).astype(np.float32) - 8.0
    return (np.concatenate([lo, hi], axis=1) * d).astype(np.float32).reshape(-1)[:dim]


class RefChain:
    """One model on one GPU, decoded by the reference's kernels in its order."""

    def __init__(self, gguf_path: str, n_ctx: int, device: int = 0):
        import torch
        from gguf import GGUFReader

        self.torch = torch
        self.dev = torch.device(f"cuda:{device}")
        torch.cuda.set_device(self.dev)
        self.L = ref_dev_lib()
        rd = GGUFReader(gguf_path)
        self._t = {t.name: t for t in rd.tensors}

        def scalar(name, default):
            t = self._t.get(name)
            return default if t is None else np.asarray(t.data).reshape(-1)[0].item()

        self.n_layers = int(scalar("n_layers", 0))
        self.n_embd = int(scalar("n_embd", 0))
        self.n_heads = int(scalar("n_heads", 0))
        self.head_dim = int(scalar("head_dim", self.n_embd // max(self.n_heads, 1)))
        self.theta = float(scalar("rope_theta", 10000.0))
        self.eps = float(scalar("norm_eps", 1e-8))
        self.n_ctx = n_ctx
        q_dim = self.n_heads * self.head_dim
        qkv_rows = self._rows(f"transformer_layers_0_self_attn_in_proj_weight")
        self.n_kv = (qkv_rows - q_dim) // 2 // self.head_dim
        self.ffn = self._rows("transformer_layers_0_gating_linear_in_weight") // 2
        self.text_vocab = self._rows("text_linear.weight") if "text_linear.weight" in self._t else 0
        self.dep_q = sum(1 for k in range(64) if f"depformer_in.{k}.weight" in self._t)
        self.dep_dim = self._rows("depformer_in.0.weight") if self.dep_q else 0
        self.dep_heads = int(scalar("depformer_num_heads", 16))
        self.dep_hd = self.dep_dim // self.dep_heads if self.dep_q else 0
        self.dep_ffn = self._rows("depformer_layers_0_gating_0_linear_in_weight") // 2 if self.dep_q else 0
        self.audio_vocab = self._rows("linears.0.weight") if self.dep_q else 0
        self.dep_n_ctx = self.dep_q

        self._w = {}
        dev = self.dev
        f32 = torch.float32
        self.k_cache = torch.zeros(self.n_layers * self.n_kv * n_ctx * self.head_dim, dtype=torch.float16, device=dev)
        self.v_cache = torch.zeros_like(self.k_cache)
        dn = 6 * self.dep_heads * self.dep_n_ctx * self.dep_hd
        self.dk_cache = torch.zeros(max(dn, 1), dtype=torch.float16, device=dev)
        self.dv_cache = torch.zeros_like(self.dk_cache)
        big = max(self.n_embd, q_dim + 2 * self.n_kv * self.head_dim, 2 * self.ffn, self.text_vocab,
                  3 * self.dep_dim, 2 * self.dep_ffn, self.audio_vocab, 64)
        self.q8 = torch.zeros(big // 32 * 36 + 64, dtype=torch.uint8, device=dev)
        self.buf = [torch.zeros(big, dtype=f32, device=dev) for _ in range(8)]
        self.pos_dev = torch.zeros(1, dtype=torch.int32, device=dev)

    # ---- weights ----
    def _rows(self, name: str) -> int:
        return int(self._t[name].shape[1]) if len(self._t[name].shape) > 1 else 1

    def _dev(self, name: str):
        """Device copy of a tensor's raw bytes (Q4_0 blocks or f32 values)."""
        if name not in self._w:
            t = self._t[name]
            raw = np.ascontiguousarray(np.asarray(t.data)).view(np.uint8).reshape(-1)
            self._w[name] = self.torch.from_numpy(raw.copy()).to(self.dev)
        return self._w[name]

    def _emb_row(self, name: str, tok: int, dim: int):
        """One embedding row as fp32 (the reference's to_float), or None when the
        token is outside the table or the table's width is not `dim`."""
        t = self._t.get(name)
        if t is None or tok < 0:
            return None
        cols, rows = int(t.shape[0]), int(t.shape[1])
        if cols != dim or tok >= rows:
            return None
        raw = np.asarray(t.data).view(np.uint8).reshape(rows, -1)[tok]
        tt = int(t.tensor_type)
        if tt == 0:
            return raw.view(np.float32).copy()
        if tt == 1:
            return _f16_to_f32(raw)
        if tt == 2:
            return _q4_0_rows_to_f32(raw, dim)
        raise ValueError(f"{name}: embedding type {tt} not handled")

    # ---- one reference launch each ----
    def _ck(self, rc, what):
        if rc != 0:
            raise RuntimeError(f"{what}: CUDA error {rc}")

    def rmsnorm(self, x, w, n, y):
        self._ck(self.L.refd_rmsnorm(x.data_ptr(), w.data_ptr(), self.eps, n, y.data_ptr()), "rmsnorm")

    def gemv(self, W, byte_off, x, y, rows, cols):
        self._ck(self.L.refd_gemv(W.data_ptr() + byte_off, x.data_ptr(), y.data_ptr(), rows, cols,
                                  self.q8.data_ptr()), "gemv")

    def residual(self, a, b, n, y):
        self._ck(self.L.refd_residual(a.data_ptr(), b.data_ptr(), n, y.data_ptr()), "residual")

    # ---- the temporal step ----
    def embed(self, tokens) -> np.ndarray:
        """bmo_embed_input_tokens_into: acc = 0, then += text row, += audio rows in channel order."""
        acc = np.zeros(self.n_embd, np.float32)
        names = ["text_emb.weight"] + [f"emb.{k}.weight" for k in range(len(tokens) - 1)]
        for name, tok in zip(names, tokens):
            row = self._emb_row(name, int(tok), self.n_embd)
            if row is not None:
                acc = (acc + row).astype(np.float32)
        return acc

    def layer(self, l: int, x, pos: int):
        """Temporal layer l on device vector x (modified in place, the residual stream)."""
        d, hd, H, nkv = self.n_embd, self.head_dim, self.n_heads, self.n_kv
        q_dim, kv_dim = H * hd, nkv * hd
        b = f"transformer_layers_{l}"
        xn, qkv, qr, kr, att, ao, tmp = self.buf[1:8]
        self.pos_dev.fill_(pos)
        self.rmsnorm(x, self._dev(f"{b}_norm1_weight"), d, xn)
        self.gemv(self._dev(f"{b}_self_attn_in_proj_weight"), 0, xn, qkv, q_dim + 2 * kv_dim, d)
        self._ck(self.L.refd_rope(qkv.data_ptr(), H, hd, self.pos_dev.data_ptr(), self.theta, qr.data_ptr()), "rope q")
        self._ck(self.L.refd_rope(qkv.data_ptr() + 4 * q_dim, nkv, hd, self.pos_dev.data_ptr(), self.theta,
                                  kr.data_ptr()), "rope k")
        self._ck(self.L.refd_attention(qr.data_ptr(), kr.data_ptr(), qkv.data_ptr() + 4 * (q_dim + kv_dim),
                                       self.k_cache.data_ptr(), self.v_cache.data_ptr(), att.data_ptr(), hd, H, nkv,
                                       self.n_ctx, pos, l, self.pos_dev.data_ptr()), "attention")
        self.gemv(self._dev(f"{b}_self_attn_out_proj_weight"), 0, att, ao, d, q_dim)
        self.residual(x, ao, d, tmp)
        x[:d].copy_(tmp[:d])
        self.rmsnorm(x, self._dev(f"{b}_norm2_weight"), d, xn)
        self.gemv(self._dev(f"{b}_gating_linear_in_weight"), 0, xn, qkv, 2 * self.ffn, d)
        self._ck(self.L.refd_swiglu(qkv.data_ptr(), self.ffn, att.data_ptr()), "swiglu")
        self.gemv(self._dev(f"{b}_gating_linear_out_weight"), 0, att, ao, d, self.ffn)
        self.residual(x, ao, d, tmp)
        x[:d].copy_(tmp[:d])

    def forward_layers(self, x_host: np.ndarray, pos: int, begin: int, end: int) -> np.ndarray:
        x = self.buf[0]
        x[: self.n_embd].copy_(self.torch.from_numpy(np.ascontiguousarray(x_host, np.float32)))
        for l in range(begin, end):
            self.layer(l, x, pos)
        self._ck(self.L.refd_sync(), "sync")
        return x[: self.n_embd].cpu().numpy()

    def forward_temporal(self, tokens, pos: int):
        """(z = out_norm(x), text logits) of one step; appends every layer's K/V."""
        d = self.n_embd
        x = self.buf[0]
        x[:d].copy_(self.torch.from_numpy(self.embed(tokens)))
        for l in range(self.n_layers):
            self.layer(l, x, pos)
        z, lg, tmp = self.buf[1], self.buf[2], self.buf[3]
        self.rmsnorm(x, self._dev("out_norm_weight"), d, z)
        logits = None
        if self.text_vocab:
            V = self.text_vocab
            self.gemv(self._dev("text_linear.weight"), 0, z, lg, V, d)
            if "text_linear.bias" in self._t:
                self.residual(lg, self._dev("text_linear.bias").view(self.torch.float32), V, tmp)
                lg = tmp
            logits = lg[:V].cpu().numpy()
        self._ck(self.L.refd_sync(), "sync")
        return z[:d].cpu().numpy(), logits

    # ---- the depformer ----
    def reset_depth_kv(self):
        self.dk_cache.zero_()
        self.dv_cache.zero_()

    def forward_depth(self, cb: int, prev_token: int, z_host: np.ndarray) -> np.ndarray:
        """Audio logits of depformer step cb (bmo_forward_depth; resets the depth KV at cb 0)."""
        if cb == 0:
            self.reset_depth_kv()
        D, d, hd, H = self.dep_dim, self.n_embd, self.dep_hd, self.dep_heads
        z, x, xn, qkv, att, ao, tmp, emb = self.buf
        z[:d].copy_(self.torch.from_numpy(np.ascontiguousarray(z_host, np.float32)))
        self.gemv(self._dev(f"depformer_in.{cb}.weight"), 0, z, x, D, d)
        name = "depformer_text_emb.weight" if cb == 0 else f"depformer_emb.{cb - 1}.weight"
        row = self._emb_row(name, int(prev_token), D)
        emb[:D].copy_(self.torch.from_numpy(row if row is not None else np.zeros(D, np.float32)))
        self.residual(x, emb, D, tmp)
        x[:D].copy_(tmp[:D])
        rb = D // 32 * 18  # bytes of one Q4_0 row of width D
        for i in range(6):
            p = f"depformer.layers.{i}"
            self.rmsnorm(x, self._dev(f"{p}.norm1.weight"), D, xn)
            self.gemv(self._dev(f"{p}.self_attn.in_proj_weight"), cb * 3 * D * rb, xn, qkv, 3 * D, D)
            self._ck(self.L.refd_attention(qkv.data_ptr(), qkv.data_ptr() + 4 * D, qkv.data_ptr() + 8 * D,
                                           self.dk_cache.data_ptr(), self.dv_cache.data_ptr(), att.data_ptr(), hd, H,
                                           H, self.dep_n_ctx, cb, i, None), "depth attention")
            self.gemv(self._dev(f"{p}.self_attn.out_proj.weight"), cb * D * rb, att, ao, D, D)
            self.residual(x, ao, D, tmp)
            x[:D].copy_(tmp[:D])
            self.rmsnorm(x, self._dev(f"{p}.norm2.weight"), D, xn)
            g = f"depformer_layers_{i}_gating_{cb}_linear"
            self.gemv(self._dev(f"{g}_in_weight"), 0, xn, qkv, 2 * self.dep_ffn, D)
            self._ck(self.L.refd_swiglu(qkv.data_ptr(), self.dep_ffn, att.data_ptr()), "depth swiglu")
            self.gemv(self._dev(f"{g}_out_weight"), 0, att, ao, D, self.dep_ffn)
            self.residual(x, ao, D, tmp)
            x[:D].copy_(tmp[:D])
        self.gemv(self._dev(f"linears.{cb}.weight"), 0, x, ao, self.audio_vocab, D)
        self._ck(self.L.refd_sync(), "sync")
        return ao[: self.audio_vocab].cpu().numpy()

    def cascade_greedy(self, text_token: int, z_host: np.ndarray):
        """dep_q greedy steps (bmo_forward_depth_cascade with top_k <= 0): tokens and each step's logits."""
        prev, toks, logits = int(text_token), [], []
        for cb in range(self.dep_q):
            lg = self.forward_depth(cb, prev, z_host)
            logits.append(lg)
            prev = int(np.argmax(lg[: min(self.audio_vocab, 2048)]))
            toks.append(prev)
        return np.array(toks, np.int32), logits

    # ---- rings ----
    def set_ring(self, k_fp16: np.ndarray, v_fp16: np.ndarray) -> None:
        """Whole temporal rings as fp16 [n_layers][n_kv][n_ctx][head_dim] (the engine's layout)."""
        self.k_cache.copy_(self.torch.from_numpy(np.ascontiguousarray(k_fp16).reshape(-1)))
        self.v_cache.copy_(self.torch.from_numpy(np.ascontiguousarray(v_fp16).reshape(-1)))

    def ring(self):
        return self.k_cache.cpu().numpy(), self.v_cache.cpu().numpy()
