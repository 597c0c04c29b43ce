"""ctypes bindings for the CPU oracle (TEST INFRASTRUCTURE ONLY).

Loads ``oracle/_build/libbmo_oracle.so`` (the C restatement of the reference
arithmetic) and, when present, ``oracle/_ref/libbmo_refkernels.so`` (the
reference's own CUDA kernels, for golden vectors on a GPU box).  Only tests,
``__graft_entry__.smoke()`` and bench.py's CPU-baseline legs import this.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(_HERE, "_build", "libbmo_oracle.so")
REF_SO = os.path.join(_HERE, "_ref", "libbmo_refkernels.so")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")

KV_F16, KV_Q4_0 = 0, 1

_lib = None


def build() -> None:
    subprocess.check_call(["make", "-s", "-C", _HERE])


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.isfile(ORACLE_SO):
            build()
        L = ctypes.CDLL(ORACLE_SO)
        L.orc_quantize_row_q8_1.argtypes = [_f32p, _u8p, ctypes.c_int]
        L.orc_quantize_row_q4_0.argtypes = [_f32p, _u8p, ctypes.c_int]
        L.orc_dequantize_row_q4_0.argtypes = [_u8p, _f32p, ctypes.c_int]
        L.orc_gemv_q4_0_q8_1.argtypes = [_u8p, _u8p, _f32p, ctypes.c_int, ctypes.c_int]
        L.orc_rmsnorm.argtypes = [_f32p, _f32p, ctypes.c_float, ctypes.c_int, _f32p]
        L.orc_rope_interleaved.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, _f32p]
        L.orc_swiglu.argtypes = [_f32p, ctypes.c_int, _f32p]
        L.orc_decode_attention_f16.argtypes = [_f32p, _f32p, _f32p, _u16p, _u16p, _f32p] + [ctypes.c_int] * 6
        L.orc_decode_attention_q4.argtypes = [_f32p, _f32p, _f32p, _u8p, _u8p, _f32p] + [ctypes.c_int] * 6
        L.orc_gemv_q4_0_q8_1_reforder.argtypes = [_u8p, _u8p, _f32p, ctypes.c_int, ctypes.c_int]
        L.orc_rmsnorm_reforder.argtypes = [_f32p, _f32p, ctypes.c_float, ctypes.c_int, _f32p]
        L.orc_decode_attention_f16_reforder.argtypes = [_f32p, _f32p, _f32p, _u16p, _u16p, _f32p] + [ctypes.c_int] * 6
        L.orc_argmax.argtypes = [_f32p, ctypes.c_int]
        L.orc_fp32_to_fp16.argtypes = [ctypes.c_float]
        L.orc_fp32_to_fp16.restype = ctypes.c_uint16
        L.orc_fp16_to_fp32.argtypes = [ctypes.c_uint16]
        L.orc_fp16_to_fp32.restype = ctypes.c_float
        L.orc_model_load.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_int]
        L.orc_model_load.restype = ctypes.c_void_p
        L.orc_model_free.argtypes = [ctypes.c_void_p]
        L.orc_model_geometry.argtypes = [ctypes.c_void_p, _i32p, ctypes.c_int]
        L.orc_model_set_threads.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.orc_reset.argtypes = [ctypes.c_void_p]
        L.orc_reset_depth_kv.argtypes = [ctypes.c_void_p]
        L.orc_forward_temporal.argtypes = [ctypes.c_void_p, _i32p, ctypes.c_int, ctypes.c_int, _f32p, _f32p,
                                           ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
        L.orc_forward_layers.argtypes = [ctypes.c_void_p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, _f32p]
        L.orc_embed.argtypes = [ctypes.c_void_p, _i32p, ctypes.c_int, _f32p]
        L.orc_text_head.argtypes = [ctypes.c_void_p, _f32p, _f32p, _f32p]
        L.orc_forward_depth.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int32, _f32p, _f32p]
        L.orc_forward_depth_cascade_greedy.argtypes = [ctypes.c_void_p, ctypes.c_int32, _f32p, _i32p]
        L.orc_kv_import.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, _f32p, _f32p]
        L.orc_kv_export.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _f32p]
        L.orc_sessions.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.orc_select_session.argtypes = [ctypes.c_void_p, ctypes.c_int]
        _lib = L
    return _lib


# ---- kernel-level helpers (numpy in, numpy out) ---------------------------

def quantize_q8_1(x: np.ndarray) -> np.ndarray:
    """Q8_1 blocks (36 bytes each: fp16 d, fp16 sum, 32 int8) as uint8[nb, 36]."""
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    out = np.zeros((x.size // 32, 36), np.uint8)
    lib().orc_quantize_row_q8_1(x, out, x.size)
    return out


def quantize_q4_0(x: np.ndarray) -> np.ndarray:
    """ggml Q4_0 blocks (18 bytes each) as uint8[..., nb*18] with x's leading shape."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(x.shape[:-1] + (x.shape[-1] // 32 * 18,), np.uint8)
    lib().orc_quantize_row_q4_0(x.ravel(), out.reshape(-1), x.size)
    return out


def dequantize_q4_0(blocks: np.ndarray, n: int) -> np.ndarray:
    b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1)
    out = np.zeros(n, np.float32)
    lib().orc_dequantize_row_q4_0(b, out, n)
    return out


def gemv_q4_0(W: np.ndarray, x: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """y = W (Q4_0 bytes, [rows, cols/32*18]) @ quantize_q8_1(x)."""
    xq = quantize_q8_1(x)
    y = np.zeros(rows, np.float32)
    lib().orc_gemv_q4_0_q8_1(np.ascontiguousarray(W, np.uint8).reshape(-1), xq.reshape(-1), y, rows, cols)
    return y


def gemv_q4_0_reforder(W: np.ndarray, xq: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """y = W (Q4_0 bytes) @ Q8_1 blocks xq in the reference kernel's own fp32 order (bit-exact)."""
    y = np.zeros(rows, np.float32)
    lib().orc_gemv_q4_0_q8_1_reforder(np.ascontiguousarray(W, np.uint8).reshape(-1),
                                      np.ascontiguousarray(xq, np.uint8).reshape(-1), y, rows, cols)
    return y


def rmsnorm_reforder(x, w, eps=1e-8):
    x = np.ascontiguousarray(x, np.float32)
    y = np.zeros_like(x)
    lib().orc_rmsnorm_reforder(x, np.ascontiguousarray(w, np.float32), eps, x.size, y)
    return y


def attention_f16_reforder(q, k, v, k_cache, v_cache, head_dim, n_heads, n_kv_heads, n_ctx, pos, layer):
    """Ring attention in the reference kernel's order; caches (uint16 fp16 bits) updated in place."""
    out = np.zeros(n_heads * head_dim, np.float32)
    lib().orc_decode_attention_f16_reforder(np.ascontiguousarray(q, np.float32), np.ascontiguousarray(k, np.float32),
                                            np.ascontiguousarray(v, np.float32), k_cache, v_cache, out,
                                            head_dim, n_heads, n_kv_heads, n_ctx, pos, layer)
    return out


def rmsnorm(x, w, eps=1e-8):
    x = np.ascontiguousarray(x, np.float32)
    y = np.zeros_like(x)
    lib().orc_rmsnorm(x, np.ascontiguousarray(w, np.float32), eps, x.size, y)
    return y


def rope(x, n_heads, head_dim, pos, theta=10000.0):
    x = np.ascontiguousarray(x, np.float32).ravel()
    y = np.zeros_like(x)
    lib().orc_rope_interleaved(x, n_heads, head_dim, pos, theta, y)
    return y


def swiglu(h):
    h = np.ascontiguousarray(h, np.float32).ravel()
    y = np.zeros(h.size // 2, np.float32)
    lib().orc_swiglu(h, h.size // 2, y)
    return y


def attention_f16(q, k, v, k_cache, v_cache, head_dim, n_heads, n_kv_heads, n_ctx, pos, layer):
    """Ring attention; k_cache/v_cache are uint16 fp16 bits, updated in place."""
    out = np.zeros(n_heads * head_dim, np.float32)
    lib().orc_decode_attention_f16(np.ascontiguousarray(q, np.float32), np.ascontiguousarray(k, np.float32),
                                   np.ascontiguousarray(v, np.float32), k_cache, v_cache, out,
                                   head_dim, n_heads, n_kv_heads, n_ctx, pos, layer)
    return out


def attention_q4(q, k, v, k_cache, v_cache, head_dim, n_heads, n_kv_heads, n_ctx, pos, layer):
    """Ring attention over Q4_0 caches (uint8 block bytes), updated in place."""
    out = np.zeros(n_heads * head_dim, np.float32)
    lib().orc_decode_attention_q4(np.ascontiguousarray(q, np.float32), np.ascontiguousarray(k, np.float32),
                                  np.ascontiguousarray(v, np.float32), k_cache, v_cache, out,
                                  head_dim, n_heads, n_kv_heads, n_ctx, pos, layer)
    return out


# ---- model-level oracle ---------------------------------------------------

GEOM_KEYS = ("n_layers", "n_embd", "n_heads", "head_dim", "n_codebooks", "dep_q", "text_vocab",
             "audio_vocab", "n_ctx", "n_kv_heads", "ffn_hidden", "dep_dim")


class OracleModel:
    """The reference decode step on the CPU, over the same GGUF file."""

    def __init__(self, gguf_path: str, n_ctx: int = 512, kv_type: int = KV_F16, threads: int = 0):
        self._L = lib()
        self._m = self._L.orc_model_load(gguf_path.encode(), n_ctx, kv_type)
        if not self._m:
            raise RuntimeError(f"oracle failed to load {gguf_path}")
        if threads:
            self._L.orc_model_set_threads(self._m, threads)
        g = np.zeros(12, np.int32)
        self._L.orc_model_geometry(self._m, g, 12)
        self.geom = dict(zip(GEOM_KEYS, (int(v) for v in g)))
        for k, v in self.geom.items():
            setattr(self, k, v)

    def close(self):
        if self._m:
            self._L.orc_model_free(self._m)
            self._m = None

    __del__ = close

    def reset(self):
        self._L.orc_reset(self._m)

    def sessions(self, n):
        """Gives the model n independent temporal rings (ring 0 is the current one)."""
        if self._L.orc_sessions(self._m, n):
            raise RuntimeError("oracle sessions failed")

    def select(self, s):
        """Points every later call at ring s."""
        if self._L.orc_select_session(self._m, s):
            raise RuntimeError(f"oracle select_session({s}) failed")

    def frame_greedy(self, tokens, pos):
        """One greedy frame of the current ring: (z, logits, text token, audio tokens)."""
        z, logits, _ = self.forward_temporal(tokens, pos)
        text = int(np.argmax(logits[:self.text_vocab]))
        return z, logits, text, self.depth_cascade_greedy(text, z)

    def embed(self, tokens):
        t = np.ascontiguousarray(tokens, np.int32)
        out = np.zeros(self.n_embd, np.float32)
        self._L.orc_embed(self._m, t, t.size, out)
        return out

    def forward_temporal(self, tokens, pos, capture=None):
        t = np.ascontiguousarray(tokens, np.int32)
        z = np.zeros(self.n_embd, np.float32)
        logits = np.zeros(max(self.text_vocab, 1), np.float32)
        cap = None
        if capture:
            cap_idx = np.ascontiguousarray(capture, np.int32)
            cap = np.zeros((len(capture), self.n_embd), np.float32)
            rc = self._L.orc_forward_temporal(self._m, t, t.size, pos, z, logits,
                                              cap_idx.ctypes.data, len(capture), cap.ctypes.data)
        else:
            rc = self._L.orc_forward_temporal(self._m, t, t.size, pos, z, logits, None, 0, None)
        if rc:
            raise RuntimeError(f"oracle forward_temporal rc={rc}")
        return z, logits, cap

    def text_head(self, x_final):
        """(z, logits) of the out_norm + text head applied to a given final residual."""
        z = np.zeros(self.n_embd, np.float32)
        logits = np.zeros(max(self.text_vocab, 1), np.float32)
        rc = self._L.orc_text_head(self._m, np.ascontiguousarray(x_final, np.float32), z, logits)
        if rc:
            raise RuntimeError(f"oracle text_head rc={rc}")
        return z, logits

    def forward_layers(self, x, pos, begin, end):
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros_like(x)
        rc = self._L.orc_forward_layers(self._m, x, pos, begin, end, out)
        if rc:
            raise RuntimeError(f"oracle forward_layers rc={rc}")
        return out

    def forward_depth(self, cb, prev, z):
        out = np.zeros(max(self.audio_vocab, 1), np.float32)
        rc = self._L.orc_forward_depth(self._m, cb, prev, np.ascontiguousarray(z, np.float32), out)
        if rc:
            raise RuntimeError(f"oracle forward_depth rc={rc}")
        return out

    def depth_cascade_greedy(self, text_token, z):
        out = np.zeros(max(self.dep_q, 1), np.int32)
        rc = self._L.orc_forward_depth_cascade_greedy(self._m, text_token, np.ascontiguousarray(z, np.float32), out)
        if rc:
            raise RuntimeError(f"oracle cascade rc={rc}")
        return out

    def kv_import(self, layer, slot0, k_rows, v_rows):
        rc = self._L.orc_kv_import(self._m, layer, slot0, k_rows.shape[0],
                                   np.ascontiguousarray(k_rows, np.float32), np.ascontiguousarray(v_rows, np.float32))
        if rc:
            raise RuntimeError(f"oracle kv_import rc={rc}")

    def kv_export(self, which, layer, slot0, n):
        out = np.zeros((n, self.n_kv_heads * self.head_dim), np.float32)
        rc = self._L.orc_kv_export(self._m, which, layer, slot0, n, out)
        if rc:
            raise RuntimeError(f"oracle kv_export rc={rc}")
        return out


# ---- the reference's own CUDA kernels (GPU box only) ---------------------

def ref_lib() -> ctypes.CDLL:
    L = ctypes.CDLL(REF_SO)
    L.ref_gemv_q4_0_q8_1.argtypes = [_u8p, _f32p, _f32p, _u8p, ctypes.c_int, ctypes.c_int]
    L.ref_rmsnorm.argtypes = [_f32p, _f32p, ctypes.c_float, ctypes.c_int, _f32p]
    L.ref_rope.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, _f32p]
    L.ref_swiglu.argtypes = [_f32p, ctypes.c_int, _f32p]
    L.ref_attention.argtypes = [_f32p, _f32p, _f32p, _u16p, _u16p, _f32p] + [ctypes.c_int] * 7
    L.ref_time_gemv.argtypes = [_u8p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    L.ref_time_gemv.restype = ctypes.c_float
    L.ref_time_gemv_cold.argtypes = [_u8p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t,
                                     ctypes.c_int]
    L.ref_time_gemv_cold.restype = ctypes.c_float
    L.ref_time_attention_cold.argtypes = [ctypes.c_int] * 4 + [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
    L.ref_time_attention_cold.restype = ctypes.c_float
    return L
