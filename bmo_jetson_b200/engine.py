"""ctypes binding of libbmo.so (the B200 decode-step engine).

``BMOEngine`` mirrors utkarshyadav009/bmo_jetson ``bmo_engine.py`` (same
methods, argument meaning and errors, tracking ``pos`` itself), so code
written against the reference binding runs unchanged; extensions
(``forward_frame_greedy``, KV import/export, device-resident frames) are
additional methods.  ``Kernels`` wraps the device-pointer kernel layer
(include/bmo_kernels.h) for parity tests.

The library is the CUDA engine itself: there is no CPU fallback, and
``bmo_init`` returns NULL (``RuntimeError`` here) without a B200.
"""
from __future__ import annotations

import ctypes
import os
from typing import List, Optional, Tuple

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("BMO_SO_PATH") or os.path.join(_HERE, "lib", "libbmo.so")

_lib = None
_c_i32p = ctypes.POINTER(ctypes.c_int32)
_c_f32p = ctypes.POINTER(ctypes.c_float)

KV_F16, KV_Q4_0 = 0, 1
FLAG_NO_GRAPHS, FLAG_NO_PDL = 1, 2
# summation order (include/bmo_ext.h): default the reference kernels' own
# fp32 order where the model allows; EXACT: double sums rounded once
FLAG_EXACT, FLAG_REF_ORDER, FLAG_DEP_CLUSTER = 8, 16, 32


def lib() -> ctypes.CDLL:
    """Loads libbmo.so (building it first if it is missing)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.isfile(LIB_PATH):
        from . import build as _build
        _build.build()
    L = ctypes.CDLL(LIB_PATH)
    vp, i, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    L.bmo_init.argtypes = [ctypes.c_char_p, i]
    L.bmo_init.restype = vp
    L.bmo_init_ex.argtypes = [ctypes.c_char_p, i, i, i, i]
    L.bmo_init_ex.restype = vp
    L.bmo_free.argtypes = [vp]
    L.bmo_free.restype = None
    L.bmo_reset.argtypes = [vp]
    L.bmo_reset.restype = None
    for name in ("bmo_get_n_layers", "bmo_get_n_embd", "bmo_get_n_codebooks", "bmo_get_dep_q", "bmo_get_text_vocab",
                 "bmo_get_audio_vocab", "bmo_get_n_attn_heads", "bmo_get_head_dim", "bmo_capture_graphs",
                 "bmo_has_cuda_graphs", "bmo_get_kv_type", "bmo_get_n_ctx", "bmo_get_n_kv_heads", "bmo_get_device",
                 "bmo_get_pos", "bmo_sync", "bmo_get_ref_order", "bmo_get_dep_mode", "bmo_get_frame_launches",
                 "bmo_get_tiled_weights"):
        fn = getattr(L, name)
        fn.argtypes = [vp]
        fn.restype = i
    L.bmo_get_stream.argtypes = [vp]
    L.bmo_get_stream.restype = vp
    L.bmo_get_device_bytes.argtypes = [vp]
    L.bmo_get_device_bytes.restype = ctypes.c_size_t
    for name in ("bmo_copy_k_cache_f32", "bmo_copy_v_cache_f32"):
        fn = getattr(L, name)
        fn.argtypes = [vp, i, i, i, _c_f32p, i]
        fn.restype = i
    L.bmo_copy_kv_raw.argtypes = [vp, i, i, i, vp, ctypes.c_longlong]
    L.bmo_copy_kv_raw.restype = ctypes.c_longlong
    L.bmo_kv_import_f32.argtypes = [vp, i, i, i, _c_f32p, _c_f32p]
    L.bmo_kv_import_f32.restype = i
    L.bmo_forward_temporal.argtypes = [vp, _c_i32p, i, i, _c_f32p, _c_f32p]
    L.bmo_forward_temporal.restype = i
    L.bmo_forward_temporal2.argtypes = [vp, _c_i32p, i, i, _c_f32p, _c_f32p, _c_i32p, i, _c_f32p]
    L.bmo_forward_temporal2.restype = i
    L.bmo_forward_depth.argtypes = [vp, i, ctypes.c_int32, _c_f32p, _c_f32p]
    L.bmo_forward_depth.restype = i
    L.bmo_forward_depth_cascade.argtypes = [vp, ctypes.c_int32, _c_f32p, f, i, _c_i32p]
    L.bmo_forward_depth_cascade.restype = i
    L.bmo_forward_frame_greedy.argtypes = [vp, _c_i32p, i, i, _c_f32p, _c_f32p, _c_i32p, _c_i32p]
    L.bmo_forward_frame_greedy.restype = i
    L.bmo_forward_layers.argtypes = [vp, _c_f32p, i, i, i, _c_f32p]
    L.bmo_forward_layers.restype = i
    L.bmo_debug_tap.argtypes = [vp, i, _c_f32p, i]
    L.bmo_debug_tap.restype = i
    L.bmo_enqueue_temporal.argtypes = [vp, vp, i, i]
    L.bmo_enqueue_temporal.restype = i
    L.bmo_enqueue_cascade.argtypes = [vp, ctypes.c_int32]
    L.bmo_enqueue_cascade.restype = i
    L.bmo_enqueue_frame.argtypes = [vp, vp, i, i, vp]
    L.bmo_enqueue_frame.restype = i
    L.bmo_tp_unique_id.argtypes = [vp]
    L.bmo_tp_unique_id.restype = i
    L.bmo_init_tp.argtypes = [ctypes.c_char_p, i, i, i, i, i, i, vp]
    L.bmo_init_tp.restype = vp
    L.bmo_get_tp_size.argtypes = [vp]
    L.bmo_get_tp_size.restype = i
    L.bmo_get_tp_rank.argtypes = [vp]
    L.bmo_get_tp_rank.restype = i
    L.bmo_get_tp_exchange.argtypes = [vp]
    L.bmo_get_tp_exchange.restype = i
    L.bmo_batch_init.argtypes = [vp, i]
    L.bmo_batch_init.restype = i
    L.bmo_batch_sessions.argtypes = [vp]
    L.bmo_batch_sessions.restype = i
    L.bmo_forward_frame_batch.argtypes = [vp, i, vp, vp, i, vp, vp, vp, vp]
    L.bmo_forward_frame_batch.restype = i
    L.bmo_enqueue_frame_batch.argtypes = [vp, i, vp, vp, i, vp, vp]
    L.bmo_enqueue_frame_batch.restype = i
    L.bmo_batch_kv_import_f32.argtypes = [vp, i, i, i, i, _c_f32p, _c_f32p]
    L.bmo_batch_kv_import_f32.restype = i
    L.bmo_batch_reset.argtypes = [vp, i]
    L.bmo_batch_reset.restype = i
    L.bmo_loop_reset.argtypes = [vp, ctypes.c_uint32]
    L.bmo_loop_reset.restype = i
    L.bmo_loop_run.argtypes = [vp, i, _c_i32p, i, f, i, f, i, _c_i32p]
    L.bmo_loop_run.restype = i
    L.bmo_loop_frame.argtypes = [vp]
    L.bmo_loop_frame.restype = i
    L.bmo_loop_supported.argtypes = [vp]
    L.bmo_loop_supported.restype = i
    L.bmo_last_error.argtypes = [vp]
    L.bmo_last_error.restype = ctypes.c_char_p
    L.bmo_rvq_decode.argtypes = [vp, vp, vp, vp]
    L.bmo_rvq_decode.restype = i
    L.bmo_rvq_encode.argtypes = [vp] * 10
    L.bmo_rvq_encode.restype = i
    # kernel layer
    sz = ctypes.c_size_t
    L.bmo_k_quantize_q8_1.argtypes = [vp, vp, i, vp]
    L.bmo_k_quantize_q8_1.restype = i
    L.bmo_k_q4_0_tiled_bytes.argtypes = [i, i, i, i]
    L.bmo_k_q4_0_tiled_bytes.restype = sz
    L.bmo_k_repack_q4_0.argtypes = [vp, vp, i, i, i, i, vp]
    L.bmo_k_repack_q4_0.restype = i
    L.bmo_k_gemv_scratch_bytes.argtypes = [i, i, i, i]
    L.bmo_k_gemv_scratch_bytes.restype = sz
    L.bmo_k_gemv_q4_0.argtypes = [vp, i, i, i, i, vp, vp, f, vp, vp, vp, vp, vp, sz, i, vp]
    L.bmo_k_gemv_q4_0.restype = i
    L.bmo_k_gemv_q4_0_static.argtypes = [vp, i, i, i, i, vp, vp, f, vp, vp, vp, vp, i, vp]
    L.bmo_k_gemv_q4_0_static.restype = i
    L.bmo_k_gemv_q4_0_ref.argtypes = [vp, i, i, i, i, vp, vp, f, vp, vp, vp, vp, vp, vp]
    L.bmo_k_gemv_q4_0_ref.restype = i
    L.bmo_k_decode_attention_ref.argtypes = [vp] * 6 + [i] * 4 + [vp, i, vp]
    L.bmo_k_decode_attention_ref.restype = i
    L.bmo_k_sample_token.argtypes = [vp, i, f, i, i, vp, vp, vp]
    L.bmo_k_sample_token.restype = i
    L.bmo_k_batch_gemm_scratch_bytes.argtypes = [i, i, i, i, i]
    L.bmo_k_batch_gemm_scratch_bytes.restype = sz
    L.bmo_k_batch_gemm_q4_0.argtypes = [vp, i, i, i, i, vp, vp, f, vp, vp, i, i, vp, sz, vp]
    L.bmo_k_batch_gemm_q4_0.restype = i
    L.bmo_k_decode_attention.argtypes = [vp] * 8 + [i] * 4 + [vp, i, i, vp]
    L.bmo_k_tp_exchange.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p)] + [vp] * 5 + \
        [i, i, i, vp]
    L.bmo_k_tp_exchange.restype = i
    L.bmo_k_decode_attention.restype = i
    _lib = L
    return L


def _preload_nccl() -> None:
    """libbmo resolves NCCL (libnccl.so.2) at run time and reuses a copy the
    process already loaded.  Load the NCCL that this Python environment ships
    (the one PyTorch links) first, so that a later `import torch` finds the
    NCCL it was built against instead of an older system copy."""
    import importlib.util
    import sys
    if "torch" in sys.modules:
        return  # torch has loaded its NCCL already
    spec = importlib.util.find_spec("nvidia.nccl")
    for base in (list(spec.submodule_search_locations) if spec and spec.submodule_search_locations else []):
        cand = os.path.join(base, "lib", "libnccl.so.2")
        if os.path.isfile(cand):
            ctypes.CDLL(cand, mode=ctypes.RTLD_GLOBAL)
            return


def tp_unique_id() -> bytes:
    """A fresh tensor-parallel group id (NCCL unique id, 128 bytes)."""
    _preload_nccl()
    buf = ctypes.create_string_buffer(128)
    rc = lib().bmo_tp_unique_id(buf)
    if rc != 0:
        raise RuntimeError(f"bmo_tp_unique_id rc={rc}")
    return buf.raw


def _err(h) -> str:
    e = lib().bmo_last_error(h)
    return e.decode() if e else "unknown"


class BMOEngine:
    """Handle on one model in one GPU's HBM (reference bmo_engine.py:112-285)."""

    def __init__(self, gguf_path: str, n_ctx: int = 1024, device: int = -1, kv_type: int = -1, flags: int = 0,
                 tp=None):
        """tp = (rank, size, group_id): rank of a tensor-parallel group (bmo_init_tp);
        group_id is the 128-byte tp_unique_id() of one rank, shared by all."""
        L = lib()
        if tp is not None:
            _preload_nccl()
            rank, size, gid = tp
            gid = bytes(gid)
            if len(gid) != 128:
                raise ValueError("tensor-parallel group id must be 128 bytes")
            self._h = L.bmo_init_tp(gguf_path.encode("utf-8"), n_ctx, device, kv_type, flags, int(rank), int(size),
                                    ctypes.c_char_p(gid))
        elif device < 0 and kv_type < 0 and flags == 0:
            self._h = L.bmo_init(gguf_path.encode("utf-8"), n_ctx)
        else:
            self._h = L.bmo_init_ex(gguf_path.encode("utf-8"), n_ctx, device, kv_type, flags)
        if not self._h:
            raise RuntimeError(f"bmo_init returned NULL for path: {gguf_path}")
        self.n_layers = L.bmo_get_n_layers(self._h)
        self.n_embd = L.bmo_get_n_embd(self._h)
        self.n_codebooks = L.bmo_get_n_codebooks(self._h)
        self.dep_q = L.bmo_get_dep_q(self._h)
        self.text_vocab = L.bmo_get_text_vocab(self._h)
        self.audio_vocab = L.bmo_get_audio_vocab(self._h)
        self.n_attn_heads = L.bmo_get_n_attn_heads(self._h)
        self.head_dim = L.bmo_get_head_dim(self._h)
        self.n_kv_heads = L.bmo_get_n_kv_heads(self._h)
        self.n_ctx = L.bmo_get_n_ctx(self._h)
        self.kv_type = L.bmo_get_kv_type(self._h)
        self._pos = 0
        self._buf_z = np.empty(self.n_embd, dtype=np.float32)
        self._buf_text = np.empty(max(self.text_vocab, 1), dtype=np.float32)
        self._buf_audio = np.empty(max(self.audio_vocab, 1), dtype=np.float32)
        self._buf_depth_audio = np.empty(max(self.dep_q, 8), dtype=np.int32)

        self.tp_size = L.bmo_get_tp_size(self._h) or 1
        self.tp_rank = L.bmo_get_tp_rank(self._h)
        self.tp_peer_exchange = bool(L.bmo_get_tp_exchange(self._h))

    # ---- reference methods -------------------------------------------------
    def reset(self) -> None:
        lib().bmo_reset(self._h)
        self._pos = 0

    @property
    def pos(self) -> int:
        return self._pos

    @pos.setter
    def pos(self, value: int) -> None:
        self._pos = int(value)

    def capture_graphs(self) -> int:
        return lib().bmo_capture_graphs(self._h)

    def has_cuda_graphs(self) -> bool:
        return bool(lib().bmo_has_cuda_graphs(self._h))

    @property
    def ref_order(self) -> bool:
        """True when the handle computes in the reference kernels' fp32 order
        (bit-identical to the reference's chain), False for the exact order."""
        return bool(lib().bmo_get_ref_order(self._h))

    @property
    def frame_launches(self) -> int:
        """Kernels one greedy frame launches on the device."""
        return int(lib().bmo_get_frame_launches(self._h))

    @property
    def tiled_weights(self) -> int:
        """GEMV weights copied from a repacked file's tiles (0 for a plain GGUF)."""
        return int(lib().bmo_get_tiled_weights(self._h))

    @property
    def dep_mode(self) -> int:
        """How greedy depformer cascades run: 0 one kernel per op, 1 one
        cluster launch, 2 one cooperative launch over every SM."""
        return int(lib().bmo_get_dep_mode(self._h))

    # ---- the caller's frame loop on the device ----
    LOOP_OUT = 17  # per frame: text token, 8 audio tokens, 8 codec tokens

    def loop_reset(self, seed: int = 1337) -> None:
        """Starts a conversation at frame 0 with the daemon's start state and
        its sampler generator std::mt19937(seed)."""
        rc = lib().bmo_loop_reset(self._h, int(seed) & 0xFFFFFFFF)
        if rc != 0:
            raise RuntimeError(f"loop_reset rc={rc}: {_err(self._h)}")

    def loop_run(self, n_frames: int, user_tokens: Optional[np.ndarray] = None, sampling: bool = False,
                 temp_text: float = 0.7, top_k_text: int = 25, temp_audio: float = 0.8,
                 top_k_audio: int = 250) -> np.ndarray:
        """Runs n_frames (1..64) frames on the device; user_tokens [n][8] or
        None for the daemon's silence tokens.  Returns int32 [n][17]."""
        out = np.zeros((int(n_frames), self.LOOP_OUT), np.int32)
        up = None
        if user_tokens is not None:
            user_tokens = np.ascontiguousarray(user_tokens, dtype=np.int32)
            assert user_tokens.shape == (n_frames, 8), user_tokens.shape
            up = user_tokens.ctypes.data_as(_c_i32p)
        rc = lib().bmo_loop_run(self._h, int(n_frames), up, 1 if sampling else 0, float(temp_text), int(top_k_text),
                                float(temp_audio), int(top_k_audio), out.ctypes.data_as(_c_i32p))
        if rc != 0:
            raise RuntimeError(f"loop_run rc={rc}: {_err(self._h)}")
        return out

    @property
    def loop_supported(self) -> bool:
        """True when the model runs the daemon's frame loop on the device
        (text head, 8 depformer steps, 9 or 17 input channels, one GPU)."""
        return bool(lib().bmo_loop_supported(self._h))

    @property
    def loop_frame(self) -> int:
        """Frames run since loop_reset (-1 before it)."""
        return int(lib().bmo_loop_frame(self._h))

    def forward_temporal(self, tokens: np.ndarray, copy: bool = False) -> Tuple[np.ndarray, np.ndarray]:
        assert tokens.dtype == np.int32 and tokens.shape == (self.n_codebooks,), (
            f"Expected int32 array of shape ({self.n_codebooks},), got {tokens.dtype} shape {tokens.shape}")
        tokens = np.ascontiguousarray(tokens)
        rc = lib().bmo_forward_temporal(self._h, tokens.ctypes.data_as(_c_i32p), int(tokens.size), int(self._pos),
                                        self._buf_z.ctypes.data_as(_c_f32p), self._buf_text.ctypes.data_as(_c_f32p))
        if rc != 0:
            raise RuntimeError(f"forward_temporal rc={rc}: {_err(self._h)}")
        self._pos += 1
        if copy:
            return self._buf_z.copy(), self._buf_text.copy()
        return self._buf_z, self._buf_text

    def forward_temporal2(self, tokens: np.ndarray, capture_layers: Optional[List[int]] = None
                          ) -> Tuple[np.ndarray, np.ndarray, Optional[np.ndarray]]:
        assert tokens.dtype == np.int32 and tokens.shape == (self.n_codebooks,), (
            f"Expected int32 array of shape ({self.n_codebooks},), got {tokens.dtype} shape {tokens.shape}")
        tokens = np.ascontiguousarray(tokens)
        if not capture_layers:
            z, text_logits = self.forward_temporal(tokens)
            return z, text_logits, None
        cap_arr = np.array(capture_layers, dtype=np.int32)
        cap_out = np.empty((len(capture_layers), self.n_embd), dtype=np.float32)
        rc = lib().bmo_forward_temporal2(self._h, tokens.ctypes.data_as(_c_i32p), int(tokens.size), int(self._pos),
                                         self._buf_z.ctypes.data_as(_c_f32p), self._buf_text.ctypes.data_as(_c_f32p),
                                         cap_arr.ctypes.data_as(_c_i32p), len(capture_layers),
                                         cap_out.ctypes.data_as(_c_f32p))
        if rc != 0:
            raise RuntimeError(f"forward_temporal2 rc={rc}: {_err(self._h)}")
        self._pos += 1
        return self._buf_z.copy(), self._buf_text.copy(), cap_out

    def forward_depth(self, cb_index: int, prev_token: int, transformer_out: np.ndarray, copy: bool = False) -> np.ndarray:
        assert transformer_out.dtype == np.float32 and transformer_out.shape == (self.n_embd,), (
            f"Expected float32 array of shape ({self.n_embd},), got {transformer_out.dtype} shape {transformer_out.shape}")
        transformer_out = np.ascontiguousarray(transformer_out)
        rc = lib().bmo_forward_depth(self._h, int(cb_index), int(prev_token), transformer_out.ctypes.data_as(_c_f32p),
                                     self._buf_audio.ctypes.data_as(_c_f32p))
        if rc != 0:
            raise RuntimeError(f"forward_depth rc={rc}: {_err(self._h)}")
        return self._buf_audio.copy() if copy else self._buf_audio

    def forward_depth_cascade(self, text_token: int, transformer_out: np.ndarray, temp: float = 0.8,
                              top_k: int = 250) -> np.ndarray:
        transformer_out = np.ascontiguousarray(transformer_out, dtype=np.float32)
        rc = lib().bmo_forward_depth_cascade(self._h, int(text_token), transformer_out.ctypes.data_as(_c_f32p),
                                             float(temp), int(top_k), self._buf_depth_audio.ctypes.data_as(_c_i32p))
        if rc != 0:
            raise RuntimeError(f"forward_depth_cascade rc={rc}: {_err(self._h)}")
        return self._buf_depth_audio[: self.dep_q].copy()

    def get_k_cache_f32(self, layer: int, t_start: int, n_positions: int) -> np.ndarray:
        """Temporal K-cache slice as float32, layout (n_positions, n_heads, head_dim)."""
        return self._cache(lib().bmo_copy_k_cache_f32, layer, t_start, n_positions)

    # ---- extensions ----------------------------------------------------------
    def get_v_cache_f32(self, layer: int, t_start: int, n_positions: int) -> np.ndarray:
        return self._cache(lib().bmo_copy_v_cache_f32, layer, t_start, n_positions)

    def _cache(self, fn, layer, t_start, n_positions):
        nh, hd = self.n_kv_heads, self.head_dim
        n_el = int(n_positions) * nh * hd
        buf = np.empty(n_el, dtype=np.float32)
        n = fn(self._h, int(layer), int(t_start), int(n_positions), buf.ctypes.data_as(_c_f32p), int(n_el))
        if n < 0:
            raise RuntimeError(f"KV cache copy failed with code {n}")
        if n != n_el:
            raise RuntimeError(f"KV cache copy expected {n_el} floats, got {n}")
        return buf.reshape(int(n_positions), nh, hd)

    def kv_raw(self, which: int, part: int, layer: int) -> np.ndarray:
        """Raw ring bytes of one layer (fp16 rows, or Q4_0 nibble/scale planes)."""
        per = self.n_kv_heads * self.n_ctx * self.head_dim
        if self.kv_type == KV_F16:
            nbytes = per * 2 if part == 0 else 0
        else:
            nbytes = per // 2 if part == 0 else per // 16
        out = np.empty(max(nbytes, 1), np.uint8)
        n = lib().bmo_copy_kv_raw(self._h, which, part, layer, out.ctypes.data, nbytes)
        if n < 0:
            raise RuntimeError(f"bmo_copy_kv_raw failed: {n}")
        return out[:n]

    def kv_import(self, layer: int, slot0: int, k_rows: np.ndarray, v_rows: np.ndarray) -> None:
        k = np.ascontiguousarray(k_rows, np.float32)
        v = np.ascontiguousarray(v_rows, np.float32)
        rc = lib().bmo_kv_import_f32(self._h, layer, slot0, k.shape[0], k.ctypes.data_as(_c_f32p),
                                     v.ctypes.data_as(_c_f32p))
        if rc != 0:
            raise RuntimeError(f"bmo_kv_import_f32 rc={rc}: {_err(self._h)}")

    def forward_frame_greedy(self, tokens: np.ndarray):
        tokens = np.ascontiguousarray(tokens, np.int32)
        text = np.zeros(1, np.int32)
        audio = np.zeros(max(self.dep_q, 1), np.int32)
        rc = lib().bmo_forward_frame_greedy(self._h, tokens.ctypes.data_as(_c_i32p), int(tokens.size), int(self._pos),
                                            self._buf_z.ctypes.data_as(_c_f32p),
                                            self._buf_text.ctypes.data_as(_c_f32p), text.ctypes.data_as(_c_i32p),
                                            audio.ctypes.data_as(_c_i32p))
        if rc != 0:
            raise RuntimeError(f"forward_frame_greedy rc={rc}: {_err(self._h)}")
        self._pos += 1
        return self._buf_z.copy(), self._buf_text.copy(), int(text[0]), audio[: self.dep_q].copy()

    def forward_layers(self, x: np.ndarray, pos: int, layer_begin: int, layer_end: int) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty(self.n_embd, np.float32)
        rc = lib().bmo_forward_layers(self._h, x.ctypes.data_as(_c_f32p), int(pos), int(layer_begin),
                                      int(layer_end), out.ctypes.data_as(_c_f32p))
        if rc != 0:
            raise RuntimeError(f"bmo_forward_layers rc={rc}: {_err(self._h)}")
        return out

    TAPS = {"q": 0, "v": 1, "attn": 2, "xmid": 3, "act": 4, "z": 5, "rope": 6, "dlogits": 7}

    def debug_tap(self, name: str) -> np.ndarray:
        """An activation buffer as left by the last call (see bmo_debug_tap)."""
        out = np.empty(1 << 16, np.float32)
        n = lib().bmo_debug_tap(self._h, self.TAPS[name], out.ctypes.data_as(_c_f32p), out.size)
        if n < 0:
            raise RuntimeError(f"bmo_debug_tap({name}) failed")
        return out[:n].copy()

    def enqueue_frame(self, tokens_dev_ptr: int, n_tokens: int, pos: int, out_tokens_dev_ptr: int) -> None:
        rc = lib().bmo_enqueue_frame(self._h, tokens_dev_ptr, n_tokens, pos, out_tokens_dev_ptr)
        if rc != 0:
            raise RuntimeError(f"bmo_enqueue_frame rc={rc}: {_err(self._h)}")

    def enqueue_temporal(self, tokens_dev_ptr: int, n_tokens: int, pos: int) -> None:
        rc = lib().bmo_enqueue_temporal(self._h, tokens_dev_ptr, n_tokens, pos)
        if rc != 0:
            raise RuntimeError(f"bmo_enqueue_temporal rc={rc}: {_err(self._h)}")

    def enqueue_cascade(self, text_token: int) -> None:
        rc = lib().bmo_enqueue_cascade(self._h, int(text_token))
        if rc != 0:
            raise RuntimeError(f"bmo_enqueue_cascade rc={rc}: {_err(self._h)}")

    # ---- batched sessions ----
    def batch_init(self, n_sessions: int) -> None:
        """Allocates n_sessions independent session rings (bmo_batch_init)."""
        rc = lib().bmo_batch_init(self._h, int(n_sessions))
        if rc != 0:
            raise RuntimeError(f"bmo_batch_init rc={rc}: {_err(self._h)}")

    @property
    def batch_sessions(self) -> int:
        return lib().bmo_batch_sessions(self._h)

    def forward_frame_batch(self, tokens: np.ndarray, pos, sess_ids=None, want_z: bool = False,
                            want_logits: bool = False):
        """One greedy frame for every row of tokens [n][K]: returns (text [n],
        audio [n][dep_q], z [n][n_embd] or None, logits [n][text_vocab] or None)."""
        tokens = np.ascontiguousarray(tokens, np.int32)
        n, K = tokens.shape
        pos = np.ascontiguousarray(pos, np.int32).reshape(n)
        sid = None if sess_ids is None else np.ascontiguousarray(sess_ids, np.int32).reshape(n)
        out = np.zeros((n, 1 + self.dep_q), np.int32)
        z = np.zeros((n, self.n_embd), np.float32) if want_z else None
        lg = np.zeros((n, self.text_vocab), np.float32) if want_logits else None
        rc = lib().bmo_forward_frame_batch(self._h, n, None if sid is None else sid.ctypes.data,
                                           tokens.ctypes.data, K, pos.ctypes.data,
                                           None if z is None else z.ctypes.data,
                                           None if lg is None else lg.ctypes.data, out.ctypes.data)
        if rc != 0:
            raise RuntimeError(f"bmo_forward_frame_batch rc={rc}: {_err(self._h)}")
        return out[:, 0].copy(), out[:, 1:].copy(), z, lg

    def enqueue_frame_batch(self, n: int, sess_dev_ptr: int, tokens_dev_ptr: int, K: int, pos_dev_ptr: int,
                            out_tokens_dev_ptr: int) -> None:
        rc = lib().bmo_enqueue_frame_batch(self._h, int(n), sess_dev_ptr or None, tokens_dev_ptr, int(K),
                                           pos_dev_ptr, out_tokens_dev_ptr or None)
        if rc != 0:
            raise RuntimeError(f"bmo_enqueue_frame_batch rc={rc}: {_err(self._h)}")

    def batch_kv_import(self, session: int, layer: int, slot0: int, k_rows: np.ndarray, v_rows: np.ndarray) -> None:
        k = np.ascontiguousarray(k_rows, np.float32)
        v = np.ascontiguousarray(v_rows, np.float32)
        rc = lib().bmo_batch_kv_import_f32(self._h, int(session), layer, slot0, k.shape[0],
                                           k.ctypes.data_as(_c_f32p), v.ctypes.data_as(_c_f32p))
        if rc != 0:
            raise RuntimeError(f"bmo_batch_kv_import_f32 rc={rc}: {_err(self._h)}")

    def batch_reset(self, session: int = -1) -> None:
        rc = lib().bmo_batch_reset(self._h, int(session))
        if rc != 0:
            raise RuntimeError(f"bmo_batch_reset rc={rc}: {_err(self._h)}")

    def sync(self) -> None:
        rc = lib().bmo_sync(self._h)
        if rc != 0:
            raise RuntimeError(f"bmo_sync rc={rc}: {_err(self._h)}")

    @property
    def stream(self) -> int:
        return lib().bmo_get_stream(self._h) or 0

    @property
    def device(self) -> int:
        return lib().bmo_get_device(self._h)

    @property
    def device_bytes(self) -> int:
        return lib().bmo_get_device_bytes(self._h)

    def last_error(self) -> Optional[str]:
        e = lib().bmo_last_error(self._h)
        return e.decode() if e else None

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().bmo_free(self._h)
            self._h = None

    def __del__(self):
        # at interpreter shutdown the module globals may already be gone
        try:
            self.close()
        except TypeError:
            pass
