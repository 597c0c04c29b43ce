"""Times the reference's own CUDA kernels (src/bmo_cuda_kernels.cu, compiled
unmodified for sm_100a into oracle/_ref/libbmo_refkernels.so) against this
package's kernels on the same shapes, on one B200.  TEST INFRASTRUCTURE: a
measurement script, not part of the product path.

Every launch is timed alone with CUDA events after a 256 MB rewrite of a flush
buffer (so weights and caches come from HBM, as in a decode frame); the median
of 20 launches is reported.  Work per row:
  GEMV  -- reference: launch_gemv_q4_0_q8_1 (its Q8_1 quantiser + GEMV
           kernels); here: bmo_k_gemv_q4_0 (quantiser fused into the GEMV
           prologue), plain store epilogue; the 7B Moshi shapes of the temporal
           layer and the text head.
  ATTN  -- one layer at pos 700 over a 512-slot fp16 ring, 32 heads x 128:
           reference launch_decode_attention vs bmo_k_decode_attention.
Prints one JSON object.  Run: python tests/ref_kernel_timing.py
"""
import ctypes
import json
import os
import sys

import numpy as np
import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from bmo_jetson_b200 import engine  # noqa: E402
from oracle import oracle as orc  # noqa: E402

PEAK_GBS = 6541.8  # MEASURED_PEAKS.json hbm_gbs on this pool
SHAPES = {"qkv": (12288, 4096), "o_proj": (4096, 4096), "ffn_in": (22528, 4096), "ffn_out": (4096, 11264),
          "text_head": (32000, 4096)}
ITERS = 20
FLUSH = 256 << 20


def median_event_us(fn, flush, stream):
    ts = []
    for i in range(ITERS):
        flush.fill_(i & 0xFF)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        fn()
        b.record(stream)
        b.synchronize()
        ts.append(a.elapsed_time(b) * 1e3)
    return float(np.median(ts))


def ggml_q4_0(rows, cols, rng):
    w = rng.integers(0, 256, (rows, cols // 32, 18), dtype=np.uint8)
    w[:, :, 0], w[:, :, 1] = 0x00, 0x20  # fp16 scale 2^-7
    return np.ascontiguousarray(w.reshape(-1))


def main():
    dev = torch.device("cuda:0")
    L = engine.lib()
    R = orc.ref_lib()
    s = torch.cuda.current_stream(dev)
    flush = torch.empty(FLUSH, dtype=torch.uint8, device=dev)
    rng = np.random.default_rng(0)
    out = {"gpu": torch.cuda.get_device_name(dev), "iters": ITERS, "l2_flush_bytes": FLUSH, "gemv": {}, "attention": {}}
    for name, (rows, cols) in SHAPES.items():
        W = ggml_q4_0(rows, cols, rng)
        x = rng.standard_normal(cols, dtype=np.float32)
        ref_us = R.ref_time_gemv_cold(W, x, rows, cols, ctypes.c_void_p(flush.data_ptr()), FLUSH, ITERS)
        assert ref_us > 0, "reference GEMV failed"
        src = torch.from_numpy(W).to(dev)
        tiled = torch.empty(L.bmo_k_q4_0_tiled_bytes(rows, cols, 0, 0), dtype=torch.uint8, device=dev)
        assert L.bmo_k_repack_q4_0(src.data_ptr(), tiled.data_ptr(), rows, cols, 0, 0, s.cuda_stream) == 0
        del src
        xd = torch.from_numpy(x).to(dev)
        y = torch.empty(rows, device=dev)
        sb = L.bmo_k_gemv_scratch_bytes(rows, cols, 0, 0)
        scratch = torch.zeros(sb, dtype=torch.uint8, device=dev)

        def ours():
            rc = L.bmo_k_gemv_q4_0(tiled.data_ptr(), rows, cols, 0, 0, xd.data_ptr(), None, 1e-8, None, y.data_ptr(),
                                   None, None, scratch.data_ptr(), sb, 0, s.cuda_stream)
            assert rc == 0, rc
        for _ in range(3):
            ours()
        our_us = median_event_us(ours, flush, s)
        alg = rows * cols // 32 * 18 + cols * 4 + rows * 4
        out["gemv"][name] = {"rows": rows, "cols": cols, "bytes": alg,
                             "reference_us": ref_us, "reference_gbs": alg / ref_us / 1e3,
                             "ours_us": our_us, "ours_gbs": alg / our_us / 1e3,
                             "speedup": ref_us / our_us, "ours_frac_of_measured_peak": alg / our_us / 1e3 / PEAK_GBS}
        print(name, json.dumps(out["gemv"][name]), flush=True)
        del tiled, scratch
    # attention, one layer, pos 700, 512-slot fp16 ring
    hd, nh, n_ctx, pos = 128, 32, 512, 700
    ref_us = R.ref_time_attention_cold(hd, nh, n_ctx, pos, ctypes.c_void_p(flush.data_ptr()), FLUSH, ITERS)
    assert ref_us > 0, "reference attention failed"
    q = torch.zeros(nh * hd, device=dev)
    kc = torch.zeros(nh * n_ctx * hd, dtype=torch.float16, device=dev)
    vc = torch.zeros_like(kc)
    o = torch.empty(nh * hd, device=dev)
    pos_d = torch.tensor([pos], dtype=torch.int32, device=dev)

    def ours_attn():
        rc = L.bmo_k_decode_attention(q.data_ptr(), q.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), None, None,
                                      o.data_ptr(), hd, nh, nh, n_ctx, pos_d.data_ptr(), 0, 0, s.cuda_stream)
        assert rc == 0, rc
    for _ in range(3):
        ours_attn()
    our_us = median_event_us(ours_attn, flush, s)
    kv = 2 * nh * n_ctx * hd * 2
    out["attention"] = {"head_dim": hd, "heads": nh, "n_ctx": n_ctx, "pos": pos, "kv_bytes": kv,
                        "reference_us": ref_us, "ours_us": our_us, "speedup": ref_us / our_us}
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
