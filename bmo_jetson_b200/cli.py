"""Command-line harness with the modes of the reference's `bmo_engine` binary
(src/main.cpp:47-400), run on this package's engine:

  temporal_cascade  layer i alone (i in [--layer_begin, --layer_end)) at
                    position 0, fed the previous layer's output, starting from
                    a vector of ones (main.cpp:103-155); --debug-dumps writes
                    each layer's output as raw fp32 to cpp_out_layer_<i>.bin
  depth_cascade     depformer step 0 on a temporal output of ones with text
                    token 0 (main.cpp:157-261); --debug-dumps writes its audio
                    logits to cpp_depth_out.bin
  stress_test       --n-iterations times: all temporal layers at position 0 on
                    the running state, then the dep_q depformer steps with
                    token 0 (main.cpp:262-380), printing per-iteration wall
                    time and resident memory

Usage: python -m bmo_jetson_b200.cli model.gguf --mode temporal_cascade
The reference's graph-build and arena diagnostics have no counterpart here
(frames run as captured CUDA graphs); --n-threads is accepted and ignored.
"""
import argparse
import os
import sys
import time

import numpy as np

MODES = ("temporal_cascade", "depth_cascade", "stress_test")


def parse_args(argv=None):
    ap = argparse.ArgumentParser(prog="python -m bmo_jetson_b200.cli", description=__doc__.split("\n\n")[0])
    ap.add_argument("model", nargs="?", default="bmo_weights.gguf", help="GGUF path (default bmo_weights.gguf)")
    ap.add_argument("--mode", default="depth_cascade", choices=MODES)
    ap.add_argument("--n-iterations", type=int, default=100)
    ap.add_argument("--n-threads", type=int, default=32, help="accepted for compatibility; unused")
    ap.add_argument("--layer_begin", type=int, default=0)
    ap.add_argument("--layer_end", type=int, default=-1)
    ap.add_argument("--debug-dumps", action="store_true")
    ap.add_argument("--n-ctx", type=int, default=2048, help="KV ring slots (the reference allocates 2048)")
    ap.add_argument("--device", type=int, default=-1)
    ap.add_argument("--out-dir", default=".", help="where --debug-dumps writes (default: the working directory)")
    a = ap.parse_args(argv)
    if a.n_iterations < 0:
        ap.error("--n-iterations must be >= 0")
    return a


def rss_mb():
    try:
        with open("/proc/self/status") as f:
            for line in f:
                if line.startswith("VmRSS:"):
                    return int(line.split()[1]) // 1024
    except OSError:
        pass
    return 0


def dump(path, arr):
    np.ascontiguousarray(arr, np.float32).tofile(path)
    print(f"[bmo_main] Dumped {path}")


def run(a):
    from bmo_jetson_b200 import engine
    print("[bmo_main] === BMO Forward Pass Test ===")
    print(f"[bmo_main] Loading model from: {a.model}")
    e = engine.BMOEngine(a.model, n_ctx=a.n_ctx, device=a.device)
    print(f"[bmo_main] n_layers={e.n_layers} n_heads={e.n_attn_heads} n_embd={e.n_embd} head_dim={e.head_dim}")
    print(f"[bmo_main] device_bytes = {e.device_bytes / 2**30:.3f} GB")
    e.capture_graphs()
    try:
        if a.mode == "temporal_cascade":
            print("[bmo_main] Running Temporal Cascade...")
            x = np.ones(e.n_embd, np.float32)
            begin = max(0, a.layer_begin)
            end = e.n_layers if a.layer_end < 0 else min(a.layer_end, e.n_layers)
            for i in range(begin, end):
                x = e.forward_layers(x, 0, i, i + 1)
                if not np.isfinite(x).all():
                    raise RuntimeError(f"temporal_cascade: non-finite output at layer {i}")
                if a.debug_dumps:
                    dump(os.path.join(a.out_dir, f"cpp_out_layer_{i}.bin"), x)
            print("[SUCCESS] Temporal validation cascade completed!")
        elif a.mode == "depth_cascade":
            print("[bmo_main] Running Depth Cascade (Step 0)...")
            logits = e.forward_depth(0, 0, np.ones(e.n_embd, np.float32), copy=True)
            if not np.isfinite(logits).all():
                raise RuntimeError("depth_cascade: non-finite logits")
            if a.debug_dumps:
                dump(os.path.join(a.out_dir, "cpp_depth_out.bin"), logits)
            print("[SUCCESS] Depth-step 0 validation completed!")
        else:
            print(f"[bmo_main] Running Stress Test ({a.n_iterations} iterations)...")
            state = np.ones(e.n_embd, np.float32)
            t_loop = time.perf_counter()
            for it in range(a.n_iterations):
                t0 = time.perf_counter()
                state = e.forward_layers(state, 0, 0, e.n_layers)
                t1 = time.perf_counter()
                print(f"[prof] iter={it} phase=temporal compute_ms={(t1 - t0) * 1e3:.3f}", file=sys.stderr)
                for step in range(e.dep_q):
                    t0 = time.perf_counter()
                    e.forward_depth(step, 0, state)
                    print(f"[prof] iter={it} phase=depth step={step} compute_ms={(time.perf_counter() - t0) * 1e3:.3f}",
                          file=sys.stderr)
                now = time.perf_counter()
                print(f"[stress] iter={it + 1} iter_ms={(now - t_loop) * 1e3:.3f} rss_mb={rss_mb()}", flush=True)
                t_loop = now
            print("[SUCCESS] Stress test completed!")
    finally:
        print("[bmo_main] Cleaning up...")
        e.close()
    print("[bmo_main] Test completed successfully!")
    return 0


def main(argv=None):
    a = parse_args(argv)
    try:
        return run(a)
    except Exception as ex:  # the reference prints the error and exits 1
        print(f"[bmo_main] ERROR: {ex}", file=sys.stderr)
        return 1


if __name__ == "__main__":
    sys.exit(main())
