"""Benchmark: Moshi decode frames/s at batch 1 on B200 (workload configs 2 + 3).

One step = one decode frame: the 32-layer temporal transformer (d 4096,
32x128 heads, FFN 11264, Q4_0) at the next position, its 32000-way text head
and greedy text token, then the 8-step depformer cascade (6 layers, d 1024,
greedy audio tokens).  The 512-slot KV ring of every layer is pre-filled
with 512 seeded prior positions and decoding starts at position 700, so the
ring has wrapped.  Weights (4.1 GB) exceed L2 (126 MB), so every frame
streams them from HBM.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

`value`: frames/s with inputs resident in HBM (device token buffers, one
CUDA graph per frame, CUDA events on the engine's stream, max over ranks).
`e2e`: the same frames through the reference C ABI (bmo_forward_temporal +
host argmax + bmo_forward_depth_cascade) with host buffers, wall clock.
With N GPUs (torchrun), every rank runs its own session on its own GPU
(data-parallel sessions, no collective): weak scaling.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

N_CTX = 512
START_POS = 700
HBM_FALLBACK_GBS = 6650.0


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return HBM_FALLBACK_GBS, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu = gpu_id
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.3)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for name, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def smi_id(local: int) -> str:
    """nvidia-smi id of CUDA device `local` (its UUID; CUDA and nvidia-smi
    indices differ under CUDA_VISIBLE_DEVICES)."""
    try:
        import torch
        u = str(torch.cuda.get_device_properties(local).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        return str(local)


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def init_dist(world, local, backend=None):
    """One process group per run: NCCL over the GPUs, or gloo on the host
    (backend="gloo", or BMO_DIST_BACKEND=gloo) for the host-side logic."""
    if world <= 1:
        return None
    import datetime

    import torch
    import torch.distributed as dist
    backend = backend or os.environ.get("BMO_DIST_BACKEND", "nccl")
    if backend == "nccl":
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    else:
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120))
    return dist


def _dist_device(dist):
    return "cuda" if dist.get_backend() == "nccl" else "cpu"


def barrier(dist):
    if dist is not None:
        dist.barrier()


def reduce_max(dist, v):
    """The maximum of v over the ranks (every rank gets it)."""
    if dist is None:
        return v
    import torch
    t = torch.tensor([float(v)], device=_dist_device(dist))
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def broadcast_bytes(dist, data, n, src=0):
    """Rank src's n bytes `data` on every rank (the tensor-parallel group id)."""
    if dist is None:
        return bytes(data)
    import torch
    t = torch.zeros(n, dtype=torch.uint8)
    if dist.get_rank() == src:
        t = torch.frombuffer(bytearray(data), dtype=torch.uint8).clone()
    t = t.to(_dist_device(dist))
    dist.broadcast(t, src)
    return bytes(t.cpu().numpy())


def whole_job_rate(dist, world, ms_local):
    """Frames/s of the whole job: every rank's frames over the slowest rank's
    time (max over ranks), and that time."""
    ms = reduce_max(dist, ms_local)
    return world * 1000.0 / ms, ms


def prepare_model(rank, dist):
    from bmo_jetson_b200 import synth
    d = os.environ.get("BMO_MODEL_DIR") or os.path.join(os.environ.get("TMPDIR", "/tmp"), "bmo_models")
    if rank == 0:
        t0 = time.time()
        path = synth.ensure_model("config2", d)
        sys.stderr.write(f"[bench] model ready in {time.time() - t0:.1f}s: {path}\n")
    barrier(dist)
    return synth.ensure_model("config2", d)


def frame_tokens(n, K, text_vocab, audio_vocab, seed=1):
    rng = np.random.default_rng(seed)
    t = np.empty((n, K), np.int32)
    t[:, 0] = rng.integers(0, text_vocab, n)
    t[:, 1:] = rng.integers(0, audio_vocab, (n, K - 1))
    return t


def fill_history(e, seed=7):
    """512 seeded prior positions of N(0,1) K/V in every layer's ring."""
    rng = np.random.default_rng(seed)
    width = e.n_kv_heads * e.head_dim
    for layer in range(e.n_layers):
        k = rng.standard_normal((N_CTX, width), dtype=np.float32)
        v = rng.standard_normal((N_CTX, width), dtype=np.float32)
        e.kv_import(layer, 0, k, v)


def frame_bytes(e):
    """Algorithmic HBM bytes of one frame: Q4_0 weights streamed once, the KV
    window read once, activations negligible."""
    d, F, V = e.n_embd, 11264, e.text_vocab
    q4 = lambda r, c: r * c // 32 * 18
    per_layer = q4(3 * d, d) + q4(d, d) + q4(2 * F, d) + q4(d, F)
    temporal = e.n_layers * per_layer + q4(V, d)
    D, DF = 1024, 2816
    dep_step = q4(D, d) + 6 * (q4(3 * D, D) + q4(D, D) + q4(2 * DF, D) + q4(D, DF)) + q4(2048, D)
    kv_elem = 2 if e.kv_type == 0 else 18 / 32
    kv = 2 * e.n_layers * e.n_kv_heads * N_CTX * e.head_dim * kv_elem
    return temporal + 8 * dep_step + kv, temporal, 8 * dep_step, kv


def gemv_roofline(local, peak_gbs, iters=40, exact=False):
    """Times the dominant kernel of the default path (the reference-order Q4_0
    GEMV, FFN-in shape 22528x4096 with the fused RMSNorm + SwiGLU) on resident buffers: 8 distinct weight copies
    (415 MB > L2) rotated per launch, `iters` back-to-back launches captured in
    one CUDA graph (as the decode frame runs them), CUDA events on the
    replaying stream.  The same launches issued one by one from the host are
    reported beside it (`eager_us_per_launch`).  exact=True times the
    exact-order GEMV (bmo_k_gemv_q4_0, double sums) on the same shape."""
    import torch
    from bmo_jetson_b200 import engine
    L = engine.lib()
    rows, cols, F = 22528, 4096, 11264
    dev = torch.device("cuda", local)
    s = torch.cuda.current_stream(dev)
    nbytes = L.bmo_k_q4_0_tiled_bytes(rows, cols, 1, F)
    mats = [torch.randint(0, 255, (nbytes,), dtype=torch.uint8, device=dev) for _ in range(8)]
    for m in mats:  # sane fp16 scales: 0x2000 ~ 0.0078
        m.view(-1, 4608)[:, 4096:].fill_(0x20)
    x = torch.randn(cols, device=dev)
    g = torch.ones(cols, device=dev)
    y = torch.empty(F, device=dev)
    sbytes = L.bmo_k_gemv_scratch_bytes(rows, cols, 1, F)
    scratch = torch.zeros(max(sbytes, 1), dtype=torch.uint8, device=dev)

    def launch(i, st):
        if exact:
            rc = L.bmo_k_gemv_q4_0(mats[i % 8].data_ptr(), rows, cols, 1, F, x.data_ptr(), g.data_ptr(), 1e-8, None,
                                   y.data_ptr(), None, None, scratch.data_ptr(), sbytes, 0, st.cuda_stream)
        else:
            rc = L.bmo_k_gemv_q4_0_ref(mats[i % 8].data_ptr(), rows, cols, 1, F, x.data_ptr(), g.data_ptr(), 1e-8,
                                       None, y.data_ptr(), None, None, None, st.cuda_stream)
        assert rc == 0, rc

    for i in range(8):
        launch(i, s)
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(s)
    for i in range(iters):
        launch(i, s)
    b.record(s)
    torch.cuda.synchronize(dev)
    eager_ms = a.elapsed_time(b) / iters
    graph = torch.cuda.CUDAGraph()
    cs = torch.cuda.Stream(dev)
    with torch.cuda.graph(graph, stream=cs):
        for i in range(iters):
            launch(i, cs)
    graph.replay()
    torch.cuda.synchronize(dev)
    a.record(s)
    graph.replay()
    b.record(s)
    torch.cuda.synchronize(dev)
    ms = a.elapsed_time(b) / iters
    del graph
    alg = rows * cols // 32 * 18 + cols * 4 * 2 + F * 4
    achieved = alg / (ms * 1e-3) / 1e9
    name = ("gemv_q4_kernel<kProNorm,kEpiSwiGLU> (FFN-in 22528x4096 Q4_0, exact order" if exact else
            "gemv_ref_kernel<kProNorm,kEpiSwiGLU> (FFN-in 22528x4096 Q4_0 in the reference's fp32 order")
    return {"kernel": name + ", fused RMSNorm+Q8_1, SwiGLU)",
            "bytes_per_launch": alg, "us_per_launch": ms * 1e3, "achieved_gbs": achieved,
            "eager_us_per_launch": eager_ms * 1e3, "timing": f"{iters} launches in one CUDA graph, weights rotated "
                                                           "over 8 copies (415 MB > L2)"}


def dep_gemv_timing(local, peak_gbs, iters=40, copies=48):
    """--kernel dep_ffn_in: a depformer GEMV alone, the FFN-in of one step
    (5632x1024 Q4_0, fused RMSNorm + SwiGLU, reference order) through
    bmo_k_gemv_q4_0_ref, weights rotated over `copies` copies (156 MB > L2)
    so each launch streams its 3.2 MB from HBM; CUDA events around `iters`
    back-to-back launches, eager and captured in one CUDA graph."""
    import torch
    from bmo_jetson_b200 import engine
    L = engine.lib()
    rows, cols, F = 5632, 1024, 2816
    dev = torch.device("cuda", local)
    s = torch.cuda.current_stream(dev)
    nbytes = L.bmo_k_q4_0_tiled_bytes(rows, cols, 1, F)
    mats = [torch.randint(0, 255, (nbytes,), dtype=torch.uint8, device=dev) for _ in range(copies)]
    for m in mats:  # sane fp16 scales: 0x2000 ~ 0.0078
        m.view(-1, 4608)[:, 4096:].fill_(0x20)
    x = torch.randn(cols, device=dev)
    g = torch.ones(cols, device=dev)
    y = torch.empty(F, device=dev)

    def launch(i, st):
        rc = L.bmo_k_gemv_q4_0_ref(mats[i % copies].data_ptr(), rows, cols, 1, F, x.data_ptr(), g.data_ptr(), 1e-8,
                                   None, y.data_ptr(), None, None, None, st.cuda_stream)
        assert rc == 0, rc

    for i in range(copies):
        launch(i, s)
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(s)
    for i in range(iters):
        launch(i, s)
    b.record(s)
    torch.cuda.synchronize(dev)
    eager_ms = a.elapsed_time(b) / iters
    graph = torch.cuda.CUDAGraph()
    cs = torch.cuda.Stream(dev)
    with torch.cuda.graph(graph, stream=cs):
        for i in range(iters):
            launch(i, cs)
    graph.replay()
    torch.cuda.synchronize(dev)
    a.record(s)
    graph.replay()
    b.record(s)
    torch.cuda.synchronize(dev)
    ms = a.elapsed_time(b) / iters
    del graph
    alg = rows * cols // 32 * 18 + cols * 4 * 2 + F * 4
    return {"kernel": "gemv_ref_kernel<kProNorm,kEpiSwiGLU> (depformer FFN-in 5632x1024 Q4_0, reference order, "
                      "fused RMSNorm+Q8_1, SwiGLU)",
            "bytes_per_launch": alg, "us_per_launch": ms * 1e3, "achieved_gbs": alg / (ms * 1e-3) / 1e9,
            "frac": alg / (ms * 1e-3) / 1e9 / peak_gbs, "eager_us_per_launch": eager_ms * 1e3,
            "timing": f"{iters} launches in one CUDA graph, weights rotated over {copies} copies (156 MB > L2)"}


def batch_gemm_timing(local, peak_gbs, iters=20, sessions=64):
    """--kernel batch_qkv: one batched GEMM through the kernel-level entry point
    bmo_k_batch_gemm_q4_0 (tensor cores, exact form) on the temporal QKV shape
    12288x4096 with the RMSNorm prologue, `sessions` sessions, weights rotated
    over 8 copies (226 MB > L2) so each launch streams its weights from HBM;
    CUDA events around `iters` back-to-back launches on the launching stream.
    Each call is a stage kernel (norm + Q8_1 of every session) and the GEMM."""
    import torch
    from bmo_jetson_b200 import engine
    L = engine.lib()
    rows, cols = 12288, 4096
    dev = torch.device("cuda", local)
    s = torch.cuda.current_stream(dev)
    nbytes = L.bmo_k_q4_0_tiled_bytes(rows, cols, 0, 0)
    mats = [torch.randint(0, 255, (nbytes,), dtype=torch.uint8, device=dev) for _ in range(8)]
    for m in mats:  # sane fp16 scales: 0x2000 ~ 0.0078
        m.view(-1, 4608)[:, 4096:].fill_(0x20)
    x = torch.randn(sessions, cols, device=dev)
    g = torch.ones(cols, device=dev)
    y = torch.empty(sessions, rows, device=dev)
    sbytes = L.bmo_k_batch_gemm_scratch_bytes(rows, cols, 0, 0, sessions)
    scratch = torch.zeros(max(sbytes, 1), dtype=torch.uint8, device=dev)

    def launch(i):
        rc = L.bmo_k_batch_gemm_q4_0(mats[i % 8].data_ptr(), rows, cols, 0, 0, x.data_ptr(), g.data_ptr(), 1e-8,
                                     None, y.data_ptr(), sessions, 1, scratch.data_ptr(), sbytes, s.cuda_stream)
        assert rc == 0, rc

    for i in range(8):
        launch(i)
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(s)
    for i in range(iters):
        launch(i)
    b.record(s)
    torch.cuda.synchronize(dev)
    ms = a.elapsed_time(b) / iters
    alg = rows * cols // 32 * 18 + sessions * (cols + rows) * 4 + cols * 4
    return {"kernel": f"batch_stage_kernel + batch_mma_kernel (QKV 12288x4096 Q4_0, {sessions} sessions, "
                      "tensor cores, exact form, RMSNorm prologue)",
            "bytes_per_launch": alg, "us_per_launch": ms * 1e3, "achieved_gbs": alg / (ms * 1e-3) / 1e9,
            "frac": alg / (ms * 1e-3) / 1e9 / peak_gbs,
            "timing": f"{iters} eager launches, weights rotated over 8 copies (226 MB > L2)"}


def attn_ref_timing(local, peak_gbs, iters=20, n_layers=32):
    """--kernel attn_ref: the default path's temporal decode attention through
    bmo_k_decode_attention_ref (32 heads x 128, fp16 ring of 512 slots, pos
    700 so the ring has wrapped), the layer rotated over `n_layers` rings
    (268 MB > L2) so each launch reads its K/V window from HBM; CUDA events
    around `iters` back-to-back launches on the launching stream."""
    import torch
    from bmo_jetson_b200 import engine
    L = engine.lib()
    hd, nh, n_ctx, pos = 128, 32, N_CTX, START_POS
    dev = torch.device("cuda", local)
    s = torch.cuda.current_stream(dev)
    q, k, v = (torch.randn(nh * hd, device=dev) for _ in range(3))
    kc = (0.5 * torch.randn(n_layers * nh * n_ctx * hd, device=dev)).half()
    vc = (0.5 * torch.randn(n_layers * nh * n_ctx * hd, device=dev)).half()
    o = torch.empty(nh * hd, device=dev)
    pos_d = torch.tensor([pos], dtype=torch.int32, device=dev)

    def launch(i):
        rc = L.bmo_k_decode_attention_ref(q.data_ptr(), k.data_ptr(), v.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                          o.data_ptr(), hd, nh, nh, n_ctx, pos_d.data_ptr(), i % n_layers,
                                          s.cuda_stream)
        assert rc == 0, rc

    for i in range(n_layers):
        launch(i)
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(s)
    for i in range(iters):
        launch(i)
    b.record(s)
    torch.cuda.synchronize(dev)
    ms = a.elapsed_time(b) / iters
    alg = 2 * nh * n_ctx * hd * 2 + 4 * nh * hd * 4
    return {"kernel": "attn_ref_kernel<128, 8> (32 heads x 128, fp16 ring of 512 slots, pos 700, reference order)",
            "bytes_per_launch": alg, "us_per_launch": ms * 1e3, "achieved_gbs": alg / (ms * 1e-3) / 1e9,
            "frac": alg / (ms * 1e-3) / 1e9 / peak_gbs,
            "timing": f"{iters} eager launches, layers rotated over {n_layers} rings (268 MB > L2)"}


def bench_batch(path, local, dist, sessions, steps, warmup, rank):
    """Config 4: `sessions` independent sessions on this GPU, each with its own
    512-slot Q4_0 ring, at seeded positions uniform in [0, 3000), stepped
    together (one weight stream per frame for all of them).  Device-resident
    inputs for `value`; host arrays through bmo_forward_frame_batch for e2e."""
    import torch
    from bmo_jetson_b200 import engine
    e = engine.BMOEngine(path, n_ctx=N_CTX, device=local, kv_type=engine.KV_Q4_0)
    e.batch_init(sessions)
    K = e.n_codebooks
    dev = torch.device("cuda", local)
    rng = np.random.default_rng(1000 + rank)
    n = warmup + steps
    pos0 = rng.integers(0, 3000, sessions).astype(np.int32)
    pos = np.stack([pos0 + i for i in range(2 * n + 1)]).astype(np.int32)       # [frame][row]
    toks = np.stack([frame_tokens(sessions, K, e.text_vocab, e.audio_vocab, seed=2000 + 97 * rank + i)
                     for i in range(2 * n + 1)])                                # [frame][row][K]
    pos_d = torch.from_numpy(pos).to(dev)
    toks_d = torch.from_numpy(toks).to(dev)
    out_d = torch.zeros((n, sessions, 1 + e.dep_q), dtype=torch.int32, device=dev)
    stream = torch.cuda.ExternalStream(e.stream, device=dev)
    for i in range(warmup):
        e.enqueue_frame_batch(sessions, 0, toks_d[i].data_ptr(), K, pos_d[i].data_ptr(), out_d[i].data_ptr())
    e.sync()
    barrier(dist)
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for i in range(steps):
        f = warmup + i
        e.enqueue_frame_batch(sessions, 0, toks_d[f].data_ptr(), K, pos_d[f].data_ptr(), out_d[f].data_ptr())
    b.record(stream)
    e.sync()
    torch.cuda.synchronize(dev)
    barrier(dist)
    ms = reduce_max(dist, a.elapsed_time(b) / steps)
    out = out_d.cpu().numpy()
    assert (out[:, :, 0] >= 0).all() and (out[:, :, 0] < e.text_vocab).all()
    # end to end: host tokens and positions in, host tokens out, every frame
    for i in range(min(warmup, 3)):
        e.forward_frame_batch(toks[n + i], pos[n + i])
    barrier(dist)
    t0 = time.perf_counter()
    for i in range(steps):
        e.forward_frame_batch(toks[n + i], pos[n + i])
    e2e_s = reduce_max(dist, time.perf_counter() - t0)
    world = 1 if dist is None else dist.get_world_size()
    # algorithmic bytes: weights once + every session's Q4 KV window (positions advance during the run)
    d, F, V = e.n_embd, 11264, e.text_vocab
    q4 = lambda r, c: r * c // 32 * 18
    w = e.n_layers * (q4(3 * d, d) + q4(d, d) + q4(2 * F, d) + q4(d, F)) + q4(V, d)
    D, DF = 1024, 2816
    w += 8 * (q4(D, d) + 6 * (q4(3 * D, D) + q4(D, D) + q4(2 * DF, D) + q4(D, DF)) + q4(2048, D))
    win = np.minimum(pos[warmup:warmup + steps] + 1, N_CTX).mean(axis=0).sum()
    kv = 2 * e.n_layers * e.n_kv_heads * e.head_dim * 18 / 32 * win
    frame_b = w + kv
    launches = 1 + e.n_layers * 9 + 2 + e.dep_q * (2 + 6 * 9 + 2) + 1
    # bytes bmo_forward_frame_batch moves per frame: its fixed input block (session ids, positions and
    # tokens of up to 64 rows x 64 channels, the channel count; one copy) in, the tokens and status out
    batch_max, max_tokens = 64, 64
    h2d = 4 * (batch_max + batch_max + batch_max * max_tokens + 4)
    d2h = sessions * (1 + e.dep_q) * 4 + 4
    e.close()
    return {"sessions_per_gpu": sessions, "value": world * sessions * 1000.0 / ms, "unit": "frames/s",
            "ms_per_step": ms, "frame_hbm_bytes": frame_b, "weight_bytes": w, "kv_bytes": kv,
            "frame_hbm_gbs": frame_b / (ms * 1e-3) / 1e9,
            "e2e": {"value": world * sessions * steps / e2e_s, "unit": "frames/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "path": "bmo_forward_frame_batch (host arrays), wall clock"},
            "gpu_launches": launches * steps,
            "config": "config4: independent sessions, each a 512-slot Q4_0 ring, positions uniform in [0,3000), "
                      "greedy frame (temporal + text head + 8-step depformer) per session per step"}


def tp_measure(path, dist, rank, world, local, kv, frames, warmup, check_frames=64):
    """Config 5: one session split over the world's GPUs (attention heads and
    FFN columns per rank, the double partial sums of each O-projection and
    FFN-out summed over the ranks -- over peer memory by default, NCCL with
    BMO_TP_P2P=0).  Every rank decodes the same `frames` frames; returns (on
    every rank) frames/s of the single stream, mean/p50/p99 frame times (device
    events per frame, max over ranks) and whether the first `check_frames`
    tokens equal a one-GPU handle's (rank 0 re-decodes them alone; tensor
    parallel computes in the exact-reduction order, so the one-GPU handle does too)."""
    import torch
    from bmo_jetson_b200 import engine
    gid = broadcast_bytes(dist, engine.tp_unique_id() if rank == 0 else b"", 128)
    kv_type = engine.KV_F16 if kv == "f16" else engine.KV_Q4_0
    e = engine.BMOEngine(path, n_ctx=N_CTX, device=local, kv_type=kv_type, tp=(rank, world, gid))
    rng = np.random.default_rng(7)
    width = e.n_kv_heads * e.head_dim
    hist = []
    for layer in range(e.n_layers):  # the same history on every rank, each keeps its heads
        k = rng.standard_normal((N_CTX, width * world), dtype=np.float32)
        v = rng.standard_normal((N_CTX, width * world), dtype=np.float32)
        e.kv_import(layer, 0, k[:, rank * width:(rank + 1) * width], v[:, rank * width:(rank + 1) * width])
        if rank == 0:
            hist.append((k[:, :], v[:, :]))
    assert e.capture_graphs() == 0
    K = e.n_codebooks
    dev = torch.device("cuda", local)
    toks = frame_tokens(warmup + frames, K, e.text_vocab, e.audio_vocab)
    toks_d = torch.from_numpy(toks).to(dev)
    out_d = torch.zeros((warmup + frames, 1 + e.dep_q), dtype=torch.int32, device=dev)
    stream = torch.cuda.ExternalStream(e.stream, device=dev)
    pos = START_POS
    for i in range(warmup):
        e.enqueue_frame(toks_d[i].data_ptr(), K, pos, out_d[i].data_ptr())
        pos += 1
    e.sync()
    barrier(dist)
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(frames + 1)]
    evs[0].record(stream)
    for i in range(frames):
        e.enqueue_frame(toks_d[warmup + i].data_ptr(), K, pos, out_d[warmup + i].data_ptr())
        evs[i + 1].record(stream)
        pos += 1
    e.sync()
    torch.cuda.synchronize(dev)
    per = np.array([evs[i].elapsed_time(evs[i + 1]) for i in range(frames)])
    ms = reduce_max(dist, float(per.mean()))
    p50, p99 = reduce_max(dist, float(np.percentile(per, 50))), reduce_max(dist, float(np.percentile(per, 99)))
    tp_tokens = out_d.cpu().numpy()
    exchange = "NVLink peer memory (IPC-mapped partial buffers, fused sum + residual kernel)" \
        if e.tp_peer_exchange else "NCCL all-reduce"
    e.close()
    barrier(dist)
    equal = None
    if rank == 0 and check_frames > 0:
        n = min(check_frames, warmup + frames)
        one = engine.BMOEngine(path, n_ctx=N_CTX, device=local, kv_type=kv_type, flags=engine.FLAG_EXACT)
        for layer, (k, v) in enumerate(hist):
            one.kv_import(layer, 0, k, v)
        ones = np.zeros((n, 1 + one.dep_q), np.int32)
        for i in range(n):
            one.pos = START_POS + i
            _, _, text, audio = one.forward_frame_greedy(toks[i])
            ones[i, 0], ones[i, 1:] = text, audio
        one.close()
        equal = bool((ones == tp_tokens[:n]).all())
    barrier(dist)
    return {"value": 1000.0 / ms, "unit": "frames/s", "n_gpus": world, "frames": frames, "ms_per_step": ms,
            "p50_ms": p50, "p99_ms": p99, "exchange": exchange, "parallelism": f"tp{world}",
            "tokens_equal_1gpu": equal, "tokens_checked": check_frames,
            "config": "config5: one session, 32-layer temporal + text head + 8-step depformer per frame, heads and "
                      "FFN columns split over the GPUs, one exchange after each O-projection and FFN-out"}


def run_tp(args, rank, world, local):
    """--tp: only the tensor-parallel measurement, as its own JSON line."""
    import torch
    dist = init_dist(world, local)
    torch.cuda.set_device(local)
    path = prepare_model(rank, dist)
    r = tp_measure(path, dist, rank, world, local, args.kv, args.steps, args.warmup)
    if rank == 0:
        print(json.dumps({"metric": "Moshi decode frames/s (B=1, tensor parallel)", "value": r["value"],
                          "unit": "frames/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                          "ms_per_step": r["ms_per_step"], "p50_ms": r["p50_ms"], "p99_ms": r["p99_ms"],
                          "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "impl": "ours",
                          "dtype": "int8 (Q4_0 x Q8_1 integer dot, fp32 scales), double partial sums over ranks",
                          "data": "synthetic: seeded weights, tokens and KV history",
                          "config": {"workload": r["config"], "parallelism": r["parallelism"], "n_ctx": N_CTX,
                                     "start_pos": START_POS, "kv": args.kv, "exchange": r["exchange"]},
                          "tokens_equal_1gpu": r["tokens_equal_1gpu"]}), flush=True)
    if dist is not None:
        dist.destroy_process_group()
    return 0


def traffic_from_profile():
    p = os.path.join(ROOT, "profiles", "gemv_ffn_in_traffic.json")
    try:
        with open(p) as f:
            return float(json.load(f)["dram_bytes_per_launch"])
    except Exception:
        return None


def cpu_baseline(model_path, n_frames=2):
    """The CPU oracle (C restatement of the reference arithmetic, OpenMP on
    all host threads) on `n_frames` full frames of the same workload."""
    from oracle import oracle as orc
    o = orc.OracleModel(model_path, n_ctx=N_CTX)
    threads = os.cpu_count() or 1
    rng = np.random.default_rng(7)
    width = o.n_kv_heads * o.head_dim
    for layer in range(o.n_layers):
        o.kv_import(layer, 0, rng.standard_normal((N_CTX, width), dtype=np.float32),
                    rng.standard_normal((N_CTX, width), dtype=np.float32))
    toks = frame_tokens(n_frames + 1, o.n_codebooks, o.text_vocab, o.audio_vocab)
    z, lg, _ = o.forward_temporal(toks[0], START_POS)  # page in the weights
    t0 = time.perf_counter()
    for i in range(n_frames):
        z, lg, _ = o.forward_temporal(toks[i + 1], START_POS + 1 + i)
        o.depth_cascade_greedy(int(np.argmax(lg)), z)
    dt = time.perf_counter() - t0
    o.close()
    return {"value": n_frames / dt, "unit": "frames/s", "cores": threads, "kind": "port",
            "sample": f"{n_frames} full frames (32-layer temporal + text head + 8-step depformer) of the same "
                      f"model at pos {START_POS + 1}.., oracle in C with OpenMP"}


def ref_kernel_timing(peak_gbs, iters=20, flush_bytes=256 << 20):
    """--ref-kernels: the reference's own CUDA kernels (src/bmo_cuda_kernels.cu,
    compiled unmodified into oracle/_ref) against the kernels of the default
    path, which compute the same results bit for bit, on the temporal layer's
    GEMV shapes, the text head and one layer's decode attention at pos 700 of a
    512-slot fp16 ring.  Each launch alone after a rewrite of a flush buffer
    larger than L2 (weights and caches come from HBM), median of `iters`, CUDA
    events on the launching stream.  Reference GEMV = its Q8_1 quantiser +
    GEMV kernels (launch_gemv_q4_0_q8_1); ours = bmo_k_gemv_q4_0_ref (quantiser
    in the prologue).  Attention: reference launch_decode_attention; ours
    bmo_k_decode_attention_ref (K/V append + attention)."""
    import ctypes
    import torch
    from bmo_jetson_b200 import engine
    from oracle import oracle as orc
    dev = torch.device("cuda:0")
    L, R = engine.lib(), orc.ref_lib()
    s = torch.cuda.current_stream(dev)
    flush = torch.empty(flush_bytes, dtype=torch.uint8, device=dev)
    rng = np.random.default_rng(0)

    def median_us(fn):
        ts = []
        for i in range(iters):
            flush.fill_(i & 0xFF)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(s)
            fn()
            b.record(s)
            b.synchronize()
            ts.append(a.elapsed_time(b) * 1e3)
        return float(np.median(ts))

    out = {"mode": "ref_kernels", "gpu": torch.cuda.get_device_name(dev), "iters": iters,
           "l2_flush_bytes": flush_bytes, "peak_gbs": peak_gbs, "gemv": {}, "attention": {}}
    shapes = {"qkv": (12288, 4096), "o_proj": (4096, 4096), "ffn_in": (22528, 4096), "ffn_out": (4096, 11264),
              "text_head": (32000, 4096)}
    for name, (rows, cols) in shapes.items():
        sys.stderr.write(f"[ref-kernels] {name} {rows}x{cols}\n")
        sys.stderr.flush()
        w = rng.integers(0, 256, (rows, cols // 32, 18), dtype=np.uint8)
        w[:, :, 0], w[:, :, 1] = 0x00, 0x20  # fp16 scale 2^-7
        W = np.ascontiguousarray(w.reshape(-1))
        x = rng.standard_normal(cols, dtype=np.float32)
        ref_us = R.ref_time_gemv_cold(W, x, rows, cols, ctypes.c_void_p(flush.data_ptr()), flush_bytes, iters)
        assert ref_us > 0, "reference GEMV failed"
        sys.stderr.write(f"[ref-kernels]   reference {ref_us:.1f} us\n")
        sys.stderr.flush()
        src = torch.from_numpy(W).to(dev)
        tiled = torch.empty(L.bmo_k_q4_0_tiled_bytes(rows, cols, 0, 0), dtype=torch.uint8, device=dev)
        assert L.bmo_k_repack_q4_0(src.data_ptr(), tiled.data_ptr(), rows, cols, 0, 0, s.cuda_stream) == 0
        del src
        xd = torch.from_numpy(x).to(dev)
        y = torch.empty(rows, device=dev)

        def ours():
            rc = L.bmo_k_gemv_q4_0_ref(tiled.data_ptr(), rows, cols, 0, 0, xd.data_ptr(), None, 1e-8, None,
                                       y.data_ptr(), None, None, None, s.cuda_stream)
            assert rc == 0, rc
        for _ in range(3):
            ours()
        our_us = median_us(ours)
        sys.stderr.write(f"[ref-kernels]   ours {our_us:.1f} us\n")
        sys.stderr.flush()
        alg = rows * cols // 32 * 18 + cols * 4 + rows * 4
        out["gemv"][name] = {"rows": rows, "cols": cols, "bytes": alg, "reference_us": ref_us,
                             "reference_gbs": alg / ref_us / 1e3, "ours_us": our_us, "ours_gbs": alg / our_us / 1e3,
                             "speedup": ref_us / our_us, "ours_frac": alg / our_us / 1e3 / peak_gbs}
        del tiled
    hd, nh, n_ctx, pos = 128, 32, 512, 700
    sys.stderr.write("[ref-kernels] attention\n")
    sys.stderr.flush()
    ref_us = R.ref_time_attention_cold(hd, nh, n_ctx, pos, ctypes.c_void_p(flush.data_ptr()), flush_bytes, iters)
    assert ref_us > 0, "reference attention failed"
    q = torch.zeros(nh * hd, device=dev)
    kc = torch.zeros(nh * n_ctx * hd, dtype=torch.float16, device=dev)
    vc = torch.zeros_like(kc)
    o = torch.empty(nh * hd, device=dev)
    pos_d = torch.tensor([pos], dtype=torch.int32, device=dev)

    def ours_attn():
        rc = L.bmo_k_decode_attention_ref(q.data_ptr(), q.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                          o.data_ptr(), hd, nh, nh, n_ctx, pos_d.data_ptr(), 0, s.cuda_stream)
        assert rc == 0, rc
    for _ in range(3):
        ours_attn()
    our_us = median_us(ours_attn)
    out["attention"] = {"head_dim": hd, "heads": nh, "n_ctx": n_ctx, "pos": pos, "kv_bytes": 2 * nh * n_ctx * hd * 2,
                        "reference_us": ref_us, "ours_us": our_us, "speedup": ref_us / our_us}
    return out


def loop_measure(e, steps, warmup, tokens):
    """The daemon's whole frame (bmo_daemon.cpp:727-816: interleave, temporal
    step, text draw, 8 depformer steps each with its audio draw at the
    daemon's defaults temp 0.7 / top-k 25 and 0.8 / 250, codec input) through
    bmo_loop_run, up to 64 frames per call, wall clock around the calls (the
    host copies of inputs and results included), from frame 0 as the daemon
    starts.  Beside it the same library driven the daemon's way: per frame
    bmo_forward_temporal, the text argmax on the host, then
    bmo_forward_depth_cascade with its host sampler (eight logits round
    trips)."""
    params = (0.7, 25, 0.8, 250)

    def run_loop(sampling):
        e.loop_reset(1337)
        e.loop_run(max(warmup, 3), None, sampling, *params)
        done, t0 = 0, time.perf_counter()
        while done < steps:
            n = min(64, steps - done)
            e.loop_run(n, None, sampling, *params)
            done += n
        return steps / (time.perf_counter() - t0)

    sampled = run_loop(True)
    greedy = run_loop(False)
    e.reset()
    K, pos = e.n_codebooks, 0
    for i in range(max(warmup, 3)):
        e.pos = pos
        z, lg = e.forward_temporal(tokens[i % len(tokens)][:K])
        e.forward_depth_cascade(int(np.argmax(lg[:32000])), z, 0.8, 250)
        pos += 1
    t0 = time.perf_counter()
    for i in range(steps):
        e.pos = pos
        z, lg = e.forward_temporal(tokens[i % len(tokens)][:K])
        e.forward_depth_cascade(int(np.argmax(lg[:32000])), z, 0.8, 250)
        pos += 1
    host = steps / (time.perf_counter() - t0)
    return {"value": sampled, "unit": "frames/s", "greedy_value": greedy,
            "path": "bmo_loop_run (one graph per frame, daemon sampling defaults), wall clock",
            "h2d_bytes_per_step": 60, "d2h_bytes_per_step": 68 + 4,
            "host_driven": {"value": host, "unit": "frames/s",
                            "path": "bmo_forward_temporal + host text argmax + bmo_forward_depth_cascade "
                                    "(host top-k sampling, temp 0.8, top-k 250), wall clock"}}


def workload_config(kv, world):
    """The `config` object both arms print (the same workload, same keys)."""
    return {"workload": "config2+3: 32-layer temporal (d4096, 32x128, FFN 11264) + 32000 text head + greedy 8-step "
                        "depformer (6x d1024) per frame, B=1, one session per GPU",
            "n_ctx": N_CTX, "start_pos": START_POS, "kv": kv,
            "l2": "weights 4.1 GB per frame > 126 MB L2 (no flush needed)",
            "parallelism": f"dp{world} (independent sessions)"}


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU arithmetic (the oracle port, C with
    OpenMP on every host core) on full frames of the same workload.  The model
    file is written with the oracle's copy of the synthetic generator, so this
    process loads no library of the engine."""
    if rank != 0:
        return 0
    cores = os.cpu_count() or 1
    os.environ["OMP_NUM_THREADS"] = str(cores)  # torchrun gives its workers 1
    from bmo_jetson_b200 import synth
    from oracle import oracle as orc
    synth.use_generator(orc.lib(), "orc_synth_")
    d = os.environ.get("BMO_MODEL_DIR") or os.path.join(os.environ.get("TMPDIR", "/tmp"), "bmo_models")
    path = synth.ensure_model("config2", d)
    o = orc.OracleModel(path, n_ctx=N_CTX, threads=cores)
    rng = np.random.default_rng(7)
    width = o.n_kv_heads * o.head_dim
    for layer in range(o.n_layers):
        o.kv_import(layer, 0, rng.standard_normal((N_CTX, width), dtype=np.float32),
                    rng.standard_normal((N_CTX, width), dtype=np.float32))
    toks = frame_tokens(args.warmup + args.steps, o.n_codebooks, o.text_vocab, o.audio_vocab)
    pos = START_POS
    for i in range(args.warmup):
        z, lg, _ = o.forward_temporal(toks[i], pos)
        o.depth_cascade_greedy(int(np.argmax(lg)), z)
        pos += 1
    t0 = time.perf_counter()
    for i in range(args.steps):
        z, lg, _ = o.forward_temporal(toks[args.warmup + i], pos)
        o.depth_cascade_greedy(int(np.argmax(lg)), z)
        pos += 1
    dt = time.perf_counter() - t0
    v = args.steps / dt
    line = {"metric": "Moshi decode frames/s (B=1)", "value": v, "unit": "frames/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "impl": "reference",
            "dtype": "int8 (Q4_0 x Q8_1 integer dot, fp32 scales)",
            "data": "synthetic: seeded N(0,0.02) Q4_0 weights, N(0,1) f16 embeddings, seeded tokens and KV history",
            "config": workload_config("f16", world),
            "cpu_baseline": {"value": v, "unit": "frames/s", "cores": cores, "kind": "port",
                             "sample": f"{args.steps} full frames after {args.warmup} warm-up frames on rank 0 only; "
                                       "the reference's ggml CPU path cannot be built here (llama.cpp not vendored), "
                                       "so this is the C restatement of its arithmetic (oracle/) with OpenMP on "
                                       f"{cores} threads"},
            "e2e": {"value": v, "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    o.close()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--kv", default="f16", choices=["f16", "q4_0"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--kernel-only", action="store_true",
                    help="only the standalone timing of one kernel (profiling); which one: --kernel")
    ap.add_argument("--kernel", default="ffn_in",
                    choices=["ffn_in", "ffn_in_exact", "dep_ffn_in", "batch_qkv", "attn_ref"],
                    help="--kernel-only: FFN-in GEMV in the reference order (default) or the exact order, a "
                         "depformer FFN-in GEMV, the batched 64-session QKV GEMM, or the reference-order temporal "
                         "attention")
    ap.add_argument("--sessions", type=int, default=64,
                    help="config 4: sessions per GPU of the batched measurement (0: skip it)")
    ap.add_argument("--batch-only", action="store_true", help="only the batched-sessions measurement")
    ap.add_argument("--ref-kernels", action="store_true",
                    help="only the per-kernel timing of the reference's CUDA kernels against ours (one GPU)")
    ap.add_argument("--tp", action="store_true",
                    help="config 5: one session tensor-parallel over the --gpus ranks (prints its own line)")
    ap.add_argument("--tp-frames", type=int, default=3000,
                    help="N > 1: frames of the tensor-parallel session measured after the data-parallel one (0: skip)")
    ap.add_argument("--loop-only", action="store_true",
                    help="only the frame loop on the device (bmo_loop_run, daemon sampling) and its host-driven twin")
    ap.add_argument("--profile-frames", type=int, default=0,
                    help="profiling: run --warmup frames then this many device-resident frames, print nothing else")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 0)
    rank, world, local = dist_env()
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.tp:
        return run_tp(args, rank, world, local)

    import torch
    peak, peak_kind = measured_peaks()
    if args.ref_kernels:
        torch.cuda.set_device(local)
        print(json.dumps(ref_kernel_timing(peak, iters=max(args.steps, 5))), flush=True)
        return 0
    if args.kernel_only:
        torch.cuda.set_device(local)
        iters = max(args.steps, 1)
        if args.kernel == "batch_qkv":
            r = batch_gemm_timing(local, peak, iters=iters)
        elif args.kernel == "attn_ref":
            r = attn_ref_timing(local, peak, iters=iters)
        elif args.kernel == "dep_ffn_in":
            r = dep_gemv_timing(local, peak, iters=iters)
        else:
            r = gemv_roofline(local, peak, iters=iters, exact=args.kernel == "ffn_in_exact")
        print(json.dumps(r), flush=True)
        return 0

    dist = init_dist(world, local)
    torch.cuda.set_device(local)
    path = prepare_model(rank, dist)
    if args.batch_only:
        r = bench_batch(path, local, dist, args.sessions, args.steps, args.warmup, rank)
        if rank == 0:
            print(json.dumps(r), flush=True)
        if dist is not None:
            dist.destroy_process_group()
        return 0
    from bmo_jetson_b200 import engine
    kv_type = engine.KV_F16 if args.kv == "f16" else engine.KV_Q4_0
    e = engine.BMOEngine(path, n_ctx=N_CTX, device=local, kv_type=kv_type)
    ref_order = e.ref_order
    fill_history(e)
    assert e.capture_graphs() == 0
    K = e.n_codebooks
    if args.loop_only:
        toks = frame_tokens(max(args.steps, 8), K, e.text_vocab, e.audio_vocab)
        r = loop_measure(e, args.steps, args.warmup, toks)
        e.close()
        if rank == 0:
            print(json.dumps({"loop": r, "steps": args.steps, "warmup": args.warmup,
                              "config": workload_config(args.kv, world)}), flush=True)
        if dist is not None:
            dist.destroy_process_group()
        return 0
    if args.profile_frames > 0:
        n = args.warmup + args.profile_frames
        toks = torch.from_numpy(frame_tokens(n, K, e.text_vocab, e.audio_vocab)).to(torch.device("cuda", local))
        out = torch.zeros((n, 1 + e.dep_q), dtype=torch.int32, device=toks.device)
        for i in range(n):
            e.enqueue_frame(toks[i].data_ptr(), K, START_POS + i, out[i].data_ptr())
        e.sync()
        print(json.dumps({"profile_frames": args.profile_frames, "warmup": args.warmup,
                          "text_tokens": out[:, 0].cpu().tolist()}), flush=True)
        e.close()
        return 0
    n_frames = args.warmup + args.steps
    toks = frame_tokens(2 * n_frames + 2, K, e.text_vocab, e.audio_vocab, seed=1 + rank)
    dev = torch.device("cuda", local)
    toks_d = torch.from_numpy(toks).to(dev)
    out_d = torch.zeros((n_frames, 1 + e.dep_q), dtype=torch.int32, device=dev)
    stream = torch.cuda.ExternalStream(e.stream, device=dev)

    # ---- device-resident frames (value) ----
    pos = START_POS
    for i in range(args.warmup):
        e.enqueue_frame(toks_d[i].data_ptr(), K, pos, out_d[i].data_ptr())
        pos += 1
    e.sync()
    barrier(dist)
    torch.cuda.synchronize(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(smi_id(local)) as clocks:
        ev0.record(stream)
        for i in range(args.steps):
            e.enqueue_frame(toks_d[args.warmup + i].data_ptr(), K, pos, out_d[args.warmup + i].data_ptr())
            pos += 1
        ev1.record(stream)
        e.sync()
        torch.cuda.synchronize(dev)
    barrier(dist)
    ms_local = ev0.elapsed_time(ev1) / args.steps
    value, ms = whole_job_rate(dist, world, ms_local)
    out_tokens = out_d.cpu().numpy()
    assert (out_tokens[:, 0] >= 0).all() and (out_tokens[:, 0] < e.text_vocab).all()

    # ---- end to end through the reference C ABI (e2e) ----
    z = np.empty(e.n_embd, np.float32)
    audio = np.empty(e.dep_q, np.int32)
    for i in range(min(args.warmup, 3)):
        e.pos = pos
        z, lg = e.forward_temporal(toks[n_frames + i])
        e.forward_depth_cascade(int(np.argmax(lg)), z, 0.0, 0)
        pos += 1
    barrier(dist)
    t0 = time.perf_counter()
    for i in range(args.steps):
        e.pos = pos
        z, lg = e.forward_temporal(toks[n_frames + (i % n_frames)])
        audio = e.forward_depth_cascade(int(np.argmax(lg)), z, 0.0, 0)
        pos += 1
    e2e_s = reduce_max(dist, time.perf_counter() - t0)
    e2e_value = world * args.steps / e2e_s
    fin_bytes = 64 * 4 + 16
    h2d = fin_bytes + (fin_bytes + e.n_embd * 4)
    d2h = e.n_embd * 4 + e.text_vocab * 4 + 4 + (1 + 8) * 4 + 4

    # ---- per-part device time: temporal step alone, depformer cascade alone ----
    def timed(fn, n):
        e.sync()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for i in range(n):
            fn(i)
        b.record(stream)
        e.sync()
        return a.elapsed_time(b) / n
    n_part = max(5, min(args.steps, 20))
    temporal_ms = timed(lambda i: e.enqueue_temporal(toks_d[i % n_frames].data_ptr(), K, pos + i), n_part)
    pos += n_part
    depth_ms = timed(lambda i: e.enqueue_cascade(int(out_tokens[i % n_frames, 0])), n_part)

    # ---- roofline of the dominant kernel ----
    rl = gemv_roofline(local, peak)
    total_b, temporal_b, dep_b, kv_b = frame_bytes(e)
    launches_per_frame = e.frame_launches
    loop = loop_measure(e, args.steps, args.warmup, toks) if e.loop_supported else None

    e.close()
    batch = None
    if args.sessions > 0:
        batch = bench_batch(path, local, dist, args.sessions, max(5, min(args.steps, 20)), max(3, min(args.warmup, 3)),
                            rank)
    # N > 1: config 4 as written (64 sessions in total, split over the GPUs)
    # and config 5 (one session tensor-parallel over the GPUs)
    batch_split = tp = None
    if world > 1 and args.sessions > 0 and 64 % world == 0:
        batch_split = bench_batch(path, local, dist, 64 // world, max(5, min(args.steps, 20)),
                                  max(3, min(args.warmup, 3)), rank)
    if world > 1 and args.tp_frames > 0:
        tp = tp_measure(path, dist, rank, world, local, "f16", args.tp_frames, max(args.warmup, 3))

    line = None
    if rank == 0:
        cpu = None
        if not args.no_cpu_baseline and world == 1:
            try:
                cpu = cpu_baseline(path)
            except Exception as ex:  # reported, not fatal
                cpu = {"value": None, "unit": "frames/s", "cores": os.cpu_count(), "kind": "port",
                       "sample": f"failed: {ex}"}
        line = {
            "metric": "Moshi decode frames/s (B=1)", "value": value, "unit": "frames/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "int8 (Q4_0 x Q8_1 integer dot, fp32 scales)",
            "data": "synthetic: seeded N(0,0.02) Q4_0 weights, N(0,1) f16 embeddings, seeded tokens and KV history",
            "config": workload_config(args.kv, world),
            "frame": {"semantics": "reference order" if ref_order else "exact order",
                      "frame_hbm_bytes": total_b, "temporal_bytes": temporal_b, "depformer_bytes": dep_b,
                      "kv_bytes": kv_b, "frame_hbm_gbs": total_b / (ms * 1e-3) / 1e9,
                      "frame_hbm_frac": total_b / (ms * 1e-3) / 1e9 / peak,
                      "temporal_ms": temporal_ms, "depformer_ms": depth_ms,
                      "temporal_hbm_gbs": (temporal_b + kv_b) / (temporal_ms * 1e-3) / 1e9,
                      "temporal_hbm_frac": (temporal_b + kv_b) / (temporal_ms * 1e-3) / 1e9 / peak},
            "roofline": {"bound": "hbm", "achieved": rl["achieved_gbs"], "peak": peak, "unit": "GB/s",
                         "frac": rl["achieved_gbs"] / peak, "traffic": traffic_from_profile(),
                         "kernel": rl["kernel"], "bytes_per_launch": rl["bytes_per_launch"],
                         "us_per_launch": rl["us_per_launch"], "eager_us_per_launch": rl["eager_us_per_launch"],
                         "timing": rl["timing"], "peak_source": peak_kind},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "frames/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "path": "bmo_forward_temporal + host argmax + bmo_forward_depth_cascade (greedy), wall clock"},
            "gpu_launches": launches_per_frame * args.steps,
            "clocks": clocks.summary(),
            "loop": loop,
            "batch": batch,
            "batch_split": batch_split,
            "tp": tp,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
