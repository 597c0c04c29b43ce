"""CPU-side checks of libbmo.so: it loads, exports the declared ABI, its
synthetic-data generator and Q4_0 quantiser are exact, and the GGUF files it
writes parse with gguf-py.  Nothing here launches a kernel."""
import ctypes
import os
import re

import numpy as np
import pytest
from gguf import GGMLQuantizationType, GGUFReader, quants

from bmo_jetson_b200 import engine, synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", h) for h in ("bmo_api.h", "bmo_ext.h", "bmo_kernels.h")]

# the reference ABI (utkarshyadav009/bmo_jetson src/bmo_api.h:39-160)
REFERENCE_SYMBOLS = [
    "bmo_init", "bmo_free", "bmo_reset", "bmo_get_n_layers", "bmo_get_n_embd", "bmo_get_n_codebooks",
    "bmo_get_dep_q", "bmo_get_text_vocab", "bmo_get_audio_vocab", "bmo_get_n_attn_heads", "bmo_get_head_dim",
    "bmo_copy_k_cache_f32", "bmo_capture_graphs", "bmo_has_cuda_graphs", "bmo_forward_temporal",
    "bmo_forward_temporal2", "bmo_forward_depth", "bmo_forward_depth_cascade", "bmo_last_error",
    "bmo_rvq_decode", "bmo_rvq_encode",
]


def declared_symbols():
    names = []
    for h in HEADERS:
        text = open(h).read()
        names += re.findall(r"BMO_API\s+[\w\s\*]*?\b(bmo_\w+)\s*\(", text)
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    L = engine.lib()
    declared = declared_symbols()
    assert len(declared) >= 40
    missing = [n for n in declared if not hasattr(L, n)]
    assert not missing, missing


def test_reference_abi_is_a_subset():
    declared = declared_symbols()
    assert set(REFERENCE_SYMBOLS) <= set(declared)


def test_init_without_gpu_fails_loudly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    assert engine.lib().bmo_init(b"/nonexistent.gguf", 512) is None
    with pytest.raises(RuntimeError):
        engine.BMOEngine("/nonexistent.gguf", 512)


def test_null_handle_getters_return_zero():
    L = engine.lib()
    for name in ("bmo_get_n_layers", "bmo_get_n_embd", "bmo_get_n_codebooks", "bmo_get_dep_q",
                 "bmo_get_text_vocab", "bmo_get_audio_vocab", "bmo_get_n_attn_heads", "bmo_get_head_dim",
                 "bmo_has_cuda_graphs"):
        assert getattr(L, name)(None) == 0
    assert L.bmo_capture_graphs(None) == 1
    assert L.bmo_last_error(None) is None
    L.bmo_free(None)
    L.bmo_reset(None)
    assert L.bmo_forward_temporal(None, None, 1, 0, None, None) == 1
    assert L.bmo_forward_depth(None, 0, 0, None, None) == 1
    assert L.bmo_forward_depth_cascade(None, 0, None, 0.0, 0, None) == 1
    assert L.bmo_copy_k_cache_f32(None, 0, 0, 1, None, 1) == -1
    assert L.bmo_rvq_decode(None, None, None, None) == 1
    assert L.bmo_rvq_encode(*([None] * 10)) == 1


@pytest.mark.parametrize("seed", [0, 9])
def test_library_q4_0_quantiser_bit_exact(seed):
    rng = np.random.default_rng(seed)
    x = rng.normal(0, 0.02, (33, 320)).astype(np.float32)
    x[0, :32] = 0.0
    x[1, :32] = -1.0
    x[2, 3] = 1e30
    np.testing.assert_array_equal(synth.quantize_q4_0(x), quants.quantize(x, GGMLQuantizationType.Q4_0))


def test_synth_q4_fill_is_quantised_normal_fill():
    rows, cols = 17, 256
    normals = synth.normal_f32(5, 77, rows * cols, 0.0, 0.02).reshape(rows, cols)
    assert abs(float(normals.std()) - 0.02) < 0.003
    blocks = synth.q4_0_normal(5, 77, rows, cols, 0.02)
    np.testing.assert_array_equal(blocks, quants.quantize(normals, GGMLQuantizationType.Q4_0))
    # deterministic and stream-dependent
    np.testing.assert_array_equal(blocks, synth.q4_0_normal(5, 77, rows, cols, 0.02))
    assert not np.array_equal(blocks, synth.q4_0_normal(5, 78, rows, cols, 0.02))


def test_gguf_writer_round_trip(tiny_model):
    r = GGUFReader(tiny_model)
    by_name = {t.name: t for t in r.tensors}
    cfg = synth.PRESETS["tiny"]
    specs = synth.tensor_specs(cfg)
    assert set(by_name) == {s.name for s in specs}
    qkv = by_name["transformer_layers_0_self_attn_in_proj_weight"]
    assert qkv.tensor_type == GGMLQuantizationType.Q4_0
    assert list(qkv.shape) == [cfg.n_embd, 3 * cfg.n_embd]
    expect = synth.q4_0_normal(cfg.seed, synth._stream_id(qkv.name), 3 * cfg.n_embd, cfg.n_embd, cfg.weight_sigma)
    np.testing.assert_array_equal(np.asarray(qkv.data).reshape(expect.shape), expect)
    assert int(np.asarray(by_name["n_layers"].data)[0]) == cfg.n_layers
    emb = by_name["emb.0.weight"]
    assert emb.tensor_type == GGMLQuantizationType.F16
    assert list(emb.shape) == [cfg.n_embd, cfg.audio_vocab + 1]


def test_cli_arguments_follow_the_reference_harness():
    from bmo_jetson_b200 import cli
    a = cli.parse_args([])
    assert (a.model, a.mode, a.n_iterations, a.layer_begin, a.layer_end, a.debug_dumps) == (
        "bmo_weights.gguf", "depth_cascade", 100, 0, -1, False)
    a = cli.parse_args(["m.gguf", "--mode", "stress_test", "--n-iterations", "5", "--n-threads", "8",
                        "--layer_begin", "2", "--layer_end", "4", "--debug-dumps"])
    assert (a.model, a.mode, a.n_iterations, a.layer_begin, a.layer_end, a.debug_dumps) == (
        "m.gguf", "stress_test", 5, 2, 4, True)
    with pytest.raises(SystemExit):
        cli.parse_args(["--mode", "bogus"])
    with pytest.raises(SystemExit):
        cli.parse_args(["--n-iterations", "-1"])


def test_cli_reports_a_missing_model_and_exits_1(tmp_path, capsys):
    from bmo_jetson_b200 import cli
    assert cli.main([str(tmp_path / "absent.gguf"), "--mode", "depth_cascade"]) == 1
    assert "[bmo_main] ERROR:" in capsys.readouterr().err


def test_oracle_synth_generator_matches_library():
    """The oracle's restatement of the synthetic generator writes the same
    tensors as libbmo's, bit for bit (the CPU-only benchmark arm uses it)."""
    from bmo_jetson_b200 import engine, synth
    from oracle import oracle as orc
    L, O = engine.lib(), orc.lib()
    synth.use_generator(L, "bmo_synth_")
    a = (synth.normal_f32(3, 77, 1001, 0.5, 2.0), synth.f16_normal(3, 78, 999), synth.q4_0_normal(3, 79, 5, 256, 0.02))
    synth.use_generator(O, "orc_synth_")
    try:
        b = (synth.normal_f32(3, 77, 1001, 0.5, 2.0), synth.f16_normal(3, 78, 999), synth.q4_0_normal(3, 79, 5, 256, 0.02))
    finally:
        synth.use_generator(L, "bmo_synth_")
    for x, y in zip(a, b):
        np.testing.assert_array_equal(x.view(np.uint8), y.view(np.uint8))
