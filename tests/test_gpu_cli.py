"""The bmo_engine-style harness (python -m bmo_jetson_b200.cli) on a GPU: its
temporal_cascade and depth_cascade dumps equal the same calls made directly on
the engine, and stress_test runs its iterations."""
import os

import numpy as np
import pytest

from bmo_jetson_b200 import cli, engine

pytestmark = pytest.mark.gpu


def test_temporal_cascade_dumps_match_engine(tiny_model, tmp_path, capsys):
    rc = cli.main([tiny_model, "--mode", "temporal_cascade", "--debug-dumps", "--n-ctx", "16",
                   "--out-dir", str(tmp_path)])
    out = capsys.readouterr().out
    assert rc == 0 and "[SUCCESS] Temporal validation cascade completed!" in out
    e = engine.BMOEngine(tiny_model, n_ctx=16)
    x = np.ones(e.n_embd, np.float32)
    for i in range(e.n_layers):
        x = e.forward_layers(x, 0, i, i + 1)
        got = np.fromfile(os.path.join(tmp_path, f"cpp_out_layer_{i}.bin"), np.float32)
        np.testing.assert_array_equal(got, x)
    e.close()


def test_temporal_cascade_layer_range(tiny_model, tmp_path, capsys):
    rc = cli.main([tiny_model, "--mode", "temporal_cascade", "--layer_begin", "1", "--layer_end", "2",
                   "--debug-dumps", "--n-ctx", "16", "--out-dir", str(tmp_path)])
    assert rc == 0
    assert sorted(os.listdir(tmp_path)) == ["cpp_out_layer_1.bin"]


def test_depth_cascade_dump_matches_engine(tiny_model, tmp_path, capsys):
    rc = cli.main([tiny_model, "--mode", "depth_cascade", "--debug-dumps", "--n-ctx", "16", "--out-dir", str(tmp_path)])
    assert rc == 0 and "[SUCCESS] Depth-step 0 validation completed!" in capsys.readouterr().out
    e = engine.BMOEngine(tiny_model, n_ctx=16)
    want = e.forward_depth(0, 0, np.ones(e.n_embd, np.float32), copy=True)
    np.testing.assert_array_equal(np.fromfile(os.path.join(tmp_path, "cpp_depth_out.bin"), np.float32), want)
    e.close()


def test_stress_test_iterations(tiny_model, capsys):
    rc = cli.main([tiny_model, "--mode", "stress_test", "--n-iterations", "3", "--n-ctx", "16"])
    out = capsys.readouterr().out
    assert rc == 0 and "[SUCCESS] Stress test completed!" in out
    assert sum(line.startswith("[stress] iter=") for line in out.splitlines()) == 3
