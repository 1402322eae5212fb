"""bench.py's reference arm on the CPU: the JSON line the round-end driver
reads beside the GPU arm's (same metric, unit and direction; a cpu_baseline
object describing the run; an e2e object with no host-device copies).

The reference arm times the reference's own compiled I2_S projections
(oracle/_ref) on this machine's cores, so this runs without a GPU."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def test_reference_arm_json_line():
    import oracle
    if not oracle.reference_available():
        pytest.skip("oracle/_ref is not built")
    import bench
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                          "--steps", "1", "--warmup", "1"],
                         cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout[-2000:]
    d = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference"
    assert d["metric"] == bench.METRIC
    assert d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert d["n_gpus"] == 1 and d["steps"] == 1
    assert d["value"] > 0
    cb = d["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] >= 1 and cb["sample"]
    assert cb["value"] == d["value"] and cb["unit"] == d["unit"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert d["config"]["workload"] == "layer_projections_2b4t"


def test_headline_algorithmic_bytes():
    """The roofline numerator of the headline: per 2B-4T layer, the seven
    tensors' 2-bit codes with their 32-byte scale tails, each GEMV's input
    and norm vector once, each f32 output once -- 17,636,576 bytes, so
    564,370,432 bytes per step of 32 layer copies."""
    import importlib
    import bench
    synth = importlib.import_module("saphira-llm_b200.synth")
    cfg = synth.Config(n_layer=1, n_vocab=256)
    m = synth.SynthModel(cfg, seed=1)
    E, F, G = cfg.n_embd, cfg.n_ff, cfg.n_embd_gqa
    assert (E, F, G) == (2560, 6912, 640)
    codes = (2 * E * E + 2 * G * E + 3 * F * E) // 4 + 7 * 32
    closed = codes + 2 * 4 * (6 * E + F) + 4 * (3 * E + 2 * G + 2 * F)
    assert bench.projection_bytes(cfg, m) == closed == 17_636_576
    assert bench.projection_bytes(cfg, m) * bench.N_COPIES == 564_370_432
