"""Loaders for the committed golden fixtures in tests/golden/.

The fixtures hold outputs of the reference saphira-llm library (compiled from
its own sources, oracle/_ref) on seeded synthetic inputs; the inputs are
regenerated here from their seeds and checked against stored SHA-256 digests,
so a drift in the generator is reported as such rather than as a parity
failure. tests/golden/make_golden.py writes them.
"""
import hashlib
import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def fnv1a64(data: bytes) -> str:
    """FNV-1a 64 (the hash saphira-llm's golden files use, tests/test_i2s.c:41-48)."""
    h = 0xCBF29CE484222325
    arr = np.frombuffer(data, np.uint8)
    # vectorised in blocks would change nothing; keep it plain and exact
    for b in arr.tobytes():
        h ^= b
        h = (h * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return f"{h:016x}"


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def probe_sha(image) -> str:
    """SHA-256 of the first and last 16 MiB of a model image: enough to show
    that a seeded generator still produces the bytes a fixture was made from,
    without hashing a 1.2 GB image on every run."""
    a = np.ascontiguousarray(image).view(np.uint8)
    k = 16 << 20
    return hashlib.sha256(a[:k].tobytes() + a[-k:].tobytes()).hexdigest()


def load_large_decode_cases():
    with open(os.path.join(GOLDEN, "decode_large.json")) as f:
        return {c["name"]: c for c in json.load(f)}


def large_decode_model(synth, case):
    cfg = synth.Config(**case["config"])
    m = synth.SynthModel(cfg, seed=case["seed"])
    assert m.image.nbytes == case["image_bytes"], f"{case['name']}: model size drifted"
    assert probe_sha(m.image) == case["image_probe_sha256"], f"{case['name']}: model generator drifted"
    return m


def gemv_inputs(synth, case):
    rng = np.random.default_rng(case["seed"])
    w = synth.random_i2s(rng, case["rows"], case["n"])
    x = (rng.standard_normal(case["n"]).astype(np.float32) * np.float32(case.get("x_scale", 1.0))).astype(np.float32)
    assert sha(w) == case["w_sha256"], f"{case['name']}: weight generator drifted"
    assert sha(x) == case["x_sha256"], f"{case['name']}: activation generator drifted"
    return w, x


def load_gemv_cases():
    with open(os.path.join(GOLDEN, "gemv_cases.json")) as f:
        cases = json.load(f)
    for c in cases:
        c["dots"] = np.array(c["dots"], np.int32)
        c["y_bits"] = np.array(c["y_bits"], np.uint32)
    return cases


def load_decode_cases():
    with open(os.path.join(GOLDEN, "decode_cases.json")) as f:
        return json.load(f)


def decode_model(synth, case):
    cfg = synth.small_config(**case["config"])
    m = synth.SynthModel(cfg, seed=case["seed"])
    assert sha(m.image) == case["image_sha256"], f"{case['name']}: model generator drifted"
    return m
