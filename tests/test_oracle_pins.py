"""Pin the oracle restatement (oracle/sllm_oracle.c) before trusting it.

Three sources, in order of authority:
  1. the reference's own golden vectors and known-answer tests
     (tests/golden/i2s-converter.txt, tests/golden/i2s-reference.txt and
     tests/test_i2s.c of saphira-llm);
  2. the reference library compiled from its own sources (oracle/_ref), run
     here on seeded inputs: every kernel and the whole decode chain must agree
     bit for bit;
  3. the committed fixtures under tests/golden/, generated from the compiled
     reference by tests/golden/make_golden.py (these also travel to the GPU).
"""
import json
import os
import struct

import numpy as np
import pytest

import oracle
from conftest import bits

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


# ---------------------------------------------------------------------------
# 1. the reference's own golden vectors and known answers
# ---------------------------------------------------------------------------
def lcg_activation(n):
    """The fixed activation of tests/test_i2s.c:253-264 (seed 0xBEEF01)."""
    rng = 0xBEEF01
    x = np.empty(n, np.float32)
    for i in range(n):
        rng = (rng * 1664525 + 1013904223) & 0xFFFFFFFF
        v = np.float32((rng >> 8) & 0xFFFF) / np.float32(32768.0)
        x[i] = (v - np.float32(1.0)) * np.float32(3.0)
    return x


# tests/golden/i2s-reference.txt (saphira-llm): act_scale / act_sum that the
# quantiser must produce for the fixed activation, captured from upstream.
@pytest.mark.parametrize("n,scale,act_sum", [(2560, "42.3747139", 6643), (6912, "42.3359184", 1818)])
def test_quantiser_matches_upstream_golden_act(orc, n, scale, act_sum):
    q, s, total = orc.quant_act(lcg_activation(n))
    assert s == np.float32(float(scale))
    assert total == act_sum
    assert int(q.astype(np.int64).sum()) == act_sum


def test_epilogue_known_answers(orc):
    # tests/test_i2s.c:431-456
    dots = [0, 1, -1, 1000, -1000, 123456, -123456]
    sums = [0, 5, -5, 0, 0, 77, -77]
    scales = [1.0, 2.0, 0.5, 127.0, 0.007874, 42.0, 3.5]
    ws = [1.0, -1.0, 0.25, 2.16316128, 1.21885478, 2.17397785, 0.5]
    for d, s, a, w in zip(dots, sums, scales, ws):
        post = np.float32(w) / np.float32(a)
        want = np.float32(d - s) * post
        assert bits(orc.epilogue(d, s, a, w)) == bits(want)
    assert orc.epilogue(1000, 100, 1.0, 1.0) == 900.0
    assert orc.epilogue(1000, 0, 1.0, 1.0) == 1000.0


def test_quantiser_known_answers(orc):
    # tests/test_i2s.c:458-483: zero row -> scale 0; max 2 -> scale 63.5 and
    # roundf halves away from zero (127, -64)
    q, s, total = orc.quant_act(np.zeros(256, np.float32))
    assert s == 0.0 and total == 0 and not q.any()
    u = np.array([2.0 if i % 3 == 0 else -1.0 for i in range(256)], np.float32)
    q, s, total = orc.quant_act(u)
    assert s == np.float32(63.5)
    want = np.array([127 if i % 3 == 0 else -64 for i in range(256)], np.int8)
    assert np.array_equal(q, want) and total == int(want.astype(np.int64).sum())


def _converter_cases():
    path = os.path.join(oracle.REFERENCE_DIR, "tests/golden/i2s-converter.txt")
    if not os.path.exists(path):
        return []
    cases = []
    for line in open(path):
        if not line.startswith("case "):
            continue
        parts = [p.split() for p in line.split("|")]
        head = parts[0]
        n, nbytes, scale_hex = int(head[1]), int(head[2]), head[3]
        src = np.array([int(h, 16) for h in head[4:]], np.uint32).astype(np.uint16)
        packed_py = bytes(int(h, 16) for h in parts[3])
        decoded_py = np.array([int(h, 16) for h in parts[4]], np.uint32)
        cases.append((n, nbytes, int(scale_hex, 16), src, packed_py, decoded_py))
    return cases


@pytest.mark.skipif(not _converter_cases(), reason="reference tree with tests/golden/i2s-converter.txt absent")
def test_packer_matches_upstream_converter_golden(orc):
    """All 17 cases of tests/golden/i2s-converter.txt, GGUF-python rule: the
    packed bytes, and the read-back through the layout decoder."""
    for n, nbytes, scale_u, src_bf16, packed_py, decoded_py in _converter_cases():
        src = (src_bf16.astype(np.uint32) << 16).view(np.float32)
        scale = np.uint32(scale_u).view(np.float32)
        dst = np.zeros(n // 4 + 32, np.uint8)
        assert orc.lib.orc_i2s_quantize_scaled_py(src, n, scale, dst) == 0
        assert len(packed_py) == nbytes == dst.size
        assert bytes(dst) == packed_py, f"case n={n}"
        # the recorded read-back is the ternary value of each code
        # (dequantize_row_i2_s's map {-1, 0, 1, 0}), without the scale
        m = np.array([-1.0, 0.0, 1.0, 0.0], np.float32)
        dec = np.array([m[orc.lib.orc_i2s_code(dst, k)] for k in range(n)], np.float32)
        assert np.array_equal(bits(dec), decoded_py), f"case n={n}"


# ---------------------------------------------------------------------------
# 2. against the compiled reference
# ---------------------------------------------------------------------------
def test_quant_act_matches_reference(orc, ref):
    rng = np.random.default_rng(1)
    cases = [rng.standard_normal(n).astype(np.float32) * 3 for n in (1, 7, 128, 2560, 6912, 28672)]
    cases += [np.zeros(300, np.float32),
              np.array([1e-40, -1e-41, 0.0, 3e-41] * 64, np.float32),     # scale overflows to inf
              np.array([np.inf, 1, -2, 0] * 64, np.float32),
              np.array([np.nan, 1, -2, 0] * 64, np.float32),
              np.array([-np.inf, 5, 0, 1e30] * 64, np.float32),
              (np.arange(-254, 255, dtype=np.float32) / 2)]                # exact halves
    for x in cases:
        a, b = orc.quant_act(x), ref.quant_act(x)
        assert np.array_equal(a[0], b[0]) and bits(a[1]) == bits(b[1]) and a[2] == b[2]


@pytest.mark.parametrize("rows,n", [(6912, 2560), (2560, 6912), (640, 2560), (37, 128), (5, 8192), (64, 28672)])
def test_gemv_matches_reference(orc, ref, synth, rows, n):
    rng = np.random.default_rng(rows * 7 + n)
    w = synth.random_i2s(rng, rows, n)
    q, _, _ = orc.quant_act(rng.standard_normal(n).astype(np.float32))
    a = orc.gemv(w, rows, n, q)
    b = ref.gemv(w, rows, n, q)
    assert np.array_equal(a, b)
    # and the scalar oracle of the reference on a few rows
    for r in (0, rows // 2, rows - 1):
        assert a[r] == ref.lib.sllm_i2s_dot_scalar(np.ascontiguousarray(w[r * n // 4:]), q, n)


def test_numpy_packer_matches_reference_layout(orc, ref, synth):
    rng = np.random.default_rng(5)
    rows, n = 9, 640
    codes = rng.integers(0, 3, size=(rows, n)).astype(np.uint8)
    packed = synth.pack_codes(codes)
    assert np.array_equal(synth.unpack_codes(packed, rows, n), codes)
    flat = np.concatenate([packed, np.zeros(32, np.uint8)])
    for k in range(0, rows * n, 97):
        assert ref.lib.sllm_i2s_code(flat, k) == codes.reshape(-1)[k] == orc.lib.orc_i2s_code(flat, k)
    # the reference packer with the GGUF-python rule on ternary*scale floats
    s = np.float32(0.05)
    src = ((codes.astype(np.float32) - 1) * s).reshape(-1)
    dst = np.zeros(rows * n // 4 + 32, np.uint8)
    assert ref.lib.sllm_i2s_quantize_scaled(src, src.size, dst, s, 0) == 0
    assert np.array_equal(dst[: rows * n // 4], packed)


@pytest.mark.parametrize("n", [1, 7, 8, 13, 100, 128, 2560, 6912, 8192, 28672])
def test_vector_ops_match_reference(orc, ref, n):
    rng = np.random.default_rng(n)
    v = (rng.standard_normal(n) * 3).astype(np.float32)
    w = (1 + 0.02 * rng.standard_normal(n)).astype(np.float32)
    assert np.array_equal(bits(orc.rms_norm(v, w, 1e-5)), bits(ref.rms_norm(v, w, 1e-5)))
    assert np.array_equal(bits(orc.rms_norm(v, None, 1e-5)), bits(ref.rms_norm(v, None, 1e-5)))
    assert np.array_equal(bits(orc.softmax(v)), bits(ref.softmax(v)))
    assert np.array_equal(bits(orc.silu(v)), bits(ref.silu(v)))
    if n % 2 == 0 or n == 7:
        for pos in (0, 1, 63, 319, 4095):
            assert np.array_equal(bits(orc.rope(v[:128] if n >= 128 else v, min(n, 128), pos, 500000.0)),
                                  bits(ref.rope(v[:128] if n >= 128 else v, min(n, 128), pos, 500000.0)))
    row = (rng.standard_normal(n) * 0.02).astype(np.float16).view(np.uint16)
    assert bits(orc.dot_f16(row, v)) == bits(ref.dot_f16(row, v))


def test_fp16_conversions(orc, ref):
    """Every f16 bit pattern: the exact conversion (src/quant.c) and the
    embedding's, which halves subnormals (src/forward.c:239-263)."""
    for h in range(0, 65536, 1):
        a = orc.lib.orc_fp16_to_fp32(h)
        b = ref.lib.sllm_fp16_to_fp32(h)
        assert bits(np.float32(a)) == bits(np.float32(b)) or (np.isnan(a) and np.isnan(b))
    assert orc.lib.orc_fp16_to_fp32_embd(0x0001) == np.float32(2.0 ** -25)
    assert orc.lib.orc_fp16_to_fp32_embd(0x8200) == -np.float32(2.0 ** -16)
    assert orc.lib.orc_fp16_to_fp32_embd(0x3c00) == 1.0


@pytest.mark.parametrize("cfg_kw,seed,n_new", [
    (dict(n_layer=3, n_embd=256, n_ff=512, n_head=2, n_head_kv=1, n_vocab=1000), 7, 20),
    (dict(n_layer=2, n_embd=384, n_ff=768, n_head=3, n_head_kv=3, n_vocab=3001), 11, 12),
])
def test_decode_matches_reference(orc, ref, synth, cfg_kw, seed, n_new):
    cfg = synth.small_config(**cfg_kw)
    m = synth.SynthModel(cfg, seed=seed)
    rm = ref.model(m.image, 64, 2)
    oc = orc.ctx(m.desc(), 64)
    prompt = np.random.default_rng(seed).integers(0, cfg.n_vocab, 9).astype(np.int32)
    r1, t1 = rm.generate(prompt, n_new)
    r2, t2 = oc.generate(prompt, n_new)
    assert r1 == r2 == 0 and np.array_equal(t1, t2)
    assert np.array_equal(bits(rm.last_logits(cfg.n_vocab)), bits(oc.last_logits()))
    # continuation with no prompt, then a chunk after a reset
    r1, t1 = rm.generate(np.zeros(0, np.int32), 5)
    r2, t2 = oc.generate(np.zeros(0, np.int32), 5)
    assert r1 == r2 == 0 and np.array_equal(t1, t2)
    rm.reset(); oc.reset()
    r1, a = rm.forward_chunk(prompt, 0, cfg.n_vocab)
    r2, b = oc.forward_chunk(prompt, 0)
    assert r1 == r2 == 0 and np.array_equal(bits(a), bits(b))
    # argument rules (src/forward.c:592-608)
    assert oc.forward_chunk(prompt, 0)[0] == rm.forward_chunk(prompt, 0, cfg.n_vocab)[0] == -1
    assert oc.forward_chunk(np.array([cfg.n_vocab], np.int32), 9)[0] == -1


def test_layer_chain_matches_reference(orc, ref, synth):
    cfg = synth.small_config(n_layer=2, n_embd=512, n_ff=1024, n_head=4, n_head_kv=2, n_vocab=300)
    m = synth.SynthModel(cfg, seed=3)
    d = m.desc()
    x = np.random.default_rng(3).standard_normal(cfg.n_embd).astype(np.float32)
    pool = ref.pool(2)
    xr = x.copy()
    E, F, G = cfg.n_embd, cfg.n_ff, cfg.n_embd_gqa
    scratch = np.zeros(4 * E + 2 * G + 3 * F, np.float32)
    qbuf = np.zeros(max(E, F), np.int8)
    dots = np.zeros(max(E, F), np.int32)
    for layer in range(cfg.n_layer):
        pool.layer_chain(d, layer, xr, scratch, qbuf, dots)
        x = orc.layer_chain(d, layer, x)
        assert np.array_equal(bits(x), bits(xr))


# ---------------------------------------------------------------------------
# 3. the committed fixtures
# ---------------------------------------------------------------------------
def test_oracle_matches_committed_fixtures(orc, synth):
    import fixtures
    for case in fixtures.load_gemv_cases():
        w, x = fixtures.gemv_inputs(synth, case)
        y, d = orc.gemv_f32(w, case["rows"], case["n"], x)
        assert np.array_equal(d, case["dots"]), case["name"]
        assert np.array_equal(bits(y), case["y_bits"]), case["name"]
    for case in fixtures.load_decode_cases():
        m = fixtures.decode_model(synth, case)
        oc = orc.ctx(m.desc(), case["n_ctx"])
        rc, toks = oc.generate(np.array(case["prompt"], np.int32), case["n_new"])
        assert rc == 0 and toks.tolist() == case["tokens"], case["name"]
        assert fixtures.fnv1a64(bits(oc.last_logits()).tobytes()) == case["last_logits_fnv"], case["name"]


def test_fp16_rounding_matches_numpy(orc):
    """The oracle's float -> half conversion (its fp16-KV variant, not part of
    the reference) is IEEE round-to-nearest-even: numpy's astype(float16) on
    every float of a seeded sample, the half boundaries, the subnormal range,
    ties and overflow."""
    rng = np.random.default_rng(5)
    xs = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * np.float32(3.0),
        (rng.standard_normal(5000) * 1e-5).astype(np.float32),
        (rng.standard_normal(5000) * 3e4).astype(np.float32),
        np.array([0.0, -0.0, 65504.0, 65519.996, 65520.0, -65520.0, 1e9, np.inf, -np.inf,
                  2.0 ** -24, 2.0 ** -25, 3 * 2.0 ** -26, 2.0 ** -14, 2.0 ** -14 * 1.00048828125,
                  1.0 + 2.0 ** -11, 1.0 + 3 * 2.0 ** -11, 6.1035156e-05, 5.9604645e-08], np.float32),
    ])
    got = np.array([orc.fp32_to_fp16(v) for v in xs], np.uint16)
    want = xs.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, want)
