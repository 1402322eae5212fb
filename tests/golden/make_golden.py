"""Regenerate tests/golden/*.json from the reference saphira-llm library.

Run in a tree where the reference sources exist (oracle/Makefile builds
oracle/_ref/libsllm_ref.so from them):

    python tests/golden/make_golden.py            # gemv_cases.json, decode_cases.json
    python tests/golden/make_golden.py --large    # decode_large.json (a few minutes)

Every output here comes from the REFERENCE's own functions
(sllm_i2s_quant_act, sllm_i2s_gemv, sllm_i2s_epilogue, sllm_generate_greedy
on a synthetic GGUF loaded by sllm_model_load), never from this project's
code, so the fixtures pin both the oracle restatement and the CUDA backend.
"""
import importlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [ROOT, os.path.join(ROOT, "oracle"), os.path.dirname(HERE)]

import oracle  # noqa: E402
import fixtures  # noqa: E402

synth = importlib.import_module("saphira-llm_b200.synth")


def gemv_case(ref, name, rows, n, seed, x_scale=1.0):
    rng = np.random.default_rng(seed)
    w = synth.random_i2s(rng, rows, n)
    x = (rng.standard_normal(n).astype(np.float32) * np.float32(x_scale)).astype(np.float32)
    q, s, total = ref.quant_act(x)
    dots = ref.gemv(w, rows, n, q)
    ws = np.frombuffer(w[rows * n // 4: rows * n // 4 + 4].tobytes(), np.float32)[0]
    y = np.array([ref.lib.sllm_i2s_epilogue(int(d), total, float(s), float(ws)) for d in dots], np.float32)
    return dict(name=name, rows=rows, n=n, seed=seed, x_scale=x_scale, w_sha256=fixtures.sha(w),
                x_sha256=fixtures.sha(x), act_scale_bits=int(np.float32(s).view(np.uint32)), act_sum=total,
                dots=dots.tolist(), y_bits=y.view(np.uint32).tolist())


def decode_case(ref, name, cfg_kw, seed, n_prompt, n_new, n_ctx):
    cfg = synth.small_config(**cfg_kw)
    m = synth.SynthModel(cfg, seed=seed)
    prompt = np.random.default_rng(seed + 1).integers(0, cfg.n_vocab, n_prompt).astype(np.int32)
    rm = ref.model(m.image, n_ctx, 4)
    rc, toks = rm.generate(prompt, n_new)
    assert rc == 0
    last = rm.last_logits(cfg.n_vocab)
    return dict(name=name, config=cfg_kw, seed=seed, n_ctx=n_ctx, prompt=prompt.tolist(), n_new=n_new,
                image_sha256=fixtures.sha(m.image), tokens=toks.tolist(),
                last_logits_fnv=fixtures.fnv1a64(last.view(np.uint32).tobytes()))


def large_decode_case(ref, name, cfg_kw, seed, prompt_seed, n_prompt, n_new, n_ctx, threads):
    """A decode at a BASELINE configuration's full geometry. The model image is
    too large to hash whole on every test run, so its first and last 16 MiB
    are hashed instead (any drift of the seeded generator changes both)."""
    cfg = synth.Config(**cfg_kw)
    m = synth.SynthModel(cfg, seed=seed)
    prompt = np.random.default_rng(prompt_seed).integers(0, cfg.n_vocab, n_prompt).astype(np.int32)
    rm = ref.model(m.image, n_ctx, threads)
    rc, toks = rm.generate(prompt, n_new)
    assert rc == 0
    last = rm.last_logits(cfg.n_vocab)
    return dict(name=name, config=cfg_kw, seed=seed, prompt_seed=prompt_seed, n_ctx=n_ctx,
                prompt=prompt.tolist(), n_new=n_new, image_bytes=int(m.image.nbytes),
                image_probe_sha256=fixtures.probe_sha(m.image), tokens=toks.tolist(),
                last_logits_fnv=fixtures.fnv1a64(last.view(np.uint32).tobytes()))


def make_large(ref):
    """decode_large.json: configs[2] exactly as stated (the 2B-4T geometry with
    30 layers, 64-token prompt, 256 greedy tokens, 320 positions; the model
    and prompt seeds bench.py's decode leg uses), and configs[4]'s geometry
    (n_embd 8192, n_ff 28672, 64 query / 8 kv heads) with 2 layers and a small
    vocabulary, which the reference's loader accepts (80 layers it refuses)."""
    threads = os.cpu_count() or 1
    cases = [
        large_decode_case(ref, "configs2-2b4t-30l-64+256", {}, 4242, 7, 64, 256, 320, threads),
        large_decode_case(ref, "configs4-geometry-2l",
                          dict(n_layer=2, n_embd=8192, n_ff=28672, n_head=64, n_head_kv=8, n_vocab=4099),
                          4343, 8, 24, 24, 64, threads),
    ]
    with open(os.path.join(HERE, "decode_large.json"), "w") as f:
        json.dump(cases, f, indent=1)
    print("wrote", len(cases), "large decode cases")


def main():
    oracle.build(ref=True)
    if "--large" in sys.argv:
        make_large(oracle.Reference())
        return
    ref = oracle.Reference()
    gemv = [
        gemv_case(ref, "q-rows-2560", 40, 2560, 101),
        gemv_case(ref, "down-rows-6912", 24, 6912, 102),
        gemv_case(ref, "k128", 33, 128, 103, x_scale=1e-3),
        gemv_case(ref, "wide-8192", 8, 8192, 104, x_scale=50.0),
    ]
    decode = [
        decode_case(ref, "tiny-3l", dict(n_layer=3, n_embd=256, n_ff=512, n_head=2, n_head_kv=1, n_vocab=1000),
                    21, 13, 24, 48),
        decode_case(ref, "gqa-2l", dict(n_layer=2, n_embd=512, n_ff=1536, n_head=4, n_head_kv=2, n_vocab=5003),
                    22, 11, 16, 40),
    ]
    with open(os.path.join(HERE, "gemv_cases.json"), "w") as f:
        json.dump(gemv, f)
    with open(os.path.join(HERE, "decode_cases.json"), "w") as f:
        json.dump(decode, f, indent=1)
    print("wrote", len(gemv), "gemv cases and", len(decode), "decode cases")


if __name__ == "__main__":
    main()
