"""GPU parity of the model-level C ABI: the decode chain against the oracle
restatement (and, where committed, the reference library's own outputs).

Bar: greedy tokens identical; logits bit-identical (north_star asks for
1e-3 relative; the device reproduces the reference's float order, so the
test demands exact bits and would report the largest relative difference
if that ever broke).
"""
import numpy as np
import pytest

from conftest import bits

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float(np.max(np.abs(a - b) / np.maximum(np.abs(b), 1e-30)))


def _pair(cuda, orc, synth, cfg_kw, seed, n_ctx):
    cfg = synth.small_config(**cfg_kw)
    m = synth.SynthModel(cfg, seed=seed)
    model = cuda.Model(m.desc())
    return cfg, m, model, model.ctx(n_ctx), orc.ctx(m.desc(), n_ctx)


CONFIGS = [
    (dict(n_layer=3, n_embd=256, n_ff=512, n_head=2, n_head_kv=1, n_vocab=1000), 7),
    (dict(n_layer=2, n_embd=512, n_ff=1536, n_head=4, n_head_kv=2, n_vocab=5003), 8),
    (dict(n_layer=2, n_embd=1024, n_ff=2816, n_head=8, n_head_kv=8, n_vocab=777), 9),
]


@pytest.mark.parametrize("cfg_kw,seed", CONFIGS)
def test_greedy_decode_matches_oracle(cuda, orc, synth, cfg_kw, seed):
    cfg, m, model, gc, oc = _pair(cuda, orc, synth, cfg_kw, seed, 96)
    prompt = np.random.default_rng(seed).integers(0, cfg.n_vocab, 13).astype(np.int32)
    r1, t1 = gc.generate(prompt, 40)
    r2, t2 = oc.generate(prompt, 40)
    assert r1 == r2 == 0
    assert t1.tolist() == t2.tolist()
    g, o = gc.last_logits(), oc.last_logits()
    assert np.array_equal(bits(g), bits(o)), f"max rel diff {_rel(g, o)}"
    assert gc.n_past() == oc.n_past() == 53
    # continuation from the last logits, with no prompt (src/forward.c:910-920)
    r1, t1 = gc.generate(np.zeros(0, np.int32), 9)
    r2, t2 = oc.generate(np.zeros(0, np.int32), 9)
    assert r1 == r2 == 0 and t1.tolist() == t2.tolist()


@pytest.mark.parametrize("cfg_kw,seed", CONFIGS[:2])
def test_forward_chunk_logits_bit_exact(cuda, orc, synth, cfg_kw, seed):
    cfg, m, model, gc, oc = _pair(cuda, orc, synth, cfg_kw, seed, 64)
    toks = np.random.default_rng(seed + 5).integers(0, cfg.n_vocab, 17).astype(np.int32)
    r1, lg, am = gc.forward_chunk(toks, 0)
    r2, lo = oc.forward_chunk(toks, 0)
    assert r1 == r2 == 0
    assert np.array_equal(bits(lg), bits(lo)), f"max rel diff {_rel(lg, lo)}"
    assert am.tolist() == [int(np.argmax(r)) for r in lo]
    # a second chunk continues the same sequence
    r1, lg, _ = gc.forward_chunk(toks[:5], 17)
    r2, lo = oc.forward_chunk(toks[:5], 17)
    assert r1 == r2 == 0 and np.array_equal(bits(lg), bits(lo))
    # reset, then the same chunk reproduces the first result exactly
    gc.reset(); oc.reset()
    r1, lg2, _ = gc.forward_chunk(toks, 0)
    r2, lo2 = oc.forward_chunk(toks, 0)
    assert np.array_equal(bits(lg2), bits(lo2))


def test_argument_rules_match_the_reference(cuda, orc, synth):
    cfg, m, model, gc, oc = _pair(cuda, orc, synth, CONFIGS[0][0], 3, 16)
    toks = np.array([1, 2, 3], np.int32)
    assert gc.forward_chunk(toks, 0)[0] == 0
    assert gc.forward_chunk(toks, 0)[0] == -1           # rewinding behind n_past
    assert gc.forward_chunk(toks, 14)[0] == -1          # past n_ctx
    assert gc.forward_chunk(np.array([cfg.n_vocab], np.int32), 3)[0] == -1
    assert gc.generate(toks, 20)[0] == -36              # SLLM_ERR_TOO_LARGE
    gc.reset()
    assert gc.generate(np.zeros(0, np.int32), 2)[0] == -1   # BOS 128000 outside a 1000-token vocabulary


def test_certified_sum_fallback_gives_the_same_bits(cuda, orc, synth):
    """Force every certified f64 sum (RMSNorm mean, softmax normaliser) onto
    its reference-order fallback: outputs must not change."""
    cfg_kw, seed = CONFIGS[0]
    cfg, m, model, gc, oc = _pair(cuda, orc, synth, cfg_kw, seed, 48)
    prompt = np.random.default_rng(seed).integers(0, cfg.n_vocab, 11).astype(np.int32)
    r0, t0 = gc.generate(prompt, 12)
    before = cuda.fallback_count()
    cuda.set_force_fallback(True)
    try:
        fc = model.ctx(48)                               # graph captured with the hook on
        r1, t1 = fc.generate(prompt, 12)
        after = cuda.fallback_count()
        l1 = fc.last_logits()
    finally:
        cuda.set_force_fallback(False)
    r2, t2 = oc.generate(prompt, 12)
    assert r0 == r1 == r2 == 0
    assert t0.tolist() == t1.tolist() == t2.tolist()
    assert np.array_equal(bits(l1), bits(oc.last_logits()))
    assert after > before


def test_committed_reference_decode_fixtures(cuda, synth):
    """Tokens and last-logit hashes produced by the reference library itself."""
    import fixtures
    for case in fixtures.load_decode_cases():
        m = fixtures.decode_model(synth, case)
        model = cuda.Model(m.desc())
        c = model.ctx(case["n_ctx"])
        rc, toks = c.generate(np.array(case["prompt"], np.int32), case["n_new"])
        assert rc == 0 and toks.tolist() == case["tokens"], case["name"]
        assert fixtures.fnv1a64(bits(c.last_logits()).tobytes()) == case["last_logits_fnv"], case["name"]


def test_bitnet_2b_shape_two_layers(cuda, orc, synth):
    """The 2B-4T geometry (E 2560, F 6912, 20/5 heads, 128256-token head) with
    two layers: every GEMV shape and the full lm_head of the real model."""
    cfg = synth.Config(n_layer=2)
    m = synth.SynthModel(cfg, seed=2024)
    model = cuda.Model(m.desc())
    gc, oc = model.ctx(40), orc.ctx(m.desc(), 40)
    prompt = np.random.default_rng(4).integers(0, cfg.n_vocab, 6).astype(np.int32)
    r1, t1 = gc.generate(prompt, 4)
    r2, t2 = oc.generate(prompt, 4)
    assert r1 == r2 == 0 and t1.tolist() == t2.tolist()
    assert np.array_equal(bits(gc.last_logits()), bits(oc.last_logits()))


def test_layer_chain_matches_oracle(cuda, orc, synth):
    cfg = synth.Config(n_layer=3, n_vocab=512)
    m = synth.SynthModel(cfg, seed=77)
    model = cuda.Model(m.desc())
    c = model.ctx(8)
    x = np.random.default_rng(77).standard_normal(cfg.n_embd).astype(np.float32)
    got = c.layer_chain(0, 3, x)
    want = x
    for layer in range(3):
        want = orc.layer_chain(m.desc(), layer, want)
    assert np.array_equal(bits(got), bits(want))


def test_layer_projections_match_oracle(cuda, orc, synth):
    """The seven projections on independent inputs (benchmark configuration
    1): each output equals the oracle's norm -> quant -> GEMV -> epilogue."""
    import importlib
    cfg = synth.Config(n_layer=2, n_vocab=256)
    m = synth.SynthModel(cfg, seed=55)
    model = cuda.Model(m.desc())
    c = model.ctx(8)
    xs_n, ys_n = cuda.projection_sizes(model)
    E, F, G = cfg.n_embd, cfg.n_ff, cfg.n_embd_gqa
    assert xs_n == 6 * E + F and ys_n == 3 * E + 2 * G + 2 * F
    x = np.random.default_rng(5).standard_normal(xs_n).astype(np.float32)
    y = c.layer_projections(0, 2, x)
    specs = [("attn_q", E, E, "attn_norm"), ("attn_k", G, E, "attn_norm"), ("attn_v", G, E, "attn_norm"),
             ("attn_output", E, E, "attn_sub_norm"), ("ffn_gate", F, E, "ffn_norm"),
             ("ffn_up", F, E, "ffn_norm"), ("ffn_down", E, F, "ffn_sub_norm")]
    for il in range(2):
        xo = yo = 0
        for name, rows, n, norm in specs:
            xn = orc.rms_norm(x[xo:xo + n], m.tensors[f"blk.{il}.{norm}.weight"].view(np.float32), cfg.eps)
            want, _ = orc.gemv_f32(m.tensors[f"blk.{il}.{name}.weight"], rows, n, xn)
            assert np.array_equal(bits(y[il, yo:yo + rows]), bits(want)), (il, name)
            xo += n
            yo += rows


def test_layer_projections_in_pieces(cuda, orc, synth):
    """The host-buffer call over 16 or more layers runs the layers as pieces
    whose outputs return while the next piece computes: every layer's outputs
    equal the oracle's and the device entry point's, into pageable and pinned
    host memory, for spans that do not start at layer 0 or divide evenly."""
    import torch
    cfg = synth.small_config(n_layer=20, n_embd=256, n_ff=512, n_head=2, n_head_kv=1, n_vocab=64)
    m = synth.SynthModel(cfg, seed=31)
    model = cuda.Model(m.desc())
    c = model.ctx(8)
    xs_n, ys_n = cuda.projection_sizes(model)
    E, F, G = cfg.n_embd, cfg.n_ff, cfg.n_embd_gqa
    specs = [("attn_q", E, E, "attn_norm"), ("attn_k", G, E, "attn_norm"), ("attn_v", G, E, "attn_norm"),
             ("attn_output", E, E, "attn_sub_norm"), ("ffn_gate", F, E, "ffn_norm"),
             ("ffn_up", F, E, "ffn_norm"), ("ffn_down", E, F, "ffn_sub_norm")]
    x = np.random.default_rng(31).standard_normal(xs_n).astype(np.float32)
    for begin, n in [(0, 20), (3, 17), (0, 16)]:
        y = c.layer_projections(begin, n, x)
        for il in range(n):
            xo = yo = 0
            for name, rows, k, norm in specs:
                xn = orc.rms_norm(x[xo:xo + k], m.tensors[f"blk.{begin + il}.{norm}.weight"].view(np.float32),
                                  cfg.eps)
                want, _ = orc.gemv_f32(m.tensors[f"blk.{begin + il}.{name}.weight"], rows, k, xn)
                assert np.array_equal(bits(y[il, yo:yo + rows]), bits(want)), (begin, il, name)
                xo += k
                yo += rows
        xd = torch.from_numpy(x).cuda()
        yd = torch.empty(n * ys_n, dtype=torch.float32, device="cuda")
        c.layer_projections_device(begin, n, xd, yd)
        torch.cuda.synchronize()
        assert np.array_equal(bits(y.reshape(-1)), bits(yd.cpu().numpy())), (begin, n)
        xp = torch.from_numpy(x).pin_memory()
        yp = torch.full((n * ys_n,), float("nan"), dtype=torch.float32).pin_memory()
        assert cuda.lib().sllm_cuda_layer_projections(model.h, c.h, begin, n, xp.data_ptr(), yp.data_ptr()) == 0
        assert np.array_equal(bits(yp.numpy()), bits(y.reshape(-1))), (begin, n)


@pytest.mark.parametrize("cfg_kw", [
    dict(n_layer=2, n_embd=256, n_ff=512, n_head=2, n_head_kv=1, n_vocab=64),
    dict(n_layer=2, n_embd=1152, n_ff=3072, n_head=9, n_head_kv=3, n_vocab=64),
    dict(n_layer=1, n_embd=8192, n_ff=8192, n_head=64, n_head_kv=8, n_vocab=64),
    dict(n_layer=2, n_embd=640, n_ff=1280, n_head=5, n_head_kv=5, n_vocab=64),   # widths (2, 3): fallback path
])
def test_engine_shapes_chain_and_projections(cuda, orc, synth, cfg_kw):
    """The persistent engine on widths the 2B model does not use (K = 256 to
    8192, odd head counts), for the dependent chain and the projections, and
    the per-GEMV fallback for a width pair the engine is not compiled for."""
    cfg = synth.small_config(**cfg_kw)
    m = synth.SynthModel(cfg, seed=17)
    model = cuda.Model(m.desc())
    c = model.ctx(8)
    x = np.random.default_rng(17).standard_normal(cfg.n_embd).astype(np.float32)
    got = c.layer_chain(0, cfg.n_layer, x)
    want = x
    for layer in range(cfg.n_layer):
        want = orc.layer_chain(m.desc(), layer, want)
    assert np.array_equal(bits(got), bits(want))
    xs_n, ys_n = cuda.projection_sizes(model)
    xp = np.random.default_rng(18).standard_normal(xs_n).astype(np.float32)
    y = c.layer_projections(0, cfg.n_layer, xp)
    E, F, G = cfg.n_embd, cfg.n_ff, cfg.n_embd_gqa
    specs = [("attn_q", E, E, "attn_norm"), ("attn_k", G, E, "attn_norm"), ("attn_v", G, E, "attn_norm"),
             ("attn_output", E, E, "attn_sub_norm"), ("ffn_gate", F, E, "ffn_norm"),
             ("ffn_up", F, E, "ffn_norm"), ("ffn_down", E, F, "ffn_sub_norm")]
    for il in range(cfg.n_layer):
        xo = yo = 0
        for name, rows, n, norm in specs:
            xn = orc.rms_norm(xp[xo:xo + n], m.tensors[f"blk.{il}.{norm}.weight"].view(np.float32), cfg.eps)
            want_y, _ = orc.gemv_f32(m.tensors[f"blk.{il}.{name}.weight"], rows, n, xn)
            assert np.array_equal(bits(y[il, yo:yo + rows]), bits(want_y)), (il, name)
            xo += n
            yo += rows


def test_engine_fallback_path(cuda, orc, synth):
    """The engine's certified-sum fallback gives the same bits."""
    cfg = synth.Config(n_layer=2, n_vocab=64)
    m = synth.SynthModel(cfg, seed=23)
    model = cuda.Model(m.desc())
    x = np.random.default_rng(23).standard_normal(cfg.n_embd).astype(np.float32)
    cuda.set_force_fallback(True)
    try:
        c = model.ctx(8)                  # programs are built (and the hook read) on first use
        before = cuda.fallback_count()
        got = c.layer_chain(0, 2, x)
        after = cuda.fallback_count()
    finally:
        cuda.set_force_fallback(False)
    want = orc.layer_chain(m.desc(), 1, orc.layer_chain(m.desc(), 0, x))
    assert np.array_equal(bits(got), bits(want))
    assert after > before


def test_decode_step_runs_on_the_engine(cuda, orc, synth):
    """The decode step is one engine launch for every layer (attention as a
    stage) between the embedding and the head: 3 kernels per token, and the
    tokens and logits stay the oracle's. (A one-token prompt: longer prompts
    run as chunks on the tensor cores.)"""
    cfg, m, model, gc, oc = _pair(cuda, orc, synth, CONFIGS[1][0], 41, 64)
    prompt = np.random.default_rng(41).integers(0, cfg.n_vocab, 1).astype(np.int32)
    r1, t1 = gc.generate(prompt, 1)           # builds the step graph
    gc.reset()
    k0 = cuda.kernel_launches()
    r1, t1 = gc.generate(prompt, 10)
    per_step = (cuda.kernel_launches() - k0) / (len(prompt) + 10)
    r2, t2 = oc.generate(prompt, 10)
    assert r1 == r2 == 0 and t1.tolist() == t2.tolist()
    assert np.array_equal(bits(gc.last_logits()), bits(oc.last_logits()))
    assert per_step == 3, per_step


def test_chunk_path_long_prompt_and_boundaries(cuda, orc, synth):
    """The multi-token chunk path on the tensor cores: a 300-token prompt
    runs as two chunks (256 + 44), a forward_chunk split at another boundary
    gives the same bits as one chunk, and decoding continues from either,
    all equal to the oracle's one-token-at-a-time order (a chunk is not a
    semantic boundary, src/forward.c:572-588)."""
    cfg = synth.small_config(n_layer=2, n_embd=512, n_ff=1536, n_head=4, n_head_kv=2, n_vocab=2003)
    m = synth.SynthModel(cfg, seed=303)
    model = cuda.Model(m.desc())
    gc, oc = model.ctx(340), orc.ctx(m.desc(), 340)
    prompt = np.random.default_rng(303).integers(0, cfg.n_vocab, 300).astype(np.int32)
    r1, t1 = gc.generate(prompt, 12)
    r2, t2 = oc.generate(prompt, 12)
    assert r1 == r2 == 0 and t1.tolist() == t2.tolist()
    assert np.array_equal(bits(gc.last_logits()), bits(oc.last_logits()))
    # the same 40 tokens as one chunk and as chunks of 23 + 17
    toks = prompt[:40]
    a = model.ctx(64)
    r, la, _ = a.forward_chunk(toks, 0)
    assert r == 0
    b = model.ctx(64)
    r, lb1, _ = b.forward_chunk(toks[:23], 0)
    assert r == 0
    r, lb2, _ = b.forward_chunk(toks[23:], 23)
    assert r == 0
    assert np.array_equal(bits(la), bits(np.concatenate([lb1, lb2])))
    ra, ta = a.generate(np.zeros(0, np.int32), 6)
    rb, tb = b.generate(np.zeros(0, np.int32), 6)
    o2 = orc.ctx(m.desc(), 64)
    ro, lo = o2.forward_chunk(toks, 0)
    ro2, to = o2.generate(np.zeros(0, np.int32), 6)
    assert ra == rb == ro2 == 0 and ta.tolist() == tb.tolist() == to.tolist()
    assert np.array_equal(bits(la), bits(lo))
    for c in (gc, a, b):
        c.close()
    model.close()
