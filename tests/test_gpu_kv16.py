"""The fp16 KV cache option (sllm_cuda_ctx_new_kv with SLLM_CUDA_KV_F16).

The reference keeps an fp32 cache, so this option has no reference output.
It is pinned instead to the oracle restatement with the same rounding
(every cached K and V value rounded to the nearest half, ties to even, and
widened back exactly; everything else in the reference's order): tokens and
logits bit for bit, on the persistent-engine decode step and on the
per-GEMV step with the standalone attention kernel. Against the fp32 path it
only reports how many greedy tokens agree (the benchmark does the same at
configs[2]'s size)."""
import numpy as np
import pytest

from conftest import bits

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape", [
    dict(n_layer=2, n_embd=256, n_ff=512, n_head=2, n_head_kv=1, n_vocab=1000),      # the engine step
    dict(n_layer=2, n_embd=1024, n_ff=2048, n_head=8, n_head_kv=2, n_vocab=3000),    # per-GEMV kernels
])
def test_kv16_decode_matches_rounded_oracle(cuda, orc, synth, shape):
    cfg = synth.small_config(**shape)
    m = synth.SynthModel(cfg, seed=161)
    model = cuda.Model(m.desc())
    c16 = model.ctx(64, kv_f16=True)
    o16 = orc.ctx(m.desc(), 64, kv_f16=True)
    prompt = np.random.default_rng(161).integers(0, cfg.n_vocab, 9).astype(np.int32)
    rc1, t1 = c16.generate(prompt, 24)
    rc2, t2 = o16.generate(prompt, 24)
    assert rc1 == rc2 == 0
    assert t1.tolist() == t2.tolist()
    assert np.array_equal(bits(c16.last_logits()), bits(o16.last_logits()))
    # the fp32 context of the same model, for the agreement figure only
    c32 = model.ctx(64)
    rc3, t3 = c32.generate(prompt, 24)
    assert rc3 == 0
    agree = int(np.sum(t1 == t3))
    print(f"fp16 KV: {agree}/24 greedy tokens as the fp32 cache's")
    c16.close()
    c32.close()
    model.close()


def test_kv16_state_round_trip(cuda, orc, synth, tmp_path):
    """State files keep f32 values: an f16 context's export widens exactly, so
    saving and loading it into another f16 context continues identically."""
    cfg = synth.small_config(n_layer=2, n_embd=256, n_ff=512, n_head=2, n_head_kv=1, n_vocab=700)
    m = synth.SynthModel(cfg, seed=162)
    model = cuda.Model(m.desc())
    a = model.ctx(40, kv_f16=True)
    prompt = np.arange(3, 12, dtype=np.int32)
    assert a.generate(prompt, 5)[0] == 0
    f = str(tmp_path / "kv16.slkv")
    assert a.state_save(f) == 0
    b = model.ctx(40, kv_f16=True)
    assert b.state_load(f) == 0
    ra = a.generate(np.zeros(0, np.int32), 6)
    rb = b.generate(np.zeros(0, np.int32), 6)
    assert ra[0] == rb[0] == 0 and ra[1].tolist() == rb[1].tolist()
    assert np.array_equal(bits(a.last_logits()), bits(b.last_logits()))
    a.close()
    b.close()
    model.close()


def test_kv16_2b_shape_matches_rounded_oracle(cuda, orc, synth):
    """The 2B-4T widths: the fp16 instance of the engine the benchmark runs."""
    cfg = synth.Config(n_layer=2)
    m = synth.SynthModel(cfg, seed=2024)
    model = cuda.Model(m.desc())
    c16 = model.ctx(40, kv_f16=True)
    o16 = orc.ctx(m.desc(), 40, kv_f16=True)
    prompt = np.random.default_rng(4).integers(0, cfg.n_vocab, 6).astype(np.int32)
    r1, t1 = c16.generate(prompt, 4)
    r2, t2 = o16.generate(prompt, 4)
    assert r1 == r2 == 0 and t1.tolist() == t2.tolist()
    assert np.array_equal(bits(c16.last_logits()), bits(o16.last_logits()))
    c16.close()
    model.close()
