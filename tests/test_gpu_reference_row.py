"""The CUDA row selected on the reference's side of the boundary: saphira-llm
built with the two insertion-only patches (saphira-llm_b200/reference_row/)
and linked to libsllm_cuda.so, driven through its own public API
(sllm_gguf_open_memory -> sllm_model_load -> sllm_ctx_new ->
sllm_generate_greedy / sllm_forward_chunk / sllm_state_save / _load).

With the CUDA row selected every token and logit must equal the CPU row's,
the device must have done the work (this library's kernel counter moves),
and state files must cross between the rows byte for byte: a file the CUDA
row writes equals the CPU row's for the same history, and each row continues
identically from the other's file."""
import os

import numpy as np
import pytest

import reference_row as rr
from conftest import bits

pytestmark = pytest.mark.gpu

CFG = dict(n_layer=3, n_embd=512, n_ff=1536, n_head=4, n_head_kv=2, n_vocab=5003)


def _row():
    assert rr.available(), "build saphira-llm_b200/reference_row (make REF=<saphira-llm tree>) first"
    return rr.Row()


def _model(synth, seed):
    cfg = synth.small_config(**CFG)
    return cfg, synth.SynthModel(cfg, seed=seed)


def test_cuda_row_matches_cpu_row(cuda, synth):
    row = _row()
    cfg, m = _model(synth, 81)
    V = cfg.n_vocab
    prompt = np.random.default_rng(81).integers(0, V, 9).astype(np.int32)
    g = row.open(m.image, rr.CUDA, 64)
    c = row.open(m.image, rr.CPU, 64)
    assert g.rc == 0 and g.backend() == rr.CUDA
    assert c.rc == 0 and c.backend() == rr.CPU
    k0 = cuda.kernel_launches()
    rc1, t1 = g.generate(prompt, 12)
    assert cuda.kernel_launches() > k0, "the CUDA row ran no kernel of libsllm_cuda.so"
    rc2, t2 = c.generate(prompt, 12)
    assert rc1 == rc2 == 0 and t1.tolist() == t2.tolist()
    assert np.array_equal(bits(g.last_logits(V)), bits(c.last_logits(V)))
    # a chunk through sllm_forward_chunk, every position's logits
    g.reset()
    c.reset()
    rc1, l1 = g.forward_chunk(prompt[:5], 0, V)
    rc2, l2 = c.forward_chunk(prompt[:5], 0, V)
    assert rc1 == rc2 == 0 and np.array_equal(bits(l1), bits(l2))
    # the argument rules are the reference's: a rewind is refused
    rc1, _ = g.forward_chunk(prompt[:2], 1, V)
    rc2, _ = c.forward_chunk(prompt[:2], 1, V)
    assert rc1 == rc2 == -1
    # no prompt: continue from the last logits
    rc1, t1 = g.generate(np.zeros(0, np.int32), 4)
    rc2, t2 = c.generate(np.zeros(0, np.int32), 4)
    assert rc1 == rc2 == 0 and t1.tolist() == t2.tolist()
    g.close()
    c.close()


def test_state_files_cross_between_rows(cuda, synth, tmp_path):
    row = _row()
    cfg, m = _model(synth, 82)
    V = cfg.n_vocab
    prompt = np.random.default_rng(82).integers(0, V, 11).astype(np.int32)
    g = row.open(m.image, rr.CUDA, 48)
    c = row.open(m.image, rr.CPU, 48)
    assert g.rc == 0 and c.rc == 0 and g.backend() == rr.CUDA
    assert g.generate(prompt, 7)[0] == 0 and c.generate(prompt, 7)[0] == 0
    fg, fc = str(tmp_path / "cuda.slkv"), str(tmp_path / "cpu.slkv")
    assert g.save(fg) == 0 and c.save(fc) == 0
    assert open(fg, "rb").read() == open(fc, "rb").read()
    # this library's own writer gives the same bytes
    model = cuda.Model(m.desc())
    nc = model.ctx(48)
    assert nc.generate(prompt, 7)[0] == 0
    fn = str(tmp_path / "native.slkv")
    assert nc.state_save(fn) == 0
    assert open(fn, "rb").read() == open(fc, "rb").read()
    # each row continues from the other's file as it would have itself
    want = c.generate(np.zeros(0, np.int32), 6)
    g2 = row.open(m.image, rr.CUDA, 48)
    c2 = row.open(m.image, rr.CPU, 48)
    assert g2.load(fc) == 0 and c2.load(fg) == 0
    got_g = g2.generate(np.zeros(0, np.int32), 6)
    got_c = c2.generate(np.zeros(0, np.int32), 6)
    nc2 = model.ctx(48)
    assert nc2.state_load(fc) == 0
    got_n = nc2.generate(np.zeros(0, np.int32), 6)
    assert want[0] == got_g[0] == got_c[0] == got_n[0] == 0
    assert want[1].tolist() == got_g[1].tolist() == got_c[1].tolist() == got_n[1].tolist()
    assert np.array_equal(bits(g2.last_logits(V)), bits(c.last_logits(V)))
    for h in (g, c, g2, c2):
        h.close()
    nc.close()
    nc2.close()
    model.close()


def test_state_load_refusals(cuda, synth, tmp_path):
    cfg, m = _model(synth, 83)
    model = cuda.Model(m.desc())
    c = model.ctx(32)
    prompt = np.arange(1, 6, dtype=np.int32)
    assert c.generate(prompt, 3)[0] == 0
    f = str(tmp_path / "s.slkv")
    assert c.state_save(f) == 0
    data = open(f, "rb").read()
    bad = str(tmp_path / "bad.slkv")
    open(bad, "wb").write(b"XXXX" + data[4:])
    assert c.state_load(bad) == -32                       # SLLM_ERR_KV_TYPE
    open(bad, "wb").write(data[: len(data) // 2])
    assert c.state_load(bad) == -12                       # SLLM_ERR_GGUF_TRUNCATED
    other = model.ctx(40)                                 # another context depth
    assert other.state_load(f) == -34                     # SLLM_ERR_TENSOR_SHAPE
    assert c.state_load(str(tmp_path / "missing.slkv")) == -3
    # the refusals left the context usable
    assert c.state_load(f) == 0
    assert c.generate(np.zeros(0, np.int32), 2)[0] == 0
    other.close()
    c.close()
    model.close()


def test_cli_and_tgbench_on_the_cuda_row(cuda, synth, tmp_path):
    """The reference's own CLI and decode benchmark with --backend cuda: the
    same generated text as the CPU row, and tg_bench's token checksum (its
    witness that a faster row produced the same tokens) equal across rows."""
    assert rr.available() and os.path.exists(rr.CLI), "build saphira-llm_b200/reference_row first"
    cfg = synth.small_config(n_layer=2, n_embd=512, n_ff=1536, n_head=4, n_head_kv=2, n_vocab=1000)
    m = synth.SynthModel(cfg, seed=6, tokenizer=True)
    path = str(tmp_path / "synth.gguf")
    m.image.tofile(path)
    rc1, text_gpu, err1 = rr.run_cli(path, "cuda", n=16)
    rc2, text_cpu, err2 = rr.run_cli(path, "cpu", n=16)
    assert rc1 == 0, err1
    assert rc2 == 0, err2
    assert text_gpu == text_cpu and len(text_gpu) > 0
    rc1, cs_gpu, out1 = rr.run_tgbench(path, "cuda")
    rc2, cs_cpu, out2 = rr.run_tgbench(path, "cpu")
    assert rc1 == rc2 == 0, (out1, out2)
    assert cs_gpu is not None and cs_gpu == cs_cpu
