"""The CUDA row on the reference's side of the boundary, without a device:
saphira-llm built with the two insertion-only patches
(saphira-llm_b200/reference_row/) still runs its CPU row exactly as before,
refuses the CUDA row with an explained status when no sm_100 device is
present (no fallback once "cuda" is asked for), and lets "auto" choose the
CPU row. The patches add lines only: none of the reference's lines appear
in them. The GPU half is tests/test_gpu_reference_row.py."""
import os

import numpy as np
import pytest

import reference_row as rr

ROW_DIR = os.path.join(rr.ROOT, "saphira-llm_b200", "reference_row")


def _row():
    if not rr.available():
        pytest.skip("the reference row library is not built (needs the reference source tree)")
    return rr.Row()


@pytest.mark.parametrize("name", ["forward.c.patch", "dispatch.c.patch", "main.c.patch", "tg_bench.c.patch"])
def test_patches_insert_only(name):
    body = open(os.path.join(ROW_DIR, name)).read().splitlines()
    hunks = [l for l in body if l.startswith("@@")]
    assert hunks
    for h in hunks:
        old = h.split()[1]                       # -start,0: nothing of the reference replaced
        assert old.endswith(",0"), h
    assert not [l for l in body if l.startswith("-") and not l.startswith("---")]


def test_cpu_row_is_the_reference(synth, ref):
    row = _row()
    cfg = synth.small_config(n_layer=2, n_embd=256, n_ff=512, n_head=2, n_head_kv=1, n_vocab=1000)
    m = synth.SynthModel(cfg, seed=71)
    prompt = np.random.default_rng(71).integers(0, cfg.n_vocab, 7).astype(np.int32)
    rm = row.open(m.image, rr.CPU, 32)
    assert rm.rc == 0 and rm.backend() == rr.CPU
    rc, toks = rm.generate(prompt, 6)
    want_model = ref.model(m.image, 32, 1)
    rc2, want = want_model.generate(prompt, 6)
    assert rc == rc2 == 0 and toks.tolist() == want.tolist()
    assert np.array_equal(rm.last_logits(cfg.n_vocab).view(np.uint32),
                          want_model.last_logits(cfg.n_vocab).view(np.uint32))
    rm.close()


def test_cuda_row_refused_without_a_device(synth, cuda_absent):
    row = _row()
    cfg = synth.small_config(n_layer=1)
    m = synth.SynthModel(cfg, seed=72)
    rm = row.open(m.image, rr.CUDA, 16)
    assert rm.rc == -4                           # SLLM_ERR_UNSUPPORTED: no fallback to the CPU
    rm.close()
    rm = row.open(m.image, rr.AUTO, 16)          # "auto": the CPU row
    assert rm.rc == 0 and rm.backend() == rr.CPU
    rm.close()


def test_cuda_row_refuses_widths_it_does_not_run(synth):
    row = _row()
    # head dim 64: the dispatch row refuses before any device is asked
    cfg = synth.small_config(n_layer=1, n_embd=256, n_ff=512, n_head=4, n_head_kv=2)
    cfg.n_rot = 64
    m = synth.SynthModel(cfg, seed=73)
    rm = row.open(m.image, rr.CUDA, 16)
    assert rm.rc == -4
    rm.close()


def test_cli_and_tgbench_backend_flag(synth, tmp_path, cuda_absent):
    """The CLI and tg_bench take --backend: the CPU row runs, "cuda" without
    a device is refused (exit status, no output), an unknown row is a usage
    error. The model file carries a byte-level BPE vocabulary so that the
    reference's tokenizer loads it."""
    if not os.path.exists(rr.CLI):
        pytest.skip("the reference row CLI is not built (needs the reference source tree)")
    cfg = synth.small_config(n_layer=2, n_vocab=1000)
    m = synth.SynthModel(cfg, seed=5, tokenizer=True)
    path = str(tmp_path / "synth.gguf")
    m.image.tofile(path)
    rc, text, err = rr.run_cli(path, "cpu")
    assert rc == 0 and len(text) > 0, err
    rc, text, err = rr.run_cli(path, "cuda")
    assert rc != 0 and "CUDA row" in err
    rc, _, err = rr.run_cli(path, "bogus")
    assert rc == 2 and "--backend" in err
    rc, cs, out = rr.run_tgbench(path, "cpu")
    assert rc == 0 and cs is not None, out
