"""Failure detection on the GPU without a GPU fault.

* A bounded wait made to run out: a test hook shortens every engine wait to
  50 ms and makes one CTA leave out its first grid-barrier arrival, so the
  other CTAs' barrier waits give up. The call reports SLLM_CUDA_ERR_TIMEOUT
  (-61), the kernel still ends (the aborting CTAs keep reaching every barrier
  and drain their own copies), and the same context's next call, with the
  hook off, is correct again. Nothing traps, faults or spins unbounded.
* Host-injected refusals: a device allocation of a model or context
  (SLLM_CUDA_ERR_NOMEM, nothing leaked, the next try succeeds).
"""
import numpy as np
import pytest

from conftest import bits

pytestmark = pytest.mark.gpu

TIMEOUT, NOMEM = -61, -2


class _Faults:
    def __init__(self, cuda, skip_cta, wait_ms):
        self.L, self.skip, self.ms = cuda.lib(), skip_cta, wait_ms

    def __enter__(self):
        assert self.L.sllm_cuda_test_engine_faults(0, self.skip, self.ms) == 0
        return self

    def __exit__(self, *a):
        assert self.L.sllm_cuda_test_engine_faults(0, -1, 0.0) == 0


def test_layer_chain_barrier_timeout_then_correct(cuda, orc, synth):
    cfg = synth.small_config(n_layer=2, n_embd=256, n_ff=512, n_head=2, n_head_kv=1, n_vocab=64)
    m = synth.SynthModel(cfg, seed=61)
    model = cuda.Model(m.desc())
    c = model.ctx(8)
    x = np.random.default_rng(61).standard_normal(cfg.n_embd).astype(np.float32)
    want = c.layer_chain(0, 2, x)                  # the engine program, once normally
    with _Faults(cuda, 5, 50.0):
        out = np.empty_like(x)
        rc = cuda.lib().sllm_cuda_layer_chain(model.h, c.h, 0, 2, x.ctypes.data, out.ctypes.data)
        assert rc == TIMEOUT, (rc, cuda.lib().sllm_cuda_last_error())
    assert b"gave up" in cuda.lib().sllm_cuda_last_error()
    got = c.layer_chain(0, 2, x)                   # the same context, hook off
    assert np.array_equal(bits(got), bits(want))
    c.close()
    model.close()


def test_decode_barrier_timeout_then_correct(cuda, orc, synth):
    cfg = synth.small_config(n_layer=2, n_embd=256, n_ff=512, n_head=2, n_head_kv=1, n_vocab=500)
    m = synth.SynthModel(cfg, seed=62)
    model = cuda.Model(m.desc())
    c = model.ctx(32)
    prompt = np.random.default_rng(62).integers(0, cfg.n_vocab, 5).astype(np.int32)
    rc, _ = c.generate(prompt, 2)                  # builds the decode graph
    assert rc == 0
    c.reset()
    with _Faults(cuda, 3, 50.0):
        rc, _ = c.generate(prompt, 4)
        assert rc == TIMEOUT, (rc, cuda.lib().sllm_cuda_last_error())
    assert c.n_past() == 0                          # a failed call consumes nothing
    c.reset()
    rc, got = c.generate(prompt, 6)
    oc = orc.ctx(m.desc(), 32)
    rc2, want = oc.generate(prompt, 6)
    assert rc == rc2 == 0 and got.tolist() == want.tolist()
    assert np.array_equal(bits(c.last_logits()), bits(oc.last_logits()))
    c.close()
    model.close()


def test_injected_allocation_failures(cuda, synth):
    import ctypes as C
    L = cuda.lib()
    cfg = synth.small_config(n_layer=1, n_vocab=100)
    m = synth.SynthModel(cfg, seed=63)
    d = m.desc()
    h = C.c_void_p()
    L.sllm_cuda_test_fail_next(1, 1)
    assert L.sllm_cuda_model_upload(C.byref(d), 0, C.byref(h)) == NOMEM
    assert not h.value
    model = cuda.Model(d)                           # the next try succeeds
    for k in (1, 3, 7):                             # fail the k-th allocation of a context
        L.sllm_cuda_test_fail_next(1, 0)
        ch = C.c_void_p()
        L.sllm_cuda_test_fail_next(1, k)
        rc = L.sllm_cuda_ctx_new(model.h, 16, C.byref(ch))
        L.sllm_cuda_test_fail_next(1, 0)
        assert rc == NOMEM and not ch.value, (k, rc)
    c = model.ctx(16)
    rc, toks = c.generate(np.arange(1, 4, dtype=np.int32), 3)
    assert rc == 0
    tm = C.c_void_p()
    L.sllm_cuda_test_fail_next(1, 1)
    assert L.sllm_cuda_tp_model_upload(C.byref(d), 1, 0, 0, C.byref(tm)) == NOMEM
    L.sllm_cuda_test_fail_next(1, 0)
    c.close()
    model.close()
