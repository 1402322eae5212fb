"""sllm_cuda_layer_chain_device_noalloc: the layer chain for callers that
cannot call cudaMalloc (a host whose allocator already owns the device's
memory, loops that cannot take cudaMalloc's implicit synchronisation). Its
scratch is a static 128 KB device array in the library, so it must give the
same bits as the context-backed sllm_cuda_layer_chain_device, call after
call, and refuse a model whose scratch would not fit.

Collected last on purpose (file name), so a failure here cannot hide others.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import bits

pytestmark = pytest.mark.gpu


def _noalloc(cuda):
    L = cuda.lib()
    f = L.sllm_cuda_layer_chain_device_noalloc
    f.argtypes = [C.c_void_p, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p]
    f.restype = C.c_int
    return f


def test_noalloc_chain_matches_the_context_chain_twice(cuda, synth):
    import torch
    fn = _noalloc(cuda)
    cfg = synth.Config(n_layer=3, n_vocab=256)          # the 2B-4T layer geometry
    m = synth.SynthModel(cfg, seed=91)
    model = cuda.Model(m.desc())
    ctx = model.ctx(8)
    stream = torch.cuda.current_stream()
    rng = np.random.default_rng(91)
    for call in range(2):                                # two calls in a row share the scratch
        x = rng.standard_normal(cfg.n_embd).astype(np.float32) * (1 + call)
        want = ctx.layer_chain(0, 3, x)                  # the existing, context-backed entry point
        xd = torch.from_numpy(x).cuda()
        rc = fn(model.h, 0, 3, xd.data_ptr(), stream.cuda_stream)
        assert rc == 0, cuda.lib().sllm_cuda_last_error()
        torch.cuda.synchronize()
        assert np.array_equal(bits(xd.cpu().numpy()), bits(want)), f"call {call}"


def test_noalloc_chain_refuses_a_model_beyond_its_scratch(cuda, synth):
    import torch
    fn = _noalloc(cuda)
    # 2*8192 + 2*8192 + 8192 = 40960 floats > the 32768 the static scratch holds
    cfg = synth.small_config(n_layer=1, n_embd=8192, n_ff=8192, n_head=64, n_head_kv=64, n_vocab=64)
    m = synth.SynthModel(cfg, seed=3)
    model = cuda.Model(m.desc())
    xd = torch.zeros(cfg.n_embd, device="cuda")
    rc = fn(model.h, 0, 1, xd.data_ptr(), None)
    assert rc == -36                                     # SLLM_ERR_TOO_LARGE
    assert b"scratch" in cuda.lib().sllm_cuda_last_error()


def test_noalloc_chain_with_the_reference_order_fallback_forced(cuda, synth):
    """The forced reference-order RMSNorm sums (the rare ambiguous case of
    the certified sum) reach this entry point too, and give the bits of the
    context chain under the same switch."""
    import torch
    fn = _noalloc(cuda)
    cfg = synth.Config(n_layer=2, n_vocab=256)
    m = synth.SynthModel(cfg, seed=92)
    model = cuda.Model(m.desc())
    ctx = model.ctx(8)
    x = np.random.default_rng(92).standard_normal(cfg.n_embd).astype(np.float32)
    cuda.set_force_fallback(True)
    try:
        want = ctx.layer_chain(0, 2, x)
        xd = torch.from_numpy(x).cuda()
        rc = fn(model.h, 0, 2, xd.data_ptr(), torch.cuda.current_stream().cuda_stream)
        assert rc == 0, cuda.lib().sllm_cuda_last_error()
        torch.cuda.synchronize()
    finally:
        cuda.set_force_fallback(False)
    assert np.array_equal(bits(xd.cpu().numpy()), bits(want))
