"""GPU parity of the kernel-level C ABI against the oracle restatement.

int32 dot products: bit-exact. f32 outputs: bit-exact (the epilogue is one
IEEE division, one conversion and one multiply; the tolerance north_star
allows, 1e-5 relative, is not needed and not used). Device buffers come from
torch; every compute call goes through libsllm_cuda.so.
"""
import numpy as np
import pytest

from conftest import bits

pytestmark = pytest.mark.gpu

SHAPES = [
    (6912, 2560),    # config 0 / gate, up
    (2560, 6912),    # down
    (640, 2560),     # K, V
    (2560, 2560),    # Q, O
    (1, 128),        # smallest
    (3, 256),        # rows below a warp's task
    (1000, 384),     # K not a multiple of 512
    (7, 8192),       # widest K
    (100000, 128),   # many short rows
    (257, 1152),
]


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def test_quant_act_bit_exact(cuda, orc):
    import torch
    rng = np.random.default_rng(0)
    cases = [rng.standard_normal(n).astype(np.float32) * 3 for n in (1, 5, 128, 2560, 6912, 28672, 65536)]
    cases += [np.zeros(256, np.float32),
              np.array([1e-40, -1e-41, 0.0, 3e-41] * 64, np.float32),
              np.array([np.inf, 1, -2, 0] * 64, np.float32),
              np.array([np.nan, 1, -2, 0] * 64, np.float32),
              np.arange(-254, 255, dtype=np.float32) / 2]
    for x in cases:
        xd = _dev(x)
        q = torch.empty(x.size, dtype=torch.int8, device="cuda")
        act = torch.zeros(2, dtype=torch.int32, device="cuda")
        cuda.quant_act(xd, x.size, q, act)
        torch.cuda.synchronize()
        wq, ws, wsum = orc.quant_act(x)
        a = act.cpu().numpy()
        assert np.array_equal(q.cpu().numpy(), wq)
        assert a[0].view(np.float32) == ws or (np.isnan(ws) and np.isnan(a[0].view(np.float32)))
        assert a[1] == wsum


@pytest.mark.parametrize("rows,n", SHAPES)
def test_raw_gemv_bit_exact(cuda, orc, synth, rows, n):
    import torch
    rng = np.random.default_rng(rows + 31 * n)
    w = synth.random_i2s(rng, rows, n)
    q, _, _ = orc.quant_act(rng.standard_normal(n).astype(np.float32))
    out = torch.empty(rows, dtype=torch.int32, device="cuda")
    cuda.gemv(_dev(w), rows, n, _dev(q), out)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), orc.gemv(w, rows, n, q))


@pytest.mark.parametrize("rows,n", SHAPES)
def test_gemv_f32_bit_exact(cuda, orc, synth, rows, n):
    import torch
    rng = np.random.default_rng(rows * 3 + n)
    w = synth.random_i2s(rng, rows, n)
    x = rng.standard_normal(n).astype(np.float32)
    y = torch.empty(rows, dtype=torch.float32, device="cuda")
    d = torch.empty(rows, dtype=torch.int32, device="cuda")
    cuda.gemv_f32(_dev(w), rows, n, _dev(x), y, d)
    torch.cuda.synchronize()
    wy, wd = orc.gemv_f32(w, rows, n, x)
    assert np.array_equal(d.cpu().numpy(), wd)
    assert np.array_equal(bits(y.cpu().numpy()), bits(wy))


def test_gemv_extreme_activations(cuda, orc, synth):
    """All-zero row (scale 0: the epilogue divides by zero, NaN/inf reproduced),
    a single huge value, codes on every rounding half."""
    import torch
    rng = np.random.default_rng(9)
    rows, n = 96, 1024
    w = synth.random_i2s(rng, rows, n)
    xs = [np.zeros(n, np.float32),
          np.where(np.arange(n) == 17, 1e30, 1e-3).astype(np.float32),
          (np.arange(n, dtype=np.float32) - 512) / 4,
          np.full(n, -7.25, np.float32)]
    for x in xs:
        y = torch.empty(rows, dtype=torch.float32, device="cuda")
        cuda.gemv_f32(_dev(w), rows, n, _dev(x), y)
        torch.cuda.synchronize()
        wy, _ = orc.gemv_f32(w, rows, n, x)
        assert np.array_equal(bits(y.cpu().numpy()), bits(wy))


def test_committed_reference_fixtures(cuda, synth):
    """The CUDA path against outputs of the reference library itself."""
    import torch
    import fixtures
    for case in fixtures.load_gemv_cases():
        w, x = fixtures.gemv_inputs(synth, case)
        y = torch.empty(case["rows"], dtype=torch.float32, device="cuda")
        d = torch.empty(case["rows"], dtype=torch.int32, device="cuda")
        cuda.gemv_f32(_dev(w), case["rows"], case["n"], _dev(x), y, d)
        torch.cuda.synchronize()
        assert np.array_equal(d.cpu().numpy(), case["dots"]), case["name"]
        assert np.array_equal(bits(y.cpu().numpy()), case["y_bits"]), case["name"]


def test_argument_errors(cuda):
    import torch
    w = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    q = torch.zeros(256, dtype=torch.int8, device="cuda")
    out = torch.zeros(16, dtype=torch.int32, device="cuda")
    with pytest.raises(cuda.SllmCudaError) as e:
        cuda.gemv(w, 16, 200, q, out)
    assert e.value.status == -1
    with pytest.raises(cuda.SllmCudaError) as e:
        cuda.gemv(w, 16, 256, q[1:], out)              # misaligned activation
    assert e.value.status == -1


@pytest.mark.parametrize("shared_x", [True, False])
def test_gemv_batch_matches_single_gemvs(cuda, orc, synth, shared_x):
    """configs[0]'s shape as a batch of independent GEMVs in one persistent
    launch: every output equals the single-GEMV entry point's and the oracle's,
    bit for bit, on two runs (the second reuses the launch tables)."""
    import torch
    rows, n, count = 6912, 2560, 5
    rng = np.random.default_rng(4040 + shared_x)
    ws = [synth.random_i2s(rng, rows, n) for _ in range(count)]
    wd = [_dev(w) for w in ws]
    xs = rng.standard_normal((count, n)).astype(np.float32)
    xs[2] *= 40.0
    xd = _dev(xs)
    b = cuda.GemvBatch(wd, rows, n)
    y = torch.empty((count, rows), dtype=torch.float32, device="cuda")
    for _ in range(2):
        y.zero_()
        b.run(xd, y, 0 if shared_x else n)
        torch.cuda.synchronize()
        assert b.error() == 0
        got = y.cpu().numpy()
        for i in range(count):
            x = xs[0] if shared_x else xs[i]
            one = torch.empty(rows, dtype=torch.float32, device="cuda")
            cuda.gemv_f32(wd[i], rows, n, _dev(x), one)
            torch.cuda.synchronize()
            want, _ = orc.gemv_f32(ws[i], rows, n, x)
            assert np.array_equal(bits(got[i]), bits(one.cpu().numpy())), i
            assert np.array_equal(bits(got[i]), bits(want)), i
    b.close()


def test_gemv_batch_argument_errors(cuda, synth):
    import ctypes as C
    L = cuda.lib()
    w = _dev(synth.random_i2s(np.random.default_rng(1), 64, 256))
    h = C.c_void_p()
    arr = (C.c_void_p * 1)(w.data_ptr())
    assert L.sllm_cuda_gemv_batch_new(arr, 0, 64, 256, 0, C.byref(h)) == -1
    assert L.sllm_cuda_gemv_batch_new(arr, 1, 64, 200, 0, C.byref(h)) == -1
    assert L.sllm_cuda_gemv_batch_new(arr, 1, 64, 256, 0, C.byref(h)) == 0
    assert L.sllm_cuda_gemv_batch_run(h, None, 0, None, None) == -1
    L.sllm_cuda_gemv_batch_free(h)
