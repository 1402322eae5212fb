"""Prefill GEMM on the tcgen05 tensor cores, against the oracle.

The reference has no GEMM: its prefill quantises each token and runs the
GEMV once per token (src/forward.c:756-793). So every int32 dot of the GEMM
must equal the oracle's per-token GEMV exactly, and every f32 output the
per-token epilogue's bits; the gate/up form must give silu(gate) * up as the
reference's sllm_silu_inplace and product compute it.
"""
import numpy as np
import pytest

from conftest import bits

pytestmark = pytest.mark.gpu

# (weight rows, K, tokens): one tile; ragged tokens and rows; several k-steps
# and M tiles; the config-3 widths at a reduced token count
SHAPES = [(128, 128, 128), (256, 384, 200), (200, 256, 70), (640, 2560, 130), (384, 6912, 256)]


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _quant_rows(cuda, x):
    import torch
    m, n = x.shape
    xd = _dev(x)
    q = torch.empty((m, n), dtype=torch.int8, device="cuda")
    acts = torch.empty((m, 2), dtype=torch.int32, device="cuda")
    cuda.quant_act_rows(xd, m, n, q, acts)
    return q, acts


@pytest.mark.parametrize("n", [384, 2560, 6912, 8192, 130])
def test_quant_act_rows_bit_exact(cuda, orc, n):
    """Per-token quantisation of a batch: every row length of the models
    (the vectorised kernel, one to eight float4 per thread) and a length that
    is not a multiple of 4 (the scalar kernel); a zero row, NaN and inf."""
    import torch
    rng = np.random.default_rng(5 + n)
    x = (rng.standard_normal((37, n)) * 2).astype(np.float32)
    x[3] = 0.0
    x[7, 5] = np.nan
    x[9, 11] = np.inf
    q, acts = _quant_rows(cuda, x)
    torch.cuda.synchronize()
    q = q.cpu().numpy()
    a = acts.cpu().numpy()
    for t in range(x.shape[0]):
        wq, ws, wsum = orc.quant_act(x[t])
        assert np.array_equal(q[t], wq), t
        assert bits(a[t, :1].view(np.float32))[0] == bits(np.array([ws], np.float32))[0], t
        assert a[t, 1] == wsum, t


@pytest.mark.parametrize("rows,n,m", SHAPES)
def test_gemm_bit_exact(cuda, orc, synth, rows, n, m):
    import torch
    rng = np.random.default_rng(rows + 7 * n + 13 * m)
    w = synth.random_i2s(rng, rows, n)
    x = rng.standard_normal((m, n)).astype(np.float32)
    q, acts = _quant_rows(cuda, x)
    dots = torch.empty((m, rows), dtype=torch.int32, device="cuda")
    y = torch.empty((m, rows), dtype=torch.float32, device="cuda")
    cuda.gemm(_dev(w), rows, n, m, q, acts, dots, y)
    assert cuda.gemm_error() == 0
    d = dots.cpu().numpy()
    yy = y.cpu().numpy()
    for t in range(m):
        wy, wd = orc.gemv_f32(w, rows, n, x[t])
        assert np.array_equal(d[t], wd), f"token {t}"
        assert np.array_equal(bits(yy[t]), bits(wy)), f"token {t}"


@pytest.mark.parametrize("rows,n,m", [(256, 384, 200), (384, 2560, 130)])
def test_gemm_silu_bit_exact(cuda, orc, synth, rows, n, m):
    import torch
    rng = np.random.default_rng(rows * 5 + n + m)
    wg = synth.random_i2s(rng, rows, n)
    wu = synth.random_i2s(rng, rows, n)
    x = rng.standard_normal((m, n)).astype(np.float32)
    q, acts = _quant_rows(cuda, x)
    h = torch.empty((m, rows), dtype=torch.float32, device="cuda")
    cuda.gemm_silu(_dev(wg), _dev(wu), rows, n, m, q, acts, h)
    assert cuda.gemm_error() == 0
    hh = h.cpu().numpy()
    for t in range(m):
        g, _ = orc.gemv_f32(wg, rows, n, x[t])
        u, _ = orc.gemv_f32(wu, rows, n, x[t])
        want = (orc.silu(g) * u).astype(np.float32)
        assert np.array_equal(bits(hh[t]), bits(want)), f"token {t}"


@pytest.mark.parametrize("rows,n", [(6912, 2560), (2560, 6912)])
def test_gemm_config3_sizes_match_per_token_gemv(cuda, orc, synth, rows, n):
    """configs[3] at full size (512 tokens): every int32 dot equals the GPU
    GEMV of that token (an independent kernel), and a sample of tokens equals
    the oracle."""
    import torch
    m = 512
    rng = np.random.default_rng(rows + n)
    w = synth.random_i2s(rng, rows, n)
    x = rng.standard_normal((m, n)).astype(np.float32)
    wd_dev = _dev(w)
    q, acts = _quant_rows(cuda, x)
    dots = torch.empty((m, rows), dtype=torch.int32, device="cuda")
    cuda.gemm(wd_dev, rows, n, m, q, acts, dots, None)
    per = torch.empty((m, rows), dtype=torch.int32, device="cuda")
    for t in range(m):
        cuda.gemv(wd_dev, rows, n, q[t], per[t])
    assert cuda.gemm_error() == 0
    assert torch.equal(dots, per)
    d = dots.cpu().numpy()
    qh = q.cpu().numpy()
    for t in (0, 1, 255, 511):
        assert np.array_equal(d[t], orc.gemv(w, rows, n, qh[t])), f"token {t}"


# (weight rows, K, tokens) of the skinny form (at most 16 tokens): one tile
# and one token; ragged rows; the contraction split over clusters of 2 and 8
# CTAs; the tensor-parallel widths of configs[4]; more tiles than resident
# CTAs (the persistent grid, two tiles for some CTAs)
SKINNY = [(128, 128, 1), (200, 256, 5), (8192, 1024, 16), (640, 2560, 7), (1024, 8192, 16), (3584, 1024, 3),
          (8192, 3584, 16), (40000, 256, 16)]


@pytest.fixture
def skinny(cuda):
    cuda.set_gemm_form(2)
    yield
    cuda.set_gemm_form(0)


@pytest.mark.parametrize("rows,n,m", SKINNY)
def test_gemm_skinny_bit_exact(cuda, orc, synth, skinny, rows, n, m):
    """At most 16 tokens, weight rows as the MMA's M operand: the same dots
    and epilogue bits as the per-token GEMV."""
    import torch
    rng = np.random.default_rng(rows + 3 * n + 17 * m)
    w = synth.random_i2s(rng, rows, n)
    x = rng.standard_normal((m, n)).astype(np.float32)
    q, acts = _quant_rows(cuda, x)
    dots = torch.empty((m, rows), dtype=torch.int32, device="cuda")
    y = torch.empty((m, rows), dtype=torch.float32, device="cuda")
    cuda.gemm(_dev(w), rows, n, m, q, acts, dots, y)
    assert cuda.gemm_error() == 0
    d = dots.cpu().numpy()
    yy = y.cpu().numpy()
    for t in range(m):
        wy, wd = orc.gemv_f32(w, rows, n, x[t])
        assert np.array_equal(d[t], wd), f"token {t}"
        assert np.array_equal(bits(yy[t]), bits(wy)), f"token {t}"


@pytest.mark.parametrize("rows,n,m", [(256, 384, 16), (3584, 8192, 16), (384, 2560, 1), (20000, 256, 9)])
def test_gemm_skinny_silu_bit_exact(cuda, orc, synth, skinny, rows, n, m):
    import torch
    rng = np.random.default_rng(rows * 3 + n + m)
    wg = synth.random_i2s(rng, rows, n)
    wu = synth.random_i2s(rng, rows, n)
    x = rng.standard_normal((m, n)).astype(np.float32)
    q, acts = _quant_rows(cuda, x)
    h = torch.empty((m, rows), dtype=torch.float32, device="cuda")
    cuda.gemm_silu(_dev(wg), _dev(wu), rows, n, m, q, acts, h)
    assert cuda.gemm_error() == 0
    hh = h.cpu().numpy()
    for t in range(m):
        g, _ = orc.gemv_f32(wg, rows, n, x[t])
        u, _ = orc.gemv_f32(wu, rows, n, x[t])
        want = (orc.silu(g) * u).astype(np.float32)
        assert np.array_equal(bits(hh[t]), bits(want)), f"token {t}"


@pytest.mark.parametrize("form", [1, 2])
def test_gemm_strided_columns(cuda, orc, synth, form):
    """A contraction over columns [c0, c0 + k) of a wider activation matrix
    (the tensor-parallel slice of O or down): both forms give the oracle's
    dots of that slice."""
    import torch
    rows, k, width, c0, m = 512, 1024, 4096, 2048, 12
    rng = np.random.default_rng(99 + form)
    w = synth.random_i2s(rng, rows, k)
    x = rng.standard_normal((m, width)).astype(np.float32)
    q, acts = _quant_rows(cuda, x)
    dots = torch.empty((m, rows), dtype=torch.int32, device="cuda")
    cuda.set_gemm_form(form)
    try:
        cuda.gemm_strided(_dev(w), rows, k, m, q[:, c0:], width, acts, dots, None)
        assert cuda.gemm_error() == 0
    finally:
        cuda.set_gemm_form(0)
    d = dots.cpu().numpy()
    qh = q.cpu().numpy()
    for t in range(m):
        assert np.array_equal(d[t], orc.gemv(w, rows, k, qh[t, c0:c0 + k])), f"token {t}"
