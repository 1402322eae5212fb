"""The persistent engine's work split on the CPU (no device): the host code
that cuts every stage of an engine program into one contiguous range of rows
per CTA. A wrong cut runs a row twice or never, so the split is checked for
what the kernel relies on -- each stage starts at its first op's row 0 and
ends at the next stage's first op, the cursors never go backwards, every
cursor names a real row, so every row runs exactly once -- and for balance:
no CTA costs more than the average plus a few prologues and rows, in the
split's own cost model (a row streams K/4 bytes, twice for a gate/up pair;
an attention head counts as 64 KB; entering an input group costs its
RMSNorm + quantisation prologue, worth 192 KB). Also the host-buffer
projections' cut of a call into two engine launches."""
import ctypes as C

import numpy as np
import pytest

PROLOGUE = 192.0 * 1024.0
EPI_DOTS, EPI_F32, EPI_RESID, EPI_SILU, EPI_ATTN = 0, 1, 2, 3, 4


@pytest.fixture(scope="module")
def split(pkg):
    import os
    if not os.path.exists(pkg.LIB_PATH):
        pkg.build()
    L = pkg.lib()

    def run(ops, stage_first, grid):
        n = len(ops)
        arr = lambda v: (C.c_int32 * max(1, len(v)))(*v)
        rows = arr([o[0] for o in ops])
        K = arr([o[1] for o in ops])
        epi = arr([o[2] for o in ops])
        group = arr([o[3] for o in ops])
        sf = arr(stage_first)
        n_stages = len(stage_first) - 1
        out = (C.c_int32 * (2 * n_stages * (grid + 1)))()
        rc = L.sllm_cuda_test_engine_split(rows, K, epi, group, n, sf, n_stages, grid, out)
        cur = np.frombuffer(out, dtype=np.int32).reshape(n_stages, grid + 1, 2) if rc == 0 else None
        return rc, cur

    return run


def row_cost(op):
    rows, K, epi, _ = op
    if epi == EPI_ATTN:
        return 65536.0
    return (K // 4) * (2.0 if epi == EPI_SILU else 1.0)


def check(ops, stage_first, grid, cur):
    n_stages = len(stage_first) - 1
    for s in range(n_stages):
        o0, o1 = stage_first[s], stage_first[s + 1]
        c = [tuple(x) for x in cur[s]]
        assert c[grid] == (o1, 0), (s, c[grid])
        if o1 > o0:
            assert c[0] == (o0, 0), (s, c[0])
        for a, b in zip(c, c[1:]):
            assert a <= b, (s, a, b)                     # lexicographic: never backwards
        for op, row in c:
            assert o0 <= op <= o1, (s, op)
            if op < o1:
                assert 0 <= row < ops[op][0], (s, op, row)
            else:
                assert row == 0
        # walk every CTA's range: each row exactly once, and its cost
        seen = {o: np.zeros(ops[o][0], dtype=np.int32) for o in range(o0, o1)}
        costs = []
        for k in range(grid):
            (oa, ra), (ob, rb) = c[k], c[k + 1]
            cost, last_group = 0.0, None
            o, r = oa, ra
            while (o, r) < (ob, rb):
                end = rb if o == ob else ops[o][0]
                seen[o][r:end] += 1
                if ops[o][3] != last_group:
                    cost += PROLOGUE
                    last_group = ops[o][3]
                cost += (end - r) * row_cost(ops[o])
                o, r = o + 1, 0
            costs.append(cost)
        for o in range(o0, o1):
            assert np.all(seen[o] == 1), (s, o)
        if o1 > o0:
            # every run of ops on one input group pays its prologue at least
            # once; cutting a run adds one more per CTA boundary
            runs = 1 + sum(ops[o][3] != ops[o - 1][3] for o in range(o0 + 1, o1))
            total = sum(ops[o][0] * row_cost(ops[o]) for o in range(o0, o1)) + runs * PROLOGUE
            max_rc = max(row_cost(ops[o]) for o in range(o0, o1))
            bound = total / grid + 3 * PROLOGUE + 2 * max_rc + 1.0
            assert max(costs) <= bound, (s, max(costs), bound)


def test_headline_projections_program(split):
    """32 copies of a 2B-4T layer's seven projections, every
    GEMV its own input group, one stage on 148 CTAs."""
    E, G, F = 2560, 640, 6912
    ops = []
    for layer in range(32):
        for rows, K in [(E, E), (G, E), (G, E), (E, E), (F, E), (F, E), (E, F)]:
            ops.append((rows, K, EPI_F32, len(ops)))
    rc, cur = split(ops, [0, len(ops)], 148)
    assert rc == 0
    check(ops, [0, len(ops)], 148, cur)


def test_decode_step_program(split):
    """30 layers x five stages (Q/K/V on one group, attention
    heads, O + residual, the gate/up pair, down + residual)."""
    E, G, F, H = 2560, 640, 6912, 20
    ops, stage_first, g = [], [0], 0
    for layer in range(30):
        for rows in (E, G, G):
            ops.append((rows, E, EPI_F32, g))
        g += 1
        stage_first.append(len(ops))
        ops.append((H, 128, EPI_ATTN, g)); g += 1
        stage_first.append(len(ops))
        ops.append((E, E, EPI_RESID, g)); g += 1
        stage_first.append(len(ops))
        ops.append((F, E, EPI_SILU, g)); g += 1
        stage_first.append(len(ops))
        ops.append((E, F, EPI_RESID, g)); g += 1
        stage_first.append(len(ops))
    rc, cur = split(ops, stage_first, 148)
    assert rc == 0
    check(ops, stage_first, 148, cur)


def test_random_programs(split):
    """Seeded random programs: single-row ops, empty stages, more CTAs than
    rows, one CTA, shared and separate input groups."""
    rng = np.random.default_rng(20)
    for case in range(200):
        n_stages = int(rng.integers(1, 5))
        ops, stage_first, g = [], [0], 0
        for s in range(n_stages):
            for _ in range(int(rng.integers(0, 6))):
                epi = int(rng.integers(0, 5))
                rows = int(rng.choice([1, 2, 7, 64, 640, 2560, 6912]))
                K = int(rng.choice([128, 256, 2560, 6912, 8192]))
                if rng.random() < 0.5:
                    g += 1
                ops.append((rows, K, epi, g))
            stage_first.append(len(ops))
        grid = int(rng.choice([1, 2, 3, 17, 148, 1000]))
        rc, cur = split(ops, stage_first, grid)
        assert rc == 0, case
        check(ops, stage_first, grid, cur)


def test_bad_arguments(split):
    ops = [(4, 128, EPI_F32, 0)]
    assert split(ops, [0, 2], 4)[0] == -1                 # stages past the op list
    assert split([(0, 128, EPI_F32, 0)], [0, 1], 4)[0] == -1   # an op with no rows
    assert split([(4, 128, 9, 0)], [0, 1], 4)[0] == -1    # unknown epilogue
    assert split(ops, [0, 1], 0)[0] == -1                 # no CTAs


def test_host_projection_split(pkg):
    """The host-buffer projections' two-piece cut: none under 16 layers;
    otherwise the second piece holds at least one layer and at most half,
    sized so that the first piece's copy-back (f32 outputs at ~54 GB/s)
    hides behind the second piece's compute (2-bit codes at ~5.6 TB/s):
    20 + 12 layers for the 2B-4T benchmark's 32."""
    L = pkg.lib()
    E, F, G = 2560, 6912, 640
    assert L.sllm_cuda_test_projection_split(E, F, G, 32) == 20
    for n in range(0, 16):
        assert L.sllm_cuda_test_projection_split(E, F, G, n) == 0
    for n in range(16, 200):
        split = L.sllm_cuda_test_projection_split(E, F, G, n)
        last = n - split
        assert 1 <= last <= n // 2, (n, split)
        copy = 4.0 * (3 * E + 2 * G + 2 * F) / 54e9
        compute = (2.0 * E * E + 2.0 * G * E + 3.0 * E * F) / 4.0 / 5.6e12
        assert split * copy <= last * compute * 1.0001 or last == n // 2, n   # the first copy hides
    assert L.sllm_cuda_test_projection_split(640, 1280, 640, 32) == 0       # widths the engine lacks
    assert L.sllm_cuda_test_projection_split(0, F, G, 32) == -1
