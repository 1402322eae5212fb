"""The tensor-parallel shard plan on the CPU (no device): for every rank
count the upload accepts, the ranks' shards partition every tensor exactly
-- query and kv heads, O's n_embd columns, gate/up's n_ff rows, down's n_ff
columns in chunks the engine can run, and the vocabulary rows of the
head -- and the geometries it cannot shard are refused with the upload's
own errors."""
import ctypes as C
import os

import pytest

ERR_ARG, ERR_UNSUPPORTED = -1, -4

# (name, n_embd, n_ff, n_head, n_head_kv, n_vocab)
MODELS = [
    ("configs[4] 80L 8192", 8192, 28672, 64, 8, 128256),
    ("2B-4T", 2560, 6912, 20, 5, 128256),
    ("small, odd vocabulary", 1024, 2816, 8, 8, 777),
]


@pytest.fixture(scope="module")
def plan(pkg):
    if not os.path.exists(pkg.LIB_PATH):
        pkg.build()
    L = pkg.lib()

    def run(E, F, H, Hkv, V, n, r, n_layer=2):
        out = (C.c_int32 * 8)()
        rc = L.sllm_cuda_test_tp_plan(n_layer, E, F, H, Hkv, V, n, r, out)
        return rc, list(out)

    return run


@pytest.mark.parametrize("model", MODELS, ids=[m[0] for m in MODELS])
@pytest.mark.parametrize("n", [1, 2, 4, 8])
def test_shards_partition_every_tensor(plan, model, n):
    _, E, F, H, Hkv, V = model
    shardable = H % n == 0 and Hkv % n == 0 and (E // n) % 128 == 0 and (F // n) % 128 == 0
    vocab = []
    for r in range(n):
        rc, (hq, hk, e_loc, f_loc, down_c, down_k, v0, v_loc) = plan(E, F, H, Hkv, V, n, r)
        if not shardable:
            assert rc == ERR_UNSUPPORTED, (n, r, rc)
            continue
        assert rc == 0, (n, r, rc)
        assert hq * n == H and hk * n == Hkv
        assert hq // hk == H // Hkv              # each rank's query heads read its own kv heads
        assert e_loc * n == E and e_loc == hq * 128
        assert f_loc * n == F
        assert down_c * down_k == f_loc and down_k <= 8192 and down_k % 128 == 0
        vocab.append((v0, v_loc))
    if shardable:
        # the head's rows: consecutive, in rank order, covering [0, V) once
        pos = 0
        for v0, v_loc in vocab:
            assert v0 == pos and v_loc >= 0
            pos += v_loc
        assert pos == V


def test_refused_geometries(plan):
    assert plan(8192, 28672, 64, 8, 1000, 2, 2)[0] == ERR_ARG           # rank outside the group
    assert plan(8192, 28672, 64, 8, 1000, 16, 0)[0] == ERR_ARG          # more ranks than supported
    assert plan(8192, 28672, 64, 8, 1000, 1, 0, n_layer=0)[0] == ERR_ARG
    assert plan(8192, 28672, 32, 8, 1000, 1, 0)[0] == ERR_UNSUPPORTED   # head dim 256
    assert plan(8192, 28672, 64, 6, 1000, 1, 0)[0] == ERR_UNSUPPORTED   # 64 % 6 heads
    assert plan(8192, 40960, 64, 8, 1000, 1, 0)[0] == ERR_UNSUPPORTED   # n_ff above one quantisation pass
