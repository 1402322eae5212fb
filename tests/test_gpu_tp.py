"""Tensor-parallel decode (the configs[4] path): shards of one model on N ranks.

The sharding changes where each value is computed, never how: Q/K/V and
gate/up rows split by heads and FFN rows, O and down split by contraction
columns with an int32 sum of the partial dots (exact in any order), the head
split by vocabulary rows with a first-maximum argmax across slices. So:
  * TP = 1 equals the oracle (the reference's forward pass) bit for bit;
  * a group of N ranks equals TP = 1 bit for bit (tokens and logits), on one
    GPU with the exchanges done by device copies;
  * on two GPUs with the peer-memory exchange and with NCCL, the same
    (skipped when the box has one GPU).
"""
import os

import numpy as np
import pytest

from conftest import bits

pytestmark = pytest.mark.gpu

TP_CFG = dict(n_layer=2, n_embd=512, n_ff=1024, n_head=4, n_head_kv=2, n_vocab=1000)


def _tokens(seed, n, vocab):
    return np.random.default_rng(seed).integers(0, vocab, n).astype(np.int32)


def test_tp1_matches_oracle(cuda, orc, synth):
    cfg = synth.small_config(**TP_CFG)
    m = synth.SynthModel(cfg, seed=21)
    tm = cuda.TpModel(1, 0, 0, desc=m.desc())
    tc = tm.ctx(64)
    oc = orc.ctx(m.desc(), 64)
    prompt = _tokens(3, 11, cfg.n_vocab)
    r1, t1 = tc.generate(prompt, 20)
    r2, t2 = oc.generate(prompt, 20)
    assert r1 == r2 == 0
    assert t1.tolist() == t2.tolist()
    v0, lg = tc.last_logits()
    assert v0 == 0 and np.array_equal(bits(lg), bits(oc.last_logits()))
    # continuation from the last logits, with no prompt
    r1, t1 = tc.generate(np.zeros(0, np.int32), 5)
    r2, t2 = oc.generate(np.zeros(0, np.int32), 5)
    assert r1 == r2 == 0 and t1.tolist() == t2.tolist()
    assert cuda.gemm_error() == 0
    tc.close()
    tm.close()


@pytest.mark.parametrize("n", [2])
def test_tp_group_matches_oracle(cuda, orc, synth, n):
    cfg = synth.small_config(**TP_CFG)
    m = synth.SynthModel(cfg, seed=22)
    shards = [cuda.TpModel(n, r, 0, desc=m.desc()) for r in range(n)]
    ctxs = [s.ctx(64) for s in shards]
    oc = orc.ctx(m.desc(), 64)
    prompt = _tokens(4, 9, cfg.n_vocab)
    r1, t1 = cuda.tp_generate_group(ctxs, prompt, 16)
    r2, t2 = oc.generate(prompt, 16)
    assert r1 == r2 == 0
    assert t1.tolist() == t2.tolist()
    parts = [c.last_logits() for c in ctxs]
    assert [p[0] for p in parts] == [r * (cfg.n_vocab // n) for r in range(n)]
    lg = np.concatenate([p[1] for p in parts])
    assert np.array_equal(bits(lg), bits(oc.last_logits()))
    for c in ctxs:
        c.close()
    for s in shards:
        s.close()


def _synth_desc(cuda):
    # n_ff / 1 = 16384 > 8192: the single rank's down projection runs as two
    # column chunks, so the chunked contraction is covered too
    return cuda.abi.TpSynthDesc(n_layer=2, n_embd=1024, n_ff=16384, n_head=8, n_head_kv=4, n_vocab=3001,
                                f_rms_eps=1e-5, rope_freq_base=500000.0, seed=1234)


def _group_run(cuda, sd, n, prompt, n_new):
    shards = [cuda.TpModel(n, r, 0, synth=sd) for r in range(n)]
    ctxs = [s.ctx(64) for s in shards]
    if n == 1:
        rc, toks = ctxs[0].generate(prompt, n_new)
    else:
        rc, toks = cuda.tp_generate_group(ctxs, prompt, n_new)
    lg = np.concatenate([c.last_logits()[1] for c in ctxs])
    for c in ctxs:
        c.close()
    for s in shards:
        s.close()
    return rc, toks, lg


def test_tp_synth_ranks_agree(cuda):
    """A device-generated model: every rank count gives TP = 1's tokens and
    logits, bit for bit (the shards are slices of one model)."""
    sd = _synth_desc(cuda)
    prompt = _tokens(5, 7, sd.n_vocab)
    rc1, t1, l1 = _group_run(cuda, sd, 1, prompt, 12)
    assert rc1 == 0
    for n in (2, 4):
        rc, t, lg = _group_run(cuda, sd, n, prompt, 12)
        assert rc == 0
        assert t.tolist() == t1.tolist(), f"TP={n}"
        assert np.array_equal(bits(lg), bits(l1)), f"TP={n}"


WIDE_CFG = dict(n_layer=2, n_embd=8192, n_ff=16384, n_head=64, n_head_kv=8, n_vocab=3001)


def test_tp_engine_path_matches_oracle(cuda, orc, synth):
    """configs[4]'s widths (n_embd 8192): the layer GEMVs run as persistent-
    engine programs (pre-quantised slices, raw partial dots); TP = 1 must still
    equal the oracle exactly."""
    cfg = synth.small_config(**WIDE_CFG)
    m = synth.SynthModel(cfg, seed=31)
    tm = cuda.TpModel(1, 0, 0, desc=m.desc())
    tc = tm.ctx(32)
    assert tc.uses_engine()
    assert tc.fused_layers() == cfg.n_layer       # one rank: each layer is one four-stage program
    oc = orc.ctx(m.desc(), 32)
    prompt = _tokens(8, 5, cfg.n_vocab)
    r1, t1 = tc.generate(prompt, 6)
    r2, t2 = oc.generate(prompt, 6)
    assert r1 == r2 == 0
    assert t1.tolist() == t2.tolist()
    _, lg = tc.last_logits()
    assert np.array_equal(bits(lg), bits(oc.last_logits()))
    tc.close()
    tm.close()


def test_tp_engine_ranks_agree(cuda):
    sd = cuda.abi.TpSynthDesc(n_layer=2, n_embd=8192, n_ff=16384, n_head=64, n_head_kv=8, n_vocab=3001,
                              f_rms_eps=1e-5, rope_freq_base=500000.0, seed=77)
    prompt = _tokens(9, 6, sd.n_vocab)
    rc1, t1, l1 = _group_run(cuda, sd, 1, prompt, 8)
    assert rc1 == 0
    # 8 ranks: one kv head and 1024 O columns per rank (the widths the
    # eight-GPU run uses)
    for n in (2, 4, 8):
        rc, t, lg = _group_run(cuda, sd, n, prompt, 8)
        assert rc == 0
        assert t.tolist() == t1.tolist(), f"TP={n}"
        assert np.array_equal(bits(lg), bits(l1)), f"TP={n}"


def _wide_desc(cuda):
    # n_embd 8192: the widths with an exchanging engine instance, so two
    # ranks over peer memory run the fused exchange
    return cuda.abi.TpSynthDesc(n_layer=2, n_embd=8192, n_ff=16384, n_head=64, n_head_kv=8, n_vocab=3001,
                                f_rms_eps=1e-5, rope_freq_base=500000.0, seed=77)


def _nccl_rank(rank, n, uid, prompt, n_new, kind, q, wide=False):
    import importlib
    import torch  # noqa: F401  (a process with torch keeps one NCCL copy)
    try:
        os.environ["SLLM_CUDA_TP_EXCHANGE"] = kind
        cuda = importlib.import_module("saphira-llm_b200")
        comm = cuda.TpComm(uid, n, rank, rank)
        tm = cuda.TpModel(n, rank, rank, synth=_wide_desc(cuda) if wide else _synth_desc(cuda))
        tc = tm.ctx(64, comm)
        got = tc.exchange_kind()
        if wide and kind == "p2p" and not tc.fused_exchange():
            got = "not fused"
        rc, toks = tc.generate(prompt, n_new)
        v0, lg = tc.last_logits()
        q.put((rank, rc if got == kind else -998, toks.tolist(), v0, lg))
        tc.close()
        tm.close()
        comm.close()
    except Exception as e:  # report, never hang the parent
        q.put((rank, -999, repr(e), 0, None))


@pytest.mark.parametrize("kind", ["p2p", "nccl"])
def test_tp_two_gpus_matches_one(cuda, kind):
    """Two processes, one GPU each: the one-shot peer-memory exchange (P2P
    stores and epoch flags) and NCCL's collectives give TP = 1's bits."""
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("one GPU on this box: the NCCL exchange is covered by the multi-GPU bench and runs")
    sd = _synth_desc(cuda)
    prompt = _tokens(6, 7, sd.n_vocab)
    rc1, t1, l1 = _group_run(cuda, sd, 1, prompt, 12)
    assert rc1 == 0
    uid = cuda.tp_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_nccl_rank, args=(r, 2, uid, prompt, 12, kind, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(2):
            rank, rc, toks, v0, lg = q.get(timeout=300)
            res[rank] = (rc, toks, v0, lg)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(res[r][0] == 0 for r in range(2)), res
    assert res[0][1] == res[1][1] == t1.tolist()
    lg = np.concatenate([res[r][3] for r in range(2)])
    assert np.array_equal(bits(lg), bits(l1))


@pytest.mark.parametrize("kind", ["p2p", "nccl"])
def test_tp_two_gpus_wide_matches_one(cuda, kind):
    """The 8192-wide model on two GPUs: with the peer exchange the step runs
    the fused exchange (stores into every rank's memory and flag waits inside
    the layer programs); with NCCL the per-phase collectives. Both give the
    single-GPU bits, tokens and logits."""
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("one GPU on this box: the exchange is covered by the multi-GPU bench and runs")
    sd = _wide_desc(cuda)
    prompt = _tokens(10, 7, sd.n_vocab)
    rc1, t1, l1 = _group_run(cuda, sd, 1, prompt, 12)
    assert rc1 == 0
    uid = cuda.tp_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_nccl_rank, args=(r, 2, uid, prompt, 12, kind, q, True)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(2):
            rank, rc, toks, v0, lg = q.get(timeout=300)
            res[rank] = (rc, toks, v0, lg)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(res[r][0] == 0 for r in range(2)), res
    assert res[0][1] == res[1][1] == t1.tolist()
    lg = np.concatenate([res[r][3] for r in range(2)])
    assert np.array_equal(bits(lg), bits(l1))
