"""Batch decode (configs[4] at batch 16): B sequences stepped together over a
shard, every layer GEMV one skinny GEMM over the B tokens.

The reference serves a batch as one context per sequence, so each sequence of
a batch must give, bit for bit, the tokens and logits of its own batch-1 run:
  * on one rank, against the single-sequence tensor-parallel context (which
    equals the oracle) and the oracle itself;
  * on a group of ranks on one GPU (exchanges by device copies);
  * at the configs[4] widths (8192 / 28672, two layers), every one of 16
    sequences against its own batch-1 run.
"""
import numpy as np
import pytest

from conftest import bits

pytestmark = pytest.mark.gpu

TP_CFG = dict(n_layer=2, n_embd=512, n_ff=1024, n_head=4, n_head_kv=2, n_vocab=1000)


def _prompts(seed, b, n, vocab):
    return np.random.default_rng(seed).integers(0, vocab, (b, n)).astype(np.int32)


def _single(model, prompt, n_new, n_ctx=64):
    c = model.ctx(n_ctx)
    rc, toks = c.generate(prompt, n_new)
    assert rc == 0
    lg = c.last_logits()[1]
    c.close()
    return toks, lg


def test_batch_one_rank_matches_single_and_oracle(cuda, orc, synth):
    cfg = synth.small_config(**TP_CFG)
    m = synth.SynthModel(cfg, seed=41)
    tm = cuda.TpModel(1, 0, 0, desc=m.desc())
    prompts = _prompts(5, 5, 9, cfg.n_vocab)
    b = tm.batch(5, 64)
    rc, toks = b.generate(prompts, 12)
    assert rc == 0
    assert cuda.gemm_error() == 0
    for s in range(5):
        want, lg = _single(tm, prompts[s], 12)
        assert toks[s].tolist() == want.tolist(), f"sequence {s}"
        assert np.array_equal(bits(b.last_logits(s)[1]), bits(lg)), f"sequence {s}"
    oc = orc.ctx(m.desc(), 64)
    r2, t2 = oc.generate(prompts[3], 12)
    assert r2 == 0 and toks[3].tolist() == t2.tolist()
    b.close()
    tm.close()


def test_batch_continuation(cuda, synth):
    """A second call with no prompt continues every sequence: 6 + 6 new
    tokens equal 12 in one call."""
    cfg = synth.small_config(**TP_CFG)
    m = synth.SynthModel(cfg, seed=42)
    tm = cuda.TpModel(1, 0, 0, desc=m.desc())
    prompts = _prompts(6, 3, 7, cfg.n_vocab)
    b = tm.batch(3, 64)
    rc, whole = b.generate(prompts, 12)
    assert rc == 0
    b.reset()
    rc1, first = b.generate(prompts, 6)
    rc2, second = b.generate(np.zeros((3, 0), np.int32), 6)
    assert rc1 == rc2 == 0
    assert np.concatenate([first, second], axis=1).tolist() == whole.tolist()
    # too long for the cache: refused, nothing run
    assert b.generate(prompts, 64)[0] == cuda.abi.ERR_TOO_LARGE
    b.close()
    tm.close()


@pytest.mark.parametrize("n", [2, 4])
def test_batch_group_matches_one_rank(cuda, synth, n):
    sd = cuda.abi.TpSynthDesc(n_layer=2, n_embd=1024, n_ff=16384, n_head=8, n_head_kv=4, n_vocab=3001,
                              f_rms_eps=1e-5, rope_freq_base=500000.0, seed=1234)
    prompts = _prompts(7, 6, 5, sd.n_vocab)
    one = cuda.TpModel(1, 0, 0, synth=sd)
    b1 = one.batch(6, 32)
    rc, t1 = b1.generate(prompts, 8)
    assert rc == 0
    l1 = [b1.last_logits(s)[1] for s in range(6)]
    b1.close()
    one.close()
    shards = [cuda.TpModel(n, r, 0, synth=sd) for r in range(n)]
    bs = [s.batch(6, 32) for s in shards]
    rc, t = cuda.tp_batch_generate_group(bs, prompts, 8)
    assert rc == 0
    assert t.tolist() == t1.tolist()
    for s in range(6):
        lg = np.concatenate([b.last_logits(s)[1] for b in bs])
        assert np.array_equal(bits(lg), bits(l1[s])), f"sequence {s}"
    for b in bs:
        b.close()
    for s in shards:
        s.close()


def test_batch16_config4_widths(cuda):
    """configs[4]'s layer geometry (8192 / 28672, 64 / 8 heads) at batch 16:
    every sequence equals its own batch-1 run, tokens and logits."""
    sd = cuda.abi.TpSynthDesc(n_layer=2, n_embd=8192, n_ff=28672, n_head=64, n_head_kv=8, n_vocab=128256,
                              f_rms_eps=1e-5, rope_freq_base=500000.0, seed=4242)
    tm = cuda.TpModel(1, 0, 0, synth=sd)
    prompts = _prompts(8, 16, 6, sd.n_vocab)
    b = tm.batch(16, 32)
    rc, toks = b.generate(prompts, 6)
    assert rc == 0
    assert cuda.gemm_error() == 0
    for s in range(16):
        want, lg = _single(tm, prompts[s], 6, n_ctx=32)
        assert toks[s].tolist() == want.tolist(), f"sequence {s}"
        assert np.array_equal(bits(b.last_logits(s)[1]), bits(lg)), f"sequence {s}"
    b.close()
    tm.close()


def _nccl_batch_rank(rank, n, uid, prompts, n_new, q):
    import importlib
    import torch  # noqa: F401  (a process with torch keeps one NCCL copy)
    try:
        cuda = importlib.import_module("saphira-llm_b200")
        comm = cuda.TpComm(uid, n, rank, rank)
        sd = cuda.abi.TpSynthDesc(n_layer=2, n_embd=1024, n_ff=16384, n_head=8, n_head_kv=4, n_vocab=3001,
                                  f_rms_eps=1e-5, rope_freq_base=500000.0, seed=1234)
        tm = cuda.TpModel(n, rank, rank, synth=sd)
        b = tm.batch(prompts.shape[0], 32, comm)
        rc, toks = b.generate(prompts, n_new)
        lg = [b.last_logits(s)[1] for s in range(prompts.shape[0])]
        q.put((rank, rc, toks.tolist(), lg))
        b.close()
        tm.close()
        comm.close()
    except Exception as e:  # report, never hang the parent
        q.put((rank, -999, repr(e), None))


def test_batch_two_gpus_nccl_matches_one(cuda):
    """Two processes, one GPU each, the exchanges NCCL collectives carrying
    every sequence's rows: the one-GPU batch's tokens and logits."""
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("one GPU on this box: the NCCL batch exchange is covered by the multi-GPU bench")
    sd = cuda.abi.TpSynthDesc(n_layer=2, n_embd=1024, n_ff=16384, n_head=8, n_head_kv=4, n_vocab=3001,
                              f_rms_eps=1e-5, rope_freq_base=500000.0, seed=1234)
    prompts = _prompts(12, 5, 6, sd.n_vocab)
    one = cuda.TpModel(1, 0, 0, synth=sd)
    b1 = one.batch(5, 32)
    rc, t1 = b1.generate(prompts, 8)
    assert rc == 0
    l1 = [b1.last_logits(s)[1] for s in range(5)]
    b1.close()
    one.close()
    uid = cuda.tp_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_nccl_batch_rank, args=(r, 2, uid, prompts, 8, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(2):
            rank, rc, toks, lg = q.get(timeout=300)
            res[rank] = (rc, toks, lg)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(res[r][0] == 0 for r in range(2)), res
    assert res[0][1] == res[1][1] == t1.tolist()
    for s in range(5):
        lg = np.concatenate([res[r][2][s] for r in range(2)])
        assert np.array_equal(bits(lg), bits(l1[s])), f"sequence {s}"


def test_batch_group_eight_ranks_config4_widths(cuda):
    """Eight ranks of the configs[4] layer geometry (one kv head, 1024 O
    columns, 3584 FFN rows and one down chunk per rank: the shapes of the
    eight-GPU run), batch 16, on one GPU: TP = 1's tokens and logits."""
    sd = cuda.abi.TpSynthDesc(n_layer=2, n_embd=8192, n_ff=28672, n_head=64, n_head_kv=8, n_vocab=3001,
                              f_rms_eps=1e-5, rope_freq_base=500000.0, seed=99)
    prompts = _prompts(13, 16, 5, sd.n_vocab)
    one = cuda.TpModel(1, 0, 0, synth=sd)
    b1 = one.batch(16, 32)
    rc, t1 = b1.generate(prompts, 6)
    assert rc == 0
    l1 = [b1.last_logits(s)[1] for s in range(16)]
    b1.close()
    one.close()
    shards = [cuda.TpModel(8, r, 0, synth=sd) for r in range(8)]
    bs = [s.batch(16, 32) for s in shards]
    rc, t = cuda.tp_batch_generate_group(bs, prompts, 6)
    assert rc == 0
    assert cuda.gemm_error() == 0
    assert t.tolist() == t1.tolist()
    for s in range(16):
        lg = np.concatenate([b.last_logits(s)[1] for b in bs])
        assert np.array_equal(bits(lg), bits(l1[s])), f"sequence {s}"
    for b in bs:
        b.close()
    for s in shards:
        s.close()
