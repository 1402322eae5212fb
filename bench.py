"""Benchmark: I2_S GEMV HBM GB/s on a bitnet-b1.58-2B-4T layer chain (B200).

Workload: the seven I2_S GEMVs of one 2B-4T layer
at batch 1 -- Q 2560x2560, K/V 640x2560, O 2560x2560, gate/up 6912x2560,
down 2560x6912 -- with RMSNorm + int8 quantisation before every projection
(attn_norm, attn_sub_norm, ffn_norm, ffn_sub_norm), SiLU gating and the two
residual adds: the decode layer without attention, run by
sllm_cuda_layer_chain_device. One STEP runs that chain through 32 distinct
layer copies (556 MB of packed weights, more than 4x the 126 MB L2), so every
step streams its weights from HBM and no L2 flush is needed.

  value     whole-job GB/s: algorithmic bytes of all ranks / max device time
  e2e       the same metric through the host-buffer C ABI call
            sllm_cuda_layer_chain (pinned input copied in, output copied back
            every step), wall clock
  roofline  the GEMV kernel (every launch in the step is one): algorithmic
            bytes per launch / average launch time, against the measured HBM
            copy bandwidth
  cpu_baseline  the reference saphira-llm library (oracle/_ref, compiled
            from its own sources) running the same chain on the host cores

  python bench.py [--gpus N --steps K --warmup W] [--impl reference]
Multi-GPU: one process per GPU (torchrun); each rank runs its own replica
(the chain does not shard: replicas only), weak scaling.
"""
import argparse
import importlib
import json
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "oracle")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

N_COPIES = 32
METRIC = "I2_S GEMV HBM GB/s (bitnet-b1.58-2B-4T layer chain: 7 GEMVs + RMSNorm, batch 1)"
FALLBACK_HBM_GBS = 6650.0


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def chain_bytes(cfg, m):
    """Algorithmic bytes of one layer's chain: every weight byte once (packed
    codes with their scale tail, the four norm vectors) plus every activation
    vector each GEMV reads or writes once."""
    E, F, G = cfg.n_embd, cfg.n_ff, cfg.n_embd_gqa
    w = m.layer_weight_bytes(0)
    act = 4 * ((E + E + 2 * G)           # QKV: x in, q k v out
               + (E + E + E)             # O: q in, residual in, ffn_inp out
               + (E + F)                 # gate/up: ffn_inp in, h out
               + (F + E + E))            # down: h in, residual in, x out
    return w + act


def clocks_start():
    """Sample SM clocks and throttle reasons while the timed region runs."""
    try:
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        import tempfile
        tmp = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        p = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits", "-lms", "100"],
                             stdout=tmp, stderr=subprocess.DEVNULL)
        return p, tmp.name
    except Exception:
        return None, None


def clocks_stop(handle, dev_index):
    p, path = handle
    if p is None:
        return None
    p.terminate()
    try:
        p.wait(timeout=5)
    except Exception:
        p.kill()
    sm, mx, reasons = [], None, set()
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    try:
        for line in open(path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9 or f[0] != str(dev_index):
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(path)
    except Exception:
        return None
    if not sm:
        return None
    return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def dist_init():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def reference_arm(args, world, rank):
    """The reference CPU implementation on this box's host cores."""
    if rank != 0:
        return
    import oracle
    synth = importlib.import_module("saphira-llm_b200.synth")
    if not oracle.reference_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libsllm_ref.so was not built"}))
        return
    ref = oracle.Reference()
    cfg = synth.Config(n_layer=N_COPIES, n_vocab=256)
    m = synth.SynthModel(cfg, seed=1)
    d = m.desc()
    cores = os.cpu_count() or 1
    pool = ref.pool(cores)
    E, F, G = cfg.n_embd, cfg.n_ff, cfg.n_embd_gqa
    x = np.random.default_rng(0).standard_normal(E).astype(np.float32)
    scratch = np.zeros(4 * E + 2 * G + 3 * F, np.float32)
    qbuf = np.zeros(max(E, F), np.int8)
    dots = np.zeros(max(E, F), np.int32)
    # a step is a bounded sample of the chain: 8 of the 32 layer copies
    per_step = 8

    def step(i):
        for j in range(per_step):
            pool.layer_chain(d, (i * per_step + j) % N_COPIES, x, scratch, qbuf, dots)

    for i in range(args.warmup):
        step(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        step(args.warmup + i)
    dt = time.perf_counter() - t0
    gbs = chain_bytes(cfg, m) * per_step * args.steps / dt / 1e9
    sample = f"{per_step} of the {N_COPIES} layer copies per step, {args.steps} steps"
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8xternary->int32, f32",
        "data": "synthetic (seeded random-init 2B-4T layers)",
        "config": {"workload": "layer_chain_2b4t", "layers_per_step": per_step, "threads": pool.threads,
                   "isa_level": ref.isa},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": pool.threads, "kind": "reference",
                         "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


def cpu_baseline_sample(cfg, m):
    """Rank 0 only: the reference library on the host cores, ~10 s bounded."""
    import oracle
    if not oracle.reference_available():
        return None
    ref = oracle.Reference()
    cores = os.cpu_count() or 1
    pool = ref.pool(cores)
    d = m.desc()
    E, F, G = cfg.n_embd, cfg.n_ff, cfg.n_embd_gqa
    x = np.random.default_rng(0).standard_normal(E).astype(np.float32)
    scratch = np.zeros(4 * E + 2 * G + 3 * F, np.float32)
    qbuf = np.zeros(max(E, F), np.int8)
    dots = np.zeros(max(E, F), np.int32)
    for layer in range(2):
        pool.layer_chain(d, layer, x, scratch, qbuf, dots)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < 10.0:
        pool.layer_chain(d, n % cfg.n_layer, x, scratch, qbuf, dots)
        n += 1
    dt = time.perf_counter() - t0
    return {"value": round(chain_bytes(cfg, m) * n / dt / 1e9, 3), "unit": "GB/s", "cores": pool.threads,
            "kind": "reference",
            "sample": f"{n} layer chains over the same {cfg.n_layer} layer copies in {dt:.1f} s "
                      f"(reference ISA level {ref.isa})"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    world, rank, local = dist_init()
    if args.impl == "reference":
        reference_arm(args, world, rank)
        return

    import torch
    pkg = importlib.import_module("saphira-llm_b200")
    synth = importlib.import_module("saphira-llm_b200.synth")
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))

    cfg = synth.Config(n_layer=N_COPIES, n_vocab=256)
    m = synth.SynthModel(cfg, seed=1 + rank)
    model = pkg.Model(m.desc(), local)
    ctx = model.ctx(8)
    E = cfg.n_embd
    x0 = torch.from_numpy(np.random.default_rng(rank).standard_normal(E).astype(np.float32)).cuda()
    x = x0.clone()
    stream = torch.cuda.current_stream()
    per_step_bytes = chain_bytes(cfg, m) * N_COPIES
    launches_per_step = 4 * N_COPIES

    def step():
        ctx.layer_chain_device(0, N_COPIES, x, stream)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    clk = clocks_start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    torch.cuda.synchronize()
    start.record(stream)
    ev[0].record(stream)
    for i in range(args.steps):
        step()
        ev[i + 1].record(stream)
    end.record(stream)
    torch.cuda.synchronize()
    clocks = clocks_stop(clk, local)
    ms = start.elapsed_time(end)
    per_step_ms = [ev[i].elapsed_time(ev[i + 1]) for i in range(args.steps)]
    t = torch.tensor([ms], dtype=torch.float64, device="cuda")
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms_max = float(t.item())
    value = per_step_bytes * args.steps * world / (ms_max / 1e3) / 1e9

    # e2e through the host-buffer C ABI (pinned input, output read back)
    host_in = torch.from_numpy(np.random.default_rng(rank).standard_normal(E).astype(np.float32)).pin_memory()
    host_out = torch.empty(E, dtype=torch.float32).pin_memory()
    lib = pkg.lib()
    for _ in range(2):
        lib.sllm_cuda_layer_chain(model.h, ctx.h, 0, N_COPIES, host_in.data_ptr(), host_out.data_ptr())
    if world > 1:
        torch.distributed.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        rc = lib.sllm_cuda_layer_chain(model.h, ctx.h, 0, N_COPIES, host_in.data_ptr(), host_out.data_ptr())
        assert rc == 0
    e2e_s = time.perf_counter() - t0
    te = torch.tensor([e2e_s], dtype=torch.float64, device="cuda")
    if world > 1:
        torch.distributed.all_reduce(te, op=torch.distributed.ReduceOp.MAX)
    e2e = per_step_bytes * args.steps * world / float(te.item()) / 1e9

    peak, peak_kind = peaks()
    per_launch_bytes = per_step_bytes / launches_per_step
    per_launch_s = (ms / 1e3) / (args.steps * launches_per_step)
    achieved = per_launch_bytes / per_launch_s / 1e9
    traffic = None
    prof = os.path.join(ROOT, "profiles", "i2s_gemv_layer_chain_traffic.txt")
    if os.path.exists(prof):
        for line in open(prof):
            if line.startswith("traffic_bytes_per_launch"):
                traffic = int(line.split()[1])
    out = {
        "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": round(ms_max / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8xternary->int32, f32", "data": "synthetic (seeded random-init 2B-4T layers)",
        "config": {"workload": "layer_chain_2b4t", "layer_copies_per_step": N_COPIES,
                   "weights_mb_per_step": round(m.layer_weight_bytes(0) * N_COPIES / 1e6, 1),
                   "bytes_per_step": per_step_bytes,
                   "l2": "inputs larger than L2: 32 distinct layer copies (>4x the 126 MB L2) per step, no flush",
                   "parallelism": f"replicas x{world}", "batch": 1},
        "roofline": {"bound": "hbm", "kernel": "i2s_gemv_kernel (all 4 launches per layer)",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                     "bytes_per_launch": int(per_launch_bytes), "traffic": traffic},
        "e2e": {"value": round(e2e, 3), "unit": "GB/s", "h2d_bytes_per_step": 4 * E, "d2h_bytes_per_step": 4 * E,
                "api": "sllm_cuda_layer_chain (host buffers, wall clock)"},
        "gpu_launches": launches_per_step * args.steps,
        "step_ms_min_median_max": [round(min(per_step_ms), 4), round(float(np.median(per_step_ms)), 4),
                                   round(max(per_step_ms), 4)],
        "clocks": clocks,
    }
    if rank == 0 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline_sample(cfg, m)
    if rank == 0:
        print(json.dumps(out))
    ctx.close()
    model.close()
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
