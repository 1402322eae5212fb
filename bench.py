"""Benchmark: I2_S GEMV HBM GB/s on bitnet-b1.58-2B-4T layers, plus the other configs (B200).

Headline workload (as stated there): the seven I2_S
GEMV shapes of one 2B-4T layer at batch 1 -- Q 2560x2560, K/V 640x2560,
O 2560x2560, gate/up 6912x2560, down 2560x6912 -- each on its own f32 N(0,1)
activation, RMSNorm'd (eps 1e-5, norm weights N(1, 0.02)) and int8-quantised
per token, run back to back (sllm_cuda_layer_projections_device). One STEP
runs them through 32 distinct layer copies (564 MB of algorithmic bytes, more
than 4x the 126 MB L2), so every step streams its weights from HBM and no
L2 flush is needed. Inputs are seeded synthetic data of the configs' shapes.

Also in the same JSON line, measured in the same run:
  chain      the decode layer's projection chain (each GEMV's input is the
             previous one's output: norm -> QKV -> O + residual -> gate/up,
             SiLU -> down + residual), sllm_cuda_layer_chain_device
  prefill    configs[3]: 512 tokens through gate/up (SiLU fused) and down on
             the tcgen05 tensor cores, int8 TOP/s, with the reference CPU path
  gemv       configs[0]: the single 6912x2560 GEMV over 128 distinct weight
             copies per step (L2-cold), as 128 back-to-back launches and as
             one persistent launch, with the reference CPU GEMV beside it
  tp_decode  configs[4]: the 80-layer 8192 model, tensor-parallel over the
             ranks (NCCL between GPUs), tokens/s at batch 1, with the
             reference kernels chained on the CPU beside it (one rank)
  decode     configs[2]: random-init 2B-4T model, 64-token prompt, 256 greedy
             tokens, tokens/s through sllm_cuda_generate_greedy, with a bounded
             sample of the reference CPU decode beside it

  value         whole-job GB/s: algorithmic bytes of all ranks / max device time
  e2e           the same metric through the host-buffer C ABI call
                sllm_cuda_layer_projections (pinned inputs copied in, every
                output copied back each step), wall clock
  roofline      the persistent engine kernel (one launch per step)
  cpu_baseline  the reference saphira-llm library (oracle/_ref, compiled from
                its own sources) running the same projections on the host
                cores (rank 0, one GPU only)

  python bench.py [--gpus N --steps K --warmup W] [--impl reference]
                  [--no-cpu-baseline] [--no-gemv] [--no-prefill] [--no-tp] [--no-decode]
                  [--leg decode|prefill|tp|gemv]   (one leg only, for profiler captures)
Multi-GPU: one process per GPU (torchrun); each rank runs its own replica of
configs 0-3 (the projections do not shard: replicas only, weak scaling);
configs[4] is sharded over all ranks.
"""
import argparse
import importlib
import json
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "oracle")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

N_COPIES = 32
METRIC = "I2_S GEMV HBM GB/s (bitnet-b1.58-2B-4T: the 7 GEMVs of a layer with RMSNorm + int8 quant, batch 1)"
FALLBACK_HBM_GBS = 6650.0


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def cpu_model():
    """The host CPU's model name (the CPU baselines run on it)."""
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def projection_bytes(cfg, m):
    """Algorithmic bytes of one layer's seven independent projections: every
    packed weight byte (with its scale tail) once, every GEMV's input vector
    and norm vector once, every output once."""
    E, F, G = cfg.n_embd, cfg.n_ff, cfg.n_embd_gqa
    w = sum(m.tensors[f"blk.0.{n}.weight"].nbytes for n in
            ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"))
    inputs = 2 * 4 * (6 * E + F)                       # input vectors + their norm vectors
    outputs = 4 * (3 * E + 2 * G + 2 * F)
    return w + inputs + outputs


def chain_bytes(cfg, m):
    """Algorithmic bytes of one layer's dependent chain: every weight byte once
    (codes with scale tails, the four norm vectors) plus every activation
    vector each GEMV reads or writes once."""
    E, F, G = cfg.n_embd, cfg.n_ff, cfg.n_embd_gqa
    act = 4 * ((E + E + 2 * G) + (E + E + E) + (E + F) + (F + E + E))
    return m.layer_weight_bytes(0) + act


# ---------------------------------------------------------------------------
# clocks: NVML polled every 5 ms on this rank's GPU while the workload runs
# ---------------------------------------------------------------------------
_REASONS = {  # NVML clocks-event (throttle) reason bits
    0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown", 0x4: "sw_power_cap",
    0x80: "hw_power_brake_slowdown",
}


class ClockSampler:
    """SM clock and throttle reasons of this rank's GPU, sampled in a thread."""

    def __init__(self, local):
        import threading
        self.samples, self.reasons, self.max_mhz, self.err = [], set(), None, None
        self._stop = threading.Event()
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            want = str(torch.cuda.get_device_properties(local).uuid)
            self.h = None
            for i in range(pynvml.nvmlDeviceGetCount()):
                h = pynvml.nvmlDeviceGetHandleByIndex(i)
                u = pynvml.nvmlDeviceGetUUID(h)
                u = u.decode() if isinstance(u, bytes) else u
                if want in u or u.replace("GPU-", "") == want.replace("GPU-", ""):
                    self.h = h
            if self.h is None:
                self.h = pynvml.nvmlDeviceGetHandleByIndex(local)
            self.nvml = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.t = threading.Thread(target=self._run, daemon=True)
        except Exception as e:          # no NVML: report why instead of a number
            self.err, self.t = repr(e), None

    def _run(self):
        p = self.nvml
        while not self._stop.is_set():
            try:
                self.samples.append(p.nvmlDeviceGetClockInfo(self.h, p.NVML_CLOCK_SM))
                bits = p.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for b, name in _REASONS.items():
                    if bits & b:
                        self.reasons.add(name)
            except Exception as e:
                self.err = repr(e)
            self._stop.wait(0.005)

    def __enter__(self):
        if self.t is not None:
            self.t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self.t is not None:
            self.t.join()

    def summary(self):
        if not self.samples:
            return {"error": self.err or "no samples"}
        return {"sm_mhz": float(np.median(self.samples)), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples), "source": "NVML, 5 ms"}


# ---------------------------------------------------------------------------
# reference (CPU) legs
# ---------------------------------------------------------------------------
class RefProjections:
    """The reference library on the host cores, same inputs and layers."""

    def __init__(self, cfg, m, x):
        import oracle
        self.ref = oracle.Reference()
        self.cores = os.cpu_count() or 1
        self.pool = self.ref.pool(self.cores)
        self.cfg, self.m, self.d = cfg, m, m.desc()
        E, F = cfg.n_embd, cfg.n_ff
        self.x = [x[i * E:(i + 1) * E] for i in range(6)] + [x[6 * E: 6 * E + F]]
        self.dots = np.zeros(max(E, F), np.int32)

    def layer(self, il):
        """One layer: for each projection sllm_rms_norm -> sllm_i2s_quant_act ->
        pooled sllm_i2s_gemv -> the epilogue of src/forward.c:653-655."""
        cfg = self.cfg
        E, F, G = cfg.n_embd, cfg.n_ff, cfg.n_embd_gqa
        L = self.m.tensors
        p = f"blk.{il}."
        specs = [("attn_q", E, E, "attn_norm"), ("attn_k", G, E, "attn_norm"), ("attn_v", G, E, "attn_norm"),
                 ("attn_output", E, E, "attn_sub_norm"), ("ffn_gate", F, E, "ffn_norm"),
                 ("ffn_up", F, E, "ffn_norm"), ("ffn_down", E, F, "ffn_sub_norm")]
        out = []
        for (name, rows, n, norm), xin in zip(specs, self.x):
            xn = self.ref.rms_norm(xin, L[p + norm + ".weight"].view(np.float32), cfg.eps)
            q, s, total = self.ref.quant_act(xn)
            w = L[p + name + ".weight"]
            self.pool.gemv(w, rows, n, q, self.dots)
            ws = np.float32(w[rows * n // 4: rows * n // 4 + 4].view(np.float32)[0])
            post = ws / np.float32(s)
            out.append((self.dots[:rows] - total).astype(np.float32) * post)
        return out


def cpu_baseline_sample(cfg, m, x, seconds=10.0):
    import oracle
    if not oracle.reference_available():
        return None
    rp = RefProjections(cfg, m, x)
    rp.layer(0)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        rp.layer(n % cfg.n_layer)
        n += 1
    dt = time.perf_counter() - t0
    return {"value": round(projection_bytes(cfg, m) * n / dt / 1e9, 3), "unit": "GB/s", "cores": rp.pool.threads,
            "kind": "reference", "cpu": cpu_model(),
            "sample": f"{n} layers' seven projections (of the same {cfg.n_layer} layer copies) in {dt:.1f} s, "
                      f"reference ISA level {rp.ref.isa}"}


def reference_arm(args, world, rank):
    """bench.py --impl reference: the reference CPU implementation on this box."""
    if rank != 0:
        return
    import oracle
    synth = importlib.import_module("saphira-llm_b200.synth")
    if not oracle.reference_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libsllm_ref.so was not built"}))
        return
    cfg = synth.Config(n_layer=N_COPIES, n_vocab=256)
    m = synth.SynthModel(cfg, seed=1)
    xs = np.random.default_rng(0).standard_normal(6 * cfg.n_embd + cfg.n_ff).astype(np.float32)
    rp = RefProjections(cfg, m, xs)
    per_step = 8          # a bounded sample: 8 of the 32 layer copies per step
    for i in range(args.warmup):
        for j in range(per_step):
            rp.layer((i * per_step + j) % N_COPIES)
    t0 = time.perf_counter()
    for i in range(args.steps):
        for j in range(per_step):
            rp.layer(((args.warmup + i) * per_step + j) % N_COPIES)
    dt = time.perf_counter() - t0
    gbs = projection_bytes(cfg, m) * per_step * args.steps / dt / 1e9
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8 x ternary -> int32, f32",
        "data": "synthetic (seeded random-init 2B-4T layers)",
        "config": {"workload": "layer_projections_2b4t", "layers_per_step": per_step, "threads": rp.pool.threads,
                   "isa_level": rp.ref.isa},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": rp.pool.threads, "kind": "reference",
                         "cpu": cpu_model(),
                         "sample": f"{per_step} of the {N_COPIES} layer copies per step, {args.steps} steps"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


# ---------------------------------------------------------------------------
# GPU legs
# ---------------------------------------------------------------------------
def time_device(fn, steps, warmup, stream, world):
    """Device time of `steps` back-to-back calls of fn() after `warmup`, from
    an idle device to the end of the last step (synchronize, barrier, one
    event before and one after: an event between steps would serialise the
    launches and hide how consecutive steps overlap), max over ranks."""
    import torch
    for _ in range(max(warmup, 3)):
        fn()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(steps):
        fn()
    ev1.record(stream)
    torch.cuda.synchronize()
    return max_over_ranks(ev0.elapsed_time(ev1), world), None


def max_over_ranks(value, world, device="cuda"):
    """The largest of every rank's `value` (a duration): a multi-GPU figure
    is the slowest rank's. One rank: the value itself, with no collective."""
    if world <= 1:
        return float(value)
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


PREFILL_TOKENS = 512


INT8_NOMINAL_TOPS = 4500.0


def int8_peak():
    """Dense int8 tensor peak. The pool's measured peaks carry no int8 figure,
    so this is the nominal B200 dense rate (4.5 P ops/s, the sparse figure
    halved); 2x the measured bf16 burst rate is reported beside it."""
    return INT8_NOMINAL_TOPS, "nominal B200 dense int8 (4.5 P ops/s; no measured int8 peak on this pool)"


def bf16_x2_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return 2.0 * float(json.load(f)["bf16_tflops"])
    except Exception:
        return 2.0 * 1590.0


def prefill_leg(pkg, synth, local, rank, world, args):
    """512 tokens of fp32 N(0,1) activations through one 2B-4T
    layer's FFN projections on the tcgen05 tensor cores: per-token int8
    quantisation, gate/up with the SiLU product fused, then down. One step =
    the four launches; ops = 2 * 512 * (6912*2560*2 + 2560*6912)."""
    import torch
    cfg = synth.Config(n_layer=1, n_vocab=256)
    m = synth.SynthModel(cfg, seed=77 + rank)
    E, F, M = cfg.n_embd, cfg.n_ff, PREFILL_TOKENS
    L = m.tensors
    wg, wu, wd = (torch.from_numpy(np.ascontiguousarray(L[f"blk.0.{n}.weight"])).cuda()
                  for n in ("ffn_gate", "ffn_up", "ffn_down"))
    rng = np.random.default_rng(100 + rank)
    xa_h = rng.standard_normal((M, E)).astype(np.float32)
    xd_h = rng.standard_normal((M, F)).astype(np.float32)
    xa, xd = torch.from_numpy(xa_h).cuda(), torch.from_numpy(xd_h).cuda()
    qa = torch.empty((M, E), dtype=torch.int8, device="cuda")
    qd = torch.empty((M, F), dtype=torch.int8, device="cuda")
    aa = torch.empty((M, 2), dtype=torch.int32, device="cuda")
    ad = torch.empty((M, 2), dtype=torch.int32, device="cuda")
    h = torch.empty((M, F), dtype=torch.float32, device="cuda")
    y = torch.empty((M, E), dtype=torch.float32, device="cuda")
    st = torch.cuda.current_stream()

    def gemms():
        pkg.gemm_silu(wg, wu, F, E, M, qa, aa, h, st)
        pkg.gemm(wd, E, F, M, qd, ad, None, y, st)

    def step():
        pkg.quant_act_rows(xa, M, E, qa, aa, st)
        pkg.quant_act_rows(xd, M, F, qd, ad, st)
        gemms()

    ops = 2.0 * M * (2 * F * E + E * F)
    ms, _ = time_device(step, args.steps, args.warmup, st, world)
    gms, _ = time_device(gemms, args.steps, args.warmup, st, world)
    err = pkg.gemm_error()
    peak, kind = int8_peak()
    tops = ops * args.steps * world / (ms / 1e3) / 1e12
    gtops = ops * args.steps / (gms / 1e3) / 1e12
    # e2e: host activations in (pinned), the down projection's outputs back,
    # every step, through the same C-ABI calls
    xa_p, xd_p = torch.from_numpy(xa_h).pin_memory(), torch.from_numpy(xd_h).pin_memory()
    y_p = torch.empty((M, E), dtype=torch.float32).pin_memory()

    def e2e_step():
        xa.copy_(xa_p, non_blocking=True)
        xd.copy_(xd_p, non_blocking=True)
        step()
        y_p.copy_(y, non_blocking=True)
        st.synchronize()

    for _ in range(max(args.warmup, 3)):
        e2e_step()
    if world > 1:
        torch.distributed.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    te = max_over_ranks(time.perf_counter() - t0, world)
    out = {"workload": "prefill_ffn_2b4t (512 tokens: quant + gate/up SiLU + quant + down)",
           "value": round(tops, 2), "unit": "int8 TOP/s", "ms_per_step": round(ms / args.steps, 4),
           "ops_per_step": ops, "device_error": err,
           "e2e": {"value": round(ops * args.steps * world / te / 1e12, 2), "unit": "int8 TOP/s",
                   "h2d_bytes_per_step": int(xa_h.nbytes + xd_h.nbytes), "d2h_bytes_per_step": int(4 * M * E),
                   "api": "sllm_cuda_i2s_quant_act_rows + sllm_cuda_i2s_gemm_silu + sllm_cuda_i2s_gemm, "
                          "pinned host activations in and outputs back every step, wall clock"},
           "roofline": {"bound": "tensor", "kernel": "i2s_gemm_kernel (gate/up pair + down)",
                        "achieved": round(gtops, 1), "peak": round(peak, 1), "unit": "TOP/s",
                        "frac": round(gtops / peak, 4), "peak_source": kind,
                        "frac_of_2x_measured_bf16": round(gtops / bf16_x2_peak(), 4),
                        "gemm_ms_per_step": round(gms / args.steps, 4)}}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:     # N = 1 only
        import oracle
        if oracle.reference_available():
            ref = oracle.Reference()
            pool = ref.pool(os.cpu_count() or 1)
            dots = np.zeros(F, np.int32)
            wgh, wuh, wdh = (L[f"blk.0.{n}.weight"] for n in ("ffn_gate", "ffn_up", "ffn_down"))
            n_tok, t0 = 0, time.perf_counter()
            while time.perf_counter() - t0 < 5.0 and n_tok < M:
                # per token, as the reference's prefill: quantise, GEMV (pooled)
                q, _, _ = ref.quant_act(xa_h[n_tok])
                pool.gemv(wgh, F, E, q, dots)
                pool.gemv(wuh, F, E, q, dots)
                q, _, _ = ref.quant_act(xd_h[n_tok])
                pool.gemv(wdh, E, F, q, dots)
                n_tok += 1
            dt = time.perf_counter() - t0
            out["cpu_reference"] = {"value": round(2.0 * (2 * F * E + E * F) * n_tok / dt / 1e12, 4),
                                    "unit": "int8 TOP/s", "cores": pool.threads, "kind": "reference",
                                    "cpu": cpu_model(),
                                    "sample": f"{n_tok} of the 512 tokens, per-token quant + 3 pooled GEMVs, "
                                              f"{dt:.1f} s"}
    del m
    return out


GEMV_COPIES = 128


def gemv_bytes(rows, n):
    """Algorithmic bytes of one configs[0] GEMV: the packed codes, the f32
    scale after them, the f32 input and the f32 outputs."""
    return rows * n // 4 + 4 + 4 * n + 4 * rows


def gemv_leg(pkg, synth, local, rank, world, args):
    """the single 6912 x 2560 GEMV (quantise, ternary dot,
    epilogue), L2-cold: a step runs it over 128 distinct weight copies
    (566 MB, 4.5x the L2) with one shared f32 N(0,1) input. Timed two ways:
    128 back-to-back sllm_cuda_i2s_gemv_f32 launches (one CUDA graph per step,
    plain launches as a caller makes them), and one sllm_cuda_gemv_batch_run
    (the 128 GEMVs as one persistent engine launch)."""
    import torch
    rows, n, count = 6912, 2560, GEMV_COPIES
    nb = rows * n // 4
    stride = (nb + 32 + 255) // 256 * 256
    rng = np.random.default_rng(500 + rank)
    host = np.zeros((count, stride), np.uint8)
    host[:, :nb] = synth.LUT81[rng.integers(0, 81, size=(count, nb), dtype=np.uint8)]
    scales = rng.uniform(0.01, 0.1, count).astype(np.float32)
    host[:, nb:nb + 4] = scales.view(np.uint8).reshape(count, 4)
    wdev = torch.from_numpy(host).cuda()
    del host
    ws = [wdev[i] for i in range(count)]
    x_h = np.random.default_rng(600 + rank).standard_normal(n).astype(np.float32)
    x = torch.from_numpy(x_h).cuda()
    y = torch.empty((count, rows), dtype=torch.float32, device="cuda")
    y1 = torch.empty((count, rows), dtype=torch.float32, device="cuda")
    unit = gemv_bytes(rows, n)
    side = torch.cuda.Stream()

    # (a) back-to-back launches, recorded once into a graph
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        for i in range(count):               # warm-up outside the capture
            pkg.gemv_f32(ws[i], rows, n, x, y1[i], None, side)
        side.synchronize()
        with torch.cuda.graph(g, stream=side):
            for i in range(count):
                pkg.gemv_f32(ws[i], rows, n, x, y1[i], None, side)
    st = torch.cuda.current_stream()
    ms_l, _ = time_device(g.replay, args.steps, args.warmup, st, world)

    # (b) the same 128 GEMVs as one engine launch
    batch = pkg.GemvBatch(ws, rows, n, local)
    run = lambda: batch.run(x, y, 0, st)
    ms_e, _ = time_device(run, args.steps, args.warmup, st, world)
    torch.cuda.synchronize()
    err = batch.error()
    same = bool(torch.equal(y.view(torch.int32), y1.view(torch.int32)))

    # e2e: the input up from pinned memory, the 128 GEMVs, every output back
    x_p = torch.from_numpy(x_h).pin_memory()
    y_p = torch.empty((count, rows), dtype=torch.float32).pin_memory()

    def e2e_step():
        x.copy_(x_p, non_blocking=True)
        batch.run(x, y, 0, st)
        y_p.copy_(y, non_blocking=True)
        st.synchronize()

    for _ in range(max(args.warmup, 3)):
        e2e_step()
    if world > 1:
        torch.distributed.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    te = max_over_ranks(time.perf_counter() - t0, world)
    peak, peak_kind = peaks()
    step_bytes = unit * count
    gbs_e = step_bytes * args.steps * world / (ms_e / 1e3) / 1e9
    gbs_l = step_bytes * args.steps * world / (ms_l / 1e3) / 1e9
    per_e = step_bytes * args.steps / (ms_e / 1e3) / 1e9       # this rank's kernel
    per_l = step_bytes * args.steps / (ms_l / 1e3) / 1e9
    out = {"workload": "gemv_6912x2560 (configs[0]: one GEMV, 128 distinct weight copies per step, shared x)",
           "value": round(gbs_e, 1), "unit": "GB/s", "bytes_per_gemv": unit, "gemvs_per_step": count,
           "l2": "inputs larger than L2: 128 distinct copies (566 MB, 4.5x the 126 MB L2) per step, no flush",
           "engine": {"api": "sllm_cuda_gemv_batch_run (one persistent launch of 128 GEMVs)",
                      "ms_per_step": round(ms_e / args.steps, 4), "us_per_gemv": round(ms_e / args.steps / count * 1e3, 3),
                      "gbs": round(gbs_e, 1), "device_error": err, "outputs_equal_launches": same},
           "launches": {"api": "128 x sllm_cuda_i2s_gemv_f32 (plain launches, one CUDA graph per step)",
                        "ms_per_step": round(ms_l / args.steps, 4),
                        "us_per_gemv": round(ms_l / args.steps / count * 1e3, 3), "gbs": round(gbs_l, 1),
                        "frac": round(per_l / peak, 4)},
           "e2e": {"value": round(step_bytes * args.steps * world / te / 1e9, 1), "unit": "GB/s",
                   "h2d_bytes_per_step": 4 * n, "d2h_bytes_per_step": 4 * rows * count,
                   "api": "sllm_cuda_gemv_batch_run, pinned input up and every output back per step, wall clock"},
           "roofline": {"bound": "hbm", "kernel": "i2s_engine_kernel<5,14> (128 GEMVs, one launch)",
                        "achieved": round(per_e, 1), "peak": peak, "unit": "GB/s", "frac": round(per_e / peak, 4),
                        "peak_source": peak_kind, "bytes_per_launch": step_bytes}}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import oracle
        if oracle.reference_available():
            ref = oracle.Reference()
            pool = ref.pool(os.cpu_count() or 1)
            hw = wdev[:16].cpu().numpy()
            dots = np.zeros(rows, np.int32)
            k, t0 = 0, time.perf_counter()
            while time.perf_counter() - t0 < 5.0:
                # sllm_i2s_quant_act, pooled sllm_i2s_gemv (src/forward.c:196-205), the epilogue
                q, s_, total = ref.quant_act(x_h)
                w = hw[k % 16]
                pool.gemv(w, rows, n, q, dots)
                ws_ = np.float32(w[nb:nb + 4].view(np.float32)[0])
                _ = (dots - total).astype(np.float32) * (ws_ / np.float32(s_))
                k += 1
            dt = time.perf_counter() - t0
            out["cpu_reference"] = {"value": round(unit * k / dt / 1e9, 3), "unit": "GB/s", "cores": pool.threads,
                                    "kind": "reference", "cpu": cpu_model(),
                                    "sample": f"{k} GEMVs over 16 of the copies (70 MB, beyond the host caches) "
                                              f"in {dt:.1f} s"}
    batch.close()
    del g
    return out


def tp_decode_leg(pkg, local, rank, world, args):
    """greedy decode of the 80-layer 8192 / 28672 ternary model
    (64 / 8 heads, vocab 128256), weights generated on each GPU from a seeded
    hash, tensor-parallel over the `world` ranks with NCCL (one rank: no
    exchange). Prompt 128 ids, 128 greedy tokens, batch 1; wall clock, max
    over ranks. The token checksum is the same for every rank count."""
    import torch
    sd = pkg.abi.TpSynthDesc(n_layer=80, n_embd=8192, n_ff=28672, n_head=64, n_head_kv=8, n_vocab=128256,
                             f_rms_eps=1e-5, rope_freq_base=500000.0, seed=4242)
    n_prompt, n_new = 128, 128
    comm = None
    if world > 1:
        obj = [pkg.tp_unique_id() if rank == 0 else None]
        torch.distributed.broadcast_object_list(obj, src=0)
        comm = pkg.TpComm(obj[0], world, rank, local)
    t0 = time.perf_counter()
    model = pkg.TpModel(world, rank, local, synth=sd)
    build_s = time.perf_counter() - t0
    ctx = model.ctx(n_prompt + n_new + 8, comm)
    prompt = np.random.default_rng(7).integers(0, sd.n_vocab, n_prompt).astype(np.int32)
    rc, _ = ctx.generate(prompt[:8], 8)          # warm-up: builds the step graph
    assert rc == 0, rc
    ctx.reset()
    if world > 1:
        torch.distributed.barrier()
    t0 = time.perf_counter()
    rc, toks = ctx.generate(prompt, n_new)
    dt = time.perf_counter() - t0
    assert rc == 0, rc
    dev_ms = max_over_ranks(ctx.last_run_ms(), world)
    dt = max_over_ranks(dt, world)
    E, F, H, Hkv, V = sd.n_embd, sd.n_ff, sd.n_head, sd.n_head_kv, sd.n_vocab
    i2s_layer = (E * E * 2 + 2 * (Hkv * 128) * E + 3 * F * E) // 4
    per_gpu_bytes = (sd.n_layer * i2s_layer + V * E * 2) / world
    steps = n_prompt + n_new
    kv_row = 2 * sd.n_layer * Hkv * 128 * 4 / world
    run_bytes_gpu = per_gpu_bytes * steps + kv_row * sum(range(1, steps + 1))
    peak, peak_kind = peaks()
    achieved = run_bytes_gpu / (dev_ms / 1e3) / 1e9
    out = {"workload": "tp_decode_80L_8192 (configs[4], batch 1)", "tp": world,
           "tokens_per_s": round(steps / dt, 2), "ms_per_token": round(dt / steps * 1e3, 4),
           "steps": f"{n_prompt} prompt + {n_new} greedy, one token per step",
           "weight_gbs_per_gpu": round(per_gpu_bytes * steps / dt / 1e9, 1),
           "model_gb_per_gpu": round(model.bytes() / 1e9, 2), "build_s": round(build_s, 2),
           "token_checksum": int(sum((i + 1) * int(v) for i, v in enumerate(toks))),
           "device_ms_per_token": round(dev_ms / steps, 4),
           "roofline": {"bound": "hbm", "kernel": "per-token step graph (engine layer programs, attention, "
                                                  "exchanges, head), device time, slowest rank",
                        "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s per GPU",
                        "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                        "bytes_per_step_per_gpu": int(run_bytes_gpu / steps)},
           "layer_gemvs": ("persistent engine: per layer one program of four stages (Q/K/V, attention, O, "
                           "gate/up) and one for down" if ctx.fused_layers() > 0 else
                           "persistent engine (one program per phase)") if ctx.uses_engine() else "per-GEMV kernels",
           "exchange": {"none": "none (one rank)", "nccl": "NCCL all-gather / int32 all-reduce in the step graph",
                        "p2p": ("fused peer exchange: per layer one engine program storing into every rank's "
                                "memory and waiting on flags inside its stages" if ctx.fused_exchange() else
                                "one-shot peer-memory exchange kernels (P2P stores + epoch flags) in the step "
                                "graph")}[ctx.exchange_kind()]}
    ctx.close()
    out["batch16"] = tp_batch_run(pkg, model, comm, sd, prompt, n_new, world, rank, per_gpu_bytes, kv_row)
    model.close()
    if comm is not None:
        comm.close()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_reference"] = tp_cpu_reference(sd, steps)
    return out


def tp_batch_run(pkg, model, comm, sd, prompt, n_new, world, rank, per_gpu_bytes, kv_row, n_seq=16):
    """configs[4] at batch 16: 16 sequences (the batch-1 prompt and 15 more
    seeded prompts of the same length) stepped together, every layer GEMV one
    16-token GEMM on the tensor cores. tokens/s counts every sequence's
    tokens (prompt and generated) over the wall clock of the generate call,
    max over ranks. Sequence 0's tokens are the batch-1 run's."""
    import torch
    n_prompt = len(prompt)
    prompts = np.random.default_rng(11).integers(0, sd.n_vocab, (n_seq, n_prompt)).astype(np.int32)
    prompts[0] = prompt
    b = model.batch(n_seq, n_prompt + n_new + 8, comm)
    rc, _ = b.generate(prompts[:, :8], 8)          # warm-up: builds the step graph
    assert rc == 0, rc
    b.reset()
    if world > 1:
        torch.distributed.barrier()
    t0 = time.perf_counter()
    rc, toks = b.generate(prompts, n_new)
    dt = time.perf_counter() - t0
    assert rc == 0, rc
    dev_ms = max_over_ranks(b.last_run_ms(), world)
    dt = max_over_ranks(dt, world)
    b.close()
    steps = n_prompt + n_new
    run_bytes_gpu = per_gpu_bytes * steps + n_seq * kv_row * sum(range(1, steps + 1))
    peak, peak_kind = peaks()
    achieved = run_bytes_gpu / (dev_ms / 1e3) / 1e9
    return {"workload": f"tp_decode_80L_8192 (configs[4], batch {n_seq})", "tp": world, "batch": n_seq,
            "tokens_per_s": round(n_seq * steps / dt, 1), "ms_per_step": round(dt / steps * 1e3, 4),
            "device_ms_per_step": round(dev_ms / steps, 4),
            "steps": f"{n_prompt} prompt + {n_new} greedy positions per sequence, {n_seq} sequences per step",
            "token_checksum_seq0": int(sum((i + 1) * int(v) for i, v in enumerate(toks[0]))),
            "token_checksum_all": int(sum((i + 1) * int(v) for i, v in enumerate(toks.reshape(-1)))),
            "roofline": {"bound": "hbm", "kernel": "batch step graph (skinny tcgen05 GEMMs, attention, exchanges, "
                                                  "batched head), device time, slowest rank",
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s per GPU",
                         "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                         "bytes_per_step_per_gpu": int(run_bytes_gpu / steps)},
            "layer_gemms": "skinny tcgen05 kind::i8 GEMM: 128 weight rows (M) x 16 tokens (N) per CTA"}


def tp_cpu_reference(sd, steps):
    """configs[4] on the host cores with the reference's own kernels. Its model
    API refuses 80 layers (SLLM_LAYER_MAX 64), so the reference kernels run
    chained per layer, pooled as src/forward.c:196-205 pools them: one layer
    of the configs[4] geometry (sllm_rms_norm, sllm_i2s_quant_act, pooled
    sllm_i2s_gemv and the epilogue for all seven projections, SiLU, residual
    adds) is timed and multiplied by 80, and the pooled F16 head
    (sllm_dot_f16_f32 per row, src/forward.c:215-233) is timed on 16384 of the
    128256 rows and scaled. Attention at these lengths is a small share and
    is left out, so the figure is an upper bound on the reference's speed."""
    import oracle
    if not oracle.reference_available():
        return None
    synth = importlib.import_module("saphira-llm_b200.synth")
    ref = oracle.Reference()
    cores = os.cpu_count() or 1
    pool = ref.pool(cores)
    cfg = synth.Config(n_layer=1, n_embd=sd.n_embd, n_ff=sd.n_ff, n_head=sd.n_head, n_head_kv=sd.n_head_kv,
                       n_vocab=64)
    m = synth.SynthModel(cfg, seed=sd.seed)
    d = m.desc()
    E, F, G = cfg.n_embd, cfg.n_ff, cfg.n_embd_gqa
    x = np.random.default_rng(1).standard_normal(E).astype(np.float32)
    scratch = np.zeros(4 * E + 2 * G + 3 * F, np.float32)
    qbuf = np.zeros(max(E, F), np.int8)
    dots = np.zeros(max(E, F), np.int32)
    pool.layer_chain(d, 0, x, scratch, qbuf, dots)
    n_l, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < 4.0:
        pool.layer_chain(d, 0, x, scratch, qbuf, dots)
        n_l += 1
    t_layer = (time.perf_counter() - t0) / n_l
    rows = 16384
    embd = (np.random.default_rng(2).standard_normal(rows * E).astype(np.float32) * 0.02).astype(np.float16)
    embd = embd.view(np.uint16)
    logits = np.zeros(rows, np.float32)
    xn = np.random.default_rng(3).standard_normal(E).astype(np.float32)
    pool.lm_head(embd, rows, E, xn, logits)
    n_h, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < 2.0:
        pool.lm_head(embd, rows, E, xn, logits)
        n_h += 1
    t_head = (time.perf_counter() - t0) / n_h * (sd.n_vocab / rows)
    t_tok = sd.n_layer * t_layer + t_head
    return {"tokens_per_s": round(1.0 / t_tok, 3), "ms_per_token": round(t_tok * 1e3, 1), "cores": pool.threads,
            "cpu": cpu_model(), "kind": "reference",
            "sample": f"one {E}/{F} layer chained {n_l} times ({t_layer * 1e3:.1f} ms each) x {sd.n_layer} layers, "
                      f"plus the F16 head timed on {rows} rows x {n_h} and scaled to {sd.n_vocab}; "
                      "attention left out (upper bound on the reference's speed)"}


def decode_leg(pkg, synth, local, rank, world, args):
    """2B-4T random init, prompt 64, 256 greedy tokens."""
    import torch
    cfg = synth.Config()
    m = synth.SynthModel(cfg, seed=4242 + rank)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    model = pkg.Model(m.desc(), local)           # sllm_cuda_model_upload: pinned, double-buffered staging
    up_s = time.perf_counter() - t0
    t0 = time.perf_counter()
    plain = torch.from_numpy(m.image).to(f"cuda:{local}")   # one pageable copy of the same image, for scale
    torch.cuda.synchronize()
    pg_s = time.perf_counter() - t0
    del plain
    ctx = model.ctx(64 + 256)
    prompt = np.random.default_rng(7 + rank).integers(0, cfg.n_vocab, 64).astype(np.int32)
    rc, toks = ctx.generate(prompt, 256)         # warm-up (captures the step graph)
    assert rc == 0, pkg.lib().sllm_cuda_last_error()
    runs, dev = [], []
    for _ in range(3):
        ctx.reset()
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        t0 = time.perf_counter()
        rc, toks2 = ctx.generate(prompt, 256)
        runs.append(time.perf_counter() - t0)
        dev.append(ctx.last_run_ms())
        assert rc == 0 and toks2.tolist() == toks.tolist()
    best = min(runs)
    best = max_over_ranks(best, world)
    dev_ms = max_over_ranks(min(dev), world)
    # algorithmic bytes of the 320 steps: every weight once per step, and at
    # step t the KV rows of positions 0..t (fp32 K and V of every layer)
    kv_row = 2 * cfg.n_layer * cfg.n_embd_gqa * 4
    run_bytes = model.weight_bytes() * 320 + kv_row * sum(range(1, 321))
    peak, peak_kind = peaks()
    achieved = run_bytes / (dev_ms / 1e3) / 1e9
    out = {"workload": "greedy_decode_2b4t", "prompt": 64, "new_tokens": 256,
           "tokens_per_s": round((64 + 256) * world / best, 1), "ms_per_token": round(best / 320 * 1e3, 4),
           "weight_gbs": round(model.weight_bytes() * 320 * world / best / 1e9, 1),
           "api": "sllm_cuda_generate_greedy (host prompt in, ids out, wall clock; best of 3)",
           "device_ms_per_token": round(dev_ms / 320, 4),
           "roofline": {"bound": "hbm", "kernel": "decode step graph (embed, i2s_engine_kernel<5,14> over the "
                                                  "30 layers, lm_head_kernel), device time of the 320 steps",
                        "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                        "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                        "bytes_per_step": int(run_bytes / 320)},
           "token_checksum": int(np.sum(toks.astype(np.int64) * np.arange(1, 257)) % 1000003),
           "upload": {"api": "sllm_cuda_model_upload (pinned double-buffered staging, host copy threads)",
                      "bytes": int(model.weight_bytes()), "s": round(up_s, 3),
                      "gbs": round(model.weight_bytes() / up_s / 1e9, 2),
                      "pageable_copy_gbs": round(m.image.nbytes / pg_s / 1e9, 2)}}
    # the fp16 KV option: the same decode with every cached value rounded to
    # half; it has no reference output, so it reports its token agreement
    c16 = model.ctx(64 + 256, kv_f16=True)
    rc16, t16 = c16.generate(prompt, 256)
    c16.reset()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    rc16, t16 = c16.generate(prompt, 256)
    w16 = time.perf_counter() - t0
    if rc16 == 0:
        first = next((i for i in range(256) if t16[i] != toks[i]), 256)
        out["kv_f16"] = {"tokens_per_s": round(320 / w16, 1), "device_ms_per_token": round(c16.last_run_ms() / 320, 4),
                         "tokens_equal_to_fp32": int(np.sum(t16 == toks)), "first_difference": first,
                         "kv_bytes_per_position": int(kv_row // 2)}
    c16.close()
    # the reference's own 256 tokens for this model and prompt (the fixture
    # tests/golden/make_golden.py --large wrote from the compiled reference)
    fx = os.path.join(ROOT, "tests", "golden", "decode_large.json")
    if rank == 0 and os.path.exists(fx):
        case = {c["name"]: c for c in json.load(open(fx))}.get("configs2-2b4t-30l-64+256")
        if case is not None and case["prompt"] == prompt.tolist():
            out["tokens_identical_to_reference"] = toks.tolist() == case["tokens"]
            out["reference_tokens"] = "tests/golden/decode_large.json (all 256, same model seed and prompt)"
    if rank == 0 and world == 1 and not args.no_cpu_baseline:     # N = 1 only
        import oracle
        if oracle.reference_available():
            ref = oracle.Reference()
            cores = os.cpu_count() or 1
            rm = ref.model(m.image, 64, cores)
            n_new = 8
            rm.generate(prompt[:8], 1)
            rm.reset()
            t0 = time.perf_counter()
            rcr, rt = rm.generate(prompt[:8], n_new)
            dt = time.perf_counter() - t0
            ctx.reset()
            rc, g = ctx.generate(prompt[:8], n_new)
            out["cpu_reference"] = {"tokens_per_s": round((8 + n_new) / dt, 2), "cores": cores, "cpu": cpu_model(),
                                    "kind": "reference",
                                    "sample": f"prompt 8 + {n_new} greedy tokens through sllm_generate_greedy",
                                    "tokens_identical": bool(rcr == 0 and g.tolist() == rt.tolist())}
            del rm
    ctx.close()
    model.close()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-tp", action="store_true")
    ap.add_argument("--no-gemv", action="store_true")
    ap.add_argument("--copies", type=int, default=N_COPIES,
                    help="layer copies per step (default 32; smaller only for profiler captures)")
    ap.add_argument("--leg", choices=["decode", "prefill", "tp", "gemv"], default=None,
                    help="run only this secondary leg and print its object (for profiler captures; "
                         "no headline line)")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
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

    if args.leg is not None:
        leg = {"decode": lambda: decode_leg(pkg, synth, local, rank, world, args),
               "prefill": lambda: prefill_leg(pkg, synth, local, rank, world, args),
               "tp": lambda: tp_decode_leg(pkg, local, rank, world, args),
               "gemv": lambda: gemv_leg(pkg, synth, local, rank, world, args)}[args.leg]()
        if rank == 0:
            print(json.dumps({"leg": args.leg, **leg}))
        if world > 1:
            torch.distributed.destroy_process_group()
        return

    copies = args.copies
    cfg = synth.Config(n_layer=copies, n_vocab=256)
    m = synth.SynthModel(cfg, seed=1 + rank)
    model = pkg.Model(m.desc(), local)
    ctx = model.ctx(8)
    E = cfg.n_embd
    stream = torch.cuda.current_stream()
    xs_n, ys_n = pkg.projection_sizes(model)
    xs_host = np.random.default_rng(rank).standard_normal(xs_n).astype(np.float32)
    xs = torch.from_numpy(xs_host).cuda()
    ys = torch.empty(ys_n * copies, dtype=torch.float32, device="cuda")
    step_bytes = projection_bytes(cfg, m) * copies

    # headline: independent projections. The clock sampler runs over a second
    # of the same workload right before the timed region and over the timed
    # region itself (a timed region of ~10 ms is too short to sample alone).
    fn = lambda: ctx.layer_projections_device(0, copies, xs, ys, stream)
    with ClockSampler(local) as clk:
        t_end = time.perf_counter() + 1.0
        while time.perf_counter() < t_end:
            for _ in range(20):
                fn()
            torch.cuda.synchronize()
        fn()
        torch.cuda.synchronize()
        k0 = pkg.kernel_launches()
        fn()
        torch.cuda.synchronize()
        launches = pkg.kernel_launches() - k0      # kernels per step, as the library counts them
        ms, per = time_device(fn, args.steps, args.warmup, stream, world)
    clocks = clk.summary()
    value = step_bytes * args.steps * world / (ms / 1e3) / 1e9
    # one launch alone (idle device before and after, events around it): the
    # figure without the overlap of consecutive launches that `value` includes
    singles = []
    for _ in range(10):
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        fn()
        e1.record(stream)
        torch.cuda.synchronize()
        singles.append(e0.elapsed_time(e1))
    single_ms = float(np.median(singles))

    # e2e: host buffers through sllm_cuda_layer_projections
    host_in = torch.from_numpy(xs_host).pin_memory()
    host_out = torch.empty(ys_n * copies, dtype=torch.float32).pin_memory()
    lib = pkg.lib()
    for _ in range(2):
        assert lib.sllm_cuda_layer_projections(model.h, ctx.h, 0, copies, host_in.data_ptr(),
                                               host_out.data_ptr()) == 0
    if world > 1:
        torch.distributed.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        assert lib.sllm_cuda_layer_projections(model.h, ctx.h, 0, copies, host_in.data_ptr(),
                                               host_out.data_ptr()) == 0
    te = max_over_ranks(time.perf_counter() - t0, world)
    e2e = step_bytes * args.steps * world / te / 1e9

    # secondary: the dependent chain
    xc = torch.from_numpy(np.random.default_rng(rank).standard_normal(E).astype(np.float32)).cuda()
    cms, _ = time_device(lambda: ctx.layer_chain_device(0, copies, xc, stream), args.steps, args.warmup,
                         stream, world)
    chain_gbs = chain_bytes(cfg, m) * copies * args.steps * world / (cms / 1e3) / 1e9

    peak, peak_kind = peaks()
    per_launch_bytes = step_bytes / launches
    achieved = per_launch_bytes / ((ms / 1e3) / (args.steps * launches)) / 1e9
    traffic = None
    prof = os.path.join(ROOT, "profiles", "i2s_engine_projections_traffic.txt")
    if os.path.exists(prof):
        for line in open(prof):
            if line.startswith("traffic_bytes_per_launch"):
                traffic = int(line.split()[1])
    out = {
        "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": round(ms / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8 x ternary -> int32, f32", "data": "synthetic (seeded random-init 2B-4T layers, N(0,1) inputs)",
        "config": {"workload": "layer_projections_2b4t", "layer_copies_per_step": copies,
                   "weights_mb_per_step": round(step_bytes / 1e6, 1), "bytes_per_step": step_bytes,
                   "l2": "inputs larger than L2: 32 distinct layer copies (4.4x the 126 MB L2) per step, no flush",
                   "parallelism": f"replicas x{world}", "batch": 1},
        "roofline": {"bound": "hbm",
                     "kernel": ("i2s_engine_kernel (one persistent launch per step: "
                                f"{copies} layers x 7 GEMVs)") if launches == 1 else
                               f"i2s_gemv_kernel ({launches} launches per step)",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                     "bytes_per_launch": int(per_launch_bytes), "traffic": traffic,
                     "timing": f"{args.steps} back-to-back launches between two events (consecutive launches "
                               "overlap: each takes the SMs as the previous one's CTAs exit)",
                     "single_launch": {"ms": round(single_ms, 4),
                                       "achieved": round(step_bytes / (single_ms / 1e3) / 1e9, 1),
                                       "frac": round(step_bytes / (single_ms / 1e3) / 1e9 / peak, 4),
                                       "timing": "one launch between two events on an idle device, median of 10"}},
        "e2e": {"value": round(e2e, 3), "unit": "GB/s", "h2d_bytes_per_step": 4 * xs_n,
                "d2h_bytes_per_step": 4 * ys_n * copies,
                "api": "sllm_cuda_layer_projections (host buffers, wall clock)"},
        "gpu_launches": launches * args.steps,
        "clocks": clocks,
        "chain": {"workload": "layer_chain_2b4t (dependent: decode layer without attention)",
                  "value": round(chain_gbs, 3), "unit": "GB/s", "frac": round(chain_gbs / world / peak, 4),
                  "ms_per_step": round(cms / args.steps, 4),
                  "us_per_layer": round(cms / args.steps / copies * 1e3, 3)},
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:     # N = 1 only
        out["cpu_baseline"] = cpu_baseline_sample(cfg, m, xs_host)
    ctx.close()
    model.close()
    del m
    if not args.no_gemv:
        out["gemv"] = gemv_leg(pkg, synth, local, rank, world, args)
    if not args.no_prefill:
        out["prefill"] = prefill_leg(pkg, synth, local, rank, world, args)
    if not args.no_tp:
        out["tp_decode"] = tp_decode_leg(pkg, local, rank, world, args)
    if not args.no_decode:
        out["decode"] = decode_leg(pkg, synth, local, rank, world, args)
    if rank == 0:
        print(json.dumps(out))
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
