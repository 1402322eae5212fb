"""The C ABI without a GPU: the library builds, loads, exports exactly what
include/*.h declares, and rejects bad arguments before touching a device."""
import ctypes as C
import os
import re
import subprocess

import pytest

from conftest import ROOT

HEADERS = [os.path.join(ROOT, "include", h) for h in ("sllm_cuda.h", "sllm_cuda_testing.h")]


def declared():
    names = set()
    for h in HEADERS:
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names |= set(re.findall(r"\b(sllm_cuda_\w+)\s*\(", src))
    return sorted(names)


def exported(path):
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T " in line}


@pytest.fixture(scope="module")
def built(pkg):
    if not os.path.exists(pkg.LIB_PATH):
        pkg.build()
    return pkg


def test_every_declared_symbol_is_exported(built):
    names = declared()
    assert len(names) >= 20
    syms = exported(built.LIB_PATH)
    missing = [n for n in names if n not in syms]
    assert not missing, missing
    # and nothing else leaks out of the library's C ABI
    extra = [s for s in syms if s.startswith("sllm_") and s not in names]
    assert not extra, extra


def test_library_loads_without_a_cuda_runtime_dependency(built):
    out = subprocess.run(["ldd", built.LIB_PATH], capture_output=True, text=True).stdout
    assert "libcudart" not in out          # static runtime: loads on a host without a driver
    built.lib()


def test_argument_errors_need_no_device(built, synth):
    L = built.lib()
    vp = C.c_void_p()
    assert L.sllm_cuda_model_upload(None, 0, C.byref(vp)) == -1
    assert L.sllm_cuda_i2s_gemv(None, 10, 256, None, None, None) == -1
    assert L.sllm_cuda_i2s_gemv(1024, 10, 200, 2048, 4096, None) == -1       # n % 128
    assert L.sllm_cuda_i2s_gemv(1024, 10, 65536, 2048, 4096, None) == -4     # above the widest K
    assert L.sllm_cuda_i2s_quant_act(None, 5, None, None, None) == -1
    assert L.sllm_cuda_ctx_new(None, 16, C.byref(vp)) == -1
    assert L.sllm_cuda_forward_chunk(None, None, None, 1, 0, None, None) == -1
    assert L.sllm_cuda_generate_greedy(None, None, None, 0, 1, None) == -1
    assert L.sllm_cuda_status_string(-61) == b"device wait timed out"
    assert b"generate_greedy" in L.sllm_cuda_last_error()
    assert L.sllm_cuda_i2s_gemv(1024, 10, 200, 2048, 4096, None) == -1
    assert b"multiple of 128" in L.sllm_cuda_last_error()
    # the batch decode API: no shard, too many sequences, no batch
    assert L.sllm_cuda_tp_batch_new(None, None, 16, 64, C.byref(vp)) == -1
    assert L.sllm_cuda_tp_batch_new(None, None, 17, 64, C.byref(vp)) == -1
    assert L.sllm_cuda_tp_batch_generate_greedy(None, None, 4, 4, None) == -1
    assert L.sllm_cuda_tp_batch_last_logits(None, 0, None) == -1


def test_unsupported_shapes_are_refused(built, synth):
    """Shape rules of sllm_cuda_model_upload, checked before any device call."""
    L = built.lib()
    cfg = synth.small_config(n_layer=1, n_embd=256, n_ff=512, n_head=4, n_head_kv=2, n_vocab=50)  # head dim 64
    m = synth.SynthModel(cfg, seed=1)
    vp = C.c_void_p()
    assert L.sllm_cuda_model_upload(C.byref(m.desc()), 0, C.byref(vp)) == -4
    d = synth.SynthModel(synth.small_config(n_layer=1, n_vocab=50), seed=1).desc()
    d.n_head_kv = 3                                         # 2 % 3 != 0
    assert L.sllm_cuda_model_upload(C.byref(d), 0, C.byref(vp)) == -1


def test_probe_reports_no_device_here(built):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a device is present; covered by the gpu tests")
    rc, n, cc = built.probe()
    assert rc == -4 and n == 0


def test_c11_caller_links_and_runs(built, tmp_path):
    """The headers compile as strict C11 (no C++ in any declaration) and a C
    program linked against the library runs the device-free calls:
    tests/c/abi_caller.c, the way saphira-llm's own C host code binds it."""
    exe = tmp_path / "abi_caller"
    lib_dir = os.path.dirname(built.LIB_PATH)
    cmd = ["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-pedantic", "-I", os.path.join(ROOT, "include"),
           os.path.join(ROOT, "tests", "c", "abi_caller.c"), built.LIB_PATH, "-Wl,-rpath," + lib_dir, "-o", str(exe)]
    out = subprocess.run(cmd, capture_output=True, text=True)
    assert out.returncode == 0, out.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0 and run.stdout.strip() == "ok", run.stdout + run.stderr
