"""Per-thread resources of the persistent engine, read from ptxas on a CPU.

The engine kernel hands its by-value parameter block to helpers by reference.
Without `__grid_constant__` on that parameter every thread copied the whole
block into local memory at launch: a 232-248-byte stack frame per thread that
cost 0.07-0.36 ms per token in the 80-layer tensor-parallel decode as the
block grew. With it the block stays in the parameter space and only a few
spilled registers remain on the stack. This test compiles engine.cu with the
library's own flags and `-Xptxas -v` and checks every engine instance.
"""
import os
import re
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "saphira-llm_b200")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

# the flags of saphira-llm_b200/Makefile (NVFLAGS), plus the resource report
FLAGS = ["-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-fmad=false",
         "-prec-div=true", "-prec-sqrt=true", "-ftz=false", "-Xcompiler", "-fPIC", "-Xcompiler",
         "-ffp-contract=off", "-Xptxas", "-v"]

# a copy of the parameter block alone is over 200 bytes; spills are tens
MAX_STACK = 64


def _ptxas_report(src):
    if not (os.path.exists(NVCC) or shutil.which("nvcc")):
        pytest.skip("nvcc not available")
    nvcc = NVCC if os.path.exists(NVCC) else shutil.which("nvcc")
    r = subprocess.run([nvcc, *FLAGS, "-c", os.path.join(PKG, "csrc", src), "-o", os.devnull],
                       cwd=PKG, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    return r.stdout + r.stderr


def _stack_frames(report):
    """{mangled kernel name: stack frame bytes} from a ptxas -v report."""
    out, name = {}, None
    for line in report.splitlines():
        m = re.search(r"Compiling entry function '([^']+)'", line)
        if m:
            name = m.group(1)
            continue
        m = re.search(r"(\d+) bytes stack frame", line)
        if m and name is not None:
            out[name] = int(m.group(1))
            name = None
    return out


def test_engine_instances_keep_their_parameters_out_of_local_memory():
    frames = _stack_frames(_ptxas_report("engine.cu"))
    engine = {k: v for k, v in frames.items() if "i2s_engine_kernel" in k}
    assert len(engine) >= 10, sorted(frames)      # every compiled width pair, plain, f16-cache and exchange
    big = {k: v for k, v in engine.items() if v > MAX_STACK}
    assert not big, f"stack frames over {MAX_STACK} bytes (a local copy of the parameter block?): {big}"
