"""The device softmax's libm expf restatement (saphira-llm_b200/csrc/libm_expf.h)
must equal the host libm's expf -- the one the reference softmax tail calls
(src/ops.c:413-417) -- on every float. Exhaustive: 2^32 inputs, a few seconds
with OpenMP."""
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))


def test_expf_restatement_is_bit_exact_on_every_float(tmp_path):
    exe = tmp_path / "expf_check"
    subprocess.run(["gcc", "-O2", "-fopenmp", "-ffp-contract=off", "-march=x86-64-v3",
                    os.path.join(HERE, "libm_expf_check.c"), "-o", str(exe), "-lm"], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "mismatch 0 " in r.stdout
