"""Failure injection on the host, without a device: a communicator set-up
that NCCL refuses is reported as SLLM_CUDA_ERR_COMM (-62) with its message,
and the next set-up is not affected by the injection."""
import ctypes as C

import pytest


def test_injected_comm_init_failure(pkg):
    L = pkg.lib()
    L.sllm_cuda_test_fail_next(2, 1)
    uid = (C.c_uint8 * 128)()
    h = C.c_void_p()
    rc = L.sllm_cuda_tp_comm_init(uid, 2, 0, 0, C.byref(h))
    L.sllm_cuda_test_fail_next(2, 0)
    if rc == -4:
        pytest.skip("no libnccl.so.2 on this machine")
    assert rc == -62 and not h.value
    assert b"injected" in L.sllm_cuda_last_error()
