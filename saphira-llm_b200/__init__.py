"""saphira-llm B200 backend: Python binding of libsllm_cuda.so (include/sllm_cuda.h).

The product is the C ABI in libsllm_cuda.so; saphira-llm's C11 host code calls
it directly. This module binds the same entry points with
ctypes for the tests, the benchmark and Python callers. Device buffers are
passed as raw pointers (or torch CUDA tensors, whose data_ptr() is used); the
library never falls back to the CPU: loading fails loudly if the built library
is missing, and every call returns its status as an exception.
"""
import ctypes as C
import os

import numpy as np

from . import abi

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libsllm_cuda.so")

_lib = None


class SllmCudaError(RuntimeError):
    def __init__(self, status, where, msg=""):
        self.status = status
        super().__init__(f"{where}: {abi.STATUS_NAMES.get(status, status)} ({status}) {msg}".rstrip())


def build():
    """Compile libsllm_cuda.so in place (nvcc, sm_100a)."""
    import subprocess
    subprocess.run(["make", "-s", "-C", HERE, "-j4"], check=True)


def lib():
    """The loaded libsllm_cuda.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise FileNotFoundError(f"{LIB_PATH} is not built: run `make -C saphira-llm_b200`")
    L = C.CDLL(LIB_PATH)
    vp, sz, i32 = C.c_void_p, C.c_size_t, C.c_int32
    L.sllm_cuda_status_string.argtypes = [C.c_int]
    L.sllm_cuda_status_string.restype = C.c_char_p
    L.sllm_cuda_last_error.restype = C.c_char_p
    L.sllm_cuda_probe.argtypes = [C.POINTER(C.c_int)] * 3
    L.sllm_cuda_i2s_quant_act.argtypes = [vp, sz, vp, vp, vp]
    L.sllm_cuda_i2s_gemv.argtypes = [vp, sz, sz, vp, vp, vp]
    L.sllm_cuda_i2s_gemv_f32.argtypes = [vp, sz, sz, vp, vp, vp, vp]
    L.sllm_cuda_i2s_quant_act_rows.argtypes = [vp, sz, sz, vp, vp, vp]
    L.sllm_cuda_i2s_gemm.argtypes = [vp, sz, sz, sz, vp, vp, vp, vp, vp]
    L.sllm_cuda_i2s_gemm_silu.argtypes = [vp, vp, sz, sz, sz, vp, vp, vp, vp]
    L.sllm_cuda_test_gemm_error.restype = C.c_int
    L.sllm_cuda_test_gemm_form.argtypes = [C.c_int]
    L.sllm_cuda_test_gemm_form.restype = None
    L.sllm_cuda_test_gemm_strided.argtypes = [vp, i32, i32, i32, vp, i32, vp, vp, vp, vp]
    L.sllm_cuda_tp_unique_id.argtypes = [vp]
    L.sllm_cuda_tp_comm_init.argtypes = [vp, i32, i32, i32, C.POINTER(vp)]
    L.sllm_cuda_tp_comm_free.argtypes = [vp]
    L.sllm_cuda_tp_model_upload.argtypes = [C.POINTER(abi.ModelDesc), i32, i32, i32, C.POINTER(vp)]
    L.sllm_cuda_tp_model_synth.argtypes = [C.POINTER(abi.TpSynthDesc), i32, i32, i32, C.POINTER(vp)]
    L.sllm_cuda_tp_model_free.argtypes = [vp]
    L.sllm_cuda_tp_model_bytes.argtypes = [vp]
    L.sllm_cuda_tp_model_bytes.restype = sz
    L.sllm_cuda_tp_vocab_range.argtypes = [vp, C.POINTER(i32), C.POINTER(i32)]
    L.sllm_cuda_tp_ctx_new.argtypes = [vp, vp, i32, C.POINTER(vp)]
    L.sllm_cuda_tp_ctx_free.argtypes = [vp]
    L.sllm_cuda_tp_batch_new.argtypes = [vp, vp, i32, i32, C.POINTER(vp)]
    L.sllm_cuda_tp_batch_free.argtypes = [vp]
    L.sllm_cuda_tp_batch_free.restype = None
    L.sllm_cuda_tp_batch_reset.argtypes = [vp]
    L.sllm_cuda_tp_batch_generate_greedy.argtypes = [vp, vp, i32, i32, vp]
    L.sllm_cuda_tp_batch_last_logits.argtypes = [vp, i32, vp]
    L.sllm_cuda_test_tp_batch_last_run_ms.argtypes = [vp]
    L.sllm_cuda_test_tp_batch_last_run_ms.restype = C.c_float
    L.sllm_cuda_test_tp_batch_generate_group.argtypes = [vp, i32, vp, i32, i32, vp]
    L.sllm_cuda_tp_ctx_reset.argtypes = [vp]
    L.sllm_cuda_tp_generate_greedy.argtypes = [vp, vp, i32, i32, vp]
    L.sllm_cuda_tp_last_logits.argtypes = [vp, vp]
    L.sllm_cuda_test_tp_generate_group.argtypes = [C.POINTER(vp), i32, vp, i32, i32, vp]
    L.sllm_cuda_test_tp_uses_engine.argtypes = [vp]
    L.sllm_cuda_test_tp_fused_layers.argtypes = [vp]
    L.sllm_cuda_test_tp_exchange_kind.argtypes = [vp]
    L.sllm_cuda_test_tp_fused_exchange.argtypes = [vp]
    L.sllm_cuda_model_upload.argtypes = [C.POINTER(abi.ModelDesc), C.c_int, C.POINTER(vp)]
    L.sllm_cuda_model_free.argtypes = [vp]
    L.sllm_cuda_model_weight_bytes.argtypes = [vp]
    L.sllm_cuda_model_weight_bytes.restype = sz
    L.sllm_cuda_ctx_new.argtypes = [vp, i32, C.POINTER(vp)]
    L.sllm_cuda_ctx_new_kv.argtypes = [vp, i32, i32, C.POINTER(vp)]
    L.sllm_cuda_ctx_free.argtypes = [vp]
    L.sllm_cuda_ctx_reset.argtypes = [vp]
    L.sllm_cuda_ctx_n_past.argtypes = [vp]
    L.sllm_cuda_ctx_n_past.restype = i32
    L.sllm_cuda_forward_chunk.argtypes = [vp, vp, vp, i32, i32, vp, vp]
    L.sllm_cuda_generate_greedy.argtypes = [vp, vp, vp, i32, i32, vp]
    L.sllm_cuda_ctx_last_logits.argtypes = [vp, vp]
    L.sllm_cuda_layer_chain.argtypes = [vp, vp, i32, i32, vp, vp]
    L.sllm_cuda_layer_chain_device.argtypes = [vp, vp, i32, i32, vp, vp]
    L.sllm_cuda_layer_projections_sizes.argtypes = [vp, C.POINTER(sz)]
    L.sllm_cuda_layer_projections_sizes.restype = sz
    L.sllm_cuda_layer_projections.argtypes = [vp, vp, i32, i32, vp, vp]
    L.sllm_cuda_layer_projections_device.argtypes = [vp, vp, i32, i32, vp, vp, vp]
    L.sllm_cuda_test_set_force_fallback.argtypes = [C.c_int]
    L.sllm_cuda_test_fallback_count.restype = C.c_int
    L.sllm_cuda_test_kernel_launches.restype = C.c_longlong
    L.sllm_cuda_test_engine_split.argtypes = [vp, vp, vp, vp, i32, vp, i32, i32, vp]
    L.sllm_cuda_test_tp_plan.argtypes = [i32, i32, i32, i32, i32, i32, i32, i32, vp]
    L.sllm_cuda_test_projection_split.argtypes = [i32, i32, i32, i32]
    L.sllm_cuda_test_fail_next.argtypes = [C.c_int, C.c_int]
    L.sllm_cuda_test_engine_faults.argtypes = [C.c_int, C.c_int, C.c_double]
    L.sllm_cuda_state_save.argtypes = [vp, vp, C.c_char_p]
    L.sllm_cuda_state_load.argtypes = [vp, vp, C.c_char_p]
    L.sllm_cuda_ctx_kv_export.argtypes = [vp, vp, vp]
    L.sllm_cuda_ctx_kv_import.argtypes = [vp, vp, vp, i32, vp]
    L.sllm_cuda_gemv_batch_new.argtypes = [vp, sz, sz, sz, C.c_int, C.POINTER(vp)]
    L.sllm_cuda_gemv_batch_run.argtypes = [vp, vp, sz, vp, vp]
    L.sllm_cuda_gemv_batch_free.argtypes = [vp]
    L.sllm_cuda_test_gemv_batch_error.argtypes = [vp]
    L.sllm_cuda_test_ctx_last_run_ms.argtypes = [vp]
    L.sllm_cuda_test_ctx_last_run_ms.restype = C.c_float
    L.sllm_cuda_test_tp_ctx_last_run_ms.argtypes = [vp]
    L.sllm_cuda_test_tp_ctx_last_run_ms.restype = C.c_float
    _lib = L
    return L


def _check(rc, where):
    if rc != abi.OK:
        raise SllmCudaError(rc, where, lib().sllm_cuda_last_error().decode(errors="replace"))


def _ptr(t):
    """A raw device (or host) address from a torch tensor, numpy array or int."""
    if t is None:
        return None
    if isinstance(t, int):
        return t
    if hasattr(t, "data_ptr"):
        return t.data_ptr()
    if hasattr(t, "ctypes"):
        return t.ctypes.data
    raise TypeError(type(t))


def _stream(s):
    if s is None:
        return None
    if isinstance(s, int):
        return s
    return s.cuda_stream


def probe():
    n, ma, mi = C.c_int(), C.c_int(), C.c_int()
    rc = lib().sllm_cuda_probe(C.byref(n), C.byref(ma), C.byref(mi))
    return rc, n.value, (ma.value, mi.value)


# kernel level (device pointers, asynchronous) ---------------------------------
def quant_act(x, n, q, act, stream=None):
    _check(lib().sllm_cuda_i2s_quant_act(_ptr(x), n, _ptr(q), _ptr(act), _stream(stream)), "quant_act")


def gemv(w, n_rows, n, q, out, stream=None):
    _check(lib().sllm_cuda_i2s_gemv(_ptr(w), n_rows, n, _ptr(q), _ptr(out), _stream(stream)), "gemv")


def gemv_f32(w, n_rows, n, x, y, dots=None, stream=None):
    _check(lib().sllm_cuda_i2s_gemv_f32(_ptr(w), n_rows, n, _ptr(x), _ptr(y), _ptr(dots), _stream(stream)),
           "gemv_f32")


def quant_act_rows(x, m, n, q, acts, stream=None):
    """Per-token quantisation of a row-major [m][n] batch (device pointers)."""
    _check(lib().sllm_cuda_i2s_quant_act_rows(_ptr(x), m, n, _ptr(q), _ptr(acts), _stream(stream)),
           "quant_act_rows")


def gemm(w, n_rows, n, m, q, acts, dots=None, y=None, stream=None):
    """Prefill GEMM on the tensor cores: per-token GEMV dots and/or the f32
    epilogue for m tokens at once (device pointers)."""
    _check(lib().sllm_cuda_i2s_gemm(_ptr(w), n_rows, n, m, _ptr(q), _ptr(acts), _ptr(dots), _ptr(y),
                                    _stream(stream)), "gemm")


def gemm_silu(w_gate, w_up, n_rows, n, m, q, acts, h, stream=None):
    """h = silu(gate) * up for m tokens at once (device pointers)."""
    _check(lib().sllm_cuda_i2s_gemm_silu(_ptr(w_gate), _ptr(w_up), n_rows, n, m, _ptr(q), _ptr(acts), _ptr(h),
                                         _stream(stream)), "gemm_silu")


class GemvBatch:
    """`count` independent GEMVs of one shape as one persistent launch
    (sllm_cuda_gemv_batch_*). `ws` are device tensors or addresses."""

    def __init__(self, ws, n_rows, n, device=0):
        arr = (C.c_void_p * len(ws))(*[_ptr(w) for w in ws])
        self._keep = ws
        self.h = C.c_void_p()
        _check(lib().sllm_cuda_gemv_batch_new(arr, len(ws), n_rows, n, device, C.byref(self.h)), "gemv_batch_new")

    def run(self, x, y, x_stride=0, stream=None):
        _check(lib().sllm_cuda_gemv_batch_run(self.h, _ptr(x), x_stride, _ptr(y), _stream(stream)), "gemv_batch_run")

    def error(self):
        return lib().sllm_cuda_test_gemv_batch_error(self.h)

    def close(self):
        if getattr(self, "h", None):
            lib().sllm_cuda_gemv_batch_free(self.h)
            self.h = None


def gemm_strided(w, n_rows, k, m, q, lda, acts, dots=None, y=None, stream=None):
    """The GEMM over k columns of a row-major activation matrix whose rows
    are lda bytes apart (device pointers)."""
    _check(lib().sllm_cuda_test_gemm_strided(_ptr(w), n_rows, k, m, _ptr(q), lda, _ptr(acts), _ptr(dots), _ptr(y),
                                             _stream(stream)), "gemm_strided")


def set_gemm_form(form):
    """0: by size; 1: the 128-token tiles; 2: the skinny (<= 16 tokens) form."""
    lib().sllm_cuda_test_gemm_form(int(form))


def gemm_error():
    """The prefill kernels' device error word (0 = every bounded wait
    completed); synchronises and clears it."""
    return lib().sllm_cuda_test_gemm_error()


def set_force_fallback(on):
    lib().sllm_cuda_test_set_force_fallback(1 if on else 0)


def fallback_count():
    return lib().sllm_cuda_test_fallback_count()


def kernel_launches():
    """Kernels the library has put on streams in this process (graph launches
    count their kernel nodes)."""
    return lib().sllm_cuda_test_kernel_launches()


# model level (host pointers) -------------------------------------------------
class Model:
    """A model uploaded to one device (sllm_cuda_model_upload)."""

    def __init__(self, desc, device=0):
        self.desc = desc
        self.h = C.c_void_p()
        _check(lib().sllm_cuda_model_upload(C.byref(desc), device, C.byref(self.h)), "model_upload")

    def weight_bytes(self):
        return lib().sllm_cuda_model_weight_bytes(self.h)

    def close(self):
        if getattr(self, "h", None):
            try:
                lib().sllm_cuda_model_free(self.h)
            except (TypeError, AttributeError):      # interpreter shutdown
                pass
            self.h = None

    def __del__(self):
        self.close()

    def ctx(self, n_ctx, kv_f16=False):
        return Ctx(self, n_ctx, kv_f16)


class Ctx:
    """One sequence's device state: KV cache, scratch, decode graph."""

    def __init__(self, model, n_ctx, kv_f16=False):
        import numpy as np
        self._np = np
        self.model = model
        self.n_vocab = model.desc.n_vocab
        self.n_embd = model.desc.n_embd
        self.h = C.c_void_p()
        _check(lib().sllm_cuda_ctx_new_kv(model.h, n_ctx, 1 if kv_f16 else 0, C.byref(self.h)), "ctx_new")

    def close(self):
        if getattr(self, "h", None):
            try:
                lib().sllm_cuda_ctx_free(self.h)
            except (TypeError, AttributeError):      # interpreter shutdown
                pass
            self.h = None

    def __del__(self):
        self.close()

    def reset(self):
        lib().sllm_cuda_ctx_reset(self.h)

    def n_past(self):
        return lib().sllm_cuda_ctx_n_past(self.h)

    def forward_chunk(self, tokens, base, want_logits=True):
        np = self._np
        tokens = np.ascontiguousarray(tokens, np.int32)
        logits = np.empty((tokens.size, self.n_vocab), np.float32) if want_logits else None
        am = np.empty(tokens.size, np.int32)
        rc = lib().sllm_cuda_forward_chunk(self.model.h, self.h, tokens.ctypes.data, tokens.size, base,
                                           None if logits is None else logits.ctypes.data, am.ctypes.data)
        return rc, logits, am

    def generate(self, prompt, n_new):
        np = self._np
        prompt = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(max(n_new, 1), np.int32)
        rc = lib().sllm_cuda_generate_greedy(self.model.h, self.h, prompt.ctypes.data if prompt.size else None,
                                             prompt.size, n_new, out.ctypes.data)
        return rc, out[:n_new]

    def last_logits(self):
        np = self._np
        out = np.empty(self.n_vocab, np.float32)
        rc = lib().sllm_cuda_ctx_last_logits(self.h, out.ctypes.data)
        return None if rc != 0 else out

    def state_save(self, path):
        """sllm_cuda_state_save: the reference's SLKV v1 file."""
        return lib().sllm_cuda_state_save(self.model.h, self.h, os.fsencode(path))

    def state_load(self, path):
        return lib().sllm_cuda_state_load(self.model.h, self.h, os.fsencode(path))

    def last_run_ms(self):
        """Device time of the decode steps of the last forward / generate call."""
        return float(lib().sllm_cuda_test_ctx_last_run_ms(self.h))

    def layer_chain(self, layer_begin, n_layers, x):
        np = self._np
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty_like(x)
        _check(lib().sllm_cuda_layer_chain(self.model.h, self.h, layer_begin, n_layers, x.ctypes.data,
                                           out.ctypes.data), "layer_chain")
        return out

    def layer_projections(self, layer_begin, n_layers, x):
        np = self._np
        xs, ys = projection_sizes(self.model)
        x = np.ascontiguousarray(x, np.float32)
        assert x.size == xs
        y = np.empty(ys * n_layers, np.float32)
        _check(lib().sllm_cuda_layer_projections(self.model.h, self.h, layer_begin, n_layers, x.ctypes.data,
                                                 y.ctypes.data), "layer_projections")
        return y.reshape(n_layers, ys)

    def layer_projections_device(self, layer_begin, n_layers, x_dev, y_dev, stream=None):
        _check(lib().sllm_cuda_layer_projections_device(self.model.h, self.h, layer_begin, n_layers, _ptr(x_dev),
                                                        _ptr(y_dev), _stream(stream)), "layer_projections_device")

    def layer_chain_device(self, layer_begin, n_layers, x_dev, stream=None):
        _check(lib().sllm_cuda_layer_chain_device(self.model.h, self.h, layer_begin, n_layers, _ptr(x_dev),
                                                  _stream(stream)), "layer_chain_device")


def projection_sizes(model):
    """(input floats, output floats per layer) of the layer-projection API."""
    ys = C.c_size_t()
    xs = lib().sllm_cuda_layer_projections_sizes(model.h, C.byref(ys))
    return int(xs), int(ys.value)


# tensor parallel (one rank per GPU) ---------------------------------------------
def tp_unique_id():
    """The group identity rank 0 creates and hands to the other ranks (bytes)."""
    buf = (C.c_uint8 * abi.TP_ID_BYTES)()
    _check(lib().sllm_cuda_tp_unique_id(buf), "tp_unique_id")
    return bytes(buf)


class TpComm:
    def __init__(self, uid, n_ranks, rank, device):
        self.h = C.c_void_p()
        buf = (C.c_uint8 * abi.TP_ID_BYTES).from_buffer_copy(uid)
        _check(lib().sllm_cuda_tp_comm_init(buf, n_ranks, rank, device, C.byref(self.h)), "tp_comm_init")

    def close(self):
        if self.h:
            lib().sllm_cuda_tp_comm_free(self.h)
            self.h = C.c_void_p()


class TpModel:
    """Rank `rank`'s shard of a model: from host tensors (`desc`, a ModelDesc)
    or generated on the device (`synth`, a TpSynthDesc)."""

    def __init__(self, n_ranks, rank, device=0, desc=None, synth=None):
        self.h = C.c_void_p()
        self._keep = desc
        if desc is not None:
            _check(lib().sllm_cuda_tp_model_upload(C.byref(desc), n_ranks, rank, device, C.byref(self.h)),
                   "tp_model_upload")
        else:
            _check(lib().sllm_cuda_tp_model_synth(C.byref(synth), n_ranks, rank, device, C.byref(self.h)),
                   "tp_model_synth")

    def vocab_range(self):
        v0, n = C.c_int32(), C.c_int32()
        _check(lib().sllm_cuda_tp_vocab_range(self.h, C.byref(v0), C.byref(n)), "tp_vocab_range")
        return v0.value, n.value

    def bytes(self):
        return lib().sllm_cuda_tp_model_bytes(self.h)

    def ctx(self, n_ctx, comm=None):
        return TpCtx(self, n_ctx, comm)

    def batch(self, n_seq, n_ctx, comm=None):
        return TpBatch(self, n_seq, n_ctx, comm)

    def close(self):
        if self.h:
            lib().sllm_cuda_tp_model_free(self.h)
            self.h = C.c_void_p()


class TpCtx:
    def __init__(self, model, n_ctx, comm=None):
        self.model = model
        self.h = C.c_void_p()
        _check(lib().sllm_cuda_tp_ctx_new(model.h, comm.h if comm is not None else None, n_ctx, C.byref(self.h)),
               "tp_ctx_new")

    def generate(self, prompt, n_new):
        prompt = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(max(n_new, 1), np.int32)
        rc = lib().sllm_cuda_tp_generate_greedy(self.h, prompt.ctypes.data if prompt.size else None, prompt.size,
                                                 n_new, out.ctypes.data)
        return rc, out[:n_new]

    def last_logits(self):
        v0, n = self.model.vocab_range()
        out = np.zeros(n, np.float32)
        _check(lib().sllm_cuda_tp_last_logits(self.h, out.ctypes.data), "tp_last_logits")
        return v0, out

    def reset(self):
        _check(lib().sllm_cuda_tp_ctx_reset(self.h), "tp_ctx_reset")

    def last_run_ms(self):
        """Device time of the decode steps of the last generate call on this rank."""
        return float(lib().sllm_cuda_test_tp_ctx_last_run_ms(self.h))

    def uses_engine(self):
        return bool(lib().sllm_cuda_test_tp_uses_engine(self.h))

    def fused_layers(self):
        return int(lib().sllm_cuda_test_tp_fused_layers(self.h))

    def fused_exchange(self):
        return bool(lib().sllm_cuda_test_tp_fused_exchange(self.h))

    def exchange_kind(self):
        """'none' (one rank), 'nccl' or 'p2p' (the one-shot peer-memory exchange)."""
        return ("none", "nccl", "p2p")[lib().sllm_cuda_test_tp_exchange_kind(self.h)]

    def close(self):
        if self.h:
            lib().sllm_cuda_tp_ctx_free(self.h)
            self.h = C.c_void_p()


class TpBatch:
    """n_seq <= 16 sequences decoded together over one shard
    (sllm_cuda_tp_batch_*), each with its own KV cache."""

    def __init__(self, model, n_seq, n_ctx, comm=None):
        self.model = model
        self.n_seq = n_seq
        self.h = C.c_void_p()
        _check(lib().sllm_cuda_tp_batch_new(model.h, comm.h if comm is not None else None, n_seq, n_ctx,
                                            C.byref(self.h)), "tp_batch_new")

    def generate(self, prompts, n_new):
        """prompts: [n_seq][n_prompt] token ids; returns (status, [n_seq][n_new])."""
        prompts = np.ascontiguousarray(prompts, np.int32).reshape(self.n_seq, -1)
        out = np.zeros((self.n_seq, max(n_new, 1)), np.int32)
        rc = lib().sllm_cuda_tp_batch_generate_greedy(self.h, prompts.ctypes.data if prompts.size else None,
                                                      prompts.shape[1], n_new, out.ctypes.data)
        return rc, out[:, :n_new].copy() if n_new > 0 else out[:, :0]

    def last_logits(self, seq):
        v0, n = self.model.vocab_range()
        out = np.zeros(n, np.float32)
        _check(lib().sllm_cuda_tp_batch_last_logits(self.h, seq, out.ctypes.data), "tp_batch_last_logits")
        return v0, out

    def reset(self):
        _check(lib().sllm_cuda_tp_batch_reset(self.h), "tp_batch_reset")

    def last_run_ms(self):
        return float(lib().sllm_cuda_test_tp_batch_last_run_ms(self.h))

    def close(self):
        if self.h:
            lib().sllm_cuda_tp_batch_free(self.h)
            self.h = C.c_void_p()


def tp_batch_generate_group(batches, prompts, n_new):
    """Batch decode over the batches of ranks 0..N-1 on one device (device
    copies instead of NCCL)."""
    n_seq = batches[0].n_seq
    prompts = np.ascontiguousarray(prompts, np.int32).reshape(n_seq, -1)
    arr = (C.c_void_p * len(batches))(*[b.h.value for b in batches])
    out = np.zeros((n_seq, max(n_new, 1)), np.int32)
    rc = lib().sllm_cuda_test_tp_batch_generate_group(arr, len(batches), prompts.ctypes.data if prompts.size else None,
                                                      prompts.shape[1], n_new, out.ctypes.data)
    return rc, out[:, :n_new].copy()


def tp_generate_group(ctxs, prompt, n_new):
    """Greedy decode over the contexts of ranks 0..N-1 on one device (device
    copies instead of NCCL; a test of the sharding on one GPU)."""
    prompt = np.ascontiguousarray(prompt, np.int32)
    arr = (C.c_void_p * len(ctxs))(*[c.h.value for c in ctxs])
    out = np.zeros(max(n_new, 1), np.int32)
    rc = lib().sllm_cuda_test_tp_generate_group(arr, len(ctxs), prompt.ctypes.data if prompt.size else None,
                                                prompt.size, n_new, out.ctypes.data)
    return rc, out[:n_new]
