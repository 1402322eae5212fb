"""TEST INFRASTRUCTURE ONLY: ctypes access to the two CPU checkers.

* ``Oracle``    -- oracle/liboracle.so, this project's restatement of the
                   reference arithmetic (oracle/sllm_oracle.c).
* ``Reference`` -- oracle/_ref/libsllm_ref.so, the reference saphira-llm
                   library compiled from its own sources (oracle/Makefile),
                   driven through its public API (plus oracle/ref_glue.c).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module. The product path never does.
"""
import ctypes as C
import importlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
abi = importlib.import_module("saphira-llm_b200.abi")

# Where the reference source tree lies. Read in this one place; the Makefile,
# the build entry point and the tests take it from here.
REFERENCE_DIR = os.environ.get("SLLM_REFERENCE_DIR", "/root/reference")

ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libsllm_ref.so")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")


def build(ref=True):
    """Compile the restatement (and the reference, when its sources exist)."""
    import subprocess
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)
    if ref and os.path.isdir(os.path.join(REFERENCE_DIR, "src")):
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF={REFERENCE_DIR}"], check=True)


def _a(x, dt):
    return np.ascontiguousarray(x, dtype=dt)


class Oracle:
    def __init__(self, path=ORACLE_SO):
        if not os.path.exists(path):
            build(ref=False)
        L = self.lib = C.CDLL(path)
        L.orc_i2s_quant_act.argtypes = [_f32p, C.c_size_t, _i8p, C.POINTER(abi.Act)]
        L.orc_i2s_dot.argtypes = [_u8p, _i8p, C.c_size_t]
        L.orc_i2s_dot.restype = C.c_int32
        L.orc_i2s_gemv.argtypes = [_u8p, C.c_size_t, C.c_size_t, _i8p, _i32p]
        L.orc_i2s_gemv_f32.argtypes = [_u8p, C.c_size_t, C.c_size_t, _f32p, _f32p, _i32p]
        L.orc_i2s_epilogue.argtypes = [C.c_int32, C.c_int32, C.c_float, C.c_float]
        L.orc_i2s_epilogue.restype = C.c_float
        L.orc_i2s_pack_codes.argtypes = [_u8p, C.c_size_t, C.c_float, _u8p]
        L.orc_i2s_quantize_scaled_py.argtypes = [_f32p, C.c_size_t, C.c_float, _u8p]
        L.orc_i2s_code.argtypes = [_u8p, C.c_size_t]
        L.orc_i2s_code.restype = C.c_uint8
        L.orc_fp16_to_fp32.argtypes = [C.c_uint16]
        L.orc_fp16_to_fp32.restype = C.c_float
        L.orc_fp16_to_fp32_embd.argtypes = [C.c_uint16]
        L.orc_fp16_to_fp32_embd.restype = C.c_float
        L.orc_rms_norm.argtypes = [_f32p, _f32p, C.c_void_p, C.c_size_t, C.c_float]
        L.orc_v_expf.argtypes = [C.c_float]
        L.orc_v_expf.restype = C.c_float
        L.orc_softmax.argtypes = [_f32p, C.c_size_t]
        L.orc_silu.argtypes = [_f32p, C.c_size_t]
        L.orc_rope_neox.argtypes = [_f32p, C.c_size_t, C.c_int32, C.c_float]
        L.orc_dot_f16.argtypes = [_u16p, _f32p, C.c_size_t]
        L.orc_dot_f16.restype = C.c_float
        L.orc_argmax.argtypes = [_f32p, C.c_int32]
        L.orc_argmax.restype = C.c_int32
        L.orc_ctx_new.argtypes = [C.POINTER(abi.ModelDesc), C.c_int32, C.POINTER(C.c_void_p)]
        L.orc_ctx_free.argtypes = [C.c_void_p]
        L.orc_ctx_reset.argtypes = [C.c_void_p]
        L.orc_ctx_set_kv_f16.argtypes = [C.c_void_p, C.c_int]
        L.orc_fp32_to_fp16.argtypes = [C.c_float]
        L.orc_fp32_to_fp16.restype = C.c_uint16
        L.orc_ctx_n_past.argtypes = [C.c_void_p]
        L.orc_ctx_n_past.restype = C.c_int32
        L.orc_ctx_last_logits.argtypes = [C.c_void_p]
        L.orc_ctx_last_logits.restype = C.POINTER(C.c_float)
        L.orc_forward_chunk.argtypes = [C.POINTER(abi.ModelDesc), C.c_void_p, _i32p, C.c_int32,
                                        C.c_int32, _f32p]
        L.orc_generate_greedy.argtypes = [C.POINTER(abi.ModelDesc), C.c_void_p, _i32p, C.c_int32,
                                          C.c_int32, _i32p]
        L.orc_layer_chain.argtypes = [C.POINTER(abi.ModelDesc), C.c_int32, _f32p, _f32p]
        L.orc_set_threads.argtypes = [C.c_int]

    # kernels -----------------------------------------------------------
    def quant_act(self, x):
        x = _a(x, np.float32)
        q = np.empty(x.size, np.int8)
        act = abi.Act()
        self.lib.orc_i2s_quant_act(x, x.size, q, C.byref(act))
        return q, np.float32(act.scale), int(act.sum)

    def gemv(self, w, rows, n, q):
        out = np.empty(rows, np.int32)
        self.lib.orc_i2s_gemv(_a(w, np.uint8), rows, n, _a(q, np.int8), out)
        return out

    def gemv_f32(self, w, rows, n, x):
        y = np.empty(rows, np.float32)
        d = np.empty(rows, np.int32)
        self.lib.orc_i2s_gemv_f32(_a(w, np.uint8), rows, n, _a(x, np.float32), y, d)
        return y, d

    def epilogue(self, dot, s, act_scale, w_scale):
        return np.float32(self.lib.orc_i2s_epilogue(dot, s, act_scale, w_scale))

    def rms_norm(self, x, w, eps):
        x = _a(x, np.float32)
        dst = np.empty_like(x)
        wp = None if w is None else _a(w, np.float32)
        self.lib.orc_rms_norm(dst, x, None if wp is None else wp.ctypes.data, x.size, eps)
        return dst

    def softmax(self, x):
        x = _a(x, np.float32).copy()
        self.lib.orc_softmax(x, x.size)
        return x

    def silu(self, x):
        x = _a(x, np.float32).copy()
        self.lib.orc_silu(x, x.size)
        return x

    def rope(self, x, n_rot, pos, theta):
        x = _a(x, np.float32).copy()
        self.lib.orc_rope_neox(x, n_rot, pos, theta)
        return x

    def dot_f16(self, row, x):
        return np.float32(self.lib.orc_dot_f16(_a(row, np.uint16), _a(x, np.float32), row.size))

    def set_threads(self, n):
        self.lib.orc_set_threads(n)

    def layer_chain(self, desc, layer, x):
        x = _a(x, np.float32).copy()
        E, F = desc.n_embd, desc.n_ff
        G = (E // desc.n_head) * desc.n_head_kv
        scratch = np.zeros(4 * E + 2 * G + 3 * F, np.float32)
        self.lib.orc_layer_chain(C.byref(desc), layer, x, scratch)
        return x

    def ctx(self, desc, n_ctx, kv_f16=False):
        return OracleCtx(self, desc, n_ctx, kv_f16)

    def fp32_to_fp16(self, f):
        return int(self.lib.orc_fp32_to_fp16(float(f)))


class OracleCtx:
    def __init__(self, orc, desc, n_ctx, kv_f16=False):
        self.orc, self.desc, self.n_vocab = orc, desc, desc.n_vocab
        self.h = C.c_void_p()
        rc = orc.lib.orc_ctx_new(C.byref(desc), n_ctx, C.byref(self.h))
        if rc != 0:
            raise RuntimeError(f"orc_ctx_new: {rc}")
        if kv_f16:
            orc.lib.orc_ctx_set_kv_f16(self.h, 1)

    def __del__(self):
        if getattr(self, "h", None):
            self.orc.lib.orc_ctx_free(self.h)
            self.h = None

    def forward_chunk(self, tokens, base):
        tokens = _a(tokens, np.int32)
        logits = np.empty((tokens.size, self.n_vocab), np.float32)
        rc = self.orc.lib.orc_forward_chunk(C.byref(self.desc), self.h, tokens, tokens.size, base,
                                            logits.reshape(-1))
        return rc, logits

    def generate(self, prompt, n_new):
        prompt = _a(prompt, np.int32)
        out = np.zeros(max(n_new, 1), np.int32)
        rc = self.orc.lib.orc_generate_greedy(C.byref(self.desc), self.h, prompt, prompt.size,
                                              n_new, out)
        return rc, out[:n_new]

    def reset(self):
        self.orc.lib.orc_ctx_reset(self.h)

    def n_past(self):
        return self.orc.lib.orc_ctx_n_past(self.h)

    def last_logits(self):
        p = self.orc.lib.orc_ctx_last_logits(self.h)
        if not p:
            return None
        return np.ctypeslib.as_array(p, shape=(self.n_vocab,)).copy()


class Reference:
    """The compiled reference (oracle/_ref/libsllm_ref.so)."""

    def __init__(self, path=REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        L = self.lib = C.CDLL(path)
        L.sllm_i2s_quant_act.argtypes = [_f32p, C.c_size_t, _i8p, C.POINTER(abi.Act)]
        L.sllm_i2s_dot_scalar.argtypes = [_u8p, _i8p, C.c_size_t]
        L.sllm_i2s_dot_scalar.restype = C.c_int32
        L.sllm_i2s_dot.argtypes = [_u8p, _i8p, C.c_size_t]
        L.sllm_i2s_dot.restype = C.c_int32
        L.sllm_i2s_gemv.argtypes = [_u8p, C.c_size_t, C.c_size_t, _i8p, _i32p]
        L.sllm_i2s_epilogue.argtypes = [C.c_int32, C.c_int32, C.c_float, C.c_float]
        L.sllm_i2s_epilogue.restype = C.c_float
        L.sllm_i2s_quantize_scaled.argtypes = [_f32p, C.c_size_t, _u8p, C.c_float, C.c_int]
        L.sllm_i2s_quantize_scaled.restype = C.c_int
        L.sllm_i2s_scale.argtypes = [_u8p, C.c_size_t]
        L.sllm_i2s_scale.restype = C.c_float
        L.sllm_i2s_code.argtypes = [_u8p, C.c_size_t]
        L.sllm_i2s_code.restype = C.c_uint8
        L.sllm_fp16_to_fp32.argtypes = [C.c_uint16]
        L.sllm_fp16_to_fp32.restype = C.c_float
        L.sllm_rms_norm.argtypes = [_f32p, _f32p, C.c_void_p, C.c_size_t, C.c_float]
        L.sllm_softmax_inplace.argtypes = [_f32p, C.c_size_t]
        L.sllm_silu_inplace.argtypes = [_f32p, C.c_size_t]
        L.sllm_rope_inplace.argtypes = [_f32p, C.c_size_t, C.c_int32, C.c_float, C.c_float, C.c_int]
        L.sllm_dot_f16_f32.argtypes = [_u16p, _f32p, C.c_size_t]
        L.sllm_dot_f16_f32.restype = C.c_float
        L.sllm_argmax.argtypes = [_f32p, C.c_int32]
        L.sllm_argmax.restype = C.c_int32
        L.sllm_i2s_select_auto.argtypes = []
        L.refg_select_auto.restype = C.c_int
        L.refg_pool_create.argtypes = [C.c_int]
        L.refg_pool_create.restype = C.c_void_p
        L.refg_pool_destroy.argtypes = [C.c_void_p]
        L.refg_pool_threads.argtypes = [C.c_void_p]
        L.refg_model_open.argtypes = [C.c_void_p, C.c_size_t, C.c_int32, C.c_int, C.POINTER(C.c_void_p),
                                      C.c_char_p, C.c_size_t]
        L.refg_model_close.argtypes = [C.c_void_p]
        L.refg_ctx_reset.argtypes = [C.c_void_p]
        L.refg_forward_chunk.argtypes = [C.c_void_p, _i32p, C.c_int32, C.c_int32, _f32p]
        L.refg_generate_greedy.argtypes = [C.c_void_p, _i32p, C.c_int32, C.c_int32, _i32p]
        L.refg_last_logits.argtypes = [C.c_void_p, _f32p, C.c_int32]
        L.refg_gemv_pooled.argtypes = [C.c_void_p, _u8p, C.c_size_t, C.c_size_t, _i8p, _i32p]
        L.refg_layer_chain.argtypes = [C.c_void_p, C.POINTER(abi.ModelDesc), C.c_int32, _f32p, _f32p,
                                       _i8p, _i32p]
        L.refg_lm_head_pooled.argtypes = [C.c_void_p, _u16p, C.c_size_t, C.c_size_t, _f32p, _f32p]
        self.isa = L.refg_select_auto()

    def quant_act(self, x):
        x = _a(x, np.float32)
        q = np.empty(x.size, np.int8)
        act = abi.Act()
        self.lib.sllm_i2s_quant_act(x, x.size, q, C.byref(act))
        return q, np.float32(act.scale), int(act.sum)

    def gemv(self, w, rows, n, q):
        out = np.empty(rows, np.int32)
        self.lib.sllm_i2s_gemv(_a(w, np.uint8), rows, n, _a(q, np.int8), out)
        return out

    def rms_norm(self, x, w, eps):
        x = _a(x, np.float32)
        dst = np.empty_like(x)
        wp = None if w is None else _a(w, np.float32)
        self.lib.sllm_rms_norm(dst, x, None if wp is None else wp.ctypes.data, x.size, eps)
        return dst

    def softmax(self, x):
        x = _a(x, np.float32).copy()
        self.lib.sllm_softmax_inplace(x, x.size)
        return x

    def silu(self, x):
        x = _a(x, np.float32).copy()
        self.lib.sllm_silu_inplace(x, x.size)
        return x

    def rope(self, x, n_rot, pos, theta):
        x = _a(x, np.float32).copy()
        self.lib.sllm_rope_inplace(x, n_rot, pos, theta, 1.0, 0)   # SLLM_ROPE_NEOX == 0
        return x

    def dot_f16(self, row, x):
        return np.float32(self.lib.sllm_dot_f16_f32(_a(row, np.uint16), _a(x, np.float32), row.size))

    def pool(self, n_threads):
        return RefPool(self, n_threads)

    def model(self, image, n_ctx, n_threads=1):
        return RefModel(self, image, n_ctx, n_threads)


class RefPool:
    def __init__(self, ref, n):
        self.ref = ref
        self.p = ref.lib.refg_pool_create(n)
        self.threads = ref.lib.refg_pool_threads(self.p)

    def __del__(self):
        if getattr(self, "p", None):
            self.ref.lib.refg_pool_destroy(self.p)
            self.p = None

    def gemv(self, w, rows, n, q, out):
        self.ref.lib.refg_gemv_pooled(self.p, w, rows, n, q, out)

    def layer_chain(self, desc, layer, x, scratch, qbuf, dots):
        self.ref.lib.refg_layer_chain(self.p, C.byref(desc), layer, x, scratch, qbuf, dots)

    def lm_head(self, embd, n_rows, n_embd, x, out):
        self.ref.lib.refg_lm_head_pooled(self.p, embd, n_rows, n_embd, x, out)


class RefModel:
    def __init__(self, ref, image, n_ctx, n_threads):
        self.ref, self.image = ref, image       # the image must outlive the model
        self.h = C.c_void_p()
        err = C.create_string_buffer(512)
        rc = ref.lib.refg_model_open(image.ctypes.data, image.nbytes, n_ctx, n_threads,
                                     C.byref(self.h), err, 512)
        if rc != 0:
            raise RuntimeError(f"reference model load failed ({rc}): {err.value.decode()}")
        # n_vocab from the GGUF is not exposed by glue; callers pass it.

    def __del__(self):
        if getattr(self, "h", None):
            self.ref.lib.refg_model_close(self.h)
            self.h = None

    def forward_chunk(self, tokens, base, n_vocab):
        tokens = _a(tokens, np.int32)
        logits = np.empty((tokens.size, n_vocab), np.float32)
        rc = self.ref.lib.refg_forward_chunk(self.h, tokens, tokens.size, base, logits.reshape(-1))
        return rc, logits

    def generate(self, prompt, n_new):
        prompt = _a(prompt, np.int32)
        out = np.zeros(max(n_new, 1), np.int32)
        rc = self.ref.lib.refg_generate_greedy(self.h, prompt, prompt.size, n_new, out)
        return rc, out[:n_new]

    def reset(self):
        self.ref.lib.refg_ctx_reset(self.h)

    def last_logits(self, n_vocab):
        out = np.empty(n_vocab, np.float32)
        rc = self.ref.lib.refg_last_logits(self.h, out, n_vocab)
        return None if rc != 0 else out


def reference_available():
    return os.path.exists(REF_SO)
