"""ctypes mirror of include/sllm_cuda.h: the structs and status codes of the C ABI.

Only plain data lives here, so both the product binding (``__init__.py``) and
the test-side oracle wrapper can describe a model the same way.
"""
import ctypes as C

OK = 0
ERR_ARG = -1
ERR_NOMEM = -2
ERR_IO = -3
ERR_UNSUPPORTED = -4
ERR_TOO_LARGE = -36
ERR_DEVICE = -60
ERR_TIMEOUT = -61
ERR_COMM = -62

STATUS_NAMES = {
    OK: "ok", ERR_ARG: "bad argument", ERR_NOMEM: "out of memory", ERR_IO: "io error",
    ERR_UNSUPPORTED: "unsupported", ERR_TOO_LARGE: "too large", ERR_DEVICE: "device error",
    ERR_TIMEOUT: "device wait timed out", ERR_COMM: "collective failed",
}


class Act(C.Structure):
    """sllm_cuda_act == sllm_i2s_act (include/saphira_llm/i2s_gemm.h:37-40)."""
    _fields_ = [("scale", C.c_float), ("sum", C.c_int32)]


class LayerDesc(C.Structure):
    """sllm_cuda_layer_desc (the reference's sllm_layer, src/forward.c:47-54)."""
    _fields_ = [
        ("wq", C.c_void_p), ("wk", C.c_void_p), ("wv", C.c_void_p), ("wo", C.c_void_p),
        ("ffn_gate", C.c_void_p), ("ffn_up", C.c_void_p), ("ffn_down", C.c_void_p),
        ("attn_norm", C.c_void_p), ("attn_sub_norm", C.c_void_p),
        ("ffn_norm", C.c_void_p), ("ffn_sub_norm", C.c_void_p),
    ]


class ModelDesc(C.Structure):
    """sllm_cuda_model_desc (the reference's sllm_model, src/forward.c:56-76)."""
    _fields_ = [
        ("n_layer", C.c_int32), ("n_embd", C.c_int32), ("n_ff", C.c_int32),
        ("n_head", C.c_int32), ("n_head_kv", C.c_int32), ("n_vocab", C.c_int32),
        ("n_rot", C.c_int32), ("n_ctx_train", C.c_int32),
        ("f_rms_eps", C.c_float), ("rope_freq_base", C.c_float),
        ("tok_embd", C.c_void_p), ("output_norm", C.c_void_p),
        ("layers", C.POINTER(LayerDesc)),
    ]


LAYER_I2S = ("wq", "wk", "wv", "wo", "ffn_gate", "ffn_up", "ffn_down")
LAYER_NORMS = ("attn_norm", "attn_sub_norm", "ffn_norm", "ffn_sub_norm")


class TpSynthDesc(C.Structure):
    """sllm_cuda_tp_synth_desc: a seeded synthetic model generated on the device."""
    _fields_ = [
        ("n_layer", C.c_int32), ("n_embd", C.c_int32), ("n_ff", C.c_int32),
        ("n_head", C.c_int32), ("n_head_kv", C.c_int32), ("n_vocab", C.c_int32),
        ("f_rms_eps", C.c_float), ("rope_freq_base", C.c_float), ("seed", C.c_uint64),
    ]


TP_ID_BYTES = 128
