"""ctypes access to saphira-llm built with the CUDA row
(saphira-llm_b200/reference_row/_build/libsaphira_llm_row.so): the
reference's own public API (src/gguf.c, src/forward.c), with the backend
chosen through sllm_backend_request. Test helper only."""
import ctypes as C
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ROW_DIR = os.path.join(ROOT, "saphira-llm_b200", "reference_row", "_build")
ROW_SO = os.path.join(ROW_DIR, "libsaphira_llm_row.so")
CLI = os.path.join(ROW_DIR, "saphira-llm")
TGBENCH = os.path.join(ROW_DIR, "saphira-llm-tgbench")
CPU, CUDA, AUTO = 0, 1, 2

_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")


def available():
    return os.path.exists(ROW_SO)


class Row:
    def __init__(self):
        L = self.lib = C.CDLL(ROW_SO)
        vp = C.c_void_p
        L.sllm_gguf_open_memory.argtypes = [vp, C.c_size_t, vp, C.c_char_p, C.c_size_t]
        L.sllm_gguf_close.argtypes = [vp]
        L.sllm_model_load.argtypes = [vp, C.POINTER(vp)]
        L.sllm_model_free.argtypes = [vp]
        L.sllm_model_backend.argtypes = [vp]
        L.sllm_ctx_new.argtypes = [vp, C.c_int32, C.POINTER(vp)]
        L.sllm_ctx_free.argtypes = [vp]
        L.sllm_ctx_reset.argtypes = [vp]
        L.sllm_ctx_last_logits.argtypes = [vp]
        L.sllm_ctx_last_logits.restype = C.POINTER(C.c_float)
        L.sllm_forward_chunk.argtypes = [vp, vp, _i32p, C.c_int32, C.c_int32, _f32p]
        L.sllm_generate_greedy.argtypes = [vp, vp, vp, C.c_int32, C.c_int32, _i32p]
        L.sllm_state_save.argtypes = [vp, vp, C.c_char_p]
        L.sllm_state_load.argtypes = [vp, vp, C.c_char_p]
        L.sllm_backend_request.argtypes = [C.c_int]

    def open(self, image, backend, n_ctx):
        return RowModel(self, image, backend, n_ctx)


class RowModel:
    """A model loaded through sllm_model_load on the requested backend row,
    with one context. `rc` is sllm_model_load's status."""

    def __init__(self, row, image, backend, n_ctx):
        L = self.L = row.lib
        self.image = image                       # borrowed by the gguf: keep it alive
        self.g = (C.c_uint8 * 256)()             # sllm_gguf is 80 bytes
        self.m, self.c = C.c_void_p(), C.c_void_p()
        err = C.create_string_buffer(256)
        assert L.sllm_gguf_open_memory(image.ctypes.data, image.nbytes, self.g, err, 256) == 0, err.value
        L.sllm_backend_request(backend)
        self.rc = L.sllm_model_load(self.g, C.byref(self.m))
        self.n_vocab = None
        if self.rc == 0:
            self.rc = L.sllm_ctx_new(self.m, n_ctx, C.byref(self.c))

    def backend(self):
        return self.L.sllm_model_backend(self.m)

    def generate(self, prompt, n_new):
        prompt = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(max(n_new, 1), np.int32)
        rc = self.L.sllm_generate_greedy(self.m, self.c, prompt.ctypes.data if prompt.size else None,
                                         prompt.size, n_new, out)
        return rc, out[:n_new]

    def forward_chunk(self, tokens, base, n_vocab):
        tokens = np.ascontiguousarray(tokens, np.int32)
        logits = np.zeros(tokens.size * n_vocab, np.float32)
        rc = self.L.sllm_forward_chunk(self.m, self.c, tokens, tokens.size, base, logits)
        return rc, logits.reshape(tokens.size, n_vocab)

    def last_logits(self, n_vocab):
        p = self.L.sllm_ctx_last_logits(self.c)
        return np.ctypeslib.as_array(p, shape=(n_vocab,)).copy()

    def save(self, path):
        return self.L.sllm_state_save(self.m, self.c, path.encode())

    def load(self, path):
        return self.L.sllm_state_load(self.m, self.c, path.encode())

    def reset(self):
        self.L.sllm_ctx_reset(self.c)

    def close(self):
        if self.c:
            self.L.sllm_ctx_free(self.c)
            self.c = C.c_void_p()
        if self.m:
            self.L.sllm_model_free(self.m)
            self.m = C.c_void_p()
        self.L.sllm_gguf_close(self.g)


def run_cli(model_path, backend, prompt="Hello world", n=8):
    """The reference's CLI (src/main.c with --backend): (exit code, generated text, stderr)."""
    import subprocess
    r = subprocess.run([CLI, "-m", model_path, "-p", prompt, "-n", str(n), "-t", "1", "--backend", backend],
                       capture_output=True, text=True, timeout=300)
    text = r.stdout.split("\nsllm_bench")[0]
    return r.returncode, text, r.stderr


def run_tgbench(model_path, backend, n=16):
    """The reference's decode benchmark (bench/tg_bench.c with --backend):
    (exit code, token checksum or None, stdout)."""
    import subprocess
    r = subprocess.run([TGBENCH, "-m", model_path, "-n", str(n), "-t", "1", "-r", "2", "-w", "1", "--no-calibrate",
                        "--backend", backend], capture_output=True, text=True, timeout=300)
    cs = None
    for line in r.stdout.splitlines():
        if line.startswith("token_checksum"):
            cs = int(line.split()[1])
    return r.returncode, cs, r.stdout
