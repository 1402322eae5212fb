"""Seeded synthetic bitnet-b1.58 models, written as a GGUF v3 image.

The benchmark configurations have no real checkpoint, so every weight is drawn
from a seeded generator with the distributions the benchmark specifies:

* I2_S tensors: codes i.i.d. uniform on {0, 1, 2} (ternary {-1, 0, +1} with
  p = 1/3 each) in the interleaved I2_S layout (src/quant.c:77-100,
  src/i2s_convert.c:137-176 of saphira-llm), followed by the f32 per-tensor
  scale ~ U(0.01, 0.1) and 28 zero bytes (src/i2s_convert.c:31-35).
  Because the four 2-bit fields of a packed byte are four independent
  elements, a byte is drawn directly as one of the 81 base-3 digit patterns,
  which is the same distribution as drawing and packing element codes.
* norm weights: f32 1 + 0.02 N(0, 1); token embedding / tied head: f16 of
  0.02 N(0, 1).

The whole model lives in one GGUF v3 byte image (FORMAT.md:9-30 of
saphira-llm), so the reference loads exactly these bytes through its own
sllm_gguf_open_memory + sllm_model_load, while the CUDA backend and the
restated oracle read the same tensors through a ModelDesc of pointers into
the image.
"""
import ctypes as C
import struct
from dataclasses import dataclass

import numpy as np

from . import abi

GGUF_ALIGN = 32
TYPE_F32, TYPE_F16, TYPE_I2_S = 0, 1, 36
VT_UINT32, VT_FLOAT32, VT_STRING, VT_ARRAY = 4, 6, 8, 9
ARCH = "bitnet-b1.58"


def _lut81():
    lut = np.zeros(81, np.uint8)
    for i in range(81):
        d, v = i, 0
        for f in range(4):
            v |= (d % 3) << (6 - 2 * f)
            d //= 3
        lut[i] = v
    return lut


LUT81 = _lut81()


def i2s_nbytes(rows, cols):
    return rows * cols // 4 + 32


def fill_i2s(rng, out, rows, cols, scale=None):
    """Fill `out` (uint8, i2s_nbytes long) with random ternary codes + scale."""
    nb = rows * cols // 4
    out[:nb] = LUT81[rng.integers(0, 81, size=nb, dtype=np.uint8)]
    if scale is None:
        scale = rng.uniform(0.01, 0.1)
    out[nb:nb + 32] = 0
    out[nb:nb + 4] = np.frombuffer(np.float32(scale).tobytes(), np.uint8)
    return np.float32(scale)


def random_i2s(rng, rows, cols):
    buf = np.empty(i2s_nbytes(rows, cols), np.uint8)
    fill_i2s(rng, buf, rows, cols)
    return buf


def unpack_codes(packed, rows, cols):
    """Codes [rows, cols] (0..2) of a packed I2_S tensor (numpy, for tests)."""
    b = packed[: rows * cols // 4].reshape(rows, cols // 128, 32)
    f = np.stack([(b >> (6 - 2 * i)) & 3 for i in range(4)], axis=2)  # [r, blk, 4, 32]
    return f.reshape(rows, cols)


def pack_codes(codes):
    """Inverse of unpack_codes, without the scale tail."""
    rows, cols = codes.shape
    c = codes.reshape(rows, cols // 128, 4, 32).astype(np.uint8)
    b = (c[:, :, 0] << 6) | (c[:, :, 1] << 4) | (c[:, :, 2] << 2) | c[:, :, 3]
    return b.reshape(-1)


@dataclass
class Config:
    n_layer: int = 30
    n_embd: int = 2560
    n_ff: int = 6912
    n_head: int = 20
    n_head_kv: int = 5
    n_vocab: int = 128256
    n_rot: int = 128
    n_ctx_train: int = 4096
    eps: float = 1e-5
    rope_base: float = 500000.0

    @property
    def head_dim(self):
        return self.n_embd // self.n_head

    @property
    def n_embd_gqa(self):
        return self.head_dim * self.n_head_kv


BITNET_2B = Config()


def small_config(**kw):
    base = dict(n_layer=2, n_embd=256, n_ff=512, n_head=2, n_head_kv=1, n_vocab=1000)
    base.update(kw)
    return Config(**base)


def _layer_tensors(cfg, il):
    E, F, G = cfg.n_embd, cfg.n_ff, cfg.n_embd_gqa
    p = f"blk.{il}."
    return [
        (p + "attn_q.weight", TYPE_I2_S, (E, E)),
        (p + "attn_k.weight", TYPE_I2_S, (E, G)),
        (p + "attn_v.weight", TYPE_I2_S, (E, G)),
        (p + "attn_output.weight", TYPE_I2_S, (E, E)),
        (p + "ffn_gate.weight", TYPE_I2_S, (E, F)),
        (p + "ffn_up.weight", TYPE_I2_S, (E, F)),
        (p + "ffn_down.weight", TYPE_I2_S, (F, E)),
        (p + "attn_norm.weight", TYPE_F32, (E,)),
        (p + "attn_sub_norm.weight", TYPE_F32, (E,)),
        (p + "ffn_norm.weight", TYPE_F32, (E,)),
        (p + "ffn_sub_norm.weight", TYPE_F32, (F,)),
    ]


_FIELD = {"attn_q": "wq", "attn_k": "wk", "attn_v": "wv", "attn_output": "wo",
          "ffn_gate": "ffn_gate", "ffn_up": "ffn_up", "ffn_down": "ffn_down",
          "attn_norm": "attn_norm", "attn_sub_norm": "attn_sub_norm",
          "ffn_norm": "ffn_norm", "ffn_sub_norm": "ffn_sub_norm"}


def _nbytes(ttype, dims):
    n = int(np.prod(dims))
    return {TYPE_F32: 4 * n, TYPE_F16: 2 * n, TYPE_I2_S: n // 4 + 32}[ttype]


def byte_level_tokens():
    """The 256 single-byte tokens of a GPT-2 byte-level BPE vocabulary: the
    published byte -> printable-character mapping (printable Latin-1 bytes map
    to themselves, the other 68 to U+0100 upwards, in byte order)."""
    keep = list(range(0x21, 0x7F)) + list(range(0xA1, 0xAD)) + list(range(0xAE, 0x100))
    table, extra = {}, 0
    for b in range(256):
        if b in keep:
            table[b] = b
        else:
            table[b] = 0x100 + extra
            extra += 1
    return [chr(table[b]) for b in range(256)]


def _kv_bytes(cfg, tokenizer=False):
    out = bytearray()

    def key(k):
        kb = k.encode()
        out.extend(struct.pack("<Q", len(kb)) + kb)

    def s(k, v):
        key(k); vb = v.encode()
        out.extend(struct.pack("<IQ", VT_STRING, len(vb)) + vb)

    def u32(k, v):
        key(k); out.extend(struct.pack("<II", VT_UINT32, v))

    def f32(k, v):
        key(k); out.extend(struct.pack("<If", VT_FLOAT32, v))

    s("general.architecture", ARCH)
    a = ARCH + "."
    u32(a + "block_count", cfg.n_layer)
    u32(a + "embedding_length", cfg.n_embd)
    u32(a + "feed_forward_length", cfg.n_ff)
    u32(a + "attention.head_count", cfg.n_head)
    u32(a + "attention.head_count_kv", cfg.n_head_kv)
    u32(a + "rope.dimension_count", cfg.n_rot)
    u32(a + "context_length", cfg.n_ctx_train)
    u32(a + "vocab_size", cfg.n_vocab)
    f32(a + "attention.layer_norm_rms_epsilon", cfg.eps)
    f32(a + "rope.freq_base", cfg.rope_base)
    n_kv = 11
    if tokenizer:
        # a byte-level BPE vocabulary without merges: every byte its own token
        # (the first 256 ids), the rest placeholders, so that the reference's
        # tokenizer loads it (src/tokenizer.c: model "gpt2", >= 256 tokens)
        s("tokenizer.ggml.model", "gpt2")
        toks = byte_level_tokens() + [f"<|synthetic_{i}|>" for i in range(256, cfg.n_vocab)]
        key("tokenizer.ggml.tokens")
        out.extend(struct.pack("<IIQ", VT_ARRAY, VT_STRING, len(toks)))
        for t in toks:
            tb = t.encode()
            out.extend(struct.pack("<Q", len(tb)) + tb)
        n_kv += 2
    return bytes(out), n_kv


class SynthModel:
    """A seeded random-init bitnet-b1.58 model held as one GGUF v3 image.

    `tensors[name]` are numpy views into `image`; `desc()` is the ModelDesc the
    C ABI takes (pointers into the image, which must stay alive).
    """

    def __init__(self, cfg: Config, seed: int = 1234, tokenizer: bool = False):
        self.cfg = cfg
        self.seed = seed
        rng = np.random.Generator(np.random.PCG64(seed))
        specs = [("token_embd.weight", TYPE_F16, (cfg.n_embd, cfg.n_vocab)),
                 ("output_norm.weight", TYPE_F32, (cfg.n_embd,))]
        for il in range(cfg.n_layer):
            specs += _layer_tensors(cfg, il)
        kv, n_kv = _kv_bytes(cfg, tokenizer)
        info = bytearray()
        offs, off = [], 0
        for name, tt, dims in specs:
            nb = name.encode()
            info.extend(struct.pack("<Q", len(nb)) + nb + struct.pack("<I", len(dims)))
            info.extend(struct.pack(f"<{len(dims)}Q", *dims))
            info.extend(struct.pack("<IQ", tt, off))
            offs.append(off)
            off += (_nbytes(tt, dims) + GGUF_ALIGN - 1) // GGUF_ALIGN * GGUF_ALIGN
        head = b"GGUF" + struct.pack("<IQQ", 3, len(specs), n_kv) + kv + bytes(info)
        data_off = (len(head) + GGUF_ALIGN - 1) // GGUF_ALIGN * GGUF_ALIGN
        self.image = np.zeros(data_off + off, np.uint8)
        self.image[: len(head)] = np.frombuffer(head, np.uint8)
        self.tensors = {}
        for (name, tt, dims), o in zip(specs, offs):
            view = self.image[data_off + o: data_off + o + _nbytes(tt, dims)]
            self.tensors[name] = view
            n = int(np.prod(dims))
            if tt == TYPE_I2_S:
                fill_i2s(rng, view, dims[1], dims[0])
            elif tt == TYPE_F16:
                v = (rng.standard_normal(n, dtype=np.float32) * np.float32(0.02)).astype(np.float16)
                view.view(np.uint16)[:] = v.view(np.uint16)
            else:
                view.view(np.float32)[:] = np.float32(1.0) + np.float32(0.02) * rng.standard_normal(n, dtype=np.float32)
        self._desc = None

    def weight_bytes(self):
        """Every tensor payload, the per-token weight traffic of decode."""
        return int(sum(v.nbytes for v in self.tensors.values()))

    def layer_weight_bytes(self, il=0):
        return int(sum(v.nbytes for k, v in self.tensors.items() if k.startswith(f"blk.{il}.")))

    def tensor(self, name):
        return self.tensors[name]

    def desc(self):
        if self._desc is None:
            cfg = self.cfg
            layers = (abi.LayerDesc * cfg.n_layer)()
            for il in range(cfg.n_layer):
                for name, _, _ in _layer_tensors(cfg, il):
                    short = name.split(".")[2]
                    setattr(layers[il], _FIELD[short], self.tensors[name].ctypes.data)
            d = abi.ModelDesc()
            d.n_layer, d.n_embd, d.n_ff = cfg.n_layer, cfg.n_embd, cfg.n_ff
            d.n_head, d.n_head_kv, d.n_vocab = cfg.n_head, cfg.n_head_kv, cfg.n_vocab
            d.n_rot, d.n_ctx_train = cfg.n_rot, cfg.n_ctx_train
            d.f_rms_eps, d.rope_freq_base = cfg.eps, cfg.rope_base
            d.tok_embd = self.tensors["token_embd.weight"].ctypes.data
            d.output_norm = self.tensors["output_norm.weight"].ctypes.data
            d.layers = C.cast(layers, C.POINTER(abi.LayerDesc))
            self._desc = (d, layers)
        return self._desc[0]


def random_activation(rng, n, dtype=np.float32):
    return rng.standard_normal(n, dtype=np.float32).astype(dtype)
