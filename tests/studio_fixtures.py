"""Test infrastructure for the trainer API (smollm2.c_b200/liblora_train.so):
files in the reference's formats and the ctypes glue.

- write_gguf: a GGUF v3 file (the public format the reference's
  src/gguf.c reads: magic, version 3, tensor and key/value counts, the
  key/value table, the tensor table, data aligned to 32 bytes).
- write_packed: a packed dataset as src/data.c writes it: <path> holds the
  int32 token ids, <path>.idx the 16-byte sample_idx records
  {int32 n_tokens, pad, int64 offset} and the 20-byte trailer
  {int32 n_samples, int32 total_tokens, int32 fmt, "STUDIO\\0\\0"}.
- TrainerEnv: loads oracle/_ref/libstudio_env.so (the stand-in body forward
  plus the reference's gguf / gguf_write / hw_probe code) into the global
  symbol scope, then liblora_train.so, which resolves against it.
"""
from __future__ import annotations

import ctypes as C
import os
import struct

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
ENV_SO = os.path.join(REPO, "oracle", "_ref", "libstudio_env.so")
TRAIN_SO = os.path.join(REPO, "smollm2.c_b200", "liblora_train.so")

GGUF_F32, GGUF_F16 = 0, 1
GGUF_V_UINT32, GGUF_V_FLOAT32, GGUF_V_STRING, GGUF_V_ARRAY = 4, 6, 8, 9


def _gguf_str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def write_gguf(path: str, tensors, kv=()) -> None:
    """tensors: (name, dims (innermost first), dtype, raw bytes); kv:
    (key, "u32" | "f32" | "str" | "str_arr", value)."""
    head = struct.pack("<IIQQ", 0x46554747, 3, len(tensors), len(kv))
    for key, typ, val in kv:
        head += _gguf_str(key)
        if typ == "u32":
            head += struct.pack("<II", GGUF_V_UINT32, val)
        elif typ == "f32":
            head += struct.pack("<If", GGUF_V_FLOAT32, val)
        elif typ == "str_arr":
            head += struct.pack("<IIQ", GGUF_V_ARRAY, GGUF_V_STRING, len(val))
            head += b"".join(_gguf_str(x) for x in val)
        else:
            head += struct.pack("<I", GGUF_V_STRING) + _gguf_str(val)
    offs, off = [], 0
    for _, _, _, raw in tensors:
        offs.append(off)
        off = (off + len(raw) + 31) // 32 * 32
    for (name, dims, dtype, _), o in zip(tensors, offs):
        head += _gguf_str(name) + struct.pack("<I", len(dims))
        head += b"".join(struct.pack("<Q", x) for x in dims)
        head += struct.pack("<IQ", dtype, o)
    pad = (-len(head)) % 32
    with open(path, "wb") as f:
        f.write(head + b"\0" * pad)
        for (_, _, _, raw), o in zip(tensors, offs):
            f.write(raw)
            f.write(b"\0" * ((-len(raw)) % 32))


def write_packed(path: str, samples) -> None:
    idx = b""
    off = 0
    total = 0
    with open(path, "wb") as f:
        for s in samples:
            a = np.asarray(s, np.int32)
            f.write(a.tobytes())
            idx += struct.pack("<iiq", len(a), 0, off)
            off += a.nbytes
            total += len(a)
    with open(path + ".idx", "wb") as f:
        f.write(idx + struct.pack("<iii", len(samples), total, 0) + b"STUDIO\0\0")


class TrainParams(C.Structure):
    """src/train.h:11-23."""
    _fields_ = [("mode", C.c_int), ("lora_rank", C.c_int), ("lora_alpha", C.c_int),
                ("seq_max", C.c_int), ("batch", C.c_int), ("lr", C.c_float),
                ("epochs", C.c_int), ("checkpoint_every", C.c_int), ("max_steps", C.c_int),
                ("seed", C.c_int), ("simulate_mem_kb", C.c_long)]


def available() -> bool:
    return os.path.exists(ENV_SO) and os.path.exists(TRAIN_SO)


class TrainerEnv:
    def __init__(self) -> None:
        vp = C.c_void_p
        self.env = C.CDLL(ENV_SO, mode=C.RTLD_GLOBAL)
        self.lib = C.CDLL(TRAIN_SO)
        self.libc = C.CDLL(None)
        e, t = self.env, self.lib
        e.env_forward_create.argtypes = [C.c_int, C.c_int, vp, C.c_int]
        e.env_forward_create.restype = vp
        e.env_forward_free.argtypes = [vp]
        e.env_forward_calls.argtypes = [vp, C.POINTER(C.c_int)]
        e.env_gguf_open.argtypes = [C.c_char_p]
        e.env_gguf_open.restype = vp
        e.env_gguf_close.argtypes = [vp]
        e.env_gguf_tensor.argtypes = [C.c_char_p, C.c_char_p, C.POINTER(C.c_uint64),
                                      C.POINTER(C.c_int), vp, C.c_size_t]
        e.gguf_patch_tensor.argtypes = [C.c_char_p, C.c_char_p, C.c_char_p, vp, C.c_size_t]
        t.train_create.argtypes = [vp, C.POINTER(TrainParams)]
        t.train_create.restype = vp
        t.train_free.argtypes = [vp]
        t.train_step.argtypes = [vp, vp, C.c_int]
        t.train_step.restype = C.c_float
        t.train_save.argtypes = [vp, C.c_char_p]
        t.train_load.argtypes = [vp, C.c_char_p]
        t.train_run.argtypes = [vp, C.c_char_p, C.POINTER(TrainParams), C.c_char_p]
        t.train_merge.argtypes = [C.c_char_p, C.c_char_p, C.c_char_p]
        t.lora_train_set_lm_head.argtypes = [vp, vp]
        t.lora_train_set_lm_head_gguf.argtypes = [vp, vp]

    def forward(self, H: np.ndarray, vocab: int):
        """A stand-in forward serving the rows of H (kept alive by the caller)."""
        return self.env.env_forward_create(H.shape[1], vocab, H.ctypes.data, H.shape[0])

    def forward_calls(self, f):
        c = (C.c_int * 3)()
        self.env.env_forward_calls(f, c)
        return tuple(c)

    def gguf_tensor(self, path: str, name: str, nbytes: int):
        dims = (C.c_uint64 * 2)()
        dt = C.c_int()
        out = np.empty(nbytes, np.uint8)
        rc = self.env.env_gguf_tensor(path.encode(), name.encode(), dims, C.byref(dt),
                                      out.ctypes.data, nbytes)
        return rc, (dims[0], dims[1]), dt.value, out

    def flush(self) -> None:
        self.libc.fflush(None)


def params(rank=4, alpha=8, seq_max=256, lr=1e-3, epochs=1, checkpoint_every=0, max_steps=0,
           seed=42, simulate_mem_kb=0, batch=1) -> TrainParams:
    return TrainParams(0, rank, alpha, seq_max, batch, lr, epochs, checkpoint_every, max_steps,
                       seed, simulate_mem_kb)


def write_smollm_gguf(path: str, seed: int, n_layers: int = 2, dim: int = 576, heads: int = 9,
                      kv_heads: int = 3, ffn: int = 1536, vocab: int = 49152,
                      norm_spread: float = 0.0, return_tensors: bool = False):
    """A SmolLM2-135M-shaped model file with random weights: the llama
    metadata and tensor names the reference's forward_load reads
    (src/forward.c:671-880), f16 matrices ~ N(0, 0.02) from a seed, f32
    norms of 1.0, RMSNorm eps 1e-5, RoPE theta 1e5, tied embeddings, and a
    token list of `vocab` placeholder strings.  `n_layers` is 30 in the
    real model; fewer keep the CPU body quick.  norm_spread > 0 draws the
    norm weights from 1 + U(-spread, spread) instead.  Returns token_embd
    [V][d] as f16 bits, or with return_tensors (token_embd, output_norm,
    [per layer {attn_norm, wq, wk, wv, wo, ffn_norm, gate, up, down}]) with
    the matrices as f16 bits [outputs][inputs]."""
    rng = np.random.default_rng(seed)

    def f16(*shape):
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)).astype(np.float16)

    kv_dim = dim // heads * kv_heads
    embd = f16(vocab, dim)

    def norm():
        if norm_spread <= 0:
            return np.ones(dim, np.float32)
        return (1.0 + rng.uniform(-norm_spread, norm_spread, dim)).astype(np.float32)

    out_norm = norm()
    tensors = [("token_embd.weight", [dim, vocab], GGUF_F16, embd.tobytes()),
               ("output_norm.weight", [dim], GGUF_F32, out_norm.tobytes())]
    layers = []
    for L in range(n_layers):
        b = f"blk.{L}."
        ly = dict(attn_norm=norm(), wq=f16(dim, dim), wk=f16(kv_dim, dim), wv=f16(kv_dim, dim),
                  wo=f16(dim, dim), ffn_norm=norm(), gate=f16(ffn, dim), up=f16(ffn, dim),
                  down=f16(dim, ffn))
        layers.append({k: (v.view(np.uint16) if v.dtype == np.float16 else v)
                       for k, v in ly.items()})
        tensors += [(b + "attn_norm.weight", [dim], GGUF_F32, ly["attn_norm"].tobytes()),
                    (b + "attn_q.weight", [dim, dim], GGUF_F16, ly["wq"].tobytes()),
                    (b + "attn_k.weight", [dim, kv_dim], GGUF_F16, ly["wk"].tobytes()),
                    (b + "attn_v.weight", [dim, kv_dim], GGUF_F16, ly["wv"].tobytes()),
                    (b + "attn_output.weight", [dim, dim], GGUF_F16, ly["wo"].tobytes()),
                    (b + "ffn_norm.weight", [dim], GGUF_F32, ly["ffn_norm"].tobytes()),
                    (b + "ffn_gate.weight", [dim, ffn], GGUF_F16, ly["gate"].tobytes()),
                    (b + "ffn_up.weight", [dim, ffn], GGUF_F16, ly["up"].tobytes()),
                    (b + "ffn_down.weight", [ffn, dim], GGUF_F16, ly["down"].tobytes())]
    kv = [("general.architecture", "str", "llama"),
          ("llama.embedding_length", "u32", dim), ("llama.block_count", "u32", n_layers),
          ("llama.attention.head_count", "u32", heads),
          ("llama.attention.head_count_kv", "u32", kv_heads),
          ("llama.feed_forward_length", "u32", ffn),
          ("llama.attention.layer_norm_rms_epsilon", "f32", 1e-5),
          ("llama.rope.freq_base", "f32", 1e5),
          ("tokenizer.ggml.tokens", "str_arr", [f"t{i}" for i in range(vocab)])]
    write_gguf(path, tensors, kv)
    if return_tensors:
        return embd.view(np.uint16), out_norm, layers
    return embd.view(np.uint16)
