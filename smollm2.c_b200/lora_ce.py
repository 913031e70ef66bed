"""Python binding of the lora_ce C ABI (include/lora_ce.h), through ctypes.

This mirrors the reference's trainer interface for the LoRA head
(src/train.h: train_create / train_step / train_save / train_load /
train_free) on top of the CUDA library:

* ``LoraCE(cfg)``           ~ train_create (adapter + optimizer state on GPU)
* ``set_weight(W16)``       the tied lm_head, [V][d] f16 bit patterns
* ``set_adapter(A, B, step)`` / ``get_adapter()``  reference layouts
  (A [d][r], B [r][V], src/train.c:35-36)
* ``step(H, targets)``      one train_step on pre-gathered hidden states;
  returns the mean loss (train_step's return value)
* ``train_step_tokens(H, tokens, seq_max)`` the reference's target indexing
  (src/train.c:198-229): positions 0..use_n-2 predict tokens[pos+1],
  use_n = min(n, seq_max); returns -1.0 when fewer than 2 tokens remain,
  exactly as train_step does.
* ``save(path)`` / ``load(path)`` the LORA0001 adapter file
  (src/train.c:244-283), byte-identical to the reference's writer.

There is no CPU fallback: if the shared library is missing or no B200 is
present, construction raises.
"""
from __future__ import annotations

import ctypes as C
import os
import struct
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
LIB_PATH = os.path.join(HERE, "liblora_ce.so")

BF16, F16, F32 = 0, 1, 2
ERRORS = {0: "ok", -1: "EINVAL", -2: "ENOMEM", -3: "ECUDA", -4: "ENCCL", -5: "EDEVICE",
          -6: "ESTATE"}

# Symbols declared in include/lora_ce.h (checked by the CPU tests).
EXPORTS = [
    "lora_ce_default_config", "lora_ce_create", "lora_ce_destroy", "lora_ce_set_weight_f16",
    "lora_ce_set_adapter", "lora_ce_get_adapter", "lora_ce_step", "lora_ce_step_device",
    "lora_ce_get_grads", "lora_ce_get_token_loss", "lora_ce_nccl_unique_id",
    "lora_ce_comm_init", "lora_ce_sync", "lora_ce_stream", "lora_ce_last_launches",
    "lora_ce_last_error", "lora_ce_set_profiling", "lora_ce_phase_times", "lora_ce_phase_name",
    "lora_ce_token_loss_noalloc", "lora_ce_noalloc_last_error", "lora_ce_merge_weight",
    "lora_ce_merge_weight_device", "lora_ce_merge_last_error", "lora_ce_set_scale",
    "lora_ce_set_weight_q4k", "lora_ce_q4k_dequant", "lora_ce_q4k_dequant_device",
    "lora_ce_q4k_last_error", "lora_ce_apply_grads", "lora_ce_set_copy_timing",
    "lora_ce_copy_times", "lora_ce_set_comm_timeout",
]

# Symbols declared in include/lora_body.h.
BODY_EXPORTS = [
    "lora_body_create", "lora_body_destroy", "lora_body_set_embedding", "lora_body_set_layer",
    "lora_body_set_window", "lora_body_hidden", "lora_body_hidden_device", "lora_body_sync",
    "lora_body_stream", "lora_body_last_error", "lora_body_train_step",
]

NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
              "-Xcompiler", "-fPIC", "-shared"]


def build(verbose: bool = False) -> str:
    """Compile csrc/ into liblora_ce.so (sm_100a) next to this file."""
    srcs = [os.path.join(HERE, "csrc", f) for f in ("lora_ce_api.cu", "lora_ce_noalloc.cu", "lora_ce_merge.cu",
                                                         "lora_ce_q4k.cu", "lora_body.cu")]
    cmd = ["nvcc", *NVCC_FLAGS, "-I" + os.path.join(REPO, "include"), "-o", LIB_PATH, *srcs,
           "-ldl"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    if os.path.exists(LIB_PATH):
        os.remove(LIB_PATH)  # a failed build must not leave a stale library behind
    subprocess.run(cmd, check=True)
    return LIB_PATH


class Config(C.Structure):
    _fields_ = [("dim", C.c_int32), ("vocab", C.c_int32), ("rank", C.c_int32),
                ("scale", C.c_float), ("lr", C.c_float), ("beta1", C.c_float),
                ("beta2", C.c_float), ("eps", C.c_float), ("weight_decay", C.c_float),
                ("clip_norm", C.c_float), ("max_tokens", C.c_int32), ("device", C.c_int32)]


class BodyConfig(C.Structure):
    _fields_ = [("n_layers", C.c_int32), ("dim", C.c_int32), ("n_heads", C.c_int32),
                ("n_kv_heads", C.c_int32), ("ffn_hidden", C.c_int32), ("vocab", C.c_int32),
                ("rms_eps", C.c_float), ("rope_theta", C.c_float), ("max_seq", C.c_int32),
                ("max_tokens", C.c_int32), ("device", C.c_int32)]


class LoraCEError(RuntimeError):
    pass


_lib = None


def load_library() -> C.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise LoraCEError(f"{LIB_PATH} is missing: run __graft_entry__.build() first")
    lib = C.CDLL(LIB_PATH)
    vp = C.c_void_p
    lib.lora_ce_default_config.argtypes = [C.POINTER(Config), C.c_int32, C.c_int32, C.c_int32,
                                           C.c_int32]
    lib.lora_ce_default_config.restype = None
    lib.lora_ce_create.argtypes = [C.POINTER(Config), C.POINTER(vp)]
    lib.lora_ce_destroy.argtypes = [vp]
    lib.lora_ce_set_weight_f16.argtypes = [vp, vp]
    lib.lora_ce_set_adapter.argtypes = [vp, vp, vp, C.c_int32]
    lib.lora_ce_set_scale.argtypes = [vp, C.c_float]
    lib.lora_ce_set_weight_q4k.argtypes = [vp, vp]
    lib.lora_ce_q4k_dequant.argtypes = [vp, C.c_int64, vp, C.c_int32, C.c_int32]
    lib.lora_ce_q4k_dequant_device.argtypes = [vp, C.c_int64, vp, C.c_int32, vp]
    lib.lora_ce_q4k_last_error.argtypes = []
    lib.lora_ce_q4k_last_error.restype = C.c_char_p
    lib.lora_ce_get_adapter.argtypes = [vp, vp, vp, C.POINTER(C.c_int32)]
    lib.lora_ce_step.argtypes = [vp, vp, C.c_int32, C.c_int32, vp, C.POINTER(C.c_float)]
    lib.lora_ce_step_device.argtypes = [vp, vp, C.c_int32, C.c_int32, vp, vp]
    lib.lora_ce_get_grads.argtypes = [vp, vp, vp, C.POINTER(C.c_float), C.POINTER(C.c_float)]
    lib.lora_ce_get_token_loss.argtypes = [vp, vp, C.c_int32]
    lib.lora_ce_apply_grads.argtypes = [vp, vp, vp, C.c_float]
    lib.lora_body_create.argtypes = [C.POINTER(BodyConfig), C.POINTER(vp)]
    lib.lora_body_destroy.argtypes = [vp]
    lib.lora_body_set_embedding.argtypes = [vp, vp, vp]
    lib.lora_body_set_layer.argtypes = [vp, C.c_int32] + [vp] * 9
    lib.lora_body_set_window.argtypes = [vp, C.c_int32, C.c_int32]
    lib.lora_body_hidden.argtypes = [vp, vp, vp, C.c_int32, vp]
    lib.lora_body_hidden_device.argtypes = [vp, vp, vp, C.c_int32, vp, C.c_int32]
    lib.lora_body_sync.argtypes = [vp]
    lib.lora_body_train_step.argtypes = [vp, vp, vp, vp, C.c_int32, vp, C.POINTER(C.c_float)]
    lib.lora_body_stream.argtypes = [vp]
    lib.lora_body_stream.restype = vp
    lib.lora_body_last_error.argtypes = []
    lib.lora_body_last_error.restype = C.c_char_p
    lib.lora_ce_set_copy_timing.argtypes = [vp, C.c_int32]
    lib.lora_ce_set_comm_timeout.argtypes = [vp, C.c_int32]
    lib.lora_ce_copy_times.argtypes = [vp, C.POINTER(C.c_float), C.c_int32]
    lib.lora_ce_copy_times.restype = C.c_int32
    lib.lora_ce_nccl_unique_id.argtypes = [vp]
    lib.lora_ce_comm_init.argtypes = [vp, C.c_int32, C.c_int32, vp]
    lib.lora_ce_sync.argtypes = [vp]
    lib.lora_ce_stream.argtypes = [vp]
    lib.lora_ce_stream.restype = vp
    lib.lora_ce_last_launches.argtypes = [vp]
    lib.lora_ce_last_launches.restype = C.c_int32
    lib.lora_ce_set_profiling.argtypes = [vp, C.c_int32]
    lib.lora_ce_set_profiling.restype = C.c_int
    lib.lora_ce_phase_times.argtypes = [vp, C.POINTER(C.c_float), C.c_int32]
    lib.lora_ce_phase_times.restype = C.c_int32
    lib.lora_ce_phase_name.argtypes = [C.c_int32]
    lib.lora_ce_phase_name.restype = C.c_char_p
    lib.lora_ce_token_loss_noalloc.argtypes = [vp, C.c_int32, C.c_int32, vp, vp, C.c_float, vp,
                                               C.c_int32, C.c_int32, vp, vp, vp]
    lib.lora_ce_token_loss_noalloc.restype = C.c_int
    lib.lora_ce_noalloc_last_error.argtypes = []
    lib.lora_ce_noalloc_last_error.restype = C.c_char_p
    lib.lora_ce_merge_weight.argtypes = [vp, vp, vp, C.c_int32, C.c_int32, C.c_int32, C.c_float,
                                         vp, C.c_int32]
    lib.lora_ce_merge_weight.restype = C.c_int
    lib.lora_ce_merge_weight_device.argtypes = [vp, vp, vp, C.c_int32, C.c_int32, C.c_int32,
                                                C.c_float, vp, vp]
    lib.lora_ce_merge_weight_device.restype = C.c_int
    lib.lora_ce_merge_last_error.argtypes = []
    lib.lora_ce_merge_last_error.restype = C.c_char_p
    lib.lora_ce_last_error.argtypes = []
    lib.lora_ce_last_error.restype = C.c_char_p
    for name in ["lora_ce_create", "lora_ce_destroy", "lora_ce_set_weight_f16",
                 "lora_ce_set_adapter", "lora_ce_get_adapter", "lora_ce_step",
                 "lora_ce_step_device", "lora_ce_get_grads", "lora_ce_get_token_loss",
                 "lora_ce_nccl_unique_id", "lora_ce_comm_init", "lora_ce_sync"]:
        getattr(lib, name).restype = C.c_int
    _lib = lib
    return lib


def _check(rc: int, what: str) -> None:
    if rc != 0:
        msg = load_library().lora_ce_last_error().decode(errors="replace")
        raise LoraCEError(f"{what} failed: {ERRORS.get(rc, rc)}: {msg}")


def _ptr(a: np.ndarray) -> C.c_void_p:
    return C.c_void_p(a.ctypes.data)


def merge_weight(W16: np.ndarray, A_dr: np.ndarray, B_rv: np.ndarray, scale: float,
                 device: int = 0) -> np.ndarray:
    """LoRA merge into the tied lm_head on the GPU (lora_patched_weight's
    arithmetic, bit-exact): returns the patched [V][d] f16 bit patterns."""
    W16 = np.ascontiguousarray(W16, np.uint16)
    A = np.ascontiguousarray(A_dr, np.float32)
    B = np.ascontiguousarray(B_rv, np.float32)
    V, d = W16.shape
    r = A.shape[1]
    assert A.shape == (d, r) and B.shape == (r, V)
    out = np.empty_like(W16)
    lib = load_library()
    rc = lib.lora_ce_merge_weight(_ptr(W16), _ptr(A), _ptr(B), d, r, V, float(scale), _ptr(out),
                                  device)
    if rc != 0:
        msg = lib.lora_ce_merge_last_error().decode(errors="replace")
        raise LoraCEError(f"lora_ce_merge_weight failed: {ERRORS.get(rc, rc)}: {msg}")
    return out


def q4k_dequant(blocks: np.ndarray, dtype: int = 2, device: int = 0) -> np.ndarray:
    """Q4_K super-blocks -> f32 (dtype F32) or f16 bits (dtype F16) on the GPU."""
    b = np.ascontiguousarray(blocks, np.uint8).ravel()
    assert b.size % 144 == 0
    n = b.size // 144
    out = np.empty(n * 256, np.float32 if dtype == F32 else np.uint16)
    lib = load_library()
    rc = lib.lora_ce_q4k_dequant(_ptr(b), n, _ptr(out), dtype, device)
    if rc != 0:
        msg = lib.lora_ce_q4k_last_error().decode(errors="replace")
        raise LoraCEError(f"lora_ce_q4k_dequant failed: {ERRORS.get(rc, rc)}: {msg}")
    return out


def token_loss_noalloc(d_W: int, vocab: int, dim: int, d_A: int, d_B: int, scale: float,
                       d_H: int, h_dtype: int, T: int, d_targets: int, d_loss: int,
                       stream: int = 0) -> None:
    """lora_ce_token_loss_noalloc on device pointers (see include/lora_ce.h):
    the per-position loss without any allocation, for callers that cannot
    allocate GPU memory at call time.  Rank 4, T <= 4096, V <= 49152."""
    lib = load_library()
    rc = lib.lora_ce_token_loss_noalloc(
        C.c_void_p(d_W), vocab, dim, C.c_void_p(d_A), C.c_void_p(d_B), float(scale),
        C.c_void_p(d_H), h_dtype, T, C.c_void_p(d_targets), C.c_void_p(d_loss),
        C.c_void_p(stream or None))
    if rc != 0:
        msg = lib.lora_ce_noalloc_last_error().decode(errors="replace")
        raise LoraCEError(f"lora_ce_token_loss_noalloc failed: {ERRORS.get(rc, rc)}: {msg}")


def default_config(dim, vocab, rank, max_tokens, **kw) -> Config:
    cfg = Config()
    load_library().lora_ce_default_config(C.byref(cfg), dim, vocab, rank, max_tokens)
    for k, v in kw.items():
        setattr(cfg, k, v)
    return cfg


LORA_MAGIC = b"LORA0001"


def save_lora0001(path: str, A_dr: np.ndarray, B_rv: np.ndarray, scale: float, step: int) -> None:
    """LORA0001 writer: magic, int32 {dim, vocab, rank, step}, f32 scale,
    f32 A [d][r], f32 B [r][V] (src/train.c:244-259)."""
    d, r = A_dr.shape
    V = B_rv.shape[1]
    with open(path, "wb") as f:
        f.write(LORA_MAGIC)
        f.write(struct.pack("<4i", d, V, r, step))
        f.write(struct.pack("<f", scale))
        f.write(np.ascontiguousarray(A_dr, np.float32).tobytes())
        f.write(np.ascontiguousarray(B_rv, np.float32).tobytes())


def load_lora0001(path: str, dim: int | None = None, vocab: int | None = None,
                  rank: int | None = None):
    """LORA0001 reader with train_load's checks (src/train.c:261-283):
    bad magic or a dim/vocab/rank mismatch raise ValueError."""
    with open(path, "rb") as f:
        if f.read(8) != LORA_MAGIC:
            raise ValueError("bad LORA0001 magic")
        d, V, r, step = struct.unpack("<4i", f.read(16))
        if (dim is not None and d != dim) or (vocab is not None and V != vocab) or (
                rank is not None and r != rank):
            raise ValueError("train_load: shape mismatch")
        (scale,) = struct.unpack("<f", f.read(4))
        A = np.frombuffer(f.read(4 * d * r), np.float32).reshape(d, r).copy()
        B = np.frombuffer(f.read(4 * r * V), np.float32).reshape(r, V).copy()
    return dict(A=A, B=B, scale=scale, step=step, dim=d, vocab=V, rank=r)


class LoraCE:
    """One GPU's LoRA-on-lm_head trainer state (see module docstring)."""

    def __init__(self, cfg: Config):
        self.lib = load_library()
        self.cfg = cfg
        self.h = C.c_void_p()
        _check(self.lib.lora_ce_create(C.byref(cfg), C.byref(self.h)), "lora_ce_create")

    def close(self) -> None:
        if self.h:
            self.lib.lora_ce_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- state
    def set_weight(self, W16: np.ndarray) -> None:
        W16 = np.ascontiguousarray(W16, np.uint16)
        assert W16.shape == (self.cfg.vocab, self.cfg.dim)
        _check(self.lib.lora_ce_set_weight_f16(self.h, _ptr(W16)), "set_weight")

    def set_adapter(self, A_dr: np.ndarray, B_rv: np.ndarray, step: int = 0) -> None:
        A = np.ascontiguousarray(A_dr, np.float32)
        B = np.ascontiguousarray(B_rv, np.float32)
        assert A.shape == (self.cfg.dim, self.cfg.rank)
        assert B.shape == (self.cfg.rank, self.cfg.vocab)
        _check(self.lib.lora_ce_set_adapter(self.h, _ptr(A), _ptr(B), step), "set_adapter")

    def set_weight_q4k(self, blocks: np.ndarray) -> None:
        """lm_head as Q4_K super-blocks (uint8, V*d/256 x 144)."""
        b = np.ascontiguousarray(blocks, np.uint8)
        assert b.size == self.cfg.vocab * self.cfg.dim // 256 * 144
        _check(self.lib.lora_ce_set_weight_q4k(self.h, _ptr(b)), "set_weight_q4k")

    def set_scale(self, scale: float) -> None:
        _check(self.lib.lora_ce_set_scale(self.h, float(scale)), "set_scale")
        self.cfg.scale = float(scale)

    def get_adapter(self):
        A = np.empty((self.cfg.dim, self.cfg.rank), np.float32)
        B = np.empty((self.cfg.rank, self.cfg.vocab), np.float32)
        step = C.c_int32()
        _check(self.lib.lora_ce_get_adapter(self.h, _ptr(A), _ptr(B), C.byref(step)),
               "get_adapter")
        return A, B, step.value

    def get_grads(self):
        gA = np.empty((self.cfg.dim, self.cfg.rank), np.float32)
        gB = np.empty((self.cfg.rank, self.cfg.vocab), np.float32)
        ls, npred = C.c_float(), C.c_float()
        _check(self.lib.lora_ce_get_grads(self.h, _ptr(gA), _ptr(gB), C.byref(ls),
                                          C.byref(npred)), "get_grads")
        return gA, gB, ls.value, npred.value

    def token_loss(self, T: int) -> np.ndarray:
        out = np.empty(T, np.float32)
        _check(self.lib.lora_ce_get_token_loss(self.h, _ptr(out), T), "get_token_loss")
        return out

    def apply_grads(self, gA_sum: np.ndarray, gB_sum: np.ndarray, n_pred: float) -> None:
        """One optimizer step from gradient sums over n_pred positions
        (lora_ce_apply_grads)."""
        gA = np.ascontiguousarray(gA_sum, np.float32)
        gB = np.ascontiguousarray(gB_sum, np.float32)
        assert gA.shape == (self.cfg.dim, self.cfg.rank)
        assert gB.shape == (self.cfg.rank, self.cfg.vocab)
        _check(self.lib.lora_ce_apply_grads(self.h, _ptr(gA), _ptr(gB), float(n_pred)),
               "apply_grads")

    # -- steps
    def step(self, H: np.ndarray, targets: np.ndarray, dtype: int | None = None) -> float:
        """H: [T][d] as bf16 bits (uint16, dtype BF16 by default), float16 or
        float32; targets: [T] int32."""
        if dtype is None:
            dtype = {np.dtype(np.uint16): BF16, np.dtype(np.float16): F16,
                     np.dtype(np.float32): F32}[H.dtype]
        H = np.ascontiguousarray(H)
        tg = np.ascontiguousarray(targets, np.int32)
        T = tg.shape[0]
        assert H.shape == (T, self.cfg.dim)
        loss = C.c_float()
        _check(self.lib.lora_ce_step(self.h, _ptr(H), dtype, T, _ptr(tg), C.byref(loss)),
               "lora_ce_step")
        return loss.value

    def step_device(self, dH_ptr: int, dtype: int, T: int, dtg_ptr: int, dloss_ptr: int = 0) -> None:
        _check(self.lib.lora_ce_step_device(self.h, C.c_void_p(dH_ptr), dtype, T,
                                            C.c_void_p(dtg_ptr), C.c_void_p(dloss_ptr or None)),
               "lora_ce_step_device")

    def train_step_tokens(self, H: np.ndarray, tokens: np.ndarray, seq_max: int) -> float:
        n = len(tokens)
        if n < 2:
            return -1.0
        use_n = min(n, seq_max)
        if use_n < 2:
            return -1.0
        n_pred = use_n - 1
        targets = np.ascontiguousarray(np.asarray(tokens, np.int32)[1:use_n])
        return self.step(np.ascontiguousarray(H[:n_pred]), targets)

    def sync(self) -> None:
        _check(self.lib.lora_ce_sync(self.h), "lora_ce_sync")

    def set_profiling(self, enable: bool = True) -> None:
        _check(self.lib.lora_ce_set_profiling(self.h, 1 if enable else 0), "set_profiling")

    def phase_times(self) -> dict:
        """{phase name: ms} of the last step (needs set_profiling(True))."""
        buf = (C.c_float * 16)()
        n = self.lib.lora_ce_phase_times(self.h, buf, 16)
        if n < 0:
            _check(n, "phase_times")
        return {self.lib.lora_ce_phase_name(i).decode(): float(buf[i]) for i in range(n)}

    def set_comm_timeout(self, ms: int) -> None:
        _check(self.lib.lora_ce_set_comm_timeout(self.h, int(ms)), "set_comm_timeout")

    def set_copy_timing(self, enable: bool = True) -> None:
        _check(self.lib.lora_ce_set_copy_timing(self.h, int(enable)), "set_copy_timing")

    def copy_times(self) -> dict:
        """Where the last host-input step's time went (needs
        set_copy_timing(True)): host_us (enqueue), wait_us (host waiting for
        the result), copy_wait_ms, chunk_ms [...], step_ms."""
        buf = (C.c_float * 16)()
        n = self.lib.lora_ce_copy_times(self.h, buf, 16)
        if n < 0:
            _check(n, "copy_times")
        v = [float(buf[i]) for i in range(n)]
        if n == 2:  # timing off: the host's times only
            return {"host_us": v[0], "wait_us": v[1]}
        return {"host_us": v[0], "wait_us": v[1], "copy_wait_ms": v[2], "chunk_ms": v[3:-1],
                "step_ms": v[-1]}

    @property
    def stream(self) -> int:
        return self.lib.lora_ce_stream(self.h) or 0

    @property
    def last_launches(self) -> int:
        return int(self.lib.lora_ce_last_launches(self.h))

    # -- multi-GPU
    @staticmethod
    def nccl_unique_id() -> bytes:
        buf = C.create_string_buffer(128)
        _check(load_library().lora_ce_nccl_unique_id(buf), "nccl_unique_id")
        return buf.raw

    def comm_init(self, nranks: int, rank: int, uid: bytes) -> None:
        buf = C.create_string_buffer(uid, 128)
        _check(self.lib.lora_ce_comm_init(self.h, nranks, rank, buf), "comm_init")

    # -- adapter files
    def save(self, path: str) -> None:
        A, B, step = self.get_adapter()
        save_lora0001(path, A, B, self.cfg.scale, step)

    def load(self, path: str) -> None:
        ad = load_lora0001(path, self.cfg.dim, self.cfg.vocab, self.cfg.rank)
        self.set_adapter(ad["A"], ad["B"], ad["step"])


def _bcheck(rc: int, what: str) -> None:
    if rc != 0:
        msg = load_library().lora_body_last_error().decode(errors="replace")
        raise LoraCEError(f"{what} failed: {ERRORS.get(rc, rc)}: {msg}")


class LoraBody:
    """The body forward on the GPU (include/lora_body.h): hidden states of
    every position of a batch of token sequences."""

    def __init__(self, n_layers, dim=576, n_heads=9, n_kv_heads=3, ffn_hidden=1536,
                 vocab=49152, rms_eps=1e-5, rope_theta=1e5, max_seq=256, max_tokens=1024,
                 device=0):
        self.lib = load_library()
        self.cfg = BodyConfig(n_layers, dim, n_heads, n_kv_heads, ffn_hidden, vocab, rms_eps,
                              rope_theta, max_seq, max_tokens, device)
        self.h = C.c_void_p()
        _bcheck(self.lib.lora_body_create(C.byref(self.cfg), C.byref(self.h)), "lora_body_create")

    def close(self) -> None:
        if self.h:
            self.lib.lora_body_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_embedding(self, token_embd_f16: np.ndarray, output_norm: np.ndarray) -> None:
        e = np.ascontiguousarray(token_embd_f16, np.uint16)
        n = np.ascontiguousarray(output_norm, np.float32)
        _bcheck(self.lib.lora_body_set_embedding(self.h, _ptr(e), _ptr(n)), "set_embedding")

    def set_layer(self, L: int, t: dict) -> None:
        """t: attn_norm, wq, wk, wv, wo, ffn_norm, gate, up, down (f16 bits
        as uint16 with rows = outputs; norms float32)."""
        a = [np.ascontiguousarray(t[k], np.float32 if k.endswith("norm") else np.uint16)
             for k in ("attn_norm", "wq", "wk", "wv", "wo", "ffn_norm", "gate", "up", "down")]
        _bcheck(self.lib.lora_body_set_layer(self.h, L, *[_ptr(x) for x in a]), "set_layer")

    def set_window(self, L: int, window: int) -> None:
        _bcheck(self.lib.lora_body_set_window(self.h, L, window), "set_window")

    def hidden(self, tokens: np.ndarray, offsets) -> np.ndarray:
        tok = np.ascontiguousarray(tokens, np.int32)
        off = np.ascontiguousarray(offsets, np.int32)
        out = np.empty((int(off[-1]), self.cfg.dim), np.float32)
        _bcheck(self.lib.lora_body_hidden(self.h, _ptr(tok), _ptr(off), len(off) - 1, _ptr(out)),
                "lora_body_hidden")
        return out

    def hidden_device(self, d_tokens: int, offsets, d_H: int, dtype: int) -> None:
        off = np.ascontiguousarray(offsets, np.int32)
        _bcheck(self.lib.lora_body_hidden_device(self.h, C.c_void_p(d_tokens), _ptr(off),
                                                 len(off) - 1, C.c_void_p(d_H), dtype),
                "lora_body_hidden_device")

    def train_step(self, ce: "LoraCE", tokens, offsets, targets) -> float:
        """lora_body_train_step: body forward of the packed samples, then one
        LoRA step on `ce`; the mean loss."""
        tok = np.ascontiguousarray(tokens, np.int32)
        off = np.ascontiguousarray(offsets, np.int32)
        tg = np.ascontiguousarray(targets, np.int32)
        loss = C.c_float()
        _bcheck(self.lib.lora_body_train_step(self.h, ce.h, _ptr(tok), _ptr(off), len(off) - 1,
                                              _ptr(tg), C.byref(loss)), "lora_body_train_step")
        return loss.value

    def sync(self) -> None:
        _bcheck(self.lib.lora_body_sync(self.h), "lora_body_sync")

    @property
    def stream(self) -> int:
        return self.lib.lora_body_stream(self.h) or 0
