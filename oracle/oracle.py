"""ctypes front end of the CPU checker (test infrastructure only).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg
import this module; the product library never does.  It wraps

* ``oracle/liblora_oracle.so`` — our C restatement of the reference's
  LoRA-on-lm_head step (see lora_oracle.c for the file:line of each
  reference function it follows), and
* ``oracle/_ref/libref_train.so`` — the reference's own ``src/train.c`` and
  ``src/backward.c`` compiled unmodified by ``oracle/Makefile``, used to pin
  the restatement (present wherever it was built; the reference sources are
  only needed to build it).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liblora_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libref_train.so")
REF_BODY_SO = os.path.join(HERE, "_ref", "libref_body.so")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")


def build(ref: bool = True) -> None:
    """Compile the restatement (and the reference harness when the
    reference tree is present)."""
    targets = ["oracle", "ref"] if ref else ["oracle"]
    tree = os.environ.get("SMOLLM2_REF", "") or os.path.join(os.path.dirname(os.path.dirname(HERE)),
                                                             "reference")
    subprocess.run(["make", "-s", "-C", HERE, "REF=" + tree] + targets, check=True)


def _load(path: str) -> C.CDLL:
    if not os.path.exists(path):
        build(ref=(path == REF_SO))
    return C.CDLL(path)


class Oracle:
    """Our restatement (lora_oracle.c)."""

    def __init__(self) -> None:
        lib = _load(ORACLE_SO)
        lib.oracle_base_logits.argtypes = [_u16p, _f32p, C.c_int, C.c_int, _f32p]
        lib.oracle_base_logits.restype = None
        lib.oracle_accumulate.argtypes = [
            C.c_int, C.c_int, C.c_int, C.c_float, _u16p, _f32p, _f32p, _f32p,
            _i32p, C.c_int, C.c_int, _f32p, _f32p, _f32p]
        lib.oracle_accumulate.restype = C.c_int
        lib.oracle_adam.argtypes = [
            C.c_int, C.c_int, C.c_int, C.c_float, C.c_float, C.c_float, C.c_int,
            C.POINTER(C.c_int), _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p]
        lib.oracle_adam.restype = None
        lib.oracle_train_step.argtypes = [
            C.c_int, C.c_int, C.c_int, C.c_float, C.c_float, C.c_float, C.c_float,
            C.c_int, _u16p, _f32p, _i32p, C.c_int, C.c_int, C.POINTER(C.c_int),
            _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p]
        lib.oracle_train_step.restype = C.c_float
        lib.oracle_kaiming_init.argtypes = [C.c_int, C.c_int, C.c_int, _f32p]
        lib.oracle_kaiming_init.restype = None
        lib.oracle_grad_check_softmax_ce.argtypes = [C.c_int, C.c_float]
        lib.oracle_grad_check_softmax_ce.restype = C.c_float
        lib.oracle_merge.argtypes = [_u16p, _f32p, _f32p, C.c_int, C.c_int, C.c_int,
                                     C.c_float, _u16p]
        lib.oracle_merge.restype = None
        lib.oracle_q4k_dequant.argtypes = [C.c_void_p, C.c_int64, _f32p]
        lib.oracle_q4k_dequant.restype = None
        self.lib = lib

    def base_logits(self, W16: np.ndarray, h: np.ndarray) -> np.ndarray:
        V, d = W16.shape
        out = np.empty(V, np.float32)
        self.lib.oracle_base_logits(W16, np.ascontiguousarray(h, np.float32), d, V, out)
        return out

    def accumulate(self, W16, A_dr, B_rv, H, targets, scale, nthreads=1):
        """Summed (not averaged) gA [d][r], gB [r][V] and per-position loss."""
        V, d = W16.shape
        r = A_dr.shape[1]
        T = H.shape[0]
        gA = np.empty((d, r), np.float32)
        gB = np.empty((r, V), np.float32)
        loss = np.empty(T, np.float32)
        rc = self.lib.oracle_accumulate(
            d, V, r, float(scale), W16, np.ascontiguousarray(A_dr, np.float32),
            np.ascontiguousarray(B_rv, np.float32), np.ascontiguousarray(H, np.float32),
            np.ascontiguousarray(targets, np.int32), T, int(nthreads), gA, gB, loss)
        if rc != 0:
            raise ValueError("oracle_accumulate rejected its arguments")
        return gA, gB, loss

    def step(self, W16, A_dr, B_rv, H, targets, scale, lr, wd=0.0, clip=0.0,
             nthreads=1, state=None):
        """One optimizer step on pre-gathered (H, targets).

        Returns dict(loss, gA, gB (mean gradients applied), A, B, state).
        ``state`` carries Adam moments and the step counter between calls."""
        V, d = W16.shape
        r = A_dr.shape[1]
        T = H.shape[0]
        gA, gB, loss_tok = self.accumulate(W16, A_dr, B_rv, H, targets, scale, nthreads)
        if state is None:
            state = dict(step=0, mA=np.zeros((d, r), np.float32), vA=np.zeros((d, r), np.float32),
                         mB=np.zeros((r, V), np.float32), vB=np.zeros((r, V), np.float32))
        A = np.array(A_dr, np.float32, copy=True, order="C")
        B = np.array(B_rv, np.float32, copy=True, order="C")
        stp = C.c_int(state["step"])
        self.lib.oracle_adam(d, V, r, float(lr), float(wd), float(clip), T, C.byref(stp),
                             A, B, gA, gB, state["mA"], state["vA"], state["mB"], state["vB"])
        state["step"] = stp.value
        total = np.float32(0.0)
        for x in loss_tok:  # sequential f32 sum, as train_step does
            total = np.float32(total + x)
        loss = np.float32(total * np.float32(np.float32(1.0) / np.float32(T)))
        return dict(loss=float(loss), loss_tok=loss_tok, gA=gA, gB=gB, A=A, B=B, state=state)

    def adam(self, A_dr, B_rv, gA_sum, gB_sum, n_pred, lr, wd=0.0, clip=0.0, state=None):
        """The optimizer part alone (oracle_adam): mean over n_pred, the
        extensions, Adam.  Returns (A, B, state)."""
        d, r = A_dr.shape
        V = B_rv.shape[1]
        if state is None:
            state = dict(step=0, mA=np.zeros((d, r), np.float32), vA=np.zeros((d, r), np.float32),
                         mB=np.zeros((r, V), np.float32), vB=np.zeros((r, V), np.float32))
        A = np.array(A_dr, np.float32, copy=True, order="C")
        B = np.array(B_rv, np.float32, copy=True, order="C")
        gA = np.array(gA_sum, np.float32, copy=True, order="C")
        gB = np.array(gB_sum, np.float32, copy=True, order="C")
        stp = C.c_int(state["step"])
        self.lib.oracle_adam(d, V, r, float(lr), float(wd), float(clip), int(n_pred), C.byref(stp),
                             A, B, gA, gB, state["mA"], state["vA"], state["mB"], state["vB"])
        state["step"] = stp.value
        return A, B, state

    def train_step_tokens(self, W16, A_dr, B_rv, H, tokens, seq_max, scale, lr,
                          wd=0.0, clip=0.0, nthreads=1, state=None):
        """train_step semantics on a raw token sample (target indexing
        included): H must hold at least min(n, seq_max)-1 rows."""
        V, d = W16.shape
        r = A_dr.shape[1]
        if state is None:
            state = dict(step=0, mA=np.zeros((d, r), np.float32), vA=np.zeros((d, r), np.float32),
                         mB=np.zeros((r, V), np.float32), vB=np.zeros((r, V), np.float32))
        A = np.array(A_dr, np.float32, copy=True, order="C")
        B = np.array(B_rv, np.float32, copy=True, order="C")
        gA = np.empty((d, r), np.float32)
        gB = np.empty((r, V), np.float32)
        stp = C.c_int(state["step"])
        tokens = np.ascontiguousarray(tokens, np.int32)
        loss = self.lib.oracle_train_step(
            d, V, r, float(scale), float(lr), float(wd), float(clip), int(seq_max), W16,
            np.ascontiguousarray(H, np.float32), tokens, len(tokens), int(nthreads),
            C.byref(stp), A, B, gA, gB, state["mA"], state["vA"], state["mB"], state["vB"])
        state["step"] = stp.value
        return dict(loss=float(loss), gA=gA, gB=gB, A=A, B=B, state=state)

    def kaiming_init(self, seed: int, d: int, r: int) -> np.ndarray:
        A = np.empty((d, r), np.float32)
        self.lib.oracle_kaiming_init(int(seed), d, r, A)
        return A

    def grad_check_softmax_ce(self, vocab: int = 32, eps: float = 1e-3) -> float:
        return float(self.lib.oracle_grad_check_softmax_ce(vocab, eps))

    def q4k_dequant(self, blocks: np.ndarray) -> np.ndarray:
        """Q4_K super-blocks (uint8, 144 bytes each) -> f32 weights."""
        blocks = np.ascontiguousarray(blocks, np.uint8).ravel()
        assert blocks.size % 144 == 0
        n = blocks.size // 144
        out = np.empty(n * 256, np.float32)
        self.lib.oracle_q4k_dequant(blocks.ctypes.data, n, out)
        return out

    def merge(self, W16, A_dr, B_rv, scale) -> np.ndarray:
        V, d = W16.shape
        r = A_dr.shape[1]
        out = np.empty_like(W16)
        self.lib.oracle_merge(W16, np.ascontiguousarray(A_dr, np.float32),
                              np.ascontiguousarray(B_rv, np.float32), d, r, V, float(scale), out)
        return out


def ref_available() -> bool:
    return os.path.exists(REF_SO)


class RefHarness:
    """The reference's own train.c / backward.c (oracle/_ref)."""

    def __init__(self) -> None:
        lib = _load(REF_SO)
        lib.ref_train_steps.argtypes = [
            C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, C.c_int, C.c_int, _u16p,
            _f32p, _i32p, C.c_int, C.c_int, C.c_int, _f32p, _f32p, _f32p, _f32p,
            _f32p, C.POINTER(C.c_int)]
        lib.ref_train_steps.restype = C.c_int
        lib.ref_save_adapter.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                         _f32p, _f32p, C.c_char_p]
        lib.ref_save_adapter.restype = C.c_int
        lib.ref_grad_check_softmax_ce.argtypes = [C.c_int, C.c_float]
        lib.ref_grad_check_softmax_ce.restype = C.c_float
        lib.ref_adam_steps.argtypes = [C.c_int, C.c_int, C.c_int, C.c_float, C.c_int, C.c_int,
                                       _f32p, _f32p, _i32p, _f32p, _f32p]
        lib.ref_adam_steps.restype = C.c_int
        self.lib = lib

    def adam_steps(self, A_dr, B_rv, gA_sums, gB_sums, n_pred, lr, step0=0):
        """The reference's mean + adam_update on given gradient sums:
        gA_sums [k][d][r], gB_sums [k][r][V], n_pred [k]; returns (A, B)."""
        d, r = A_dr.shape
        V = B_rv.shape[1]
        A = np.array(A_dr, np.float32, order="C")
        B = np.array(B_rv, np.float32, order="C")
        k = len(n_pred)
        rc = self.lib.ref_adam_steps(d, V, r, float(lr), int(step0), k,
                                     np.ascontiguousarray(gA_sums, np.float32),
                                     np.ascontiguousarray(gB_sums, np.float32),
                                     np.ascontiguousarray(n_pred, np.int32), A, B)
        if rc != 0:
            raise RuntimeError("reference adam_update harness failed")
        return A, B

    def train_steps(self, W16, H, tokens, rank, alpha, lr, seq_max, n_steps=1,
                    A_dr=None, B_rv=None, seed=42):
        V, d = W16.shape
        tokens = np.ascontiguousarray(tokens, np.int32)
        A = np.zeros((d, rank), np.float32) if A_dr is None else np.array(A_dr, np.float32, order="C")
        B = np.zeros((rank, V), np.float32) if B_rv is None else np.array(B_rv, np.float32, order="C")
        gA = np.empty((d, rank), np.float32)
        gB = np.empty((rank, V), np.float32)
        losses = np.empty(max(n_steps, 1), np.float32)
        stp = C.c_int(0)
        Hc = np.ascontiguousarray(H, np.float32)
        rc = self.lib.ref_train_steps(d, V, rank, alpha, float(lr), int(seq_max), int(seed), W16,
                                      Hc, tokens, len(tokens), n_steps,
                                      1 if A_dr is not None else 0, A, B, gA, gB, losses,
                                      C.byref(stp))
        if rc != 0:
            raise RuntimeError("reference train_step returned -1")
        return dict(losses=losses, A=A, B=B, gA=gA, gB=gB, step=stp.value)

    def save_adapter(self, path, A_dr, B_rv, alpha, step):
        d, r = A_dr.shape
        V = B_rv.shape[1]
        return self.lib.ref_save_adapter(d, V, r, alpha, step, np.ascontiguousarray(A_dr, np.float32),
                                         np.ascontiguousarray(B_rv, np.float32), path.encode())

    def grad_check_softmax_ce(self, vocab: int = 32, eps: float = 1e-3) -> float:
        return float(self.lib.ref_grad_check_softmax_ce(vocab, eps))


def ref_body_available() -> bool:
    return os.path.exists(REF_BODY_SO)


class RefBody:
    """The reference's own body forward (src/forward.c via
    oracle/_ref/libref_body.so), driven as train_step drives it: every
    position's forward_last_hidden."""

    def __init__(self, model_path: str, max_seq: int) -> None:
        lib = _load(REF_BODY_SO)
        lib.ref_body_load.argtypes = [C.c_char_p, C.c_int]
        lib.ref_body_load.restype = C.c_int
        lib.ref_body_hidden.argtypes = [_i32p, C.c_int, _f32p]
        lib.ref_body_hidden.restype = C.c_double
        lib.ref_body_free.argtypes = []
        lib.ref_body_free.restype = None
        if lib.ref_body_load(model_path.encode(), int(max_seq)) != 0:
            raise RuntimeError("reference forward_load failed")
        self.lib = lib

    def hidden(self, tokens, dim: int):
        """(H [n][dim] of one sequence, seconds in the reference forward)."""
        tok = np.ascontiguousarray(tokens, np.int32)
        out = np.empty((len(tok), dim), np.float32)
        secs = self.lib.ref_body_hidden(tok, len(tok), out)
        if secs < 0:
            raise RuntimeError("reference forward failed")
        return out, float(secs)

    def close(self) -> None:
        self.lib.ref_body_free()
