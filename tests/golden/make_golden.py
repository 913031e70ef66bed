"""Generate the golden fixtures in this directory from the reference's OWN
code (oracle/_ref/libref_train.so: src/train.c and src/backward.c compiled
unmodified from the reference tree by oracle/Makefile).

Run from the repository root, where the reference tree is available:
    python tests/golden/make_golden.py

Inputs are re-generated from seeds by smollm2.c_b200/workload.py, so only
outputs are stored: full arrays for the small cases, SHA-256 digests of the
f32 bytes (plus a few values) for the full-vocabulary cases.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "oracle"))
sys.path.insert(0, os.path.join(REPO, "smollm2.c_b200"))

import oracle as orc  # noqa: E402
import workload as wl  # noqa: E402

# name, V, d, r, alpha, T (predicted positions), n_steps, seq_max, seed
CASES = [
    ("small_r4", 2048, 128, 4, 8, 33, 3, 4096, 5),
    ("small_r8_seqcap", 1000, 64, 8, 16, 40, 2, 17, 6),
    ("small_r16", 1031, 128, 16, 32, 9, 2, 4096, 7),
    ("full_r4", 49152, 576, 4, 8, 8, 2, 4096, 8),
]


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


EDGE_F16 = [0x0001, 0x8001, 0x03FF, 0x83FF, 0x0200, 0x7C00, 0xFC00, 0x7E00, 0x0000, 0x8000,
            0x7BFF, 0xFBFF, 0x0400, 0x8400]


def merge_inputs():
    """Seeded W (4099 x 576) with f16 edge patterns, A [576][8], B [8][4099]."""
    W = wl.make_weight(77, 4099, 576)
    W[0, :len(EDGE_F16)] = np.array(EDGE_F16, np.uint16)
    W[4098, -len(EDGE_F16):] = np.array(EDGE_F16, np.uint16)
    rng = np.random.default_rng(77)
    A = rng.standard_normal((576, 8), dtype=np.float32)
    B = (rng.standard_normal((8, 4099), dtype=np.float32) * np.float32(0.3)).astype(np.float32)
    return W, A, B


def case_inputs(V, d, r, T, seed):
    W = wl.make_weight(seed, V, d)
    h, tgt, A, B = wl.make_step_inputs(seed, T, V, d, r)
    H = wl.oracle_hidden(h)
    tokens = np.concatenate([[int(tgt[0]) ^ 1], tgt]).astype(np.int32)
    return W, H, tokens, A, B


def main() -> None:
    ref = orc.RefHarness()
    meta = {"cases": {}}
    for name, V, d, r, alpha, T, n_steps, seq_max, seed in CASES:
        W, H, tokens, A, B = case_inputs(V, d, r, T, seed)
        out = ref.train_steps(W, H, tokens, r, alpha, 1e-3, seq_max, n_steps=n_steps,
                              A_dr=A, B_rv=B)
        entry = dict(V=V, d=d, r=r, alpha=alpha, T=T, n_steps=n_steps, seq_max=seq_max,
                     seed=seed, lr=1e-3, losses=[float(x) for x in out["losses"]],
                     step=out["step"])
        for k in ("A", "B", "gA", "gB"):
            entry["sha_" + k] = sha(out[k])
            entry["head_" + k] = [float(x) for x in out[k].ravel()[:4]]
        if V * d <= 1 << 20:
            np.savez_compressed(os.path.join(HERE, f"{name}.npz"), A=out["A"], B=out["B"],
                                gA=out["gA"], gB=out["gB"], losses=out["losses"])
        meta["cases"][name] = entry
        print(name, entry["losses"])
    # softmax-CE finite-difference check, vocab 32, eps 1e-4 (cmd_grad_check default)
    meta["grad_check_softmax_ce"] = ref.grad_check_softmax_ce(32, 1e-4)
    # train_create's Kaiming init (seed 42, d 576, r 4) and train_save's bytes
    init = ref.train_steps(wl.make_weight(1, 64, 576), np.zeros((1, 576), np.float32),
                           np.array([0, 1], np.int32), 4, 8, 1e-3, 4096, n_steps=0)
    meta["kaiming_seed42_sha"] = sha(init["A"])
    meta["kaiming_seed42_head"] = [float(x) for x in init["A"].ravel()[:4]]
    rng = np.random.default_rng(9)
    A = rng.standard_normal((576, 4), dtype=np.float32)
    B = rng.standard_normal((4, 49152), dtype=np.float32)
    with tempfile.TemporaryDirectory() as td:
        p = os.path.join(td, "a.bin")
        ref.save_adapter(p, A, B, 8, 7)
        data = open(p, "rb").read()
    meta["lora0001_seed9"] = {"size": len(data), "sha": hashlib.sha256(data).hexdigest(),
                              "alpha": 8, "step": 7}
    # the reference's merge (lora_patched_weight): seeded W with f16 edge
    # patterns (subnormals, inf, NaN, zeros), A, B, scale 2
    Wm, Am, Bm = merge_inputs()
    out = np.empty_like(Wm)
    f = ref.lib.ref_merge_weight
    u16 = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
    f32 = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
    import ctypes as C
    f.argtypes = [u16, f32, f32, C.c_int, C.c_int, C.c_int, C.c_float, u16]
    f.restype = C.c_int
    assert f(Wm, Am, Bm, Wm.shape[1], Am.shape[1], Wm.shape[0], 2.0, out) == 0
    meta["merge_4099x576_r8"] = {"sha": sha(out), "changed": int((out != Wm).sum())}
    # Q4_K has no reference implementation: the digest pins the restatement
    # of the public format against drift
    meta["q4k_seed4_49152x576_sha"] = sha(orc.Oracle().q4k_dequant(wl.make_weight_q4k(4, 49152, 576)))
    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)
    print("grad_check", meta["grad_check_softmax_ce"], "lora0001 bytes", len(data))


if __name__ == "__main__":
    main()
