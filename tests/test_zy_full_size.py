"""Parity at the full sizes of the rank-16, Q4_K and rank-64 workloads.

The kernels take different tile, segment and chunk plans at 32,768 and
65,536 positions than at the few hundred positions of test_gpu_parity.py
(pass-1 slot counts, the tensor-core passes' 192- and 128-column plans,
lce_combine_wide, the rank-64 resident layout), so each workload runs here
once at its exact shape, through the C ABI, against the oracle on all host
cores.  Tolerances as everywhere: loss 1e-4 relative; per-position loss,
dA, dB and the updated A, B 1e-3 relative L2.  Collected after the fast
tests (and before the allocation-free entry point's file), so a failure
here does not hide them."""
import os

import numpy as np
import pytest

import lora_ce
import workload as wl

pytestmark = pytest.mark.gpu

NTHREADS = os.cpu_count() or 8
LOSS_RTOL = 1e-4
L2_RTOL = 1e-3
V, D = 49152, 576


def rel(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / max(np.linalg.norm(b), 1e-30))


def check_step(m, ref, loss, T, k):
    gA, gB, _, n_pred = m.get_grads()
    A1, B1, step = m.get_adapter()
    assert step == k + 1 and n_pred == T
    assert abs(loss - ref["loss"]) <= LOSS_RTOL * abs(ref["loss"]), (k, loss, ref["loss"])
    assert rel(m.token_loss(T), ref["loss_tok"]) <= LOSS_RTOL
    for name, a, b in (("dA", gA, ref["gA"]), ("dB", gB, ref["gB"]), ("A", A1, ref["A"]),
                       ("B", B1, ref["B"])):
        e = rel(a, b)
        assert e <= L2_RTOL, f"step {k}: {name} rel L2 {e:.3e}"


def run_workload(oracle, r, alpha, T, steps, wd, clip, q4k=False, seed=1000):
    h, tgt, _, _ = wl.make_step_inputs(seed, T, V, D, r)
    _, _, A, B = wl.make_step_inputs(seed, 8, V, D, r)
    Hor = wl.oracle_hidden(h)
    if q4k:
        blocks = wl.make_weight_q4k(1, V, D)
        W16 = oracle.q4k_dequant(blocks).astype(np.float16).view(np.uint16).reshape(V, D)
    else:
        W16 = wl.make_weight(1, V, D)
    scale = alpha / r
    cfg = lora_ce.default_config(D, V, r, T, scale=scale, lr=1e-3, weight_decay=wd,
                                 clip_norm=clip)
    m = lora_ce.LoraCE(cfg)
    if q4k:
        m.set_weight_q4k(blocks)
    else:
        m.set_weight(W16)
    m.set_adapter(A, B, 0)
    state, Ao, Bo = None, A, B
    try:
        for k in range(steps):  # Adam moments carried on both sides
            loss = m.step(h, tgt)
            ref = oracle.step(W16, Ao, Bo, Hor, tgt, scale, 1e-3, wd=wd, clip=clip,
                              nthreads=NTHREADS, state=state)
            state, Ao, Bo = ref["state"], ref["A"], ref["B"]
            check_step(m, ref, loss, T, k)
    finally:
        m.close()


def test_rank16_65536_positions(oracle):
    """Rank 16, alpha 32, 65,536 positions on one GPU (the strong-scaling
    workload's total), AdamW wd 0.01: one step."""
    run_workload(oracle, r=16, alpha=32, T=65536, steps=1, wd=0.01, clip=0.0)


def test_q4k_rank8_32768_positions(oracle):
    """Q4_K lm_head (dequantised on the GPU), rank 8, alpha 16, 32,768
    positions, AdamW wd 0.01: one step against the oracle on the same f16
    weights (the oracle's own dequantisation)."""
    run_workload(oracle, r=8, alpha=16, T=32768, steps=1, wd=0.01, clip=0.0, q4k=True)


def test_rank64_long_context_three_steps(oracle):
    """The long-context batch: 32 x 2048 = 65,536 positions, rank 64,
    alpha 128, AdamW wd 0.01 with grad-clip 1.0: three steps with the Adam
    moments carried on both sides."""
    run_workload(oracle, r=64, alpha=128, T=65536, steps=3, wd=0.01, clip=1.0)
