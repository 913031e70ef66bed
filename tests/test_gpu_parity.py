"""Parity of the CUDA path (through the C ABI) with the oracle on seeded
inputs.  Tolerances: loss within 1e-4 relative; dA, dB and the updated A, B
within 1e-3 relative L2; target indexing exact."""
import os

import numpy as np
import pytest

import lora_ce
import workload as wl

pytestmark = pytest.mark.gpu

NTHREADS = os.cpu_count() or 8
LOSS_RTOL = 1e-4
L2_RTOL = 1e-3


def rel(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / max(np.linalg.norm(b), 1e-30))


def make(V, d, r, T, seed, dtype="bf16"):
    W = wl.make_weight(seed, V, d)
    h, tgt, A, B = wl.make_step_inputs(seed, T, V, d, r)
    Hor = wl.oracle_hidden(h)
    if dtype == "bf16":
        H = h
    elif dtype == "f16":
        H = Hor.astype(np.float16)
    else:
        H = Hor.copy()  # f32 values already f16-representable
    return W, H, Hor, tgt, A, B


def run_case(oracle, V, d, r, T, seed, dtype="bf16", steps=1, scale=2.0, lr=1e-3, wd=0.0,
             clip=0.0):
    W, H, Hor, tgt, A, B = make(V, d, r, T, seed, dtype)
    cfg = lora_ce.default_config(d, V, r, T, scale=scale, lr=lr, weight_decay=wd,
                                 clip_norm=clip)
    m = lora_ce.LoraCE(cfg)
    m.set_weight(W)
    m.set_adapter(A, B, 0)
    state, Ao, Bo = None, A, B
    for k in range(steps):
        loss = m.step(H, tgt)
        ref = oracle.step(W, Ao, Bo, Hor, tgt, scale, lr, wd=wd, clip=clip, nthreads=NTHREADS,
                          state=state)
        state, Ao, Bo = ref["state"], ref["A"], ref["B"]
        gA, gB, loss_sum, n_pred = m.get_grads()
        A1, B1, step = m.get_adapter()
        assert step == k + 1 and n_pred == T
        assert abs(loss - ref["loss"]) <= LOSS_RTOL * abs(ref["loss"]), (k, loss, ref["loss"])
        tl = m.token_loss(T)
        assert rel(tl, ref["loss_tok"]) <= LOSS_RTOL
        for name, a, b in (("dA", gA, ref["gA"]), ("dB", gB, ref["gB"]), ("A", A1, Ao),
                           ("B", B1, Bo)):
            e = rel(a, b)
            assert e <= L2_RTOL, f"step {k}: {name} rel L2 {e:.3e}"
        # continue both from the GPU state so later steps test one update each
        Ao, Bo = A1, B1
        m.set_adapter(A1, B1, step)
        state["mA"], state["vA"], state["mB"], state["vB"] = (np.zeros_like(state["mA"]),
                                                              np.zeros_like(state["vA"]),
                                                              np.zeros_like(state["mB"]),
                                                              np.zeros_like(state["vB"]))
    m.close()


@pytest.mark.parametrize(
    "V,d,r,T,dtype",
    [
        (49152, 576, 4, 256, "bf16"),   # the isolated-op shape at reduced T
        (49152, 576, 4, 1, "bf16"),     # a single position
        (4099, 128, 4, 129, "f16"),     # V and T off the tile grid
        (1000, 64, 8, 300, "f32"),      # small d, rank 8, f32 input
        (2048, 576, 16, 513, "bf16"),   # rank 16
        (49152, 576, 8, 127, "bf16"),
        (3000, 128, 1, 77, "bf16"),     # ranks padded to the kernels' 4 / 8 / 16
        (3000, 192, 3, 40, "f16"),
        (2048, 576, 13, 100, "bf16"),
        (49152, 576, 16, 700, "bf16"),  # rank augmentation at full vocabulary
        (4099, 128, 32, 100, "bf16"),   # rank chunks: 2 x 16, augmentation layout 2
        (3000, 192, 20, 77, "f16"),     # padded to 32
        (2048, 576, 40, 260, "bf16"),   # padded to 64
        (49152, 576, 64, 300, "bf16"),  # rank 64 at full vocabulary (11 resident K-blocks)
        (49152, 576, 100, 300, "bf16"),  # wide-rank path (kernel rank 128)
        (3000, 192, 65, 77, "f16"),
        (4099, 128, 256, 129, "f32"),  # LORA_MAX_RANK, vocabulary and positions off the tiles
        (49152, 576, 256, 1, "bf16"),
    ],
)
def test_step_matches_oracle(oracle, V, d, r, T, dtype):
    run_case(oracle, V, d, r, T, seed=V + T + r, dtype=dtype, steps=2)


@pytest.mark.parametrize("tc", ["0", "1"])
@pytest.mark.parametrize(
    "V,d,r,T,dtype",
    [
        (1000, 64, 8, 300, "f32"),
        (2048, 576, 13, 100, "bf16"),
        (2048, 576, 16, 513, "bf16"),
        (4099, 128, 32, 300, "bf16"),   # vocabulary and positions off both tile grids
        (3000, 192, 20, 77, "f16"),
        (49152, 576, 64, 300, "bf16"),
    ],
)
def test_step_matches_oracle_both_rank_paths(oracle, monkeypatch, tc, V, d, r, T, dtype):
    """Ranks 8..64 down both paths: the tensor-core rank sums (LORA_CE_TC=1
    uses them from rank 8) and the per-logit epilogues with rank chunks
    above 16 (LORA_CE_TC=0)."""
    monkeypatch.setenv("LORA_CE_TC", tc)
    run_case(oracle, V, d, r, T, seed=V + T + r + 1, dtype=dtype, steps=2)


def test_adamw_and_clip_extensions(oracle):
    run_case(oracle, 49152, 576, 4, 300, seed=77, wd=0.01, clip=1.0, steps=2)
    run_case(oracle, 3000, 128, 4, 50, seed=78, wd=0.01, clip=1e-4, steps=1)  # clip active


def test_wide_rank_adamw_clip_and_position_blocks(oracle):
    """Ranks above 64 (the wide-rank path): AdamW with an active clip, and a
    vocabulary large enough that 3000 positions run as three position
    blocks (512 MB of logit rows hold 1280 positions at V = 100,000)."""
    run_case(oracle, 3000, 128, 128, 200, seed=91, wd=0.01, clip=1e-4, steps=2)
    run_case(oracle, 100000, 64, 72, 3000, seed=92, steps=1)


def test_adam_state_carries_over_steps(oracle):
    """Three consecutive steps with the Adam moments kept on both sides."""
    V, d, r, T = 8192, 576, 4, 200
    W, H, Hor, tgt, A, B = make(V, d, r, T, 5)
    m = lora_ce.LoraCE(lora_ce.default_config(d, V, r, T, scale=2.0, lr=1e-3))
    m.set_weight(W)
    m.set_adapter(A, B, 0)
    state = None
    Ao, Bo = A, B
    for k in range(3):
        loss = m.step(H, tgt)
        ref = oracle.step(W, Ao, Bo, Hor, tgt, 2.0, 1e-3, nthreads=NTHREADS, state=state)
        state, Ao, Bo = ref["state"], ref["A"], ref["B"]
        assert abs(loss - ref["loss"]) <= LOSS_RTOL * ref["loss"]
    A1, B1, step = m.get_adapter()
    assert step == 3
    assert rel(A1, Ao) <= L2_RTOL and rel(B1, Bo) <= L2_RTOL
    m.close()


def test_target_indexing_matches_train_step(oracle):
    """tokens -> targets: positions 0..use_n-2 predict tokens[pos+1] with
    use_n = min(n, seq_max) (src/train.c:198-229)."""
    V, d, r = 4096, 128, 4
    W, H, Hor, tgt, A, B = make(V, d, r, 64, 9)
    tokens = np.concatenate([[3], tgt]).astype(np.int32)
    for seq_max in (65, 30, 2):
        m = lora_ce.LoraCE(lora_ce.default_config(d, V, r, 64, scale=2.0, lr=1e-3))
        m.set_weight(W)
        m.set_adapter(A, B, 0)
        loss = m.train_step_tokens(H, tokens, seq_max)
        ref = oracle.train_step_tokens(W, A, B, Hor, tokens, seq_max, 2.0, 1e-3)
        _, _, _, n_pred = m.get_grads()
        assert n_pred == min(len(tokens), seq_max) - 1
        assert abs(loss - ref["loss"]) <= LOSS_RTOL * ref["loss"]
        m.close()
    m = lora_ce.LoraCE(lora_ce.default_config(d, V, r, 64))
    m.set_weight(W)
    assert m.train_step_tokens(H, tokens[:1], 10) == -1.0
    m.close()


def test_deterministic():
    V, d, r, T = 49152, 576, 4, 1000
    W, H, _, tgt, A, B = make(V, d, r, T, 21)
    outs = []
    for _ in range(2):
        m = lora_ce.LoraCE(lora_ce.default_config(d, V, r, T, scale=2.0, lr=1e-3))
        m.set_weight(W)
        m.set_adapter(A, B, 0)
        loss = m.step(H, tgt)
        outs.append((loss,) + m.get_grads()[:2] + m.get_adapter()[:2])
        m.close()
    for a, b in zip(outs[0], outs[1]):
        np.testing.assert_array_equal(a, b)


def test_adapter_roundtrip_and_lora0001(tmp_path):
    V, d, r = 2048, 128, 8
    W, _, _, _, A, B = make(V, d, r, 4, 3)
    m = lora_ce.LoraCE(lora_ce.default_config(d, V, r, 16))
    m.set_weight(W)
    m.set_adapter(A, B, 17)
    A1, B1, s = m.get_adapter()
    np.testing.assert_array_equal(A1, A)
    np.testing.assert_array_equal(B1, B)
    assert s == 17
    p = str(tmp_path / "lora.bin")
    m.save(p)
    assert os.path.getsize(p) == 28 + 4 * d * r + 4 * r * V
    m2 = lora_ce.LoraCE(lora_ce.default_config(d, V, r, 16))
    m2.load(p)
    A2, B2, s2 = m2.get_adapter()
    np.testing.assert_array_equal(A2, A)
    np.testing.assert_array_equal(B2, B)
    assert s2 == 17
    m.close()
    m2.close()


def test_errors_are_reported_not_raised_on_device():
    V, d, r, T = 1024, 64, 4, 32
    W, H, _, tgt, A, B = make(V, d, r, T, 4)
    m = lora_ce.LoraCE(lora_ce.default_config(d, V, r, T))
    with pytest.raises(lora_ce.LoraCEError, match="ESTATE"):
        m.step(H, tgt)  # no weight yet
    m.set_weight(W)
    with pytest.raises(lora_ce.LoraCEError, match="EINVAL"):
        m.step(np.zeros((T + 1, d), np.uint16), np.zeros(T + 1, np.int32))  # T > max_tokens
    bad = tgt.copy()
    bad[5] = V  # caught by the kernel's range check, clamped, reported
    with pytest.raises(lora_ce.LoraCEError, match="EDEVICE"):
        m.step(H, bad)
    with pytest.raises(lora_ce.LoraCEError, match="ESTATE"):
        m.step(H, tgt)  # poisoned
    m.close()
    # the context is still usable
    m = lora_ce.LoraCE(lora_ce.default_config(d, V, r, T))
    m.set_weight(W)
    m.set_adapter(A, B, 0)
    assert np.isfinite(m.step(H, tgt))
    m.close()


def test_full_size_isolated_op(oracle):
    """h [8192x576], W [49152x576], r = 4: one step against the oracle
    (all host cores), plus the additivity of the gradient sums over two
    halves of the positions."""
    V, d, r, T = 49152, 576, 4, 8192
    W, H, Hor, tgt, A, B = make(V, d, r, T, 2024)
    m = lora_ce.LoraCE(lora_ce.default_config(d, V, r, T, scale=2.0, lr=1e-3))
    m.set_weight(W)
    m.set_adapter(A, B, 0)
    loss = m.step(H, tgt)
    gA, gB, lsum, n = m.get_grads()
    A1, B1, _ = m.get_adapter()
    ref = oracle.step(W, A, B, Hor, tgt, 2.0, 1e-3, nthreads=NTHREADS)
    assert abs(loss - ref["loss"]) <= LOSS_RTOL * ref["loss"]
    for name, a, b in (("dA", gA, ref["gA"]), ("dB", gB, ref["gB"]), ("A", A1, ref["A"]),
                       ("B", B1, ref["B"])):
        assert rel(a, b) <= L2_RTOL, (name, rel(a, b))
    # sums over the halves add up to the sum over all positions
    sums = []
    for sl in (slice(0, T // 2), slice(T // 2, T)):
        m.set_adapter(A, B, 0)
        m.step(np.ascontiguousarray(H[sl]), np.ascontiguousarray(tgt[sl]))
        ga, gb, ls, nn = m.get_grads()
        sums.append((ga * nn, gb * nn, ls))
    assert rel(sums[0][0] + sums[1][0], gA * n) <= 1e-5
    assert rel(sums[0][1] + sums[1][1], gB * n) <= 1e-5
    assert abs(sums[0][2] + sums[1][2] - lsum) <= 1e-5 * lsum
    m.close()


@pytest.mark.parametrize("rank", [4, 64, 256])
def test_merge_bit_exact(oracle, rank):
    """GPU merge == the reference's merge arithmetic, bit for bit, on the
    full 49152 x 576 lm_head with f16 edge patterns."""
    V, d = 49152, 576
    W = wl.make_weight(90 + rank, V, d)
    edge = np.array([0x0001, 0x8001, 0x03FF, 0x83FF, 0x0200, 0x7C00, 0xFC00, 0x7E00, 0x0000,
                     0x8000, 0x7BFF, 0xFBFF, 0x0400, 0x8400], np.uint16)
    W[0, :len(edge)] = edge
    W[V - 1, -len(edge):] = edge
    rng = np.random.default_rng(rank)
    A = rng.standard_normal((d, rank), dtype=np.float32) * np.float32(1.0 / np.sqrt(d))
    B = rng.standard_normal((rank, V), dtype=np.float32) * np.float32(1e-2)
    got = lora_ce.merge_weight(W, A, B, 16.0 / rank)
    if rank == 4:
        ref = oracle.merge(W, A, B, 16.0 / rank)
    else:  # the full oracle merge at rank 256 takes minutes; check a row sample
        rows = np.r_[0:64, V - 64:V]
        ref_rows = oracle.merge(np.ascontiguousarray(W[rows]), A, np.ascontiguousarray(B[:, rows]),
                                16.0 / rank)
        got, ref = got[rows], ref_rows
    np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("V,d,r", [(4099, 1096, 256), (1000, 64, 1), (333, 2048, 5)])
def test_merge_ragged_shapes(oracle, V, d, r):
    """Column tiles that do not divide d, V off the row tile, rank 1, and
    the k-chunked path (rank 256 at d = 1096)."""
    W = wl.make_weight(V + d + r, V, d)
    rng = np.random.default_rng(V * r)
    A = rng.standard_normal((d, r), dtype=np.float32) * np.float32(0.05)
    B = rng.standard_normal((r, V), dtype=np.float32) * np.float32(0.05)
    np.testing.assert_array_equal(lora_ce.merge_weight(W, A, B, 8.0 / r),
                                  oracle.merge(W, A, B, 8.0 / r))


def test_q4k_dequant_bit_exact(oracle):
    """Q4_K -> f32 on the GPU == the oracle's restatement, bit for bit, over
    the QLoRA lm_head (110,592 super-blocks); the f16 output is that value
    rounded to nearest."""
    blocks = wl.make_weight_q4k(4, 49152, 576)
    want = oracle.q4k_dequant(blocks)
    got = lora_ce.q4k_dequant(blocks, lora_ce.F32)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    got16 = lora_ce.q4k_dequant(blocks, lora_ce.F16)
    np.testing.assert_array_equal(got16, want.astype(np.float16).view(np.uint16))


def test_q4k_step_matches_oracle(oracle):
    """The QLoRA step (r 8, Q4_K lm_head dequantised once into the f16
    operand) against the oracle on the same f16 weights."""
    V, d, r, T = 49152, 576, 8, 512
    blocks = wl.make_weight_q4k(6, V, d)
    W16 = oracle.q4k_dequant(blocks).astype(np.float16).view(np.uint16).reshape(V, d)
    h, tgt, A, B = wl.make_step_inputs(6, T, V, d, r)
    m = lora_ce.LoraCE(lora_ce.default_config(d, V, r, T, scale=2.0, lr=1e-3))
    m.set_weight_q4k(blocks)
    m.set_adapter(A, B, 0)
    loss = m.step(h, tgt)
    gA, gB, _, _ = m.get_grads()
    A1, B1, _ = m.get_adapter()
    m.close()
    ref = oracle.step(W16, A, B, wl.oracle_hidden(h), tgt, 2.0, 1e-3, nthreads=NTHREADS)
    assert abs(loss - ref["loss"]) <= LOSS_RTOL * ref["loss"]
    for name, a, b in (("dA", gA, ref["gA"]), ("dB", gB, ref["gB"]), ("A", A1, ref["A"]),
                       ("B", B1, ref["B"])):
        assert rel(a, b) <= L2_RTOL, (name, rel(a, b))


def test_chunked_host_step_matches_device_step():
    """lora_ce_step copies h in chunks and runs pass 1 per chunk (T 8192: four
    launches); lora_ce_step_device runs it as one launch.  The two differ
    only in how the pass-1 partials are grouped: 1e-5 apart."""
    import torch
    V, d, r, T = 49152, 576, 4, 8192
    W, H, _, tgt, A, B = make(V, d, r, T, 55)
    outs = []
    for mode in ("host", "device"):
        m = lora_ce.LoraCE(lora_ce.default_config(d, V, r, T, scale=2.0, lr=1e-3))
        m.set_weight(W)
        m.set_adapter(A, B, 0)
        if mode == "host":
            loss = m.step(H, tgt)
        else:
            dH = torch.from_numpy(H.view(np.int16)).cuda()
            dT = torch.from_numpy(tgt).cuda()
            dL = torch.zeros(2, dtype=torch.float32, device="cuda")
            m.step_device(dH.data_ptr(), lora_ce.BF16, T, dT.data_ptr(), dL.data_ptr())
            m.sync()
            loss = float(dL[0].item())
        gA, gB, _, n = m.get_grads()
        A1, B1, _ = m.get_adapter()
        outs.append((loss, gA, gB, A1, B1))
        m.close()
    (l0, *a0), (l1, *a1) = outs
    assert abs(l0 - l1) <= 1e-5 * abs(l1)
    for x, y in zip(a0, a1):
        assert rel(x, y) <= 1e-5


def test_graph_replay_reads_current_inputs(oracle):
    """Steps are CUDA-graph replays once (T, dtype, buffers) repeat: a replay
    must copy the buffers' current contents and apply this step's Adam bias
    corrections.  Three steps with new data in the same host buffers, with
    graphs on and off."""
    V, d, r, T = 8192, 576, 4, 512
    W = wl.make_weight(70, V, d)
    _, _, A, B = wl.make_step_inputs(70, T, V, d, r)
    batches = [wl.make_step_inputs(71 + k, T, V, d, r)[:2] for k in range(3)]
    results = []
    for graphs in ("1", "0"):
        os.environ["LORA_CE_GRAPHS"] = graphs
        try:
            m = lora_ce.LoraCE(lora_ce.default_config(d, V, r, T, scale=2.0, lr=1e-3))
        finally:
            os.environ.pop("LORA_CE_GRAPHS", None)
        m.set_weight(W)
        m.set_adapter(A, B, 0)
        H = np.empty_like(batches[0][0])
        tg = np.empty_like(batches[0][1])
        losses = []
        for h, t in batches:
            H[...] = h
            tg[...] = t
            losses.append(m.step(H, tg))
        A1, B1, step = m.get_adapter()
        assert step == 3
        results.append((losses, A1, B1))
        m.close()
    (l_g, A_g, B_g), (l_d, A_d, B_d) = results
    np.testing.assert_array_equal(np.float32(l_g), np.float32(l_d))
    np.testing.assert_array_equal(A_g, A_d)
    np.testing.assert_array_equal(B_g, B_d)
    # and the losses follow the oracle step by step
    state, Ao, Bo = None, A, B
    for (h, t), lg in zip(batches, l_g):
        ref = oracle.step(W, Ao, Bo, wl.oracle_hidden(h), t, 2.0, 1e-3, nthreads=NTHREADS,
                          state=state)
        state, Ao, Bo = ref["state"], ref["A"], ref["B"]
        assert abs(lg - ref["loss"]) <= LOSS_RTOL * ref["loss"]


def test_rank64_adamw_clip_and_graph_replay(oracle):
    """Rank 64 (16-rank chunks, augmentation layout 2) with weight decay and
    an active clip over three steps (graph replays after the first), and
    bit-identical results on a second handle."""
    V, d, r, T = 8192, 576, 64, 384
    W, H, Hor, tgt, A, B = make(V, d, r, T, 64)
    runs = []
    for _ in range(2):
        m = lora_ce.LoraCE(lora_ce.default_config(d, V, r, T, scale=2.0, lr=1e-3,
                                                  weight_decay=0.01, clip_norm=1e-3))
        m.set_weight(W)
        m.set_adapter(A, B, 0)
        losses = [m.step(H, tgt) for _ in range(3)]
        A1, B1, step = m.get_adapter()
        assert step == 3
        runs.append((losses, A1, B1))
        m.close()
    np.testing.assert_array_equal(np.float32(runs[0][0]), np.float32(runs[1][0]))
    np.testing.assert_array_equal(runs[0][1], runs[1][1])
    np.testing.assert_array_equal(runs[0][2], runs[1][2])
    state, Ao, Bo = None, A, B
    for k in range(3):
        ref = oracle.step(W, Ao, Bo, Hor, tgt, 2.0, 1e-3, wd=0.01, clip=1e-3, nthreads=NTHREADS,
                          state=state)
        state, Ao, Bo = ref["state"], ref["A"], ref["B"]
        assert abs(runs[0][0][k] - ref["loss"]) <= LOSS_RTOL * ref["loss"]
    assert rel(runs[0][1], Ao) <= L2_RTOL and rel(runs[0][2], Bo) <= L2_RTOL


@pytest.mark.parametrize("V,d,r", [(49152, 576, 4), (3001, 64, 13), (49152, 576, 64)])
def test_adam_kernel_bit_exact_with_reference_adam_update(V, d, r):
    """lce_adam (through lora_ce_apply_grads) against the reference's own
    mean + adam_update (src/train.c:230-239, 175-196; oracle/_ref) on
    identical gradient sums: three updates with the moments carried, the
    adapter bit-equal after each run (weight decay 0, no clip: the
    reference's Adam)."""
    import oracle as orc

    k = 3
    A, B, gA, gB, n_pred = wl.make_adam_inputs(V + r, d, V, r, k)
    m = lora_ce.LoraCE(lora_ce.default_config(d, V, r, 16, scale=2.0, lr=1e-3))
    m.set_adapter(A, B, 0)
    for i in range(k):
        m.apply_grads(gA[i], gB[i], float(n_pred[i]))
    A1, B1, step = m.get_adapter()
    m.close()
    Ar, Br = orc.RefHarness().adam_steps(A, B, gA, gB, n_pred, 1e-3)
    assert step == k
    assert np.array_equal(A1.view(np.uint32), Ar.view(np.uint32))
    assert np.array_equal(B1.view(np.uint32), Br.view(np.uint32))


def test_copy_timing_of_host_steps():
    """lora_ce_set_copy_timing: timed host-input steps launch directly with
    events between the copies; the step's results do not change, and the
    reported times are consistent (chunk copies inside the step)."""
    V, d, r, T = 49152, 576, 4, 8192
    W, H, _, tgt, A, B = make(V, d, r, T, 91)
    res = []
    for timing in (False, True):
        m = lora_ce.LoraCE(lora_ce.default_config(d, V, r, T, scale=2.0, lr=1e-3))
        m.set_weight(W)
        m.set_adapter(A, B, 0)
        m.set_copy_timing(timing)
        losses = [m.step(H, tgt) for _ in range(3)]
        if timing:
            t = m.copy_times()
            assert len(t["chunk_ms"]) == 4
            assert t["host_us"] > 0 and t["wait_us"] >= 0
            assert 0 < sum(t["chunk_ms"]) < t["step_ms"]
        res.append((losses, m.get_adapter()[1]))
        m.close()
    assert res[0][0] == res[1][0]
    assert np.array_equal(res[0][1], res[1][1])
