"""The CPU checker is pinned before it is trusted: bit-exact against the
committed fixtures (made by the reference's own src/train.c, see
tests/golden/make_golden.py), against the reference built here when its
sources are present, and against the published grad-check value."""
import hashlib
import os
import tempfile

import numpy as np
import pytest

import oracle as orc
import workload as wl
import lora_ce

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def case_inputs(V, d, r, T, seed):
    W = wl.make_weight(seed, V, d)
    h, tgt, A, B = wl.make_step_inputs(seed, T, V, d, r)
    H = wl.oracle_hidden(h)
    tokens = np.concatenate([[int(tgt[0]) ^ 1], tgt]).astype(np.int32)
    return W, H, tokens, A, B


@pytest.mark.parametrize("name", ["small_r4", "small_r8_seqcap", "small_r16", "full_r4"])
def test_oracle_matches_reference_fixtures(oracle, golden, name):
    c = golden["cases"][name]
    W, H, tokens, A, B = case_inputs(c["V"], c["d"], c["r"], c["T"], c["seed"])
    state = None
    losses = []
    for _ in range(c["n_steps"]):
        out = oracle.train_step_tokens(W, A, B, H, tokens, c["seq_max"], c["alpha"] / c["r"],
                                       c["lr"], state=state)
        state = out["state"]
        A, B = out["A"], out["B"]
        losses.append(out["loss"])
    np.testing.assert_array_equal(np.float32(losses), np.float32(c["losses"]))
    assert state["step"] == c["step"]
    for k in ("A", "B", "gA", "gB"):
        assert sha(out[k]) == c["sha_" + k], k
    npz = os.path.join(GOLDEN, f"{name}.npz")
    if os.path.exists(npz):
        ref = np.load(npz)
        for k in ("A", "B", "gA", "gB"):
            np.testing.assert_array_equal(out[k], ref[k])


def test_grad_check_softmax_ce_known_answer(oracle, golden):
    # published: 1.651e-05 (vocab 32, srand(42)); same bits as the reference here
    e = oracle.grad_check_softmax_ce(32, 1e-4)
    assert e == pytest.approx(1.651e-05, abs=5e-9)
    assert np.float32(e) == np.float32(golden["grad_check_softmax_ce"])


def test_kaiming_init_matches_train_create(oracle, golden):
    A = oracle.kaiming_init(42, 576, 4)
    assert sha(A) == golden["kaiming_seed42_sha"]


def test_lora0001_writer_is_byte_identical(golden):
    g = golden["lora0001_seed9"]
    rng = np.random.default_rng(9)
    A = rng.standard_normal((576, 4), dtype=np.float32)
    B = rng.standard_normal((4, 49152), dtype=np.float32)
    with tempfile.TemporaryDirectory() as td:
        p = os.path.join(td, "a.bin")
        lora_ce.save_lora0001(p, A, B, g["alpha"] / 4, g["step"])
        data = open(p, "rb").read()
        assert len(data) == g["size"] == 795676  # spec/014: ~795 KB at rank 4
        assert hashlib.sha256(data).hexdigest() == g["sha"]
        ad = lora_ce.load_lora0001(p, 576, 49152, 4)
        np.testing.assert_array_equal(ad["A"], A)
        np.testing.assert_array_equal(ad["B"], B)
        assert ad["step"] == g["step"]
        with pytest.raises(ValueError):
            lora_ce.load_lora0001(p, 576, 49152, 8)


def test_threaded_oracle_close_to_sequential(oracle):
    W, H, tokens, A, B = case_inputs(2048, 128, 4, 40, 3)
    tg = tokens[1:]
    a = oracle.accumulate(W, A, B, H, tg, 2.0, nthreads=1)
    b = oracle.accumulate(W, A, B, H, tg, 2.0, nthreads=4)
    np.testing.assert_array_equal(a[2], b[2])  # per-position loss is per-row work
    for x, y in zip(a[:2], b[:2]):
        assert np.linalg.norm(x - y) <= 1e-6 * np.linalg.norm(x)


def test_oracle_rejects_bad_targets(oracle):
    W, H, tokens, A, B = case_inputs(512, 64, 4, 5, 1)
    bad = tokens[1:].copy()
    bad[2] = 512
    with pytest.raises(ValueError):
        oracle.accumulate(W, A, B, H, bad, 2.0)


@pytest.mark.skipif(not orc.ref_available(), reason="reference not built here")
@pytest.mark.parametrize("V,d,r,T,seq_max", [(777, 64, 4, 12, 4096), (3000, 128, 8, 20, 9)])
def test_oracle_bit_exact_with_reference_build(oracle, V, d, r, T, seq_max):
    ref = orc.RefHarness()
    W, H, tokens, A, B = case_inputs(V, d, r, T, V + T)
    a = ref.train_steps(W, H, tokens, r, 2 * r, 1e-3, seq_max, n_steps=1, A_dr=A, B_rv=B)
    b = oracle.train_step_tokens(W, A, B, H, tokens, seq_max, 2.0, 1e-3)
    assert np.float32(a["losses"][0]) == np.float32(b["loss"])
    for k in ("A", "B", "gA", "gB"):
        np.testing.assert_array_equal(a[k], b[k])


def test_target_indexing_edge_cases(oracle):
    # fewer than two usable tokens -> -1.0, as train_step returns
    W, H, tokens, A, B = case_inputs(512, 64, 4, 5, 2)
    assert oracle.train_step_tokens(W, A, B, H, tokens[:1], 4096, 2.0, 1e-3)["loss"] == -1.0
    assert oracle.train_step_tokens(W, A, B, H, tokens, 1, 2.0, 1e-3)["loss"] == -1.0


def test_merge_matches_reference_fixture(oracle, golden):
    """oracle/lora_oracle.c's merge reproduces the reference's
    lora_patched_weight bit for bit (f16 edge patterns included)."""
    import sys
    sys.path.insert(0, GOLDEN)
    from make_golden import merge_inputs
    W, A, B = merge_inputs()
    out = oracle.merge(W, A, B, 2.0)
    assert sha(out) == golden["merge_4099x576_r8"]["sha"]
    assert int((out != W).sum()) == golden["merge_4099x576_r8"]["changed"]


def _pack_q4k_scales(sc, m):
    """Inverse of the Q4_K 6-bit (scale, min) packing, from the format's definition."""
    q = np.zeros(12, np.uint8)
    for j in range(4):
        q[j] = (sc[j] & 63) | ((sc[j + 4] >> 4) << 6)
        q[j + 4] = (m[j] & 63) | ((m[j + 4] >> 4) << 6)
        q[j + 8] = (sc[j + 4] & 15) | ((m[j + 4] & 15) << 4)
    return q


def test_q4k_known_answer(oracle):
    """A hand-packed super-block whose weights follow from the format:
    sub-block j holds d*sc_j*q - dmin*m_j, runs of 64 = (low, high) nibbles."""
    sc = [1, 2, 3, 63, 17, 33, 48, 5]
    m = [0, 1, 62, 63, 16, 32, 7, 40]
    qs = (np.arange(128) * 7 % 256).astype(np.uint8)
    blk = np.concatenate([np.array([1.0, 0.5], np.float16).view(np.uint8), _pack_q4k_scales(sc, m),
                          qs])
    assert blk.size == 144
    want = np.empty(256, np.float64)
    for c in range(4):
        for l in range(32):
            want[64 * c + l] = 1.0 * sc[2 * c] * (qs[32 * c + l] & 15) - 0.5 * m[2 * c]
            want[64 * c + 32 + l] = 1.0 * sc[2 * c + 1] * (qs[32 * c + l] >> 4) - 0.5 * m[2 * c + 1]
    np.testing.assert_array_equal(oracle.q4k_dequant(blk), want.astype(np.float32))
    np.testing.assert_array_equal(wl.q4k_dequant_np(blk), want.astype(np.float32))


def test_q4k_restatements_agree(oracle, golden):
    """The C restatement and the independent numpy one, bit for bit, on the
    seeded QLoRA weight (110,592 blocks), and the committed digest."""
    blocks = wl.make_weight_q4k(4, 49152, 576)
    a = oracle.q4k_dequant(blocks)
    np.testing.assert_array_equal(a.view(np.uint32), wl.q4k_dequant_np(blocks).view(np.uint32))
    assert sha(a) == golden["q4k_seed4_49152x576_sha"]


@pytest.mark.skipif(not orc.ref_available(), reason="reference not built here")
def test_oracle_adam_bit_exact_with_reference_adam_update(oracle):
    """The oracle's mean + Adam against the reference's own adam_update
    (src/train.c:175-196, via oracle/_ref) on identical gradient sums, three
    updates with the moments carried: bit-equal."""
    d, V, r, k = 64, 3001, 5, 3
    A, B, gA, gB, n_pred = wl.make_adam_inputs(11, d, V, r, k)
    Ar, Br = orc.RefHarness().adam_steps(A, B, gA, gB, n_pred, 1e-3)
    Ao, Bo, state = A, B, None
    for i in range(k):
        Ao, Bo, state = oracle.adam(Ao, Bo, gA[i], gB[i], n_pred[i], 1e-3, state=state)
    assert state["step"] == k
    assert np.array_equal(Ao.view(np.uint32), Ar.view(np.uint32))
    assert np.array_equal(Bo.view(np.uint32), Br.view(np.uint32))
