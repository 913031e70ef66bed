"""The trainer API of the reference's src/train.h on the GPU
(smollm2.c_b200/liblora_train.so): the drop-in for src/train.c.

CPU: the library exports the seven train.h functions and the two additions
of include/lora_train.h; the GGUF and packed-dataset fixtures are read by
the reference's own code (gguf_load, train_run); without a GPU train_create
fails and returns NULL.

GPU: train_step against the oracle (loss 1e-4 relative, adapter 1e-3
relative L2) with the reference's Kaiming init bit for bit; train_save /
train_load round trips and byte-identical LORA0001 files; train_run against
the reference's own train_run (same printed lines, same files); train_merge
against the reference's own train_merge (byte-identical GGUF).
"""
import os
import re

import numpy as np
import pytest

import oracle as orc
import workload as wl
import lora_ce
import studio_fixtures as sf

pytestmark = pytest.mark.skipif(not sf.available(), reason="trainer library or test env not built")

TRAIN_H_API = ["train_create", "train_free", "train_step", "train_save", "train_load", "train_run",
               "train_merge"]
REPO = sf.REPO


@pytest.fixture(scope="module")
def env():
    return sf.TrainerEnv()


def test_exports_match_headers(env):
    with open(os.path.join(REPO, "include", "lora_train.h")) as f:
        extra = re.findall(r"^int\s+(lora_train_\w+)\s*\(", f.read(), re.M)
    assert extra == ["lora_train_set_lm_head", "lora_train_set_lm_head_gguf",
                     "lora_train_set_body_gguf"]
    for name in TRAIN_H_API + extra:
        assert hasattr(env.lib, name), name


def test_gguf_fixture_reads_back_through_reference(env, tmp_path):
    d, V = 64, 100
    W = wl.make_weight(3, V, d)
    other = np.arange(10, dtype=np.float32)
    p = str(tmp_path / "m.gguf")
    sf.write_gguf(p, [("output_norm.weight", [10], sf.GGUF_F32, other.tobytes()),
                      ("token_embd.weight", [d, V], sf.GGUF_F16, W.tobytes())],
                  kv=[("general.architecture", "str", "llama")])
    rc, dims, dt, raw = env.gguf_tensor(p, "token_embd.weight", W.nbytes)
    assert rc == 0 and dims == (d, V) and dt == sf.GGUF_F16
    np.testing.assert_array_equal(raw.view(np.uint16).reshape(V, d), W)
    rc, dims, dt, raw = env.gguf_tensor(p, "output_norm.weight", other.nbytes)
    assert rc == 0 and dims == (10, 1) and dt == sf.GGUF_F32
    np.testing.assert_array_equal(raw.view(np.float32), other)


def _run_inputs(seed=5, d=128, V=3000, n_pos=63):
    W = wl.make_weight(seed, V, d)
    h, tgt, _, _ = wl.make_step_inputs(seed, n_pos, V, d, 4)
    H = np.ascontiguousarray(wl.oracle_hidden(h))
    rng = np.random.default_rng(seed)
    samples = [rng.integers(0, V, 64), rng.integers(0, V, 1), rng.integers(0, V, 40),
               rng.integers(0, V, 64), rng.integers(0, V, 30)]
    return W, H, samples


def _ref_train_run(W, H, samples, tmp, d, V, max_steps, checkpoint_every):
    ref = orc.RefHarness()
    import ctypes as C
    f = ref.lib.ref_train_run
    f.argtypes = [C.c_int] * 4 + [C.c_float] + [C.c_int] * 5 + [C.c_void_p, C.c_void_p, C.c_int,
                                                                C.c_char_p, C.c_char_p]
    packed = os.path.join(tmp, "data.bin")
    sf.write_packed(packed, samples)
    out = os.path.join(tmp, "ref_out")
    rc = f(d, V, 4, 8, 1e-3, 64, 42, 1, max_steps, checkpoint_every, W.ctypes.data, H.ctypes.data,
           H.shape[0], packed.encode(), out.encode())
    return rc, packed, out


STEP_RE = re.compile(r"^step=(\d+) epoch=(\d+) sample=(\d+) loss=([0-9.]+)$")
DONE_RE = re.compile(r"^train: done steps=(\d+) first_loss=([0-9.]+) last_loss=([0-9.]+) "
                     r"adapter=(\S+)$")


@pytest.mark.skipif(not orc.ref_available(), reason="reference not built here")
def test_packed_fixture_runs_through_reference_train_run(tmp_path, capfd):
    d, V = 128, 3000
    W, H, samples = _run_inputs(d=d, V=V)
    rc, _, out = _ref_train_run(W, H, samples, str(tmp_path), d, V, 3, 2)
    lines = capfd.readouterr().out.strip().splitlines()
    assert rc == 0
    steps = [STEP_RE.match(x).groups() for x in lines if x.startswith("step=")]
    # sample 1 has one token and is skipped; max_steps 3 stops after sample 3
    assert [(int(a), int(b), int(c)) for a, b, c, _ in steps] == [(1, 0, 0), (2, 0, 2), (3, 0, 3)]
    assert DONE_RE.match(lines[-1])
    assert sorted(os.listdir(out)) == ["lora_2.bin", "lora_final.bin"]


def test_train_create_fails_without_gpu(env):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    H = np.zeros((4, 64), np.float32)
    f = env.forward(H, 128)
    p = sf.params(seq_max=8)
    assert env.lib.train_create(f, p) is None
    env.env.env_forward_free(f)


# ------------------------------------------------------------------- GPU
def _read_adapter(path, d, V, r):
    ad = lora_ce.load_lora0001(path, d, V, r)
    return ad["A"], ad["B"], ad["step"], ad["scale"]


@pytest.mark.gpu
@pytest.mark.parametrize("r", [4, 128])  # 128: the wide-rank path (ranks above 64)
def test_train_step_matches_oracle(env, oracle, tmp_path, r):
    d, V, n = 576, 49152, 256
    W = wl.make_weight(31, V, d)
    h, tgt, _, _ = wl.make_step_inputs(31, n - 1, V, d, r)
    H = np.ascontiguousarray(wl.oracle_hidden(h))
    tokens = np.concatenate([[7], tgt]).astype(np.int32)
    f = env.forward(H, V)
    t = env.lib.train_create(f, sf.params(rank=r, alpha=2 * r, seq_max=n, lr=1e-3, seed=42))
    assert t
    assert env.lib.train_step(t, tokens.ctypes.data, n) == -1.0  # no lm_head yet
    assert env.lib.lora_train_set_lm_head(t, W.ctypes.data) == 0
    p0 = str(tmp_path / "init.bin")
    assert env.lib.train_save(t, p0.encode()) == 0
    A0, B0, s0, scale = _read_adapter(p0, d, V, r)
    np.testing.assert_array_equal(A0, oracle.kaiming_init(42, d, r))  # train_create's init
    assert not B0.any() and s0 == 0 and scale == 2.0
    state, A, B = None, A0, B0
    for k in range(3):
        loss = env.lib.train_step(t, tokens.ctypes.data, n)
        ref = oracle.train_step_tokens(W, A, B, H, tokens, n, 2.0, 1e-3, state=state)
        state, A, B = ref["state"], ref["A"], ref["B"]
        assert abs(loss - ref["loss"]) <= 1e-4 * ref["loss"], (k, loss, ref["loss"])
    p1 = str(tmp_path / "after.bin")
    assert env.lib.train_save(t, p1.encode()) == 0
    A1, B1, s1, _ = _read_adapter(p1, d, V, r)
    assert s1 == 3
    for a, b in ((A1, A), (B1, B)):
        assert np.linalg.norm(a - b) <= 1e-3 * np.linalg.norm(b)
    # one prefill and n-2 decodes per step, in order
    assert env.forward_calls(f) == (3, 3 * (n - 2), 0)
    # seq_max caps the positions; fewer than two tokens is -1
    assert env.lib.train_step(t, tokens.ctypes.data, 1) == -1.0
    bad = tokens.copy()
    bad[5] = V
    assert env.lib.train_step(t, bad.ctypes.data, n) == -1.0  # target out of range
    assert env.lib.train_step(t, tokens.ctypes.data, n) > 0  # still usable
    env.lib.train_free(t)
    env.env.env_forward_free(f)


@pytest.mark.gpu
def test_save_load_roundtrip_and_lora0001_bytes(env, tmp_path):
    d, V, r = 128, 3000, 8
    W = wl.make_weight(8, V, d)
    H = np.ascontiguousarray(wl.oracle_hidden(wl.make_step_inputs(8, 31, V, d, r)[0]))
    tokens = np.random.default_rng(8).integers(0, V, 32).astype(np.int32)
    f = env.forward(H, V)
    t = env.lib.train_create(f, sf.params(rank=r, alpha=16, seq_max=32, seed=9))
    assert env.lib.lora_train_set_lm_head(t, W.ctypes.data) == 0
    for _ in range(2):
        assert env.lib.train_step(t, tokens.ctypes.data, 32) > 0
    p = str(tmp_path / "a.bin")
    assert env.lib.train_save(t, p.encode()) == 0
    A, B, step, scale = _read_adapter(p, d, V, r)
    q = str(tmp_path / "b.bin")
    lora_ce.save_lora0001(q, A, B, scale, step)  # the reference's writer, byte for byte
    assert open(p, "rb").read() == open(q, "rb").read()
    assert os.path.getsize(p) == 28 + 4 * (d * r + r * V)
    # load into a fresh trainer (different seed, scale from the file)
    t2 = env.lib.train_create(f, sf.params(rank=r, alpha=4, seq_max=32, seed=1))
    assert env.lib.train_load(t2, p.encode()) == 0
    p2 = str(tmp_path / "c.bin")
    assert env.lib.train_save(t2, p2.encode()) == 0
    assert open(p2, "rb").read() == open(p, "rb").read()
    t3 = env.lib.train_create(f, sf.params(rank=4, seq_max=32))
    assert env.lib.train_load(t3, p.encode()) == -1  # rank mismatch
    assert env.lib.train_load(t3, str(tmp_path / "missing").encode()) == -1
    for x in (t, t2, t3):
        env.lib.train_free(x)
    env.env.env_forward_free(f)


@pytest.mark.gpu
@pytest.mark.skipif(not orc.ref_available(), reason="reference not built here")
def test_train_run_matches_reference_train_run(env, tmp_path, capfd):
    d, V = 128, 3000
    W, H, samples = _run_inputs(d=d, V=V)
    rc, packed, ref_out = _ref_train_run(W, H, samples, str(tmp_path), d, V, 4, 2)
    assert rc == 0
    ref_lines = capfd.readouterr().out.strip().splitlines()
    f = env.forward(H, V)
    p = sf.params(rank=4, alpha=8, seq_max=64, lr=1e-3, max_steps=4, checkpoint_every=2, seed=42)
    t = env.lib.train_create(f, p)
    assert env.lib.lora_train_set_lm_head(t, W.ctypes.data) == 0
    out = str(tmp_path / "gpu_out")
    assert env.lib.train_run(t, packed.encode(), p, out.encode()) == 0
    env.flush()
    lines = capfd.readouterr().out.strip().splitlines()
    env.lib.train_free(t)
    env.env.env_forward_free(f)
    assert len(lines) == len(ref_lines) == 5
    for a, b in zip(lines[:-1], ref_lines[:-1]):
        ga, gb = STEP_RE.match(a).groups(), STEP_RE.match(b).groups()
        assert ga[:3] == gb[:3]
        assert abs(float(ga[3]) - float(gb[3])) <= 1e-4 * float(gb[3]) + 1e-4
    da, db = DONE_RE.match(lines[-1]).groups(), DONE_RE.match(ref_lines[-1]).groups()
    assert da[0] == db[0]
    assert da[3] == os.path.join(out, "lora_final.bin") and db[3].endswith("lora_final.bin")
    assert sorted(os.listdir(out)) == sorted(os.listdir(ref_out)) == [
        "lora_2.bin", "lora_4.bin", "lora_final.bin"]
    for name in ("lora_2.bin", "lora_final.bin"):
        A, B, s, sc = _read_adapter(os.path.join(out, name), d, V, 4)
        Ar, Br, sr, scr = _read_adapter(os.path.join(ref_out, name), d, V, 4)
        assert (s, sc) == (sr, scr)
        for a, b in ((A, Ar), (B, Br)):
            assert np.linalg.norm(a - b) <= 1e-3 * np.linalg.norm(b)


@pytest.mark.gpu
@pytest.mark.skipif(not orc.ref_available(), reason="reference not built here")
def test_train_merge_matches_reference_train_merge(env, tmp_path, capfd):
    d, V, r = 576, 49152, 8
    W = wl.make_weight(41, V, d)
    W[0, :4] = [0x0001, 0x8001, 0x7c00, 0x0000]  # subnormals and inf take the quirky paths
    rng = np.random.default_rng(41)
    A = rng.standard_normal((d, r), dtype=np.float32) * np.float32(0.05)
    B = rng.standard_normal((r, V), dtype=np.float32) * np.float32(0.01)
    base = str(tmp_path / "base.gguf")
    norm = np.ones(d, np.float32)
    sf.write_gguf(base, [("output_norm.weight", [d], sf.GGUF_F32, norm.tobytes()),
                         ("token_embd.weight", [d, V], sf.GGUF_F16, W.tobytes())],
                  kv=[("general.architecture", "str", "llama"), ("general.alignment", "u32", 32)])
    adapter = str(tmp_path / "lora.bin")
    lora_ce.save_lora0001(adapter, A, B, 2.0, 20)
    ours, theirs = str(tmp_path / "ours.gguf"), str(tmp_path / "ref.gguf")
    assert env.lib.train_merge(base.encode(), adapter.encode(), ours.encode()) == 0
    env.flush()
    out_ours = capfd.readouterr().out
    import ctypes as C
    ref = orc.RefHarness()
    ref.lib.ref_train_merge.argtypes = [C.c_char_p] * 3
    assert ref.lib.ref_train_merge(base.encode(), adapter.encode(), theirs.encode()) == 0
    out_ref = capfd.readouterr().out
    assert open(ours, "rb").read() == open(theirs, "rb").read()
    assert out_ours.replace(ours, "OUT") == out_ref.replace(theirs, "OUT")
    # errors: missing adapter, bad magic, shape mismatch
    assert env.lib.train_merge(base.encode(), b"/nonexistent", ours.encode()) == -1
    bad = str(tmp_path / "bad.bin")
    open(bad, "wb").write(b"NOTLORA!" + bytes(40))
    assert env.lib.train_merge(base.encode(), bad.encode(), ours.encode()) == -1
    small = str(tmp_path / "small.bin")
    lora_ce.save_lora0001(small, A[:64], B, 2.0, 1)
    assert env.lib.train_merge(base.encode(), small.encode(), ours.encode()) == -1


@pytest.mark.gpu
def test_lm_head_from_gguf(env, tmp_path):
    d, V, r = 128, 3000, 4
    W = wl.make_weight(12, V, d)
    H = np.ascontiguousarray(wl.oracle_hidden(wl.make_step_inputs(12, 15, V, d, r)[0]))
    tokens = np.random.default_rng(12).integers(0, V, 16).astype(np.int32)
    p = str(tmp_path / "m.gguf")
    sf.write_gguf(p, [("token_embd.weight", [d, V], sf.GGUF_F16, W.tobytes())])
    g = env.env.env_gguf_open(p.encode())
    assert g
    f = env.forward(H, V)
    t1 = env.lib.train_create(f, sf.params(rank=r, seq_max=16))
    t2 = env.lib.train_create(f, sf.params(rank=r, seq_max=16))
    assert env.lib.lora_train_set_lm_head_gguf(t1, g) == 0
    assert env.lib.lora_train_set_lm_head(t2, W.ctypes.data) == 0
    assert env.lib.train_step(t1, tokens.ctypes.data, 16) == env.lib.train_step(
        t2, tokens.ctypes.data, 16)
    p_small = str(tmp_path / "small.gguf")
    sf.write_gguf(p_small, [("token_embd.weight", [d, 100], sf.GGUF_F16, W[:100].tobytes())])
    g2 = env.env.env_gguf_open(p_small.encode())
    assert env.lib.lora_train_set_lm_head_gguf(t1, g2) == -1  # wrong vocab
    for x in (t1, t2):
        env.lib.train_free(x)
    env.env.env_gguf_close(g)
    env.env.env_gguf_close(g2)
    env.env.env_forward_free(f)


@pytest.mark.gpu
def test_qlora_lm_head_from_gguf(env, oracle, tmp_path):
    """A Q4_K token_embd.weight in the model file (QLoRA): dequantised on
    the GPU, the step matches the oracle on the dequantised f16 weight."""
    d, V, r, n = 576, 4096, 8, 64
    blocks = wl.make_weight_q4k(13, V, d)
    W16 = oracle.q4k_dequant(blocks).astype(np.float16).view(np.uint16).reshape(V, d)
    h, tgt, _, _ = wl.make_step_inputs(13, n - 1, V, d, r)
    H = np.ascontiguousarray(wl.oracle_hidden(h))
    tokens = np.concatenate([[1], tgt]).astype(np.int32)
    p = str(tmp_path / "q.gguf")
    sf.write_gguf(p, [("token_embd.weight", [d, V], 12, blocks.tobytes())])
    g = env.env.env_gguf_open(p.encode())
    assert g
    f = env.forward(H, V)
    t = env.lib.train_create(f, sf.params(rank=r, alpha=16, seq_max=n, seed=42))
    assert env.lib.lora_train_set_lm_head_gguf(t, g) == 0
    loss = env.lib.train_step(t, tokens.ctypes.data, n)
    A0 = oracle.kaiming_init(42, d, r)
    ref = oracle.train_step_tokens(W16, A0, np.zeros((r, V), np.float32), H, tokens, n, 2.0, 1e-4)
    assert abs(loss - ref["loss"]) <= 1e-4 * ref["loss"]
    env.lib.train_free(t)
    env.env.env_gguf_close(g)
    env.env.env_forward_free(f)


@pytest.mark.gpu
def test_train_run_packs_samples_when_asked(env, oracle, tmp_path, capfd):
    """LORA_TRAIN_PACK=1 with batch 3: train_run makes one step per three
    usable samples (the last step takes what is left), each step one Adam
    update over all their predicted positions, checked against the oracle
    on the concatenated positions.  Without it, one sample per step."""
    d, V = 128, 3000
    W, H, samples = _run_inputs(d=d, V=V)  # lengths 64, 1, 40, 64, 30
    packed = str(tmp_path / "data.bin")
    sf.write_packed(packed, samples)
    f = env.forward(H, V)
    p = sf.params(rank=4, alpha=8, seq_max=64, lr=1e-3, batch=3, seed=42)
    os.environ["LORA_TRAIN_PACK"] = "1"
    try:
        t = env.lib.train_create(f, p)
    finally:
        os.environ.pop("LORA_TRAIN_PACK", None)
    assert env.lib.lora_train_set_lm_head(t, W.ctypes.data) == 0
    out = str(tmp_path / "out")
    assert env.lib.train_run(t, packed.encode(), p, out.encode()) == 0
    env.flush()
    lines = capfd.readouterr().out.strip().splitlines()
    steps = [STEP_RE.match(x).groups() for x in lines if x.startswith("step=")]
    assert [(int(a), int(c)) for a, _, c, _ in steps] == [(1, 0), (2, 4)]
    # the oracle on the same positions: rows 0..n-2 of H for each sample
    groups = [[0, 2, 3], [4]]
    state, A, B = None, oracle.kaiming_init(42, d, 4), np.zeros((4, V), np.float32)
    for (_, _, _, loss), grp in zip(steps, groups):
        Hs = np.concatenate([H[:len(samples[i]) - 1] for i in grp])
        tg = np.concatenate([np.asarray(samples[i][1:], np.int32) for i in grp])
        ref = oracle.step(W, A, B, Hs, tg, 2.0, 1e-3, state=state)
        state, A, B = ref["state"], ref["A"], ref["B"]
        assert abs(float(loss) - ref["loss"]) <= 1e-4 * ref["loss"] + 1e-4
    A1, B1, s1, _ = _read_adapter(os.path.join(out, "lora_final.bin"), d, V, 4)
    assert s1 == 2
    for a, b in ((A1, A), (B1, B)):
        assert np.linalg.norm(a - b) <= 1e-3 * np.linalg.norm(b)
    env.lib.train_free(t)
    env.env.env_forward_free(f)


# ------------------------------------------------------- failure paths (GPU)
@pytest.mark.gpu
@pytest.mark.skipif(not orc.ref_available(), reason="reference not built here")
def test_train_run_emergency_save_matches_reference(env, tmp_path, capfd):
    """train_run's watchdog (src/train.c:355-369) with simulate_mem_kb below
    the emergency threshold: after the first step both trainers write
    emergency_1.bin, print the same lines and return 0 without a final
    save."""
    import ctypes as C
    d, V = 128, 3000
    W, H, samples = _run_inputs(d=d, V=V)
    ref = orc.RefHarness()
    f = ref.lib.ref_train_run_mem
    f.argtypes = [C.c_int] * 4 + [C.c_float] + [C.c_int] * 5 + [C.c_void_p, C.c_void_p, C.c_int,
                                                                C.c_char_p, C.c_char_p, C.c_long]
    packed = str(tmp_path / "data.bin")
    sf.write_packed(packed, samples)
    ref_out = str(tmp_path / "ref_out")
    rc = f(d, V, 4, 8, 1e-3, 64, 42, 1, 4, 2, W.ctypes.data, H.ctypes.data, H.shape[0],
           packed.encode(), ref_out.encode(), 1024)
    assert rc == 0
    ref_cap = capfd.readouterr()
    fw = env.forward(H, V)
    p = sf.params(rank=4, alpha=8, seq_max=64, lr=1e-3, max_steps=4, checkpoint_every=2, seed=42,
                  simulate_mem_kb=1024)
    t = env.lib.train_create(fw, p)
    assert env.lib.lora_train_set_lm_head(t, W.ctypes.data) == 0
    out = str(tmp_path / "gpu_out")
    assert env.lib.train_run(t, packed.encode(), p, out.encode()) == 0
    env.flush()
    cap = capfd.readouterr()
    env.lib.train_free(t)
    env.env.env_forward_free(fw)
    lines, ref_lines = cap.out.strip().splitlines(), ref_cap.out.strip().splitlines()
    assert len(lines) == len(ref_lines) == 1
    a, b = STEP_RE.match(lines[0]).groups(), STEP_RE.match(ref_lines[0]).groups()
    assert a[:3] == b[:3] and abs(float(a[3]) - float(b[3])) <= 1e-4 * float(b[3]) + 1e-4
    emerg = [x for x in cap.err.splitlines() if x.startswith("train: emergency save")]
    ref_emerg = [x for x in ref_cap.err.splitlines() if x.startswith("train: emergency save")]
    assert emerg == ref_emerg and len(emerg) == 1
    assert sorted(os.listdir(out)) == sorted(os.listdir(ref_out)) == ["emergency_1.bin"]
    A, B, s, sc = _read_adapter(os.path.join(out, "emergency_1.bin"), d, V, 4)
    Ar, Br, sr, scr = _read_adapter(os.path.join(ref_out, "emergency_1.bin"), d, V, 4)
    assert (s, sc) == (sr, scr) == (1, 2.0)
    for x, y in ((A, Ar), (B, Br)):
        assert np.linalg.norm(x - y) <= 1e-3 * np.linalg.norm(y)


@pytest.mark.gpu
def test_train_create_host_allocation_failure(tmp_path):
    """A host allocation that fails inside train_create (the buffer of
    gathered hidden states, made to fail by a preloaded malloc fake in a
    child process) makes it return NULL, as the reference's does, after
    releasing the GPU handle it had created; a second train_create in the
    same process then succeeds."""
    import subprocess
    import sys
    so = str(tmp_path / "libfail_alloc.so")
    subprocess.run(["gcc", "-O2", "-fPIC", "-shared", "-o", so,
                    os.path.join(REPO, "tests", "fault", "fail_alloc.c")], check=True)
    d, seq_max = 128, 1237
    size = (seq_max - 1) * d * 4  # train_create's t->H: max_pred x dim floats
    script = f"""
import sys, numpy as np
sys.path[:0] = {[REPO, os.path.join(REPO, 'tests'), os.path.join(REPO, 'smollm2.c_b200'),
                 os.path.join(REPO, 'oracle')]!r}
import studio_fixtures as sf
env = sf.TrainerEnv()
H = np.zeros((4, {d}), np.float32)
f = env.forward(H, 1000)
p = sf.params(seq_max={seq_max})
t = env.lib.train_create(f, p)
print("first", t is None)
import os
os.environ["FAIL_ALLOC_SIZE"] = "0"
t = env.lib.train_create(f, p)
print("second", t is not None)
env.lib.train_free(t)
env.env.env_forward_free(f)
"""
    envv = dict(os.environ, LD_PRELOAD=so, FAIL_ALLOC_SIZE=str(size))
    r = subprocess.run([sys.executable, "-c", script], env=envv, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "first True" in r.stdout and "second True" in r.stdout


@pytest.mark.gpu
def test_device_allocation_failure_is_enomem(oracle):
    """A handle whose buffers cannot be allocated on the device (a vocabulary
    whose weight alone would need 1.2 TB) is refused with LORA_CE_ENOMEM, the
    failed allocation leaves no error behind, and the next handle on the same
    device steps correctly."""
    with pytest.raises(lora_ce.LoraCEError, match="ENOMEM"):
        lora_ce.LoraCE(lora_ce.default_config(576, 1 << 30, 4, 16))
    with pytest.raises(lora_ce.LoraCEError, match="EINVAL"):
        lora_ce.LoraCE(lora_ce.default_config(576, 49152, 4, (1 << 24) + 1))
    V, d, T = 1000, 64, 40
    W = wl.make_weight(2, V, d)
    h, tgt, A, B = wl.make_step_inputs(2, T, V, d, 4)
    m = lora_ce.LoraCE(lora_ce.default_config(d, V, 4, T, scale=2.0, lr=1e-3))
    m.set_weight(W)
    m.set_adapter(A, B, 0)
    loss = m.step(h, tgt)
    m.close()
    ref = oracle.step(W, A, B, wl.oracle_hidden(h), tgt, 2.0, 1e-3)
    assert abs(loss - ref["loss"]) <= 1e-4 * ref["loss"]
