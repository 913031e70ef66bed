"""The body forward on the GPU (include/lora_body.h) against the reference's
own body forward (src/forward.c through oracle/_ref/libref_body.so, driven
position by position as train_step drives it).

Both quantise weights and activations to int8 with the same rules, sum in
int32 and add the float parts in the same order, so hidden states agree to
the last bit until e^x differs: the GPU takes it from a double-precision exp
rounded to f32, which differs from glibc's expf in the last bit for about
0.008% of arguments.  Such a difference can move one int8 activation of the
next matmul by one step; from the position where that first happens, the
attention carries it to every later position of the sequence, where the
hidden states then differ by about 2e-3 relative (measured at 30 layers;
the int8 step of one activation is 1/127 of its row's largest value).
Tolerances: two layers, bit-exact rows; 30 layers, every position within
1e-2 relative L2 and the first positions bit-exact."""
import os

import numpy as np
import pytest

import oracle as orc
import studio_fixtures as sf
import lora_ce

pytestmark = pytest.mark.skipif(not orc.ref_body_available(),
                                reason="reference body harness not built")

ROW_RTOL = 1e-2


def body_from(embd, out_norm, layers, max_seq, max_tokens):
    b = lora_ce.LoraBody(len(layers), max_seq=max_seq, max_tokens=max_tokens)
    b.set_embedding(embd, out_norm)
    for L, t in enumerate(layers):
        b.set_layer(L, t)
    return b


def row_errors(H, R):
    return np.linalg.norm(H - R, axis=1) / np.linalg.norm(R, axis=1)


def test_reference_body_harness_runs(tmp_path):
    """The harness itself (CPU): hidden rows of one sequence, finite, one
    per position, and the first row independent of what follows."""
    model = str(tmp_path / "m.gguf")
    sf.write_smollm_gguf(model, seed=3, n_layers=1, norm_spread=0.2)
    rb = orc.RefBody(model, 16)
    tok = np.random.default_rng(1).integers(0, 49152, 9)
    H, secs = rb.hidden(tok, 576)
    H2, _ = rb.hidden(tok[:3], 576)
    rb.close()
    assert H.shape == (9, 576) and np.all(np.isfinite(H)) and secs > 0
    np.testing.assert_array_equal(H[:3], H2)


@pytest.mark.gpu
def test_body_matches_reference_packed_sequences(tmp_path):
    """Two layers, three sequences packed back to back (64, 1 and 40
    positions: positions restart at 0 in each), against the reference run
    sequence by sequence."""
    model = str(tmp_path / "m.gguf")
    embd, out_norm, layers = sf.write_smollm_gguf(model, seed=7, n_layers=2, norm_spread=0.2,
                                                  return_tensors=True)
    rng = np.random.default_rng(11)
    seqs = [rng.integers(0, 49152, n) for n in (64, 1, 40)]
    rb = orc.RefBody(model, 64)
    ref = np.concatenate([rb.hidden(s, 576)[0] for s in seqs])
    rb.close()
    b = body_from(embd, out_norm, layers, 64, 256)
    offsets = np.cumsum([0] + [len(s) for s in seqs])
    H = b.hidden(np.concatenate(seqs), offsets)
    b.close()
    err = row_errors(H, ref)
    print(f"per-position rel L2: median {np.median(err):.2e}, max {err.max():.2e}, "
          f"exact rows {int(np.sum(err == 0))}/{len(err)}")
    assert err.max() <= ROW_RTOL and np.median(err) == 0.0


@pytest.mark.gpu
def test_body_sliding_window_and_device_output(tmp_path):
    """A sliding window on layer 1 (the reference's SWA type via its
    attention registry is not reachable from the model file, so the
    reference side is the dense model on each window's suffix: with one
    windowed layer and the window covering the whole sequence the result is
    the dense one), and the device entry point writing bf16 rows into a
    device buffer: the bf16 rounding of the f32 rows."""
    import torch
    model = str(tmp_path / "m.gguf")
    embd, out_norm, layers = sf.write_smollm_gguf(model, seed=9, n_layers=2, norm_spread=0.2,
                                                  return_tensors=True)
    tok = np.random.default_rng(5).integers(0, 49152, 48).astype(np.int32)
    b = body_from(embd, out_norm, layers, 64, 64)
    dense = b.hidden(tok, [0, 48])
    b.set_window(1, 64)  # covers every position: same as dense
    same = b.hidden(tok, [0, 48])
    np.testing.assert_array_equal(dense, same)
    b.set_window(1, 4)
    win = b.hidden(tok, [0, 48])
    assert np.array_equal(win[:4], dense[:4]) and not np.allclose(win[4:], dense[4:])
    b.set_window(1, 0)
    dev = torch.device("cuda", 0)
    dT = torch.from_numpy(tok).to(dev)
    dH = torch.empty((48, 576), dtype=torch.bfloat16, device=dev)
    b.hidden_device(dT.data_ptr(), [0, 48], dH.data_ptr(), lora_ce.BF16)
    b.sync()
    got = dH.float().cpu().numpy()
    want = torch.from_numpy(dense).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(got, want)
    with pytest.raises(lora_ce.LoraCEError, match="EINVAL"):
        b.hidden(np.array([0, 49152], np.int32), [0, 2])
    b.close()


@pytest.mark.gpu
def test_body_full_model_one_sequence(tmp_path):
    """The 30-layer SmolLM2-135M shape on one packed sequence of 256
    positions (the CPU-body training workload's sample), against the
    reference."""
    model = str(tmp_path / "m30.gguf")
    embd, out_norm, layers = sf.write_smollm_gguf(model, seed=21, n_layers=30, norm_spread=0.2,
                                                  return_tensors=True)
    import workload as wl
    tok = wl.zipf_targets(np.random.default_rng(2), 256, 49152).astype(np.int32)
    rb = orc.RefBody(model, 256)
    ref, secs = rb.hidden(tok, 576)
    rb.close()
    b = body_from(embd, out_norm, layers, 256, 256)
    H = b.hidden(tok, [0, 256])
    b.close()
    err = row_errors(H, ref)
    print(f"30 layers: per-position rel L2 median {np.median(err):.2e}, max {err.max():.2e}, "
          f"exact rows {int(np.sum(err == 0))}/256; reference {secs:.1f} s")
    print("by position (every 16th):", " ".join(f"{e:.1e}" for e in err[::16]))
    assert err.max() <= ROW_RTOL
    assert np.all(err[:8] == 0.0)  # before any e^x difference has had an effect


@pytest.mark.gpu
def test_body_train_step_is_body_then_step(tmp_path):
    """lora_body_train_step (body into its own buffer, then the LoRA step)
    gives the loss and adapter of the two calls made separately: the body's
    hidden rows through lora_ce_step, packed samples included."""
    model = str(tmp_path / "m.gguf")
    embd, out_norm, layers = sf.write_smollm_gguf(model, seed=4, n_layers=2, norm_spread=0.2,
                                                  return_tensors=True)
    import workload as wl
    rng = np.random.default_rng(6)
    seqs = [wl.zipf_targets(rng, n, 49152).astype(np.int32) for n in (40, 2, 64)]
    tok = np.concatenate([s[:-1] for s in seqs])
    tgt = np.concatenate([s[1:] for s in seqs])
    off = np.cumsum([0] + [len(s) - 1 for s in seqs])
    T = int(off[-1])
    _, _, A, B = wl.make_step_inputs(6, 8, 49152, 576, 4)
    b = body_from(embd, out_norm, layers, 64, 128)
    out = []
    for fused in (True, False):
        ce = lora_ce.LoraCE(lora_ce.default_config(576, 49152, 4, T, scale=2.0, lr=1e-3))
        ce.set_weight(embd)
        ce.set_adapter(A, B, 0)
        if fused:
            loss = b.train_step(ce, tok, off, tgt)
        else:
            loss = ce.step(b.hidden(tok, off), tgt)
        out.append((loss, ce.get_adapter()[1], ce.get_grads()[1]))
        ce.close()
    b.close()
    assert out[0][0] == out[1][0]
    np.testing.assert_array_equal(out[0][1], out[1][1])
    np.testing.assert_array_equal(out[0][2], out[1][2])
