"""The allocation-free loss entry point (lora_ce_token_loss_noalloc), for
callers that cannot allocate GPU memory at call time: a serving or
evaluation process whose device memory is reserved up front, or a runtime
that must never fail or stall in an allocation in the middle of a request.

Through the C ABI, its per-position losses match the oracle's (and the
training step's, lora_ce_step + lora_ce_get_token_loss) on the same inputs,
on calls in a row that share its static scratch arrays; uneven shapes (one
position, a partial last tile, d = 64, f32 hidden states) take the same
route; a target outside [0, V) gives NaN losses instead of a fault; and a
call leaves the device's free memory unchanged.  Collected last on
purpose, so that a run stopping at the first failure has run every other
test before it."""
import os

import numpy as np
import pytest

import lora_ce
import workload as wl

pytestmark = pytest.mark.gpu

LOSS_RTOL = 1e-4
NTHREADS = os.cpu_count() or 8


def _run(torch, dev, W, A, B, H, h_dtype, tgt, scale):
    V, d = W.shape
    T = tgt.shape[0]
    dW = torch.from_numpy(W.view(np.int16)).to(dev)
    dA = torch.from_numpy(np.ascontiguousarray(A)).to(dev)
    dB = torch.from_numpy(np.ascontiguousarray(B)).to(dev)
    if h_dtype == lora_ce.F32:
        dH = torch.from_numpy(np.ascontiguousarray(H, np.float32)).to(dev)
    else:
        dH = torch.from_numpy(np.ascontiguousarray(H).view(np.int16)).to(dev)
    dT = torch.from_numpy(np.ascontiguousarray(tgt, np.int32)).to(dev)
    dL = torch.full((T,), float("nan"), dtype=torch.float32, device=dev)
    lora_ce.token_loss_noalloc(dW.data_ptr(), V, d, dA.data_ptr(), dB.data_ptr(), scale,
                               dH.data_ptr(), h_dtype, T, dT.data_ptr(), dL.data_ptr(),
                               torch.cuda.current_stream(dev).cuda_stream)
    torch.cuda.synchronize(dev)
    return dL.cpu().numpy()


def _rel(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / np.linalg.norm(b))


def test_noalloc_loss_matches_oracle_and_step(oracle):
    import torch

    V, d, r = 49152, 576, 4
    W = wl.make_weight(31, V, d)
    dev = torch.device("cuda", 0)
    for call, T in enumerate((1000, 257)):  # two calls in a row
        h, tgt, A, B = wl.make_step_inputs(40 + call, T, V, d, r)
        m = lora_ce.LoraCE(lora_ce.default_config(d, V, r, T, scale=2.0, lr=1e-3))
        m.set_weight(W)
        m.set_adapter(A, B, 0)
        m.step(h, tgt)
        step_loss = m.token_loss(T)
        m.close()
        _, _, ref = oracle.accumulate(W, A, B, wl.oracle_hidden(h), tgt, 2.0, nthreads=NTHREADS)
        got = _run(torch, dev, W, A, B, h, lora_ce.BF16, tgt, 2.0)
        assert np.all(np.isfinite(got))
        assert _rel(got, ref) <= LOSS_RTOL, (call, _rel(got, ref))
        assert _rel(got, step_loss) <= LOSS_RTOL, (call, _rel(got, step_loss))


@pytest.mark.parametrize("V,d,T,dtype", [
    (1000, 64, 1, "f32"),     # one position; the last vocabulary tile partial
    (1000, 64, 129, "f32"),   # positions off the tile grid
    (4099, 128, 129, "bf16"),
    (49152, 576, 4096, "bf16"),  # the largest T it accepts
])
def test_noalloc_uneven_shapes_match_oracle(oracle, V, d, T, dtype):
    import torch

    dev = torch.device("cuda", 0)
    W = wl.make_weight(7 + V, V, d)
    h, tgt, A, B = wl.make_step_inputs(9 + T, T, V, d, 4)
    Hor = wl.oracle_hidden(h)
    H, hd = (Hor, lora_ce.F32) if dtype == "f32" else (h, lora_ce.BF16)
    _, _, ref = oracle.accumulate(W, A, B, Hor, tgt, 2.0, nthreads=NTHREADS)
    got = _run(torch, dev, W, A, B, H, hd, tgt, 2.0)
    assert np.all(np.isfinite(got))
    assert _rel(got, ref) <= LOSS_RTOL


def test_noalloc_target_out_of_range_gives_nan():
    """A target id equal to V is clamped inside the kernel and flagged, so
    the GPU reads nothing out of bounds; the call's losses come back NaN.
    The next call starts from a cleared flag."""
    import torch

    dev = torch.device("cuda", 0)
    V, d, T = 1000, 64, 50
    W = wl.make_weight(3, V, d)
    h, tgt, A, B = wl.make_step_inputs(4, T, V, d, 4)
    bad = tgt.copy()
    bad[17] = V
    got = _run(torch, dev, W, A, B, h, lora_ce.BF16, bad, 2.0)
    assert np.all(np.isnan(got))
    again = _run(torch, dev, W, A, B, h, lora_ce.BF16, tgt, 2.0)
    assert np.all(np.isfinite(again))


def test_noalloc_call_allocates_nothing():
    """After a first call (which resolves the static arrays' addresses), a
    call leaves the device's free memory exactly where it was."""
    import torch

    dev = torch.device("cuda", 0)
    V, d, T = 49152, 576, 2048
    W = wl.make_weight(5, V, d)
    h, tgt, A, B = wl.make_step_inputs(6, T, V, d, 4)
    dW = torch.from_numpy(W.view(np.int16)).to(dev)
    dA = torch.from_numpy(A).to(dev)
    dB = torch.from_numpy(B).to(dev)
    dH = torch.from_numpy(h.view(np.int16)).to(dev)
    dT = torch.from_numpy(tgt).to(dev)
    dL = torch.empty((T,), dtype=torch.float32, device=dev)
    st = torch.cuda.current_stream(dev).cuda_stream

    def call():
        lora_ce.token_loss_noalloc(dW.data_ptr(), V, d, dA.data_ptr(), dB.data_ptr(), 2.0,
                                   dH.data_ptr(), lora_ce.BF16, T, dT.data_ptr(),
                                   dL.data_ptr(), st)
        torch.cuda.synchronize(dev)

    call()
    free0, _ = torch.cuda.mem_get_info(dev)
    for _ in range(3):
        call()
    free1, _ = torch.cuda.mem_get_info(dev)
    assert free1 == free0, (free0, free1)


def test_noalloc_rejects_sizes_beyond_its_limits():
    with pytest.raises(lora_ce.LoraCEError, match="EINVAL"):
        lora_ce.token_loss_noalloc(16, 49152, 576, 16, 16, 2.0, 16, lora_ce.BF16, 4097, 16, 16)
    with pytest.raises(lora_ce.LoraCEError, match="EINVAL"):
        lora_ce.token_loss_noalloc(16, 49153, 576, 16, 16, 2.0, 16, lora_ce.BF16, 16, 16, 16)
    with pytest.raises(lora_ce.LoraCEError, match="aligned"):  # rejected before any work
        lora_ce.token_loss_noalloc(16, 1000, 64, 16, 16, 2.0, 8, lora_ce.BF16, 16, 16, 16)
