"""The allocation-free loss entry point (lora_ce_token_loss_noalloc) for
callers that cannot allocate GPU memory at call time: through the C ABI,
its per-position losses match those of the training step
(lora_ce_step + lora_ce_get_token_loss) on the same inputs, on two calls in
a row that share its static scratch arrays.  Collected last on purpose."""
import numpy as np
import pytest

import lora_ce
import workload as wl

pytestmark = pytest.mark.gpu

LOSS_RTOL = 1e-4


def test_noalloc_loss_matches_step_loss():
    import torch

    V, d, r = 49152, 576, 4
    W = wl.make_weight(31, V, d)
    dev = torch.device("cuda", 0)
    dW = torch.from_numpy(W.view(np.int16)).to(dev)
    for call, T in enumerate((1000, 257)):  # two calls in a row
        h, tgt, A, B = wl.make_step_inputs(40 + call, T, V, d, r)
        m = lora_ce.LoraCE(lora_ce.default_config(d, V, r, T, scale=2.0, lr=1e-3))
        m.set_weight(W)
        m.set_adapter(A, B, 0)
        m.step(h, tgt)
        ref = m.token_loss(T)
        m.close()
        dA = torch.from_numpy(A).to(dev)
        dB = torch.from_numpy(B).to(dev)
        dH = torch.from_numpy(h.view(np.int16)).to(dev)
        dT = torch.from_numpy(tgt).to(dev)
        dL = torch.full((T,), float("nan"), dtype=torch.float32, device=dev)
        lora_ce.token_loss_noalloc(dW.data_ptr(), V, d, dA.data_ptr(), dB.data_ptr(), 2.0,
                                   dH.data_ptr(), lora_ce.BF16, T, dT.data_ptr(), dL.data_ptr(),
                                   torch.cuda.current_stream(dev).cuda_stream)
        torch.cuda.synchronize(dev)
        got = dL.cpu().numpy()
        assert np.all(np.isfinite(got))
        err = np.linalg.norm(got - ref) / np.linalg.norm(ref)
        assert err <= LOSS_RTOL, (call, err)


def test_noalloc_rejects_sizes_beyond_its_limits():
    with pytest.raises(lora_ce.LoraCEError, match="EINVAL"):
        lora_ce.token_loss_noalloc(1, 49152, 576, 1, 1, 2.0, 1, lora_ce.BF16, 4097, 1, 1)
    with pytest.raises(lora_ce.LoraCEError, match="EINVAL"):
        lora_ce.token_loss_noalloc(1, 49153, 576, 1, 1, 2.0, 1, lora_ce.BF16, 16, 1, 1)
