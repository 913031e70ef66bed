"""Data-parallel token sharding.

CPU (gloo, world size 2): every rank accumulates the oracle gradient sums on
its own positions, the packed buffer [dA | dB | loss sum | n_pred] is summed
with one all-reduce (the library's one exchange step), and the mean + Adam
then reproduce the single-process step over all positions.

GPU (two B200s, NCCL through the library's own communicator): the same
comparison for the CUDA path.  Skipped when fewer than two GPUs are visible.
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

import oracle as orc
import workload as wl

V, D, R = 3000, 128, 4
T_TOTAL = 96
SCALE, LR = 2.0, 1e-3


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def inputs(r=R):
    W = wl.make_weight(61, V, D)
    h, tgt, A, B = wl.make_step_inputs(61, T_TOTAL, V, D, r)
    return W, h, tgt, A, B


def shard(rank, world, n):
    return slice(n * rank // world, n * (rank + 1) // world)


def _gloo_rank(rank, world, port, out):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    o = orc.Oracle()
    W, h, tgt, A, B = inputs()
    sl = shard(rank, world, T_TOTAL)
    H = wl.oracle_hidden(h)[sl]
    gA, gB, loss = o.accumulate(W, A, B, H, tgt[sl], SCALE)
    G = np.concatenate([gA.ravel(), gB.ravel(), [loss.astype(np.float64).sum(), len(loss)]])
    Gt = torch.from_numpy(G.astype(np.float64))
    dist.all_reduce(Gt)
    G = Gt.numpy()
    nA = D * R
    gA = G[:nA].astype(np.float32).reshape(D, R)
    gB = G[nA:nA + R * V].astype(np.float32).reshape(R, V)
    n_pred = int(G[-1])
    state = dict(step=0, mA=np.zeros_like(gA), vA=np.zeros_like(gA), mB=np.zeros_like(gB),
                 vB=np.zeros_like(gB))
    A1, B1 = A.copy(), B.copy()
    import ctypes as C
    stp = C.c_int(0)
    o.lib.oracle_adam(D, V, R, LR, 0.0, 0.0, n_pred, C.byref(stp), A1, B1, gA, gB, state["mA"],
                      state["vA"], state["mB"], state["vB"])
    out[rank] = dict(A=A1, B=B1, gA=gA, gB=gB, loss=G[-2] / n_pred, n=n_pred)
    dist.destroy_process_group()


def test_gloo_two_ranks_reproduce_single_process_step(oracle):
    world = 2
    port = free_port()
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_gloo_rank, args=(world, port, out), nprocs=world, join=True)
    W, h, tgt, A, B = inputs()
    ref = oracle.step(W, A, B, wl.oracle_hidden(h), tgt, SCALE, LR)
    for rank in range(world):
        r = out[rank]
        assert r["n"] == T_TOTAL
        assert abs(r["loss"] - ref["loss"]) <= 1e-6 * ref["loss"]
        for k in ("gA", "gB", "A", "B"):
            assert np.linalg.norm(r[k] - ref[k]) <= 1e-5 * np.linalg.norm(ref[k]), k
    # both ranks applied the identical update
    for k in ("A", "B"):
        np.testing.assert_array_equal(out[0][k], out[1][k])


def _gpu_rank(rank, world, uid_path, out, r):
    import time
    import lora_ce
    W, h, tgt, A, B = inputs(r)
    m = lora_ce.LoraCE(lora_ce.default_config(D, V, r, T_TOTAL, scale=SCALE, lr=LR,
                                              device=rank))
    m.set_weight(W)
    m.set_adapter(A, B, 0)
    if rank == 0:
        uid = lora_ce.LoraCE.nccl_unique_id()
        with open(uid_path + ".tmp", "wb") as f:
            f.write(uid)
        os.rename(uid_path + ".tmp", uid_path)
    else:
        for _ in range(600):
            if os.path.exists(uid_path):
                break
            time.sleep(0.05)
        with open(uid_path, "rb") as f:
            uid = f.read()
    m.comm_init(world, rank, uid)
    sl = shard(rank, world, T_TOTAL)
    loss = m.step(np.ascontiguousarray(h[sl]), np.ascontiguousarray(tgt[sl]))
    gA, gB, lsum, n = m.get_grads()
    A1, B1, _ = m.get_adapter()
    m.close()
    out[rank] = dict(loss=loss, gA=gA, gB=gB, A=A1, B=B1, n=n)


@pytest.mark.gpu
# rank 64: the tensor-core rank-sum passes; rank 100: the wide-rank path (kernel rank 128)
@pytest.mark.parametrize("r", [4, 64, 100])
def test_two_gpus_match_oracle(oracle, tmp_path, r):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    world = 2
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_gpu_rank, args=(world, str(tmp_path / "uid"), out, r), nprocs=world, join=True)
    W, h, tgt, A, B = inputs(r)
    ref = oracle.step(W, A, B, wl.oracle_hidden(h), tgt, SCALE, LR)
    for rank in range(world):
        r = out[rank]
        assert r["n"] == T_TOTAL
        assert abs(r["loss"] - ref["loss"]) <= 1e-4 * ref["loss"]
        for k in ("gA", "gB", "A", "B"):
            assert np.linalg.norm(r[k] - ref[k]) <= 1e-3 * np.linalg.norm(ref[k]), k
    for k in ("A", "B"):
        np.testing.assert_array_equal(out[0][k], out[1][k])

