"""The sharded MLP and head with the output exchange over peer memory, on
two GPUs (one process each, NCCL only for set-up): bit-identical to the
unsharded single-GPU calls.  Skipped with fewer than two GPUs."""
import os
import pathlib
import socket
import tempfile

import numpy as np
import pytest
import torch

from qmr import synth

pytestmark = pytest.mark.gpu

H, F, V, B = 5120, 17408, 152064 // 8, 3  # the config-2 MLP; a vocabulary slice for the head


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _mats():
    return (synth.affine_matrix(F, H, 4, 64, seed=71), synth.affine_matrix(F, H, 4, 64, seed=72),
            synth.affine_matrix(H, F, 4, 64, seed=73), synth.affine_matrix(V, H, 4, 64, seed=74))


def _rows(m, r0, r1):
    """Rows [r0, r1) of a synthetic packed matrix (weights and metadata)."""
    return {k: np.ascontiguousarray(m[k][r0:r1]) for k in ("weight", "scales", "biases")}


def _rank_main(rank, world, port, outdir, steps):
    import datetime

    import torch.distributed as dist

    import qmr
    from qmr import parallel
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    qmr.ops.init(rank)
    mlp = hd = None
    try:
        gate, up, down, head = _mats()
        f0, f1 = parallel.shard_range(F, world, rank)
        h0, h1 = parallel.shard_range(H, world, rank)
        v0, v1 = parallel.shard_range(V, world, rank)
        dm = lambda m, r0, r1, c: synth.to_device(_rows(m, r0, r1), r1 - r0, c, 4, 64, dev)  # noqa: E731
        mlp = parallel.ShardedMLP(dm(gate, f0, f1, H), dm(up, f0, f1, H), dm(down, h0, h1, F), H, F, qmr.ops,
                                  exchange="p2p")
        hd = parallel.ShardedHead(dm(head, v0, v1, H), V, v0, qmr.ops, exchange="p2p")
        x = torch.from_numpy(synth.activations(B, H, seed=75).ravel()).to(dev)
        ys, ids = [], []
        for _ in range(steps):  # both output buffers, more than one epoch
            y = mlp(x, B).clone()
            idx, _ = hd(y, B)
            ys.append(y.cpu().numpy())
            ids.append(idx.cpu().numpy())
        torch.cuda.synchronize()
        err = qmr.ops.device_error()
        np.savez(pathlib.Path(outdir) / f"rank{rank}.npz", y=np.stack(ys), idx=np.stack(ids), err=err)
    finally:
        torch.cuda.synchronize()
        if mlp is not None:
            mlp.close()
        if hd is not None:
            hd.close()
        dist.destroy_process_group()


def test_p2p_sharded_mlp_and_head_equal_the_unsharded_calls():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    import qmr
    world, steps = 2, 3
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_rank_main, args=(world, _free_port(), d, steps), nprocs=world, start_method="spawn",
                           join=True)
        res = [np.load(pathlib.Path(d) / f"rank{r}.npz") for r in range(world)]
    gate, up, down, head = _mats()
    dev = torch.device("cuda", 0)
    qmr.ops.init(0)
    tm = lambda m, r, c: synth.to_device(m, r, c, 4, 64, dev)  # noqa: E731
    x = torch.from_numpy(synth.activations(B, H, seed=75).ravel()).to(dev)
    act = torch.empty(B * F, dtype=torch.float32, device=dev)
    qmr.gateup_swiglu(tm(gate, F, H), tm(up, F, H), x, act, B)
    y = torch.empty(B * H, dtype=torch.float32, device=dev)
    qmr.matmul_affine(tm(down, H, F), act, y, B)
    lg = torch.empty(B * V, dtype=torch.float32, device=dev)
    idx = torch.empty(B, dtype=torch.int32, device=dev)
    qmr.head_argmax(tm(head, V, H), y, lg, idx, B)
    torch.cuda.synchronize()
    want_y, want_idx = y.cpu().numpy(), idx.cpu().numpy()
    for r in range(world):
        assert int(res[r]["err"]) == 0
        for s in range(steps):
            assert np.array_equal(res[r]["y"][s].view(np.uint32), want_y.view(np.uint32)), (r, s)
            assert np.array_equal(res[r]["idx"][s], want_idx), (r, s)
