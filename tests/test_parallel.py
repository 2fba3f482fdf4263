"""Host logic of the sharded MLP and head (qmr.parallel) on world-size-2 gloo
ranks on the CPU, with the FP64 oracle standing in for the kernels."""
import os
import pathlib
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from qmr import parallel, synth

from _cpu_ops import CpuMatrix, CpuOps, total_order_key

H, F, V, B = 256, 512, 1024, 3


def _matrix(rows, cols, seed):
    d = synth.affine_matrix(rows, cols, 4, 64, seed=seed)
    return CpuMatrix(d["weight"], d["scales"], d["biases"], rows, cols, 4, 64)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, outdir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        gate, up, down, head = _matrix(F, H, 11), _matrix(F, H, 12), _matrix(H, F, 13), _matrix(V, H, 14)
        f0, f1 = parallel.shard_range(F, world, rank)
        h0, h1 = parallel.shard_range(H, world, rank)
        v0, v1 = parallel.shard_range(V, world, rank)
        mlp = parallel.ShardedMLP(gate.shard(f0, f1), up.shard(f0, f1), down.shard(h0, h1), H, F, CpuOps)
        x = torch.from_numpy(synth.activations(B, H, seed=15).ravel())
        y = mlp(x, B)
        hd = parallel.ShardedHead(head.shard(v0, v1), V, v0, CpuOps)
        idx, keys = hd(y, B)
        np.savez(pathlib.Path(outdir) / f"rank{rank}.npz", y=y.numpy(), idx=idx.numpy(), keys=keys.numpy())
    finally:
        dist.destroy_process_group()


def test_sharded_mlp_and_head_match_the_unsharded_computation():
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_rank_main, args=(world, _free_port(), d), nprocs=world, start_method="spawn", join=True)
        res = [np.load(pathlib.Path(d) / f"rank{r}.npz") for r in range(world)]
    gate, up, down, head = _matrix(F, H, 11), _matrix(F, H, 12), _matrix(H, F, 13), _matrix(V, H, 14)
    x = torch.from_numpy(synth.activations(B, H, seed=15).ravel())
    act = torch.empty(B * F, dtype=torch.float32)
    CpuOps.gateup_swiglu(gate, up, x, act, B)
    y = torch.empty(B * H, dtype=torch.float32)
    CpuOps.matmul_affine(down, act, y, B)
    lg = torch.empty(B * V, dtype=torch.float32)
    idx = torch.empty(B, dtype=torch.int32)
    CpuOps.head_argmax(head, y, lg, idx, B)
    for r in res:
        # Row sharding keeps every row whole: the same values, bit for bit.
        assert np.array_equal(r["y"].view(np.uint32), y.numpy().view(np.uint32))
        assert r["idx"].tolist() == idx.tolist()
    assert res[0]["keys"].tolist() == res[1]["keys"].tolist()


def test_argmax_keys_merge_to_the_highest_logit_and_lowest_index():
    vals = np.array([[1.5, -2.0, 3.0], [1.5, 7.0, -1.0], [0.5, 7.0, 3.0]], np.float32)  # rank x RHS
    idxs = np.array([[10, 5, 900], [4, 600, 3], [700, 100, 50]], np.uint64)
    keys = (total_order_key(vals) << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - idxs)
    best = parallel.merge_argmax_keys(torch.from_numpy(keys.view(np.int64)))
    assert parallel.key_index(best).tolist() == [4, 100, 50]  # ties -> lowest index


def test_shard_range_keeps_whole_tiles():
    assert parallel.shard_range(17408, 8, 3) == (6528, 8704)
    assert parallel.shard_range(152064, 4, 1) == (38016, 76032)
    with pytest.raises(ValueError):
        parallel.shard_range(5120, 3, 0)
