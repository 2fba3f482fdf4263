"""The sharded MLP and head with the output exchange over peer memory, on
2, 4 and 8 GPUs (one process each, NCCL only for set-up and for the
comparison exchange).  Each world size is skipped when the box has fewer
GPUs.

What must hold: the exchange moves every row exactly (all ranks end with
the same bits, and the peer-memory exchange gives the same bits as NCCL
all-gathers of the same shards); the merged argmax is the argmax of the
ranks' logits with the lowest-index tie rule; and every stage meets the
FP64 oracle bound.  (A shard is a different matrix shape, whose launch plan
may split a tile's windows between warps differently, so sharded outputs
are not required to equal the unsharded call bit for bit.)"""
import os
import pathlib
import socket
import tempfile

import numpy as np
import pytest
import torch

import oracle
from qmr import synth

pytestmark = pytest.mark.gpu

H, F, V, B = 5120, 17408, 152064 // 4, 3  # the config-2 MLP; a vocabulary slice (16-row tiles at 8 ranks)
NS_RTOL = 2e-5


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
    mods = []
    try:
        gate, up, down, head = _mats()
        f0, f1 = parallel.shard_range(F, world, rank)
        h0, h1 = parallel.shard_range(H, world, rank)
        v0, v1 = parallel.shard_range(V, world, rank)
        dm = lambda m, r0, r1, c: synth.to_device(_rows(m, r0, r1), r1 - r0, c, 4, 64, dev)  # noqa: E731
        g, u, d, h = dm(gate, f0, f1, H), dm(up, f0, f1, H), dm(down, h0, h1, F), dm(head, v0, v1, H)
        x = torch.from_numpy(synth.activations(B, H, seed=75).ravel()).to(dev)
        out = {}
        for ex in ("p2p", "nccl"):
            mlp = parallel.ShardedMLP(g, u, d, H, F, qmr.ops, exchange=ex)
            hd = parallel.ShardedHead(h, V, v0, qmr.ops, exchange=ex)
            mods += [mlp, hd]
            ys, ids, lgs, acts = [], [], [], []
            for _ in range(steps):  # p2p: both output buffers, several epochs
                y = mlp(x, B).clone()
                lg = torch.empty(B * (v1 - v0), dtype=torch.float32, device=dev)
                idx, _ = hd(y, B, logits=lg)
                if ex == "p2p":
                    acts.append(mlp.xa.output(mlp.xa.parity ^ 1, dev)[:B * F].cpu().numpy())
                ys.append(y.cpu().numpy())
                ids.append(idx.cpu().numpy())
                lgs.append(lg.cpu().numpy())
            out[ex] = (np.stack(ys), np.stack(ids), np.stack(lgs), np.stack(acts) if acts else np.zeros(1))
        torch.cuda.synchronize()
        np.savez(pathlib.Path(outdir) / f"rank{rank}.npz", y_p2p=out["p2p"][0], idx_p2p=out["p2p"][1],
                 lg_p2p=out["p2p"][2], act_p2p=out["p2p"][3], y_nccl=out["nccl"][0], idx_nccl=out["nccl"][1],
                 lg_nccl=out["nccl"][2], err=qmr.ops.device_error())
    finally:
        torch.cuda.synchronize()
        for m in mods:
            m.close()
        dist.destroy_process_group()


def _bound(got, want, mag, slack, what):
    ratio, i = oracle.tolerance_ratio(got, want, mag + slack, rtol=1.0)
    assert ratio <= 1.0, f"{what}: output {i} got {np.ravel(got)[i]} want {np.ravel(want)[i]} ratio {ratio}"


@pytest.mark.parametrize("world", [2, 4, 8])
def test_p2p_sharded_mlp_and_head_exchange_exactly_and_meet_the_bound(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    steps = 3
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_rank_main, args=(world, _free_port(), d, steps), nprocs=world, start_method="spawn",
                           join=True)
        res = [np.load(pathlib.Path(d) / f"rank{r}.npz") for r in range(world)]
    for r in range(world):
        assert int(res[r]["err"]) == 0
        # The peer-memory exchange and NCCL all-gathers of the same shards agree bit for bit,
        # every rank holds the same full output, and repeated steps are reproducible.
        assert np.array_equal(res[r]["y_p2p"].view(np.uint32), res[r]["y_nccl"].view(np.uint32)), r
        assert np.array_equal(res[r]["idx_p2p"], res[r]["idx_nccl"]), r
        assert np.array_equal(res[r]["lg_p2p"].view(np.uint32), res[r]["lg_nccl"].view(np.uint32)), r
        assert np.array_equal(res[r]["y_p2p"].view(np.uint32), res[0]["y_p2p"].view(np.uint32)), r
        assert np.array_equal(res[r]["act_p2p"].view(np.uint32), res[0]["act_p2p"].view(np.uint32)), r
        assert np.array_equal(res[r]["idx_p2p"], res[0]["idx_p2p"]), r
        for s in range(1, steps):
            assert np.array_equal(res[r]["y_p2p"][s].view(np.uint32), res[r]["y_p2p"][0].view(np.uint32))
    act = res[0]["act_p2p"][0].reshape(B, F)
    y = res[0]["y_p2p"][0].reshape(B, H)
    logits = np.concatenate([res[r]["lg_p2p"][0].reshape(B, V // world) for r in range(world)], axis=1)
    idx = res[0]["idx_p2p"][0]
    # The merged argmax is the argmax of all ranks' logits (f32 total order, lowest index on ties).
    assert [oracle.argmax_f32(logits[b]) for b in range(B)] == idx.tolist()
    # Each stage against FP64 on its own input.
    gate, up, down, head = _mats()
    x = synth.activations(B, H, seed=75)
    want, mag = oracle.swiglu_f64(gate["weight"], gate["scales"], gate["biases"], up["weight"], up["scales"],
                                  up["biases"], x, F, H, 4, 64, B)
    _bound(act, want, NS_RTOL * mag, 0.05 * np.abs(want), "sharded gate/up")
    want, mag = oracle.matmul_f64(down["weight"], down["scales"], down["biases"], act, H, F, 4, 64, batch=B)
    _bound(y, want, NS_RTOL * mag, 0.0, "sharded down")
    want, mag = oracle.matmul_f64(head["weight"], head["scales"], head["biases"], y, V, H, 4, 64, batch=B)
    _bound(logits, want, NS_RTOL * mag, 0.0, "sharded head")
