"""Tensor-parallel decode of the synthetic model over 2, 4 and 8 GPUs (one
process per GPU, torch.distributed on gloo only for the IPC handles and the
final barrier; the data path is the library's peer-memory exchange).

What must hold:
* every rank emits the same tokens, and they are the FP64 oracle's greedy
  tokens: step-by-step forward over a prompt, device-side greedy decode, and
  verification rounds of 3 with right drafts (all accepted) and wrong
  drafts (none accepted);
* each rank's logits are the oracle's logits of its vocabulary rows, within
  the single-GPU engine's bound (the all-reduce sums the ranks' partial
  products in rank order, a different order from one GPU's, so the bits
  are not required to equal the unsharded engine's);
* the step graph holds the one-GPU launches plus the head's key wait: each
  all-reduce rides in the image build of the next matrix that reads x.

Each world size is skipped when the box has fewer GPUs.  Shapes: the small
layer graph at 2 ranks (column slices of 4 groups, padded metadata rows),
and 4 layers of the 27B-shaped model at 2, 4 and 8 ranks (8 ranks replicate
each of its 4 KV heads on 2 ranks; the down projection's 2176-column slices
have 34 groups, padded to 40)."""
import datetime
import os
import pathlib
import socket
import tempfile

import numpy as np
import pytest
import torch

import oracle
import qmr
from qmr import engine as qeng

pytestmark = pytest.mark.gpu

SEED, CONTEXT, N_NEW, BLOCK = 29, 64, 12, 3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _config(name):
    if name == "small":
        from test_engine_gpu import small_config
        return small_config()
    return qeng.qwen27b_config(layers=4)


def _prompt(cfg):
    from qmr import synth
    return [int(v % cfg["vocab"]) for v in synth.splitmix64(31, 5)]


def _rank_main(rank, world, port, outdir, name, table):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    qmr.ops.init(rank)
    cfg = _config(name)
    prompt = _prompt(cfg)
    eng = qmr.Engine.synthetic_sharded(cfg, SEED, CONTEXT)
    try:
        _, _, vbase, vrows = eng.shard
        lgs, nxts = [], []
        for t in prompt:
            lg, nx = eng.forward(t)
            lgs.append(lg)
            nxts.append(nx)
        gen, _, _ = eng.generate([nxts[-1]], N_NEW)
        eng.reset()
        mtp, rounds, acc, _, _ = eng.mtp_generate(prompt, N_NEW, BLOCK, table)
        eng.reset()
        wrong = [(t + 1) % cfg["vocab"] for t in table]
        mtp_w, rounds_w, acc_w, _, _ = eng.mtp_generate(prompt, N_NEW, BLOCK, wrong)
        launches = eng.step_launches()
        np.savez(pathlib.Path(outdir) / f"rank{rank}.npz", lgs=np.stack(lgs), nxts=np.array(nxts), gen=np.array(gen),
                 mtp=np.array(mtp), mtp_w=np.array(mtp_w), stats=np.array([rounds, acc, rounds_w, acc_w]),
                 shard=np.array([vbase, vrows]), launches=np.array(launches), err=qmr.ops.device_error())
    finally:
        eng.close()
        dist.destroy_process_group()


_oracle_cache = {}


def _oracle_run(name):
    """The unsharded model's FP64 logits over the prompt and its greedy tokens."""
    if name not in _oracle_cache:
        cfg = _config(name)
        oracle.set_threads(len(os.sched_getaffinity(0)))
        o = oracle.synthetic_decode_oracle(cfg, SEED, CONTEXT, qeng.synthetic_mid, qeng.MID_EMBED, qeng.MID_HEAD)
        prompt = _prompt(cfg)
        lgs = [o.forward(t) for t in prompt]
        cur = oracle.argmax_f64(lgs[-1])
        seq = [cur]
        for _ in range(N_NEW):
            cur = oracle.argmax_f64(o.forward(cur))
            seq.append(cur)
        _oracle_cache[name] = (cfg, prompt, np.stack(lgs), seq)
    return _oracle_cache[name]


@pytest.mark.parametrize("name,world", [("small", 2), ("qwen27b-4", 2), ("qwen27b-4", 4), ("qwen27b-4", 8)])
def test_sharded_decode_gives_the_oracle_tokens_on_every_rank(name, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    cfg, prompt, want_lgs, seq = _oracle_run(name)
    # Greedy tokens: seq[0] follows the prompt, seq[1:] continue from it.
    table = [0] * CONTEXT
    for k, t in enumerate(seq[:N_NEW]):
        table[len(prompt) + k] = t
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_rank_main, args=(world, _free_port(), d, name, table), nprocs=world,
                           start_method="spawn", join=True)
        res = [np.load(pathlib.Path(d) / f"rank{r}.npz") for r in range(world)]
    tol = 1e-4 if name == "small" else 1e-3
    vrows = cfg["vocab"] // world
    L = cfg["layers"]
    for r in range(world):
        x = res[r]
        assert int(x["err"]) == 0, r
        assert x["shard"].tolist() == [r * vrows, vrows]
        # Same tokens on every rank, and the oracle's.
        assert x["nxts"][-1] == seq[0], (r, x["nxts"].tolist())
        assert x["gen"].tolist() == seq[1:], (r, x["gen"].tolist(), seq)
        assert x["mtp"].tolist() == seq[:N_NEW], (r, x["mtp"].tolist())
        assert x["mtp_w"].tolist() == seq[:N_NEW], (r, x["mtp_w"].tolist())
        rounds, acc, rounds_w, acc_w = x["stats"].tolist()
        assert acc == rounds * (BLOCK - 1) and rounds == -(-(N_NEW - 1) // BLOCK)
        assert acc_w == 0 and rounds_w == N_NEW - 1
        # This rank's vocabulary rows of every prompt position's logits.
        want = want_lgs[:, r * vrows:(r + 1) * vrows]
        scale = np.max(np.abs(want_lgs), axis=1, keepdims=True)
        err = np.max(np.abs(x["lgs"] - want) / scale)
        assert err <= tol, (r, err)
        # embed + per layer (in-proj, mixer, out, gate/up, down: one streaming kernel per
        # matrix; each all-reduce rides in the image build of the next matrix that reads x)
        # + head (matmul, key wait) + advance; without the head, the last all-reduce runs as
        # wait + sum.
        with_head, without = x["launches"].tolist()
        assert with_head == 1 + 5 * L + 2 + 1 and without == with_head
