"""Row-sharded SwiGLU MLP and vocabulary-sharded head over several GPUs.

One process per GPU (torch.distributed, NCCL over NVLink on B200).  The
matrices are split by output rows, so every packed row stays whole on one
rank and each shard is an ordinary matrix for the library's kernels:

* MLP (src/engine.rs:755-763 run on n GPUs): rank r holds rows
  [r*F/n, (r+1)*F/n) of gate and up, computes silu(gate x) * (up x) for them
  with the fused gate/up kernel, the ranks all-gather the activations, and
  rank r computes rows [r*H/n, (r+1)*H/n) of down from the full activation
  vector; a second all-gather assembles the output.  Both exchanges are the
  activation vectors only (F*B and H*B floats); no weight moves.
* Head (src/engine.rs:777-780 + src/chat.rs:383-390): rank r holds vocabulary
  rows [r*V/n, (r+1)*V/n); each rank's fused logits+argmax kernel returns its
  best (value, index) as one packed key per RHS, the ranks all-gather the
  keys and take the largest: the highest logit under f32 total order, ties
  to the lowest vocabulary index, exactly the single-GPU rule.

The kernels are passed in as `ops` (qmr.ops on GPUs); the host logic here is
the same for any backend that implements those calls.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

SIGN = -(1 << 63)  # flips an unsigned 64-bit order onto signed int64 order


def shard_range(total: int, world: int, rank: int, align: int = 16):
    """Equal contiguous shard [r0, r1) of `total` rows; every shard is a
    multiple of `align` rows (the kernels' 16-row tiles), so `total` must
    divide into `world * align`-row pieces."""
    if total % (world * align):
        raise ValueError(f"{total} rows do not split into {world} shards of whole {align}-row tiles")
    per = total // world
    return rank * per, (rank + 1) * per


def merge_argmax_keys(keys: torch.Tensor) -> torch.Tensor:
    """[world, B] packed argmax keys (uint64 bits in int64) -> the winning key
    per RHS: the maximum as unsigned 64-bit numbers."""
    flipped = keys ^ SIGN
    return flipped.max(dim=0).values ^ SIGN


def key_index(key: torch.Tensor) -> torch.Tensor:
    """Vocabulary index of packed keys: the low word holds 0xffffffff - index."""
    return (0xFFFFFFFF - (key & 0xFFFFFFFF)).to(torch.int32)


def _gather_rows(local: torch.Tensor, batch: int, group) -> torch.Tensor:
    """All-gather token-major [batch][rows_r] shards into [batch][world*rows_r]."""
    world = dist.get_world_size(group)
    rows_r = local.numel() // batch
    stacked = torch.empty(world * local.numel(), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(stacked, local, group=group)
    return stacked.view(world, batch, rows_r).permute(1, 0, 2).reshape(batch * world * rows_r)


class ShardedMLP:
    """down(silu(gate x) * (up x)) with gate/up/down row-sharded over the
    group's ranks.  gate, up: this rank's [F/n, H] shards; down: its [H/n, F]
    shard (ops.PackedMatrix-like objects)."""

    def __init__(self, gate, up, down, hidden: int, inter: int, ops, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        if gate.rows * self.world != inter or down.rows * self.world != hidden:
            raise ValueError("shards do not tile the MLP")
        if gate.cols != hidden or up.cols != hidden or down.cols != inter:
            raise ValueError("shard widths do not match the MLP")
        self.gate, self.up, self.down = gate, up, down
        self.hidden, self.inter = hidden, inter
        self.ops = ops

    def __call__(self, x: torch.Tensor, batch: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        dev = x.device
        act_r = torch.empty(batch * self.gate.rows, dtype=torch.float32, device=dev)
        self.ops.gateup_swiglu(self.gate, self.up, x, act_r, batch)
        act = _gather_rows(act_r, batch, self.group)
        y_r = torch.empty(batch * self.down.rows, dtype=torch.float32, device=dev)
        self.ops.matmul_affine(self.down, act, y_r, batch)
        y = _gather_rows(y_r, batch, self.group)
        if out is not None:
            out.copy_(y)
            return out
        return y


class ShardedHead:
    """Greedy next token over a vocabulary-sharded head: `head` is this rank's
    [V/n, H] shard whose first row is vocabulary row `row_base`."""

    def __init__(self, head, vocab: int, row_base: int, ops, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        if head.rows * self.world != vocab:
            raise ValueError("shards do not tile the vocabulary")
        self.head, self.vocab, self.row_base, self.ops = head, vocab, row_base, ops

    def __call__(self, x: torch.Tensor, batch: int, logits: Optional[torch.Tensor] = None):
        """Returns (token index per RHS as int32 [batch], winning keys int64
        [batch]); `logits` receives this rank's [batch][V/n] logits if given."""
        dev = x.device
        lg = logits if logits is not None else torch.empty(batch * self.head.rows, dtype=torch.float32, device=dev)
        idx = torch.empty(batch, dtype=torch.int32, device=dev)
        keys = torch.empty(batch, dtype=torch.int64, device=dev)
        self.ops.head_argmax(self.head, x, lg, idx, batch, best_key=keys, row_base=self.row_base)
        gathered = torch.empty(self.world * batch, dtype=torch.int64, device=dev)
        dist.all_gather_into_tensor(gathered, keys, group=self.group)
        best = merge_argmax_keys(gathered.view(self.world, batch))
        return key_index(best), best
