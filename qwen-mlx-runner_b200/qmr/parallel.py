"""Row-sharded SwiGLU MLP and vocabulary-sharded head over several GPUs.

One process per GPU (torch.distributed, NCCL over NVLink on B200).  The
matrices are split by output rows, so every packed row stays whole on one
rank and each shard is an ordinary matrix for the library's kernels:

* MLP (src/engine.rs:755-763 run on n GPUs): rank r holds rows
  [r*F/n, (r+1)*F/n) of gate and up, computes silu(gate x) * (up x) for them
  with the fused gate/up kernel, the ranks exchange the activations, and
  rank r computes rows [r*H/n, (r+1)*H/n) of down from the full activation
  vector; a second exchange assembles the output.  Both exchanges are the
  activation vectors only (F*B and H*B floats); no weight moves.
* Head (src/engine.rs:777-780 + src/chat.rs:383-390): rank r holds vocabulary
  rows [r*V/n, (r+1)*V/n); each rank's fused logits+argmax kernel returns its
  best (value, index) as one packed key per RHS, the ranks exchange the
  keys and take the largest: the highest logit under f32 total order, ties
  to the lowest vocabulary index, exactly the single-GPU rule.

Two ways to exchange the shards:

* `exchange="p2p"` (what bench.py uses on GPUs): the streaming kernel
  itself stores each finished row into every rank's full output buffer over
  NVLink (CUDA IPC mappings of buffers the library allocated, PeerExchange)
  and its last CTA publishes an epoch; a one-warp kernel on each rank waits
  (bounded) for every rank's epoch before the consumer, and for the head
  merges the keys.  No collective library call on the data path.
* `exchange="nccl"`: torch.distributed all-gathers (any backend: the CPU
  tests run it on gloo with an oracle-backed `ops`).

The kernels are passed in as `ops` (qmr.ops on GPUs); the host logic here is
the same for any backend that implements those calls.
"""
from __future__ import annotations

import ctypes
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


class _DeviceArray:
    """A view of library-allocated device memory that torch can wrap without
    a copy (__cuda_array_interface__)."""

    def __init__(self, ptr: int, n: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False), "version": 3}


class PeerExchange:
    """The buffers of one output exchange over peer memory (QmrExchange in
    include/qmr.h), set up collectively by every rank of `group`.

    Every rank allocates, with the library, two full outputs [4][total_rows]
    f32 (or, for a head, two key arrays [world][4]), a flag array and an
    epoch word; the IPC handles are all-gathered and every peer's buffers are
    mapped.  Calls alternate between the two output buffers (`next()`), so a
    rank can run one exchange ahead of the slowest peer without overwriting
    data that peer has not consumed yet."""

    def __init__(self, total_rows: int, row_base: int, head: bool = False, group=None):
        from . import _lib
        self._lib = _lib
        L = _lib.lib()
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if not 2 <= self.world <= _lib.QMR_MAX_RANKS:
            raise ValueError(f"peer exchange supports 2..{_lib.QMR_MAX_RANKS} ranks")
        self.group, self.head, self.total_rows = group, head, total_rows
        self._own, self._mapped = [], []

        def alloc(nbytes: int) -> int:
            p = ctypes.c_void_p()
            _lib.check(L.qmr_exchange_alloc(nbytes, ctypes.byref(p)))
            self._own.append(p.value)
            return p.value

        if head:
            self.out = [None, None]
            self.keys = [alloc(self.world * 4 * 8) for _ in range(2)]
        else:
            self.out = [alloc(4 * total_rows * 4) for _ in range(2)]
            self.keys = [None, None]
        self.flags = alloc(max(4 * self.world, 16))
        self.epoch = alloc(16)
        mine = []
        for ptr in self.out + self.keys + [self.flags]:
            if ptr is None:
                mine.append(None)
                continue
            h = ctypes.create_string_buffer(_lib.QMR_IPC_HANDLE_BYTES)
            _lib.check(L.qmr_ipc_handle(ptr, h))
            mine.append(h.raw)
        handles = [None] * self.world
        dist.all_gather_object(handles, mine, group=group)
        ptrs = []
        for r in range(self.world):
            if r == self.rank:
                ptrs.append(self.out + self.keys + [self.flags])
                continue
            row = []
            for h in handles[r]:
                if h is None:
                    row.append(None)
                    continue
                p = ctypes.c_void_p()
                _lib.check(L.qmr_ipc_open(h, ctypes.byref(p)))
                self._mapped.append(p.value)
                row.append(p.value)
            ptrs.append(row)
        self.structs = []
        for par in range(2):
            ex = _lib.QmrExchange()
            ex.world, ex.rank, ex.total_rows, ex.row_base = self.world, self.rank, total_rows, row_base
            for r in range(self.world):
                ex.out[r] = ptrs[r][par]
                ex.keys[r] = ptrs[r][2 + par]
                ex.flags[r] = ptrs[r][4]
            ex.epoch = self.epoch
            self.structs.append(ex)
        self.parity = 0
        self._views = None

    def next(self):
        """(exchange struct, parity) of the next call; parities alternate."""
        par = self.parity
        self.parity ^= 1
        return self.structs[par], par

    def output(self, par: int, device) -> torch.Tensor:
        """Full output buffer `par` as a float32 tensor [4 * total_rows]."""
        if self._views is None:
            self._views = [torch.as_tensor(_DeviceArray(p, 4 * self.total_rows, "<f4"), device=device)
                           for p in self.out]
        return self._views[par]

    def close(self):
        """Unmap the peers' buffers, then (after every rank did) free ours."""
        L = self._lib.lib()
        for p in self._mapped:
            L.qmr_ipc_close(p)
        self._mapped = []
        dist.barrier(group=self.group)
        for p in self._own:
            L.qmr_exchange_free(p)
        self._own = []


class ShardedMLP:
    """down(silu(gate x) * (up x)) with gate/up/down row-sharded over the
    group's ranks.  gate, up: this rank's [F/n, H] shards; down: its [H/n, F]
    shard (ops.PackedMatrix-like objects)."""

    def __init__(self, gate, up, down, hidden: int, inter: int, ops, group=None, exchange: str = "nccl"):
        self.group = group
        self.world = dist.get_world_size(group)
        if gate.rows * self.world != inter or down.rows * self.world != hidden:
            raise ValueError("shards do not tile the MLP")
        if gate.cols != hidden or up.cols != hidden or down.cols != inter:
            raise ValueError("shard widths do not match the MLP")
        if exchange not in ("nccl", "p2p"):
            raise ValueError("exchange must be nccl or p2p")
        self.gate, self.up, self.down = gate, up, down
        self.hidden, self.inter = hidden, inter
        self.ops = ops
        self.exchange = exchange
        if exchange == "p2p":
            rank = dist.get_rank(group)
            self.xa = PeerExchange(inter, rank * gate.rows, group=group)
            self.xy = PeerExchange(hidden, rank * down.rows, group=group)

    def close(self):
        if self.exchange == "p2p":
            self.xa.close()
            self.xy.close()

    def __call__(self, x: torch.Tensor, batch: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        dev = self.gate.weight.device  # x may be a pinned host tensor
        if self.exchange == "p2p":
            ea, par = self.xa.next()
            self.ops.gateup_swiglu_exchange(self.gate, self.up, x, batch, ea)
            self.ops.exchange_wait(ea, batch)
            ey, _ = self.xy.next()
            self.ops.matmul_affine_exchange(self.down, self.xa.output(par, dev), batch, ey)
            self.ops.exchange_wait(ey, batch)
            y = self.xy.output(par, dev)[:batch * self.hidden]
            if out is not None:
                out.copy_(y)
                return out
            return y
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

    def __init__(self, head, vocab: int, row_base: int, ops, group=None, exchange: str = "nccl"):
        self.group = group
        self.world = dist.get_world_size(group)
        if head.rows * self.world != vocab:
            raise ValueError("shards do not tile the vocabulary")
        if exchange not in ("nccl", "p2p"):
            raise ValueError("exchange must be nccl or p2p")
        self.head, self.vocab, self.row_base, self.ops = head, vocab, row_base, ops
        self.exchange = exchange
        if exchange == "p2p":
            self.xk = PeerExchange(vocab, row_base, head=True, group=group)

    def close(self):
        if self.exchange == "p2p":
            self.xk.close()

    def __call__(self, x: torch.Tensor, batch: int, logits: Optional[torch.Tensor] = None):
        """Returns (token index per RHS as int32 [batch], winning keys int64
        [batch]); `logits` receives this rank's [batch][V/n] logits if given."""
        dev = self.head.weight.device  # x may be a pinned host tensor
        lg = logits if logits is not None else torch.empty(batch * self.head.rows, dtype=torch.float32, device=dev)
        if self.exchange == "p2p":
            ek, _ = self.xk.next()
            idx = torch.empty(batch, dtype=torch.int32, device=dev)
            keys = torch.empty(batch, dtype=torch.int64, device=dev)
            self.ops.head_argmax_exchange(self.head, x, lg, batch, ek)
            self.ops.exchange_wait(ek, batch, argmax=idx, best_key=keys)
            return idx, keys
        idx = torch.empty(batch, dtype=torch.int32, device=dev)
        keys = torch.empty(batch, dtype=torch.int64, device=dev)
        self.ops.head_argmax(self.head, x, lg, idx, batch, best_key=keys, row_base=self.row_base)
        gathered = torch.empty(self.world * batch, dtype=torch.int64, device=dev)
        dist.all_gather_into_tensor(gathered, keys, group=self.group)
        best = merge_argmax_keys(gathered.view(self.world, batch))
        return key_index(best), best
